"""dance_b200.search: GPU search of a DiskANN memory index and recall against
ground truth, the role of DiskANN's search_memory_index for the graphs
written here (reference README.md:78,92).

CPU tests cover the file decoding and the recall arithmetic; GPU tests
build small indexes, write them in DiskANN layout, and check that the tool
returns exactly what the library's query search returns on the same graph.
"""
import numpy as np
import pytest

from dance_b200 import formats, search as SR, stitched as S


def test_decode_graph_round_trip(tmp_path):
    rng = np.random.default_rng(3)
    n, R = 300, 12
    deg = rng.integers(0, R + 1, n).astype(np.uint32)
    g = np.full((n, R), 0xFFFFFFFF, np.uint32)
    for i in range(n):
        g[i, :deg[i]] = rng.choice(n, deg[i], replace=False)
    formats.write_graph(tmp_path / "idx", g, deg, 17)
    g2, d2, start = SR.decode_graph(tmp_path / "idx")
    R2 = int(deg.max())
    assert start == 17 and np.array_equal(d2, deg) and g2.shape == (n, R2)
    assert np.array_equal(g2, g[:, :R2])


def test_load_memory_index_checks(tmp_path):
    x = np.arange(40, dtype=np.uint8).reshape(10, 4)
    g = np.full((10, 2), 0xFFFFFFFF, np.uint32)
    g[:, 0] = (np.arange(10) + 1) % 10
    formats.save_memory_index(tmp_path / "ok", x, g, np.ones(10, np.uint32), 3)
    data, graph, degree, start = SR.load_memory_index(tmp_path / "ok", "uint8")
    assert np.array_equal(data, x) and start == 3 and graph.shape == (10, 1)
    formats.save_memory_index(tmp_path / "bad", x[:9], g, np.ones(10, np.uint32), 3)
    with pytest.raises(ValueError, match="graph has 10 rows"):
        SR.load_memory_index(tmp_path / "bad", "uint8")


def test_label_sidecars_parse(tmp_path):
    names, l2i, i2l, pts = S.parse_label_lines(["b", "a,c", "c", "a"])
    side = S.sidecar_texts(names, l2i, i2l, [1, 2, 0])
    for k, text in side.items():
        (tmp_path / ("idx" + k)).write_text(text)
    offs, labs, name_to_id, medoids = SR.load_label_sidecars(tmp_path / "idx")
    rows = [sorted(l2i[nm] for nm in r) for r in names]
    assert offs.tolist() == np.cumsum([0] + [len(r) for r in rows]).tolist()
    assert labs.tolist() == [v for r in rows for v in r]
    assert name_to_id == {nm: i + 1 for i, nm in enumerate(i2l)}
    assert medoids == {1: 1, 2: 2, 3: 0}


def test_recall_arithmetic():
    found = np.array([[1, 2, 3], [4, 5, 0xFFFFFFFF]], np.uint32)
    truth = np.array([[3, 2, 9], [4, 7, 8]], np.uint32)
    assert SR.recall_at(found, truth, 3) == pytest.approx(3 / 6)
    assert SR.recall_at(found, truth, 1) == pytest.approx(1 / 2)
    with pytest.raises(ValueError, match="fewer than K"):
        SR.recall_at(found, truth[:, :2], 3)


def _clusters(rng, n, dim, k=32):
    c = rng.integers(0, 256, (k, dim))
    return np.clip(np.rint(c[rng.integers(0, k, n)] + rng.normal(0, 18, (n, dim))), 0, 255).astype(np.uint8)


def _truth(x, q, k, allowed=None):
    d = ((q.astype(np.int64)[:, None, :] - x.astype(np.int64)[None, :, :]) ** 2).sum(-1)
    if allowed is not None:
        d = np.where(allowed, d, np.iinfo(np.int64).max)
    return np.argsort(d, axis=1, kind="stable")[:, :k].astype(np.uint32)


@pytest.mark.gpu
def test_search_tool_matches_library_search(dance_lib, tmp_path, capsys):
    import torch
    from dance_b200 import vamana
    rng = np.random.default_rng(21)
    n, dim, nq = 4000, 32, 200
    x = _clusters(rng, n, dim)
    q = _clusters(rng, nq, dim)
    g, deg = vamana.gpu_vamana_vnew2_build(x, 32, 64, 48, 32)
    med = vamana.gpu_vamana_vnew2_get_last_medoid()
    prefix = tmp_path / "idx"
    formats.save_memory_index(prefix, x, g, deg, med)
    gt = _truth(x, q, 10)
    formats.write_bin(tmp_path / "q.u8bin", q)
    formats.write_groundtruth(tmp_path / "gt.bin", gt, np.zeros(gt.shape, np.float32))
    rows = SR.search_memory_index(prefix, "uint8", q, 10, [10, 64], gt)
    store, stride = vamana.padded_store(torch.from_numpy(x).cuda())
    gd = torch.from_numpy(g[:, :int(deg.max())].copy().view(np.int32)).cuda()
    for r in rows:
        ids, _ = vamana.search_queries(store, dim, stride, gd, int(deg.max()), med, torch.from_numpy(q).cuda(),
                                       r["L"], 10)
        assert np.array_equal(r["ids"], ids.cpu().numpy().view(np.uint32))
        assert r["recall"] == pytest.approx(vamana.recall_at_k(r["ids"], gt))
    assert rows[1]["recall"] > 0.9 and rows[1]["recall"] >= rows[0]["recall"]
    assert SR.main(["--data_type", "uint8", "--index_path_prefix", str(prefix), "--query_file",
                    str(tmp_path / "q.u8bin"), "--gt_file", str(tmp_path / "gt.bin"), "-K", "10", "-L", "10",
                    "64"]) == 0
    out = capsys.readouterr().out.strip().splitlines()
    assert out[0].split()[0] == "Ls" and [int(l.split()[0]) for l in out[1:]] == [10, 64]
    assert float(out[2].split()[-1]) == pytest.approx(100 * rows[1]["recall"], abs=0.01)


@pytest.mark.gpu
def test_search_tool_filtered_on_stitched_index(dance_lib, tmp_path):
    import torch
    from dance_b200 import vamana
    rng = np.random.default_rng(22)
    n, dim, nl, nq = 3000, 24, 6, 120
    x = _clusters(rng, n, dim)
    assign = rng.integers(0, nl, n)
    dp = tmp_path / "base.u8bin"
    formats.write_bin(dp, x)
    lf = tmp_path / "labels.txt"
    lf.write_text("".join(f"lab{int(a)}\n" for a in assign))
    prefix = tmp_path / "st"
    S.build_gpu_stitched("uint8", dp, lf, prefix, Rsmall=16, Lsmall=40, Rstitched=16, C=24, steps=24)
    q = _clusters(rng, nq, dim)
    qlab = rng.integers(0, nl, nq)
    names = [f"lab{int(a)}" for a in qlab]
    gt = _truth(x, q, 10, allowed=(assign[None, :] == qlab[:, None]))
    rows = SR.search_memory_index(prefix, "uint8", q, 10, [40], gt, query_filters=names)
    # the same search through the library call, from the label medoids
    offs, labs, name_to_id, medoids = SR.load_label_sidecars(prefix)
    graph, degree, _ = SR.decode_graph(prefix)
    store, stride = vamana.padded_store(torch.from_numpy(x).cuda())
    ql = np.array([name_to_id[nm] for nm in names], np.uint32)
    qs = np.array([medoids[int(l)] for l in ql], np.uint32)
    dev = [torch.from_numpy(a.view(np.int32)).cuda() for a in (offs, labs, ql, qs)]
    ids, _ = vamana.search_queries_filtered(store, dim, stride, torch.from_numpy(graph.view(np.int32)).cuda(),
                                            graph.shape[1], *dev, torch.from_numpy(q).cuda(), 40, 10)
    assert np.array_equal(rows[0]["ids"], ids.cpu().numpy().view(np.uint32))
    found = rows[0]["ids"]
    # every answer carries the query's label
    ok = found != 0xFFFFFFFF
    assert np.all(assign[found[ok].astype(np.int64)] == np.repeat(qlab, 10).reshape(nq, 10)[ok])
    assert rows[0]["recall"] > 0.9
