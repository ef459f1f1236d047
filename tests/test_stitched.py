"""GPU-StitchedVamana: label rules, files, and GPU parity with the oracle.

Reference: apps/utils/gpu_stitched_vamana_index.cpp (parse_labels :111-160,
write_sidecars :162-199, write_graph :200-227, label loop :276-341) and the
gate validator tools/validate_gpu_stitched_gate.py:26-145.
"""
import os

import numpy as np
import pytest

import oracle
from dance_b200 import stitched as S
from dance_b200.formats import GRAPH_HEADER, read_graph, write_bin


# ------------------------------------------------------------------ CPU
def test_parse_labels_rules():
    names, l2i, i2l, pts = S.parse_label_lines(["b, a\r\n", "a\n", "c,c,b\n", " a , b\n"])
    assert names == [["b", "a"], ["a"], ["c", "b"], ["a", "b"]]
    assert l2i == {"b": 1, "a": 2, "c": 3} and i2l == ["b", "a", "c"]
    assert pts == [[0, 2, 3], [0, 1, 3], [2]]
    for bad in (["a", "\n"], ["a,,b"], ["a,"], [",a"]):
        with pytest.raises(ValueError, match="empty label"):
            S.parse_label_lines(bad)
    with pytest.raises(ValueError, match="universal"):
        S.parse_label_lines(["a", "0,b"], universal_label="0")
    # the universal label only matters when it is given
    assert S.parse_label_lines(["0"])[2] == ["0"]


def test_sidecar_texts_known_answer():
    names, l2i, i2l, _ = S.parse_label_lines(["red", "blue,red", "green"])
    side = S.sidecar_texts(names, l2i, i2l, [7, 1, 2])
    assert side["_labels.txt"] == "1\n2,1\n3\n"
    assert side["_label_formatted.txt"] == side["_labels.txt"]
    assert side["_labels_map.txt"] == "red\t1\nblue\t2\ngreen\t3\n"
    assert side["_labels_to_medoids.txt"] == "1, 7\n2, 1\n3, 2\n"


def test_csr_graph_header_and_round_trip():
    offs = np.array([0, 2, 2, 5], np.uint64)
    ids = np.array([1, 2, 0, 1, 9], np.uint32)
    blob = S.encode_csr_graph(offs, ids)
    size, maxdeg, start, frozen = GRAPH_HEADER.unpack_from(blob, 0)
    assert (size, maxdeg, start, frozen) == (len(blob), 3, 0, 0)
    assert len(blob) == 24 + 4 * 3 + 4 * 5
    words = np.frombuffer(blob, np.uint32, offset=24).tolist()
    assert words == [2, 1, 2, 0, 3, 0, 1, 9]


def test_labels_csr_and_lpt():
    offs, pts = S.labels_csr([[0, 3], [], [1, 2, 4]])
    assert offs.tolist() == [0, 2, 2, 5] and pts.tolist() == [0, 3, 1, 2, 4]
    sizes = [50, 40, 30, 20, 10, 10]
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint64)
    owner = S.lpt_assignment(offs, 2)
    assert owner.tolist() == [0, 1, 1, 0, 0, 1]
    loads = [sum(s for s, o in zip(sizes, owner) if o == r) for r in range(2)]
    assert loads == [80, 80]
    assert S.lpt_assignment(offs, 1).tolist() == [0] * 6


def test_oracle_remap_rule():
    # two overlapping labels over global points 10..13 (4 points, N = 14)
    rows = [[] for _ in range(14)]
    ctr = dict(remap_invalid_local_ids=0, remap_self_loops=0, remap_duplicate_edges=0)
    INV = 0xFFFFFFFF
    ids_a = [10, 11, 12]
    g_a = np.array([[1, 2, INV], [0, 1, 2], [5, 0, 1]], np.uint32)  # row 1 has a self loop, row 2 an out-of-range id
    oracle.stitched_remap(rows, ids_a, g_a, np.array([3, 3, 3]), 3, 3, ctr)
    ids_b = [11, 13]
    g_b = np.array([[1, 1], [0, 0]], np.uint32)  # duplicates inside a row
    oracle.stitched_remap(rows, ids_b, g_b, np.array([2, 1]), 2, 3, ctr)
    assert rows[10] == [11, 12] and rows[11] == [10, 12, 13] and rows[12] == [10, 11] and rows[13] == [11]
    assert ctr == dict(remap_invalid_local_ids=2, remap_self_loops=1, remap_duplicate_edges=1)
    # Rstitched caps what each label contributes
    rows2 = [[] for _ in range(14)]
    oracle.stitched_remap(rows2, ids_a, g_a, np.array([3, 3, 3]), 3, 1, ctr)
    assert rows2[10] == [11] and rows2[11] == [10]


def _zipf_labels(n, nl, rng, min_size=1):
    w = 1.0 / np.arange(1, nl + 1)
    sizes = np.maximum(min_size, np.floor(w / w.sum() * n)).astype(int)
    sizes[0] += n - sizes.sum()
    assign = np.repeat(np.arange(nl), sizes)
    rng.shuffle(assign)
    return assign


def _line_store(pos, dim=16):
    x = np.zeros((len(pos), dim), np.uint8)
    x[:, 0] = pos
    return x


def test_point_label_csr():
    offs, labs = S.point_label_csr([[2, 0], [], [0, 1, 1]], 4)
    assert offs.tolist() == [0, 2, 3, 4, 4] and labs.tolist() == [0, 2, 2, 0]


def test_oracle_global_prune_rules():
    """Hand cases for the restated DiskANN prune_all_neighbors (patched)."""
    # points on a line; row 0 at 0 has neighbours 1..5
    x = _line_store([0, 10, 12, 30, 31, 60])
    offs = np.array([0, 5, 5, 5, 5, 5, 5], np.uint64)
    ids = np.array([5, 1, 3, 2, 4], np.uint32)
    # no labels, alpha 1: 1 (d=100) occludes 2 (d(1,2)=4 < 144), 3 and 4 and 5 -> [1]
    rows, deg = oracle.stitched_global_prune(x, offs, ids, None, None, 4, 750, 1.0)
    assert deg[0] == 1 and rows[0, 0] == 1
    # rows with at most `range` neighbours are copied as they are
    rows, deg = oracle.stitched_global_prune(x, offs, ids, None, None, 5, 750, 1.0)
    assert deg[0] == 5 and rows[0].tolist() == [5, 1, 3, 2, 4]
    # labels: row 0 and point 2 share label 7 which point 1 lacks, so 1 cannot
    # occlude 2 any more (patch rule (F_p n F_x) in F_s)
    lo = np.array([0, 2, 3, 5, 6, 7, 8], np.uint32)
    lb = np.array([3, 7, 3, 3, 7, 3, 3, 3], np.uint32)
    rows, deg = oracle.stitched_global_prune(x, offs, ids, lo, lb, 4, 750, 1.0)
    assert rows[0, :deg[0]].tolist() == [1, 2]
    # later passes: entries whose occlusion factor lies in (1, a] enter in the
    # pass with that a (a = 1, 1.2, 1.44, ... while a <= alpha)
    z = np.zeros((4, 16), np.uint8)
    z[1, 0] = 100            # s, d(0,s) = 10000
    z[2, 0], z[2, 1] = 100, 200  # x: d(0,x) = 50000, d(s,x) = 40000 -> factor 1.25
    z[3, 0], z[3, 1] = 100, 210  # w: d(0,w) = 54100, d(s,w) = 44100 -> factor 1.2268
    o2 = np.array([0, 3, 3, 3, 3], np.uint64)
    i2 = np.array([1, 2, 3], np.uint32)
    rows, deg = oracle.stitched_global_prune(z, o2, i2, None, None, 2, 750, 1.2)
    assert rows[0, :deg[0]].tolist() == [1]  # both factors above 1.2
    rows, deg = oracle.stitched_global_prune(z, o2, i2, None, None, 2, 750, 1.3)
    # pass 2 (a = 1.2): nothing new; a = 1.44 > 1.3 stops: still [1]
    assert rows[0, :deg[0]].tolist() == [1]
    rows, deg = oracle.stitched_global_prune(z, o2, i2, None, None, 2, 750, 1.5)
    # a = 1.44 <= 1.5: x (1.25) is selected, then the range of 2 is full
    assert rows[0, :deg[0]].tolist() == [1, 2]
    # shortlist: row 0 with labels {1, 2}; its three nearest carry only label 1,
    # so with range 2 the quota (1 per label) admits the nearest label-2 carrier
    w = _line_store([0, 1, 2, 3, 10, 50])
    o3 = np.array([0, 5, 5, 5, 5, 5, 5], np.uint64)
    i3 = np.array([1, 2, 3, 4, 5], np.uint32)
    lo3 = np.array([0, 2, 3, 4, 5, 6, 7], np.uint32)
    lb3 = np.array([1, 2, 1, 1, 1, 2, 2], np.uint32)
    rows, deg = oracle.stitched_global_prune(w, o3, i3, lo3, lb3, 2, 750, 1.2)
    assert rows[0, :deg[0]].tolist() == [1, 4]
    rows, deg = oracle.stitched_global_prune(w, o3, i3, None, None, 2, 750, 1.2)
    # unlabelled: 1 occludes 2, 3 and 4 (factor 100/81 > 1.2); 5 (2500/2401) enters at a = 1.2
    assert rows[0, :deg[0]].tolist() == [1, 5]


def test_write_and_audit_index(tmp_path):
    names, l2i, i2l, pts = S.parse_label_lines(["a", "b", "a", "b"])
    offs = np.array([0, 1, 2, 3, 4], np.uint64)
    ids = np.array([2, 3, 0, 1], np.uint32)
    data = np.zeros((4, 8), np.float32)
    dp = tmp_path / "x.fbin"
    write_bin(dp, data)
    prefix = tmp_path / "idx"
    S.write_stitched_index(prefix, dp, offs, ids, names, l2i, i2l, [0, 1])
    a = S.audit_stitched_index(prefix, 64)
    assert a["size_matches"] and a["nodes"] == 4 and a["edges"] == 4 and a["start_node"] == 0
    for k in ("invalid_ids", "self_loops", "duplicate_edges", "degree_overflow_rows", "incompatible_label_edges"):
        assert a[k] == 0, k
    assert a["sidecar_rows_match"] and a["medoid_labels_match_map"] and a["invalid_label_medoids"] == []
    assert (tmp_path / "idx.data").read_bytes() == dp.read_bytes()
    with pytest.raises(FileExistsError):
        S.write_stitched_index(prefix, dp, offs, ids, names, l2i, i2l, [0, 1])
    # an edge across labels is reported
    bad = tmp_path / "bad"
    S.write_stitched_index(bad, dp, offs, np.array([1, 3, 0, 1], np.uint32), names, l2i, i2l, [0, 1])
    assert S.audit_stitched_index(bad, 64)["incompatible_label_edges"] == 1


# ------------------------------------------------------------------ GPU
def _rows_of(offs, ids):
    return [ids[int(offs[i]):int(offs[i + 1])].tolist() for i in range(len(offs) - 1)]


def _dataset(dtype, n, dim, rng):
    if dtype == np.uint8:
        c = rng.integers(0, 256, (16, dim))
        x = c[rng.integers(0, 16, n)] + rng.normal(0, 20, (n, dim))
        return np.clip(np.rint(x), 0, 255).astype(np.uint8)
    c = rng.standard_normal((16, dim))
    return (c[rng.integers(0, 16, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,dim", [(np.float32, 24), (np.uint8, 40)])
def test_stitched_single_label_matches_oracle(dance_lib, dtype, dim):
    rng = np.random.default_rng(7)
    n, nl = 3000, 12
    x = _dataset(dtype, n, dim, rng)
    assign = _zipf_labels(n - 6, nl, rng)
    # three tiny labels (1, 2 and 3 points) at the end
    assign = np.concatenate([assign, [nl, nl + 1, nl + 1, nl + 2, nl + 2, nl + 2]])
    label_points = S.labels_from_assignment(assign, nl + 3)
    offs, pts = S.labels_csr(label_points)
    args = dict(r_small=16, l_small=40, r_stitched=24, C=32, steps=24)
    row_offsets, row_ids, medoids, st = S.stitched_build(x, offs, pts, streams=3, **args)
    rows, omed, ctr = oracle.stitched(x, label_points, 16, 40, 24, 32, 24)
    assert medoids.tolist() == omed
    got = _rows_of(row_offsets, row_ids)
    bad = [i for i in range(n) if got[i] != rows[i]]
    assert not bad, f"{len(bad)} rows differ, first {bad[:5]}"
    for k, v in ctr.items():
        assert st[k] == v, k
    assert st["output_edges"] == sum(len(r) for r in rows)
    assert st["num_labels"] == nl + 3 and st["npts_per_label_min"] == 1 and st["streams"] == 3
    assert st["total_label_memberships"] == n == st["processed_label_memberships"]


@pytest.mark.gpu
def test_stitched_overlapping_labels_union_order(dance_lib):
    rng = np.random.default_rng(11)
    n, dim = 1500, 16
    x = _dataset(np.float32, n, dim, rng)
    lines = []
    for i in range(n):
        k = 1 + int(rng.integers(0, 3))
        lines.append(",".join(f"L{int(v)}" for v in rng.choice(6, k, replace=False)))
    names, l2i, i2l, label_points = S.parse_label_lines(lines)
    offs, pts = S.labels_csr(label_points)
    row_offsets, row_ids, medoids, st = S.stitched_build(x, offs, pts, 12, 32, 12, 24, 16)
    rows, omed, ctr = oracle.stitched(x, label_points, 12, 32, 12, 24, 16)
    assert medoids.tolist() == omed
    assert _rows_of(row_offsets, row_ids) == rows
    assert st["remap_duplicate_edges"] == ctr["remap_duplicate_edges"] > 0
    assert st["max_degree"] == max(len(r) for r in rows) > 12


@pytest.mark.gpu
def test_stitched_remap_device_rule(dance_lib):
    """dance_stitched_remap on hand-made local graphs with invalid ids, self
    loops and duplicates, against the oracle rule."""
    import ctypes
    import torch
    from dance_b200 import DanceStitchedStats, check
    rng = np.random.default_rng(3)
    n, nl, rs = 700, 5, 40
    label_points = [sorted(rng.choice(n, int(rng.integers(1, 300)), replace=False).tolist()) for _ in range(nl)]
    offs, pts = S.labels_csr(label_points)
    M = int(offs[-1])
    lg = np.empty((M, rs), np.uint32)
    ld = rng.integers(0, rs + 1, M).astype(np.uint32)
    for l in range(nl):
        a, b = int(offs[l]), int(offs[l + 1])
        sz = b - a
        lg[a:b] = rng.integers(0, sz + 2, (sz, rs))  # ids >= sz are out of range
        lg[a:b][rng.random((sz, rs)) < 0.05] = 0xFFFFFFFF
    for r_out in (rs, 33, 7):
        rows = [[] for _ in range(n)]
        ctr = dict(remap_invalid_local_ids=0, remap_self_loops=0, remap_duplicate_edges=0)
        for l in range(nl):
            a, b = int(offs[l]), int(offs[l + 1])
            oracle.stitched_remap(rows, label_points[l], lg[a:b], ld[a:b], rs, max(r_out, rs), ctr)
        d_lg = torch.from_numpy(lg.view(np.int32)).cuda()
        d_ld = torch.from_numpy(ld.view(np.int32)).cuda()
        ro = np.zeros(n + 1, np.uint64)
        ri = np.zeros(M * rs, np.uint32)
        st = DanceStitchedStats()
        lib = dance_lib
        rc = lib.dance_stitched_remap(n, nl, S._ptr(offs), S._ptr(pts), ctypes.c_void_p(d_lg.data_ptr()),
                                      ctypes.c_void_p(d_ld.data_ptr()), rs, r_out, S._ptr(ro), S._ptr(ri), M * rs,
                                      ctypes.byref(st), None)
        check(rc)
        assert _rows_of(ro, ri) == rows  # r_out below Rsmall is raised to Rsmall
        assert (st.remap_invalid_local_ids, st.remap_self_loops, st.remap_duplicate_edges) == (
            ctr["remap_invalid_local_ids"], ctr["remap_self_loops"], ctr["remap_duplicate_edges"])
        # too small an output buffer is an error, not an overrun
        if r_out == rs and st.output_edges > 1:
            rc = lib.dance_stitched_remap(n, nl, S._ptr(offs), S._ptr(pts), ctypes.c_void_p(d_lg.data_ptr()),
                                          ctypes.c_void_p(d_ld.data_ptr()), rs, r_out, S._ptr(ro), S._ptr(ri),
                                          st.output_edges - 1, None, None)
            assert rc == -3


@pytest.mark.gpu
def test_stitched_fp16_build_matches_oracle(dance_lib, monkeypatch):
    rng = np.random.default_rng(5)
    n, dim, nl = 1200, 32, 4
    x = _dataset(np.float32, n, dim, rng)
    label_points = S.labels_from_assignment(_zipf_labels(n, nl, rng), nl)
    offs, pts = S.labels_csr(label_points)
    monkeypatch.setenv("DANCE_FLOAT16_BUILD", "1")
    row_offsets, row_ids, medoids, _ = S.stitched_build(x, offs, pts, 12, 32, 16, 24, 16)
    rows, omed, _ = oracle.stitched(x.astype(np.float16), label_points, 12, 32, 16, 24, 16)
    assert medoids.tolist() == omed
    assert _rows_of(row_offsets, row_ids) == rows


@pytest.mark.gpu
def test_stitched_app_end_to_end(dance_lib, tmp_path):
    rng = np.random.default_rng(9)
    n, dim, nl = 2500, 16, 8
    x = _dataset(np.uint8, n, dim, rng)
    assign = _zipf_labels(n, nl, rng)
    dp = tmp_path / "base.u8bin"
    write_bin(dp, x)
    lf = tmp_path / "labels.txt"
    lf.write_text("".join(f"lab{int(a)}\n" for a in assign))
    prefix = tmp_path / "stitched"
    tj = tmp_path / "timing.json"
    timing = S.build_gpu_stitched("uint8", dp, lf, prefix, timing_json=str(tj), Rsmall=16, Lsmall=32,
                                  Rstitched=16, C=24, steps=16)
    import json
    saved = json.loads(tj.read_text())
    assert list(saved) == S.TIMING_KEYS and saved["num_labels"] == nl
    audit = S.audit_stitched_index(prefix, 16)
    for k in ("invalid_ids", "self_loops", "duplicate_edges", "degree_overflow_rows", "incompatible_label_edges"):
        assert audit[k] == 0, (k, audit)
    assert audit["size_matches"] and audit["nodes"] == n and audit["invalid_label_medoids"] == []
    assert audit["edges"] == timing["output_edges"]
    rows, _, _, _ = read_graph(prefix)
    _, _, _, label_points = S.parse_labels(lf)
    orows, omed, _ = oracle.stitched(x, label_points, 16, 32, 16, 24, 16)
    assert [r.tolist() for r in rows] == orows


@pytest.mark.gpu
def test_stitched_app_multi_label_prunes_on_gpu(dance_lib, tmp_path):
    """Multi-label input: the union graph is kept as <prefix>_full and the
    index is the label-aware global prune of it (the DiskANN step of the
    reference app, run here on the GPU), equal to the oracle's."""
    rng = np.random.default_rng(19)
    n, dim = 2500, 16
    x = _dataset(np.uint8, n, dim, rng)
    dp = tmp_path / "base.u8bin"
    write_bin(dp, x)
    lines = [",".join(f"t{int(v)}" for v in rng.choice(7, 1 + int(rng.integers(0, 3)), replace=False))
             for _ in range(n)]
    lf = tmp_path / "labels.txt"
    lf.write_text("".join(ln + "\n" for ln in lines))
    prefix = tmp_path / "multi"
    timing = S.build_gpu_stitched("uint8", dp, lf, prefix, Rsmall=16, Lsmall=32, Rstitched=16, C=24, steps=16)
    assert timing["final_prune_seconds"] > 0
    full, _, _, _ = read_graph(str(prefix) + "_full")
    pruned, _, _, _ = read_graph(prefix)
    _, _, _, label_points = S.parse_labels(lf)
    urows, _, _ = oracle.stitched(x, label_points, 16, 32, 16, 24, 16)
    assert [r.tolist() for r in full] == urows
    assert max(len(r) for r in full) > 16
    offs = np.zeros(n + 1, np.uint64)
    offs[1:] = np.cumsum([len(r) for r in urows])
    ids = np.array([v for r in urows for v in r], np.uint32)
    lo, lb = S.point_label_csr(label_points, n)
    orows, odeg = oracle.stitched_global_prune(x, offs, ids, lo, lb, 16, 750, 1.2)
    assert [r.tolist() for r in pruned] == [orows[v, :odeg[v]].tolist() for v in range(n)]
    audit = S.audit_stitched_index(prefix, 16)
    for k in ("invalid_ids", "self_loops", "duplicate_edges", "degree_overflow_rows"):
        assert audit[k] == 0, (k, audit)
    # allow_unpruned writes the union graph as the index
    S.build_gpu_stitched("uint8", dp, lf, tmp_path / "u", Rsmall=16, Lsmall=32, Rstitched=16, C=24, steps=16,
                         allow_unpruned=True)
    assert [r.tolist() for r in read_graph(tmp_path / "u")[0]] == urows


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,dim", [(np.uint8, 32), (np.float32, 24), (np.float32, 100)])
def test_global_prune_kernel_matches_oracle(dance_lib, dtype, dim):
    """dance_stitched_global_prune against the oracle restatement on a random
    multi-label union graph with long rows (up to 300 neighbours, duplicate
    and self ids), with and without labels."""
    rng = np.random.default_rng(23)
    n = 3000
    x = _dataset(dtype, n, dim, rng)
    deg = rng.integers(0, 300, n)
    deg[:50] = rng.integers(40, 80, 50)
    offs = np.zeros(n + 1, np.uint64)
    offs[1:] = np.cumsum(deg)
    ids = rng.integers(0, n, int(offs[-1])).astype(np.uint32)
    ids[rng.random(len(ids)) < 0.01] = 0  # repeated ids (and self loops on row 0)
    label_points = [sorted(rng.choice(n, int(rng.integers(200, 1500)), replace=False).tolist()) for _ in range(9)]
    lo, lb = S.point_label_csr(label_points, n)
    for labels in (True, False):
        L0, L1 = (lo, lb) if labels else (None, None)
        for R, alpha in ((32, 1.2), (64, 1.5), (17, 1.0)):
            go, gi, npr = S.global_prune(x, offs, ids, L0, L1, R, 750, alpha)
            orows, odeg = oracle.stitched_global_prune(x, offs, ids, L0, L1, R, 750, alpha)
            assert np.array_equal(np.diff(go.astype(np.int64)), odeg.astype(np.int64)), (labels, R)
            assert gi.tolist() == orows[np.arange(R)[None, :] < odeg[:, None]].tolist(), (labels, R)
            assert npr == int((deg > R).sum())
    # shorter pool cap (max_candidates) on the unlabelled path
    go, gi, _ = S.global_prune(x, offs, ids, None, None, 32, 40, 1.2)
    orows, odeg = oracle.stitched_global_prune(x, offs, ids, None, None, 32, 40, 1.2)
    assert gi.tolist() == orows[np.arange(32)[None, :] < odeg[:, None]].tolist()
