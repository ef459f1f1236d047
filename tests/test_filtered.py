"""GPU-FilteredVamana: oracle pinned to the reference, GPU kernels against both.

Reference: src/gpu_vamana_filtered.cu, canonical path
(canonical_round0_from_host_backbone_typed :5663-6483).  The fixtures come
from the reference's own kernels on a B200 (tests/golden/make_golden_filtered.py):
the random initial graph and, for three rounds, every intermediate of a round
run on the reference's own input graph.

Parity bar: bit-exact everywhere -- task and union search outputs (ids,
distances, slot order), merged work rows, forward-pruned rows -- except the
reverse-repaired rows whose candidate range the reference's fill kernel
overwrites with the forward row of a row that has no reverse source
(src/gpu_vamana_filtered.cu:5071-5105, a race between concurrent stores);
those rows follow the rule "forward row, then new reverse sources" here, and
the tests check that every other row matches.
"""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
INVALID = 0xFFFFFFFF


def _cases():
    man = json.loads((GOLDEN / "manifest_filtered.json").read_text())
    return [c for c in man if "file" in c]


def _load(c):
    z = np.load(GOLDEN / c["file"])
    x = z["data"]
    xs = oracle.float_to_half(x) if x.dtype == np.float32 else x
    lab = oracle.FilteredLabels(z["offsets"], z["labels"], z["starts"], c["num_labels"], c["universal"],
                                c["global_start"])
    return z, x, xs, lab


def spill_rows(fg, fd):
    """Rows whose reverse-repair candidate range the reference's fill kernel
    overwrites: for every row u without reverse sources, its forward row is
    written at the start of the next list, covering [off[u], off[u] + deg(u))."""
    n = len(fd)
    rev = [[] for _ in range(n)]
    for s in range(n):
        for t in fg[s, :fd[s]]:
            if t < n and t != s:
                rev[t].append(int(s))
    cnt = np.array([0 if not rev[r] else int(fd[r]) + sum(1 for s in rev[r] if s not in set(fg[r, :fd[r]].tolist()))
                    for r in range(n)])
    off = np.concatenate([[0], np.cumsum(cnt)])
    hit = np.zeros(n, bool)
    starts = off[:-1]
    for u in range(n):
        if not rev[u] and fd[u] > 0:
            lo, hi = off[u], off[u] + int(fd[u])
            hit |= (cnt > 0) & (starts < hi) & (starts + cnt > lo)
    return hit


def rows_equal(g1, d1, g2, d2):
    return np.array([d1[i] == d2[i] and np.array_equal(g1[i, :d1[i]], g2[i, :d2[i]]) for i in range(len(d1))])


# ------------------------------------------------------------------ CPU: oracle pinned
@pytest.mark.parametrize("c", _cases(), ids=lambda c: c["file"])
def test_oracle_random_graph_matches_reference(c):
    z = np.load(GOLDEN / c["file"])
    n = len(z["offsets"]) - 1
    g, d = oracle.filtered_random_graph(n, c["R"], min(16, c["R"]), 42)
    assert np.array_equal(g, z["random_graph"]) and np.array_equal(d, z["random_degree"])


@pytest.mark.parametrize("c", _cases(), ids=lambda c: c["file"])
def test_oracle_rounds_match_reference(c):
    z, _, xs, lab = _load(c)
    R, L, FL, C, S = c["R"], c["L"], c["FL"], oracle.filtered_work_width(c["C"]), c["STEPS"]
    for rnd in range(3):
        k = f"r{rnd}_"
        g, d = z[k + "graph_in"], z[k + "degree_in"]
        ti, td = oracle.filtered_task_search(xs, lab, R, FL, S, g, d)
        assert np.array_equal(ti, z[k + "ti"]) and np.array_equal(td, z[k + "td"]), f"task search, round {rnd}"
        oi, od = oracle.filtered_ordinary_search(xs, lab, R, L, FL, S, g, d)
        assert np.array_equal(oi, z[k + "oi"]) and np.array_equal(od, z[k + "od"]), f"union search, round {rnd}"
        o = oracle.filtered_round(xs, lab, R, L, FL, C, S, c["alpha"], g, d)
        w_ok = rows_equal(o["work"], o["work_deg"], z[k + "wi"], z[k + "wdeg"])
        wd_ok = all(np.array_equal(o["work_d"][i, :o["work_deg"][i]], z[k + "wd"][i, :o["work_deg"][i]])
                    for i in range(len(d)))
        assert w_ok.all() and wd_ok, f"merged work rows, round {rnd}"
        assert rows_equal(o["fwd"], o["fwd_deg"], z[k + "fg"], z[k + "fd"]).all(), f"forward prune, round {rnd}"
        same = rows_equal(o["graph"], o["degree"], z[k + "go"], z[k + "do"])
        spill = spill_rows(z[k + "fg"], z[k + "fd"])
        assert not (~same & ~spill).any(), f"reverse repair differs outside the spill rows, round {rnd}"
        assert same.mean() > 0.95


def test_filtered_prune_coverage_rule():
    """FilteredRobustPrune: a selection only occludes candidates whose shared
    labels with the row it also carries (include/filtered_label_coverage.cuh)."""
    # row 0 {1,2}; 1 {1} nearest; 2 {1,2} and 3 {1} both next to 1
    x = np.zeros((4, 16), np.uint8)
    x[1, 0] = 10
    x[2, 0], x[2, 1] = 12, 2
    x[3, 0], x[3, 2] = 12, 2
    offs = np.array([0, 2, 3, 5, 6], np.uint32)
    labs = np.array([1, 2, 1, 1, 2, 1], np.uint32)
    lab = oracle.FilteredLabels(offs, labs, np.full(3, INVALID, np.uint32), 3)
    cand = np.array([1, 2, 3], np.uint32)
    cd = np.array([oracle.distance(x[0], x[i]) for i in cand], np.float32)
    g, d = oracle.filtered_prune_lists(x, lab, 4, 1.2, [0], [cand], [cd])
    # 3 shares only label 1 with the row, which 1 carries: occluded; 2 shares 2: kept
    assert d[0] == 2 and g[0, :2].tolist() == [1, 2]


def test_work_width_below_2R_is_status_1(dance_lib):
    """min(C, 128) < 2R returns 1 before any device work, as the reference does."""
    man = json.loads((GOLDEN / "manifest_filtered.json").read_text())
    status = [c for c in man if c.get("status_case")][0]
    assert status["status"] == 1
    n, dim = 50, 8
    x = np.zeros((n, dim), np.float32)
    offs = np.arange(n + 1, dtype=np.uint32)
    labs = np.zeros(n, np.uint32)
    starts = np.zeros(1, np.uint32)
    g = np.zeros((n, status["R"]), np.uint32)
    d = np.zeros(n, np.uint32)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    rc = dance_lib.gpu_vamana_filtered_build_float(p(x), n, dim, status["R"], 64, 64, status["C"], 32, 1.2, p(offs),
                                                   p(labs), n, p(starts), 1, INVALID, 0, None, None, 0, p(g), p(d))
    assert rc == 1
    # labels out of order are refused with -1, also before any device work
    offs2 = np.array([0] + [2] * n, np.uint32)
    bad2 = np.array([1, 0], np.uint32)
    rc = dance_lib.gpu_vamana_filtered_build_float(p(x), n, dim, 8, 64, 64, 64, 32, 1.2, p(offs2), p(bad2), 2,
                                                   p(starts), 2, INVALID, 0, None, None, 0, p(g), p(d))
    assert rc == -1 and "strictly increasing" in dance_lib.dance_last_error().decode()


# ------------------------------------------------------------------ GPU
def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32 if a.dtype == np.uint32 else a.dtype)).cuda()


def _store(x):
    import torch
    from dance_b200 import vamana
    t = torch.from_numpy(x).cuda()
    if x.dtype == np.float32:
        t = t.half()
    store, stride = vamana.padded_store(t)
    return store, stride, (0 if x.dtype == np.uint8 else 1)


def _stage_round(lib, x, lab, c, g_in, d_in):
    import torch
    n, dim = x.shape
    R, L, FL, C, S = c["R"], c["L"], c["FL"], oracle.filtered_work_width(c["C"]), c["STEPS"]
    T = len(lab.labels)
    keep, okeep = min(min(FL, 32), 8), min(R, L)
    store, stride, dt = _store(x)
    gi, di = _dev(g_in), _dev(d_in)
    out = dict(ti=torch.zeros((T, keep), dtype=torch.int32, device="cuda"),
               td=torch.zeros((T, keep), dtype=torch.float32, device="cuda"),
               oi=torch.zeros((n, okeep), dtype=torch.int32, device="cuda"),
               od=torch.zeros((n, okeep), dtype=torch.float32, device="cuda"),
               wi=torch.zeros((n, C), dtype=torch.int32, device="cuda"),
               wd=torch.zeros((n, C), dtype=torch.float32, device="cuda"),
               wdeg=torch.zeros(n, dtype=torch.int32, device="cuda"),
               fg=torch.zeros((n, R), dtype=torch.int32, device="cuda"),
               fd=torch.zeros(n, dtype=torch.int32, device="cuda"),
               go=torch.zeros((n, R), dtype=torch.int32, device="cuda"),
               do=torch.zeros(n, dtype=torch.int32, device="cuda"))
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    H = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    torch.cuda.synchronize()
    rc = lib.dance_filtered_stage_round(dt, P(store), stride, n, dim, R, L, FL, C, S, c["alpha"], H(lab.offsets),
                                        H(lab.labels), H(lab.starts), lab.num_labels, lab.universal,
                                        lab.global_start, P(gi), P(di),
                                        *[P(out[k]) for k in ("ti", "td", "oi", "od", "wi", "wd", "wdeg", "fg", "fd",
                                                              "go", "do")], None)
    assert rc == 0, lib.dance_last_error().decode()
    torch.cuda.synchronize()
    res = {}
    for k, t in out.items():
        a = t.cpu().numpy()
        res[k] = a.view(np.uint32) if a.dtype == np.int32 else a
    return res


@pytest.mark.gpu
@pytest.mark.parametrize("c", _cases(), ids=lambda c: c["file"])
def test_gpu_random_graph_matches_reference(dance_lib, c):
    import torch
    z = np.load(GOLDEN / c["file"])
    n, R = len(z["offsets"]) - 1, c["R"]
    g = torch.zeros((n, R), dtype=torch.int32, device="cuda")
    d = torch.zeros(n, dtype=torch.int32, device="cuda")
    assert dance_lib.dance_filtered_random_graph(n, R, min(16, R), 42, ctypes.c_void_p(g.data_ptr()),
                                                 ctypes.c_void_p(d.data_ptr()), None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(g.cpu().numpy().view(np.uint32), z["random_graph"])
    assert np.array_equal(d.cpu().numpy().view(np.uint32), z["random_degree"])


@pytest.mark.gpu
@pytest.mark.parametrize("c", _cases(), ids=lambda c: c["file"])
def test_gpu_rounds_match_reference(dance_lib, c):
    z, x, xs, lab = _load(c)
    R, L, FL, C, S = c["R"], c["L"], c["FL"], oracle.filtered_work_width(c["C"]), c["STEPS"]
    for rnd in range(3):
        k = f"r{rnd}_"
        r = _stage_round(dance_lib, x, lab, c, z[k + "graph_in"], z[k + "degree_in"])
        for key in ("ti", "td", "oi", "od"):
            assert np.array_equal(r[key], z[k + key]), f"{key}, round {rnd}"
        assert rows_equal(r["wi"], r["wdeg"], z[k + "wi"], z[k + "wdeg"]).all(), f"work rows, round {rnd}"
        assert all(np.array_equal(r["wd"][i, :r["wdeg"][i]], z[k + "wd"][i, :r["wdeg"][i]])
                   for i in range(len(r["wdeg"]))), f"work distances, round {rnd}"
        assert rows_equal(r["fg"], r["fd"], z[k + "fg"], z[k + "fd"]).all(), f"forward prune, round {rnd}"
        o = oracle.filtered_round(xs, lab, R, L, FL, C, S, c["alpha"], z[k + "graph_in"], z[k + "degree_in"])
        assert rows_equal(r["go"], r["do"], o["graph"], o["degree"]).all(), f"reverse repair vs oracle, round {rnd}"
        same = rows_equal(r["go"], r["do"], z[k + "go"], z[k + "do"])
        assert not (~same & ~spill_rows(z[k + "fg"], z[k + "fd"])).any(), f"reverse repair, round {rnd}"


@pytest.mark.gpu
@pytest.mark.parametrize("c", _cases(), ids=lambda c: c["file"])
def test_gpu_whole_build_matches_oracle(dance_lib, c):
    from dance_b200 import GPUFilteredVamanaStats
    z, x, xs, lab = _load(c)
    n, dim = x.shape
    R = c["R"]
    g = np.zeros((n, R), np.uint32)
    d = np.zeros(n, np.uint32)
    H = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    fn = dance_lib.gpu_vamana_filtered_build_float if x.dtype == np.float32 else dance_lib.gpu_vamana_filtered_build_uint8
    rc = fn(H(x), n, dim, R, c["L"], c["FL"], c["C"], c["STEPS"], c["alpha"], H(lab.offsets), H(lab.labels),
            len(lab.labels), H(lab.starts), lab.num_labels, lab.universal, lab.global_start, None, None, 0, H(g), H(d))
    assert rc == 0, dance_lib.dance_last_error().decode()
    og, od = oracle.filtered_build(xs, lab, R, c["L"], c["FL"], c["C"], c["STEPS"], c["alpha"])
    assert rows_equal(g, d, og, od).all()
    assert (g[np.arange(R)[None, :] >= d[:, None]] == INVALID).all()
    st = GPUFilteredVamanaStats()
    dance_lib.gpu_vamana_filtered_get_last_stats(ctypes.byref(st))
    assert st.semantic_complete == 1 and st.invalid_neighbor_count == 0 and st.self_loop_count == 0
    assert st.out_degree_max <= R and abs(st.out_degree_avg - d.mean()) < 1e-9
    assert st.reverse_touched_rows > 0 and st.filtered_search_distance_count > 0


@pytest.mark.gpu
def test_gpu_hub_rows_take_the_block_prune(dance_lib):
    """A point at the centre of the data is every row's nearest neighbour, so
    its reverse-repair list is far longer than one warp's shared-memory list
    and goes through the block-per-row prune."""
    rng = np.random.default_rng(17)
    n, dim, R = 1500, 32, 16
    x = rng.standard_normal((n, dim)).astype(np.float32)
    x[0] = 0.0
    labs_per = [sorted(rng.choice(3, int(rng.integers(1, 3)), replace=False).tolist()) for _ in range(n)]
    offs = np.concatenate([[0], np.cumsum([len(v) for v in labs_per])]).astype(np.uint32)
    labs = np.concatenate(labs_per).astype(np.uint32)
    starts = np.array([next(i for i in range(n) if l in labs_per[i]) for l in range(3)], np.uint32)
    lab = oracle.FilteredLabels(offs, labs, starts, 3, INVALID, 0)
    c = dict(R=R, L=32, FL=32, C=48, STEPS=16, alpha=1.2)
    g0, d0 = oracle.filtered_random_graph(n, R, 16, 42)
    xs = oracle.float_to_half(x)
    o = oracle.filtered_round(xs, lab, R, 32, 32, 48, 16, 1.2, g0, d0)
    indeg = np.bincount(o["fwd"][np.arange(R)[None, :] < o["fwd_deg"][:, None]], minlength=n)
    assert indeg.max() > 256
    r = _stage_round(dance_lib, x, lab, c, g0, d0)
    assert rows_equal(r["fg"], r["fd"], o["fwd"], o["fwd_deg"]).all()
    assert rows_equal(r["go"], r["do"], o["graph"], o["degree"]).all()


@pytest.mark.gpu
def test_gpu_resident_build_with_given_graph_matches_oracle(dance_lib):
    """dance_filtered_build_resident from a caller's initial graph (the
    DISKANN_GPU_FILTERED_HANDOFF=0 route starts from a vnew2 graph this way)."""
    import torch
    rng = np.random.default_rng(23)
    n, dim, R = 1200, 24, 16
    x = rng.integers(0, 256, (n, dim)).astype(np.uint8)
    labs_per = [sorted(rng.choice(6, int(rng.integers(1, 4)), replace=False).tolist()) for _ in range(n)]
    offs = np.concatenate([[0], np.cumsum([len(v) for v in labs_per])]).astype(np.uint32)
    labs = np.concatenate(labs_per).astype(np.uint32)
    starts = np.array([next(i for i in range(n) if l in labs_per[i]) for l in range(6)], np.uint32)
    lab = oracle.FilteredLabels(offs, labs, starts, 6, 2, starts[1])
    g0 = np.full((n, R), INVALID, np.uint32)
    d0 = rng.integers(0, R + 1, n).astype(np.uint32)
    for i in range(n):
        g0[i, :d0[i]] = rng.choice(n, d0[i], replace=False)
    store, stride, dt = _store(x)
    gi, di = _dev(g0), _dev(d0)
    go = torch.zeros((n, R), dtype=torch.int32, device="cuda")
    do = torch.zeros(n, dtype=torch.int32, device="cuda")
    H = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    torch.cuda.synchronize()
    rc = dance_lib.dance_filtered_build_resident(dt, P(store), stride, n, dim, R, 32, 24, 40, 16, 1.2, H(offs),
                                                 H(labs), H(starts), 6, 2, int(starts[1]), P(gi), P(di), 2, P(go),
                                                 P(do), None, None)
    assert rc == 0, dance_lib.dance_last_error().decode()
    torch.cuda.synchronize()
    og, od = oracle.filtered_build(x, lab, R, 32, 24, 40, 16, 1.2, graph=g0, degree=d0, rounds=2)
    assert rows_equal(go.cpu().numpy().view(np.uint32), do.cpu().numpy().view(np.uint32), og, od).all()


# ---------------------------------------------------------------- inputs computed before the hook
def test_label_points_csr_with_universal_label():
    from dance_b200 import filtered as F
    offs, labs = F.labels_csr([[0, 2], [1], [2, 5], [5], [0]])
    lo, lp = F.label_points_csr(offs, labs, 3)
    assert lo.tolist() == [0, 2, 3, 5] and lp.tolist() == [0, 4, 1, 0, 2]
    lo, lp = F.label_points_csr(offs, labs, 3, universal_label_id=5)
    assert lo.tolist() == [0, 4, 7, 10] and lp.tolist() == [0, 2, 3, 4, 1, 2, 3, 0, 2, 3]


def test_oracle_entry_point_and_label_start_rules():
    rng = np.random.default_rng(4)
    x = rng.normal(size=(500, 12)).astype(np.float32)
    c = np.zeros(12, np.float32)
    for row in x:  # point by point, in float
        c = (c + row).astype(np.float32)
    c = (c / np.float32(500)).astype(np.float32)
    assert oracle.entry_point(x) == int(np.argmin(((x.astype(np.float64) - c) ** 2).sum(1)))
    # least-chosen rule: with one candidate point per label every start is that point
    lo = np.array([0, 1, 2, 4], np.uint32)
    lp = np.array([7, 7, 3, 9], np.uint32)
    s = oracle.label_starts(lo, lp, 10, 25, 42)
    assert s[0] == 7 and s[1] == 7 and s[2] in (3, 9)
    # two labels over the same two points: the second label avoids the first's start
    lo = np.array([0, 2, 4], np.uint32)
    lp = np.array([1, 2, 1, 2], np.uint32)
    s = oracle.label_starts(lo, lp, 3, 25, 42)
    assert sorted(s.tolist()) == [1, 2]
    assert oracle.label_starts(np.array([0, 0], np.uint32), np.zeros(0, np.uint32), 3)[0] == 0xFFFFFFFF


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [np.uint8, np.float16, np.float32])
def test_gpu_entry_point_matches_oracle(dance_lib, dtype):
    import torch
    from dance_b200 import filtered as F, vamana, workloads
    if dtype == np.uint8:
        x = workloads.clustered_u8(20000, 64, centroids=50, seed=8).numpy()
    else:
        x = workloads.gaussian_mixture_f32(20000, 96, centroids=50, seed=8).numpy().astype(dtype)
    st, stride = vamana.padded_store(torch.from_numpy(x).cuda())
    assert F.calculate_entry_point(st, x.shape[1], stride) == oracle.entry_point(x)


@pytest.mark.gpu
def test_gpu_label_starts_match_oracle(dance_lib):
    from dance_b200 import filtered as F, workloads
    n, vocab = 30000, 300
    offs, labs = workloads.zipf_multilabels(n, vocab, seed=5)
    lo, lp = F.label_points_csr(offs, labs, vocab + 2)  # two empty labels at the end
    got = F.select_label_starts(lo, lp, n, 25, 42)
    want = oracle.label_starts(lo, lp, n, 25, 42)
    assert np.array_equal(got, want)
    assert (got[-2:] == 0xFFFFFFFF).all() and (got[:vocab] < n).all()
    # every start carries its label
    for l in range(0, vocab, 17):
        assert got[l] in set(lp[lo[l]:lo[l + 1]].tolist())
