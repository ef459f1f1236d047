"""GPU parity: every CUDA stage against the CPU oracle on identical inputs.

Bar: integer/index outputs (ids, degrees, medoid, expansion sequences) are
bit-exact; distances are bit-exact as well because the kernels reproduce the
reference's lane-order arithmetic (checked against float64 to 1e-5 relative
separately).  All calls go through the C ABI of libdance_b200.so.
"""
import ctypes

import numpy as np
import pytest

import oracle
from dance_b200 import load, default_params, check, vamana, workloads, formats

pytestmark = pytest.mark.gpu
INVALID = 0xFFFFFFFF
FMAX = np.finfo(np.float32).max


def _t():
    import torch
    return torch


def dev(a):
    torch = _t()
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    return torch.from_numpy(a).cuda()


def host(t, dtype=None):
    a = t.cpu().numpy()
    if dtype == np.uint32:
        return a.view(np.uint32)
    return a


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def _cudart():
    """The CUDA runtime shipped with torch, for raw cudaMemcpy/cudaFree of hand-off pointers."""
    import glob
    import os
    import torch
    base = os.path.dirname(os.path.dirname(torch.__file__))
    cands = sorted(glob.glob(os.path.join(base, "nvidia", "cuda_runtime", "lib", "libcudart.so*")))
    rt = ctypes.CDLL(cands[-1] if cands else "libcudart.so")
    rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    rt.cudaFree.argtypes = [ctypes.c_void_p]
    return rt


def make(dtype, n, dim=None, seed=11, centroids=40):
    if dtype == np.uint8:
        return workloads.clustered_u8(n, dim or 128, centroids=centroids, seed=seed).numpy()
    x = workloads.gaussian_mixture_f32(n, dim or 96, centroids=centroids, seed=seed).numpy()
    return x.astype(np.float16) if dtype == np.float16 else x


def store(x):
    """Device store with 16-byte row stride, as the oracle pads it."""
    torch = _t()
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    s, stride = vamana.padded_store(t)
    return s, stride, vamana.dtype_code(t)


DTYPES = [np.uint8, np.float32, np.float16]


@pytest.fixture(scope="module", autouse=True)
def _lib(dance_lib):
    return dance_lib


@pytest.mark.parametrize("dtype", DTYPES)
def test_medoid_bit_exact(dtype):
    torch = _t()
    lib = load()
    x = make(dtype, 5000)
    s, stride, dt = store(x)
    sc = torch.zeros(1024, dtype=torch.float32, device="cuda")
    cand = torch.zeros(1024, dtype=torch.int32, device="cuda")
    med = torch.zeros(1, dtype=torch.int32, device="cuda")
    check(lib.dance_stage_medoid(dt, P(s), stride, len(x), x.shape[1], 1024, 4096, P(sc), P(cand), P(med), None))
    torch.cuda.synchronize()
    m, osc, ocand = oracle.medoid(x)
    assert np.array_equal(host(cand, np.uint32), ocand)
    assert np.array_equal(host(sc), osc)
    assert int(host(med, np.uint32)[0]) == m


@pytest.mark.parametrize("dtype", DTYPES)
def test_init_bit_exact(dtype):
    torch = _t()
    lib = load()
    x = make(dtype, 3000)
    s, stride, dt = store(x)
    R = 40
    ids = torch.zeros((len(x), R), dtype=torch.int32, device="cuda")
    ds = torch.zeros((len(x), R), dtype=torch.float32, device="cuda")
    deg = torch.zeros(len(x), dtype=torch.int32, device="cuda")
    check(lib.dance_stage_init(dt, P(s), stride, len(x), x.shape[1], R, P(ids), P(ds), P(deg), None))
    oi, od, og = oracle.init(x, R)
    assert np.array_equal(host(ids, np.uint32), oi)
    assert np.array_equal(host(ds), od)
    assert np.array_equal(host(deg, np.uint32), og)


def _round_inputs(x, R, rounds=1, C=None, L=64, S=32):
    """Oracle graph state after `rounds` full rounds (init if 0)."""
    m, _, _ = oracle.medoid(x)
    ids, ds, deg = oracle.init(x, R)
    C = C or R + 16
    for it in range(rounds):
        e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
        w = oracle.replay(x, R, C, np.float32(1.0), ids, ds, deg, *e)
        w = oracle.reverse_merge(x, R, C, *w)[:3]
        ids, ds, deg = oracle.prune(x, R, C, np.float32(1.0), 0, *w)
    return m, ids, ds, deg


def _gpu_search(x, R, L, steps, entry, ids, ds, deg, S, log2h=11):
    torch = _t()
    lib = load()
    s, stride, dt = store(x)
    n = len(x)
    eids = torch.full((n, S), -1, dtype=torch.int32, device="cuda")
    eds = torch.zeros((n, S), dtype=torch.float32, device="cuda")
    ecnt = torch.zeros(n, dtype=torch.int32, device="cuda")
    gi, gd, gg = dev(ids), dev(ds), dev(deg)
    check(lib.dance_stage_search(dt, P(s), stride, n, x.shape[1], R, L, steps, entry, 8, log2h, P(gi), P(gd), P(gg),
                                 P(eids), P(eds), P(ecnt), S, None))
    return host(eids, np.uint32), host(eds), host(ecnt, np.uint32)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rounds", [0, 1])
def test_search_bit_exact(dtype, rounds):
    x = make(dtype, 4000)
    R, L, S = 32, 64, 32
    m, ids, ds, deg = _round_inputs(x, R, rounds)
    ge, gd, gc = _gpu_search(x, R, L, S, m, ids, ds, deg, S)
    oe, od, oc = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    assert np.array_equal(gc, oc)
    mask = np.arange(S)[None, :] < oc[:, None]
    assert np.array_equal(ge[mask], oe[mask])
    assert np.array_equal(gd[mask], od[mask])


def test_search_small_visited_table_still_exact():
    # A 256-entry visited table forgets ids constantly; the pool result must not change.
    x = make(np.uint8, 3000)
    R, L, S = 32, 64, 32
    m, ids, ds, deg = _round_inputs(x, R, 1)
    ge, gd, gc = _gpu_search(x, R, L, S, m, ids, ds, deg, S, log2h=8)
    oe, od, oc = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    assert np.array_equal(gc, oc)
    mask = np.arange(S)[None, :] < oc[:, None]
    assert np.array_equal(ge[mask], oe[mask])


def test_search_config_shape_r64_l100():
    x = make(np.float32, 6000)
    R, L, S = 64, 100, 64
    m, ids, ds, deg = _round_inputs(x, R, 1, C=80, L=L, S=S)
    ge, gd, gc = _gpu_search(x, R, L, S, m, ids, ds, deg, S)
    oe, od, oc = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    assert np.array_equal(gc, oc)
    mask = np.arange(S)[None, :] < oc[:, None]
    assert np.array_equal(ge[mask], oe[mask]) and np.array_equal(gd[mask], od[mask])


def _gpu_replay(x, R, C, alpha, ids, ds, deg, eids, eds, ecnt):
    torch = _t()
    lib = load()
    s, stride, dt = store(x)
    n = len(x)
    wid = torch.zeros((n, C), dtype=torch.int32, device="cuda")
    wd = torch.zeros((n, C), dtype=torch.float32, device="cuda")
    wdeg = torch.zeros(n, dtype=torch.int32, device="cuda")
    keep = [dev(a) for a in (ids, ds, deg, eids, eds, ecnt)]  # alive until the kernels finish
    check(lib.dance_stage_replay(dt, P(s), stride, n, x.shape[1], R, C, ctypes.c_float(alpha), *map(P, keep[:6]),
                                 eids.shape[1], P(wid), P(wd), P(wdeg), None))
    torch.cuda.synchronize()
    return host(wid, np.uint32), host(wd), host(wdeg, np.uint32)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("alpha", [1.0, 1.2])
def test_replay_bit_exact(dtype, alpha):
    x = make(dtype, 4000)
    R, L, S, C = 32, 64, 32, 48
    m, ids, ds, deg = _round_inputs(x, R, 1, C=C)
    e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    g = _gpu_replay(x, R, C, np.float32(alpha), ids, ds, deg, *e)
    o = oracle.replay(x, R, C, np.float32(alpha), ids, ds, deg, *e)
    for a, b in zip(g, o):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("dim,R,S,C", [(128, 64, 64, 80), (32, 24, 20, 56), (100, 40, 88, 128), (16, 8, 8, 12)])
def test_replay_tensor_core_shapes_u8(dim, R, S, C, monkeypatch):
    # the uint8 replay on the tcgen05 tensor cores (the default where it fits)
    # (R + S <= 128, C <= 128, rows of at most 128 bytes): the benchmarked
    # shape, small dimensions, an odd number of 16-byte chunks (zero-padded
    # K), a full 128-row cache with the widest work row, and a tiny row
    monkeypatch.setenv("DANCE_REPLAY_UMMA", "1")
    x = make(np.uint8, 3000, dim=dim, centroids=24)
    L = max(S, 32)
    m, ids, ds, deg = _round_inputs(x, R, 1, C=C)
    e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    for alpha in (1.0, 1.2):
        g = _gpu_replay(x, R, C, np.float32(alpha), ids, ds, deg, *e)
        o = oracle.replay(x, R, C, np.float32(alpha), ids, ds, deg, *e)
        for a, b in zip(g, o):
            assert np.array_equal(a, b)


def _gpu_merge(x, R, C, wid, wd, wdeg, prm=None):
    import ctypes as ct
    lib = load()
    s, stride, dt = store(x)
    n = len(x)
    a, b, c = dev(wid), dev(wd), dev(wdeg)
    edges = ct.c_uint64(0)
    p = prm or default_params()
    check(lib.dance_stage_reverse_merge(dt, P(s), stride, n, x.shape[1], R, C, ct.byref(p), None, P(a), P(b), P(c),
                                        ct.byref(edges), None))
    return host(a, np.uint32), host(b), host(c, np.uint32), int(edges.value)


@pytest.mark.parametrize("dtype", DTYPES)
def test_reverse_merge_bit_exact(dtype):
    x = make(dtype, 4000)
    R, L, S, C = 32, 64, 32, 48
    m, ids, ds, deg = _round_inputs(x, R, 1, C=C)
    e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    w = oracle.replay(x, R, C, np.float32(1.0), ids, ds, deg, *e)
    g = _gpu_merge(x, R, C, *w)
    o = oracle.reverse_merge(x, R, C, *w)
    assert g[3] == o[3]
    for a, b in zip(g[:3], o[:3]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("indeg", [600, 20000])
def test_reverse_merge_heavy_and_huge_targets(indeg):
    # Force one target with `indeg` sources: > 512 goes to the block-sorted
    # heavy path, > 16384 to the in-place global sort.
    n = indeg + 50
    x = make(np.uint8, n, dim=16, seed=3)
    R, C = 4, 8
    rng = np.random.default_rng(0)
    wid = np.full((n, C), INVALID, np.uint32)
    wd = np.full((n, C), FMAX, np.float32)
    wdeg = np.zeros(n, np.uint32)
    for s in range(1, n):
        wid[s, 0] = 0
        wid[s, 1] = rng.integers(1, n)
        if wid[s, 1] == s:
            wid[s, 1] = 0 if s != 0 else 1
        wd[s, 0] = oracle.distance(x[s], x[0])
        wd[s, 1] = oracle.distance(x[s], x[wid[s, 1]])
        wdeg[s] = 2
    g = _gpu_merge(x, R, C, wid, wd, wdeg)
    o = oracle.reverse_merge(x, R, C, wid, wd, wdeg)
    assert g[3] == o[3]
    for a, b in zip(g[:3], o[:3]):
        assert np.array_equal(a, b)
    # heavy cap option (PRO6000_100M / FILTERED_PAPER profiles)
    prm = default_params(reverse_heavy_cap=1, reverse_heavy_threshold=256, reverse_heavy_sample=384)
    oprm = oracle.params(reverse_heavy_cap=1, reverse_heavy_threshold=256, reverse_heavy_sample=384)
    g = _gpu_merge(x, R, C, wid, wd, wdeg, prm)
    o = oracle.reverse_merge(x, R, C, wid, wd, wdeg, oprm)
    for a, b in zip(g[:3], o[:3]):
        assert np.array_equal(a, b)


def _gpu_prune(x, R, C, alpha, mindeg, wid, wd, wdeg):
    torch = _t()
    lib = load()
    s, stride, dt = store(x)
    n = len(x)
    ids = torch.zeros((n, R), dtype=torch.int32, device="cuda")
    ds = torch.zeros((n, R), dtype=torch.float32, device="cuda")
    deg = torch.zeros(n, dtype=torch.int32, device="cuda")
    keep = [dev(a) for a in (wid, wd, wdeg)]  # alive until the kernel finishes
    check(lib.dance_stage_prune(dt, P(s), stride, n, x.shape[1], R, C, ctypes.c_float(alpha), mindeg, *map(P, keep),
                                P(ids), P(ds), P(deg), None))
    torch.cuda.synchronize()
    return host(ids, np.uint32), host(ds), host(deg, np.uint32)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("alpha,mindeg", [(1.0, 0), (1.2, 64)])
def test_prune_bit_exact(dtype, alpha, mindeg):
    x = make(dtype, 4000)
    R, L, S, C = 32, 64, 32, 48
    m, ids, ds, deg = _round_inputs(x, R, 1, C=C)
    e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    w = oracle.replay(x, R, C, np.float32(alpha), ids, ds, deg, *e)
    w = oracle.reverse_merge(x, R, C, *w)[:3]
    g = _gpu_prune(x, R, C, np.float32(alpha), mindeg, *w)
    o = oracle.prune(x, R, C, np.float32(alpha), mindeg, *w)
    for a, b in zip(g, o):
        assert np.array_equal(a, b)


def _gpu_build(x, R, L, C, S, prm=None):
    s, stride, dt = store(x)
    g, deg, ds, med = vamana.build_resident(s, x.shape[1], stride, R, L, C, S, params=prm)
    return host(g, np.uint32), host(deg, np.uint32), host(ds), med


@pytest.mark.parametrize("dtype", DTYPES)
def test_full_build_bit_exact(dtype):
    x = make(dtype, 6000)
    R, L, C, S = 32, 64, 48, 32
    g = _gpu_build(x, R, L, C, S)
    o = oracle.build_graph(x, R, L, C, S)
    assert g[3] == o[3]
    assert np.array_equal(g[1], o[1])
    assert np.array_equal(g[0], o[0])
    assert np.array_equal(g[2], o[2])


def test_replay_tensor_core_mask_chunks(monkeypatch):
    # the masks/bits kernels run over chunks of vertices (2^20 by default);
    # chunks of 777 vertices exercise the chunk offsets on a small input
    monkeypatch.setenv("DANCE_REPLAY_MASK_CHUNK", "777")
    x = make(np.uint8, 3000, centroids=24)
    R, L, S, C = 64, 100, 64, 80
    m, ids, ds, deg = _round_inputs(x, R, 1, C=C)
    e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    g = _gpu_replay(x, R, C, np.float32(1.2), ids, ds, deg, *e)
    o = oracle.replay(x, R, C, np.float32(1.2), ids, ds, deg, *e)
    for a, b in zip(g, o):
        assert np.array_equal(a, b)
    gb = _gpu_build(x, R, L, C, S)
    ob = oracle.build_graph(x, R, L, C, S)
    assert gb[3] == ob[3] and np.array_equal(gb[0], ob[0]) and np.array_equal(gb[1], ob[1])


@pytest.mark.parametrize("tensor_core_replay", ["0", "1"])
def test_full_build_config_shape_u8(tensor_core_replay, monkeypatch):
    # BASELINE config shape (R64 L100 C80 STEPS64) at a size the oracle
    # finishes quickly, with the pair-by-pair and the tensor-core replay
    monkeypatch.setenv("DANCE_REPLAY_UMMA", tensor_core_replay)
    x = make(np.uint8, 8000, centroids=64)
    R, L, C, S = 64, 100, 80, 64
    g = _gpu_build(x, R, L, C, S)
    o = oracle.build_graph(x, R, L, C, S)
    assert g[3] == o[3] and np.array_equal(g[0], o[0]) and np.array_equal(g[1], o[1])


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_full_build_config_shape_float(dtype):
    # float32 (QUALITY) and float16 storage (FAST_SMALL) whole builds at the
    # benchmarked shape R64 L100 C80 STEPS64: the four-lane float prune and
    # replay at C=80, the last-round fill to 64, the heavy-cap-off merge
    x = make(dtype, 8000, centroids=64)
    R, L, C, S = 64, 100, 80, 64
    g = _gpu_build(x, R, L, C, S)
    o = oracle.build_graph(x, R, L, C, S)
    assert g[3] == o[3] and np.array_equal(g[1], o[1]) and np.array_equal(g[0], o[0])
    assert np.array_equal(g[2], o[2])


def _golden_cfgshape_cases():
    import json
    from pathlib import Path
    m = Path(__file__).resolve().parent / "golden" / "manifest.json"
    cases = json.loads(m.read_text()) if m.exists() else []
    return [c for c in cases if "data_spec" in c and c.get("builder", "vnew2") == "vnew2"]


@pytest.mark.parametrize("case", _golden_cfgshape_cases(), ids=lambda c: c["file"])
def test_config_shape_build_against_reference_golden(case):
    """The GPU build at R64 L100 C80 STEPS64 (N=20000) against the reference's
    own build of the same input: bit-exact to the oracle (product rule), row
    agreement with the reference no worse than the reference's agreement with
    itself over two runs, minus the pool tie-break margin, and recall@10 at
    L=100 within 0.005 of the reference graph's on the same queries."""
    import torch
    from pathlib import Path
    from tests.golden.make_golden import case_data, case_graph, agreement, gen_queries
    z = np.load(Path(__file__).resolve().parent / "golden" / case["file"])
    x = case_data(case, z)
    if case["storage"] == "f16":
        x = x.astype(np.float16)
    R, L, C, S = case["R"], case["L"], case["C"], case["STEPS"]
    prm = default_params()
    prm.iters = case["iters"]
    g = _gpu_build(x, R, L, C, S, prm)
    o = oracle.build_graph(x, R, L, C, S, oracle.params(iters=case["iters"]))
    assert g[3] == o[3] and np.array_equal(g[0], o[0]) and np.array_equal(g[1], o[1])
    rg, rd = case_graph(z), z["degree"].astype(np.uint32)
    rows, sets = agreement(g[0], g[1], rg, rd)
    selfagr = case["reference_self_agreement"]
    assert rows >= selfagr["rows"] - 0.02, (rows, selfagr)
    assert sets >= selfagr["row_sets"] - 0.02, (sets, selfagr)
    if case["iters"] == 4:
        q = torch.from_numpy(gen_queries(case["data_spec"], 1000, seed=77).astype(x.dtype))
        xt = torch.from_numpy(np.ascontiguousarray(x))
        gt, _ = workloads.brute_force_knn(xt.cuda(), q.cuda(), 10)
        st, stride, _ = store(x)
        ours, _ = vamana.search_queries(st, x.shape[1], stride, dev(g[0]), R, g[3], q.cuda(), 100, 10)
        theirs, _ = vamana.search_queries(st, x.shape[1], stride, dev(rg), R, int(z["medoid"]), q.cuda(), 100, 10)
        r_ours = vamana.recall_at_k(ours.cpu().numpy(), gt.cpu().numpy())
        r_ref = vamana.recall_at_k(theirs.cpu().numpy(), gt.cpu().numpy())
        assert abs(r_ours - r_ref) <= 0.005, (r_ours, r_ref)


@pytest.mark.parametrize("dtype,dim", [(np.float32, 100), (np.uint8, 100), (np.float32, 20), (np.float16, 90),
                                       (np.float32, 128), (np.float16, 256)])
def test_padded_rows(dtype, dim):
    x = make(dtype, 2000, dim=dim)
    g = _gpu_build(x, 16, 32, 24, 16)
    o = oracle.build_graph(x, 16, 32, 24, 16)
    assert g[3] == o[3] and np.array_equal(g[0], o[0])


@pytest.mark.parametrize("n", [1, 2, 5, 40])
def test_tiny_inputs(n):
    x = make(np.uint8, max(n, 1), dim=16)[:n]
    g = _gpu_build(x, 8, 16, 12, 8)
    o = oracle.build_graph(x, 8, 16, 12, 8)
    assert g[3] == o[3] and np.array_equal(g[0], o[0]) and np.array_equal(g[1], o[1])


def test_reference_abi_matches_resident_build():
    x = make(np.uint8, 5000)
    R, L, C, S = 32, 64, 48, 32
    g, deg = vamana.gpu_vamana_vnew2_build(x, R, L, C, S)
    med = vamana.gpu_vamana_vnew2_get_last_medoid()
    o = oracle.build_graph(x, R, L, C, S)
    assert med == o[3] and np.array_equal(g, o[0]) and np.array_equal(deg, o[1])
    st = vamana.gpu_vamana_vnew2_get_last_stats()
    assert st["gpu_build_seconds"] > 0 and st["distance_computations"] > 0
    xf = make(np.float32, 3000)
    gf, degf = vamana.gpu_vamana_vnew2_build_float(xf, R, L, C, S)
    of = oracle.build_graph(xf, R, L, C, S)
    assert np.array_equal(gf, of[0]) and np.array_equal(degf, of[1])
    # STEPS > L is clamped, not an error
    g2, _ = vamana.gpu_vamana_vnew2_build(x[:500], 16, 16, 24, 40)
    assert formats.audit_graph(g2, _, 16, 0)["invalid"] == 0


def test_device_handoff_variant():
    torch = _t()
    lib = load()
    x = make(np.uint8, 3000)
    R, L, C, S = 32, 64, 48, 32
    dd, dg, dgr = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    rc = lib.gpu_vamana_vnew2_build_device(ctypes.c_void_p(x.ctypes.data), len(x), x.shape[1], R, L, C, S,
                                           ctypes.byref(dd), ctypes.byref(dg), ctypes.byref(dgr))
    assert rc == 0
    g = np.empty((len(x), R), np.uint32)
    d = np.empty(len(x), np.uint32)
    back = np.empty_like(x)
    rt = _cudart()
    for dst, src, nbytes in [(g, dg, g.nbytes), (d, dgr, d.nbytes), (back, dd, back.nbytes)]:
        assert rt.cudaMemcpy(ctypes.c_void_p(dst.ctypes.data), src, ctypes.c_size_t(nbytes), 2) == 0
    o = oracle.build_graph(x, R, L, C, S)
    assert np.array_equal(g, o[0]) and np.array_equal(d, o[1]) and np.array_equal(back, x)
    for p in (dd, dg, dgr):
        assert rt.cudaFree(p) == 0


@pytest.mark.parametrize("dtype", [np.uint8, np.float32])
def test_distances_within_1e5_relative_of_float64(dtype):
    x = make(dtype, 2000)
    g, deg, ds, med = _gpu_build(x, 16, 32, 24, 16)
    rows = np.repeat(np.arange(len(x)), 16).reshape(-1, 16)
    mask = g != INVALID
    a = x[rows[mask]].astype(np.float64)
    b = x[g[mask]].astype(np.float64)
    exact = ((a - b) ** 2).sum(1)
    got = ds[mask].astype(np.float64)
    assert (np.abs(got - exact) <= 1e-5 * np.maximum(exact, 1e-30)).all()


@pytest.mark.parametrize("dtype", [np.uint8, np.float32])
def test_query_search_matches_oracle_and_recall(dtype):
    torch = _t()
    x = make(dtype, 8000, centroids=64)
    q = (workloads.clustered_u8(300, 128, centroids=64, seed=11, stream_offset=1) if dtype == np.uint8 else
         workloads.gaussian_mixture_f32(300, 96, centroids=64, seed=11, stream_offset=1)).numpy()
    R, L, C, S = 32, 64, 48, 32
    g, deg, ds, med = _gpu_build(x, R, L, C, S)
    s, stride, dt = store(x)
    gdev = dev(g)
    ids, dd = vamana.search_queries(s, x.shape[1], stride, gdev, R, med, torch.from_numpy(q).cuda(), 100, 10)
    oi, od = oracle.search_queries(x, g, R, med, q, 100, 10)
    assert np.array_equal(host(ids, np.uint32), oi)
    gt, _ = workloads.brute_force_knn(torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(), 10)
    assert vamana.recall_at_k(oi, gt.cpu().numpy()) >= 0.97


def test_kernel_launches_counted():
    lib = load()
    before = lib.dance_kernel_launch_count()
    x = make(np.uint8, 1000)
    _gpu_build(x, 16, 32, 24, 16)
    assert lib.dance_kernel_launch_count() > before


def test_search_large_pool_and_degree():
    # 8 pool entries per lane (L=256) and rows wider than one 64-candidate batch (R=96)
    x = make(np.float32, 5000)
    R, L, S = 96, 256, 80
    m, ids, ds, deg = _round_inputs(x, R, 1, C=112, L=L, S=S)
    ge, gd, gc = _gpu_search(x, R, L, S, m, ids, ds, deg, S)
    oe, od, oc = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    assert np.array_equal(gc, oc)
    mask = np.arange(S)[None, :] < oc[:, None]
    assert np.array_equal(ge[mask], oe[mask]) and np.array_equal(gd[mask], od[mask])


def test_pool_capacity_limit_is_an_error():
    from dance_b200 import DanceError
    x = make(np.uint8, 500)
    with pytest.raises(DanceError):
        _gpu_build(x, 16, 300, 24, 16)
