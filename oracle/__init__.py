"""ctypes binding of the CPU parity oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference leg, never by the product.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_I = ctypes.c_int
_F = ctypes.c_float

_SIGS = {
    "oracle_default_params": (None, [_P]),
    "oracle_reset_counters": (None, []),
    "oracle_get_counters": (None, [_P]),
    "oracle_distance": (_F, [_I, _P, _P, _U32]),
    "oracle_float_to_half": (None, [_P, _P, _U64]),
    "oracle_half_selftest": (_U64, [_U64]),
    "oracle_hash_u32": (_U32, [_U32]),
    "oracle_hash_edge32": (_U32, [_U32, _U32, _U64]),
    "oracle_merge_edges": (_I, [_P, _P, _U64, _U32, _U32, _U64, _P, _P]),
    "oracle_det_neighbor": (_U32, [_U32, _U32, _U32]),
    "oracle_medoid": (_U32, [_I, _P, _U64, _U32, _U32, _U32, _U32, _P, _P, _I]),
    "oracle_init": (_I, [_I, _P, _U64, _U32, _U32, _U32, _P, _P, _P, _I]),
    "oracle_search": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _I, _P, _P, _P, _P, _P, _P,
                           _U32, _I]),
    "oracle_replay": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _F, _P, _P, _P, _P, _P, _P, _U32, _P, _P, _P,
                           _I]),
    "oracle_reverse_merge": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P, _I]),
    "oracle_prune": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _F, _U32, _P, _P, _P, _P, _P, _P, _I]),
    "oracle_build": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _P, _I, _I, _P, _P, _P, _P]),
    "oracle_search_queries": (_I, [_I, _P, _U64, _U32, _U32, _P, _U32, _U32, _P, _U64, _U32, _U32, _U32, _P, _P,
                                   _I]),
    "oracle_filtered_random_graph": (None, [_U32, _U32, _U32, _U32, _P, _P]),
    "oracle_filtered_round": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _F, _P, _P, _P, _U32,
                                   _U32, _U32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I]),
    "oracle_filtered_build": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _F, _P, _P, _P, _U32,
                                   _U32, _U32, _P, _P, _U32, _I, _P, _P]),
    "oracle_filtered_task_search": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _U32, _U32, _P,
                                         _P, _P, _P, _I]),
    "oracle_filtered_ordinary_search": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _U32,
                                             _U32, _U32, _P, _P, _P, _P, _I]),
    "oracle_entry_point": (_U32, [_I, _P, _U64, _U32, _U32]),
    "oracle_label_starts": (None, [_P, _P, _U32, _U32, _U32, _U64, _P]),
    "oracle_kmeanspp_seed": (None, [_P, _U64, _U64, _U32, _U32, _U64, _P, _P]),
    "oracle_kmeans_lloyd": (None, [_P, _U64, _U64, _U32, _U32, _U32, _P, _P, _P]),
    "oracle_partition_assign": (None, [_I, _P, _U64, _U64, _U32, _P, _U32, _U32, _P, _P]),
    "oracle_partition_buckets": (None, [_P, _U64, _U32, _U32, _P, _P]),
    "oracle_stitched_global_prune": (_I, [_I, _P, _U64, _U32, _U32, _P, _P, _P, _P, _U32, _U32, _F, _P, _P]),
    "oracle_filtered_prune_lists": (_I, [_I, _P, _U64, _U32, _U32, _U32, _F, _P, _P, _U32, _P, _U32, _P, _P, _P,
                                         _P, _P]),
}

_lib = None


def build(force: bool = False) -> Path:
    src = HERE / "vamana_oracle.cpp"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = ctypes.CDLL(str(LIB))
        for k, (r, a) in _SIGS.items():
            f = getattr(lib, k)
            f.restype = r
            f.argtypes = a
        _lib = lib
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p(0)


DTYPE = {np.dtype(np.uint8): 0, np.dtype(np.float16): 1, np.dtype(np.float32): 2}


def _store(data: np.ndarray):
    """Oracle rows use the same 16-byte padded stride as the product."""
    data = np.ascontiguousarray(data)
    n, dim = data.shape
    es = data.dtype.itemsize
    stride = (dim * es + 15) // 16 * 16
    if stride != dim * es:
        pad = np.zeros((n, stride // es), dtype=data.dtype)
        pad[:, :dim] = data
        data = pad
    return data, stride, DTYPE[np.dtype(data.dtype)]


class Params(ctypes.Structure):
    _fields_ = [("iters", _U32), ("alpha", _F), ("init_random_seeds", _U32), ("final_min_degree", _U32),
                ("medoid_candidates", _U32), ("medoid_samples", _U32), ("coarse_warmup_iters", _U32),
                ("warmup_expand_steps", _U32), ("reverse_heavy_cap", _U32), ("reverse_heavy_threshold", _U32),
                ("reverse_heavy_sample", _U32), ("visited_log2", _U32), ("reserved", _U32 * 8)]


def params(**kw) -> Params:
    p = Params()
    load().oracle_default_params(ctypes.byref(p))
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def threads() -> int:
    return int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1))


def distance(a: np.ndarray, b: np.ndarray) -> float:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b, dtype=a.dtype)
    return float(load().oracle_distance(DTYPE[a.dtype], _p(a), _p(b), a.shape[-1]))


def float_to_half(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    load().oracle_float_to_half(_p(x), _p(out), x.size)
    return out.view(np.float16)


def medoid(data, num_candidates=1024, num_samples=4096):
    d, stride, dt = _store(data)
    n, dim = data.shape
    nc = min(num_candidates, n)
    scores = np.zeros(nc, np.float32)
    cand = np.zeros(nc, np.uint32)
    m = load().oracle_medoid(dt, _p(d), stride, n, dim, num_candidates, num_samples, _p(scores), _p(cand), threads())
    return int(m), scores, cand


def init(data, R):
    d, stride, dt = _store(data)
    n, dim = data.shape
    ids = np.zeros((n, R), np.uint32)
    ds = np.zeros((n, R), np.float32)
    deg = np.zeros(n, np.uint32)
    load().oracle_init(dt, _p(d), stride, n, dim, R, _p(ids), _p(ds), _p(deg), threads())
    return ids, ds, deg


def search(data, R, L, steps, entry, seeds, cur_ids, cur_dists, degree, exp_stride, pool_mode=0):
    d, stride, dt = _store(data)
    n, dim = data.shape
    eids = np.zeros((n, exp_stride), np.uint32)
    eds = np.zeros((n, exp_stride), np.float32)
    ecnt = np.zeros(n, np.uint32)
    rc = load().oracle_search(dt, _p(d), stride, n, dim, R, L, steps, entry, seeds, pool_mode,
                              _p(np.ascontiguousarray(cur_ids, np.uint32)),
                              _p(np.ascontiguousarray(cur_dists, np.float32)),
                              _p(np.ascontiguousarray(degree, np.uint32)), _p(eids), _p(eds), _p(ecnt), exp_stride,
                              threads())
    assert rc == 0
    return eids, eds, ecnt


def replay(data, R, C, alpha, cur_ids, cur_dists, degree, exp_ids, exp_dists, exp_count):
    d, stride, dt = _store(data)
    n, dim = data.shape
    wid = np.zeros((n, C), np.uint32)
    wd = np.zeros((n, C), np.float32)
    wdeg = np.zeros(n, np.uint32)
    rc = load().oracle_replay(dt, _p(d), stride, n, dim, R, C, alpha,
                              _p(np.ascontiguousarray(cur_ids, np.uint32)),
                              _p(np.ascontiguousarray(cur_dists, np.float32)),
                              _p(np.ascontiguousarray(degree, np.uint32)),
                              _p(np.ascontiguousarray(exp_ids, np.uint32)),
                              _p(np.ascontiguousarray(exp_dists, np.float32)),
                              _p(np.ascontiguousarray(exp_count, np.uint32)), exp_ids.shape[1], _p(wid), _p(wd),
                              _p(wdeg), threads())
    assert rc == 0
    return wid, wd, wdeg


def reverse_merge(data, R, C, work_ids, work_dists, work_deg, prm=None):
    d, stride, dt = _store(data)
    n, dim = data.shape
    wid = np.array(work_ids, dtype=np.uint32, copy=True, order="C")
    wd = np.array(work_dists, dtype=np.float32, copy=True, order="C")
    wdeg = np.array(work_deg, dtype=np.uint32, copy=True, order="C")
    edges = ctypes.c_uint64(0)
    rc = load().oracle_reverse_merge(dt, _p(d), stride, n, dim, R, C, ctypes.byref(prm) if prm else None, _p(wid),
                                     _p(wd), _p(wdeg), ctypes.byref(edges), threads())
    assert rc == 0
    return wid, wd, wdeg, int(edges.value)


def prune(data, R, C, alpha, min_degree, work_ids, work_dists, work_deg):
    d, stride, dt = _store(data)
    n, dim = data.shape
    ids = np.zeros((n, R), np.uint32)
    ds = np.zeros((n, R), np.float32)
    deg = np.zeros(n, np.uint32)
    rc = load().oracle_prune(dt, _p(d), stride, n, dim, R, C, alpha, min_degree,
                             _p(np.ascontiguousarray(work_ids, np.uint32)),
                             _p(np.ascontiguousarray(work_dists, np.float32)),
                             _p(np.ascontiguousarray(work_deg, np.uint32)), _p(ids), _p(ds), _p(deg), threads())
    assert rc == 0
    return ids, ds, deg


def build_graph(data, R, L, C, STEPS, prm=None, pool_mode=0, nthreads=None):
    """Whole oracle build; returns (graph, degree, dists, medoid)."""
    d, stride, dt = _store(data)
    n, dim = data.shape
    g = np.zeros((n, R), np.uint32)
    deg = np.zeros(n, np.uint32)
    ds = np.zeros((n, R), np.float32)
    med = ctypes.c_uint32(0)
    rc = load().oracle_build(dt, _p(d), stride, n, dim, R, L, C, STEPS, ctypes.byref(prm) if prm else None,
                             pool_mode, nthreads or threads(), _p(g), _p(deg), _p(ds), ctypes.byref(med))
    assert rc == 0, rc
    return g, deg, ds, int(med.value)


def search_queries(data, graph, R, start, queries, L, K):
    d, stride, dt = _store(data)
    q, qstride, _ = _store(np.ascontiguousarray(queries, dtype=data.dtype))
    n, dim = data.shape
    nq = queries.shape[0]
    ids = np.zeros((nq, K), np.uint32)
    ds = np.zeros((nq, K), np.float32)
    load().oracle_search_queries(dt, _p(d), stride, n, dim, _p(np.ascontiguousarray(graph, np.uint32)), R, start,
                                 _p(q), qstride, nq, L, K, _p(ids), _p(ds), threads())
    return ids, ds


def merge_edges(src, dst, nnodes, max_degree, seed=0x9e3779b97f4a7c15):
    """Reference shard-merge rule on global edges -> (rows nnodes x max_degree, degrees)."""
    src = np.ascontiguousarray(src, np.uint32)
    dst = np.ascontiguousarray(dst, np.uint32)
    rows = np.zeros((nnodes, max_degree), np.uint32)
    deg = np.zeros(nnodes, np.uint32)
    load().oracle_merge_edges(_p(src), _p(dst), len(src), nnodes, max_degree, seed, _p(rows), _p(deg))
    return rows, deg


def counters():
    out = np.zeros(6, np.uint64)
    load().oracle_get_counters(_p(out))
    return dict(zip(["search_evals", "expansions", "pair_evals", "reverse_evals", "reverse_edges",
                     "seed_mismatch"], out.tolist()))


def reset_counters():
    load().oracle_reset_counters()


def stitched_remap(rows, ids, local_graph, local_degree, r_small, r_out, counters):
    """One label's rows appended to the global rows by the reference rule
    (apps/utils/gpu_stitched_vamana_index.cpp:316-341): the first
    min(deg, Rstitched) local neighbours, invalid ids and self loops skipped,
    ids already in the row not repeated."""
    n = len(ids)
    for i in range(n):
        row = rows[ids[i]]
        deg = min(int(local_degree[i]), r_out)
        for j in range(deg):
            nb = int(local_graph[i * r_small + j]) if local_graph.ndim == 1 else int(local_graph[i, j])
            if nb == 0xFFFFFFFF or nb >= n:
                counters["remap_invalid_local_ids"] += 1
                continue
            if ids[nb] == ids[i]:
                counters["remap_self_loops"] += 1
                continue
            g = int(ids[nb])
            if g not in row:
                row.append(g)
            else:
                counters["remap_duplicate_edges"] += 1


def stitched(data, label_points, r_small, l_small, r_out, C, steps, prm=None):
    """Reference label loop (:276-341) over oracle builds of each label's
    points; returns (rows: list of lists, label medoids, counters)."""
    r_out = max(r_out, r_small)
    rows = [[] for _ in range(data.shape[0])]
    medoids = []
    counters = dict(remap_invalid_local_ids=0, remap_self_loops=0, remap_duplicate_edges=0)
    for ids in label_points:
        ids = [int(i) for i in ids]
        if not ids:
            medoids.append(0)
            continue
        g, deg, _, med = build_graph(np.ascontiguousarray(data[ids]), r_small, l_small, C, steps, prm)
        medoids.append(ids[med] if med < len(ids) else ids[0])
        stitched_remap(rows, ids, g, deg, r_small, r_out, counters)
    return rows, medoids, counters


def entry_point(data) -> int:
    """DiskANN's calculate_entry_point as label_starts.cu restates it."""
    d, stride, dt = _store(data)
    n, dim = data.shape
    return int(load().oracle_entry_point(dt, _p(d), stride, n, dim))


def label_starts(label_offsets, label_points, num_points, num_candidates=25, seed=42):
    off = np.ascontiguousarray(label_offsets, np.uint32)
    pts = np.ascontiguousarray(label_points, np.uint32)
    out = np.zeros(max(len(off) - 1, 1), np.uint32)
    load().oracle_label_starts(_p(off), _p(pts), len(off) - 1, num_points, num_candidates, seed, _p(out))
    return out[:len(off) - 1]


def stitched_global_prune(data, row_offsets, row_ids, point_label_offsets, point_labels, range_, maxc=750,
                          alpha=1.2):
    """DiskANN's patched prune_all_neighbors over a union CSR graph (see the C
    restatement); labels as a per-point CSR with ascending labels, or None.
    Returns (rows N x range with 0xFFFFFFFF padding, degrees)."""
    d, stride, dt = _store(data)
    n, dim = data.shape
    ro = np.ascontiguousarray(row_offsets, np.uint64)
    ri = np.ascontiguousarray(row_ids, np.uint32)
    lo = None if point_label_offsets is None else np.ascontiguousarray(point_label_offsets, np.uint32)
    lb = None if point_labels is None else np.ascontiguousarray(point_labels, np.uint32)
    out = np.zeros((n, range_), np.uint32)
    deg = np.zeros(n, np.uint32)
    rc = load().oracle_stitched_global_prune(dt, _p(d), stride, n, dim, _p(ro), _p(ri), _p(lo), _p(lb), range_, maxc,
                                             np.float32(alpha), _p(out), _p(deg))
    assert rc == 0, rc
    return out, deg


# ---------------------------------------------------------------- GPU-FilteredVamana
class FilteredLabels:
    """Per-point label CSR (each row strictly increasing) + per-label start ids."""

    def __init__(self, offsets, labels, starts, num_labels, universal=0xFFFFFFFF, global_start=0xFFFFFFFF):
        self.offsets = np.ascontiguousarray(offsets, np.uint32)
        self.labels = np.ascontiguousarray(labels, np.uint32)
        self.starts = np.ascontiguousarray(starts, np.uint32)
        self.num_labels = int(num_labels)
        self.universal = int(universal)
        self.global_start = int(global_start)


def filtered_random_graph(n, R, initial_degree=16, seed=42):
    g = np.zeros((n, R), np.uint32)
    d = np.zeros(n, np.uint32)
    load().oracle_filtered_random_graph(n, R, initial_degree, seed, _p(g), _p(d))
    return g, d


def filtered_work_width(C):
    """The reference's GPU work width: min(C, 128) (src/gpu_vamana_filtered.cu:6563-6567)."""
    return min(int(C), 128)


def filtered_round(data, lab: FilteredLabels, R, L, FL, C, STEPS, alpha, graph, degree):
    """One canonical round; C is the work width.  Returns dict of graph, degree,
    work rows (ids, dists, lengths) and the forward-pruned graph."""
    d, stride, dt = _store(data)
    n, dim = data.shape
    out = dict(graph=np.zeros((n, R), np.uint32), degree=np.zeros(n, np.uint32),
               work=np.zeros((n, C), np.uint32), work_d=np.zeros((n, C), np.float32),
               work_deg=np.zeros(n, np.uint32), fwd=np.zeros((n, R), np.uint32), fwd_deg=np.zeros(n, np.uint32))
    rc = load().oracle_filtered_round(dt, _p(d), stride, n, dim, R, L, FL, C, STEPS, alpha, _p(lab.offsets),
                                      _p(lab.labels), _p(lab.starts), lab.num_labels, lab.universal,
                                      lab.global_start, _p(np.ascontiguousarray(graph, np.uint32)),
                                      _p(np.ascontiguousarray(degree, np.uint32)), _p(out["graph"]),
                                      _p(out["degree"]), _p(out["work"]), _p(out["work_d"]), _p(out["work_deg"]),
                                      _p(out["fwd"]), _p(out["fwd_deg"]), threads())
    assert rc == 0
    return out


def filtered_build(data, lab: FilteredLabels, R, L, FL, C, STEPS, alpha, graph=None, degree=None, rounds=3):
    """Canonical filtered build; C is the caller's C (clamped to 128 here)."""
    d, stride, dt = _store(data)
    n, dim = data.shape
    g = np.zeros((n, R), np.uint32)
    deg = np.zeros(n, np.uint32)
    gi = None if graph is None else np.ascontiguousarray(graph, np.uint32)
    di = None if degree is None else np.ascontiguousarray(degree, np.uint32)
    rc = load().oracle_filtered_build(dt, _p(d), stride, n, dim, R, L, FL, filtered_work_width(C), STEPS, alpha,
                                      _p(lab.offsets), _p(lab.labels), _p(lab.starts), lab.num_labels,
                                      lab.universal, lab.global_start, _p(gi), _p(di), rounds, threads(), _p(g),
                                      _p(deg))
    assert rc == 0
    return g, deg


def filtered_task_search(data, lab: FilteredLabels, R, FL, STEPS, graph, degree):
    d, stride, dt = _store(data)
    n, dim = data.shape
    keep = min(min(FL, 32), 8)
    T = int(lab.offsets[-1])
    ids = np.zeros((T, keep), np.uint32)
    ds = np.zeros((T, keep), np.float32)
    load().oracle_filtered_task_search(dt, _p(d), stride, n, dim, R, FL, STEPS, _p(lab.offsets), _p(lab.labels),
                                       _p(lab.starts), lab.num_labels, lab.universal,
                                       _p(np.ascontiguousarray(graph, np.uint32)),
                                       _p(np.ascontiguousarray(degree, np.uint32)), _p(ids), _p(ds), threads())
    return ids, ds


def filtered_ordinary_search(data, lab: FilteredLabels, R, L, FL, STEPS, graph, degree):
    d, stride, dt = _store(data)
    n, dim = data.shape
    keep = min(R, L)
    ids = np.zeros((n, keep), np.uint32)
    ds = np.zeros((n, keep), np.float32)
    load().oracle_filtered_ordinary_search(dt, _p(d), stride, n, dim, R, L, FL, STEPS, _p(lab.offsets),
                                           _p(lab.labels), _p(lab.starts), lab.num_labels, lab.universal,
                                           lab.global_start, _p(np.ascontiguousarray(graph, np.uint32)),
                                           _p(np.ascontiguousarray(degree, np.uint32)), _p(ids), _p(ds), threads())
    return ids, ds


def filtered_prune_lists(data, lab: FilteredLabels, R, alpha, rows, lists, dists):
    """FilteredRobustPrune of explicit candidate lists (one per row in `rows`)."""
    d, stride, dt = _store(data)
    n, dim = data.shape
    rows = np.ascontiguousarray(rows, np.uint32)
    off = np.zeros(len(rows) + 1, np.uint64)
    np.cumsum([len(x) for x in lists], out=off[1:])
    ids = np.ascontiguousarray(np.concatenate(lists) if len(lists) else np.zeros(0), np.uint32)
    ds = np.ascontiguousarray(np.concatenate(dists) if len(dists) else np.zeros(0), np.float32)
    g = np.zeros((len(rows), R), np.uint32)
    deg = np.zeros(len(rows), np.uint32)
    load().oracle_filtered_prune_lists(dt, _p(d), stride, n, dim, R, alpha, _p(lab.offsets), _p(lab.labels),
                                       lab.num_labels, _p(rows), len(rows), _p(off), _p(ids), _p(ds), _p(g),
                                       _p(deg))
    return g, deg


# ---------------------------------------------------------------- k-means partition
def kmeanspp_seed(train, k, seed=42):
    """k-means++ pivots of float32 rows as partition.cu defines them.
    Returns (centers k x dim, picked rows)."""
    t = np.ascontiguousarray(train, np.float32)
    n, dim = t.shape
    c = np.zeros((k, dim), np.float32)
    picked = np.zeros(k, np.uint64)
    load().oracle_kmeanspp_seed(_p(t), dim * 4, n, dim, k, seed, _p(c), _p(picked))
    return c, picked


def kmeans_lloyd(train, centers, iters):
    """Lloyd iterations from `centers`; returns (centers, assignment, residual)."""
    t = np.ascontiguousarray(train, np.float32)
    n, dim = t.shape
    c = np.array(centers, np.float32, copy=True, order="C")
    asg = np.zeros(n, np.uint32)
    res = ctypes.c_double(0.0)
    load().oracle_kmeans_lloyd(_p(t), dim * 4, n, dim, c.shape[0], iters, _p(c), _p(asg), ctypes.byref(res))
    return c, asg, float(res.value)


def partition_assign(data, centers, k_base):
    """Each row's k_base nearest centers (ids, squared distances)."""
    d = np.ascontiguousarray(data)
    dt = {np.dtype(np.uint8): 0, np.dtype(np.float16): 1, np.dtype(np.float32): 2}[d.dtype]
    n, dim = d.shape
    c = np.ascontiguousarray(centers, np.float32)
    ids = np.zeros((n, k_base), np.uint32)
    dists = np.zeros((n, k_base), np.float32)
    load().oracle_partition_assign(dt, _p(d), dim * d.itemsize, n, dim, _p(c), c.shape[0], k_base, _p(ids),
                                   _p(dists))
    return ids, dists


def partition_buckets(assign, num_shards):
    """Shard id lists (offsets num_shards + 1, ids) of an n x k_base assignment."""
    a = np.ascontiguousarray(assign, np.uint32)
    n, kb = a.shape
    off = np.zeros(num_shards + 1, np.uint32)
    ids = np.zeros(max(n * kb, 1), np.uint32)
    load().oracle_partition_buckets(_p(a), n, kb, num_shards, _p(off), _p(ids))
    return off, ids[:int(off[-1])]
