"""Python mirror of the GPU-FilteredVamana interface over libdance_b200.so.

gpu_vamana_filtered_build_uint8 / _float follow the reference C ABI
(DANCE include/gpu_vamana_filtered.h:79-123) one to one -- host arrays in,
host graph out, the same status codes (a non-zero status raises
``DanceError``; status 1 means the work width min(C, 128) is below 2R).
build_resident runs the same build on a padded store already on the GPU.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import DANCE_F16, DANCE_U8, DanceError, GPUFilteredVamanaStats, check, load

INVALID = 0xFFFFFFFF


def _h(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _d(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def labels_csr(label_sets):
    """Per-point label lists -> (offsets u32[N+1], labels u32), each row sorted and unique."""
    rows = [sorted(set(int(v) for v in r)) for r in label_sets]
    offs = np.zeros(len(rows) + 1, np.uint32)
    np.cumsum([len(r) for r in rows], out=offs[1:])
    labs = np.array([v for r in rows for v in r], np.uint32)
    return offs, labs


def gpu_vamana_filtered_build(data: np.ndarray, R: int, L: int, filtered_L: int, C: int, STEPS: int, alpha: float,
                              point_label_offsets, point_labels, label_to_start_id, num_labels: int,
                              universal_label_id: int = INVALID, global_start_id: int = 0):
    """Reference C ABI build; uint8 or float32 data.  Returns (graph N x R, degree N)."""
    lib = load()
    data = np.ascontiguousarray(data)
    if data.dtype == np.uint8:
        fn = lib.gpu_vamana_filtered_build_uint8
    elif data.dtype == np.float32:
        fn = lib.gpu_vamana_filtered_build_float
    else:
        raise ValueError("GPU-FilteredVamana takes uint8 or float32 vectors")
    n, dim = data.shape
    offs = np.ascontiguousarray(point_label_offsets, np.uint32)
    labs = np.ascontiguousarray(point_labels, np.uint32)
    starts = np.ascontiguousarray(label_to_start_id, np.uint32)
    graph = np.empty((n, R), np.uint32)
    degree = np.empty(n, np.uint32)
    rc = fn(_h(data), n, dim, R, L, filtered_L, C, STEPS, alpha, _h(offs), _h(labs), len(labs), _h(starts),
            num_labels, universal_label_id, global_start_id, None, None, 0, _h(graph), _h(degree))
    if rc != 0:
        raise DanceError(f"gpu_vamana_filtered_build returned {rc}: {lib.dance_last_error().decode()}")
    return graph, degree


def last_stats() -> dict:
    st = GPUFilteredVamanaStats()
    load().gpu_vamana_filtered_get_last_stats(ctypes.byref(st))
    return st.as_dict()


def build_resident(store, dim: int, stride: int, R: int, L: int, filtered_L: int, work_C: int, STEPS: int,
                   alpha: float, point_label_offsets, point_labels, label_to_start_id, num_labels: int,
                   universal_label_id: int = INVALID, global_start_id: int = 0, graph=None, degree=None,
                   init_graph=None, init_degree=None, rounds: int = 3, stream=None):
    """Canonical filtered build on a padded uint8/fp16 CUDA store.  Returns
    (graph, degree, stats dict); work_C is the work width itself."""
    import torch
    lib = load()
    dt = {torch.uint8: DANCE_U8, torch.float16: DANCE_F16}[store.dtype]
    n = store.shape[0]
    if graph is None:
        graph = torch.empty((n, R), dtype=torch.int32, device=store.device)
    if degree is None:
        degree = torch.empty(n, dtype=torch.int32, device=store.device)
    offs = np.ascontiguousarray(point_label_offsets, np.uint32)
    labs = np.ascontiguousarray(point_labels, np.uint32)
    starts = np.ascontiguousarray(label_to_start_id, np.uint32)
    st = GPUFilteredVamanaStats()
    s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
    rc = lib.dance_filtered_build_resident(dt, _d(store), stride, n, dim, R, L, filtered_L, work_C, STEPS, alpha,
                                           _h(offs), _h(labs), _h(starts), num_labels, universal_label_id,
                                           global_start_id, _d(init_graph), _d(init_degree), rounds, _d(graph),
                                           _d(degree), ctypes.byref(st), s)
    check(rc, "dance_filtered_build_resident")
    return graph, degree, st.as_dict()


def label_points_csr(point_label_offsets, point_labels, num_labels: int, universal_label_id: int = INVALID):
    """Per-label point lists (offsets u32[num_labels+1], points ascending) from
    the per-point label CSR; a point carrying the universal label is listed
    under every label, as DiskANN's label_to_points is built."""
    offs = np.asarray(point_label_offsets, np.int64)
    labs = np.asarray(point_labels, np.int64)
    n = len(offs) - 1
    pnt = np.repeat(np.arange(n, dtype=np.int64), np.diff(offs))
    keep = (labs != universal_label_id) & (labs < num_labels)
    pairs = [labs[keep] * (n + 1) + pnt[keep]]
    keep = labs != universal_label_id
    if universal_label_id != INVALID:
        upts = np.unique(pnt[~keep])
        if len(upts):
            pairs.append((np.arange(num_labels, dtype=np.int64)[:, None] * (n + 1) + upts[None, :]).ravel())
    key = np.unique(np.concatenate(pairs)) if pairs else np.zeros(0, np.int64)
    lab_of, pt_of = key // (n + 1), key % (n + 1)
    loff = np.zeros(num_labels + 1, np.uint32)
    loff[1:] = np.cumsum(np.bincount(lab_of, minlength=num_labels)[:num_labels])
    return loff, pt_of.astype(np.uint32)


def calculate_entry_point(store, dim: int, stride: int) -> int:
    """DiskANN's calculate_entry_point on a padded CUDA store
    (``dance_calculate_entry_point``)."""
    import torch
    from .vamana import dtype_code
    out = ctypes.c_uint32(0)
    rc = load().dance_calculate_entry_point(dtype_code(store), _d(store), stride, store.shape[0], dim,
                                            ctypes.byref(out), None)
    check(rc, "dance_calculate_entry_point")
    return int(out.value)


def select_label_starts(label_offsets, label_points, num_points: int, num_candidates: int = 25,
                        seed: int = 42) -> np.ndarray:
    """One start point per label (``dance_select_label_starts``; DiskANN's
    least-chosen-of-25 rule with hashed draws).  Inputs from label_points_csr."""
    import torch
    loff = torch.from_numpy(np.ascontiguousarray(label_offsets, np.uint32).view(np.int32)).cuda()
    pts = np.ascontiguousarray(label_points, np.uint32)
    dpts = torch.from_numpy((pts if len(pts) else np.zeros(1, np.uint32)).view(np.int32)).cuda()
    nl = len(label_offsets) - 1
    starts = torch.empty(max(nl, 1), dtype=torch.int32, device="cuda")
    rc = load().dance_select_label_starts(_d(loff), _d(dpts), nl, num_points, num_candidates, seed, _d(starts), None)
    check(rc, "dance_select_label_starts")
    return starts[:nl].cpu().numpy().view(np.uint32).copy()
