"""Python mirror of the DANCE builder interface over libdance_b200.so.

Host-array entry points follow the reference C ABI one to one
(include/gpu_vamana_builder.h of DANCE): same names, same argument meaning,
same status codes -- a non-zero status raises ``DanceError`` here.  Device
entry points take CUDA tensors (torch is used only to own device memory and
streams) and run the same kernels on vectors already resident in HBM.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import (DANCE_F16, DANCE_F32, DANCE_U8, DanceError, GPUVamanaStats, check, default_params, load)

INVALID = 0xFFFFFFFF


def _ptr(a) -> ctypes.c_void_p:
    if a is None:
        return ctypes.c_void_p(0)
    if isinstance(a, np.ndarray):
        return ctypes.c_void_p(a.ctypes.data)
    return ctypes.c_void_p(a.data_ptr())  # torch tensor


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        return ctypes.c_void_p(0)
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


# ----------------------------------------------------------------- reference ABI
def _host_build(fn_name: str, data: np.ndarray, R: int, L: int, C: int, STEPS: int):
    lib = load()
    if data.ndim != 2:
        raise ValueError("data must be a 2-D array (num_points x dim)")
    data = np.ascontiguousarray(data)
    n, dim = data.shape
    graph = np.empty((n, R), dtype=np.uint32)
    degree = np.empty((n,), dtype=np.uint32)
    rc = getattr(lib, fn_name)(_ptr(data), n, dim, R, L, C, STEPS, _ptr(graph), _ptr(degree))
    if rc != 0:
        raise DanceError(f"{fn_name} returned {rc}: {lib.dance_last_error().decode()}")
    return graph, degree


def gpu_vamana_vnew2_build(data: np.ndarray, R: int, L: int, C: int, STEPS: int):
    """uint8 build (reference gpu_vamana_vnew2_build); returns (graph NxR, degree N)."""
    if data.dtype != np.uint8:
        raise TypeError("gpu_vamana_vnew2_build takes uint8 data")
    return _host_build("gpu_vamana_vnew2_build", data, R, L, C, STEPS)


def gpu_vamana_vnew2_build_float(data: np.ndarray, R: int, L: int, C: int, STEPS: int):
    """float32 build (reference gpu_vamana_vnew2_build_float)."""
    if data.dtype != np.float32:
        raise TypeError("gpu_vamana_vnew2_build_float takes float32 data")
    return _host_build("gpu_vamana_vnew2_build_float", data, R, L, C, STEPS)


def gpu_vamana_build(data: np.ndarray, R: int, L: int, C: int, STEPS: int):
    """Legacy v8 entry point (reference gpu_vamana_build)."""
    return _host_build("gpu_vamana_build", np.asarray(data, dtype=np.uint8), R, L, C, STEPS)


def gpu_vamana_build_float(data: np.ndarray, R: int, L: int, C: int, STEPS: int):
    return _host_build("gpu_vamana_build_float", np.asarray(data, dtype=np.float32), R, L, C, STEPS)


def gpu_vamana_vnew2_get_last_medoid() -> int:
    return int(load().gpu_vamana_vnew2_get_last_medoid())


def gpu_vamana_vnew2_get_last_stats() -> dict:
    st = GPUVamanaStats()
    load().gpu_vamana_vnew2_get_last_stats(ctypes.byref(st))
    return {name: getattr(st, name) for name, _ in st._fields_}


# ----------------------------------------------------------------- device API
def dtype_code(t) -> int:
    import torch
    m = {torch.uint8: DANCE_U8, torch.float16: DANCE_F16, torch.float32: DANCE_F32}
    if t.dtype not in m:
        raise TypeError(f"unsupported element type {t.dtype}")
    return m[t.dtype]


def padded_store(x):
    """Return (store, stride_bytes): x with rows padded to 16 bytes (zeros)."""
    import torch
    n, dim = x.shape
    es = x.element_size()
    row = dim * es
    stride = (row + 15) // 16 * 16
    if stride == row and x.is_contiguous():
        return x, stride
    out = torch.zeros((n, stride // es), dtype=x.dtype, device=x.device)
    out[:, :dim] = x
    return out, stride


@dataclass
class Workspace:
    """Device scratch reused across builds (DanceWorkspace)."""
    handle: ctypes.c_void_p
    N: int
    R: int
    L: int
    C: int
    STEPS: int

    @classmethod
    def create(cls, N: int, R: int, L: int, C: int, STEPS: int) -> "Workspace":
        h = ctypes.c_void_p()
        check(load().dance_workspace_create(N, R, L, C, STEPS, ctypes.byref(h)), "dance_workspace_create")
        return cls(h, N, R, L, C, STEPS)

    def close(self) -> None:
        if self.handle:
            load().dance_workspace_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def build_resident(store, dim: int, stride: int, R: int, L: int, C: int, STEPS: int, params=None,
                   workspace: Workspace | None = None, graph=None, degree=None, dists=None, stream=None):
    """Whole build on a CUDA tensor already padded to ``stride`` bytes per row.

    Returns (graph, degree, dists, medoid); graph/degree/dists are CUDA tensors.
    """
    import torch
    n = store.shape[0]
    dev = store.device
    if graph is None:
        graph = torch.empty((n, R), dtype=torch.int32, device=dev)
    if degree is None:
        degree = torch.empty((n,), dtype=torch.int32, device=dev)
    if dists is None:
        dists = torch.empty((n, R), dtype=torch.float32, device=dev)
    prm = params or default_params()
    med = ctypes.c_uint32(0)
    rc = load().dance_vamana_build_resident(
        dtype_code(store), _ptr(store), stride, n, dim, R, L, C, STEPS, ctypes.byref(prm),
        workspace.handle if workspace else None, _ptr(graph), _ptr(degree), _ptr(dists),
        ctypes.byref(med), _stream(stream))
    check(rc, "dance_vamana_build_resident")
    return graph, degree, dists, int(med.value)


def search_queries(store, dim: int, stride: int, graph, R: int, start: int, queries, L_search: int, K: int,
                   visited_log2: int = 12, stream=None):
    """Best-first query search over a built graph; returns (ids, dists) CUDA tensors (nq x K)."""
    import torch
    if queries.dtype != store.dtype:
        raise ValueError(f"queries are {queries.dtype} but the store is {store.dtype}")
    q, qstride = padded_store(queries)
    nq = q.shape[0]
    ids = torch.empty((nq, K), dtype=torch.int32, device=store.device)
    dd = torch.empty((nq, K), dtype=torch.float32, device=store.device)
    rc = load().dance_search_queries(dtype_code(store), _ptr(store), stride, store.shape[0], dim, _ptr(graph), R,
                                     start, _ptr(q), qstride, nq, L_search, K, visited_log2, _ptr(ids), _ptr(dd),
                                     _stream(stream))
    check(rc, "dance_search_queries")
    return ids, dd


def search_queries_filtered(store, dim: int, stride: int, graph, R: int, label_offsets, labels, query_labels,
                            query_starts, queries, L_search: int, K: int, visited_log2: int = 12, stream=None):
    """Label-filtered query search: query i visits only points carrying
    query_labels[i], from query_starts[i].  Label arrays are CUDA tensors."""
    import torch
    if queries.dtype != store.dtype:
        raise ValueError(f"queries are {queries.dtype} but the store is {store.dtype}")
    q, qstride = padded_store(queries)
    nq = q.shape[0]
    ids = torch.empty((nq, K), dtype=torch.int32, device=store.device)
    dd = torch.empty((nq, K), dtype=torch.float32, device=store.device)
    rc = load().dance_search_queries_filtered(dtype_code(store), _ptr(store), stride, store.shape[0], dim,
                                              _ptr(graph), R, _ptr(label_offsets), _ptr(labels), _ptr(query_labels),
                                              _ptr(query_starts), _ptr(q), qstride, nq, L_search, K, visited_log2,
                                              _ptr(ids), _ptr(dd), _stream(stream))
    check(rc, "dance_search_queries_filtered")
    return ids, dd


def recall_at_k(found: np.ndarray, truth: np.ndarray, k: int = 10) -> float:
    """Mean |found[:k] & truth[:k]| / k over queries."""
    found = np.asarray(found)[:, :k].astype(np.int64)
    truth = np.asarray(truth)[:, :k].astype(np.int64)
    hits = 0
    for f, t in zip(found, truth):
        hits += len(set(f.tolist()) & set(t.tolist()))
    return hits / (k * len(truth))


# ----------------------------------------------------------------- sharded build
def shard_range(N: int, world: int, rank: int):
    """(v0, v1, chunk) of `rank`: vertices [v0, v1), chunk = ceil(N / world)."""
    a, b, c = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
    load().dance_shard_range(N, world, rank, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
    return a.value, b.value, c.value


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    check(load().dance_nccl_unique_id(buf, 128), "dance_nccl_unique_id")
    return bytes(buf)


class Comm:
    """NCCL communicator of libdance_b200 (non-blocking, bounded waits)."""

    def __init__(self, rank: int, world: int, unique_id: bytes, timeout_s: float = 120.0):
        buf = (ctypes.c_uint8 * len(unique_id)).from_buffer_copy(unique_id)
        self.handle = ctypes.c_void_p()
        check(load().dance_comm_create(rank, world, buf, len(unique_id), ctypes.c_double(timeout_s),
                                       ctypes.byref(self.handle)), "dance_comm_create")
        self.rank, self.world = rank, world

    def close(self):
        if self.handle:
            load().dance_comm_destroy(self.handle)
            self.handle = ctypes.c_void_p()


def sharded_workspace(N: int, world: int, R: int, L: int, C: int, STEPS: int) -> Workspace:
    h = ctypes.c_void_p()
    check(load().dance_workspace_create_sharded(N, world, R, L, C, STEPS, ctypes.byref(h)),
          "dance_workspace_create_sharded")
    return Workspace(h, N, R, L, C, STEPS)


def build_sharded(comm: Comm, store, dim: int, stride: int, R: int, L: int, C: int, STEPS: int, params=None,
                  workspace: Workspace | None = None, graph=None, degree=None, table_degree=None, stream=None):
    """Sharded build over the communicator's GPUs; every rank returns the
    whole graph (world*chunk rows, the first N meaningful)."""
    import torch
    n = store.shape[0]
    _, _, chunk = shard_range(n, comm.world, comm.rank)
    rows = chunk * comm.world
    dev = store.device
    if graph is None:
        graph = torch.empty((rows, R), dtype=torch.int32, device=dev)
    if degree is None:
        degree = torch.empty((rows,), dtype=torch.int32, device=dev)
    if table_degree is None:
        table_degree = torch.empty((rows,), dtype=torch.int32, device=dev)
    prm = params or default_params()
    med = ctypes.c_uint32(0)
    rc = load().dance_vamana_build_sharded(comm.handle, dtype_code(store), _ptr(store), stride, n, dim, R, L, C,
                                           STEPS, ctypes.byref(prm), workspace.handle if workspace else None,
                                           _ptr(graph), _ptr(degree), _ptr(table_degree), ctypes.byref(med),
                                           _stream(stream))
    check(rc, "dance_vamana_build_sharded")
    return graph, degree, int(med.value)
