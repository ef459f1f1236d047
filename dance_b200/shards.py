"""Sharded disk-index build on B200s: k-means partition, per-shard GPU builds
over the GPUs of one box, and the GPU shard merge.

This mirrors DiskANN's ``build_merged_vamana_index`` as the DANCE patch runs
it with ``DISKANN_USE_GPU_SHARD_BUILD=1`` and ``DISKANN_USE_GPU_MERGE=1``
(reference ``integrations/dance-diskann-78256bba.patch``):

* partition (patch lines 20629-20688, DiskANN ``partition_with_ram_budget``
  and ``shard_data_into_clusters_only_ids``): k-means on a sample, starting at
  3 parts and adding 2 while the largest shard's estimated build memory
  exceeds the budget; every point goes to its ``k_base`` nearest centers.
  Here the k-means++ seeding, the Lloyd iterations, the assignment of every
  point and the per-shard id lists run on the GPU (``dance_kmeanspp_seed``,
  ``dance_kmeans_lloyd``, ``dance_partition_assign``,
  ``dance_partition_buckets``); the files are DiskANN's:
  ``<prefix>_centroids.bin`` and ``<prefix>_subshard-<i>_ids_uint32.bin``.
* shard loop (patch lines 3270-3600, ``build_gpu_shard_index_from_data``
  lines 2811-2990): each shard's vectors are gathered from the base file and
  built on a GPU with R_shard = 2R/3 (``DISKANN_GPU_SHARD_R``), C =
  max(2 R_shard, R_shard + 32) (``DISKANN_GPU_C``) and STEPS = min(L, 20)
  (``DISKANN_GPU_STEPS``); the graph is saved in DiskANN's format with the
  shard medoid as its start (``save_gpu_vamana_graph_for_merge``, lines
  2748-2806).  ``DISKANN_SHARD_BUILD_PARALLELISM`` shards are built at once,
  one per GPU, each GPU taking the next unbuilt shard when it finishes (the
  patch's dynamic schedule).
* merge (patch lines 3015-3035 -> ``diskann::merge_shards_gpu``): the
  library's ``dance_merge_shards_gpu`` writes the merged graph and the
  medoids file.

DiskANN's PQ pivot reuse (patch lines 20689-20871) and the disk layout are
CPU code of DiskANN itself and are not part of this module; the reference's
GPU shard path also refuses ``build_PQ_bytes > 0``.

Differences from DiskANN, on purpose: DiskANN samples and seeds k-means with
``std::random_device``; here both are seeded hashes, so a partition is
reproducible.  DiskANN's CPU merge shuffles each merged row with an unseeded
generator; the GPU merge ranks edges by a seeded hash (as the reference's
own GPU merge does).
"""
from __future__ import annotations

import ctypes
import os
import queue
import threading
import time
from pathlib import Path

import numpy as np

from . import check, load
from .formats import write_graph

DANCE_U8, DANCE_F16, DANCE_F32 = 0, 1, 2
_DTYPES = {"uint8": (np.uint8, DANCE_U8), "float": (np.float32, DANCE_F32)}

# DiskANN's build-memory estimate (utils.h estimate_ram_usage): data rows
# rounded up to 8 elements, the graph with its slack factor, one lock and
# one vector header per point, times an overhead factor.
_GRAPH_SLACK_FACTOR = 1.3
_OVERHEAD_FACTOR = 1.1
_LOCK_BYTES = 40
_PTR_BYTES = 8


def _ptr(t) -> ctypes.c_void_p:
    if hasattr(t, "data_ptr"):
        return ctypes.c_void_p(t.data_ptr())
    return ctypes.c_void_p(t.ctypes.data)


def _env_u32(name: str, default: int) -> int:
    v = os.environ.get(name, "")
    try:
        return int(v) if v != "" else default
    except ValueError:
        return default


def estimate_ram_usage(size: int, dim: int, datasize: int, degree: int) -> float:
    """Bytes DiskANN reserves to build an in-memory index of `size` points."""
    data = float(size) * ((dim + 7) // 8 * 8) * datasize
    graph = float(size) * degree * 4 * _GRAPH_SLACK_FACTOR
    return _OVERHEAD_FACTOR * (data + graph + size * _LOCK_BYTES + size * _PTR_BYTES)


def splitmix64(x: np.ndarray) -> np.ndarray:
    """The splitmix64 finaliser on uint64 arrays (wrapping arithmetic)."""
    x = np.asarray(x, np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def gen_random_slice_ids(n: int, sampling_rate: float, seed: int) -> np.ndarray:
    """Ids kept by DiskANN's gen_random_slice (each point with probability
    `sampling_rate`), drawn from a seeded hash of (seed, id) so the sample is
    reproducible; at least one point is kept."""
    if not 0.0 < sampling_rate <= 1.0:
        raise ValueError(f"sampling_rate must be in (0, 1], got {sampling_rate}")
    thr = np.uint64(min(int(sampling_rate * 2.0 ** 64), 2 ** 64 - 1))
    out = []
    block = 1 << 24
    s = splitmix64(np.uint64(seed))
    for b in range(0, n, block):
        ids = np.arange(b, min(n, b + block), dtype=np.uint64)
        keep = splitmix64(ids ^ s) <= thr
        out.append(ids[keep].astype(np.int64))
    ids = np.concatenate(out) if out else np.zeros(0, np.int64)
    return ids if len(ids) else np.zeros(1, np.int64)


def read_bin_header(path) -> tuple[int, int]:
    hdr = np.fromfile(path, dtype=np.uint32, count=2)
    if len(hdr) != 2:
        raise ValueError(f"{path}: not a DiskANN .bin file")
    return int(hdr[0]), int(hdr[1])


def open_base(path, data_type: str) -> np.ndarray:
    """Memory-map a DiskANN .bin vector file (u32 n, u32 dim, rows)."""
    n, dim = read_bin_header(path)
    dt = _DTYPES[data_type][0]
    return np.memmap(path, dtype=dt, mode="r", offset=8, shape=(n, dim))


def write_idmap(path, ids: np.ndarray) -> None:
    """DiskANN idmap file: u32 count, u32 1, ids."""
    ids = np.ascontiguousarray(ids, np.uint32)
    with open(path, "wb") as f:
        np.array([len(ids), 1], np.uint32).tofile(f)
        ids.tofile(f)


def read_idmap(path) -> np.ndarray:
    hdr = np.fromfile(path, dtype=np.uint32, count=2)
    return np.fromfile(path, dtype=np.uint32, offset=8, count=int(hdr[0]))


def write_centroids(path, centers: np.ndarray) -> None:
    """DiskANN save_bin<float>: u32 rows, u32 cols, float rows."""
    c = np.ascontiguousarray(centers, np.float32)
    with open(path, "wb") as f:
        np.array(c.shape, np.uint32).tofile(f)
        c.tofile(f)


# ---------------------------------------------------------------- GPU k-means
def kmeans_centers(train, num_parts: int, max_reps: int = 10, seed: int = 42):
    """k-means++ seeding and `max_reps` Lloyd iterations of a float32 CUDA
    tensor (n x dim) on its device; returns (centers tensor, residual)."""
    import torch
    t = train.contiguous()
    n, dim = t.shape
    centers = torch.empty((num_parts, dim), dtype=torch.float32, device=t.device)
    picked = torch.empty((num_parts,), dtype=torch.int64, device=t.device)
    lib = load()
    check(lib.dance_kmeanspp_seed(_ptr(t), dim * 4, n, dim, num_parts, seed, _ptr(centers), _ptr(picked), None),
          "dance_kmeanspp_seed")
    res = ctypes.c_double(0.0)
    if max_reps:
        check(lib.dance_kmeans_lloyd(_ptr(t), dim * 4, n, dim, num_parts, max_reps, _ptr(centers), None,
                                     ctypes.byref(res), None), "dance_kmeans_lloyd")
    return centers, float(res.value)


def assign_points(x, centers, k_base: int):
    """Each row of the CUDA tensor `x` (uint8/float16/float32) to its k_base
    nearest centers; returns (ids int32 n x k_base, squared distances)."""
    import torch
    codes = {torch.uint8: DANCE_U8, torch.float16: DANCE_F16, torch.float32: DANCE_F32}
    x = x.contiguous()
    n, dim = x.shape
    ids = torch.empty((n, k_base), dtype=torch.int32, device=x.device)
    d = torch.empty((n, k_base), dtype=torch.float32, device=x.device)
    check(load().dance_partition_assign(codes[x.dtype], _ptr(x), dim * x.element_size(), n, dim,
                                        _ptr(centers), centers.shape[0], k_base, _ptr(ids), _ptr(d), None),
          "dance_partition_assign")
    return ids, d


def shard_lists(assign, num_shards: int):
    """Per-shard ascending point ids of an (n x k_base) CUDA assignment;
    returns (offsets int64 numpy, ids CUDA int32 tensor)."""
    import torch
    a = assign.contiguous()
    n, kb = a.shape
    off = torch.empty((num_shards + 1,), dtype=torch.int32, device=a.device)
    ids = torch.empty((max(n * kb, 1),), dtype=torch.int32, device=a.device)
    check(load().dance_partition_buckets(_ptr(a), n, kb, num_shards, _ptr(off), _ptr(ids), None),
          "dance_partition_buckets")
    off_h = off.cpu().numpy().view(np.uint32).astype(np.int64)
    return off_h, ids[:int(off_h[-1])]


def _rows_to_device(base: np.ndarray, ids: np.ndarray | None, device, b0: int = 0, b1: int | None = None):
    """Rows b0:b1 (or the rows `ids`) of a memory-mapped base, on `device`."""
    import torch
    block = np.array(base[b0:b1]) if ids is None else np.ascontiguousarray(base[ids])
    return torch.from_numpy(block).to(device)


def partition_with_ram_budget(data_file, data_type: str, sampling_rate: float, ram_budget_gb: float,
                              graph_degree: int, prefix_path, k_base: int = 2, seed: int = 42,
                              max_k_means_reps: int = 10, num_parts: int | None = None, device: int = 0,
                              block_points: int = 1 << 22) -> dict:
    """DiskANN partition_with_ram_budget + shard_data_into_clusters_only_ids
    on one GPU.  Writes ``<prefix>_centroids.bin`` and the shard idmaps;
    returns {"num_parts", "shard_sizes", "residual", "seconds"}.  With
    `num_parts` given, the budget loop is skipped."""
    import torch
    t0 = time.perf_counter()
    dev = torch.device("cuda", device)
    base = open_base(data_file, data_type)
    n, dim = base.shape
    es = base.dtype.itemsize
    train_ids = gen_random_slice_ids(n, sampling_rate, seed)
    test_ids = gen_random_slice_ids(n, sampling_rate, seed + 1)
    train = _rows_to_device(base, train_ids, dev).float()
    test = _rows_to_device(base, test_ids, dev)
    parts = num_parts or 3
    while True:
        centers, resid = kmeans_centers(train, parts, max_k_means_reps, seed)
        if num_parts:
            break
        a, _ = assign_points(test, centers, min(k_base, parts))
        counts = torch.bincount(a.reshape(-1).long(), minlength=parts).cpu().numpy()
        est = max(estimate_ram_usage(int(c / sampling_rate), dim, es, graph_degree) for c in counts)
        if est <= ram_budget_gb * 1024.0 ** 3:
            break
        parts += 2
        if parts > min(len(train_ids), 8192):
            raise ValueError(f"no partition of at most {parts - 2} parts fits a {ram_budget_gb} GB build budget; "
                             "raise the budget or the sampling rate")
    kb = min(k_base, parts)
    prefix = str(prefix_path)
    write_centroids(prefix + "_centroids.bin", centers.cpu().numpy())
    assign = torch.empty((n, kb), dtype=torch.int32, device=dev)
    for b in range(0, n, block_points):
        e = min(n, b + block_points)
        x = _rows_to_device(base, None, dev, b, e)
        ids, _ = assign_points(x, centers, kb)
        assign[b:e] = ids
    off, ids = shard_lists(assign, parts)
    ids_h = ids.cpu().numpy().view(np.uint32)
    sizes = []
    for s in range(parts):
        shard = ids_h[off[s]:off[s + 1]]
        write_idmap(f"{prefix}_subshard-{s}_ids_uint32.bin", shard)
        sizes.append(int(len(shard)))
    return {"num_parts": parts, "shard_sizes": sizes, "residual": resid, "seconds": time.perf_counter() - t0}


# ---------------------------------------------------------------- shard builds
def shard_build_params(R: int, L: int) -> tuple[int, int, int]:
    """(R_shard, C, STEPS) of the GPU shard build (patch lines 3270-3320)."""
    shard_r = 2 * R // 3
    req = _env_u32("DISKANN_GPU_SHARD_R", 0)
    if req > 0:
        shard_r = min(req, R)
    C = _env_u32("DISKANN_GPU_C", 0) or max(2 * shard_r, shard_r + 32)
    steps = _env_u32("DISKANN_GPU_STEPS", 0) or min(L, 20)
    C = max(C, shard_r)
    steps = min(steps, L)
    return shard_r, C, steps


def build_shard(base: np.ndarray, ids: np.ndarray, out_file, R: int, L: int, C: int, STEPS: int, device: int,
                store_fp16: bool = False, workspace=None, stream=None) -> dict:
    """One shard: gather its rows, build on `device` (on `stream`, in
    `workspace` when given), save the graph in DiskANN's format with the
    shard medoid as start."""
    import torch
    from . import vamana
    t0 = time.perf_counter()
    torch.cuda.set_device(device)
    stream = stream or torch.cuda.current_stream(device)
    with torch.cuda.stream(stream):
        x = _rows_to_device(base, ids, torch.device("cuda", device))
        if store_fp16 and x.dtype == torch.float32:
            x = x.half()
        store, stride = vamana.padded_store(x)
        stream.synchronize()
        t1 = time.perf_counter()
        graph, degree, _, medoid = vamana.build_resident(store, x.shape[1], stride, R, L, C, STEPS,
                                                         workspace=workspace, stream=stream.cuda_stream)
        stream.synchronize()
        t2 = time.perf_counter()
        g = graph.cpu().numpy().view(np.uint32)
        deg = degree.cpu().numpy().view(np.uint32)
    write_graph(out_file, g, deg, medoid)
    t3 = time.perf_counter()
    return {"points": int(len(ids)), "medoid": int(medoid), "seconds": t3 - t0, "gather_seconds": t1 - t0,
            "build_seconds": t2 - t1, "write_seconds": t3 - t2, "device": device}


def build_shards(data_file, data_type: str, prefix_path, num_parts: int, R: int, L: int,
                 devices: list[int] | None = None, store_fp16: bool = False,
                 workers_per_device: int = 2) -> list[dict]:
    """Builds every shard listed by the partition's idmaps.  Each GPU runs
    `workers_per_device` workers (own stream and build workspace, so one
    shard's file reads and writes overlap another's build), each taking the
    next unbuilt shard, largest first."""
    import torch
    from . import vamana
    if devices is None:
        par = max(1, min(_env_u32("DISKANN_SHARD_BUILD_PARALLELISM", torch.cuda.device_count()), num_parts))
        devices = list(range(min(par, torch.cuda.device_count())))
    shard_r, C, steps = shard_build_params(R, L)
    base = open_base(data_file, data_type)
    prefix = str(prefix_path)
    sizes = [int(np.fromfile(f"{prefix}_subshard-{p}_ids_uint32.bin", dtype=np.uint32, count=1)[0])
             for p in range(num_parts)]
    todo: queue.Queue[int] = queue.Queue()
    for p in sorted(range(num_parts), key=lambda q: -sizes[q]):
        todo.put(p)
    results: dict[int, dict] = {}
    errors: list[BaseException] = []

    def worker(dev: int) -> None:
        ws = None
        try:
            torch.cuda.set_device(dev)
            stream = torch.cuda.Stream(dev)
            while not errors:
                try:
                    p = todo.get_nowait()
                except queue.Empty:
                    return
                ids = read_idmap(f"{prefix}_subshard-{p}_ids_uint32.bin").astype(np.int64)
                if len(ids) == 0:
                    raise ValueError(f"shard {p} is empty")
                if ws is None:
                    ws = vamana.Workspace.create(max(sizes), shard_r, L, C, steps)
                results[p] = build_shard(base, ids, f"{prefix}_subshard-{p}_mem.index", shard_r, L, C, steps,
                                         dev, store_fp16, workspace=ws, stream=stream)
        except BaseException as e:  # reported after every worker stops
            errors.append(e)
        finally:
            if ws is not None:
                ws.close()

    threads = [threading.Thread(target=worker, args=(d,)) for d in devices for _ in range(max(1, workers_per_device))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    return [dict(results[p], shard=p, R=shard_r, C=C, STEPS=steps) for p in range(num_parts)]


def merge_shards(prefix_path, num_parts: int, R: int, mem_index_path, medoids_file) -> None:
    """The GPU shard merge over the shard graphs and idmaps of `prefix_path`."""
    prefix = str(prefix_path) + "_subshard-"
    rc = load().dance_merge_shards_gpu(prefix.encode(), b"_mem.index", prefix.encode(), b"_ids_uint32.bin",
                                       num_parts, R, str(mem_index_path).encode(), str(medoids_file).encode())
    check(rc, "dance_merge_shards_gpu")


def build_merged_vamana_index(data_file, data_type: str, R: int, L: int, ram_budget_gb: float, mem_index_path,
                              medoids_file, centroids_file=None, sampling_rate: float = 0.01, k_base: int = 2,
                              num_parts: int | None = None, devices: list[int] | None = None, seed: int = 42,
                              store_fp16: bool = False, keep_tempfiles: bool | None = None) -> dict:
    """Partition -> shard builds -> merge (DiskANN build_merged_vamana_index
    with the DANCE GPU shard build and GPU merge).  Temporary files go next to
    `mem_index_path` as ``<mem_index_path>_tempFiles_*`` and are removed
    unless `keep_tempfiles` (or DISKANN_KEEP_TEMPFILES=1)."""
    if data_type not in _DTYPES:
        raise ValueError(f"data_type must be one of {sorted(_DTYPES)}")
    prefix = str(mem_index_path) + "_tempFiles"
    timing = {}
    t0 = time.perf_counter()
    part = partition_with_ram_budget(data_file, data_type, sampling_rate, ram_budget_gb, R, prefix, k_base, seed,
                                     num_parts=num_parts, device=(devices or [0])[0])
    timing["partition_seconds"] = time.perf_counter() - t0
    if centroids_file is not None:
        os.replace(prefix + "_centroids.bin", centroids_file)
    t1 = time.perf_counter()
    shards = build_shards(data_file, data_type, prefix, part["num_parts"], R, L, devices, store_fp16)
    timing["shard_build_seconds"] = time.perf_counter() - t1
    t2 = time.perf_counter()
    merge_shards(prefix, part["num_parts"], R, mem_index_path, medoids_file)
    timing["merge_seconds"] = time.perf_counter() - t2
    if keep_tempfiles is None:
        keep_tempfiles = os.environ.get("DISKANN_KEEP_TEMPFILES") == "1"
    if not keep_tempfiles:
        for p in range(part["num_parts"]):
            for suffix in ("_ids_uint32.bin", "_mem.index"):
                f = Path(f"{prefix}_subshard-{p}{suffix}")
                if f.exists():
                    f.unlink()
        c = Path(prefix + "_centroids.bin")
        if c.exists():
            c.unlink()
    timing["total_seconds"] = time.perf_counter() - t0
    return {"num_parts": part["num_parts"], "shard_sizes": part["shard_sizes"], "shards": shards, **timing}
