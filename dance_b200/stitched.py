"""GPU-StitchedVamana: per-label graphs stitched into one filtered index.

Python mirror of the reference app ``gpu_stitched_vamana_index``
(apps/utils/gpu_stitched_vamana_index.cpp): the same label-file rules
(:111-160), the same build and remap rules (:241-341, run on the GPU by
``dance_stitched_build``), the same graph file (:200-227) and sidecars
(:162-199), the same timing keys (:378-426) and the same command-line
flags (:43-63).  ``python -m dance_b200.stitched --help`` runs it as a CLI.

The reference finishes multi-label inputs (and Rsmall > Rstitched, which its
argument parser already rules out) with DiskANN's CPU label-aware prune
(:353-372: ``Index::prune_all_neighbors(Rstitched, 750, alpha)`` with the
DANCE patch's coverage rule and label-balanced shortlist).  Here that prune
runs on the GPU (``global_prune``, ``dance_stitched_global_prune``): the
union graph is kept as ``<prefix>_full``, as the reference keeps it, and the
pruned graph is the index.  ``allow_unpruned`` writes the union graph as the
index instead.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import shutil
import sys
import time
from pathlib import Path

import numpy as np

from . import DANCE_F32, DANCE_U8, DanceError, DanceStitchedStats, check, default_params, load
from .formats import GRAPH_HEADER, _refuse_existing, read_bin

INVALID = 0xFFFFFFFF


def _ptr(a) -> ctypes.c_void_p:
    if a is None:
        return ctypes.c_void_p(0)
    if isinstance(a, np.ndarray):
        return ctypes.c_void_p(a.ctypes.data)
    return ctypes.c_void_p(a.data_ptr())


# ----------------------------------------------------------------- labels
def parse_label_lines(lines, universal_label: str = ""):
    """Label rows -> (point_label_names, label_to_id, id_to_label, label_points).

    Rules of the reference parse_labels (:111-160): carriage returns and
    spaces are removed, tokens are comma separated, an empty row or token
    is an error, the universal label is rejected, repeated names in a row
    count once, and label ids are 1-based in first-seen order.
    """
    point_label_names = []
    label_to_id: dict[str, int] = {}
    id_to_label: list[str] = []
    label_points: list[list[int]] = []
    for raw in lines:
        line = raw.rstrip("\n").replace("\r", "").replace(" ", "")
        if not line:
            raise ValueError("empty label row is not supported")
        names: list[str] = []
        for name in line.split(","):
            if not name:
                raise ValueError("empty label token is not supported")
            if universal_label and name == universal_label:
                raise ValueError("GPU StitchedMVP does not support universal-label rows")
            if name not in names:
                names.append(name)
        point = len(point_label_names)
        for name in names:
            lid = label_to_id.get(name)
            if lid is None:
                lid = len(id_to_label) + 1
                label_to_id[name] = lid
                id_to_label.append(name)
                label_points.append([])
            label_points[lid - 1].append(point)
        point_label_names.append(names)
    return point_label_names, label_to_id, id_to_label, label_points


def parse_labels(label_file, universal_label: str = ""):
    with open(label_file, "r", newline="") as f:
        return parse_label_lines(f, universal_label)


def labels_csr(label_points):
    """list of per-label point lists -> (offsets u64[L+1], points u32[M])."""
    sizes = np.array([len(p) for p in label_points], dtype=np.uint64)
    offsets = np.zeros(len(label_points) + 1, dtype=np.uint64)
    np.cumsum(sizes, out=offsets[1:])
    points = (np.concatenate([np.asarray(p, dtype=np.uint32) for p in label_points])
              if label_points and offsets[-1] else np.zeros(0, np.uint32))
    return offsets, points


def labels_from_assignment(assign: np.ndarray, num_labels: int):
    """One label per point (label index per point) -> label_points lists, points ascending."""
    order = np.argsort(assign, kind="stable")
    counts = np.bincount(assign, minlength=num_labels)
    splits = np.split(order.astype(np.uint32), np.cumsum(counts)[:-1])
    return [s.tolist() for s in splits]


# ----------------------------------------------------------------- build
def stitched_build(data: np.ndarray, label_offsets: np.ndarray, label_points: np.ndarray, r_small: int = 32,
                   l_small: int = 100, r_stitched: int = 64, C: int = 96, steps: int = 64, params=None,
                   streams: int = 4):
    """GPU build of every label's graph and the stitched CSR graph.

    Returns (row_offsets u64[N+1], row_ids u32[E], label_medoids u32[L], stats dict).
    """
    lib = load()
    data = np.ascontiguousarray(data)
    if data.dtype == np.uint8:
        dt = DANCE_U8
    elif data.dtype == np.float32:
        dt = DANCE_F32
    else:
        raise ValueError("GPU StitchedMVP supports uint8 and float in this version")
    n, dim = data.shape
    offs = np.ascontiguousarray(label_offsets, dtype=np.uint64)
    pts = np.ascontiguousarray(label_points, dtype=np.uint32)
    nl = len(offs) - 1
    row_offsets = np.zeros(n + 1, dtype=np.uint64)
    cap = int(offs[-1]) * int(r_small)
    row_ids = np.zeros(max(cap, 1), dtype=np.uint32)
    medoids = np.zeros(max(nl, 1), dtype=np.uint32)
    st = DanceStitchedStats()
    prm = params if params is not None else default_params()
    rc = lib.dance_stitched_build(dt, _ptr(data), n, dim, nl, _ptr(offs), _ptr(pts), r_small, l_small, r_stitched,
                                  C, steps, ctypes.byref(prm), streams, _ptr(row_offsets), _ptr(row_ids), cap,
                                  _ptr(medoids), ctypes.byref(st))
    check(rc, "dance_stitched_build")
    E = int(row_offsets[-1])
    return row_offsets, row_ids[:E].copy(), medoids[:nl].copy(), st.as_dict()


def point_label_csr(label_points, n: int):
    """Per-point label CSR (offsets u32[n+1], labels u32 ascending per point)
    from per-label point lists; label l of the lists is label id l."""
    pts = [np.asarray(p, dtype=np.int64) for p in label_points]
    if not pts or sum(len(p) for p in pts) == 0:
        return np.zeros(n + 1, np.uint32), np.zeros(0, np.uint32)
    pp = np.concatenate(pts)
    ll = np.concatenate([np.full(len(p), l, np.int64) for l, p in enumerate(pts)])
    pairs = np.unique(pp * (len(pts) + 1) + ll)
    pp, ll = pairs // (len(pts) + 1), pairs % (len(pts) + 1)
    offs = np.zeros(n + 1, np.uint32)
    offs[1:] = np.cumsum(np.bincount(pp, minlength=n))
    return offs, ll.astype(np.uint32)


def global_prune(data: np.ndarray, row_offsets: np.ndarray, row_ids: np.ndarray, point_label_offsets, point_labels,
                 r_stitched: int, max_candidates: int = 750, alpha: float = 1.2):
    """Label-aware global prune of a stitched union graph on the GPU
    (``dance_stitched_global_prune``; DiskANN's patched prune_all_neighbors).
    Returns (row_offsets u64[N+1], row_ids u32[E], rows pruned)."""
    import torch
    from .vamana import dtype_code, padded_store
    lib = load()
    data = np.ascontiguousarray(data)
    n, dim = data.shape
    x = torch.from_numpy(data).cuda()
    store, stride = padded_store(x)
    ro = torch.from_numpy(np.ascontiguousarray(row_offsets, np.uint64).view(np.int64)).cuda()
    ri = torch.from_numpy(np.ascontiguousarray(row_ids, np.uint32).view(np.int32)).cuda()
    if point_label_offsets is not None:
        lo = torch.from_numpy(np.ascontiguousarray(point_label_offsets, np.uint32).view(np.int32)).cuda()
        lb = torch.from_numpy(np.ascontiguousarray(point_labels, np.uint32).view(np.int32)).cuda()
        lo_p, lb_p = ctypes.c_void_p(lo.data_ptr()), ctypes.c_void_p(lb.data_ptr() if lb.numel() else lo.data_ptr())
    else:
        lo_p = lb_p = None
    out = torch.empty((n, r_stitched), dtype=torch.int32, device="cuda")
    deg = torch.empty((n,), dtype=torch.int32, device="cuda")
    pruned = ctypes.c_uint64(0)
    rc = lib.dance_stitched_global_prune(dtype_code(x), ctypes.c_void_p(store.data_ptr()), stride, n, dim,
                                         ctypes.c_void_p(ro.data_ptr()), ctypes.c_void_p(ri.data_ptr()), lo_p, lb_p,
                                         r_stitched, max_candidates, alpha, ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(deg.data_ptr()), ctypes.byref(pruned), None)
    check(rc, "dance_stitched_global_prune")
    rows = out.cpu().numpy().view(np.uint32)
    d = deg.cpu().numpy().view(np.uint32).astype(np.int64)
    offs = np.zeros(n + 1, np.uint64)
    offs[1:] = np.cumsum(d)
    ids = rows[np.arange(r_stitched)[None, :] < d[:, None]]
    return offs, ids.astype(np.uint32), int(pruned.value)


def lpt_assignment(label_offsets: np.ndarray, world: int) -> np.ndarray:
    """Rank of each label: largest label first to the least-loaded rank (ties: lower rank)."""
    sizes = np.diff(np.asarray(label_offsets, dtype=np.int64))
    owner = np.zeros(len(sizes), dtype=np.int64)
    load_ = np.zeros(world, dtype=np.int64)
    for l in sorted(range(len(sizes)), key=lambda i: (-sizes[i], i)):
        r = int(np.argmin(load_))
        owner[l] = r
        load_[r] += sizes[l]
    return owner


def stitched_build_sharded(comm, data: np.ndarray, label_offsets: np.ndarray, label_points: np.ndarray,
                           r_small: int = 32, l_small: int = 100, r_stitched: int = 64, C: int = 96, steps: int = 64,
                           params=None, streams: int = 4):
    """Label-parallel build over the GPUs of one box (``dance_stitched_build_sharded``):
    labels largest first to the least-loaded rank, each rank builds its labels,
    the local graphs go to rank 0 over NCCL and rank 0 stitches.  ``comm`` is a
    ``vamana.Comm``.  Returns (row_offsets, row_ids, label_medoids, stats) on
    rank 0 and (None, None, None, stats) on the other ranks."""
    lib = load()
    data = np.ascontiguousarray(data)
    if data.dtype == np.uint8:
        dt = DANCE_U8
    elif data.dtype == np.float32:
        dt = DANCE_F32
    else:
        raise ValueError("GPU StitchedMVP supports uint8 and float in this version")
    n, dim = data.shape
    offs = np.ascontiguousarray(label_offsets, dtype=np.uint64)
    pts = np.ascontiguousarray(label_points, dtype=np.uint32)
    nl = len(offs) - 1
    root = comm.rank == 0
    cap = int(offs[-1]) * int(r_small)
    row_offsets = np.zeros(n + 1, dtype=np.uint64) if root else None
    row_ids = np.zeros(max(cap, 1), dtype=np.uint32) if root else None
    medoids = np.zeros(max(nl, 1), dtype=np.uint32) if root else None
    st = DanceStitchedStats()
    prm = params if params is not None else default_params()
    opt = (lambda a: _ptr(a) if a is not None else None)  # noqa: E731
    rc = lib.dance_stitched_build_sharded(comm.handle, dt, _ptr(data), n, dim, nl, _ptr(offs), _ptr(pts), r_small,
                                          l_small, r_stitched, C, steps, ctypes.byref(prm), streams,
                                          opt(row_offsets), opt(row_ids), cap if root else 0, opt(medoids),
                                          ctypes.byref(st))
    check(rc, "dance_stitched_build_sharded")
    if not root:
        return None, None, None, st.as_dict()
    E = int(row_offsets[-1])
    return row_offsets, row_ids[:E].copy(), medoids[:nl].copy(), st.as_dict()


def encode_csr_graph(row_offsets: np.ndarray, row_ids: np.ndarray, start: int = 0) -> bytes:
    """DiskANN graph bytes of a CSR graph; max_degree is the largest row (:200-227)."""
    offs = np.asarray(row_offsets, dtype=np.int64)
    n = len(offs) - 1
    deg = np.diff(offs)
    total = GRAPH_HEADER.size + 4 * n + 4 * int(offs[-1])
    max_degree = int(deg.max()) if n else 0
    out = np.empty(n + int(offs[-1]), dtype=np.uint32)
    pos = offs[:-1] + np.arange(n)  # where each row's degree word goes
    out[pos] = deg
    keep = np.ones(len(out), dtype=bool)
    keep[pos] = False
    out[keep] = np.asarray(row_ids, dtype=np.uint32)
    blob = GRAPH_HEADER.pack(total, max_degree, int(start), 0) + out.tobytes()
    assert len(blob) == total
    return blob


def _publish(path: Path, payload: bytes) -> None:
    tmp = path.with_name(path.name + ".tmp")
    _refuse_existing(path, tmp)
    try:
        with open(tmp, "wb") as f:
            f.write(payload)
        os.replace(tmp, path)
    except BaseException:
        if tmp.exists():
            tmp.unlink()
        raise


def sidecar_texts(point_label_names, label_to_id, id_to_label, label_medoids) -> dict:
    """Contents of the four label sidecars (:170-198)."""
    rows = "".join(",".join(str(label_to_id[nm]) for nm in names) + "\n" for names in point_label_names)
    return {
        "_labels.txt": rows,
        "_label_formatted.txt": rows,
        "_labels_map.txt": "".join(f"{name}\t{i + 1}\n" for i, name in enumerate(id_to_label)),
        "_labels_to_medoids.txt": "".join(f"{i + 1}, {int(m)}\n" for i, m in enumerate(label_medoids)),
    }


def write_stitched_index(prefix, data_path, row_offsets, row_ids, point_label_names, label_to_id, id_to_label,
                         label_medoids) -> dict:
    """Graph at <prefix> (start node 0), <prefix>.data and the label sidecars.

    Every file is published through a temporary name and nothing existing is
    overwritten.  Returns {"write_index_seconds", "metadata_seconds"}.
    """
    prefix = Path(prefix)
    side = sidecar_texts(point_label_names, label_to_id, id_to_label, label_medoids)
    targets = [prefix, prefix.with_name(prefix.name + ".data")] + [prefix.with_name(prefix.name + k) for k in side]
    _refuse_existing(*targets)
    t0 = time.perf_counter()
    _publish(prefix, encode_csr_graph(row_offsets, row_ids, 0))
    t1 = time.perf_counter()
    data_out = targets[1]
    tmp = data_out.with_name(data_out.name + ".tmp")
    _refuse_existing(tmp)
    shutil.copyfile(data_path, tmp)
    os.replace(tmp, data_out)
    for k, text in side.items():
        _publish(prefix.with_name(prefix.name + k), text.encode())
    return {"write_index_seconds": t1 - t0, "metadata_seconds": time.perf_counter() - t1}


def _parse_rows(path):
    with open(path) as f:
        return [[int(v) for v in line.strip().split(",") if v] for line in f]


def audit_stitched_index(prefix, max_degree: int) -> dict:
    """Graph and sidecar audit after the reference's stitched gate
    (tools/validate_gpu_stitched_gate.py:26-145): header size and degree,
    invalid ids, self loops, duplicates, rows over max_degree, edges between
    points without a common label, and medoids that carry their label."""
    prefix = Path(prefix)
    labels = _parse_rows(prefix.with_name(prefix.name + "_labels.txt"))
    formatted = _parse_rows(prefix.with_name(prefix.name + "_label_formatted.txt"))
    with open(prefix.with_name(prefix.name + "_labels_map.txt")) as f:
        label_map = {a: int(b) for a, b in (line.rstrip("\n").split("\t") for line in f)}
    medoids = {}
    with open(prefix.with_name(prefix.name + "_labels_to_medoids.txt")) as f:
        for line in f:
            a, b = (int(v.strip()) for v in line.split(","))
            medoids[a] = b
    blob = prefix.read_bytes()
    size, header_degree, start, frozen = GRAPH_HEADER.unpack_from(blob, 0)
    words = np.frombuffer(blob, dtype=np.uint32, offset=GRAPH_HEADER.size)
    n = len(labels)
    label_sets = [set(r) for r in labels]
    res = dict(nodes=0, edges=0, header_max_degree=header_degree, start_node=start, frozen_points=frozen,
               size_matches=size == len(blob), invalid_ids=0, self_loops=0, duplicate_edges=0,
               degree_overflow_rows=0, incompatible_label_edges=0)
    i = 0
    while i < len(words):
        k = int(words[i])
        nb = words[i + 1:i + 1 + k]
        g = res["nodes"]
        res["degree_overflow_rows"] += int(k > max_degree)
        res["invalid_ids"] += int((nb >= n).sum())
        res["self_loops"] += int((nb == g).sum())
        res["duplicate_edges"] += k - len(set(nb.tolist()))
        src = label_sets[g] if g < n else set()
        res["incompatible_label_edges"] += sum(1 for h in nb.tolist() if h < n and not src & label_sets[h])
        res["edges"] += k
        res["nodes"] += 1
        i += 1 + k
    res["average_degree"] = res["edges"] / max(res["nodes"], 1)
    res["sidecar_rows_match"] = len(labels) == len(formatted) == res["nodes"] and all(
        set(a) == set(b) for a, b in zip(labels, formatted))
    res["medoid_labels_match_map"] = set(medoids) == set(label_map.values())
    res["invalid_label_medoids"] = sorted(l for l, m in medoids.items() if m >= n or l not in label_sets[m])
    return res


# ----------------------------------------------------------------- app
TIMING_KEYS = ["num_labels", "npts_per_label_min", "npts_per_label_mean", "npts_per_label_max",
               "total_label_memberships", "processed_label_memberships", "remap_invalid_local_ids",
               "remap_self_loops", "remap_duplicate_edges", "label_data_materialization_seconds",
               "per_label_gpu_build_sum_seconds", "per_label_gpu_build_max_seconds",
               "local_to_global_remap_seconds", "write_index_seconds", "final_prune_seconds", "metadata_seconds",
               "total_seconds", "peak_gpu_mem_gb", "output_edges"]


def build_gpu_stitched(data_type: str, data_path, label_file, index_path_prefix, universal_label: str = "",
                       timing_json: str = "", Rsmall: int = 32, Lsmall: int = 100, Rstitched: int = 64,
                       C: int = 96, steps: int = 64, num_threads: int = 32, alpha: float = 1.2, streams: int = 4,
                       allow_unpruned: bool = False) -> dict:
    """The reference app's build_gpu_stitched<T> (:241-428); returns the timing dict."""
    t0 = time.perf_counter()
    if Rstitched < Rsmall:
        Rstitched = Rsmall
    if data_type == "uint8":
        dtype = np.uint8
    elif data_type == "float":
        dtype = np.float32
    else:
        raise ValueError("GPU StitchedMVP supports uint8 and float in this version")
    data = read_bin(data_path, dtype)
    names, label_to_id, id_to_label, label_points = parse_labels(label_file, universal_label)
    if len(names) != data.shape[0]:
        raise ValueError("number of label rows does not match data points")
    single = all(len(r) == 1 for r in names)
    needs_prune = not (single and Rsmall <= Rstitched)
    offs, pts = labels_csr(label_points)
    print(f"[GPU stitched] enabled labels={len(id_to_label)} N={data.shape[0]} dim={data.shape[1]} "
          f"Rsmall={Rsmall} Lsmall={Lsmall} Rstitched={Rstitched} C={C}")
    row_offsets, row_ids, medoids, st = stitched_build(data, offs, pts, Rsmall, Lsmall, Rstitched, C, steps,
                                                       streams=streams)
    prune_seconds = 0.0
    if needs_prune and not allow_unpruned:
        # the union graph is kept as <prefix>_full (:360), the pruned graph is the index
        full = Path(str(index_path_prefix) + "_full")
        _publish(full, encode_csr_graph(row_offsets, row_ids, 0))
        pt0 = time.perf_counter()
        lo, lb = point_label_csr(label_points, data.shape[0])
        row_offsets, row_ids, pruned = global_prune(data, row_offsets, row_ids, lo, lb, Rstitched, 750, alpha)
        prune_seconds = time.perf_counter() - pt0
        print(f"[GPU stitched] global label-aware prune on the GPU: rows_pruned={pruned} seconds={prune_seconds}")
    io = write_stitched_index(index_path_prefix, data_path, row_offsets, row_ids, names, label_to_id, id_to_label,
                              medoids)
    deg = np.diff(row_offsets.astype(np.int64))
    print(f"[GPU stitched] wrote graph bytes={GRAPH_HEADER.size + 4 * len(deg) + 4 * int(row_offsets[-1])} "
          f"edges={int(row_offsets[-1])} avg_degree={int(row_offsets[-1]) / max(len(deg), 1)} "
          f"max_degree={int(deg.max()) if len(deg) else 0}")
    timing = {k: st.get(k, 0) for k in TIMING_KEYS}
    timing.update(io)
    timing["final_prune_seconds"] = prune_seconds
    timing["total_seconds"] = time.perf_counter() - t0
    timing["label_build_wall_seconds"] = st["label_build_wall_seconds"]
    timing["streams"] = st["streams"]
    if single:
        print("[GPU stitched] global label-aware prune is a no-op: single-label rows and Rsmall <= Rstitched")
    print("[GPU stitched timing] " + " ".join(f"{k}={timing[k]}" for k in TIMING_KEYS))
    if timing_json:
        with open(timing_json, "w") as f:
            json.dump({k: timing[k] for k in TIMING_KEYS}, f, indent=2)
            f.write("\n")
    return timing


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="gpu_stitched_vamana_index",
                                 description="Build GPU StitchedVamana for single- or multi-label data.")
    ap.add_argument("--data_type", required=True)
    ap.add_argument("--data_path", required=True)
    ap.add_argument("--label_file", required=True)
    ap.add_argument("--index_path_prefix", required=True)
    ap.add_argument("--universal_label", default="")
    ap.add_argument("--timing_json", default="")
    ap.add_argument("--Rsmall", type=int, default=32)
    ap.add_argument("--Lsmall", type=int, default=100)
    ap.add_argument("--Rstitched", type=int, default=64)
    ap.add_argument("--C", type=int, default=96)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--num_threads", "-T", type=int, default=32)
    ap.add_argument("--alpha", type=float, default=1.2)
    ap.add_argument("--streams", type=int, default=4, help="label builds in flight at once")
    ap.add_argument("--allow_unpruned", action="store_true")
    a = ap.parse_args(argv)
    try:
        build_gpu_stitched(a.data_type, a.data_path, a.label_file, a.index_path_prefix, a.universal_label,
                           a.timing_json, a.Rsmall, a.Lsmall, a.Rstitched, a.C, a.steps, a.num_threads, a.alpha,
                           a.streams, a.allow_unpruned)
    except Exception as e:  # the reference app prints and exits 1 (:437-446)
        print(f"[GPU stitched] failed: {e}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
