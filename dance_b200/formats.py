"""DiskANN on-disk formats used by the DANCE entry points.

Byte layouts (they must stay compatible so DiskANN's search_memory_index
loads the output unchanged):
  vectors  .fbin/.u8bin  : u32 npts, u32 dim, then npts*dim elements
                           (reference REPRODUCIBILITY.md:9-15)
  graph    <prefix>      : u64 file_size, u32 max_degree, u32 start,
                           u64 frozen_points=0, then per row u32 deg and deg
                           u32 ids (apps/utils/gpu_vamana_memory_index.cpp:217-240)
  ground truth           : u32 nq, u32 k, ids u32[nq*k], dists f32[nq*k]
                           (DATASETS.md:112)
  labels sidecars        : <prefix>_labels.txt, _label_formatted.txt,
                           _labels_map.txt, _labels_to_medoids.txt
                           (apps/utils/gpu_stitched_vamana_index.cpp:162-199)
  shard merge medoids    : u32 nshards, u32 1, u32 ids (src/gpu_merge.cu:551-569)
Writers publish atomically (temporary file + rename) and refuse to
overwrite, as the reference app does (gpu_vamana_memory_index.cpp:203-296).
"""
from __future__ import annotations

import os
import struct
from pathlib import Path

import numpy as np

GRAPH_HEADER = struct.Struct("<QIIQ")  # file_size, max_degree, start, frozen_points


def write_bin(path: str | os.PathLike, data: np.ndarray) -> None:
    data = np.ascontiguousarray(data)
    n, d = data.shape
    with open(path, "wb") as f:
        f.write(struct.pack("<II", n, d))
        f.write(data.tobytes())


def read_bin(path: str | os.PathLike, dtype) -> np.ndarray:
    with open(path, "rb") as f:
        n, d = struct.unpack("<II", f.read(8))
        expected = 8 + n * d * np.dtype(dtype).itemsize
        size = os.fstat(f.fileno()).st_size
        if size != expected:
            raise ValueError(f"{path}: header says {n}x{d} but file has {size} bytes (expected {expected})")
        return np.frombuffer(f.read(), dtype=dtype).reshape(n, d).copy()


def _refuse_existing(*paths: Path) -> None:
    for p in paths:
        if p.exists():
            raise FileExistsError(f"refusing to overwrite existing output {p}")


def graph_bytes(degree: np.ndarray, R: int) -> int:
    deg = np.minimum(degree.astype(np.int64), R)
    return GRAPH_HEADER.size + 4 * len(deg) + 4 * int(deg.sum())


def _graph_header_and_words(graph: np.ndarray, degree: np.ndarray, start: int):
    """DiskANN graph layout of an N x R graph (rows padded with 0xFFFFFFFF):
    the 24-byte header and the body words [deg, ids...] row after row."""
    n, R = graph.shape
    deg = np.minimum(degree.astype(np.int64), R).astype(np.uint32)
    max_degree = int(degree.max()) if n else 0
    total = graph_bytes(degree, R)
    header = GRAPH_HEADER.pack(total, max_degree, int(start), 0)
    # rows as [deg, id_0 .. id_{R-1}], kept up to each row's degree, read row-major
    rows = np.empty((n, R + 1), dtype=np.uint32)
    rows[:, 0] = deg
    rows[:, 1:] = graph
    keep = np.arange(R + 1, dtype=np.uint32)[None, :] <= deg[:, None]
    words = rows[keep]
    assert GRAPH_HEADER.size + 4 * len(words) == total
    return header, words


def encode_graph(graph: np.ndarray, degree: np.ndarray, start: int) -> bytes:
    """Serialise an N x R graph (rows padded with 0xFFFFFFFF) in DiskANN layout."""
    header, words = _graph_header_and_words(graph, degree, start)
    return header + words.tobytes()


def write_graph(path: str | os.PathLike, graph: np.ndarray, degree: np.ndarray, start: int) -> None:
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    _refuse_existing(path, tmp)
    header, words = _graph_header_and_words(graph, degree, start)
    total = len(header) + 4 * len(words)
    try:
        with open(tmp, "wb") as f:
            f.write(header)
            words.tofile(f)
        if tmp.stat().st_size != total:
            raise IOError(f"short write to {tmp}")
        os.replace(tmp, path)
    except BaseException:
        if tmp.exists():
            tmp.unlink()
        raise


def read_graph(path: str | os.PathLike):
    """Return (rows: list[np.ndarray], max_degree, start, frozen_points)."""
    blob = Path(path).read_bytes()
    file_size, max_degree, start, frozen = GRAPH_HEADER.unpack_from(blob, 0)
    if file_size != len(blob):
        raise ValueError(f"{path}: header file_size {file_size} != actual {len(blob)}")
    words = np.frombuffer(blob, dtype=np.uint32, offset=GRAPH_HEADER.size)
    rows = []
    i = 0
    while i < len(words):
        k = int(words[i])
        rows.append(words[i + 1:i + 1 + k].copy())
        i += 1 + k
    return rows, max_degree, start, frozen


def save_memory_index(prefix: str | os.PathLike, data: np.ndarray, graph: np.ndarray, degree: np.ndarray,
                      medoid: int) -> None:
    """Graph at <prefix> and vectors at <prefix>.data, published atomically."""
    prefix = Path(prefix)
    data_path = prefix.with_name(prefix.name + ".data")
    _refuse_existing(prefix, data_path)
    tmp_data = data_path.with_name(data_path.name + ".tmp")
    _refuse_existing(tmp_data)
    try:
        write_bin(tmp_data, data)
        write_graph(prefix, graph, degree, medoid)
        os.replace(tmp_data, data_path)
    except BaseException:
        if tmp_data.exists():
            tmp_data.unlink()
        raise


def write_groundtruth(path: str | os.PathLike, ids: np.ndarray, dists: np.ndarray) -> None:
    nq, k = ids.shape
    with open(path, "wb") as f:
        f.write(struct.pack("<II", nq, k))
        f.write(np.ascontiguousarray(ids, dtype=np.uint32).tobytes())
        f.write(np.ascontiguousarray(dists, dtype=np.float32).tobytes())


def read_groundtruth(path: str | os.PathLike):
    with open(path, "rb") as f:
        nq, k = struct.unpack("<II", f.read(8))
        ids = np.frombuffer(f.read(4 * nq * k), dtype=np.uint32).reshape(nq, k).copy()
        dists = np.frombuffer(f.read(4 * nq * k), dtype=np.float32).reshape(nq, k).copy()
    return ids, dists


def audit_graph(graph: np.ndarray, degree: np.ndarray, R: int, medoid: int) -> dict:
    """Invariant audit of the standard app (gpu_vamana_memory_index.cpp:349-384):
    invalid ids, self loops, duplicate neighbours, degree overflow, medoid range."""
    n = graph.shape[0]
    deg = degree.astype(np.int64)
    bad = {"invalid": 0, "self": 0, "duplicate": 0, "overflow": int((deg > R).sum()),
           "medoid_out_of_range": int(not (0 <= medoid < n))}
    mask = np.arange(graph.shape[1])[None, :] < np.minimum(deg, R)[:, None]
    vals = graph.astype(np.int64)
    bad["invalid"] = int(((vals >= n) & mask).sum())
    bad["self"] = int(((vals == np.arange(n)[:, None]) & mask).sum())
    srt = np.sort(np.where(mask, vals, -1 - np.arange(graph.shape[1])[None, :]), axis=1)
    bad["duplicate"] = int(((srt[:, 1:] == srt[:, :-1]) & (srt[:, 1:] >= 0)).sum())
    return bad
