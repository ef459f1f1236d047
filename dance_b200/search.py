"""Search a DiskANN memory index on the GPU and score it against ground truth.

This is the measuring end of a build: what DiskANN's ``search_memory_index``
does for the graphs the reference writes (reference README.md:78,92,
REPRODUCIBILITY.md:44-52 and :96-104 for the recall tables), here on the
same files with the library's best-first query search
(``dance_search_queries`` / ``dance_search_queries_filtered``):

* the index is ``<prefix>`` (DiskANN graph: u64 size, u32 max degree, u32
  start, u64 frozen points, then ``u32 deg`` + ids per row) and
  ``<prefix>.data`` (``u32 n, u32 dim`` + rows), as written by
  ``formats.save_memory_index`` and ``stitched.write_stitched_index``;
* queries are a ``.bin`` of the same element type, ground truth the
  ``u32 nq, u32 k, ids, dists`` file of ``formats.write_groundtruth``;
* each search starts at the index's start node and keeps a pool of L; the
  first K pool entries are the answer, recall@K is |answer & truth| / K;
* label-filtered search (``--query_filters_file``, one label name per line)
  uses the label sidecars written with the index: ``_labels_map.txt``
  (name -> id), ``_labels.txt`` (the ids of every point) and
  ``_labels_to_medoids.txt`` (id -> start); a filtered query starts at its
  label's medoid and visits only points that carry the label.

    python -m dance_b200.search --data_type uint8 --index_path_prefix IDX \
        --query_file Q.u8bin --gt_file GT.bin -K 10 -L 10 20 50 100

QPS is timed on the device (CUDA events around the search launch, queries
already resident), like a throughput benchmark rather than DiskANN's
per-thread latency loop; the table prints one line per L.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

from . import formats

DATA_TYPES = {"uint8": np.uint8, "float": np.float32}
INVALID = 0xFFFFFFFF


def decode_graph(path):
    """(graph u32 N x max_degree padded with 0xFFFFFFFF, degree u32[N], start)."""
    rows, max_degree, start, _frozen = formats.read_graph(path)
    n = len(rows)
    R = max(1, int(max_degree))
    graph = np.full((n, R), INVALID, dtype=np.uint32)
    degree = np.zeros(n, dtype=np.uint32)
    for i, r in enumerate(rows):
        k = min(len(r), R)
        graph[i, :k] = r[:k]
        degree[i] = k
    return graph, degree, int(start)


def load_memory_index(prefix, data_type: str):
    """(vectors, graph, degree, start) of a DiskANN memory index."""
    prefix = Path(prefix)
    data = formats.read_bin(prefix.with_name(prefix.name + ".data"), DATA_TYPES[data_type])
    graph, degree, start = decode_graph(prefix)
    if graph.shape[0] != data.shape[0]:
        raise ValueError(f"{prefix}: graph has {graph.shape[0]} rows but the data has {data.shape[0]} points")
    if not 0 <= start < data.shape[0]:
        raise ValueError(f"{prefix}: start node {start} outside [0, {data.shape[0]})")
    return data, graph, degree, start


def load_label_sidecars(prefix):
    """(label offsets u32[N+1], labels u32 sorted per point, name -> id, id -> medoid)."""
    prefix = Path(prefix)
    with open(prefix.with_name(prefix.name + "_labels_map.txt")) as f:
        name_to_id = {a: int(b) for a, b in (line.rstrip("\n").split("\t") for line in f if line.strip())}
    offs = [0]
    labs = []
    with open(prefix.with_name(prefix.name + "_labels.txt")) as f:
        for line in f:
            ids = sorted({int(v) for v in line.strip().split(",") if v})
            labs.extend(ids)
            offs.append(len(labs))
    medoids = {}
    with open(prefix.with_name(prefix.name + "_labels_to_medoids.txt")) as f:
        for line in f:
            if line.strip():
                a, b = (int(v.strip()) for v in line.split(","))
                medoids[a] = b
    return np.array(offs, np.uint32), np.array(labs, np.uint32), name_to_id, medoids


def search_memory_index(prefix, data_type: str, queries: np.ndarray, K: int, L_list, truth=None,
                        query_filters=None, visited_log2: int = 12):
    """Search every query at each L; returns one dict per L (ids, qps, recall
    when ``truth`` is given).  ``query_filters`` is a list of label names,
    one per query, for label-filtered search."""
    import torch
    from . import vamana

    data, graph, degree, start = load_memory_index(prefix, data_type)
    n, dim = data.shape
    if queries.shape[1] != dim or queries.dtype != data.dtype:
        raise ValueError(f"queries are {queries.dtype} x {queries.shape[1]}, the index {data.dtype} x {dim}")
    if min(L_list) < K:
        raise ValueError(f"every L must be at least K={K}")
    store, stride = vamana.padded_store(torch.from_numpy(data).cuda())
    g = torch.from_numpy(graph.view(np.int32)).cuda()
    R = graph.shape[1]
    q = torch.from_numpy(np.ascontiguousarray(queries)).cuda()
    filt = None
    if query_filters is not None:
        if len(query_filters) != len(queries):
            raise ValueError(f"{len(query_filters)} query filters for {len(queries)} queries")
        offs, labs, name_to_id, medoids = load_label_sidecars(prefix)
        if len(offs) != n + 1:
            raise ValueError(f"label file has {len(offs) - 1} rows for {n} points")
        missing = sorted({f for f in query_filters if f not in name_to_id})
        if missing:
            raise ValueError(f"query labels not in the index's label map: {missing[:5]}")
        qlab = np.array([name_to_id[f] for f in query_filters], np.uint32)
        qstart = np.array([medoids.get(int(l), start) for l in qlab], np.uint32)
        filt = [torch.from_numpy(a.view(np.int32)).cuda() for a in (offs, labs, qlab, qstart)]
    out = []
    for L in L_list:
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record()
        if filt is None:
            ids, _ = vamana.search_queries(store, dim, stride, g, R, start, q, int(L), int(K), visited_log2)
        else:
            ids, _ = vamana.search_queries_filtered(store, dim, stride, g, R, *filt, q, int(L), int(K), visited_log2)
        ev1.record()
        torch.cuda.synchronize()
        sec = ev0.elapsed_time(ev1) * 1e-3
        found = ids.cpu().numpy().view(np.uint32)
        row = {"L": int(L), "K": int(K), "queries": int(len(queries)), "seconds": sec,
               "qps": len(queries) / sec if sec > 0 else float("inf"), "ids": found}
        if truth is not None:
            row["recall"] = recall_at(found, truth, K)
        out.append(row)
    return out


def recall_at(found: np.ndarray, truth: np.ndarray, K: int) -> float:
    """Mean |found[:K] & truth[:K]| / K (INVALID answers never match)."""
    if truth.shape[0] != found.shape[0]:
        raise ValueError(f"{found.shape[0]} answers for {truth.shape[0]} ground-truth rows")
    if truth.shape[1] < K:
        raise ValueError(f"ground truth has {truth.shape[1]} neighbours per query, fewer than K={K}")
    hits = 0
    for f, t in zip(found[:, :K].tolist(), truth[:, :K].tolist()):
        hits += len(set(f) & set(t))
    return hits / (K * len(truth))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--data_type", choices=sorted(DATA_TYPES), required=True)
    ap.add_argument("--index_path_prefix", required=True)
    ap.add_argument("--query_file", required=True)
    ap.add_argument("--gt_file", default=None)
    ap.add_argument("--query_filters_file", default=None, help="one label name per query (filtered search)")
    ap.add_argument("-K", "--recall_at", type=int, default=10)
    ap.add_argument("-L", "--search_list", type=int, nargs="+", required=True)
    ap.add_argument("--json", action="store_true", help="print one JSON line per L instead of the table")
    a = ap.parse_args(argv)
    queries = formats.read_bin(a.query_file, DATA_TYPES[a.data_type])
    truth = formats.read_groundtruth(a.gt_file)[0] if a.gt_file else None
    filters = None
    if a.query_filters_file:
        with open(a.query_filters_file) as f:
            filters = [line.strip() for line in f if line.strip()]
    rows = search_memory_index(a.index_path_prefix, a.data_type, queries, a.recall_at, a.search_list, truth,
                               filters)
    if a.json:
        for r in rows:
            print(json.dumps({k: v for k, v in r.items() if k != "ids"}))
        return 0
    head = f"{'Ls':>6} {'QPS':>14} {'us per query':>14}"
    if truth is not None:
        head += f" {'Recall@' + str(a.recall_at):>10}"
    print(head)
    for r in rows:
        line = f"{r['L']:>6} {r['qps']:>14.1f} {1e6 / r['qps']:>14.3f}"
        if truth is not None:
            line += f" {100 * r['recall']:>10.2f}"
        print(line)
    return 0


if __name__ == "__main__":
    sys.exit(main())
