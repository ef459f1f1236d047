"""Generate golden fixtures for the shard merge from the reference's own merge.

Runs DANCE's diskann::merge_shards_gpu (src/gpu_merge.cu:351-871, compiled
unmodified for sm_100a into oracle/_ref/libref_merge.so by
oracle/ref/Makefile, called through the C shim oracle/ref/merge_entry.cpp)
on seeded overlapping shard files on a B200, and stores the merged graph
file and the medoids file it writes, byte for byte, in merge_*.npz plus
manifest_merge.json.  The shard files are regenerated from the seeded recipe
by write_shards(); the manifest records their sha256 so a loader can tell
that it rebuilt the same inputs.  tests/test_merge.py checks the CPU oracle
(and, on a GPU, dance_merge_shards_gpu) against these files.

    python tests/golden/make_golden_merge.py [--out DIR]   # needs a GPU
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
REF = ROOT / "oracle" / "_ref"

# (name, shard recipe, max_degree, environment of the merge call)
CASES = [
    ("merge_3shards_r24", dict(n=3000, nshards=3, width=16, overlap=2, seed=1), 24, {}),
    ("merge_4shards_r48_seed", dict(n=5000, nshards=4, width=32, overlap=2, seed=2), 48,
     {"DISKANN_GPU_MERGE_HASH_SEED": "12345"}),
    ("merge_hubs_r700_buckets", dict(n=2000, nshards=1, width=900, overlap=1, seed=3, hubs=(5, 77)), 700,
     {"DISKANN_GPU_MERGE_BUCKETS": "7"}),
]


def write_shards(dirpath: Path, n, nshards, width, overlap, seed, hubs=()):
    """Shard i: shard{i}.idx (DiskANN graph over local ids) + shard{i}_ids.bin
    (u32 k, u32 1, k global ids).  Every point is in `overlap` random shards;
    local rows are random with random degrees; `hubs` (global ids, single
    shard) get full rows.  Returns (edge sources, edge destinations, shard
    medoids) in global ids and the sha256 of all files written."""
    sys.path.insert(0, str(ROOT))
    from dance_b200 import formats
    rng = np.random.default_rng(seed)
    member = [[] for _ in range(nshards)]
    for v in range(n):
        for s in rng.choice(nshards, size=overlap, replace=False):
            member[s].append(v)
    src_all, dst_all, medoids = [], [], []
    h = hashlib.sha256()
    for s in range(nshards):
        ids = np.array(sorted(member[s]), np.uint32)
        k = len(ids)
        g = np.full((k, width), 0xFFFFFFFF, np.uint32)
        deg = rng.integers(0, min(width, 16) + 1, k).astype(np.uint32)
        for i in range(k):
            g[i, :deg[i]] = rng.integers(0, k, deg[i])
        for hub in hubs:
            i = int(np.searchsorted(ids, hub))
            deg[i] = width
            g[i] = rng.permutation(k)[:width]
        med = int(rng.integers(0, k))
        gp, ip = dirpath / f"shard{s}.idx", dirpath / f"shard{s}_ids.bin"
        formats.write_graph(gp, g, deg, med)
        ip.write_bytes(struct.pack("<II", k, 1) + ids.tobytes())
        h.update(gp.read_bytes())
        h.update(ip.read_bytes())
        for i in range(k):
            src_all.append(np.full(deg[i], ids[i], np.uint32))
            dst_all.append(ids[g[i, :deg[i]]])
        medoids.append(int(ids[med]))
    return (np.concatenate(src_all) if src_all else np.zeros(0, np.uint32),
            np.concatenate(dst_all) if dst_all else np.zeros(0, np.uint32), medoids, h.hexdigest())


def main():
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE))
    out = Path(ap.parse_args().out)
    out.mkdir(parents=True, exist_ok=True)
    lib = ctypes.CDLL(str(REF / "libref_merge.so"))
    f = lib.ref_merge_shards_gpu
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_char_p] * 4 + [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_char_p, ctypes.c_char_p]
    manifest = []
    for name, recipe, R, env in CASES:
        with tempfile.TemporaryDirectory() as td:
            d = Path(td)
            _, _, medoids, digest = write_shards(d, **recipe)
            saved = {k: os.environ.get(k) for k in env}
            os.environ.update(env)
            try:
                pre = str(d / "shard").encode()
                rc = f(pre, b".idx", pre, b"_ids.bin", recipe["nshards"], R, str(d / "merged.idx").encode(),
                       str(d / "medoids.bin").encode())
            finally:
                for k, v in saved.items():
                    if v is None:
                        os.environ.pop(k, None)
                    else:
                        os.environ[k] = v
            if rc != 0:
                raise RuntimeError(f"reference merge returned {rc} on {name}")
            graph = np.frombuffer((d / "merged.idx").read_bytes(), np.uint8)
            med = np.frombuffer((d / "medoids.bin").read_bytes(), np.uint8)
        np.savez_compressed(out / f"{name}.npz", graph_file=graph, medoids_file=med)
        manifest.append({"file": f"{name}.npz", "shards": {k: (list(v) if isinstance(v, tuple) else v)
                                                           for k, v in recipe.items()},
                         "max_degree": R, "env": env, "inputs_sha256": digest, "medoids": medoids,
                         "graph_bytes": int(graph.size)})
        print(f"{name}: merged graph {graph.size} bytes, medoids {medoids}", flush=True)
    (out / "manifest_merge.json").write_text(json.dumps(manifest, indent=1) + "\n")


if __name__ == "__main__":
    sys.exit(main())
