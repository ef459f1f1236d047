"""Golden fixtures of the reference's GPU-FilteredVamana builder.

Two reference builds run on a B200, both from DANCE src/gpu_vamana_filtered.cu
compiled unmodified for sm_100a by oracle/ref/Makefile:

  * oracle/_ref/libref_filtered.so -- the reference C ABI
    (gpu_vamana_filtered_build_uint8 / _float): whole builds, and the status
    of a call whose work width is below 2R;
  * oracle/_ref/libref_filtered_stages.so -- oracle/ref/filtered_stages.cu,
    which includes the same source and runs one canonical round at a time
    with the reference's own kernels, returning every intermediate (task
    search, union search, merged work rows, forward prune, reverse repair),
    plus the reference's random initial graph.

Each case is one .npz (inputs, the random graph, per round the input graph
and all intermediates, the whole-build output) listed in
manifest_filtered.json.  tests/test_filtered.py pins the CPU oracle to them.

    python tests/golden/make_golden_filtered.py [OUT_DIR]   # needs a GPU
"""
from __future__ import annotations

import ctypes
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = HERE.parent.parent / "oracle" / "_ref"
INVALID = 0xFFFFFFFF
U, P = ctypes.c_uint32, ctypes.c_void_p


def ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def gen_labels(n, vocab, seed, max_labels=4):
    """1..max_labels distinct labels per point by Zipf(1) popularity, rows ascending."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, vocab + 1)
    p /= p.sum()
    offs = [0]
    labs = []
    for _ in range(n):
        k = int(rng.integers(1, max_labels + 1))
        labs.extend(sorted(rng.choice(vocab, size=k, replace=False, p=p).tolist()))
        offs.append(len(labs))
    return np.array(offs, np.uint32), np.array(labs, np.uint32)


def label_starts(offs, labs, vocab, seed):
    """A deterministic member of each label as its start (INVALID when unused)."""
    rng = np.random.default_rng(seed)
    members = [[] for _ in range(vocab)]
    for pnt in range(len(offs) - 1):
        for l in labs[offs[pnt]:offs[pnt + 1]]:
            members[l].append(pnt)
    return np.array([m[int(rng.integers(0, len(m)))] if m else INVALID for m in members], np.uint32)


def gen_data(kind, n, dim, seed):
    rng = np.random.default_rng(seed)
    cent = rng.normal(size=(16, dim)) if kind == "f32" else rng.uniform(0, 255, (16, dim))
    a = rng.integers(0, 16, n)
    if kind == "f32":
        x = cent[a] + 0.3 * rng.normal(size=(n, dim))
        return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)
    return np.rint(np.clip(cent[a] + rng.normal(0, 20, (n, dim)), 0, 255)).astype(np.uint8)


def whole_build(x, offs, labs, starts, vocab, universal, global_start, R, L, FL, C, S, alpha):
    lib = ctypes.CDLL(str(REF / "libref_filtered.so"))
    fn = lib.gpu_vamana_filtered_build_float if x.dtype == np.float32 else lib.gpu_vamana_filtered_build_uint8
    fn.restype = ctypes.c_int
    fn.argtypes = [P, U, U, U, U, U, U, U, ctypes.c_float, P, P, U, P, U, U, U, P, P, U, P, P]
    n, dim = x.shape
    g = np.full((n, R), INVALID, np.uint32)
    d = np.zeros(n, np.uint32)
    rc = fn(ptr(x), n, dim, R, L, FL, C, S, alpha, ptr(offs), ptr(labs), len(labs), ptr(starts), vocab, universal,
            global_start, None, None, 0, ptr(g), ptr(d))
    return rc, g, d


def stages():
    lib = ctypes.CDLL(str(REF / "libref_filtered_stages.so"))
    lib.ref_filtered_round_stages.restype = ctypes.c_int
    lib.ref_filtered_round_stages.argtypes = ([ctypes.c_int, P, U, U, U, U, U, U, U, ctypes.c_float, P, P, U, P, U,
                                               U, U, P, P] + [P] * 11)
    lib.ref_filtered_random_graph.restype = ctypes.c_int
    lib.ref_filtered_random_graph.argtypes = [U, U, U, U, P, P]
    return lib


SPECS = [
    # name, kind, n, dim, vocab, universal, R, L, FL, C, STEPS
    ("f32_d96", "f32", 600, 96, 16, INVALID, 24, 48, 48, 64, 24),
    ("f32_d40_universal", "f32", 500, 40, 12, 3, 16, 32, 40, 40, 16),
    ("u8_d128", "u8", 600, 128, 16, INVALID, 24, 48, 48, 72, 24),
    ("u8_d64_smallpool", "u8", 500, 64, 10, INVALID, 16, 20, 20, 40, 16),
]
ROUND_KEYS = ["ti", "td", "oi", "od", "wi", "wd", "wdeg", "fg", "fd", "go", "do"]


def main():
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE
    out.mkdir(parents=True, exist_ok=True)
    lib = stages()
    cases = []
    for i, (name, kind, n, dim, vocab, universal, R, L, FL, C, S) in enumerate(SPECS):
        x = gen_data(kind, n, dim, 300 + i)
        offs, labs = gen_labels(n, vocab, 400 + i)
        starts = label_starts(offs, labs, vocab, 500 + i)
        gstart = int(starts[0]) if starts[0] != INVALID else 0
        alpha = 1.2
        Cw = min(C, 128)
        T = len(labs)
        keep, okeep = min(min(FL, 32), 8), min(R, L)
        rg = np.zeros((n, R), np.uint32)
        rd = np.zeros(n, np.uint32)
        if lib.ref_filtered_random_graph(n, R, min(16, R), 42, ptr(rg), ptr(rd)) != 0:
            raise RuntimeError("reference random graph failed")
        payload = dict(data=x, offsets=offs, labels=labs, starts=starts, random_graph=rg, random_degree=rd)
        g, d = rg, rd
        for rnd in range(3):
            bufs = dict(ti=np.zeros((T, keep), np.uint32), td=np.zeros((T, keep), np.float32),
                        oi=np.zeros((n, okeep), np.uint32), od=np.zeros((n, okeep), np.float32),
                        wi=np.zeros((n, Cw), np.uint32), wd=np.zeros((n, Cw), np.float32),
                        wdeg=np.zeros(n, np.uint32), fg=np.zeros((n, R), np.uint32), fd=np.zeros(n, np.uint32),
                        go=np.zeros((n, R), np.uint32), do=np.zeros(n, np.uint32))
            rc = lib.ref_filtered_round_stages(1 if kind == "u8" else 0, ptr(x), n, dim, R, L, FL, Cw, S, alpha,
                                               ptr(offs), ptr(labs), T, ptr(starts), vocab, universal, gstart,
                                               ptr(g), ptr(d), *[ptr(bufs[k]) for k in ROUND_KEYS])
            if rc != 0:
                raise RuntimeError(f"{name} round {rnd}: stage harness returned {rc}")
            payload[f"r{rnd}_graph_in"] = g
            payload[f"r{rnd}_degree_in"] = d
            for k in ROUND_KEYS:
                payload[f"r{rnd}_{k}"] = bufs[k]
            g, d = bufs["go"], bufs["do"]
        rc, wg, wdg = whole_build(x, offs, labs, starts, vocab, universal, gstart, R, L, FL, C, S, alpha)
        if rc != 0:
            raise RuntimeError(f"{name}: reference returned {rc}")
        payload["build_graph"] = wg
        payload["build_degree"] = wdg
        file = f"ref_filtered_{name}.npz"
        np.savez_compressed(out / file, **payload)
        cases.append({"file": file, "dtype": kind, "num_labels": vocab, "universal": universal,
                      "global_start": gstart, "R": R, "L": L, "FL": FL, "C": C, "STEPS": S, "alpha": alpha})
    # C below 2R: the reference refuses with status 1 before building
    x = gen_data("f32", 200, 32, 9)
    offs, labs = gen_labels(200, 8, 10)
    starts = label_starts(offs, labs, 8, 11)
    rc, _, _ = whole_build(x, offs, labs, starts, 8, INVALID, 0, 32, 64, 64, 48, 32, 1.2)
    cases.append({"status_case": "C < 2R", "R": 32, "C": 48, "status": rc})
    (out / "manifest_filtered.json").write_text(json.dumps(cases, indent=1) + "\n")
    print(f"wrote {len(cases)} filtered golden cases to {out}")


if __name__ == "__main__":
    sys.exit(main())
