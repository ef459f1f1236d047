"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's own vnew2 builder -- DANCE src/gpu_vamana_vnew2.cu
compiled unmodified for sm_100a into oracle/_ref/ by oracle/ref/Makefile --
on small seeded inputs on a B200 and stores inputs and outputs as .npz files
plus manifest.json in this directory.  tests/test_oracle.py then checks the
oracle (reference slot-pool mode) against them on the CPU.

    python tests/golden/make_golden.py        # needs a GPU and oracle/_ref/*.so
"""
from __future__ import annotations

import ctypes
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = HERE.parent.parent / "oracle" / "_ref"


def gen_u8(n, dim, seed):
    rng = np.random.default_rng(seed)
    cent = rng.uniform(0, 255, (24, dim))
    a = rng.integers(0, 24, n)
    x = cent[a] + rng.normal(0, 20, (n, dim))
    return np.rint(np.clip(x, 0, 255)).astype(np.uint8)


def gen_f32(n, dim, seed):
    rng = np.random.default_rng(seed)
    cent = rng.normal(size=(24, dim))
    a = rng.integers(0, 24, n)
    x = cent[a] + 0.3 * rng.normal(size=(n, dim))
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x.astype(np.float32)


def run(lib_name, fn, data, R, L, C, S):
    lib = ctypes.CDLL(str(REF / lib_name))
    f = getattr(lib, fn)
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] + [ctypes.c_uint32] * 6 + [ctypes.c_void_p] * 2
    lib.gpu_vamana_vnew2_get_last_medoid.restype = ctypes.c_uint32
    n, dim = data.shape
    g = np.zeros((n, R), np.uint32)
    d = np.zeros(n, np.uint32)
    rc = f(ctypes.c_void_p(data.ctypes.data), n, dim, R, L, C, S, ctypes.c_void_p(g.ctypes.data),
           ctypes.c_void_p(d.ctypes.data))
    if rc != 0:
        raise RuntimeError(f"{lib_name}:{fn} returned {rc}")
    return g, d, int(lib.gpu_vamana_vnew2_get_last_medoid())


def main():
    R, L, C, S, N = 32, 64, 48, 32, 1500
    cases = []
    inputs = {"u8": gen_u8(N, 128, 101), "f32": gen_f32(N, 96, 202)}
    for tag, x in inputs.items():
        fn = "gpu_vamana_vnew2_build" if tag == "u8" else "gpu_vamana_vnew2_build_float"
        for variant, iters in [("quality_it0", 0), ("quality_it1", 1), ("quality", 4)]:
            g, d, m = run(f"libref_vnew2_{variant}.so", fn, x, R, L, C, S)
            name = f"ref_vnew2_{tag}_{variant}.npz"
            payload = {"data": x, "medoid": np.uint32(m)}
            if iters == 0:
                payload["init_graph"] = g
            else:
                payload["graph"] = g
                payload["degree"] = d
            np.savez_compressed(HERE / name, **payload)
            cases.append({"file": name, "dtype": tag, "storage": tag, "R": R, "L": L, "C": C, "STEPS": S,
                          "iters": iters, "variant": variant, "min_identical_rows": 0.99})
    # FAST_SMALL profile: float input stored and searched as fp16
    x = inputs["f32"]
    g, d, m = run("libref_vnew2_fast_small.so", "gpu_vamana_vnew2_build_float", x, R, L, C, S)
    name = "ref_vnew2_f32_fast_small.npz"
    np.savez_compressed(HERE / name, data=x, medoid=np.uint32(m), graph=g, degree=d)
    cases.append({"file": name, "dtype": "f32", "storage": "f16", "R": R, "L": L, "C": C, "STEPS": S, "iters": 4,
                  "variant": "fast_small", "min_identical_rows": 0.99})
    (HERE / "manifest.json").write_text(json.dumps(cases, indent=1) + "\n")
    print(f"wrote {len(cases)} golden cases to {HERE}")


if __name__ == "__main__":
    sys.exit(main())
