"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's own builders -- DANCE src/gpu_vamana_vnew2.cu and the
older v8 builder src/gpu_vamana_uint8.cu, compiled unmodified for sm_100a
into oracle/_ref/ by oracle/ref/Makefile -- on seeded inputs on a B200 and
stores outputs as .npz files plus manifest.json in this directory.
tests/test_oracle.py then checks the oracle (reference slot-pool mode)
against them on the CPU, and tests/test_gpu_parity.py checks the GPU build.

Two shapes: a small one (N=1500, R32 L64 C48 STEPS32; inputs stored in the
.npz) and the benchmarked configuration shape (N=20000, R64 L100 C80
STEPS64; inputs regenerated from the seeded recipe in the manifest, whose
sha256 the loader checks, and graphs stored as uint16 ids).  At the
configuration shape the reference is run twice on the same input: its
reverse-edge fill order comes from atomics, so the agreement between its
own two runs is the yardstick the oracle's agreement is held to.

    python tests/golden/make_golden.py        # needs a GPU and oracle/_ref/*.so
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = HERE.parent.parent / "oracle" / "_ref"
OUT = HERE  # --out: where the new files and the manifest go


def gen_u8(n, dim, seed, centroids=24):
    rng = np.random.default_rng(seed)
    cent = rng.uniform(0, 255, (centroids, dim))
    a = rng.integers(0, centroids, n)
    x = cent[a] + rng.normal(0, 20, (n, dim))
    return np.rint(np.clip(x, 0, 255)).astype(np.uint8)


def gen_f32(n, dim, seed, centroids=24):
    rng = np.random.default_rng(seed)
    cent = rng.normal(size=(centroids, dim))
    a = rng.integers(0, centroids, n)
    x = cent[a] + 0.3 * rng.normal(size=(n, dim))
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x.astype(np.float32)


GENERATORS = {"u8": gen_u8, "f32": gen_f32}


def gen_queries(spec: dict, nq: int, seed: int) -> np.ndarray:
    """Queries from the same mixture as a data_spec input: the centroids are
    the generator's first draw from the input's seed; assignments and noise
    come from `seed`."""
    c, dim = spec["centroids"], spec["dim"]
    if spec["gen"] == "u8":
        cent = np.random.default_rng(spec["seed"]).uniform(0, 255, (c, dim))
        rng = np.random.default_rng(seed)
        x = cent[rng.integers(0, c, nq)] + rng.normal(0, 20, (nq, dim))
        return np.rint(np.clip(x, 0, 255)).astype(np.uint8)
    cent = np.random.default_rng(spec["seed"]).normal(size=(c, dim))
    rng = np.random.default_rng(seed)
    x = cent[rng.integers(0, c, nq)] + 0.3 * rng.normal(size=(nq, dim))
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x.astype(np.float32)


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def case_data(case: dict, z) -> np.ndarray:
    """The input vectors of a golden case: stored in the .npz (small shape) or
    regenerated from the manifest's recipe and checked against its sha256."""
    if "data" in z:
        return z["data"]
    spec = case["data_spec"]
    x = GENERATORS[spec["gen"]](spec["n"], spec["dim"], spec["seed"], spec["centroids"])
    if sha256(x) != spec["sha256"]:
        raise RuntimeError(f"regenerated input of {case['file']} differs from the recorded one")
    return x


def case_graph(z) -> np.ndarray:
    """Graph ids as uint32 with 0xFFFFFFFF padding (config-shape files store uint16)."""
    g = z["graph"]
    if g.dtype == np.uint16:
        g = np.where(g == 0xFFFF, np.uint32(0xFFFFFFFF), g.astype(np.uint32))
    return g


def run(lib_name, fn, data, R, L, C, S, medoid_fn="gpu_vamana_vnew2_get_last_medoid"):
    lib = ctypes.CDLL(str(REF / lib_name))
    f = getattr(lib, fn)
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] + [ctypes.c_uint32] * 6 + [ctypes.c_void_p] * 2
    getattr(lib, medoid_fn).restype = ctypes.c_uint32
    n, dim = data.shape
    g = np.zeros((n, R), np.uint32)
    d = np.zeros(n, np.uint32)
    rc = f(ctypes.c_void_p(data.ctypes.data), n, dim, R, L, C, S, ctypes.c_void_p(g.ctypes.data),
           ctypes.c_void_p(d.ctypes.data))
    if rc != 0:
        raise RuntimeError(f"{lib_name}:{fn} returned {rc}")
    return g, d, int(getattr(lib, medoid_fn)())


def agreement(g1, d1, g2, d2):
    """(identical rows, identical row sets) fractions of two graphs."""
    same = (g1 == g2).all(1) & (d1 == d2)
    sets = np.mean([set(a[:x].tolist()) == set(b[:y].tolist()) for a, b, x, y in zip(g1, g2, d1, d2)])
    return float(same.mean()), float(sets)


def config_shape_cases(cases):
    """Reference builds at the benchmarked shape R64 L100 C80 STEPS64, N=20000."""
    R, L, C, S, N = 64, 100, 80, 64, 20000
    specs = {"u8": dict(gen="u8", n=N, dim=128, seed=4242, centroids=256),
             "f32": dict(gen="f32", n=N, dim=96, seed=4243, centroids=200)}
    runs = [("u8", "quality_it1", 1, "libref_vnew2_quality_it1.so", "gpu_vamana_vnew2_build", "u8"),
            ("u8", "quality", 4, "libref_vnew2_quality.so", "gpu_vamana_vnew2_build", "u8"),
            ("f32", "quality", 4, "libref_vnew2_quality.so", "gpu_vamana_vnew2_build_float", "f32"),
            ("f32", "fast_small", 4, "libref_vnew2_fast_small.so", "gpu_vamana_vnew2_build_float", "f16")]
    for tag, variant, iters, lib, fn, storage in runs:
        spec = dict(specs[tag])
        x = GENERATORS[tag](spec["n"], spec["dim"], spec["seed"], spec["centroids"])
        spec["sha256"] = sha256(x)
        g, d, m = run(lib, fn, x, R, L, C, S)
        g2, d2, m2 = run(lib, fn, x, R, L, C, S)
        rows, sets = agreement(g, d, g2, d2)
        name = f"ref_vnew2_{tag}_{variant}_cfgshape.npz"
        np.savez_compressed(OUT / name, medoid=np.uint32(m), graph=np.where(g == 0xFFFFFFFF, 0xFFFF, g)
                            .astype(np.uint16), degree=d.astype(np.uint8))
        cases.append({"file": name, "dtype": tag, "storage": storage, "R": R, "L": L, "C": C, "STEPS": S,
                      "iters": iters, "variant": variant, "data_spec": spec,
                      "reference_self_agreement": {"rows": rows, "row_sets": sets, "medoid_equal": m == m2}})
        print(f"{name}: reference run-to-run identical rows {rows:.5f}, row sets {sets:.5f}", flush=True)
        if tag == "u8" and iters == 4:  # the v8 builder at the same shape
            g8, d8, m8 = run("libref_v8_quality.so", "gpu_vamana_build", x, R, L, C, S,
                             medoid_fn="gpu_vamana_get_last_medoid")
            rows8, sets8 = agreement(g8, d8, g, d)
            name8 = "ref_v8_u8_quality_cfgshape.npz"
            np.savez_compressed(OUT / name8, medoid=np.uint32(m8), graph=np.where(g8 == 0xFFFFFFFF, 0xFFFF, g8)
                                .astype(np.uint16), degree=d8.astype(np.uint8))
            cases.append({"file": name8, "dtype": tag, "storage": storage, "R": R, "L": L, "C": C, "STEPS": S,
                          "iters": iters, "variant": "v8_quality", "builder": "v8", "data_spec": spec,
                          "v8_vs_vnew2": {"rows": rows8, "row_sets": sets8, "medoid_equal": m8 == m}})
            print(f"{name8}: v8 vs vnew2 identical rows {rows8:.5f}, row sets {sets8:.5f}", flush=True)


def v8_cases(cases, inputs):
    """The reference's v8 builder (the default of its sharded disk build) on the
    small-shape inputs, with its agreement to the vnew2 reference build."""
    R, L, C, S = 32, 64, 48, 32
    for tag, x in inputs.items():
        fn = "gpu_vamana_build" if tag == "u8" else "gpu_vamana_build_float"
        g, d, m = run("libref_v8_quality.so", fn, x, R, L, C, S, medoid_fn="gpu_vamana_get_last_medoid")
        vfn = "gpu_vamana_vnew2_build" if tag == "u8" else "gpu_vamana_vnew2_build_float"
        g2, d2, m2 = run("libref_vnew2_quality.so", vfn, x, R, L, C, S)
        rows, sets = agreement(g, d, g2, d2)
        name = f"ref_v8_{tag}_quality.npz"
        np.savez_compressed(OUT / name, data=x, medoid=np.uint32(m), graph=g, degree=d)
        cases.append({"file": name, "dtype": tag, "storage": tag, "R": R, "L": L, "C": C, "STEPS": S, "iters": 4,
                      "variant": "v8_quality", "builder": "v8",
                      "v8_vs_vnew2": {"rows": rows, "row_sets": sets, "medoid_equal": m == m2}})
        print(f"{name}: v8 vs vnew2 identical rows {rows:.5f}, row sets {sets:.5f}, medoid {m} vs {m2}",
              flush=True)


def small_cases(cases, inputs):
    R, L, C, S = 32, 64, 48, 32
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
            np.savez_compressed(OUT / name, **payload)
            cases.append({"file": name, "dtype": tag, "storage": tag, "R": R, "L": L, "C": C, "STEPS": S,
                          "iters": iters, "variant": variant, "min_identical_rows": 0.99})
    # FAST_SMALL profile: float input stored and searched as fp16
    x = inputs["f32"]
    g, d, m = run("libref_vnew2_fast_small.so", "gpu_vamana_vnew2_build_float", x, R, L, C, S)
    name = "ref_vnew2_f32_fast_small.npz"
    np.savez_compressed(OUT / name, data=x, medoid=np.uint32(m), graph=g, degree=d)
    cases.append({"file": name, "dtype": "f32", "storage": "f16", "R": R, "L": L, "C": C, "STEPS": S, "iters": 4,
                  "variant": "fast_small", "min_identical_rows": 0.99})


def main():
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--parts", default="small,v8,cfgshape",
                    help="comma list of small, v8, cfgshape; cases of the parts not named are kept from the "
                         "existing manifest")
    ap.add_argument("--out", default=str(HERE), help="output directory (the manifest is merged from here)")
    a = ap.parse_args()
    parts = set(a.parts.split(","))
    global OUT
    OUT = Path(a.out)
    OUT.mkdir(parents=True, exist_ok=True)
    N = 1500
    inputs = {"u8": gen_u8(N, 128, 101), "f32": gen_f32(N, 96, 202)}
    made = []
    if "small" in parts:
        small_cases(made, inputs)
    if "v8" in parts:
        v8_cases(made, inputs)
    if "cfgshape" in parts:
        config_shape_cases(made)
    manifest = HERE / "manifest.json"
    old = json.loads(manifest.read_text()) if manifest.exists() else []
    names = {c["file"] for c in made}
    cases = [c for c in old if c["file"] not in names] + made
    (OUT / "manifest.json").write_text(json.dumps(cases, indent=1) + "\n")
    print(f"wrote {len(made)} golden cases ({len(cases)} in the manifest) to {OUT}")


if __name__ == "__main__":
    sys.exit(main())
