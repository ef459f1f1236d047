"""Build recipe of libdance_b200.so (sm_100a only).

    python -m dance_b200.build            # build dance_b200/libdance_b200.so
    python -m dance_b200.build --ptxas-v  # also print registers / spills

The library is built in-tree with nvcc so that it travels with the source
tree to the GPU host; there is no JIT path and no fallback.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import time
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libdance_b200.so"

SOURCES = ["vamana_build.cu", "vamana_sharded.cu", "gpu_merge.cu", "stitched.cu", "filtered.cu", "label_starts.cu"]
HEADERS = ["dance_common.cuh", "vamana_kernels.cuh", "host_common.cuh", "filtered_kernels.cuh",
           "gram_u8.cuh", "prune_quad.cuh", "stitched_prune.cuh"]
PUBLIC_HEADERS = ["dance_b200.h", "gpu_vamana_builder.h", "gpu_vamana_config.h", "gpu_merge.h",
                  "gpu_vamana_filtered.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; set NVCC or put CUDA on PATH")
    return cand


def host_compiler() -> list[str]:
    # The system g++ ships the OpenMP/libstdc++ pieces nvcc expects.
    return ["-ccbin", "/usr/bin/g++"] if Path("/usr/bin/g++").exists() else []


def _inputs() -> list[Path]:
    return ([CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS]
            + [ROOT / "include" / h for h in PUBLIC_HEADERS] + [Path(__file__)])


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs() if p.exists())


def build(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    started = time.time()
    cmd = [nvcc(), *host_compiler(), *ARCH, "-O3", "-std=c++17", "-lineinfo",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "--expt-relaxed-constexpr", "-shared",
           "-I", str(ROOT / "include"), "-o", str(LIB) + ".tmp"]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    cmd += ["--threads", "2"]
    # extra defines, e.g. DANCE_NVCC_FLAGS="-DVAMANA_ITERS=3 -DENABLE_FLOAT16_BUILD=1"
    cmd += os.environ.get("DANCE_NVCC_FLAGS", "").split()
    cmd += [str(CSRC / s) for s in SOURCES]
    cmd += ["-lnccl"]  # resolves to libnccl.so.2 (the copy torch loads when it is imported first)
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libdance_b200.so")
    if ptxas_v or verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    # stamp the library with the time the compile started, so a source edited
    # while nvcc ran leaves it stale
    os.utime(LIB, (started, started))
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    args = ap.parse_args()
    out = build(force=True if args.ptxas_v else args.force, ptxas_v=args.ptxas_v, verbose=True)
    print(out)


if __name__ == "__main__":
    main()
