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

SOURCES = ["vamana_build.cu", "vamana_sharded.cu", "gpu_merge.cu", "stitched.cu", "filtered.cu", "label_starts.cu",
           "partition.cu"]
HEADERS = ["dance_common.cuh", "vamana_kernels.cuh", "host_common.cuh", "filtered_kernels.cuh",
           "gram_u8.cuh", "prune_quad.cuh", "stitched_prune.cuh", "replay_umma.cuh", "comm.cuh"]
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


def _compile_cmd(src: Path, obj: Path, ptxas_v: bool) -> list[str]:
    cmd = [nvcc(), *host_compiler(), *ARCH, "-O3", "-std=c++17", "-lineinfo",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "--expt-relaxed-constexpr", "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    # extra defines, e.g. DANCE_NVCC_FLAGS="-DVAMANA_ITERS=3 -DENABLE_FLOAT16_BUILD=1"
    cmd += os.environ.get("DANCE_NVCC_FLAGS", "").split()
    return cmd


def build(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> Path:
    """Compile every source to an object in parallel (one nvcc per source,
    as many at once as the host has cores), then link the shared library."""
    if not force and up_to_date():
        return LIB
    started = time.time()
    objdir = ROOT / "_build" / "objs"
    objdir.mkdir(parents=True, exist_ok=True)
    jobs = []
    for s in SOURCES:
        obj = objdir / (Path(s).stem + ".o")
        cmd = _compile_cmd(CSRC / s, obj, ptxas_v)
        if verbose:
            print(" ".join(cmd), flush=True)
        jobs.append((s, obj, cmd))
    width = max(1, min(len(jobs), os.cpu_count() or 1))
    running: list = []
    failed = []
    pending = list(jobs)
    while pending or running:
        while pending and len(running) < width:
            s, obj, cmd = pending.pop(0)
            running.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        s, proc = running.pop(0)
        out, _ = proc.communicate()
        if proc.returncode != 0:
            failed.append((s, out))
        elif ptxas_v or verbose:
            sys.stderr.write(out)
    if failed:
        for s, out in failed:
            sys.stderr.write(f"--- {s}\n{out}")
        raise RuntimeError("nvcc failed building libdance_b200.so: " + ", ".join(s for s, _ in failed))
    link = [nvcc(), *host_compiler(), *ARCH, "-shared", "-o", str(LIB) + ".tmp",
            *[str(obj) for _, obj, _ in jobs], "-lnccl"]  # libnccl.so.2, the copy torch loads when imported first
    if verbose:
        print(" ".join(link), flush=True)
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("linking libdance_b200.so failed")
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
