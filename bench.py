#!/usr/bin/env python
"""Vamana build throughput on B200 (BASELINE.json metric).

One step = one complete Vamana build (medoid, random init, 4 synchronous
rounds of GreedySearch + online RobustInsert, exact reverse-edge merge,
RobustPrune) of BASELINE.json configs[1]: N=10,000,000 uint8 vectors, d=128,
4096-centroid mixture (U[0,255] centroids, N(0,20) noise, clipped, rounded),
R=64, L=100, C=80, STEPS=64, alpha=1.2, seed 42.  Synthetic data generated
on the GPU with a seeded torch generator stands in for the reference's
datasets.  The 1.28 GB vector store exceeds the 126 MB L2, so no flush is
needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Output: one JSON line on rank 0.  `value` = vectors/s of the device-resident
build (inputs already in HBM, CUDA events on the build stream, max over
ranks); `e2e` = the same metric through the reference C ABI
gpu_vamana_vnew2_build with pinned host buffers (H2D of the vectors and D2H
of graph + degrees inside the timed region).  `--impl reference` times the
reference algorithm's CPU restatement (oracle/) on the host cores on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOAD = dict(name="cfg1_u8_10M", N=10_000_000, dim=128, centroids=4096, noise=20.0, R=64, L=100, C=80, STEPS=64,
                alpha=1.2, iters=4, seed=42, queries=10_000)
REF_SAMPLE = 32_768      # vectors per step of the --impl reference CPU arm
CPU_BASELINE_SAMPLE = 65_536  # vectors of the cpu_baseline sample in our arm


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n", "--num-points", dest="n", type=int, default=WORKLOAD["N"],
                    help="override N (profiling small cases); under torchrun spell it --num-points")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-recall", action="store_true")
    ap.add_argument("--no-ref-gpu", dest="ref_gpu", action="store_false",
                    help="skip the reference's own GPU build (run by default at N=1)")
    ap.add_argument("--no-others", action="store_true",
                    help="skip the other workloads that the default N=1 line carries in other_workloads")
    ap.add_argument("--cfg0-storage", choices=["f16", "f32"], default="f16",
                    help="cfg0_f32 vector storage: f16 (the reference's FAST_SMALL) or f32 (QUALITY)")
    ap.add_argument("--ref-gpu", action="store_true", default=True,
                    help="also time the reference's own GPU builder (oracle/_ref, sm_100a) once on the workload")
    ap.add_argument("--workload", choices=["cfg1_u8_10M", "cfg0_f32", "cfg2_filtered", "cfg3_stitched",
                                           "cfg4_f32_100M", "cfg1_disk_sharded"],
                    default="cfg1_u8_10M",
                    help="cfg1_u8_10M: the headline standard build; cfg0_f32: configs[0], 1M float vectors "
                         "stored in fp16 (FAST_SMALL); cfg2_filtered: the GPU-FilteredVamana build of "
                         "BASELINE.json configs[2]; cfg3_stitched: the per-label stitched build of configs[3]; "
                         "cfg4_f32_100M: configs[4], 100M x 96 float32 over the GPUs of one box (torchrun); "
                         "cfg1_disk_sharded: the sharded disk-index pipeline (k-means partition, shard builds, "
                         "GPU merge, DiskANN files) on the configs[1] vectors")
    ap.add_argument("--ram-budget-gb", type=float, default=3.0,
                    help="cfg1_disk_sharded: DiskANN's per-shard build-memory budget (sets the part count)")
    ap.add_argument("--index-dir", default="",
                    help="cfg4: where to write (and read back) the DiskANN graph file; default: a temp dir")
    return ap.parse_args()


# ------------------------------------------------------------------ helpers
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def emit(args, line):
    """Print the JSON line, or hand it to the caller that collects the other
    workloads into the headline line (args.collect)."""
    if getattr(args, "collect", None) is not None:
        args.collect.append(line)
    else:
        print(json.dumps(line), flush=True)


def graph_digest_device(graph, degree, n):
    """64-bit polynomial digest of the first n rows and degrees, computed on
    the GPU (for graphs too large to hash on the host quickly); equal graphs
    give equal digests."""
    import torch
    w = (torch.arange(graph.shape[1], device=graph.device, dtype=torch.int64) * 2654435761 + 97) | 1
    h = 0
    for a in range(0, n, 1 << 22):  # row chunks keep the int64 temporaries near 2 GB
        e = min(n, a + (1 << 22))
        row = (graph[a:e].to(torch.int64) * w[None, :]).sum(1) + degree[a:e].to(torch.int64) * 40503
        rw = (torch.arange(a, e, device=graph.device, dtype=torch.int64) * 6364136223846793005) | 1
        h = (h + int((row * rw).sum().item())) & ((1 << 64) - 1)
    return f"poly:{h:016x}"


def graph_digest(graph, degree, n):
    """sha256 (first 16 hex digits) of the first n graph rows and degrees as
    int32 bytes: equal digests across N=1/2/4/8 show identical graphs."""
    import hashlib
    h = hashlib.sha256()
    h.update(graph[:n].contiguous().cpu().numpy().tobytes())
    h.update(degree[:n].contiguous().cpu().numpy().tobytes())
    return h.hexdigest()[:16]


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_launch(kernel: str, workload: str, n: int):
    """DRAM bytes (read+write) per launch of `kernel` at the full workload, from
    the committed ncu summary profiles/<kernel>_traffic_<workload>.md, or None."""
    import re
    if n != WORKLOAD["N"]:
        return None
    p = ROOT / "profiles" / f"{kernel}_traffic_{workload}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", p.read_text())
    return int(m.group(1)) if m else None


def make_workload(device, n, seed=WORKLOAD["seed"]):
    from dance_b200 import workloads
    return workloads.clustered_u8(n, WORKLOAD["dim"], centroids=WORKLOAD["centroids"], noise=WORKLOAD["noise"],
                                  seed=seed, device=device)


def make_queries(device):
    from dance_b200 import workloads
    return workloads.clustered_u8(WORKLOAD["queries"], WORKLOAD["dim"], centroids=WORKLOAD["centroids"],
                                  noise=WORKLOAD["noise"], seed=WORKLOAD["seed"], device=device, stream_offset=1)


def oracle_sample_rate(sample_u8, threads, iters=1):
    """Vectors/s of the CPU oracle building the sample (best of `iters`)."""
    import oracle
    best = None
    for _ in range(iters):
        t = time.perf_counter()
        oracle.build_graph(sample_u8, WORKLOAD["R"], WORKLOAD["L"], WORKLOAD["C"], WORKLOAD["STEPS"],
                           nthreads=threads)
        dt = time.perf_counter() - t
        best = dt if best is None else min(best, dt)
    return len(sample_u8) / best, best


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    import numpy as np
    import torch
    import oracle
    oracle.build()
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    sample = make_workload(dev, REF_SAMPLE).cpu().numpy()
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        oracle.build_graph(sample, WORKLOAD["R"], WORKLOAD["L"], WORKLOAD["C"], WORKLOAD["STEPS"], nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.build_graph(sample, WORKLOAD["R"], WORKLOAD["L"], WORKLOAD["C"], WORKLOAD["STEPS"], nthreads=threads)
    dt = time.perf_counter() - t0
    value = REF_SAMPLE * args.steps / dt
    sample_desc = (f"first {REF_SAMPLE} vectors of the {WORKLOAD['name']} workload, full 4-round build per step, "
                   f"{threads} OpenMP threads")
    line = {
        "impl": "reference", "metric": "vamana_build_vectors_per_s", "value": value, "unit": "vectors/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": config_dict(REF_SAMPLE),
        "cpu_baseline": {"value": value, "unit": "vectors/s", "cores": threads, "kind": "port",
                         "sample": sample_desc},
        "e2e": {"value": value, "unit": "vectors/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("DANCE has no CPU implementation of this path and DiskANN's CPU Vamana is not vendored; "
                 "this arm runs the C++ restatement of the reference algorithm (oracle/vamana_oracle.cpp)"),
    }
    emit(args, line)
    return 0


def config_dict(n):
    return {"workload": WORKLOAD["name"], "N": n, "dim": WORKLOAD["dim"], "R": WORKLOAD["R"], "L": WORKLOAD["L"],
            "C": WORKLOAD["C"], "STEPS": WORKLOAD["STEPS"], "alpha": WORKLOAD["alpha"], "iters": WORKLOAD["iters"],
            "seed": WORKLOAD["seed"], "l2": "inputs larger than L2 (1.28 GB vector store), no flush"}


# ------------------------------------------------------------------ our arm
def search_algorithmic_bytes(rep, n, row_bytes, R, iters):
    """Algorithmic DRAM bytes of the GreedySearch kernel over one build:
    one gathered vector per distance evaluation, one adjacency row + degree
    per expansion (+ the 8-byte expansion record written), and per vertex
    and round its query vector, own row ids+distances and degree."""
    per_eval = row_bytes
    per_exp = R * 4 + 4 + 8
    per_vertex = row_bytes + R * 8 + 4 + 4
    return rep["search_evals"] * per_eval + rep["expansions"] * per_exp + iters * n * per_vertex


def run_ours(args):
    import numpy as np
    import torch
    import dance_b200
    from dance_b200 import vamana, workloads
    rank, world, local = dist_env()
    if world > 1:
        return run_sharded(args)
    torch.cuda.set_device(local)
    dance_b200.load()
    lib = dance_b200.load()
    n = args.n
    R, L, C, S = WORKLOAD["R"], WORKLOAD["L"], WORKLOAD["C"], WORKLOAD["STEPS"]
    x = make_workload("cuda", n)
    store, stride = vamana.padded_store(x)
    row_bytes = stride
    ws = vamana.Workspace.create(n, R, L, C, S)
    prm = dance_b200.default_params()
    graph = torch.empty((n, R), dtype=torch.int32, device="cuda")
    degree = torch.empty((n,), dtype=torch.int32, device="cuda")
    dists = torch.empty((n, R), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def one_build():
        with torch.cuda.stream(stream):
            return vamana.build_resident(store, WORKLOAD["dim"], stride, R, L, C, S, params=prm, workspace=ws,
                                         graph=graph, degree=degree, dists=dists, stream=stream)

    for _ in range(args.warmup):
        one_build()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    launches0 = lib.dance_kernel_launch_count()
    reports = []
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        _, _, _, medoid = one_build()
        reports.append(dance_b200.last_build_report())
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = lib.dance_kernel_launch_count() - launches0
    clk = clocks.stop()
    elapsed = ev0.elapsed_time(ev1) * 1e-3
    value = n * args.steps / elapsed

    # roofline of the dominant kernel (GreedySearch), from the timed builds
    peak, peak_kind = measured_peaks()
    alg = sum(search_algorithmic_bytes(r, n, row_bytes, R, WORKLOAD["iters"]) for r in reports)
    ksec = sum(r["search_kernel_seconds"] for r in reports)
    achieved = alg / ksec / 1e9
    launches_per_build = WORKLOAD["iters"]
    stage = {k: statistics.mean(r[k] for r in reports) for k in reports[0] if k.endswith("_seconds")}
    counters = {k: reports[-1][k] for k in ("search_evals", "expansions", "replay_pairs", "reverse_evals",
                                            "prune_pairs")}
    traffic = traffic_per_launch("search_kernel", WORKLOAD["name"], n)

    line = {
        "metric": "vamana_build_vectors_per_s", "value": value, "unit": "vectors/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded GPU generator, BASELINE.json configs[1] recipe)",
        "config": config_dict(n),
        "roofline": {"kernel": "search_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": alg / (len(reports) * launches_per_build),
                     "avg_launch_ms": ksec / (len(reports) * launches_per_build) * 1e3},
        "gpu_launches": int(launches),
        "clocks": clk,
        "stage_seconds": stage,
        "counters_per_build": counters,
    }
    # ---- e2e through the reference C ABI with pinned host buffers
    if not args.no_e2e:
        hx = x.cpu().pin_memory()
        hg = torch.empty((n, R), dtype=torch.int32).pin_memory()
        hd = torch.empty((n,), dtype=torch.int32).pin_memory()
        fn = lib.gpu_vamana_vnew2_build

        def e2e_call():
            rc = fn(ctypes.c_void_p(hx.data_ptr()), n, WORKLOAD["dim"], R, L, C, S, ctypes.c_void_p(hg.data_ptr()),
                    ctypes.c_void_p(hd.data_ptr()))
            dance_b200.check(rc, "gpu_vamana_vnew2_build")

        e2e_call()  # warm-up (allocator, first-touch of pinned pages)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_call()
        torch.cuda.synchronize()
        e2e_dt = time.perf_counter() - t0
        line["e2e"] = {"value": n * args.steps / e2e_dt, "unit": "vectors/s", "h2d_bytes_per_step": int(hx.numel()),
                       "d2h_bytes_per_step": int(hg.numel() * 4 + hd.numel() * 4),
                       "api": "gpu_vamana_vnew2_build (reference C ABI), pinned host buffers, wall clock",
                       "warmup": 1}
        # the C-ABI graph equals the device-resident build's graph
        line["e2e"]["matches_resident_build"] = bool(torch.equal(hg.cuda(), graph))
        del hx
    deg = degree.cpu().numpy()
    line["graph"] = {"medoid": int(medoid), "avg_degree": float(deg.mean()), "max_degree": int(deg.max()),
                     "min_degree": int(deg.min()), "digest": graph_digest(graph, degree, n)}
    # ---- recall@10 at L_search=100 on 10k queries against brute force
    if not args.no_recall:
        q = make_queries("cuda")
        gt, _ = workloads.brute_force_knn(x, q, 10)
        ids, _ = vamana.search_queries(store, WORKLOAD["dim"], stride, graph, R, medoid, q, 100, 10)
        line["recall_at_10"] = {"L_search": 100, "queries": int(q.shape[0]),
                                "ours": vamana.recall_at_k(ids.cpu().numpy(), gt.cpu().numpy())}
    # ---- CPU baseline: the oracle restatement on the host cores, bounded sample
    if not args.no_cpu_baseline:
        sample = x[:min(CPU_BASELINE_SAMPLE, n)].cpu().numpy()
        threads = os.cpu_count() or 1
        rate, secs = oracle_sample_rate(sample, threads)
        line["cpu_baseline"] = {"value": rate, "unit": "vectors/s", "cores": threads, "kind": "port",
                                "sample": f"first {len(sample)} vectors of the workload, full 4-round build "
                                          f"({secs:.1f} s)"}
    if args.ref_gpu:
        ref = reference_gpu(x, store, stride, medoid, args)
        line["reference_gpu"] = ref
        add_recall_delta(line, ref)
    ws.close()
    if not args.no_others and n == WORKLOAD["N"]:
        del graph, degree, dists, store, x, ws
        torch.cuda.empty_cache()
        line["other_workloads"] = run_other_workloads(args)
    emit(args, line)
    return 0


def add_recall_delta(line, ref):
    """recall_at_10.reference / .delta from the reference GPU build's recall on
    the same queries, with the same searcher (north_star: |delta| <= 0.005)."""
    rec = line.get("recall_at_10")
    if rec is not None and isinstance(ref, dict) and "recall_at_10" in ref:
        rec["reference"] = ref["recall_at_10"]
        rec["delta"] = rec["ours"] - ref["recall_at_10"]
        rec["within_0.005"] = abs(rec["delta"]) <= 0.005


def run_other_workloads(args):
    """The other BASELINE.json configurations, each timed like the headline
    (same warm-up and step counts, CUDA events, e2e through the C ABI, recall,
    the reference's own GPU build on the same inputs), folded into the N=1
    line.  Their CPU-oracle samples are left to their own --workload lines."""
    import copy
    import torch
    out = {}
    plan = [("cfg0_f32_quality", run_cfg0, {"cfg0_storage": "f32"}),
            ("cfg0_f16_fast_small", run_cfg0, {"cfg0_storage": "f16"}),
            ("cfg2_filtered", run_filtered, {}),
            ("cfg3_stitched", run_stitched, {})]
    keys = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "dtype", "config", "e2e", "recall_at_10",
            "reference_gpu", "roofline", "graph", "gpu_launches", "stage_seconds", "clocks")
    for name, fn, extra in plan:
        sub = copy.copy(args)
        sub.collect = []
        sub.no_cpu_baseline = True
        sub.n = WORKLOAD["N"]  # each workload's own default size
        for k, v in extra.items():
            setattr(sub, k, v)
        t0 = time.perf_counter()
        try:
            fn(sub)
            got = sub.collect[0]
            entry = {k: got[k] for k in keys if k in got}
        except Exception as e:  # recorded, not fatal: the headline line still prints
            entry = {"error": f"{type(e).__name__}: {e}"}
        entry["wall_s"] = time.perf_counter() - t0
        out[name] = entry
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


def reference_gpu(x, store, stride, our_medoid, args):
    """The reference's own vnew2 builder (DANCE src/gpu_vamana_vnew2.cu compiled
    for sm_100a, QUALITY profile) on the same vectors through its C ABI."""
    import numpy as np
    import torch
    from dance_b200 import vamana, workloads
    lib_path = ROOT / "oracle" / "_ref" / "libref_vnew2_quality.so"
    if not lib_path.exists():
        return {"unavailable": f"{lib_path.name} not built"}
    lib = ctypes.CDLL(str(lib_path))
    f = lib.gpu_vamana_vnew2_build
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] + [ctypes.c_uint32] * 6 + [ctypes.c_void_p] * 2
    lib.gpu_vamana_vnew2_get_last_medoid.restype = ctypes.c_uint32
    n = x.shape[0]
    R, L, C, S = WORKLOAD["R"], WORKLOAD["L"], WORKLOAD["C"], WORKLOAD["STEPS"]
    hx = x.cpu().numpy()
    g = np.zeros((n, R), np.uint32)
    d = np.zeros(n, np.uint32)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = f(ctypes.c_void_p(hx.ctypes.data), n, WORKLOAD["dim"], R, L, C, S, ctypes.c_void_p(g.ctypes.data),
           ctypes.c_void_p(d.ctypes.data))
    dt = time.perf_counter() - t0
    if rc != 0:
        return {"unavailable": f"reference build returned {rc}"}
    med = int(lib.gpu_vamana_vnew2_get_last_medoid())
    q = make_queries("cuda")
    gt, _ = workloads.brute_force_knn(x, q, 10)
    gd = torch.from_numpy(g.view(np.int32)).cuda()
    ids, _ = vamana.search_queries(store, WORKLOAD["dim"], stride, gd, R, med, q, 100, 10)
    return {"e2e_vectors_per_s": n / dt, "seconds": dt, "recall_at_10": vamana.recall_at_k(ids.cpu().numpy(),
                                                                                          gt.cpu().numpy()),
            "medoid": med, "avg_degree": float(d.mean()),
            "build": "DANCE vnew2 QUALITY profile (fp32/u8 distances, VAMANA_ITERS=4), nvcc 12.9 sm_100a"}


CFG4 = dict(name="cfg4_f32_100M", N=100_000_000, dim=96, centroids=16384, sigma=0.3, R=64, L=100, C=80, STEPS=64,
            alpha=1.2, iters=4, seed=42, queries=10_000)


def sharded_ground_truth(x, q, k, rank, world):
    """Exact top-k of the queries over the whole store, each rank taking one
    slice of the base vectors; rank 0 merges the slices by (distance, id)."""
    import torch
    import torch.distributed as dist
    from dance_b200 import workloads
    n = x.shape[0]
    per = (n + world - 1) // world
    b0, b1 = min(n, rank * per), min(n, (rank + 1) * per)
    ids, d = workloads.brute_force_knn(x[b0:b1], q, k)
    ids = ids + b0
    all_i = [torch.empty_like(ids) for _ in range(world)]
    all_d = [torch.empty_like(d) for _ in range(world)]
    dist.all_gather(all_i, ids)
    dist.all_gather(all_d, d)
    ci, cd = torch.cat(all_i, 1), torch.cat(all_d, 1)
    o = torch.argsort(ci, dim=1)
    ci, cd = torch.gather(ci, 1, o), torch.gather(cd, 1, o)
    o2 = torch.argsort(cd, dim=1, stable=True)
    return torch.gather(ci, 1, o2)[:, :k]


def write_and_check_graph_file(path, graph, degree, n, start, rows_per_chunk=1 << 21):
    """Streams the graph to a DiskANN graph file (formats.GRAPH_HEADER layout,
    rows as u32 degree + ids) in row chunks, then reads it back in chunks and
    checks every row against the device graph.  Returns sizes and seconds."""
    import numpy as np
    import torch
    from dance_b200 import formats
    t0 = time.perf_counter()
    deg_all = degree[:n].to(torch.int64)
    R = graph.shape[1]
    total = formats.GRAPH_HEADER.size + 4 * n + 4 * int(deg_all.clamp(max=R).sum().item())
    max_degree = int(deg_all.max().item())
    with open(path, "wb") as f:
        f.write(formats.GRAPH_HEADER.pack(total, max_degree, int(start), 0))
        for a in range(0, n, rows_per_chunk):
            e = min(n, a + rows_per_chunk)
            # [degree, ids...] per row: an (rows, R + 1) block masked to each row's length
            blk = torch.cat([degree[a:e, None], graph[a:e]], 1).cpu().numpy().view(np.uint32)
            dg = blk[:, 0].astype(np.int64)
            f.write(blk[np.arange(R + 1)[None, :] <= dg[:, None]].tobytes())
    t1 = time.perf_counter()
    ok = True
    with open(path, "rb") as f:
        hdr = formats.GRAPH_HEADER.unpack(f.read(formats.GRAPH_HEADER.size))
        ok &= hdr == (total, max_degree, int(start), 0)
        for a in range(0, n, rows_per_chunk):
            e = min(n, a + rows_per_chunk)
            dg = degree[a:e].cpu().numpy().view(np.uint32).astype(np.int64)
            words = np.frombuffer(f.read(4 * int((dg + 1).sum())), dtype=np.uint32)
            offs = np.concatenate([[0], np.cumsum(dg + 1)[:-1]])
            ok &= bool(np.array_equal(words[offs], dg.astype(np.uint32)))
            rows = graph[a:e].cpu().numpy().view(np.uint32)
            mask = np.arange(R)[None, :] < dg[:, None]
            keep = np.ones(len(words), bool)
            keep[offs] = False
            ok &= bool(np.array_equal(words[keep], rows[mask]))
        ok &= f.read(1) == b""
    t2 = time.perf_counter()
    return {"path": str(path), "bytes": total, "write_seconds": t1 - t0, "read_back_seconds": t2 - t1,
            "read_back_equal": bool(ok), "max_degree": max_degree, "start": int(start)}


def run_sharded(args):
    """N > 1: one graph, vertex batches sharded over the ranks (strong scaling);
    every edge goes to the rank that owns its target (grouped NCCL send/recv)
    and the pruned rows are all-gathered, inside libdance_b200.  cfg1 by
    default; --workload cfg4_f32_100M runs BASELINE.json configs[4]."""
    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    import dance_b200
    from dance_b200 import vamana, workloads
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                            device_id=torch.device("cuda", local))
    lib = dance_b200.load()
    big = args.workload == "cfg4_f32_100M"
    spec = CFG4 if big else WORKLOAD
    n = args.n if (args.n != WORKLOAD["N"] or not big) else CFG4["N"]
    R, L, C, S = spec["R"], spec["L"], spec["C"], spec["STEPS"]
    dim = spec["dim"]
    t_gen = time.perf_counter()
    if big:  # the same seeded vectors on every rank
        x = workloads.gaussian_mixture_f32(n, dim, CFG4["centroids"], CFG4["sigma"], seed=CFG4["seed"], device="cuda")
    else:
        x = make_workload("cuda", n)
    store, stride = vamana.padded_store(x)
    torch.cuda.synchronize()
    gen_seconds = time.perf_counter() - t_gen
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.tensor(list(vamana.nccl_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    comm = vamana.Comm(rank, world, bytes(uid.cpu().tolist()), timeout_s=600.0)
    ws = vamana.sharded_workspace(n, world, R, L, C, S)
    _, _, chunk = vamana.shard_range(n, world, rank)
    graph = torch.empty((chunk * world, R), dtype=torch.int32, device="cuda")
    degree = torch.empty((chunk * world,), dtype=torch.int32, device="cuda")
    tdeg = torch.empty((chunk * world,), dtype=torch.int32, device="cuda")
    prm = dance_b200.default_params()
    stream = torch.cuda.Stream()

    def one_build():
        with torch.cuda.stream(stream):
            return vamana.build_sharded(comm, store, dim, stride, R, L, C, S, params=prm, workspace=ws,
                                        graph=graph, degree=degree, table_degree=tdeg, stream=stream)

    for _ in range(args.warmup):
        one_build()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
    launches0 = lib.dance_kernel_launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    reports = []
    sreports = []
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        _, _, medoid = one_build()
        reports.append(dance_b200.last_build_report())
        sreports.append(dance_b200.last_sharded_report())
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = lib.dance_kernel_launch_count() - launches0
    mine = torch.tensor([ev0.elapsed_time(ev1) * 1e-3], dtype=torch.float64, device="cuda")
    dist.all_reduce(mine, op=dist.ReduceOp.MAX)
    elapsed = float(mine.item())
    clk = clocks.stop() if clocks else None
    # per-rank search-kernel roofline (max kernel time over ranks, summed bytes)
    alg = sum(search_algorithmic_bytes(r, 0, stride, R, 0) for r in reports)
    alg += args.steps * spec["iters"] * (n // world) * (stride + R * 8 + 8)
    kt = torch.tensor([sum(r["search_kernel_seconds"] for r in reports), alg], dtype=torch.float64, device="cuda")
    kmax = kt.clone()
    dist.all_reduce(kmax, op=dist.ReduceOp.MAX)
    ksum = kt.clone()
    dist.all_reduce(ksum, op=dist.ReduceOp.SUM)
    # per-stage device time per build on every rank (mean over the timed builds), max and min over ranks
    skeys = [k for k in sreports[0] if k.endswith("_seconds")]
    sv = torch.tensor([statistics.mean(r[k] for r in sreports) for k in skeys], dtype=torch.float64, device="cuda")
    smax, smin = sv.clone(), sv.clone()
    dist.all_reduce(smax, op=dist.ReduceOp.MAX)
    dist.all_reduce(smin, op=dist.ReduceOp.MIN)
    stage_table = {k: {"max": float(smax[i]), "min": float(smin[i])} for i, k in enumerate(skeys)}
    stage_table["edge_bytes_received_per_rank"] = int(sreports[-1]["edge_bytes_received"])
    stage_table["graph_bytes_received_per_rank"] = int(sreports[-1]["graph_bytes_received"])
    digest = None
    if rank == 0:
        try:
            digest = graph_digest_device(graph, degree, n) if big else graph_digest(graph, degree, n)
        except Exception as e:
            digest = f"unavailable: {type(e).__name__}: {e}"
    free_b, total_b = torch.cuda.mem_get_info()
    used_gb = (total_b - free_b) / 1e9
    # e2e: every rank copies the vectors from pinned host memory, builds, rank 0 reads the graph back
    e2e = None
    if big:
        e2e = {"value": None, "unit": "vectors/s",
               "note": "not measured at 100M: each rank would pin a 38.4 GB host copy of the store"}
    if not args.no_e2e and not big:
        hx = x.cpu().pin_memory()
        hg = torch.empty((n, R), dtype=torch.int32).pin_memory()
        hd = torch.empty((n,), dtype=torch.int32).pin_memory()
        dx = torch.empty_like(x)
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            dx.copy_(hx, non_blocking=True)
            st2, _ = vamana.padded_store(dx)
            torch.cuda.synchronize()
            vamana.build_sharded(comm, st2, dim, stride, R, L, C, S, params=prm, workspace=ws,
                                 graph=graph, degree=degree, table_degree=tdeg)
            if rank == 0:
                hg.copy_(graph[:n])
                hd.copy_(degree[:n])
            torch.cuda.synchronize()
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device="cuda")
        dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        e2e = {"value": n * args.steps / float(dt.item()), "unit": "vectors/s",
               "h2d_bytes_per_step": int(hx.numel()) * world, "d2h_bytes_per_step": int(hg.numel() * 4 + hd.numel() * 4),
               "api": "dance_vamana_build_sharded (C ABI) on every rank; vectors copied from pinned host memory "
                      "on every rank, graph read back on rank 0; wall clock, max over ranks",
               "warmup": 0}
    rec = None
    index_file = None
    post_errors = {}
    if rank == 0:  # the measurement itself, on stderr, before anything that could fail
        print(json.dumps({"timed_builds": args.steps, "seconds": elapsed, "vectors_per_s": n * args.steps / elapsed,
                          "digest": digest}), file=sys.stderr, flush=True)
    gt_seconds = None
    if not args.no_recall:
        t_gt = time.perf_counter()
        if big:
            q = workloads.gaussian_mixture_f32(CFG4["queries"], dim, CFG4["centroids"], CFG4["sigma"],
                                               seed=CFG4["seed"], device="cuda", stream_offset=1)
        else:
            q = make_queries("cuda")
        gt = sharded_ground_truth(x, q, 10, rank, world)  # collective: every rank, also on errors below
        gt_seconds = time.perf_counter() - t_gt
        if rank == 0:
            try:
                ids, _ = vamana.search_queries(store, dim, stride, graph, R, medoid, q, 100, 10)
                rec = vamana.recall_at_k(ids.cpu().numpy(), gt.cpu().numpy())
            except Exception as e:
                post_errors["recall"] = f"{type(e).__name__}: {e}"
        del gt
        torch.cuda.empty_cache()
    if big and rank == 0:
        import tempfile
        deg = degree[:n]
        bad = 0
        for a in range(0, n, 1 << 22):
            e = min(n, a + (1 << 22))
            g = graph[a:e]
            bad += int((((g < 0) | (g >= n)) & (torch.arange(R, device="cuda")[None, :] < deg[a:e, None])).sum())
        audit = {"invalid": bad, "min_degree": int(deg.min().item()), "max_degree": int(deg.max().item()),
                 "avg_degree": float(deg.double().mean().item())}
        try:
            d = args.index_dir or tempfile.mkdtemp(prefix="cfg4_index_")
            path = os.path.join(d, "cfg4_f32_100M_R64")
            index_file = write_and_check_graph_file(path, graph, degree, n, medoid)
            os.remove(path)
            if not args.index_dir:
                os.rmdir(d)
        except Exception as e:
            index_file = {"error": f"{type(e).__name__}: {e}"}
        index_file["audit"] = audit
    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = float(ksum[1].item()) / float(kmax[0].item()) / 1e9
        if big:
            cfg = {"workload": CFG4["name"], "N": n, "dim": dim, "R": R, "L": L, "C": C, "STEPS": S,
                   "alpha": CFG4["alpha"], "iters": CFG4["iters"], "seed": CFG4["seed"],
                   "centroids": CFG4["centroids"], "storage": "fp32",
                   "l2": "inputs larger than L2 (38.4 GB vector store), no flush"}
        else:
            cfg = config_dict(n)
        cfg["parallelism"] = (f"vertex shards x{world}; edges to their target's owner by grouped NCCL send/recv; "
                              "pruned rows all-gathered")
        line = {
            "metric": "vamana_build_vectors_per_s", "value": n * args.steps / elapsed, "unit": "vectors/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32" if big else "u8",
            "data": ("synthetic (seeded GPU generator, BASELINE.json configs[4] recipe)" if big else
                     "synthetic (seeded GPU generator, BASELINE.json configs[1] recipe)"),
            "config": cfg,
            "roofline": {"kernel": "search_kernel", "bound": "hbm", "achieved": achieved, "peak": peak * world,
                         "unit": "GB/s", "frac": achieved / (peak * world), "peak_source": peak_kind + f" x{world}",
                         "traffic": None},
            "gpu_launches": int(launches), "gpu_launches_scope": "rank 0",
            "clocks": clk,
            "stage_seconds_per_build": stage_table,
            "graph": {"medoid": int(medoid), "digest": digest},
        }
        if e2e:
            line["e2e"] = e2e
        if rec is not None:
            line["recall_at_10"] = {"L_search": 100, "queries": int(q.shape[0]), "ours": rec,
                                    "ground_truth_seconds": gt_seconds}
        if post_errors:
            line["post_errors"] = post_errors
        if big:
            line["index_file"] = index_file
            line["data_generation_seconds"] = gen_seconds
            line["device_memory_used_gb_rank0"] = used_gb
        emit(args, line)
    del ws
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------ stitched
CFG0 = dict(name="cfg0_f32_1M_fp16", N=1_000_000, dim=96, centroids=1000, sigma=0.3, R=64, L=100, C=80, STEPS=64,
            alpha=1.2, iters=4, seed=42, queries=10_000)
CFG0_CPU_SAMPLE = 8_000  # vectors built by the oracle (fp16 arithmetic done in software)
# The reference's only published build number: DEEP1M (1M x 96 f32, FAST_SMALL,
# fp16 storage, same R/L/C/STEPS) on one RTX 4090 -- another dataset and GPU.
CFG0_PUBLISHED = {"seconds": 2.768, "vectors_per_s": 1e6 / 2.768,
                  "source": "DANCE REPRODUCIBILITY.md:21-42, DEEP1M on RTX 4090 (FAST_SMALL)"}


def cfg0_inputs(n):
    from dance_b200 import workloads
    C0 = CFG0
    x = workloads.gaussian_mixture_f32(n, C0["dim"], C0["centroids"], C0["sigma"], seed=C0["seed"], device="cuda")
    q = workloads.gaussian_mixture_f32(C0["queries"], C0["dim"], C0["centroids"], C0["sigma"], seed=C0["seed"],
                                       device="cuda", stream_offset=1)
    return x, q


def cfg0_config(n, storage="f16"):
    C0 = CFG0
    if storage == "f32":
        return {"workload": "cfg0_f32_1M", "N": n, "dim": C0["dim"], "R": C0["R"], "L": C0["L"], "C": C0["C"],
                "STEPS": C0["STEPS"], "alpha": C0["alpha"], "iters": C0["iters"], "seed": C0["seed"],
                "storage": "fp32 (the reference's QUALITY profile: ENABLE_FLOAT16_BUILD=0)",
                "l2": "inputs larger than L2 (384 MB fp32 vector store + graph rows), no flush"}
    return {"workload": C0["name"], "N": n, "dim": C0["dim"], "R": C0["R"], "L": C0["L"], "C": C0["C"],
            "STEPS": C0["STEPS"], "alpha": C0["alpha"], "iters": C0["iters"], "seed": C0["seed"],
            "storage": "fp16 (the reference's FAST_SMALL profile: ENABLE_FLOAT16_BUILD=1)",
            "l2": "inputs larger than L2 (192 MB fp16 vector store + graph rows), no flush"}


def run_cfg0(args):
    """1M x 96 normalised Gaussian mixture, float input
    stored and searched in fp16 like the reference's FAST_SMALL profile
    (--cfg0-storage f16, the default) or in fp32 like its QUALITY profile."""
    import torch
    import dance_b200
    from dance_b200 import vamana, workloads
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    lib = dance_b200.load()
    C0 = CFG0
    n = args.n if args.n != WORKLOAD["N"] else C0["N"]
    R, L, C, S = C0["R"], C0["L"], C0["C"], C0["STEPS"]
    x, q = cfg0_inputs(n)
    f32 = getattr(args, "cfg0_storage", "f16") == "f32"
    store, stride = vamana.padded_store(x if f32 else x.half())
    ws = vamana.Workspace.create(n, R, L, C, S)
    prm = dance_b200.default_params()
    graph = torch.empty((n, R), dtype=torch.int32, device="cuda")
    degree = torch.empty((n,), dtype=torch.int32, device="cuda")
    dists = torch.empty((n, R), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def one_build():
        with torch.cuda.stream(stream):
            return vamana.build_resident(store, C0["dim"], stride, R, L, C, S, params=prm, workspace=ws,
                                         graph=graph, degree=degree, dists=dists, stream=stream)

    for _ in range(args.warmup):
        one_build()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    launches0 = lib.dance_kernel_launch_count()
    reports = []
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    medoid = 0
    for _ in range(args.steps):
        _, _, _, medoid = one_build()
        reports.append(dance_b200.last_build_report())
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = lib.dance_kernel_launch_count() - launches0
    clk = clocks.stop()
    elapsed = ev0.elapsed_time(ev1) * 1e-3
    peak, peak_kind = measured_peaks()
    alg = sum(search_algorithmic_bytes(r, n, stride, R, C0["iters"]) for r in reports)
    ksec = sum(r["search_kernel_seconds"] for r in reports)
    achieved = alg / ksec / 1e9
    line = {
        "metric": "vamana_build_vectors_per_s", "value": n * args.steps / elapsed, "unit": "vectors/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32" if f32 else "f16",
        "data": "synthetic (seeded GPU generator, BASELINE.json configs[0] recipe)",
        "config": cfg0_config(n, "f32" if f32 else "f16"),
        "roofline": {"kernel": "search_kernel", "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_launch": alg / (len(reports) * C0["iters"]),
                     "avg_launch_ms": ksec / (len(reports) * C0["iters"]) * 1e3},
        "gpu_launches": int(launches),
        "clocks": clk,
        "stage_seconds": {k: statistics.mean(r[k] for r in reports) for k in reports[0] if k.endswith("_seconds")},
        "counters_per_build": {k: reports[-1][k] for k in ("search_evals", "expansions", "replay_pairs",
                                                           "reverse_evals", "prune_pairs")},
        "published_reference": CFG0_PUBLISHED,
    }
    if not args.no_e2e:
        # the reference's float entry point; the storage is selected at run time
        saved_env = os.environ.get("DANCE_FLOAT16_BUILD")
        os.environ["DANCE_FLOAT16_BUILD"] = "0" if f32 else "1"
        hx = x.cpu().pin_memory()
        hg = torch.empty((n, R), dtype=torch.int32).pin_memory()
        hd = torch.empty((n,), dtype=torch.int32).pin_memory()
        fn = lib.gpu_vamana_vnew2_build_float

        def e2e_call():
            rc = fn(ctypes.c_void_p(hx.data_ptr()), n, C0["dim"], R, L, C, S, ctypes.c_void_p(hg.data_ptr()),
                    ctypes.c_void_p(hd.data_ptr()))
            dance_b200.check(rc, "gpu_vamana_vnew2_build_float")

        e2e_call()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_call()
        torch.cuda.synchronize()
        e2e_dt = time.perf_counter() - t0
        line["e2e"] = {"value": n * args.steps / e2e_dt, "unit": "vectors/s", "h2d_bytes_per_step": int(hx.numel() * 4),
                       "d2h_bytes_per_step": int(hg.numel() * 4 + hd.numel() * 4),
                       "api": f"gpu_vamana_vnew2_build_float (reference C ABI, DANCE_FLOAT16_BUILD="
                              f"{0 if f32 else 1}), pinned host buffers, wall clock", "warmup": 1,
                       "matches_resident_build": bool(torch.equal(hg.cuda(), graph))}
        if saved_env is None:
            os.environ.pop("DANCE_FLOAT16_BUILD", None)
        else:
            os.environ["DANCE_FLOAT16_BUILD"] = saved_env
    if not args.no_recall:
        gt, _ = workloads.brute_force_knn(x, q, 10)
        ids, _ = vamana.search_queries(store, C0["dim"], stride, graph, R, medoid, q if f32 else q.half(), 100, 10)
        line["recall_at_10"] = {"L_search": 100, "queries": int(q.shape[0]),
                                "ours": vamana.recall_at_k(ids.cpu().numpy(), gt.cpu().numpy()),
                                "ground_truth": "brute force on the float32 vectors"}
    if not args.no_cpu_baseline:
        sample = (x[:min(CFG0_CPU_SAMPLE, n)] if f32 else x[:min(CFG0_CPU_SAMPLE, n)].half()).cpu().numpy()
        threads = os.cpu_count() or 1
        rate, secs = oracle_sample_rate(sample, threads)
        line["cpu_baseline"] = {"value": rate, "unit": "vectors/s", "cores": threads, "kind": "port",
                                "sample": f"first {len(sample)} vectors of the workload ({sample.dtype}), full 4-round "
                                          f"build ({secs:.1f} s)"}
    deg = degree.cpu().numpy()
    line["graph"] = {"medoid": int(medoid), "avg_degree": float(deg.mean()), "max_degree": int(deg.max()),
                     "min_degree": int(deg.min()), "digest": graph_digest(graph, degree, n)}
    if args.ref_gpu:
        ref = reference_gpu_cfg0(x, q, store, stride, f32)
        line["reference_gpu"] = ref
        add_recall_delta(line, ref)
    emit(args, line)
    ws.close()
    return 0


def reference_gpu_cfg0(x, q, store, stride, f32=False):
    """The reference's vnew2 builder in its FAST_SMALL profile (fp16 storage) or,
    with f32, its QUALITY profile (fp32), compiled for sm_100a, on the same
    float vectors through its C ABI."""
    import numpy as np
    import torch
    from dance_b200 import vamana, workloads
    lib_path = ROOT / "oracle" / "_ref" / ("libref_vnew2_quality.so" if f32 else "libref_vnew2_fast_small.so")
    if not lib_path.exists():
        return {"unavailable": f"{lib_path.name} not built"}
    lib = ctypes.CDLL(str(lib_path))
    f = lib.gpu_vamana_vnew2_build_float
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] + [ctypes.c_uint32] * 6 + [ctypes.c_void_p] * 2
    lib.gpu_vamana_vnew2_get_last_medoid.restype = ctypes.c_uint32
    C0 = CFG0
    n = x.shape[0]
    R, L, C, S = C0["R"], C0["L"], C0["C"], C0["STEPS"]
    hx = np.ascontiguousarray(x.cpu().numpy())
    g = np.zeros((n, R), np.uint32)
    d = np.zeros(n, np.uint32)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = f(ctypes.c_void_p(hx.ctypes.data), n, C0["dim"], R, L, C, S, ctypes.c_void_p(g.ctypes.data),
           ctypes.c_void_p(d.ctypes.data))
    dt = time.perf_counter() - t0
    if rc != 0:
        return {"unavailable": f"reference build returned {rc}"}
    med = int(lib.gpu_vamana_vnew2_get_last_medoid())
    gt, _ = workloads.brute_force_knn(x, q, 10)
    gd = torch.from_numpy(g.view(np.int32)).cuda()
    ids, _ = vamana.search_queries(store, C0["dim"], stride, gd, R, med, q if f32 else q.half(), 100, 10)
    return {"e2e_vectors_per_s": n / dt, "seconds": dt,
            "recall_at_10": vamana.recall_at_k(ids.cpu().numpy(), gt.cpu().numpy()), "medoid": med,
            "avg_degree": float(d.mean()),
            "build": ("DANCE vnew2 QUALITY profile (fp32 storage" if f32 else
                      "DANCE vnew2 FAST_SMALL profile (fp16 storage") + ", VAMANA_ITERS=4), nvcc 12.9 sm_100a"}


def run_cfg0_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    import torch
    import oracle
    oracle.build()
    C0 = CFG0
    from dance_b200 import workloads
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    sample = workloads.gaussian_mixture_f32(CFG0_CPU_SAMPLE, C0["dim"], C0["centroids"], C0["sigma"],
                                            seed=C0["seed"], device=dev).half().cpu().numpy()
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        oracle.build_graph(sample, C0["R"], C0["L"], C0["C"], C0["STEPS"], nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.build_graph(sample, C0["R"], C0["L"], C0["C"], C0["STEPS"], nthreads=threads)
    dt = time.perf_counter() - t0
    value = CFG0_CPU_SAMPLE * args.steps / dt
    desc = (f"first {CFG0_CPU_SAMPLE} vectors of the {C0['name']} workload (fp16), full 4-round build per step, "
            f"{threads} OpenMP threads")
    line = {
        "impl": "reference", "metric": "vamana_build_vectors_per_s", "value": value, "unit": "vectors/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": cfg0_config(CFG0_CPU_SAMPLE),
        "cpu_baseline": {"value": value, "unit": "vectors/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "vectors/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(args, line)
    return 0


STITCHED = dict(name="cfg3_stitched_f32_1M", N=1_000_000, dim=96, centroids=1000, sigma=0.3, labels=100,
                r_small=32, l_small=100, r_stitched=64, C=96, steps=64, alpha=1.2, seed=42, queries=10_000)
STITCHED_CPU_SAMPLE = 20_000  # label memberships built by the oracle for cpu_baseline


def stitched_inputs(n):
    import numpy as np
    from dance_b200 import stitched, workloads
    x = workloads.gaussian_mixture_f32(n, STITCHED["dim"], STITCHED["centroids"], STITCHED["sigma"],
                                       seed=STITCHED["seed"], device="cuda")
    assign = workloads.zipf_partition_labels(n, STITCHED["labels"], seed=STITCHED["seed"])
    label_points = stitched.labels_from_assignment(assign, STITCHED["labels"])
    offs, pts = stitched.labels_csr(label_points)
    return x, assign, label_points, offs, pts


def stitched_recall(x, store, stride, assign, offs, pts, row_offsets, row_ids, medoids):
    """Recall@10 at L=100 of single-label queries searched from their label's
    medoid; every stitched edge stays inside its label, so the unfiltered
    beam search is the filtered one.  Ground truth: brute force inside the label."""
    import numpy as np
    import torch
    from dance_b200 import vamana, workloads
    nq = STITCHED["queries"]
    q = workloads.gaussian_mixture_f32(nq, STITCHED["dim"], STITCHED["centroids"], STITCHED["sigma"],
                                       seed=STITCHED["seed"], device="cuda", stream_offset=1)
    qlab = workloads.zipf_partition_labels(nq, STITCHED["labels"], seed=STITCHED["seed"] + 1)
    n = x.shape[0]
    deg = np.diff(row_offsets.astype(np.int64))
    R = int(deg.max())
    padded = np.full((n, R), 0xFFFFFFFF, np.uint32)
    mask = np.arange(R)[None, :] < deg[:, None]
    padded[mask] = row_ids
    g = torch.from_numpy(padded.view(np.int32)).cuda()
    hits = 0
    for l in range(len(offs) - 1):
        qi = np.nonzero(qlab == l)[0]
        if len(qi) == 0:
            continue
        members = torch.from_numpy(pts[int(offs[l]):int(offs[l + 1])].astype(np.int64)).cuda()
        ql = q[torch.from_numpy(qi).cuda()]
        gt_local, _ = workloads.brute_force_knn(x[members], ql, 10)
        gt = members[gt_local.long()].cpu().numpy()
        ids, _ = vamana.search_queries(store, STITCHED["dim"], stride, g, R, int(medoids[l]), ql, 100, 10)
        ids = ids.cpu().numpy()
        hits += sum(len(set(a.tolist()) & set(b.tolist())) for a, b in zip(ids, gt))
    return hits / (nq * 10)


def reference_gpu_stitched(hx, label_points):
    """The reference app's label loop (apps/utils/gpu_stitched_vamana_index.cpp:276-341):
    per label, host gather, gpu_vamana_vnew2_build_float of the reference's
    own library (DANCE src/gpu_vamana_vnew2.cu built for sm_100a, QUALITY
    profile), medoid; remap done here with numpy.  Times the per-label build
    calls and the host gathers like the app's timing keys."""
    import numpy as np
    lib_path = ROOT / "oracle" / "_ref" / "libref_vnew2_quality.so"
    if not lib_path.exists():
        return {"unavailable": f"{lib_path.name} not built"}
    lib = ctypes.CDLL(str(lib_path))
    f = lib.gpu_vamana_vnew2_build_float
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] + [ctypes.c_uint32] * 6 + [ctypes.c_void_p] * 2
    lib.gpu_vamana_vnew2_get_last_medoid.restype = ctypes.c_uint32
    rs, ls, C, st = STITCHED["r_small"], STITCHED["l_small"], STITCHED["C"], STITCHED["steps"]
    n, dim = hx.shape
    point_of, counts, flats = [], [], []
    medoids = []
    build_s = mat_s = 0.0
    t0 = time.perf_counter()
    for ids in label_points:
        ids = np.asarray(ids, dtype=np.int64)
        tm = time.perf_counter()
        local = np.ascontiguousarray(hx[ids])
        mat_s += time.perf_counter() - tm
        g = np.full((len(ids), rs), 0xFFFFFFFF, np.uint32)
        d = np.zeros(len(ids), np.uint32)
        tb = time.perf_counter()
        rc = f(ctypes.c_void_p(local.ctypes.data), len(ids), dim, rs, ls, C, st, ctypes.c_void_p(g.ctypes.data),
               ctypes.c_void_p(d.ctypes.data))
        build_s += time.perf_counter() - tb
        if rc != 0:
            return {"unavailable": f"reference build returned {rc}"}
        med = int(lib.gpu_vamana_vnew2_get_last_medoid())
        medoids.append(int(ids[med if med < len(ids) else 0]))
        # remap (single-label rows: no duplicates across labels), vectorised
        k = np.minimum(d, STITCHED["r_stitched"]).astype(np.int64)
        valid = ((np.arange(rs)[None, :] < k[:, None]) & (g < len(ids))
                 & (g != np.arange(len(ids), dtype=np.uint32)[:, None]))
        point_of.append(ids)
        counts.append(valid.sum(1))
        flats.append(ids[g[valid].astype(np.int64)])
    total = time.perf_counter() - t0
    point_of = np.concatenate(point_of)
    counts = np.concatenate(counts).astype(np.int64)
    flat = np.concatenate(flats).astype(np.uint32)
    src_start = np.concatenate([[0], np.cumsum(counts)[:-1]])
    order = np.argsort(point_of, kind="stable")
    offs = np.zeros(n + 1, np.uint64)
    per_point = np.zeros(n, np.int64)
    per_point[point_of] = counts
    np.cumsum(per_point, out=offs[1:])
    c_sorted = counts[order]
    gather = np.repeat(src_start[order] - np.concatenate([[0], np.cumsum(c_sorted)[:-1]]), c_sorted) + np.arange(
        int(c_sorted.sum()))
    return {"rows": (offs, flat[gather]), "medoids": medoids,
            "per_label_gpu_build_sum_seconds": build_s, "label_data_materialization_seconds": mat_s,
            "loop_seconds": total, "e2e_vectors_per_s": n / total,
            "build": "DANCE vnew2 QUALITY profile via gpu_vamana_vnew2_build_float, nvcc 12.9 sm_100a"}


def run_stitched_sharded(args):
    """configs[3] over the GPUs of one box (torchrun): dance_stitched_build_sharded
    (labels spread largest first over the ranks, local graphs to rank 0 over
    NCCL, rank 0 stitches).  Host vectors in, host CSR out, so the timed call
    is end to end; wall clock around each call, max over ranks."""
    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    import dance_b200
    from dance_b200 import stitched, vamana
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    dance_b200.load()
    n = args.n if args.n != WORKLOAD["N"] else STITCHED["N"]
    rs, ls, rst, C, steps = (STITCHED[k] for k in ("r_small", "l_small", "r_stitched", "C", "steps"))
    x, assign, label_points, offs, pts = stitched_inputs(n)
    hx = np.ascontiguousarray(x.cpu().numpy())
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.tensor(list(vamana.nccl_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    comm = vamana.Comm(rank, world, bytes(uid.cpu().tolist()), timeout_s=600.0)

    def one():
        return stitched.stitched_build_sharded(comm, hx, offs, pts, rs, ls, rst, C, steps)

    for _ in range(args.warmup):
        one()
    times, out = [], None
    for _ in range(args.steps):
        dist.barrier()
        t0 = time.perf_counter()
        out = one()
        times.append(time.perf_counter() - t0)
    mine = torch.tensor([sum(times)], dtype=torch.float64, device="cuda")
    dist.all_reduce(mine, op=dist.ReduceOp.MAX)
    elapsed = float(mine.item())
    if rank == 0:
        ro, ri, med, st = out
        import hashlib
        line = {
            "metric": "stitched_build_vectors_per_s", "value": n * args.steps / elapsed, "unit": "vectors/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded GPU generator, BASELINE.json configs[3] recipe)",
            "config": {"workload": STITCHED["name"], "N": n, "labels": len(offs) - 1, "Rsmall": rs, "Lsmall": ls,
                       "Rstitched": rst, "C": C, "steps": steps,
                       "parallelism": f"labels over {world} ranks (largest first to the least loaded), local "
                                      "graphs to rank 0 by NCCL send/recv",
                       "timed": "dance_stitched_build_sharded, host vectors in, host CSR out (wall clock)"},
            "e2e": {"value": n * args.steps / elapsed, "unit": "vectors/s", "h2d_bytes_per_step": int(hx.nbytes),
                    "d2h_bytes_per_step": int(ro.nbytes + 4 * len(ri) + med.nbytes)},
            "stage_seconds_rank0": {k: st[k] for k in ("label_build_wall_seconds", "label_graph_exchange_seconds",
                                                        "local_to_global_remap_seconds", "total_seconds")},
            "graph": {"edges": int(ro[-1]),
                      "digest": hashlib.sha256(ro.tobytes() + ri.tobytes()).hexdigest()[:16]},
        }
        emit(args, line)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_stitched(args):
    import numpy as np
    import torch
    import dance_b200
    from dance_b200 import stitched, vamana
    rank, world, local = dist_env()
    if world > 1:
        return run_stitched_sharded(args)
    torch.cuda.set_device(local)
    lib = dance_b200.load()
    n = args.n if args.n != WORKLOAD["N"] else STITCHED["N"]
    rs, ls, rst, C, steps = (STITCHED[k] for k in ("r_small", "l_small", "r_stitched", "C", "steps"))
    x, assign, label_points, offs, pts = stitched_inputs(n)
    store, stride = vamana.padded_store(x)
    dim = STITCHED["dim"]
    M = int(offs[-1])
    nl = len(offs) - 1
    prm = dance_b200.default_params()
    lgraph = torch.zeros(M * rs, dtype=torch.int32, device="cuda")
    ldeg = torch.zeros(M, dtype=torch.int32, device="cuda")
    med_local = np.zeros(nl, np.uint32)
    row_offsets = np.zeros(n + 1, np.uint64)
    row_ids = np.zeros(M * rs, np.uint32)
    P = stitched._ptr

    def one_step():
        st = dance_b200.DanceStitchedStats()
        rc = lib.dance_stitched_label_graphs(dance_b200.DANCE_F32, P(store), stride, n, dim, nl, P(offs), P(pts),
                                             None, rs, ls, C, steps, ctypes.byref(prm), 4, P(lgraph), P(ldeg),
                                             P(med_local), ctypes.byref(st))
        dance_b200.check(rc, "dance_stitched_label_graphs")
        st2 = dance_b200.DanceStitchedStats()
        rc = lib.dance_stitched_remap(n, nl, P(offs), P(pts), P(lgraph), P(ldeg), rs, rst, P(row_offsets),
                                      P(row_ids), M * rs, ctypes.byref(st2), None)
        dance_b200.check(rc, "dance_stitched_remap")
        return st, st2

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    launches0 = lib.dance_kernel_launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    stats = []
    ev0.record()
    for _ in range(args.steps):
        stats.append(one_step())
    ev1.record()
    torch.cuda.synchronize()
    launches = lib.dance_kernel_launch_count() - launches0
    clk = clocks.stop()
    elapsed = ev0.elapsed_time(ev1) * 1e-3
    medoids = [int(pts[int(offs[l]) + int(med_local[l])]) for l in range(nl)]
    peak, peak_kind = measured_peaks()
    rep = {"search_evals": sum(a.search_evals for a, _ in stats), "expansions": sum(a.search_expansions
                                                                                   for a, _ in stats)}
    alg = search_algorithmic_bytes(rep, M * len(stats), stride, rs, 4)
    ksec = sum(a.search_kernel_seconds for a, _ in stats)
    launches_per_step = 4 * nl
    achieved = alg / ksec / 1e9
    s0, s1 = stats[-1]
    line = {
        "metric": "stitched_build_vectors_per_s", "value": n * args.steps / elapsed, "unit": "vectors/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded GPU generator, BASELINE.json configs[3] recipe)",
        "config": {"workload": STITCHED["name"], "N": n, "dim": dim, "labels": nl, "Rsmall": rs, "Lsmall": ls,
                   "Rstitched": rst, "C": C, "steps": steps, "alpha": STITCHED["alpha"], "seed": STITCHED["seed"],
                   "label_sizes": {"min": s0.npts_per_label_min, "max": s0.npts_per_label_max},
                   "l2": "inputs larger than L2 (384 MB vectors + label-major copy), no flush",
                   "timed": "dance_stitched_label_graphs (device-resident store) + dance_stitched_remap"},
        "roofline": {"kernel": "search_kernel", "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_launch": alg / (len(stats) * launches_per_step),
                     "avg_launch_ms": ksec / (len(stats) * launches_per_step) * 1e3,
                     "note": "label builds overlap on 4 streams, so launch durations overlap"},
        "gpu_launches": int(launches),
        "clocks": clk,
        "stage_seconds": {"label_build_wall": s0.label_build_wall_seconds,
                          "per_label_build_sum": s0.per_label_gpu_build_sum_seconds,
                          "per_label_build_max": s0.per_label_gpu_build_max_seconds,
                          "gather": s0.label_data_materialization_seconds,
                          "remap": s1.local_to_global_remap_seconds},
        "graph": {"edges": int(s1.output_edges), "max_degree": int(s1.max_degree),
                  "remap_invalid_local_ids": int(s1.remap_invalid_local_ids),
                  "remap_self_loops": int(s1.remap_self_loops),
                  "remap_duplicate_edges": int(s1.remap_duplicate_edges)},
    }
    hx = x.cpu().numpy()
    if not args.no_e2e:
        hxp = torch.from_numpy(hx).pin_memory()
        e_off = np.zeros(n + 1, np.uint64)
        e_ids = np.zeros(M * rs, np.uint32)
        e_med = np.zeros(nl, np.uint32)

        def e2e_call():
            st = dance_b200.DanceStitchedStats()
            rc = lib.dance_stitched_build(dance_b200.DANCE_F32, ctypes.c_void_p(hxp.data_ptr()), n, dim, nl, P(offs),
                                          P(pts), rs, ls, rst, C, steps, ctypes.byref(prm), 4, P(e_off), P(e_ids),
                                          M * rs, P(e_med), ctypes.byref(st))
            dance_b200.check(rc, "dance_stitched_build")

        e2e_call()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_call()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        line["e2e"] = {"value": n * args.steps / dt, "unit": "vectors/s", "h2d_bytes_per_step": int(hx.nbytes + pts.nbytes
                                                                                                    + offs.nbytes),
                       "d2h_bytes_per_step": int(e_off.nbytes + 4 * int(e_off[-1]) + e_med.nbytes),
                       "api": "dance_stitched_build (host in, host CSR out), pinned vectors, wall clock",
                       "matches_resident_path": bool(np.array_equal(e_off, row_offsets)
                                                     and np.array_equal(e_ids[:int(e_off[-1])],
                                                                        row_ids[:int(row_offsets[-1])])
                                                     and e_med.tolist() == medoids)}
    E = int(row_offsets[-1])
    if not args.no_recall:
        line["recall_at_10"] = {"L_search": 100, "queries": STITCHED["queries"],
                                "ours": stitched_recall(x, store, stride, assign, offs, pts, row_offsets,
                                                        row_ids[:E], medoids)}
    if not args.no_cpu_baseline:
        import oracle
        # smallest labels first until the sample holds STITCHED_CPU_SAMPLE memberships
        sizes = np.diff(offs.astype(np.int64))
        chosen, tot = [], 0
        for l in np.argsort(sizes, kind="stable"):
            if tot >= STITCHED_CPU_SAMPLE:
                break
            chosen.append(int(l))
            tot += int(sizes[l])
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        oracle.stitched(hx, [label_points[l] for l in chosen], rs, ls, rst, C, steps)
        secs = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": tot / secs, "unit": "vectors/s", "cores": threads, "kind": "port",
                                "sample": f"the {len(chosen)} smallest labels ({tot} points), per-label builds and "
                                          f"remap ({secs:.1f} s)"}
    import hashlib
    line["graph"]["digest"] = hashlib.sha256(row_offsets.tobytes() + row_ids[:E].tobytes()).hexdigest()[:16]
    if args.ref_gpu:
        ref = reference_gpu_stitched(hx, label_points)
        if "rows" in ref:
            roffs, rids = ref.pop("rows")
            ref["recall_at_10"] = stitched_recall(x, store, stride, assign, offs, pts, roffs, rids, ref["medoids"])
            ref["graph_equals_ours"] = bool(np.array_equal(roffs, row_offsets) and np.array_equal(rids,
                                                                                               row_ids[:E]))
            ref["medoids_equal_ours"] = ref.pop("medoids") == medoids
        line["reference_gpu"] = ref
        add_recall_delta(line, ref)
    emit(args, line)
    return 0


def run_stitched_reference(args, n):
    """--impl reference for the stitched workload: the oracle port of the
    app's label loop on the host cores, a bounded sample (smallest labels
    first) per step."""
    import numpy as np
    import oracle
    from dance_b200 import stitched, workloads
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    x = workloads.gaussian_mixture_f32(n, STITCHED["dim"], STITCHED["centroids"], STITCHED["sigma"],
                                       seed=STITCHED["seed"], device="cpu").numpy()
    assign = workloads.zipf_partition_labels(n, STITCHED["labels"], seed=STITCHED["seed"])
    label_points = stitched.labels_from_assignment(assign, STITCHED["labels"])
    sizes = np.array([len(p) for p in label_points])
    chosen, tot = [], 0
    for l in np.argsort(sizes, kind="stable"):
        if tot >= STITCHED_CPU_SAMPLE:
            break
        chosen.append(int(l))
        tot += int(sizes[l])
    sample = [label_points[l] for l in chosen]
    args_t = (STITCHED["r_small"], STITCHED["l_small"], STITCHED["r_stitched"], STITCHED["C"], STITCHED["steps"])
    for _ in range(args.warmup):
        oracle.stitched(x, sample[:1], *args_t)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.stitched(x, sample, *args_t)
    dt = time.perf_counter() - t0
    v = tot * args.steps / dt
    threads = os.cpu_count() or 1
    print(json.dumps({
        "impl": "reference", "metric": "stitched_build_vectors_per_s", "value": v, "unit": "vectors/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (BASELINE.json configs[3] recipe)",
        "config": {"workload": STITCHED["name"], "N": n, "labels": STITCHED["labels"]},
        "cpu_baseline": {"value": v, "unit": "vectors/s", "cores": threads, "kind": "port",
                         "sample": f"the {len(chosen)} smallest labels ({tot} points) per step"},
        "e2e": {"value": v, "unit": "vectors/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
    return 0


# ------------------------------------------------------------------ filtered
FILTERED = dict(name="cfg2_filtered_f32_1M", N=1_000_000, dim=96, centroids=1000, sigma=0.3, vocab=1000, min_labels=1,
                max_labels=5, R=64, L=100, FL=100, C=128, STEPS=64, alpha=1.2, seed=42, queries=10_000)
FILTERED_CPU_SAMPLE = 6_000  # points built by the oracle for cpu_baseline


def filtered_label_starts(x, offs, labs, vocab):
    """Label start points and the global start as DiskANN sets them before
    the GPU hook (integration patch lines 20238-20267), computed on the GPU
    by the library: per label the least-chosen of 25 hashed member draws
    (dance_select_label_starts), and the point nearest to the centroid
    (dance_calculate_entry_point)."""
    from dance_b200 import filtered as FL, vamana
    n = x.shape[0]
    loff, lpts = FL.label_points_csr(offs, labs, vocab)
    starts = FL.select_label_starts(loff, lpts, n, 25, FILTERED["seed"])
    store, stride = vamana.padded_store(x)
    g = FL.calculate_entry_point(store, x.shape[1], stride)
    return starts, g


def filtered_recall(x, store, stride, offs, labs, graph, starts, R, queries, qlabels, L_search=100, K=10):
    """Recall@10 of label-filtered queries searched from their label's start;
    ground truth is brute force among the points carrying the label."""
    import numpy as np
    import torch
    from dance_b200 import vamana, workloads
    n = x.shape[0]
    rows = np.repeat(np.arange(n), np.diff(offs.astype(np.int64)))
    order = np.argsort(labs, kind="stable")
    lab_sorted = labs[order]
    d_off = torch.from_numpy(offs.view(np.int32)).cuda()
    d_lab = torch.from_numpy(labs.view(np.int32)).cuda()
    qs = torch.from_numpy(starts[qlabels].view(np.int32)).cuda()
    ql = torch.from_numpy(qlabels.astype(np.uint32).view(np.int32)).cuda()
    # queries in the store's element type (the fp16 store searches fp16 queries)
    ids, _ = vamana.search_queries_filtered(store, x.shape[1], stride, graph, R, d_off, d_lab, ql, qs,
                                            queries.to(store.dtype), L_search, K)
    ids = ids.cpu().numpy().view(np.uint32)
    hits = total = 0
    for l in np.unique(qlabels):
        qi = np.nonzero(qlabels == l)[0]
        a, b = np.searchsorted(lab_sorted, [l, l + 1])
        members = torch.from_numpy(rows[order[a:b]].astype(np.int64)).cuda()
        k = min(K, len(members))
        gt_local, _ = workloads.brute_force_knn(x[members], queries[torch.from_numpy(qi).cuda()], k)
        gt = members[gt_local.long()].cpu().numpy()
        for j, q in enumerate(qi):
            hits += len(set(ids[q, :k].tolist()) & set(gt[j].tolist()))
            total += k
    return hits / total


def filtered_inputs(n):
    import numpy as np
    from dance_b200 import workloads
    F = FILTERED
    x = workloads.gaussian_mixture_f32(n, F["dim"], F["centroids"], F["sigma"], seed=F["seed"], device="cuda")
    offs, labs = workloads.zipf_multilabels(n, F["vocab"], F["min_labels"], F["max_labels"], seed=F["seed"])
    starts, gstart = filtered_label_starts(x, offs, labs, F["vocab"])
    q = workloads.gaussian_mixture_f32(F["queries"], F["dim"], F["centroids"], F["sigma"], seed=F["seed"],
                                       device="cuda", stream_offset=1)
    rng = np.random.default_rng(F["seed"] + 1)
    pz = 1.0 / np.arange(1, F["vocab"] + 1)
    qlabels = rng.choice(F["vocab"], size=F["queries"], p=pz / pz.sum()).astype(np.int64)
    return x, offs, labs, starts, gstart, q, qlabels


def run_filtered(args):
    import numpy as np
    import torch
    import dance_b200
    from dance_b200 import filtered, vamana
    F = FILTERED
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    lib = dance_b200.load()
    n = args.n if args.n != WORKLOAD["N"] else F["N"]
    x, offs, labs, starts, gstart, q, qlabels = filtered_inputs(n)
    store, stride = vamana.padded_store(x.half())
    R, L, FL, C, S, alpha = F["R"], F["L"], F["FL"], F["C"], F["STEPS"], F["alpha"]
    graph = torch.empty((n, R), dtype=torch.int32, device="cuda")
    degree = torch.empty(n, dtype=torch.int32, device="cuda")

    def one_build():
        return filtered.build_resident(store, F["dim"], stride, R, L, FL, min(C, 128), S, alpha, offs, labs, starts,
                                       F["vocab"], 0xFFFFFFFF, gstart, graph=graph, degree=degree)

    for _ in range(args.warmup):
        one_build()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    launches0 = lib.dance_kernel_launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    stats = []
    ev0.record()
    for _ in range(args.steps):
        stats.append(one_build()[2])
    ev1.record()
    torch.cuda.synchronize()
    launches = lib.dance_kernel_launch_count() - launches0
    clk = clocks.stop()
    elapsed = ev0.elapsed_time(ev1) * 1e-3
    peak, peak_kind = measured_peaks()
    st = stats[-1]
    # roofline of the union-label search (the largest stage): one gathered
    # fp16 row per distance evaluation over its kernel time (3 launches per build)
    alg = st["unfiltered_search_distance_count"] * stride
    ksec = st["ordinary_search_seconds"]
    achieved = alg / ksec / 1e9 if ksec else 0.0
    stage = {k: st[k] for k in ("filtered_search_seconds", "ordinary_search_seconds", "merge_seconds",
                                "forward_prune_seconds", "csr_reverse_seconds", "reverse_prune_seconds")}
    line = {
        "metric": "filtered_build_vectors_per_s", "value": n * args.steps / elapsed, "unit": "vectors/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded generators, BASELINE.json configs[2] recipe)",
        "config": {"workload": F["name"], "N": n, "dim": F["dim"], "labels": F["vocab"],
                   "label_memberships": int(offs[-1]), "R": R, "L": L, "FilteredL": FL, "C": C, "STEPS": S,
                   "alpha": alpha, "rounds": 3, "pools": [min(FL, 32), min(FL, 32, 8), min(64, FL)],
                   "l2": "inputs larger than L2 (192 MB fp16 vectors + graphs), no flush",
                   "label_starts": "DiskANN's rule on the GPU: least-chosen of 25 hashed member draws per label; global start = point nearest the centroid"},
        "roofline": {"kernel": "fl_union_search_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_launch": alg / 3, "avg_launch_ms": ksec / 3 * 1e3},
        "gpu_launches": int(launches),
        "clocks": clk,
        "stage_seconds": stage,
        "counters_per_build": {"task_search_evals": st["filtered_search_distance_count"],
                               "union_search_evals": st["unfiltered_search_distance_count"],
                               "reverse_edges": st["reverse_edges"], "reverse_touched_rows": st["reverse_touched_rows"]},
    }
    hx = x.cpu().numpy()
    if not args.no_e2e:
        hxp = torch.from_numpy(hx).pin_memory()
        hg = np.zeros((n, R), np.uint32)
        hd = np.zeros(n, np.uint32)
        P = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731

        def e2e_call():
            rc = lib.gpu_vamana_filtered_build_float(ctypes.c_void_p(hxp.data_ptr()), n, F["dim"], R, L, FL, C, S,
                                                     alpha, P(offs), P(labs), len(labs), P(starts), F["vocab"],
                                                     0xFFFFFFFF, gstart, None, None, 0, P(hg), P(hd))
            dance_b200.check(rc, "gpu_vamana_filtered_build_float")

        e2e_call()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_call()
        dt = time.perf_counter() - t0
        line["e2e"] = {"value": n * args.steps / dt, "unit": "vectors/s",
                       "h2d_bytes_per_step": int(hx.nbytes + offs.nbytes + labs.nbytes + starts.nbytes),
                       "d2h_bytes_per_step": int(hg.nbytes + hd.nbytes),
                       "api": "gpu_vamana_filtered_build_float (reference C ABI), pinned vectors, wall clock",
                       "matches_resident_build": bool(np.array_equal(hg, graph.cpu().numpy().view(np.uint32)))}
    if not args.no_recall:
        line["recall_at_10"] = {"L_search": 100, "queries": F["queries"], "search": "label-filtered, from the label start",
                                "ours": filtered_recall(x, store, stride, offs, labs, graph, starts, R, q, qlabels)}
    deg = degree.cpu().numpy()
    line["graph"] = {"avg_degree": float(deg.mean()), "max_degree": int(deg.max()), "min_degree": int(deg.min()),
                     "digest": graph_digest(graph, degree, n)}
    if not args.no_cpu_baseline:
        import oracle
        m = min(FILTERED_CPU_SAMPLE, n)
        so, sl = offs[:m + 1].copy(), labs[:int(offs[m])].copy()
        ss = np.full(F["vocab"], 0xFFFFFFFF, np.uint32)
        for pnt in range(m - 1, -1, -1):
            ss[sl[so[pnt]:so[pnt + 1]]] = pnt
        lab = oracle.FilteredLabels(so, sl, ss, F["vocab"], 0xFFFFFFFF, 0)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        oracle.filtered_build(oracle.float_to_half(hx[:m]), lab, R, L, FL, C, S, alpha)
        secs = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": m / secs, "unit": "vectors/s", "cores": threads, "kind": "port",
                                "sample": f"first {m} points with their labels, 3-round canonical build ({secs:.1f} s)"}
    if args.ref_gpu:
        ref = reference_gpu_filtered(hx, offs, labs, starts, gstart, x, store, stride, q, qlabels, graph)
        line["reference_gpu"] = ref
        add_recall_delta(line, ref)
    emit(args, line)
    return 0


def reference_gpu_filtered(hx, offs, labs, starts, gstart, x, store, stride, q, qlabels, our_graph):
    """The reference's own filtered builder (DANCE src/gpu_vamana_filtered.cu
    built for sm_100a) through its C ABI on the same inputs."""
    import numpy as np
    import torch
    lib_path = ROOT / "oracle" / "_ref" / "libref_filtered.so"
    if not lib_path.exists():
        return {"unavailable": f"{lib_path.name} not built"}
    F = FILTERED
    lib = ctypes.CDLL(str(lib_path))
    fn = lib.gpu_vamana_filtered_build_float
    fn.restype = ctypes.c_int
    U, Pv = ctypes.c_uint32, ctypes.c_void_p
    fn.argtypes = [Pv, U, U, U, U, U, U, U, ctypes.c_float, Pv, Pv, U, Pv, U, U, U, Pv, Pv, U, Pv, Pv]
    n = hx.shape[0]
    R = F["R"]
    g = np.zeros((n, R), np.uint32)
    d = np.zeros(n, np.uint32)
    P = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = fn(P(hx), n, F["dim"], R, F["L"], F["FL"], F["C"], F["STEPS"], F["alpha"], P(offs), P(labs), len(labs),
            P(starts), F["vocab"], 0xFFFFFFFF, gstart, None, None, 0, P(g), P(d))
    dt = time.perf_counter() - t0
    if rc != 0:
        return {"unavailable": f"reference build returned {rc}"}
    gd = torch.from_numpy(g.view(np.int32)).cuda()
    ours = our_graph.cpu().numpy().view(np.uint32)
    same = float(np.mean([np.array_equal(np.sort(ours[i]), np.sort(g[i])) for i in range(0, n, 97)]))
    return {"e2e_vectors_per_s": n / dt, "seconds": dt,
            "recall_at_10": filtered_recall(x, store, stride, offs, labs, gd, starts, R, q, qlabels),
            "avg_degree": float(d.mean()), "rows_equal_to_ours_sampled": same,
            "build": "DANCE GPU-FilteredVamana canonical path, nvcc 12.9 sm_100a"}


def run_filtered_reference(args):
    """--impl reference for the filtered workload: the oracle port of the
    canonical filtered build on the host cores, a bounded sample per step."""
    import numpy as np
    import oracle
    from dance_b200 import workloads
    F = FILTERED
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    m = FILTERED_CPU_SAMPLE
    x = workloads.gaussian_mixture_f32(m, F["dim"], F["centroids"], F["sigma"], seed=F["seed"], device="cpu").numpy()
    offs, labs = workloads.zipf_multilabels(m, F["vocab"], F["min_labels"], F["max_labels"], seed=F["seed"])
    ss = np.full(F["vocab"], 0xFFFFFFFF, np.uint32)
    for pnt in range(m - 1, -1, -1):
        ss[labs[offs[pnt]:offs[pnt + 1]]] = pnt
    lab = oracle.FilteredLabels(offs, labs, ss, F["vocab"], 0xFFFFFFFF, 0)
    xs = oracle.float_to_half(x)
    args_b = (F["R"], F["L"], F["FL"], F["C"], F["STEPS"], F["alpha"])
    for _ in range(args.warmup):
        oracle.filtered_build(xs[:500], oracle.FilteredLabels(offs[:501], labs[:int(offs[500])], ss, F["vocab"]),
                              *args_b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.filtered_build(xs, lab, *args_b)
    dt = time.perf_counter() - t0
    v = m * args.steps / dt
    threads = os.cpu_count() or 1
    print(json.dumps({
        "impl": "reference", "metric": "filtered_build_vectors_per_s", "value": v, "unit": "vectors/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (BASELINE.json configs[2] recipe)",
        "config": {"workload": F["name"], "N": m, "labels": F["vocab"]},
        "cpu_baseline": {"value": v, "unit": "vectors/s", "cores": threads, "kind": "port",
                         "sample": f"{m} points with their labels per step, 3-round canonical build"},
        "e2e": {"value": v, "unit": "vectors/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
    return 0


def read_graph_padded(path, R):
    """A DiskANN graph file as (N x R uint32 rows padded with 0xFFFFFFFF,
    degrees, start)."""
    import struct
    import numpy as np
    blob = np.fromfile(path, dtype=np.uint8)
    _, width, start, _ = struct.unpack_from("<QIIQ", blob.tobytes()[:24])
    words = blob[24:].view(np.uint32)
    pos = []
    i, nw = 0, len(words)
    while i < nw:
        pos.append(i)
        i += 1 + int(words[i])
    pos = np.array(pos, np.int64)
    deg = words[pos].astype(np.int64)
    g = np.full((len(pos), R), 0xFFFFFFFF, np.uint32)
    cols = np.arange(R)[None, :]
    mask = cols < np.minimum(deg, R)[:, None]
    g[mask] = words[(pos[:, None] + 1 + cols)[mask]]
    return g, deg.astype(np.uint32), int(start)


def run_disk_sharded(args):
    """The sharded disk-index pipeline (DiskANN build_merged_vamana_index with
    the DANCE GPU shard build and GPU merge) on the configs[1] vectors: one
    step is partition + shard builds + merge from a .u8bin file to the merged
    DiskANN graph, wall clock; value = N / step seconds."""
    import tempfile
    import numpy as np
    import torch
    from dance_b200 import formats, shards, vamana, workloads
    n = args.n
    R, L = WORKLOAD["R"], WORKLOAD["L"]
    x = make_workload("cuda", n)
    d = tempfile.mkdtemp(prefix="disk_sharded_")
    base = os.path.join(d, "base.u8bin")
    hx = x.cpu().numpy()
    with open(base, "wb") as f:
        np.array([n, hx.shape[1]], np.uint32).tofile(f)
        hx.tofile(f)
    runs = []
    for it in range(args.warmup + args.steps):
        prefix = os.path.join(d, f"idx{it}")
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = shards.build_merged_vamana_index(base, "uint8", R, L, args.ram_budget_gb, prefix + "_mem.index",
                                               prefix + "_medoids.bin", prefix + "_centroids.bin",
                                               sampling_rate=0.01, k_base=2, seed=WORKLOAD["seed"])
        torch.cuda.synchronize()
        res["wall_seconds"] = time.perf_counter() - t0
        if it >= args.warmup:
            runs.append(res)
    last = prefix + "_mem.index"
    secs = [r["wall_seconds"] for r in runs]
    g, deg, start = read_graph_padded(last, R)
    audit = {k: int(v) for k, v in formats.audit_graph(g, deg, R, start).items()}
    q = make_queries("cuda")
    store, stride = vamana.padded_store(x)
    gt, _ = workloads.brute_force_knn(x, q, 10)
    found, _ = vamana.search_queries(store, x.shape[1], stride, torch.from_numpy(g.view(np.int32)).cuda(), R, start,
                                     q, 100, 10)
    recall = vamana.recall_at_k(found.cpu().numpy(), gt.cpu().numpy())
    mean = float(np.mean(secs))
    r0 = runs[-1]
    line = {"metric": "vamana_disk_sharded_build_vectors_per_s", "value": n / mean, "unit": "vectors/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded GPU generator, BASELINE.json configs[1] recipe), written to a .u8bin file",
            "config": {"workload": "cfg1_disk_sharded", "N": n, "dim": hx.shape[1], "R": R, "L": L,
                       "ram_budget_gb": args.ram_budget_gb, "sampling_rate": 0.01, "k_base": 2,
                       "shard_params": dict(zip(("R_shard", "C", "STEPS"), shards.shard_build_params(R, L))),
                       "timing": "wall clock of build_merged_vamana_index (file in, DiskANN files out)"},
            "num_parts": r0["num_parts"], "shard_sizes": r0["shard_sizes"],
            "stage_seconds": {k: r0[k] for k in ("partition_seconds", "shard_build_seconds", "merge_seconds",
                                                 "total_seconds")},
            "shard_seconds_summed": {k: sum(sh[k] for sh in r0["shards"])
                                     for k in ("gather_seconds", "build_seconds", "write_seconds")},
            "graph": {"start": start, "avg_degree": float(deg.mean()), "max_degree": int(deg.max()),
                      "audit": audit},
            "recall_at_10": {"L_search": 100, "queries": int(q.shape[0]), "ours": recall}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.workload == "cfg1_disk_sharded":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "workload": "cfg1_disk_sharded",
                              "unavailable": "the reference's sharded disk pipeline runs inside DiskANN, which the "
                                             "reference repository does not contain"}), flush=True)
            return 0
        return run_disk_sharded(args)
    if args.workload == "cfg0_f32":
        if args.impl == "reference":
            return run_cfg0_reference(args)
        return run_cfg0(args)
    if args.workload == "cfg2_filtered":
        if args.impl == "reference":
            return run_filtered_reference(args)
        return run_filtered(args)
    if args.workload == "cfg3_stitched":
        if args.impl == "reference":
            return run_stitched_reference(args, args.n if args.n != WORKLOAD["N"] else STITCHED["N"])
        return run_stitched(args)
    if args.workload == "cfg4_f32_100M":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "workload": "cfg4_f32_100M",
                              "unavailable": "the reference has no multi-GPU build and its one-GPU build does not "
                                             "hold 100M float32 vectors with N x C work rows"}), flush=True)
            return 0
        if dist_env()[1] < 2:
            raise SystemExit("cfg4_f32_100M runs sharded: launch with torchrun --nproc-per-node N (N >= 2)")
        return run_sharded(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
