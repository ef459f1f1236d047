"""dance_b200 -- B200-native Vamana graph builder behind DANCE's C ABI.

The product is the shared library ``libdance_b200.so`` (sm_100a CUDA kernels
plus the C ABI of ``include/gpu_vamana_builder.h`` and ``include/dance_b200.h``).
This package loads it with ctypes and offers a thin Python mirror of the
reference interface.  There is no CPU fallback: importing ``lib`` raises if the
library has not been built.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

__all__ = ["lib", "load", "LIB_PATH", "DanceError", "DANCE_U8", "DANCE_F16", "DANCE_F32",
           "DanceVamanaParams", "GPUVamanaStats"]

LIB_PATH = Path(__file__).resolve().parent / "libdance_b200.so"

DANCE_U8, DANCE_F16, DANCE_F32 = 0, 1, 2


class DanceError(RuntimeError):
    """A libdance_b200 call returned a non-zero status."""


class DanceVamanaParams(ctypes.Structure):
    """Mirror of ``DanceVamanaParams`` in include/dance_b200.h."""
    _fields_ = [
        ("iters", ctypes.c_uint32),
        ("alpha", ctypes.c_float),
        ("init_random_seeds", ctypes.c_uint32),
        ("final_min_degree", ctypes.c_uint32),
        ("medoid_candidates", ctypes.c_uint32),
        ("medoid_samples", ctypes.c_uint32),
        ("coarse_warmup_iters", ctypes.c_uint32),
        ("warmup_expand_steps", ctypes.c_uint32),
        ("reverse_heavy_cap", ctypes.c_uint32),
        ("reverse_heavy_threshold", ctypes.c_uint32),
        ("reverse_heavy_sample", ctypes.c_uint32),
        ("visited_log2", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32 * 8),
    ]


class GPUVamanaStats(ctypes.Structure):
    """Mirror of ``GPUVamanaStats`` (reference include/gpu_vamana_builder.h:11-28)."""
    _fields_ = [
        ("medoid_seconds", ctypes.c_double),
        ("h2d_seconds", ctypes.c_double),
        ("search_online_insert_seconds", ctypes.c_double),
        ("reverse_seconds", ctypes.c_double),
        ("final_prune_seconds", ctypes.c_double),
        ("d2h_seconds", ctypes.c_double),
        ("gpu_build_seconds", ctypes.c_double),
        ("distance_computations", ctypes.c_uint64),
        ("online_insert_attempts", ctypes.c_uint64),
        ("online_insert_mutations", ctypes.c_uint64),
        ("reverse_candidate_overflows", ctypes.c_uint64),
        ("reverse_proposals", ctypes.c_uint64),
        ("reverse_touched_rows", ctypes.c_uint64),
        ("reverse_csr_seconds", ctypes.c_double),
        ("selective_active_nodes", ctypes.c_uint32),
    ]


class DanceBuildReport(ctypes.Structure):
    """Mirror of ``DanceBuildReport`` in include/dance_b200.h."""
    _fields_ = [(n, ctypes.c_double) for n in (
        "medoid_seconds", "search_seconds", "search_kernel_seconds", "replay_seconds", "reverse_seconds",
        "prune_seconds", "total_seconds")] + [(n, ctypes.c_uint64) for n in (
            "search_evals", "expansions", "replay_pairs", "reverse_evals", "prune_pairs")] + [
        ("reserved", ctypes.c_uint64 * 3)]


class DanceShardedReport(ctypes.Structure):
    """Mirror of ``DanceShardedReport`` in include/dance_b200.h."""
    _fields_ = [(n, ctypes.c_double) for n in (
        "medoid_init_seconds", "search_seconds", "replay_seconds", "edge_exchange_seconds", "reverse_seconds",
        "prune_seconds", "graph_exchange_seconds", "total_seconds")] + [(n, ctypes.c_uint64) for n in (
            "edge_bytes_sent", "edge_bytes_received", "graph_bytes_received", "rounds")] + [
        ("reserved", ctypes.c_uint64 * 4)]


class GPUFilteredVamanaStats(ctypes.Structure):
    """Mirror of ``GPUFilteredVamanaStats`` in include/gpu_vamana_filtered.h."""
    _fields_ = ([(n, ctypes.c_double) for n in (
        "gpu_build_seconds", "label_h2d_seconds", "graph_build_seconds", "diagnostics_seconds", "d2h_seconds",
        "peak_gpu_mem_gb", "backbone_seconds", "task_generation_seconds", "filtered_search_seconds",
        "ordinary_search_seconds", "merge_seconds", "forward_prune_seconds", "csr_reverse_seconds",
        "reverse_prune_seconds", "compaction_seconds")]
        + [(n, ctypes.c_uint64) for n in (
            "filtered_search_distance_count", "unfiltered_search_distance_count", "label_check_count",
            "label_reject_count", "filtered_candidate_count", "unfiltered_candidate_count", "merged_candidate_count",
            "active_rows", "original_neighbor_count", "filtered_seed_count", "filtered_visited_count",
            "filtered_visited_reserved_count", "filtered_top_reserved_count", "bridge_reserved_count",
            "unfiltered_reserved_count", "filtered_reserved_count", "label_occlusion_blocked_count",
            "geometry_occluded_count", "candidate_rejected_by_label_count", "refill_count",
            "filtered_prune_reject_count", "universal_label_pass_count", "final_prune_rows", "reverse_edges",
            "reverse_touched_rows", "filtered_reverse_edges", "filtered_reverse_touched_rows",
            "filtered_reverse_candidates_kept", "filtered_reverse_pruned_rows")]
        + [(n, ctypes.c_double) for n in (
            "avg_common_label_out_degree", "common_label_degree_before_avg", "common_label_degree_after_avg",
            "active_rows_frac")]
        + [(n, ctypes.c_uint32) for n in (
            "low_common_label_degree_count", "low_common_before", "low_common_after", "out_degree_min",
            "out_degree_max")]
        + [("out_degree_avg", ctypes.c_double)]
        + [(n, ctypes.c_uint32) for n in (
            "common_label_degree_min", "common_label_degree_max", "invalid_neighbor_count", "self_loop_count")]
        + [("prune_output_degree_avg", ctypes.c_double)]
        + [(n, ctypes.c_uint32) for n in ("filtered_seed_source", "semantic_stage", "semantic_complete")])

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


class DanceStitchedStats(ctypes.Structure):
    """Mirror of ``DanceStitchedStats`` in include/dance_b200.h."""
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "num_labels", "npts_per_label_min", "npts_per_label_max", "max_degree")] + [
        ("npts_per_label_mean", ctypes.c_double)] + [(n, ctypes.c_uint64) for n in (
            "total_label_memberships", "processed_label_memberships", "remap_invalid_local_ids", "remap_self_loops",
            "remap_duplicate_edges", "output_edges")] + [(n, ctypes.c_double) for n in (
                "label_data_materialization_seconds", "per_label_gpu_build_sum_seconds",
                "per_label_gpu_build_max_seconds", "label_build_wall_seconds", "local_to_global_remap_seconds",
                "total_seconds", "peak_gpu_mem_gb", "search_kernel_seconds")] + [
        ("search_evals", ctypes.c_uint64), ("search_expansions", ctypes.c_uint64),
        ("streams", ctypes.c_uint32), ("reserved0", ctypes.c_uint32),
        ("label_graph_exchange_seconds", ctypes.c_double), ("reserved", ctypes.c_uint64 * 3)]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_ if not k.startswith("reserved")}


_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_I = ctypes.c_int
_F = ctypes.c_float
_PU32 = ctypes.POINTER(ctypes.c_uint32)
_PU64 = ctypes.POINTER(ctypes.c_uint64)

# name -> (restype, argtypes); every entry point declared in include/*.h.
SIGNATURES = {
    # reference C ABI (include/gpu_vamana_builder.h)
    "gpu_vamana_build": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P]),
    "gpu_vamana_build_float": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P]),
    "gpu_vamana_vnew2_build": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P]),
    "gpu_vamana_vnew2_build_float": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P]),
    "gpu_vamana_vnew2_build_device": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P]),
    "gpu_vamana_vnew2_build_device_float": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P]),
    "gpu_vamana_get_last_medoid": (_U32, []),
    "gpu_vamana_get_last_stats": (None, [_P]),
    "gpu_vamana_vnew2_get_last_medoid": (_U32, []),
    "gpu_vamana_vnew2_get_last_stats": (None, [_P]),
    # reference filtered C ABI (include/gpu_vamana_filtered.h)
    "gpu_vamana_filtered_build_uint8": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _F, _P, _P, _U32, _P,
                                             _U32, _U32, _U32, _P, _P, _U32, _P, _P]),
    "gpu_vamana_filtered_build_float": (_I, [_P, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _F, _P, _P, _U32, _P,
                                             _U32, _U32, _U32, _P, _P, _U32, _P, _P]),
    "gpu_vamana_filtered_get_last_stats": (None, [_P]),
    # additive C ABI (include/dance_b200.h)
    "dance_filtered_build_resident": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _F, _P, _P, _P,
                                           _U32, _U32, _U32, _P, _P, _U32, _P, _P, _P, _P]),
    "dance_filtered_random_graph": (_I, [_U32, _U32, _U32, _U32, _P, _P, _P]),
    "dance_filtered_stage_round": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _F, _P, _P, _P,
                                        _U32, _U32, _U32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                        _P]),
    "dance_vamana_default_params": (None, [_P]),
    "dance_last_error": (ctypes.c_char_p, []),
    "dance_kernel_launch_count": (_U64, []),
    "dance_last_build_report": (_I, [_P]),
    "dance_last_sharded_report": (_I, [_P]),
    "dance_workspace_create": (_I, [_U32, _U32, _U32, _U32, _U32, _P]),
    "dance_workspace_destroy": (None, [_P]),
    "dance_vamana_build_resident": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P,
                                         _PU32, _P]),
    "dance_stage_medoid": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _P, _P, _P, _P]),
    "dance_stage_init": (_I, [_I, _P, _U64, _U32, _U32, _U32, _P, _P, _P, _P]),
    "dance_stage_search": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P,
                                _P, _U32, _P]),
    "dance_stage_replay": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _F, _P, _P, _P, _P, _P, _P, _U32, _P, _P, _P,
                                _P]),
    "dance_stage_reverse_merge": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P, _PU64, _P]),
    "dance_stage_prune": (_I, [_I, _P, _U64, _U32, _U32, _U32, _U32, _F, _U32, _P, _P, _P, _P, _P, _P, _P]),
    "dance_search_queries": (_I, [_I, _P, _U64, _U32, _U32, _P, _U32, _U32, _P, _U64, _U32, _U32, _U32, _U32, _P,
                                  _P, _P]),
    "dance_search_queries_filtered": (_I, [_I, _P, _U64, _U32, _U32, _P, _U32, _P, _P, _P, _P, _P, _U64, _U32, _U32,
                                           _U32, _U32, _P, _P, _P]),
    "dance_merge_shards_gpu": (_I, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _U64, _U32,
                                    ctypes.c_char_p, ctypes.c_char_p]),
    "dance_merge_edges_device": (_I, [_P, _P, _U64, _U32, _U32, _U32, _U64, _P, _P, _P]),
    "dance_merge_edges_device_noalloc": (_I, [_P, _P, _U64, _U32, _U32, _U32, _U64, _P, _P, _P]),
    "dance_stitched_build": (_I, [_I, _P, _U32, _U32, _U32, _P, _P, _U32, _U32, _U32, _U32, _U32, _P, _U32, _P, _P,
                                  _U64, _P, _P]),
    "dance_stitched_label_graphs": (_I, [_I, _P, _U64, _U32, _U32, _U32, _P, _P, _P, _U32, _U32, _U32, _U32, _P,
                                         _U32, _P, _P, _P, _P]),
    "dance_stitched_remap": (_I, [_U32, _U32, _P, _P, _P, _P, _U32, _U32, _P, _P, _U64, _P, _P]),
    "dance_calculate_entry_point": (_I, [_I, _P, _U64, _U32, _U32, _PU32, _P]),
    "dance_select_label_starts": (_I, [_P, _P, _U32, _U32, _U32, _U64, _P, _P]),
    "dance_kmeanspp_seed": (_I, [_P, _U64, _U64, _U32, _U32, _U64, _P, _P, _P]),
    "dance_kmeans_lloyd": (_I, [_P, _U64, _U64, _U32, _U32, _U32, _P, _P, ctypes.POINTER(ctypes.c_double), _P]),
    "dance_partition_assign": (_I, [_I, _P, _U64, _U64, _U32, _P, _U32, _U32, _P, _P, _P]),
    "dance_partition_buckets": (_I, [_P, _U64, _U32, _U32, _P, _P, _P]),
    "dance_stitched_build_sharded": (_I, [_P, _I, _P, _U32, _U32, _U32, _P, _P, _U32, _U32, _U32, _U32, _U32, _P,
                                          _U32, _P, _P, _U64, _P, _P]),
    "dance_stitched_global_prune": (_I, [_I, _P, _U64, _U32, _U32, _P, _P, _P, _P, _U32, _U32, _F, _P, _P, _P,
                                         _P]),
    "dance_shard_range": (None, [_U32, _I, _I, _PU32, _PU32, _PU32]),
    "dance_nccl_unique_id": (_I, [_P, ctypes.c_size_t]),
    "dance_comm_create": (_I, [_I, _I, _P, ctypes.c_size_t, ctypes.c_double, _P]),
    "dance_comm_destroy": (None, [_P]),
    "dance_workspace_create_sharded": (_I, [_U32, _I, _U32, _U32, _U32, _U32, _P]),
    "dance_vamana_build_sharded": (_I, [_P, _I, _P, _U64, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P,
                                        _PU32, _P]),
}

_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load libdance_b200.so and declare every exported signature.

    Raises FileNotFoundError when the library has not been built: the CUDA
    path is the only path (build it with ``python -m dance_b200.build``).
    """
    global _lib
    if _lib is not None and path is None:
        return _lib
    env = os.environ.get("DANCE_B200_LIB")
    p = Path(path) if path else (Path(env) if env else LIB_PATH)
    if not p.exists():
        raise FileNotFoundError(
            f"{p} is missing: build the CUDA library with `python -m dance_b200.build` "
            "(there is no CPU fallback)")
    cdll = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(cdll, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = cdll
    return cdll


def __getattr__(name):
    if name == "lib":
        return load()
    raise AttributeError(name)


def check(rc: int, what: str = "libdance_b200") -> None:
    """Raise DanceError with the library's last message if rc != 0."""
    if rc != 0:
        msg = load().dance_last_error()
        raise DanceError(f"{what} failed with status {rc}: {msg.decode() if msg else ''}")


def last_build_report() -> dict:
    r = DanceBuildReport()
    check(load().dance_last_build_report(ctypes.byref(r)), "dance_last_build_report")
    return {n: getattr(r, n) for n, _ in r._fields_ if n != "reserved"}


def last_sharded_report() -> dict:
    r = DanceShardedReport()
    check(load().dance_last_sharded_report(ctypes.byref(r)), "dance_last_sharded_report")
    return {n: getattr(r, n) for n, _ in r._fields_ if n != "reserved"}


def default_params(**overrides) -> DanceVamanaParams:
    p = DanceVamanaParams()
    load().dance_vamana_default_params(ctypes.byref(p))
    for k, v in overrides.items():
        setattr(p, k, v)
    return p
