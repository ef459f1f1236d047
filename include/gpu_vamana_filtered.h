/*
 * gpu_vamana_filtered.h -- GPU-FilteredVamana entry points of
 * libdance_b200.so, drop-in for DANCE include/gpu_vamana_filtered.h:11-123
 * (same struct layout, names, arguments and status codes).
 *
 * The build is the reference's canonical path: a deterministic random graph
 * (degree min(16, R), seed 42), then three rounds of label-masked search per
 * (point, label) (pool min(FilteredL, 32), first min(pool, 8) slots kept),
 * union-label search per point (pool min(64, FilteredL), first min(R, L)
 * slots), fixed-order merge with label quotas into a work row of width
 * min(C, 128), FilteredRobustPrune(alpha) and an exact CSR reverse repair.
 * Float input is searched in fp16, uint8 exactly.  Setting
 * DISKANN_GPU_FILTERED_HANDOFF=0 starts from a vnew2 graph (work width
 * min(C, 96)) instead of the random graph, as the reference does.
 *
 * point_label_offsets (num_points + 1) and point_labels (total_label_count)
 * list each point's labels, strictly increasing and below num_labels;
 * label_to_start_id[l] is label l's start point (>= num_points if none);
 * universal_label_id is never searched as a label (UINT32_MAX: none);
 * global_start_id seeds the union search when it shares a label with the
 * point.  The query anchor arguments are accepted and unused, as in the
 * reference's canonical path.  h_graph (num_points x R, INVALID padded) and
 * h_degree are caller-allocated.
 *
 * Status: 0 success; -1 invalid argument or CUDA error; 1 when the work
 * width min(C, 128) is below 2R (the reverse repair's capacity), as the
 * reference returns (src/gpu_vamana_filtered.cu:5839-5843).
 */
#ifndef GPU_VAMANA_FILTERED_H
#define GPU_VAMANA_FILTERED_H

#include <stdint.h>

#ifndef DANCE_API
#if defined(__GNUC__)
#define DANCE_API __attribute__((visibility("default")))
#else
#define DANCE_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct GPUFilteredVamanaStats
{
    double gpu_build_seconds;
    double label_h2d_seconds;
    double graph_build_seconds;
    double diagnostics_seconds;
    double d2h_seconds;
    double peak_gpu_mem_gb;
    double backbone_seconds;
    double task_generation_seconds;
    double filtered_search_seconds;
    double ordinary_search_seconds;
    double merge_seconds;
    double forward_prune_seconds;
    double csr_reverse_seconds;
    double reverse_prune_seconds;
    double compaction_seconds;

    uint64_t filtered_search_distance_count;
    uint64_t unfiltered_search_distance_count;
    uint64_t label_check_count;
    uint64_t label_reject_count;
    uint64_t filtered_candidate_count;
    uint64_t unfiltered_candidate_count;
    uint64_t merged_candidate_count;
    uint64_t active_rows;
    uint64_t original_neighbor_count;
    uint64_t filtered_seed_count;
    uint64_t filtered_visited_count;
    uint64_t filtered_visited_reserved_count;
    uint64_t filtered_top_reserved_count;
    uint64_t bridge_reserved_count;
    uint64_t unfiltered_reserved_count;
    uint64_t filtered_reserved_count;
    uint64_t label_occlusion_blocked_count;
    uint64_t geometry_occluded_count;
    uint64_t candidate_rejected_by_label_count;
    uint64_t refill_count;
    uint64_t filtered_prune_reject_count;
    uint64_t universal_label_pass_count;
    uint64_t final_prune_rows;
    uint64_t reverse_edges;
    uint64_t reverse_touched_rows;
    uint64_t filtered_reverse_edges;
    uint64_t filtered_reverse_touched_rows;
    uint64_t filtered_reverse_candidates_kept;
    uint64_t filtered_reverse_pruned_rows;

    double avg_common_label_out_degree;
    double common_label_degree_before_avg;
    double common_label_degree_after_avg;
    double active_rows_frac;
    uint32_t low_common_label_degree_count;
    uint32_t low_common_before;
    uint32_t low_common_after;
    uint32_t out_degree_min;
    uint32_t out_degree_max;
    double out_degree_avg;
    uint32_t common_label_degree_min;
    uint32_t common_label_degree_max;
    uint32_t invalid_neighbor_count;
    uint32_t self_loop_count;
    double prune_output_degree_avg;
    uint32_t filtered_seed_source;
    uint32_t semantic_stage;
    uint32_t semantic_complete;
} GPUFilteredVamanaStats;

DANCE_API int gpu_vamana_filtered_build_uint8(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R,
                                              uint32_t L, uint32_t filtered_L, uint32_t C, uint32_t STEPS,
                                              float alpha, const uint32_t *point_label_offsets,
                                              const uint32_t *point_labels, uint32_t total_label_count,
                                              const uint32_t *label_to_start_id, uint32_t num_labels,
                                              uint32_t universal_label_id, uint32_t global_start_id,
                                              const uint32_t *query_anchor_offsets, const uint32_t *query_anchor_ids,
                                              uint32_t query_anchor_count, uint32_t *h_graph, uint32_t *h_degree);

DANCE_API int gpu_vamana_filtered_build_float(const float *h_data, uint32_t num_points, uint32_t dim, uint32_t R,
                                              uint32_t L, uint32_t filtered_L, uint32_t C, uint32_t STEPS,
                                              float alpha, const uint32_t *point_label_offsets,
                                              const uint32_t *point_labels, uint32_t total_label_count,
                                              const uint32_t *label_to_start_id, uint32_t num_labels,
                                              uint32_t universal_label_id, uint32_t global_start_id,
                                              const uint32_t *query_anchor_offsets, const uint32_t *query_anchor_ids,
                                              uint32_t query_anchor_count, uint32_t *h_graph, uint32_t *h_degree);

DANCE_API void gpu_vamana_filtered_get_last_stats(GPUFilteredVamanaStats *stats);

#ifdef __cplusplus
}
#endif

#endif /* GPU_VAMANA_FILTERED_H */
