/*
 * gpu_vamana_builder.h -- standard Vamana builder C ABI (drop-in for DANCE).
 *
 * Every declaration here replaces the one of the same name in the reference
 * header include/gpu_vamana_builder.h (lines 11-81); the signatures, argument
 * meaning, ownership and return codes are kept identical so that callers such
 * as apps/utils/gpu_vamana_memory_index.cpp:316-347,
 * apps/utils/gpu_stitched_vamana_index.cpp:294-308 and DiskANN's
 * build_gpu_shard_index_from_data (integration patch lines 2811-2990) link
 * against libdance_b200.so unchanged.
 *
 * Conventions shared by all entry points:
 *   - inputs are host pointers, row-major, num_points x dim;
 *   - h_graph is caller-allocated, num_points x R uint32, padded with
 *     0xFFFFFFFF beyond each row's degree; h_degree is num_points uint32;
 *   - the current CUDA device is used (cudaGetDevice);
 *   - return 0 on success, -1 on invalid arguments or a CUDA error (a
 *     message is printed to stderr), STEPS > L is clamped to L with a warning,
 *     C < R is an error.
 */
#ifndef DANCE_B200_GPU_VAMANA_BUILDER_H
#define DANCE_B200_GPU_VAMANA_BUILDER_H

#include <stdint.h>

/* Exported with default visibility even when the library is built with
 * -fvisibility=hidden. */
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

/* Per-build timings and counters.  Same field order and types as the
 * reference struct (include/gpu_vamana_builder.h:11-28). */
typedef struct GPUVamanaStats
{
    double medoid_seconds;
    double h2d_seconds;
    double search_online_insert_seconds;
    double reverse_seconds;
    double final_prune_seconds;
    double d2h_seconds;
    double gpu_build_seconds;
    uint64_t distance_computations;
    uint64_t online_insert_attempts;
    uint64_t online_insert_mutations;
    uint64_t reverse_candidate_overflows;
    uint64_t reverse_proposals;
    uint64_t reverse_touched_rows;
    double reverse_csr_seconds;
    uint32_t selective_active_nodes;
} GPUVamanaStats;

/* Legacy "v8" builder entry points (reference src/gpu_vamana_uint8.cu:3093-3120).
 * uint8 and float input. */
DANCE_API int gpu_vamana_build(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                     uint32_t C, uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree);
DANCE_API int gpu_vamana_build_float(const float *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                           uint32_t C, uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree);

/* Standard vnew2 builder (reference src/gpu_vamana_vnew2.cu:2857-2917). */
DANCE_API int gpu_vamana_vnew2_build(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                           uint32_t C, uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree);
DANCE_API int gpu_vamana_vnew2_build_float(const float *h_data, uint32_t num_points, uint32_t dim, uint32_t R,
                                 uint32_t L, uint32_t C, uint32_t STEPS, uint32_t *h_graph,
                                 uint32_t *h_degree);

/* Device hand-off variants (reference src/gpu_vamana_vnew2_handoff.cu:110-151):
 * the build result stays on the current device.  *d_data receives the
 * device copy of the input vectors (as the element type the build used),
 * *d_graph the num_points x R graph and *d_degree the degrees.  The caller
 * owns the three allocations and releases them with cudaFree. */
DANCE_API int gpu_vamana_vnew2_build_device(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R,
                                  uint32_t L, uint32_t C, uint32_t STEPS, uint8_t **d_data,
                                  uint32_t **d_graph, uint32_t **d_degree);
DANCE_API int gpu_vamana_vnew2_build_device_float(const float *h_data, uint32_t num_points, uint32_t dim,
                                        uint32_t R, uint32_t L, uint32_t C, uint32_t STEPS,
                                        float **d_data, uint32_t **d_graph, uint32_t **d_degree);

/* Entry point (approximate medoid) and stats of the last build in this
 * process.  Like the reference these are process-global: concurrent builds
 * from several host threads overwrite each other's values. */
DANCE_API uint32_t gpu_vamana_get_last_medoid(void);
DANCE_API void gpu_vamana_get_last_stats(GPUVamanaStats *stats);
DANCE_API uint32_t gpu_vamana_vnew2_get_last_medoid(void);
DANCE_API void gpu_vamana_vnew2_get_last_stats(GPUVamanaStats *stats);

#ifdef __cplusplus
}
#endif

#endif /* DANCE_B200_GPU_VAMANA_BUILDER_H */
