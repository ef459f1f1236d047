/*
 * dance_b200.h -- additive C ABI of libdance_b200.so.
 *
 * These entry points have no one-to-one counterpart in the reference C ABI;
 * they expose what the reference keeps as compile-time macros or static
 * functions so that in-process callers (benchmarks, parity tests, the
 * multi-GPU driver) can run the same build on vectors already resident in
 * device memory, one stage at a time, or sharded over several GPUs.
 * All pointers named d_* are device pointers on the current CUDA device,
 * all streams are cudaStream_t passed as void* (NULL = legacy default).
 * Return codes: 0 success, -1 invalid argument, -2 CUDA error, -3 NCCL error,
 * -4 a bounded device wait timed out.  The message of the last failure is
 * available from dance_last_error().
 */
#ifndef DANCE_B200_H
#define DANCE_B200_H

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
#include <stddef.h>

#include "gpu_vamana_filtered.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of the vector store. */
enum
{
    DANCE_U8 = 0,  /* uint8, exact integer squared L2 */
    DANCE_F16 = 1, /* IEEE binary16 storage, half-precision diff/square as the reference */
    DANCE_F32 = 2  /* float32 */
};

/* Runtime form of the knobs in gpu_vamana_config.h (same names, lower case). */
typedef struct DanceVamanaParams
{
    uint32_t iters;               /* VAMANA_ITERS */
    float alpha;                  /* VAMANA_ALPHA, used in the last round */
    uint32_t init_random_seeds;   /* INIT_RANDOM_SEEDS */
    uint32_t final_min_degree;    /* FINAL_MIN_DEGREE (0 = no refill) */
    uint32_t medoid_candidates;   /* MEDOID_NUM_CANDIDATES */
    uint32_t medoid_samples;      /* MEDOID_NUM_SAMPLES */
    uint32_t coarse_warmup_iters; /* COARSE_WARMUP_ITERS (0 = off) */
    uint32_t warmup_expand_steps; /* WARMUP_EXPAND_STEPS */
    uint32_t reverse_heavy_cap;   /* ENABLE_REVERSE_HEAVY_CAP */
    uint32_t reverse_heavy_threshold;
    uint32_t reverse_heavy_sample;
    uint32_t visited_log2;        /* log2 of the per-search visited table (performance only) */
    uint32_t reserved[8];
} DanceVamanaParams;

DANCE_API void dance_vamana_default_params(DanceVamanaParams *params);

/* Message of the most recent failure in this thread ("" if none). */
DANCE_API const char *dance_last_error(void);

/* Number of kernels launched by this library in this process so far. */
DANCE_API uint64_t dance_kernel_launch_count(void);

/* ---- workspace --------------------------------------------------------- */
/* Opaque device scratch sized for (N, R, L, C, STEPS); reused across builds
 * of at most that size on the device that created it. */
typedef struct DanceWorkspace DanceWorkspace;
DANCE_API int dance_workspace_create(uint32_t num_points, uint32_t R, uint32_t L, uint32_t C, uint32_t STEPS,
                           DanceWorkspace **ws);
DANCE_API void dance_workspace_destroy(DanceWorkspace *ws);

/* ---- whole build on device-resident vectors ----------------------------- */
/* d_data: num_points rows of row_stride_bytes (a multiple of 16, at least
 * dim * element size; padding bytes must be zero).  Writes d_graph
 * (num_points x R, INVALID padded), d_degree, optionally d_graph_dists
 * (num_points x R, FLT_MAX padded), and *medoid_out (host).  ws may be NULL.
 * Asynchronous on stream except for the final medoid read-back. */
DANCE_API int dance_vamana_build_resident(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points,
                                uint32_t dim, uint32_t R, uint32_t L, uint32_t C, uint32_t STEPS,
                                const DanceVamanaParams *params, DanceWorkspace *ws, uint32_t *d_graph,
                                uint32_t *d_degree, float *d_graph_dists, uint32_t *medoid_out, void *stream);

/* Device-side timings (seconds, CUDA events on the build stream, summed over
 * rounds) and work counters of the last dance_vamana_build_resident call in
 * this thread.  search includes the online-insert replay (the reference's
 * search_online_insert_seconds); search_kernel is the GreedySearch kernel
 * alone.  Counters: distance evaluations of the search, expansions,
 * pair distances of the insert replay, reverse-merge evaluations, pair
 * distances of the prune. */
typedef struct DanceBuildReport
{
    double medoid_seconds, search_seconds, search_kernel_seconds, replay_seconds, reverse_seconds, prune_seconds,
        total_seconds;
    uint64_t search_evals, expansions, replay_pairs, reverse_evals, prune_pairs;
    uint64_t reserved[3];
} DanceBuildReport;
DANCE_API int dance_last_build_report(DanceBuildReport *report);

/* ---- single stages (parity tests) ---------------------------------------- */
DANCE_API int dance_stage_medoid(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points,
                       uint32_t dim, uint32_t num_candidates, uint32_t num_samples, float *d_scores,
                       uint32_t *d_candidate_ids, uint32_t *d_medoid, void *stream);
DANCE_API int dance_stage_init(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points, uint32_t dim,
                     uint32_t R, uint32_t *d_cur_ids, float *d_cur_dists, uint32_t *d_degree, void *stream);
/* Batched GreedySearch of every vertex on the frozen graph; records each
 * vertex's expansion sequence (exp_stride entries per vertex). */
DANCE_API int dance_stage_search(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points, uint32_t dim,
                       uint32_t R, uint32_t L, uint32_t steps, uint32_t entry, uint32_t init_random_seeds,
                       uint32_t visited_log2, const uint32_t *d_cur_ids, const float *d_cur_dists,
                       const uint32_t *d_degree, uint32_t *d_exp_ids, float *d_exp_dists, uint32_t *d_exp_count,
                       uint32_t exp_stride, void *stream);
/* Online RobustInsert replay of the expansion sequences into C-wide work rows. */
DANCE_API int dance_stage_replay(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points, uint32_t dim,
                       uint32_t R, uint32_t C, float alpha, const uint32_t *d_cur_ids, const float *d_cur_dists,
                       const uint32_t *d_degree, const uint32_t *d_exp_ids, const float *d_exp_dists,
                       const uint32_t *d_exp_count, uint32_t exp_stride, uint32_t *d_work_ids,
                       float *d_work_dists, uint32_t *d_work_deg, void *stream);
/* Exact CSR reverse-edge merge into the work rows (in place). */
DANCE_API int dance_stage_reverse_merge(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points,
                              uint32_t dim, uint32_t R, uint32_t C, const DanceVamanaParams *params,
                              DanceWorkspace *ws, uint32_t *d_work_ids, float *d_work_dists, uint32_t *d_work_deg,
                              uint64_t *reverse_edges_out, void *stream);
/* RobustPrune(alpha) of the work rows into the R-wide graph. */
DANCE_API int dance_stage_prune(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points, uint32_t dim,
                      uint32_t R, uint32_t C, float alpha, uint32_t min_degree, const uint32_t *d_work_ids,
                      const float *d_work_dists, const uint32_t *d_work_deg, uint32_t *d_cur_ids,
                      float *d_cur_dists, uint32_t *d_degree, void *stream);

/* ---- sharded build over the GPUs of one box (one process per GPU) -------- */
/* Rank r owns vertices [v0, v1) = [r*chunk, min(N, (r+1)*chunk)),
 * chunk = ceil(N / world).  Graph buffers are world*chunk rows. */
DANCE_API void dance_shard_range(uint32_t num_points, int world, int rank, uint32_t *v0, uint32_t *v1,
                                 uint32_t *chunk);
typedef struct DanceComm DanceComm;
/* NCCL unique id (rank 0 creates it and shares it with the other ranks). */
DANCE_API int dance_nccl_unique_id(uint8_t *out, size_t out_bytes);
/* Non-blocking NCCL communicator on the current device; every wait on it is
 * bounded by timeout_s, after which it is aborted and the call returns -4. */
DANCE_API int dance_comm_create(int rank, int world, const uint8_t *unique_id, size_t id_bytes, double timeout_s,
                                DanceComm **comm);
DANCE_API void dance_comm_destroy(DanceComm *comm);
DANCE_API int dance_workspace_create_sharded(uint32_t num_points, int world, uint32_t R, uint32_t L, uint32_t C,
                                             uint32_t STEPS, DanceWorkspace **ws);
/* The standard build with vertex batches sharded across the communicator's
 * ranks; d_data is the full store on every rank.  d_graph (world*chunk x R),
 * d_degree and d_table_degree (world*chunk) are caller buffers; on return
 * every rank holds the whole graph, bit-identical to the one-GPU build.
 * Per round each new edge goes to the rank that owns its target (grouped
 * ncclSend/ncclRecv of (target, source) pairs after an all-gather of the
 * per-owner counts), and the pruned rows are all-gathered.  d_table_degree
 * is no longer written (kept for the signature).  At most 64 ranks. */
DANCE_API int dance_vamana_build_sharded(DanceComm *comm, int dtype, const void *d_data, uint64_t row_stride_bytes,
                                         uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L, uint32_t C,
                                         uint32_t STEPS, const DanceVamanaParams *params, DanceWorkspace *ws,
                                         uint32_t *d_graph, uint32_t *d_degree, uint32_t *d_table_degree,
                                         uint32_t *medoid_out, void *stream);

/* Device time of this rank's last sharded build per stage, summed over the
 * rounds (CUDA events on the build stream): the exchange stages include the
 * time spent waiting for the slowest rank.  Bytes are this rank's own
 * traffic over the build. */
typedef struct DanceShardedReport
{
    double medoid_init_seconds, search_seconds, replay_seconds, edge_exchange_seconds, reverse_seconds,
        prune_seconds, graph_exchange_seconds, total_seconds;
    uint64_t edge_bytes_sent, edge_bytes_received, graph_bytes_received, rounds;
    uint64_t reserved[4];
} DanceShardedReport;
DANCE_API int dance_last_sharded_report(DanceShardedReport *report);

/* ---- shard merge (C form of diskann::merge_shards_gpu, include/gpu_merge.h) */
DANCE_API int dance_merge_shards_gpu(const char *vamana_prefix, const char *vamana_suffix, const char *idmaps_prefix,
                                     const char *idmaps_suffix, uint64_t nshards, uint32_t max_degree,
                                     const char *output_vamana, const char *medoids_file);
/* Device core of the merge for sources [node_begin, node_begin + node_count):
 * edges (d_src[i] -> d_dst[i]) in global ids without self loops; writes
 * each source's first max_degree distinct destinations in hash rank order
 * to d_out_neighbors (node_count x max_degree) and d_out_degrees. */
DANCE_API int dance_merge_edges_device(const uint32_t *d_src, const uint32_t *d_dst, uint64_t n_edges,
                                       uint32_t node_begin, uint32_t node_count, uint32_t max_degree, uint64_t seed,
                                       uint32_t *d_out_neighbors, uint32_t *d_out_degrees, void *stream);
/* Same merge and same results as dance_merge_edges_device, without any
 * device allocation.  No counterpart in the reference: its merge always
 * allocates.  For callers that cannot allocate device memory on this path:
 * a process whose memory is owned by another allocator (a framework's
 * caching pool that has reserved the free memory, so cudaMalloc fails), or a
 * loop that keeps other streams busy, where cudaMalloc/cudaFree would stall
 * them because cudaFree waits for the whole device.
 * Scratch is one fixed array in the library's device memory (about 4.3 MiB
 * per device): at most 16384 sources (node_count) and 1048576 edges
 * (n_edges); larger requests return -5 before any work is issued.  The
 * first call on a device (and the first after that device's context was
 * re-created, e.g. by cudaDeviceReset) looks the array's device address up
 * with cudaGetSymbolAddress; make that first call before any stream
 * capture begins.  Every call waits for its stream to finish before it
 * returns, to read the kernels' error word.  All calls on one device share
 * the array, so calls that overlap in time (from several host threads, or
 * on several streams) race on it and give wrong results: run them one after
 * another. */
DANCE_API int dance_merge_edges_device_noalloc(const uint32_t *d_src, const uint32_t *d_dst, uint64_t n_edges,
                                               uint32_t node_begin, uint32_t node_count, uint32_t max_degree,
                                               uint64_t seed, uint32_t *d_out_neighbors, uint32_t *d_out_degrees,
                                               void *stream);

/* ---- GPU-StitchedVamana (apps/utils/gpu_stitched_vamana_index.cpp:241-428) */
/* Labels are given as a CSR: label l (0-based here; the sidecar files number
 * it l + 1) holds the points label_points[label_offsets[l] ..
 * label_offsets[l + 1]), in the order the label file lists them.  Every
 * label's points form one independent vnew2 graph (Rsmall, Lsmall, C,
 * steps); a point's output row is the concatenation over its labels, in
 * label order, of the first min(local degree, Rstitched) local neighbours
 * mapped to global ids, skipping invalid ids and self loops and not
 * repeating an id (:276-341).  Rstitched below Rsmall is raised to Rsmall,
 * as the reference app does (:86-87).  The global label-aware prune that the
 * reference runs for multi-label rows (:353-372) is a separate call,
 * dance_stitched_global_prune. */
typedef struct DanceStitchedStats
{
    uint32_t num_labels;
    uint32_t npts_per_label_min;
    uint32_t npts_per_label_max;
    uint32_t max_degree; /* largest output row */
    double npts_per_label_mean;
    uint64_t total_label_memberships;
    uint64_t processed_label_memberships;
    uint64_t remap_invalid_local_ids;
    uint64_t remap_self_loops;
    uint64_t remap_duplicate_edges;
    uint64_t output_edges;
    double label_data_materialization_seconds; /* upload + label-major gather */
    double per_label_gpu_build_sum_seconds;    /* summed over labels */
    double per_label_gpu_build_max_seconds;
    double label_build_wall_seconds;           /* all labels, streams overlapped */
    double local_to_global_remap_seconds;
    double total_seconds;
    double peak_gpu_mem_gb;
    double search_kernel_seconds; /* GreedySearch kernel time summed over labels */
    uint64_t search_evals;        /* GreedySearch distance evaluations, all labels */
    uint64_t search_expansions;
    uint32_t streams; /* label builds in flight at once */
    uint32_t reserved0;
    double label_graph_exchange_seconds; /* sharded build: local graphs to rank 0 */
    uint64_t reserved[3];
} DanceStitchedStats;

/* Host in, host out.  dtype DANCE_U8 or DANCE_F32 (fp16 storage when the
 * float build is configured so, as for gpu_vamana_vnew2_build_float).
 * row_offsets has N + 1 entries; row_ids needs at most
 * label_offsets[num_labels] * Rsmall entries (error -3 when
 * row_ids_capacity is smaller than the result).  label_medoids[l] is the
 * global id of label l's medoid.  streams = 0 picks 4. */
DANCE_API int dance_stitched_build(int dtype, const void *h_data, uint32_t num_points, uint32_t dim,
                                   uint32_t num_labels, const uint64_t *label_offsets, const uint32_t *label_points,
                                   uint32_t r_small, uint32_t l_small, uint32_t r_stitched, uint32_t C,
                                   uint32_t steps, const DanceVamanaParams *params, uint32_t streams,
                                   uint64_t *row_offsets, uint32_t *row_ids, uint64_t row_ids_capacity,
                                   uint32_t *label_medoids, DanceStitchedStats *stats);
/* The same build spread over the GPUs of one box (one process per GPU, a
 * communicator from dance_comm_create): labels go largest first to the
 * least-loaded rank, every rank builds its labels from its own copy of the
 * vectors, the local graphs, degrees and medoids go to rank 0 (grouped
 * ncclSend/ncclRecv per label segment, a sum-reduce of the medoids), and
 * rank 0 stitches.  The outputs are written on rank 0 only and equal
 * dance_stitched_build's; the other ranks' output pointers may be NULL.
 * Every wait is bounded by the communicator's timeout (-4 after it). */
DANCE_API int dance_stitched_build_sharded(DanceComm *comm, int dtype, const void *h_data, uint32_t num_points,
                                           uint32_t dim, uint32_t num_labels, const uint64_t *label_offsets,
                                           const uint32_t *label_points, uint32_t r_small, uint32_t l_small,
                                           uint32_t r_stitched, uint32_t C, uint32_t steps,
                                           const DanceVamanaParams *params, uint32_t streams, uint64_t *row_offsets,
                                           uint32_t *row_ids, uint64_t row_ids_capacity, uint32_t *label_medoids,
                                           DanceStitchedStats *stats);
/* Device-resident first half, for label-parallel multi-GPU builds: builds
 * the labels with label_mask[l] != 0 (all when label_mask is NULL) from the
 * padded store d_data into d_local_graph (memberships x Rsmall, membership m
 * of label l at row label_offsets[l] + local index) and d_local_degree, and
 * writes label l's local medoid index to label_medoids_local[l] (host).  Rows
 * and medoids of unselected labels are left untouched. */
DANCE_API int dance_stitched_label_graphs(int dtype, const void *d_data, uint64_t row_stride_bytes,
                                          uint32_t num_points, uint32_t dim, uint32_t num_labels,
                                          const uint64_t *label_offsets, const uint32_t *label_points,
                                          const uint8_t *label_mask, uint32_t r_small, uint32_t l_small, uint32_t C,
                                          uint32_t steps, const DanceVamanaParams *params, uint32_t streams,
                                          uint32_t *d_local_graph, uint32_t *d_local_degree,
                                          uint32_t *label_medoids_local, DanceStitchedStats *stats);
/* Second half: local graphs (device) to the stitched CSR graph (host). */
DANCE_API int dance_stitched_remap(uint32_t num_points, uint32_t num_labels, const uint64_t *label_offsets,
                                   const uint32_t *label_points, const uint32_t *d_local_graph,
                                   const uint32_t *d_local_degree, uint32_t r_small, uint32_t r_stitched,
                                   uint64_t *row_offsets, uint32_t *row_ids, uint64_t row_ids_capacity,
                                   DanceStitchedStats *stats, void *stream);
/* Label-aware global prune of a stitched union graph: the DiskANN CPU step
 * (Index::prune_all_neighbors(Rstitched, 750, alpha) as patched by DANCE)
 * that the reference app runs when rows carry several labels or Rsmall >
 * Rstitched (apps/utils/gpu_stitched_vamana_index.cpp:353-372; coverage rule
 * integration patch lines 20009-20047, label-balanced shortlist 20055-20100).
 * Device inputs: the union graph as a CSR (d_row_offsets N+1, d_row_ids) and
 * the points' labels as a CSR with ascending labels per point (both label
 * pointers NULL = unlabelled: plain occlusion).  Rows with at most `range`
 * neighbours are copied; longer rows are pruned to at most `range`.
 * Output: d_out_rows (N x range, 0xFFFFFFFF padded) and d_out_degree.
 * Rows longer than 2048 neighbours are refused (-1).  Synchronises stream
 * (it reads the longest row's length back to size the per-warp pools). */
DANCE_API int dance_stitched_global_prune(int dtype, const void *d_data, uint64_t row_stride_bytes,
                                          uint32_t num_points, uint32_t dim, const uint64_t *d_row_offsets,
                                          const uint32_t *d_row_ids, const uint32_t *d_point_label_offsets,
                                          const uint32_t *d_point_labels, uint32_t range,
                                          uint32_t max_candidates, float alpha, uint32_t *d_out_rows,
                                          uint32_t *d_out_degree, uint64_t *pruned_rows_out, void *stream);

/* ---- inputs DiskANN computes before the filtered build hook --------------- */
/* Index entry point (DiskANN Index::calculate_entry_point, called by the
 * filtered hook at integration patch line 20267): the centroid of all points
 * (float, summed point by point in point order, divided by N), then the
 * point nearest to it by squared L2 (dimensions summed in order, no fused
 * multiply-add; lowest index on ties).  Synchronises stream. */
DANCE_API int dance_calculate_entry_point(int dtype, const void *d_data, uint64_t row_stride_bytes,
                                          uint32_t num_points, uint32_t dim, uint32_t *entry_out, void *stream);
/* One start point per label (DiskANN's _label_to_start_id, computed before
 * the hook, patch lines 20238-20241): labels in ascending id order; each
 * draws num_candidates of its points (DiskANN uses 25) and takes the one
 * chosen as a start the fewest times so far (first draw on ties).  Draw k of
 * label l is point hash(seed, l, k) mod |points of l| (DiskANN uses rand()).
 * d_label_offsets (num_labels + 1) / d_label_points: each label's points in
 * ascending order, universal-label points included in every label.  Empty
 * labels get 0xFFFFFFFF.  Synchronises stream. */
DANCE_API int dance_select_label_starts(const uint32_t *d_label_offsets, const uint32_t *d_label_points,
                                        uint32_t num_labels, uint32_t num_points, uint32_t num_candidates,
                                        uint64_t seed, uint32_t *d_starts, void *stream);

/* ---- GPU-FilteredVamana on resident vectors ------------------------------- */
/* The canonical filtered build of gpu_vamana_filtered.h on a padded store
 * already in device memory: dtype DANCE_U8 or DANCE_F16 (the float entry
 * point searches in fp16); work_C is the work width itself (no min(C, 128)
 * clamp here; it must lie in [2R, 128]).  Label arrays are host arrays as in
 * gpu_vamana_filtered.h.  d_init_graph/d_init_degree (N x R) replace the
 * random initial graph when given; rounds = 3 is the reference's schedule.
 * Status 1 when work_C < 2R. */
DANCE_API int dance_filtered_build_resident(int dtype, const void *d_data, uint64_t row_stride_bytes,
                                            uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                                            uint32_t filtered_L, uint32_t work_C, uint32_t STEPS, float alpha,
                                            const uint32_t *point_label_offsets, const uint32_t *point_labels,
                                            const uint32_t *label_to_start_id, uint32_t num_labels,
                                            uint32_t universal_label_id, uint32_t global_start_id,
                                            const uint32_t *d_init_graph, const uint32_t *d_init_degree,
                                            uint32_t rounds, uint32_t *d_graph, uint32_t *d_degree,
                                            GPUFilteredVamanaStats *stats, void *stream);
/* The reference's deterministic random initial graph (min(R, initial_degree,
 * N-1) distinct hashed neighbours per point, INVALID padded). */
DANCE_API int dance_filtered_random_graph(uint32_t num_points, uint32_t R, uint32_t initial_degree, uint32_t seed,
                                          uint32_t *d_graph, uint32_t *d_degree, void *stream);
/* One round from (d_graph_in, d_degree_in) with its intermediates copied out
 * (parity tests): per-(point, label) search outputs (total labels x
 * min(min(filtered_L, 32), 8)), union search outputs (N x min(R, L)), merged
 * work rows (N x work_C) with distances and lengths, the forward-pruned graph
 * and the reverse-repaired graph (N x R).  Any output but the last two may
 * be NULL. */
DANCE_API int dance_filtered_stage_round(int dtype, const void *d_data, uint64_t row_stride_bytes,
                                         uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                                         uint32_t filtered_L, uint32_t work_C, uint32_t STEPS, float alpha,
                                         const uint32_t *point_label_offsets, const uint32_t *point_labels,
                                         const uint32_t *label_to_start_id, uint32_t num_labels,
                                         uint32_t universal_label_id, uint32_t global_start_id,
                                         const uint32_t *d_graph_in, const uint32_t *d_degree_in,
                                         uint32_t *d_task_ids, float *d_task_dists, uint32_t *d_union_ids,
                                         float *d_union_dists, uint32_t *d_work_ids, float *d_work_dists,
                                         uint32_t *d_work_degree, uint32_t *d_forward_graph,
                                         uint32_t *d_forward_degree, uint32_t *d_graph_out, uint32_t *d_degree_out,
                                         void *stream);

/* ---- query search over a built graph (recall harness) -------------------- */
/* DiskANN-style best-first search from `start` with list size L_search; the
 * K nearest found per query go to d_out_ids / d_out_dists (nq x K). */
DANCE_API int dance_search_queries(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points,
                         uint32_t dim, const uint32_t *d_graph, uint32_t R, uint32_t start, const void *d_queries,
                         uint64_t query_stride_bytes, uint32_t num_queries, uint32_t L_search, uint32_t K,
                         uint32_t visited_log2, uint32_t *d_out_ids, float *d_out_dists, void *stream);
/* Label-filtered form (DiskANN filtered search): query i visits only points
 * carrying d_query_labels[i] (d_label_offsets/d_labels: the points' label
 * CSR on the device, ascending per point) and starts from d_query_starts[i]. */
DANCE_API int dance_search_queries_filtered(int dtype, const void *d_data, uint64_t row_stride_bytes,
                                            uint32_t num_points, uint32_t dim, const uint32_t *d_graph, uint32_t R,
                                            const uint32_t *d_label_offsets, const uint32_t *d_labels,
                                            const uint32_t *d_query_labels, const uint32_t *d_query_starts,
                                            const void *d_queries, uint64_t query_stride_bytes, uint32_t num_queries,
                                            uint32_t L_search, uint32_t K, uint32_t visited_log2,
                                            uint32_t *d_out_ids, float *d_out_dists, void *stream);

/* ---- sharded disk-index pipeline: k-means partition ---------------------- */
/* The GPU form of DiskANN's partitioner as the DANCE patch drives it before
 * the GPU shard-build loop (partition_with_ram_budget ->
 * shard_data_into_clusters_only_ids, integration patch lines 20629-20688;
 * shard loop lines 3270-3600).  Distances are squared L2 in float, summed
 * dimension by dimension without fused multiply-add; DiskANN's own
 * (GEMM-based, randomly seeded) partitioner is not in the reference, so the
 * shards match it in kind, not bit for bit.  Training rows are float32 with
 * a stride that is a multiple of 4 bytes; k * dim <= 24576.  All four
 * synchronise `stream` before they return (their scratch is freed). */
/* k-means++ seeding: d_centers (k x dim) receives the k pivots, d_picked (k)
 * the training rows they were copied from.  Pivot 0 is row
 * splitmix64(seed) mod n; pivot p is drawn with probability proportional to
 * the squared distance to the nearest earlier pivot, the weights quantised
 * to floor(w / max w * 2^31) so that the draw (splitmix64 of seed and p,
 * modulo the integer total) is exact. */
DANCE_API int dance_kmeanspp_seed(const float *d_train, uint64_t row_stride_bytes, uint64_t n, uint32_t dim,
                                  uint32_t k, uint64_t seed, float *d_centers, uint64_t *d_picked, void *stream);
/* `iters` Lloyd iterations from the centers in d_centers (replaced in
 * place): nearest center per row (lowest center on ties), then each center
 * the float64 mean of its members (summed in row order within blocks of 4096
 * rows, block sums in block order); a center without members stays.
 * d_assign (n, optional) receives the assignment to the final centers,
 * *residual_out (optional) the sum of squared distances of the last
 * iteration's assignment. */
DANCE_API int dance_kmeans_lloyd(const float *d_train, uint64_t row_stride_bytes, uint64_t n, uint32_t dim, uint32_t k,
                                 uint32_t iters, float *d_centers, uint32_t *d_assign, double *residual_out,
                                 void *stream);
/* Each point's k_base (1..8) nearest centers, nearest first, lower center on
 * ties, to d_out_centers (num_points x k_base) and, if given, their squared
 * distances to d_out_dists.  dtype DANCE_U8, DANCE_F16 or DANCE_F32; rows
 * need only be element-aligned (no 16-byte padding). */
DANCE_API int dance_partition_assign(int dtype, const void *d_data, uint64_t row_stride_bytes, uint64_t num_points,
                                     uint32_t dim, const float *d_centers, uint32_t num_centers, uint32_t k_base,
                                     uint32_t *d_out_centers, float *d_out_dists, void *stream);
/* Shard id lists from an assignment (num_points x k_base shard numbers):
 * shard s holds d_shard_ids[d_shard_offsets[s] .. d_shard_offsets[s + 1]),
 * the points that chose it, in ascending order (DiskANN's
 * <prefix>_subshard-<s>_ids_uint32.bin contents).  num_shards <= 8192;
 * choices >= num_shards are skipped; num_points * k_base < 2^32. */
DANCE_API int dance_partition_buckets(const uint32_t *d_assign, uint64_t num_points, uint32_t k_base,
                                      uint32_t num_shards, uint32_t *d_shard_offsets, uint32_t *d_shard_ids,
                                      void *stream);

#ifdef __cplusplus
}
#endif

#endif /* DANCE_B200_H */
