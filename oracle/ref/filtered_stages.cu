// Stage-level harness around the reference's GPU-FilteredVamana kernels.
//
// TEST INFRASTRUCTURE ONLY.  This file includes the reference's own
// src/gpu_vamana_filtered.cu unmodified (-I points at the reference tree) and
// runs ONE canonical round on a caller-given graph with the kernel calls and
// arguments of the reference driver (canonical_round0_from_host_backbone_typed,
// src/gpu_vamana_filtered.cu:5889-6172, defaults: no fused search, no active
// frontier, no parity/publish paths), copying every intermediate back to the
// host: task-search outputs, union-search outputs, merged work rows with their
// distances, the forward-pruned graph and the reverse-repaired graph.  The
// parity tests use these outputs to pin the CPU oracle stage by stage.
#include "src/gpu_vamana_filtered.cu"

namespace
{
template <typename SearchT>
int stage_round(const SearchT *d_data, uint32_t N, uint32_t dim, uint32_t R, uint32_t L, uint32_t FL, uint32_t C,
                uint32_t STEPS, float alpha, const uint32_t *h_offsets, const uint32_t *h_labels,
                uint32_t total_labels, const uint32_t *h_starts, uint32_t num_labels, uint32_t universal,
                uint32_t global_start, const uint32_t *h_graph_in, const uint32_t *h_degree_in, uint32_t *task_ids,
                float *task_d, uint32_t *ord_ids, float *ord_d, uint32_t *work_ids, float *work_d,
                uint32_t *work_deg, uint32_t *fwd_graph, uint32_t *fwd_deg, uint32_t *graph_out, uint32_t *deg_out)
{
    const uint32_t warps_per_block = 8, threads = warps_per_block * 32;
    const uint32_t per_label_pool = std::min(FL, 32u), per_label_keep = std::min(per_label_pool, 8u);
    const uint32_t ordinary_keep = std::min(R, L), ordinary_pool = std::min<uint32_t>(64u, FL);
    if ((size_t)N * C < (size_t)N * R * 2)
        return 1;
    std::vector<uint32_t> sizes(std::max(1u, num_labels), 0);
    for (uint32_t p = 0; p < total_labels; ++p)
        if (h_labels[p] < num_labels)
            ++sizes[h_labels[p]];
    std::vector<uint32_t> lpo((size_t)std::max(1u, num_labels) + 1, 0);
    for (uint32_t l = 0; l < num_labels; ++l)
        lpo[l + 1] = lpo[l] + sizes[l];
    std::vector<uint32_t> lp(std::max<uint32_t>(lpo[num_labels], 1)), cur(lpo.begin(), lpo.end() - 1);
    for (uint32_t row = 0; row < N; ++row)
        for (uint32_t p = h_offsets[row]; p < h_offsets[row + 1]; ++p)
            if (h_labels[p] < num_labels)
                lp[cur[h_labels[p]]++] = row;
    uint32_t *d_offsets, *d_labels, *d_starts, *d_lpo, *d_lp, *d_task_rows, *d_ga, *d_da, *d_gb, *d_db;
    uint32_t *d_task_c, *d_work, *d_work_deg, *d_ord, *d_rev_off, *d_rev_cur, *d_rev_ids = nullptr, *d_cand_off;
    uint32_t *d_touched_ids, *d_all_ids, *d_selected;
    float *d_task_d, *d_work_d, *d_ord_d;
    uint8_t *d_removed, *d_changed, *d_touched;
    const size_t T = total_labels;
    cudaMalloc(&d_offsets, (N + 1) * 4ull);
    cudaMalloc(&d_labels, std::max<size_t>(T, 1) * 4);
    cudaMalloc(&d_starts, std::max(1u, num_labels) * 4ull);
    cudaMalloc(&d_lpo, lpo.size() * 4);
    cudaMalloc(&d_lp, lp.size() * 4);
    cudaMalloc(&d_task_rows, std::max<size_t>(T, 1) * 4);
    cudaMalloc(&d_ga, (size_t)N * R * 4);
    cudaMalloc(&d_da, N * 4ull);
    cudaMalloc(&d_gb, (size_t)N * R * 4);
    cudaMalloc(&d_db, N * 4ull);
    cudaMalloc(&d_task_c, std::max<size_t>(T, 1) * per_label_keep * 4);
    cudaMalloc(&d_task_d, std::max<size_t>(T, 1) * per_label_keep * 4);
    cudaMalloc(&d_work, (size_t)N * C * 4);
    cudaMalloc(&d_work_d, (size_t)N * C * 4);
    cudaMalloc(&d_work_deg, N * 4ull);
    cudaMalloc(&d_ord, (size_t)N * C * 4);
    cudaMalloc(&d_ord_d, (size_t)N * C * 4);
    cudaMalloc(&d_removed, (size_t)N * C);
    cudaMalloc(&d_changed, N);
    cudaMalloc(&d_touched, N);
    cudaMalloc(&d_rev_off, (N + 1) * 4ull);
    cudaMalloc(&d_rev_cur, N * 4ull);
    cudaMalloc(&d_cand_off, (N + 1) * 4ull);
    cudaMalloc(&d_touched_ids, N * 4ull);
    cudaMalloc(&d_all_ids, N * 4ull);
    cudaMalloc(&d_selected, 4);
    cudaMemcpy(d_offsets, h_offsets, (N + 1) * 4ull, cudaMemcpyHostToDevice);
    cudaMemcpy(d_labels, h_labels, T * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(d_starts, h_starts, std::max(1u, num_labels) * 4ull, cudaMemcpyHostToDevice);
    cudaMemcpy(d_lpo, lpo.data(), lpo.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(d_lp, lp.data(), lp.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(d_ga, h_graph_in, (size_t)N * R * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(d_da, h_degree_in, N * 4ull, cudaMemcpyHostToDevice);
    canonical_make_task_rows<<<(N + 255) / 256, 256>>>(N, d_offsets, d_task_rows);
    canonical_init_ids<<<(N + 255) / 256, 256>>>(N, d_all_ids);
    const size_t fsh = (size_t)warps_per_block * per_label_pool * 9, osh = (size_t)warps_per_block * ordinary_pool * 9;
#define LAUNCH_BY_DIM(MACRO) \
    if (dim == 96) MACRO(96); else if (dim == 128) MACRO(128); else if (dim == 282) MACRO(282); else MACRO(0)
#define TASK(CD) canonical_filtered_task_search<CD, SearchT><<<(T + warps_per_block - 1) / warps_per_block, threads, \
        fsh>>>(d_data, N, dim, R, (uint32_t)T, per_label_pool, per_label_keep, STEPS, nullptr, d_task_rows, d_labels,  \
        d_starts, num_labels, d_lpo, d_lp, 16u, universal, d_offsets, d_labels, d_ga, d_da, d_task_c, d_task_d, 0u, 0u)
    if (T)
        LAUNCH_BY_DIM(TASK);
#define ORD(CD) canonical_ordinary_search<CD, SearchT><<<(N + warps_per_block - 1) / warps_per_block, threads, osh>>>( \
        d_data, N, dim, R, ordinary_pool, ordinary_keep, C, STEPS, global_start, nullptr, N, d_ga, d_da, d_offsets,     \
        d_labels, d_starts, num_labels, d_lpo, d_lp, 64u, d_work, d_work_d, 0u, 0u)
    LAUNCH_BY_DIM(ORD);
    cudaDeviceSynchronize();
    cudaMemcpy(d_ord, d_work, (size_t)N * C * 4, cudaMemcpyDeviceToDevice);
    cudaMemcpy(d_ord_d, d_work_d, (size_t)N * C * 4, cudaMemcpyDeviceToDevice);
    canonical_merge_candidates<<<N, 32>>>(N, R, C, per_label_keep, ordinary_keep, d_offsets, d_labels, d_lpo, d_lp,
                                          nullptr, N, d_ga, d_da, d_task_c, d_task_d, d_work, d_work_d, d_work,
                                          d_work_d, d_work_deg, 0u, 8u, 0u);
#define WD(CD) canonical_compute_work_distances<CD, SearchT><<<N, 32>>>(d_data, N, dim, C, d_work, nullptr, N, \
        d_work_deg, d_work_d)
    LAUNCH_BY_DIM(WD);
    canonical_exact_prune<SearchT><<<N, 32>>>(d_data, N, dim, R, C, alpha, d_offsets, d_labels, nullptr, N, d_ga,
                                              d_da, d_work, d_work_deg, d_work_d, d_removed, 0u, 0u, d_gb, nullptr,
                                              d_db, d_changed);
    cudaDeviceSynchronize();
    if (T)
    {
        cudaMemcpy(task_ids, d_task_c, T * per_label_keep * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(task_d, d_task_d, T * per_label_keep * 4, cudaMemcpyDeviceToHost);
    }
    cudaMemcpy2D(ord_ids, ordinary_keep * 4ull, d_ord, C * 4ull, ordinary_keep * 4ull, N, cudaMemcpyDeviceToHost);
    cudaMemcpy2D(ord_d, ordinary_keep * 4ull, d_ord_d, C * 4ull, ordinary_keep * 4ull, N, cudaMemcpyDeviceToHost);
    cudaMemcpy(work_ids, d_work, (size_t)N * C * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(work_d, d_work_d, (size_t)N * C * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(work_deg, d_work_deg, N * 4ull, cudaMemcpyDeviceToHost);
    cudaMemcpy(fwd_graph, d_gb, (size_t)N * R * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(fwd_deg, d_db, N * 4ull, cudaMemcpyDeviceToHost);
    // exact CSR reverse repair
    void *scan_tmp = nullptr, *sel_tmp = nullptr;
    size_t scan_bytes = 0, sel_bytes = 0;
    cub::DeviceScan::InclusiveSum(nullptr, scan_bytes, d_rev_off, d_rev_off, N + 1);
    cub::DeviceSelect::Flagged(nullptr, sel_bytes, d_all_ids, d_touched, d_touched_ids, d_selected, N);
    cudaMalloc(&scan_tmp, scan_bytes);
    cudaMalloc(&sel_tmp, sel_bytes);
    cudaMemset(d_touched, 0, N);
    cudaMemset(d_rev_off, 0, (N + 1) * 4ull);
    canonical_reverse_count<<<(N + 255) / 256, 256>>>(N, R, d_gb, d_db, nullptr, N, d_offsets, d_labels, universal,
                                                      d_rev_off);
    cub::DeviceScan::InclusiveSum(scan_tmp, scan_bytes, d_rev_off, d_rev_off, N + 1);
    uint32_t proposals = 0;
    cudaMemcpy(&proposals, d_rev_off + N, 4, cudaMemcpyDeviceToHost);
    cudaMalloc(&d_rev_ids, std::max(1u, proposals) * 4ull);
    cudaMemcpy(d_rev_cur, d_rev_off, N * 4ull, cudaMemcpyDeviceToDevice);
    canonical_reverse_fill<<<(N + 255) / 256, 256>>>(N, R, d_gb, d_db, d_rev_cur, d_rev_ids, nullptr, N, d_offsets,
                                                     d_labels, universal);
    cudaMemset(d_cand_off, 0, (N + 1) * 4ull);
    canonical_reverse_candidate_count<<<(N + 255) / 256, 256>>>(N, R, d_gb, d_db, d_rev_off, d_rev_ids, d_cand_off,
                                                                d_touched);
    cub::DeviceScan::InclusiveSum(scan_tmp, scan_bytes, d_cand_off, d_cand_off, N + 1);
    canonical_reverse_candidate_fill<<<(N + 255) / 256, 256>>>(N, R, d_gb, d_db, d_rev_off, d_rev_ids, d_cand_off,
                                                               d_work, nullptr, d_work_d);
    cub::DeviceSelect::Flagged(sel_tmp, sel_bytes, d_all_ids, d_touched, d_touched_ids, d_selected, N);
    uint32_t touched = 0;
    cudaMemcpy(&touched, d_selected, 4, cudaMemcpyDeviceToHost);
    if (touched)
    {
        canonical_csr_candidate_distances<SearchT><<<touched, 32>>>(d_data, N, dim, d_cand_off, d_touched_ids,
                                                                    touched, d_work, d_work_d);
        canonical_exact_prune_csr<SearchT><<<touched, 32>>>(d_data, N, dim, R, alpha, d_offsets, d_labels,
                                                            d_touched_ids, touched, d_cand_off, d_work, d_work_d,
                                                            d_removed, d_ga, d_da, d_gb, d_db, d_changed);
    }
    cudaError_t err = cudaDeviceSynchronize();
    cudaMemcpy(graph_out, d_gb, (size_t)N * R * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(deg_out, d_db, N * 4ull, cudaMemcpyDeviceToHost);
    void *bufs[] = {d_offsets, d_labels, d_starts, d_lpo, d_lp, d_task_rows, d_ga, d_da, d_gb, d_db, d_task_c,
                    d_task_d, d_work, d_work_d, d_work_deg, d_ord, d_ord_d, d_removed, d_changed, d_touched,
                    d_rev_off, d_rev_cur, d_rev_ids, d_cand_off, d_touched_ids, d_all_ids, d_selected, scan_tmp,
                    sel_tmp};
    for (void *b : bufs)
        cudaFree(b);
    return err == cudaSuccess ? 0 : -2;
}
} // namespace

extern "C" int ref_filtered_round_stages(int is_u8, const void *h_data, uint32_t N, uint32_t dim, uint32_t R,
                                         uint32_t L, uint32_t FL, uint32_t C, uint32_t STEPS, float alpha,
                                         const uint32_t *offsets, const uint32_t *labels, uint32_t total_labels,
                                         const uint32_t *starts, uint32_t num_labels, uint32_t universal,
                                         uint32_t global_start, const uint32_t *graph_in, const uint32_t *degree_in,
                                         uint32_t *task_ids, float *task_d, uint32_t *ord_ids, float *ord_d,
                                         uint32_t *work_ids, float *work_d, uint32_t *work_deg, uint32_t *fwd_graph,
                                         uint32_t *fwd_deg, uint32_t *graph_out, uint32_t *deg_out)
{
    const size_t elems = (size_t)N * dim;
    int rc;
    if (is_u8)
    {
        uint8_t *d = nullptr;
        cudaMalloc(&d, elems);
        cudaMemcpy(d, h_data, elems, cudaMemcpyHostToDevice);
        rc = stage_round<uint8_t>(d, N, dim, R, L, FL, C, STEPS, alpha, offsets, labels, total_labels, starts,
                                  num_labels, universal, global_start, graph_in, degree_in, task_ids, task_d,
                                  ord_ids, ord_d, work_ids, work_d, work_deg, fwd_graph, fwd_deg, graph_out,
                                  deg_out);
        cudaFree(d);
    }
    else
    {
        float *f = nullptr;
        __half *h = nullptr;
        cudaMalloc(&f, elems * 4);
        cudaMalloc(&h, elems * 2);
        cudaMemcpy(f, h_data, elems * 4, cudaMemcpyHostToDevice);
        canonical_convert_float_to_half<<<(elems + 255) / 256, 256>>>(f, h, elems);
        rc = stage_round<__half>(h, N, dim, R, L, FL, C, STEPS, alpha, offsets, labels, total_labels, starts,
                                 num_labels, universal, global_start, graph_in, degree_in, task_ids, task_d,
                                 ord_ids, ord_d, work_ids, work_d, work_deg, fwd_graph, fwd_deg, graph_out,
                                 deg_out);
        cudaFree(f);
        cudaFree(h);
    }
    return rc;
}

// The reference's deterministic random initial graph (:716-744).
extern "C" int ref_filtered_random_graph(uint32_t N, uint32_t R, uint32_t initial_degree, uint32_t seed,
                                         uint32_t *graph, uint32_t *degrees)
{
    uint32_t *dg = nullptr, *dd = nullptr;
    cudaMalloc(&dg, (size_t)N * R * 4);
    cudaMalloc(&dd, (size_t)N * 4);
    filtered_deterministic_random_graph_kernel<<<(N + 255) / 256, 256>>>(dg, dd, N, R, initial_degree, seed);
    cudaError_t err = cudaDeviceSynchronize();
    cudaMemcpy(graph, dg, (size_t)N * R * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(degrees, dd, (size_t)N * 4, cudaMemcpyDeviceToHost);
    cudaFree(dg);
    cudaFree(dd);
    return err == cudaSuccess ? 0 : -2;
}
