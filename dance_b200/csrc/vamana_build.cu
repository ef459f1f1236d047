// vamana_build.cu -- host orchestration and C ABI of libdance_b200.so.
//
// Replaces the round driver gpu_vamana_build_impl of the reference
// (src/gpu_vamana_vnew2.cu:2170-2855) and its exported entry points
// (:2857-2917, src/gpu_vamana_vnew2_handoff.cu:110-151,
// src/gpu_vamana_uint8.cu:3093-3120).  Differences in the plumbing, not the
// algorithm: all device memory is allocated once per build (or reused from a
// DanceWorkspace), every stage is launched on one stream with no host
// synchronisation inside the round loop (the reference syncs after every
// kernel and reads the reverse-edge count back each round), and the reverse
// CSR buffer is sized for its upper bound N*R up front.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/dance_b200.h"
#include "../../include/gpu_vamana_builder.h"
#include "../../include/gpu_vamana_config.h"
#include "host_common.cuh"

namespace dance
{
thread_local char g_err[512] = "";
std::atomic<uint64_t> g_launches{0};
thread_local DanceBuildReport g_report;

int build_resident_impl(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                        uint32_t L, uint32_t C, uint32_t STEPS, const DanceVamanaParams &prm, DanceWorkspace &ws,
                        uint32_t *graph_out, uint32_t *degree_out, float *dists_out, uint32_t *medoid_out,
                        cudaStream_t s, StageTimes *times, uint64_t *counters_out)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    if (R == 0 || L == 0 || C == 0 || STEPS == 0)
        return fail(-1, "invalid parameters: R=%u L=%u C=%u STEPS=%u", R, L, C, STEPS);
    if (C < R)
        return fail(-1, "invalid parameters: C=%u must be >= R=%u", C, R);
    if (C > 1024 || L > kMaxL || R > 1024)
        return fail(-1, "R and C are limited to 1024 and L to %d in this build", kMaxL);
    if (STEPS > L)
    {
        fprintf(stderr, "[dance_b200] STEPS=%u is larger than L=%u, clamp STEPS to L.\n", STEPS, L);
        STEPS = L;
    }
    if (prm.iters == 0)
        return fail(-1, "iters must be >= 1");
    if (prm.visited_log2 < 8 || prm.visited_log2 > 16)
        return fail(-1, "visited_log2 must be in [8, 16]");
    if (ws.N < N || ws.R != R || ws.C != C || ws.S < STEPS)
        return fail(-1, "workspace sized for N=%u R=%u C=%u S=%u cannot hold N=%u R=%u C=%u S=%u", ws.N, ws.R, ws.C,
                    ws.S, N, R, C, STEPS);
    const StoreView st = make_view(d_data, stride, N, dim, dtype);
    uint32_t *cur_ids = graph_out ? graph_out : ws.cur_ids.as<uint32_t>();
    float *cur_dists = dists_out ? dists_out : ws.cur_dists.as<float>();
    uint32_t *degree = degree_out ? degree_out : ws.degree.as<uint32_t>();
    DANCE_CUDA(cudaMemsetAsync(ws.counters.p, 0, 64, s));

    // Stage boundaries are recorded as events on the build stream and resolved
    // after the final synchronisation, so timing adds no host syncs.
    const int nev = 2 + 4 * (int)prm.iters;
    std::vector<cudaEvent_t> ev((size_t)nev + prm.iters, nullptr); // + one per search-kernel end
    struct EvGuard
    {
        std::vector<cudaEvent_t> &e;
        ~EvGuard()
        {
            for (auto x : e)
                if (x)
                    cudaEventDestroy(x);
        }
    } guard{ev};
    if (times)
        for (auto &e : ev)
            DANCE_CUDA(cudaEventCreate(&e));
    auto mark = [&](int i) -> cudaError_t { return times ? cudaEventRecord(ev[(size_t)i], s) : cudaSuccess; };

    DANCE_CUDA(mark(0));
    const uint32_t nc = std::min<uint32_t>(prm.medoid_candidates, std::min<uint32_t>(N, 4096u));
    const uint32_t ns = std::min<uint32_t>(prm.medoid_samples, N);
    uint32_t *d_medoid = ws.medoid.as<uint32_t>();
    if (nc > 0 && ns > 0)
    {
        rc = dispatch<LaunchMedoid>(dtype, st.nchunks, st, nc, ns, ws.med_scores.as<float>(),
                                    ws.med_cand.as<uint32_t>(), d_medoid, s);
        if (rc)
            return rc;
    }
    else
        DANCE_CUDA(cudaMemsetAsync(d_medoid, 0, 4, s));
    DANCE_CUDA(mark(1));
    rc = dispatch<LaunchInit>(dtype, st.nchunks, st, R, cur_ids, cur_dists, degree, 0u, N, 0u, s);
    if (rc)
        return rc;
    const uint32_t mask_vertices = replay_mask_vertices(dtype, st.nchunks, R, ws.S, C, N);
    if (mask_vertices)
        DANCE_CUDA(ws.replay_masks.ensure(replay_mask_bytes(mask_vertices, ws.S)));

    for (uint32_t it = 0; it < prm.iters; ++it)
    {
        const float alpha = (it + 1 >= prm.iters) ? prm.alpha : 1.0f;
        const uint32_t steps = steps_for_round(it, STEPS, prm);
        DANCE_CUDA(mark(2 + 4 * (int)it));
        SearchParams sp{};
        sp.st = st;
        sp.R = R;
        sp.L = L;
        sp.Lcap = lcap_of(L);
        sp.steps = steps;
        sp.seeds = std::min<uint32_t>(prm.init_random_seeds, 31u);
        sp.log2h = prm.visited_log2;
        sp.entry = 0;
        sp.entry_ptr = d_medoid;
        sp.cur_ids = cur_ids;
        sp.cur_dists = cur_dists;
        sp.degree = degree;
        sp.exp_ids = ws.exp_ids.as<uint32_t>();
        sp.exp_dists = ws.exp_dists.as<float>();
        sp.exp_count = ws.exp_count.as<uint32_t>();
        sp.exp_stride = ws.S;
        sp.v0 = 0;
        sp.v1 = N;
        sp.counters = ws.counters.as<unsigned long long>();
        rc = dispatch<LaunchSearch>(dtype, st.nchunks, sp, s);
        if (rc)
            return rc;
        if (times)
            DANCE_CUDA(cudaEventRecord(ev[(size_t)nev + it], s));
        ReplayParams rp{};
        rp.st = st;
        rp.R = R;
        rp.C = C;
        rp.alpha = alpha;
        rp.cur_ids = cur_ids;
        rp.cur_dists = cur_dists;
        rp.degree = degree;
        rp.exp_ids = sp.exp_ids;
        rp.exp_dists = sp.exp_dists;
        rp.exp_count = sp.exp_count;
        rp.exp_stride = ws.S;
        rp.work_ids = ws.work_ids.as<uint32_t>();
        rp.work_dists = ws.work_dists.as<float>();
        rp.work_deg = ws.work_deg.as<uint32_t>();
        rp.v0 = 0;
        rp.v1 = N;
        rp.row_bytes = st.nchunks * 16;
        rp.cache_rows = R + ws.S;
        rp.counters = sp.counters;
        rp.masks = mask_vertices ? ws.replay_masks.as<uint32_t>() : nullptr;
        rp.mask_vertices = mask_vertices;
        rc = dispatch<LaunchReplay>(dtype, st.nchunks, rp, s);
        if (rc)
            return rc;
        DANCE_CUDA(mark(3 + 4 * (int)it));
        rc = reverse_merge_impl(dtype, st, R, C, prm, ws, rp.work_ids, C, rp.work_deg, 0, N, rp.work_ids,
                                rp.work_dists, rp.work_deg, 0, N, s);
        if (rc)
            return rc;
        DANCE_CUDA(mark(4 + 4 * (int)it));
        PruneParams pp{};
        pp.st = st;
        pp.R = R;
        pp.C = C;
        pp.alpha = alpha;
        pp.min_degree = (it + 1 == prm.iters) ? prm.final_min_degree : 0u;
        pp.work_ids = rp.work_ids;
        pp.work_dists = rp.work_dists;
        pp.work_deg = rp.work_deg;
        pp.cur_ids = cur_ids;
        pp.cur_dists = cur_dists;
        pp.degree = degree;
        pp.v0 = 0;
        pp.v1 = N;
        pp.row_bytes = st.nchunks * 16;
        pp.counters = sp.counters;
        rc = dispatch<LaunchPrune>(dtype, st.nchunks, pp, s);
        if (rc)
            return rc;
        DANCE_CUDA(mark(5 + 4 * (int)it));

    }
    if (medoid_out)
        DANCE_CUDA(cudaMemcpyAsync(medoid_out, d_medoid, 4, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    if ((rc = replay_umma_status()))
        return rc;
    if (times)
    {
        float a = 0;
        cudaEventElapsedTime(&a, ev[0], ev[1]);
        times->medoid = a * 1e-3;
            times->search = times->replay = times->reverse = times->prune = times->search_kernel = 0;
        for (uint32_t it = 0; it < prm.iters; ++it)
        {
            const int b = 2 + 4 * (int)it;
            float t0 = 0, t1 = 0, t2 = 0, tk = 0;
            cudaEventElapsedTime(&t0, ev[b], ev[b + 1]);
            cudaEventElapsedTime(&t1, ev[b + 1], ev[b + 2]);
            cudaEventElapsedTime(&t2, ev[b + 2], ev[b + 3]);
            cudaEventElapsedTime(&tk, ev[b], ev[(size_t)nev + it]);
            times->search += t0 * 1e-3;
            times->search_kernel += tk * 1e-3;
            times->replay += (t0 - tk) * 1e-3;
            times->reverse += t1 * 1e-3;
            times->prune += t2 * 1e-3;
        }
        cudaEventElapsedTime(&a, ev[0], ev[(size_t)nev - 1]);
        times->total = a * 1e-3;
    }
    if (counters_out)
        DANCE_CUDA(cudaMemcpy(counters_out, ws.counters.p, 64, cudaMemcpyDeviceToHost));
    return 0;
}

} // namespace dance

// ====================================================================== additive C ABI

extern "C" {

void dance_vamana_default_params(DanceVamanaParams *p)
{
    if (!p)
        return;
    std::memset(p, 0, sizeof(*p));
    p->iters = VAMANA_ITERS;
    p->alpha = VAMANA_ALPHA;
    p->init_random_seeds = INIT_RANDOM_SEEDS;
    p->final_min_degree = ENABLE_FINAL_DEGREE_FILL ? FINAL_MIN_DEGREE : 0;
    p->medoid_candidates = MEDOID_NUM_CANDIDATES;
    p->medoid_samples = MEDOID_NUM_SAMPLES;
    p->coarse_warmup_iters = ENABLE_COARSE_TO_FINE_STEPS ? COARSE_WARMUP_ITERS : 0;
    p->warmup_expand_steps = WARMUP_EXPAND_STEPS;
    p->reverse_heavy_cap = ENABLE_REVERSE_HEAVY_CAP;
    p->reverse_heavy_threshold = REVERSE_HEAVY_THRESHOLD;
    p->reverse_heavy_sample = REVERSE_HEAVY_SAMPLE;
    p->visited_log2 = DANCE_VISITED_LOG2;
}

const char *dance_last_error(void) { return dance::g_err; }

int dance_last_build_report(DanceBuildReport *report)
{
    if (!report)
        return fail(-1, "null report");
    *report = g_report;
    return 0;
}

uint64_t dance_kernel_launch_count(void) { return dance::g_launches.load(); }

int dance_workspace_create(uint32_t num_points, uint32_t R, uint32_t L, uint32_t C, uint32_t STEPS,
                           DanceWorkspace **out)
{
    if (!out || num_points == 0 || R == 0 || L == 0 || C == 0 || STEPS == 0 || C < R)
        return fail(-1, "invalid workspace shape");
    DanceWorkspace *ws = new DanceWorkspace();
    cudaGetDevice(&ws->device);
    const uint32_t S = std::min(STEPS, L);
    int rc = ws->reserve(num_points, R, L, C, S);
    if (rc)
    {
        delete ws;
        return rc;
    }
    *out = ws;
    return 0;
}

void dance_workspace_destroy(DanceWorkspace *ws) { delete ws; }

int dance_vamana_build_resident(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points,
                                uint32_t dim, uint32_t R, uint32_t L, uint32_t C, uint32_t STEPS,
                                const DanceVamanaParams *params, DanceWorkspace *ws, uint32_t *d_graph,
                                uint32_t *d_degree, float *d_graph_dists, uint32_t *medoid_out, void *stream)
{
    DanceVamanaParams prm;
    if (params)
        prm = *params;
    else
        dance_vamana_default_params(&prm);
    DanceWorkspace *own = nullptr;
    if (!ws)
    {
        int rc = dance_workspace_create(num_points, R, L, C, STEPS, &own);
        if (rc)
            return rc;
        ws = own;
    }
    StageTimes tm;
    uint64_t ctr[8] = {0};
    int rc = build_resident_impl(dtype, d_data, row_stride_bytes, num_points, dim, R, L, C, STEPS, prm, *ws, d_graph,
                                 d_degree, d_graph_dists, medoid_out, as_stream(stream), &tm, ctr);
    if (!rc)
    {
        DanceBuildReport &r = g_report;
        std::memset(&r, 0, sizeof(r));
        r.medoid_seconds = tm.medoid;
        r.search_seconds = tm.search;
        r.search_kernel_seconds = tm.search_kernel;
        r.replay_seconds = tm.replay;
        r.reverse_seconds = tm.reverse;
        r.prune_seconds = tm.prune;
        r.total_seconds = tm.total;
        r.search_evals = ctr[0];
        r.expansions = ctr[1];
        r.replay_pairs = ctr[2];
        r.reverse_evals = ctr[3];
        r.prune_pairs = ctr[4];
    }
    delete own;
    return rc;
}

int dance_stage_medoid(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t nc,
                       uint32_t ns, float *d_scores, uint32_t *d_cand, uint32_t *d_medoid, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    nc = std::min(nc, N);
    ns = std::min(ns, N);
    if (nc == 0 || ns == 0 || nc > 4096)
        return fail(-1, "medoid needs 1..4096 candidates and >= 1 sample");
    StoreView st = make_view(d_data, stride, N, dim, dtype);
    return dispatch<LaunchMedoid>(dtype, st.nchunks, st, nc, ns, d_scores, d_cand, d_medoid, as_stream(stream));
}

int dance_stage_init(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                     uint32_t *d_cur_ids, float *d_cur_dists, uint32_t *d_degree, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    StoreView st = make_view(d_data, stride, N, dim, dtype);
    return dispatch<LaunchInit>(dtype, st.nchunks, st, R, d_cur_ids, d_cur_dists, d_degree, 0u, N, 0u,
                                as_stream(stream));
}

int dance_stage_search(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                       uint32_t L, uint32_t steps, uint32_t entry, uint32_t seeds, uint32_t visited_log2,
                       const uint32_t *d_cur_ids, const float *d_cur_dists, const uint32_t *d_degree,
                       uint32_t *d_exp_ids, float *d_exp_dists, uint32_t *d_exp_count, uint32_t exp_stride,
                       void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    steps = std::min(steps, L);
    if (steps > exp_stride || L == 0 || R == 0 || L > (uint32_t)kMaxL || visited_log2 < 8 || visited_log2 > 16)
        return fail(-1, "invalid search stage arguments");
    SearchParams sp{};
    sp.st = make_view(d_data, stride, N, dim, dtype);
    sp.R = R;
    sp.L = L;
    sp.Lcap = lcap_of(L);
    sp.steps = steps;
    sp.seeds = std::min<uint32_t>(seeds, 31u);
    sp.log2h = visited_log2;
    sp.entry = entry;
    sp.entry_ptr = nullptr;
    sp.cur_ids = d_cur_ids;
    sp.cur_dists = d_cur_dists;
    sp.degree = d_degree;
    sp.exp_ids = d_exp_ids;
    sp.exp_dists = d_exp_dists;
    sp.exp_count = d_exp_count;
    sp.exp_stride = exp_stride;
    sp.v0 = 0;
    sp.v1 = N;
    sp.counters = nullptr;
    return dispatch<LaunchSearch>(dtype, sp.st.nchunks, sp, as_stream(stream));
}

int dance_stage_replay(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                       uint32_t C, float alpha, const uint32_t *d_cur_ids, const float *d_cur_dists,
                       const uint32_t *d_degree, const uint32_t *d_exp_ids, const float *d_exp_dists,
                       const uint32_t *d_exp_count, uint32_t exp_stride, uint32_t *d_work_ids, float *d_work_dists,
                       uint32_t *d_work_deg, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    if (C < R || C > 1024)
        return fail(-1, "invalid replay stage arguments");
    ReplayParams rp{};
    rp.st = make_view(d_data, stride, N, dim, dtype);
    rp.R = R;
    rp.C = C;
    rp.alpha = alpha;
    rp.cur_ids = d_cur_ids;
    rp.cur_dists = d_cur_dists;
    rp.degree = d_degree;
    rp.exp_ids = d_exp_ids;
    rp.exp_dists = d_exp_dists;
    rp.exp_count = d_exp_count;
    rp.exp_stride = exp_stride;
    rp.work_ids = d_work_ids;
    rp.work_dists = d_work_dists;
    rp.work_deg = d_work_deg;
    rp.v0 = 0;
    rp.v1 = N;
    rp.row_bytes = rp.st.nchunks * 16;
    rp.cache_rows = R + exp_stride;
    rp.counters = nullptr;
    DevBuf masks; // freed (device-synchronising) on return: this stage entry point serves the parity tests
    rp.mask_vertices = replay_mask_vertices(dtype, rp.st.nchunks, R, exp_stride, C, N);
    if (rp.mask_vertices)
    {
        DANCE_CUDA(masks.ensure(replay_mask_bytes(rp.mask_vertices, exp_stride)));
        rp.masks = masks.as<uint32_t>();
    }
    if ((rc = dispatch<LaunchReplay>(dtype, rp.st.nchunks, rp, as_stream(stream))))
        return rc;
    if (rp.mask_vertices)
    {
        DANCE_CUDA(cudaStreamSynchronize(as_stream(stream)));
        return replay_umma_status();
    }
    return 0;
}

int dance_stage_reverse_merge(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                              uint32_t C, const DanceVamanaParams *params, DanceWorkspace *ws, uint32_t *d_work_ids,
                              float *d_work_dists, uint32_t *d_work_deg, uint64_t *reverse_edges_out, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    DanceVamanaParams prm;
    if (params)
        prm = *params;
    else
        dance_vamana_default_params(&prm);
    DanceWorkspace *own = nullptr;
    if (!ws)
    {
        rc = dance_workspace_create(N, R, R, C, 1, &own);
        if (rc)
            return rc;
        ws = own;
    }
    if (ws->N < N || ws->R != R || ws->C != C)
    {
        delete own;
        return fail(-1, "workspace shape mismatch");
    }
    cudaStream_t s = as_stream(stream);
    StoreView st = make_view(d_data, stride, N, dim, dtype);
    rc = reverse_merge_impl(dtype, st, R, C, prm, *ws, d_work_ids, C, d_work_deg, 0, N, d_work_ids, d_work_dists,
                            d_work_deg, 0, N, s);
    if (!rc && reverse_edges_out)
    {
        uint32_t tot = 0;
        cudaError_t e = cudaMemcpyAsync(&tot, ws->rev_off.as<uint32_t>() + N, 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess)
            e = cudaStreamSynchronize(s);
        if (e != cudaSuccess)
            rc = fail(-2, "CUDA error %s", cudaGetErrorString(e));
        *reverse_edges_out = tot;
    }
    else if (!rc)
    {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess)
            rc = fail(-2, "CUDA error %s", cudaGetErrorString(e));
    }
    delete own;
    return rc;
}

int dance_stage_prune(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                      uint32_t C, float alpha, uint32_t min_degree, const uint32_t *d_work_ids,
                      const float *d_work_dists, const uint32_t *d_work_deg, uint32_t *d_cur_ids, float *d_cur_dists,
                      uint32_t *d_degree, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    if (C < R || C > 1024)
        return fail(-1, "invalid prune stage arguments");
    PruneParams pp{};
    pp.st = make_view(d_data, stride, N, dim, dtype);
    pp.R = R;
    pp.C = C;
    pp.alpha = alpha;
    pp.min_degree = min_degree;
    pp.work_ids = d_work_ids;
    pp.work_dists = d_work_dists;
    pp.work_deg = d_work_deg;
    pp.cur_ids = d_cur_ids;
    pp.cur_dists = d_cur_dists;
    pp.degree = d_degree;
    pp.v0 = 0;
    pp.v1 = N;
    pp.row_bytes = pp.st.nchunks * 16;
    pp.counters = nullptr;
    return dispatch<LaunchPrune>(dtype, pp.st.nchunks, pp, as_stream(stream));
}

int dance_search_queries(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim,
                         const uint32_t *d_graph, uint32_t R, uint32_t start, const void *d_queries,
                         uint64_t query_stride, uint32_t nq, uint32_t L_search, uint32_t K, uint32_t visited_log2,
                         uint32_t *d_out_ids, float *d_out_dists, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    if (!d_graph || !d_queries || !d_out_ids || !d_out_dists || K == 0 || K > L_search || L_search > (uint32_t)kMaxL ||
        query_stride % 16 != 0 || visited_log2 < 8 || visited_log2 > 16)
        return fail(-1, "invalid query search arguments");
    QueryParams qp{};
    qp.st = make_view(d_data, stride, N, dim, dtype);
    qp.queries = reinterpret_cast<const uint8_t *>(d_queries);
    qp.qstride = query_stride;
    qp.nq = nq;
    qp.graph = d_graph;
    qp.R = R;
    qp.L = L_search;
    qp.Lcap = lcap_of(L_search);
    qp.K = K;
    qp.log2h = visited_log2;
    qp.start = start;
    qp.out_ids = d_out_ids;
    qp.out_dists = d_out_dists;
    if (nq == 0)
        return 0;
    return dispatch<LaunchQuery>(dtype, qp.st.nchunks, qp, as_stream(stream));
}

int dance_search_queries_filtered(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim,
                                  const uint32_t *d_graph, uint32_t R, const uint32_t *d_label_offsets,
                                  const uint32_t *d_labels, const uint32_t *d_query_labels,
                                  const uint32_t *d_query_starts, const void *d_queries, uint64_t query_stride,
                                  uint32_t nq, uint32_t L_search, uint32_t K, uint32_t visited_log2,
                                  uint32_t *d_out_ids, float *d_out_dists, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    if (!d_graph || !d_queries || !d_out_ids || !d_out_dists || !d_label_offsets || !d_labels || !d_query_labels ||
        !d_query_starts || K == 0 || K > L_search || L_search > (uint32_t)kMaxL || query_stride % 16 != 0 ||
        visited_log2 < 8 || visited_log2 > 16)
        return fail(-1, "invalid filtered query search arguments");
    QueryParams qp{};
    qp.st = make_view(d_data, stride, N, dim, dtype);
    qp.queries = reinterpret_cast<const uint8_t *>(d_queries);
    qp.qstride = query_stride;
    qp.nq = nq;
    qp.graph = d_graph;
    qp.R = R;
    qp.L = L_search;
    qp.Lcap = lcap_of(L_search);
    qp.K = K;
    qp.log2h = visited_log2;
    qp.start = kInvalid;
    qp.out_ids = d_out_ids;
    qp.out_dists = d_out_dists;
    qp.label_off = d_label_offsets;
    qp.labels = d_labels;
    qp.query_label = d_query_labels;
    qp.query_start = d_query_starts;
    if (nq == 0)
        return 0;
    return dispatch<LaunchQuery>(dtype, qp.st.nchunks, qp, as_stream(stream));
}

} // extern "C"

// ====================================================================== reference C ABI
namespace
{
uint32_t g_last_medoid = 0;
GPUVamanaStats g_last_stats;

double now_sec()
{
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

__global__ void f32_to_f16_rows(const float *src, uint32_t dim, __half *dst, uint64_t dst_stride_elems, uint64_t n)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint64_t r = i / dim, c = i % dim;
        dst[r * dst_stride_elems + c] = __float2half_rn(src[i]);
    }
}

// Host entry shared by the reference-compatible symbols.  `keep` != null
// turns it into the device hand-off variant.
int host_build(int in_dtype, const void *h_data, uint32_t N, uint32_t dim, uint32_t R, uint32_t L, uint32_t C,
               uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree, void **keep_data, uint32_t **keep_graph,
               uint32_t **keep_degree)
{
    std::memset(&g_last_stats, 0, sizeof(g_last_stats));
    const double t0 = now_sec();
    const bool handoff = keep_data != nullptr;
    if (!h_data || (!handoff && (!h_graph || !h_degree)))
        return fail(-1, "[gpu_vamana_build] null input pointer.");
    if (N == 0 || dim == 0 || R == 0 || L == 0 || C == 0 || STEPS == 0)
        return fail(-1, "[gpu_vamana_build] invalid parameters: N=%u dim=%u R=%u L=%u C=%u STEPS=%u", N, dim, R, L,
                    C, STEPS);
    if (C < R)
        return fail(-1, "[gpu_vamana_build] invalid parameters: C=%u must be >= R=%u", C, R);
    if (STEPS > L)
    {
        fprintf(stderr, "[gpu_vamana_build] STEPS=%u is larger than L=%u, clamp STEPS to L.\n", STEPS, L);
        STEPS = L;
    }
    const int store_dtype = (in_dtype == kF32 && float16_build_enabled()) ? kF16 : in_dtype;
    const int in_es = elem_size(in_dtype);
    const int st_es = elem_size(store_dtype);
    const uint64_t in_row = (uint64_t)dim * in_es;
    const uint64_t stride = ((uint64_t)dim * st_es + 15u) & ~15ull;
    DanceVamanaParams prm;
    dance_vamana_default_params(&prm);

    DevBuf input, store, graph, degree;
    cudaStream_t s = 0;
    const double th0 = now_sec();
    DANCE_CUDA(input.ensure((uint64_t)N * in_row));
    DANCE_CUDA(cudaMemcpy(input.p, h_data, (uint64_t)N * in_row, cudaMemcpyHostToDevice));
    const void *d_store = input.p;
    if (store_dtype != in_dtype)
    {
        DANCE_CUDA(store.ensure((uint64_t)N * stride));
        DANCE_CUDA(cudaMemsetAsync(store.p, 0, (uint64_t)N * stride, s));
        const uint64_t n = (uint64_t)N * dim;
        const int grid = (int)std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count() * 32);
        f32_to_f16_rows<<<grid, 256, 0, s>>>(input.as<float>(), dim, store.as<__half>(), stride / 2, n);
        DANCE_LAUNCHED();
        d_store = store.p;
    }
    else if (stride != in_row)
    {
        DANCE_CUDA(store.ensure((uint64_t)N * stride));
        DANCE_CUDA(cudaMemsetAsync(store.p, 0, (uint64_t)N * stride, s));
        DANCE_CUDA(cudaMemcpy2DAsync(store.p, stride, input.p, in_row, in_row, N, cudaMemcpyDeviceToDevice, s));
        d_store = store.p;
    }
    DANCE_CUDA(cudaStreamSynchronize(s));
    g_last_stats.h2d_seconds = now_sec() - th0;
    if (!handoff && d_store != input.p)
        input.release();

    DanceWorkspace ws;
    int rc = ws.reserve(N, R, L, C, STEPS);
    if (rc)
        return rc;
    DANCE_CUDA(graph.ensure((uint64_t)N * R * 4));
    DANCE_CUDA(degree.ensure((uint64_t)N * 4));
    StageTimes tm;
    uint64_t ctr[8] = {0};
    uint32_t medoid = 0;
    rc = build_resident_impl(store_dtype, d_store, stride, N, dim, R, L, C, STEPS, prm, ws, graph.as<uint32_t>(),
                             degree.as<uint32_t>(), nullptr, &medoid, s, &tm, ctr);
    if (rc)
        return rc;
    g_last_medoid = medoid;
    g_last_stats.medoid_seconds = tm.medoid;
    g_last_stats.search_online_insert_seconds = tm.search;
    g_last_stats.reverse_seconds = tm.reverse;
    g_last_stats.reverse_csr_seconds = tm.reverse;
    g_last_stats.final_prune_seconds = tm.prune;
    g_last_stats.distance_computations = ctr[0] + ctr[2] + ctr[3] + ctr[4];
    g_last_stats.online_insert_attempts = ctr[1];
    const double td0 = now_sec();
    if (handoff)
    {
        *keep_data = input.p;
        input.p = nullptr;
        *keep_graph = graph.as<uint32_t>();
        graph.p = nullptr;
        *keep_degree = degree.as<uint32_t>();
        degree.p = nullptr;
    }
    else
    {
        DANCE_CUDA(cudaMemcpy(h_graph, graph.p, (uint64_t)N * R * 4, cudaMemcpyDeviceToHost));
        DANCE_CUDA(cudaMemcpy(h_degree, degree.p, (uint64_t)N * 4, cudaMemcpyDeviceToHost));
    }
    g_last_stats.d2h_seconds = now_sec() - td0;
    g_last_stats.gpu_build_seconds = now_sec() - t0;
    return 0;
}
} // namespace

extern "C" {

int gpu_vamana_vnew2_build(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                           uint32_t C, uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree)
{
    // The reference returns -1 for every failure (invalid argument or CUDA error).
    return host_build(kU8, h_data, num_points, dim, R, L, C, STEPS, h_graph, h_degree, nullptr, nullptr, nullptr)
               ? -1
               : 0;
}

int gpu_vamana_vnew2_build_float(const float *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                                 uint32_t C, uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree)
{
    return host_build(kF32, h_data, num_points, dim, R, L, C, STEPS, h_graph, h_degree, nullptr, nullptr, nullptr)
               ? -1
               : 0;
}

int gpu_vamana_vnew2_build_device(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                                  uint32_t C, uint32_t STEPS, uint8_t **d_data, uint32_t **d_graph,
                                  uint32_t **d_degree)
{
    if (!d_data || !d_graph || !d_degree)
        return fail(-1, "[gpu_vamana_build] null output pointer.");
    void *dd = nullptr;
    int rc = host_build(kU8, h_data, num_points, dim, R, L, C, STEPS, nullptr, nullptr, &dd, d_graph, d_degree);
    if (!rc)
        *d_data = reinterpret_cast<uint8_t *>(dd);
    return rc ? -1 : 0;
}

int gpu_vamana_vnew2_build_device_float(const float *h_data, uint32_t num_points, uint32_t dim, uint32_t R,
                                        uint32_t L, uint32_t C, uint32_t STEPS, float **d_data, uint32_t **d_graph,
                                        uint32_t **d_degree)
{
    if (!d_data || !d_graph || !d_degree)
        return fail(-1, "[gpu_vamana_build] null output pointer.");
    void *dd = nullptr;
    int rc = host_build(kF32, h_data, num_points, dim, R, L, C, STEPS, nullptr, nullptr, &dd, d_graph, d_degree);
    if (!rc)
        *d_data = reinterpret_cast<float *>(dd);
    return rc ? -1 : 0;
}

// The legacy v8 entry points (reference src/gpu_vamana_uint8.cu) build with
// the vnew2 engine above: same rules and outputs format; the v8 file's own
// schedule (C-wide ping-pong graph buffers between rounds) is not reproduced.
int gpu_vamana_build(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L, uint32_t C,
                     uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree)
{
    return gpu_vamana_vnew2_build(h_data, num_points, dim, R, L, C, STEPS, h_graph, h_degree);
}

int gpu_vamana_build_float(const float *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                           uint32_t C, uint32_t STEPS, uint32_t *h_graph, uint32_t *h_degree)
{
    return gpu_vamana_vnew2_build_float(h_data, num_points, dim, R, L, C, STEPS, h_graph, h_degree);
}

uint32_t gpu_vamana_vnew2_get_last_medoid(void) { return g_last_medoid; }
void gpu_vamana_vnew2_get_last_stats(GPUVamanaStats *stats)
{
    if (stats)
        *stats = g_last_stats;
}
uint32_t gpu_vamana_get_last_medoid(void) { return g_last_medoid; }
void gpu_vamana_get_last_stats(GPUVamanaStats *stats)
{
    if (stats)
        *stats = g_last_stats;
}

} // extern "C"
