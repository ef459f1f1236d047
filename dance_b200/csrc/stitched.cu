// stitched.cu -- GPU-StitchedVamana: one Vamana graph per label, stitched
// into one global graph.
//
// Replaces the label loop of the reference app build_gpu_stitched
// (apps/utils/gpu_stitched_vamana_index.cpp:241-341).  The rules are the
// reference's: every label's points, in the label's point order, are built as
// an independent vnew2 graph (Rsmall, Lsmall, C, steps); the label medoid is
// the global id of the local medoid (local 0 when out of range); every point's
// row is the concatenation, over its labels in label order, of the first
// min(local degree, Rstitched) local neighbours mapped to global ids, where an
// invalid local id or a self loop is skipped and an id already in the row is
// not appended again (:316-341).
//
// The plumbing is B200-first.  The reference copies each label's vectors on
// the host, allocates, uploads, builds and downloads one label at a time
// through the host ABI.  Here the vectors go to the device once, a gather
// kernel lays every label's points out contiguously (label-major, fp16 when
// the float build is configured so), the labels are built largest first on
// several streams at once from per-stream workspaces (the per-label graphs
// are independent, so the order cannot change them), and the remap runs as
// one kernel over all points into a CSR graph.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include "../../include/dance_b200.h"
#include "comm.cuh"
#include "host_common.cuh"
#include "stitched_prune.cuh"

namespace dance
{
namespace
{

double wall()
{
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Row m of the label-major store is point points[m] of the source store.
// One warp per row; rows are padded with zeros to out_stride.  conv_f16
// converts float input to fp16 (round to nearest even, as the float entry
// points do when the fp16 build is on).
__global__ void gather_label_rows_kernel(const uint8_t *in, uint64_t in_stride, uint32_t row_bytes, int conv_f16,
                                         uint32_t dim, const uint32_t *points, uint64_t M, uint8_t *out,
                                         uint64_t out_stride)
{
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t m = blockIdx.x * (uint64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); m < M; m += warps)
    {
        const uint8_t *src = in + (uint64_t)points[m] * in_stride;
        uint8_t *dst = out + m * out_stride;
        if (conv_f16)
        {
            const float *f = reinterpret_cast<const float *>(src);
            __half *h = reinterpret_cast<__half *>(dst);
            for (uint64_t k = lane; k < out_stride / 2; k += 32)
                h[k] = k < dim ? __float2half_rn(f[k]) : __float2half_rn(0.0f);
        }
        else if ((in_stride & 3u) == 0)
        {
            const uint32_t *s4 = reinterpret_cast<const uint32_t *>(src);
            uint32_t *d4 = reinterpret_cast<uint32_t *>(dst);
            const uint32_t full = row_bytes / 4;
            for (uint64_t w = lane; w < out_stride / 4; w += 32)
            {
                uint32_t v = 0;
                if (w < full)
                    v = s4[w];
                else
                    for (int b = 0; b < 4; ++b)
                        if (4 * w + b < row_bytes)
                            v |= (uint32_t)src[4 * w + b] << (8 * b);
                d4[w] = v;
            }
        }
        else
        {
            for (uint64_t b = lane; b < out_stride; b += 32)
                dst[b] = b < row_bytes ? src[b] : 0;
        }
    }
}

struct RemapParams
{
    uint32_t N;
    const uint32_t *pm_off;     // N + 1: point -> membership CSR offsets
    const uint32_t *pm_list;    // memberships of each point, ascending (= label order)
    const uint32_t *mem_label;  // M: label of membership m
    const uint64_t *label_off;  // num_labels + 1
    const uint32_t *label_pts;  // M: global point of membership m
    const uint32_t *lgraph;     // M x r_small local graphs
    const uint32_t *ldeg;       // M
    uint32_t r_small, r_out;
    uint32_t *rows;             // scratch rows, point g at pm_off[g] * r_small
    uint32_t *row_size;         // N
    unsigned long long *counters; // [0] invalid local ids, [1] self loops, [2] duplicates
};

// One warp per point.  Candidates are taken 32 at a time in row order; a
// candidate is kept unless it equals an id already in the row or a kept-or-
// duplicate valid candidate of a lower lane, which is the reference's
// sequential "append if absent" (:330-338) done a warp at a time.
__global__ void __launch_bounds__(256) stitched_remap_kernel(RemapParams p)
{
    const int lane = threadIdx.x & 31;
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    unsigned long long n_inv = 0, n_self = 0, n_dup = 0;
    for (uint32_t g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < p.N; g += warps)
    {
        const uint32_t b0 = p.pm_off[g], b1 = p.pm_off[g + 1];
        uint32_t *row = p.rows + (uint64_t)b0 * p.r_small;
        uint32_t pos = 0;
        for (uint32_t b = b0; b < b1; ++b)
        {
            const uint32_t m = p.pm_list[b];
            const uint32_t l = p.mem_label[m];
            const uint64_t lo = p.label_off[l];
            const uint32_t nl = (uint32_t)(p.label_off[l + 1] - lo);
            const uint32_t deg = min(min(p.ldeg[m], p.r_out), p.r_small);
            for (uint32_t j0 = 0; j0 < deg; j0 += 32)
            {
                const uint32_t j = j0 + lane;
                uint32_t cand = kInvalid;
                if (j < deg)
                {
                    const uint32_t nb = p.lgraph[(uint64_t)m * p.r_small + j];
                    if (nb == kInvalid || nb >= nl)
                        ++n_inv;
                    else if (p.label_pts[lo + nb] == g)
                        ++n_self;
                    else
                        cand = p.label_pts[lo + nb];
                }
                bool dup = false;
                if (cand != kInvalid)
                    for (uint32_t k = 0; k < pos && !dup; ++k)
                        dup = row[k] == cand;
                for (int o = 0; o < 31; ++o)
                {
                    const uint32_t other = __shfl_sync(kFull, cand, o);
                    if (o < lane && other == cand && cand != kInvalid)
                        dup = true;
                }
                if (dup)
                    ++n_dup;
                const bool keep = cand != kInvalid && !dup;
                const unsigned mask = __ballot_sync(kFull, keep);
                if (keep)
                    row[pos + __popc(mask & ((1u << lane) - 1u))] = cand;
                pos += __popc(mask);
                __syncwarp();
            }
        }
        if (lane == 0)
            p.row_size[g] = pos;
    }
    for (int o = 16; o > 0; o >>= 1)
    {
        n_inv += __shfl_down_sync(kFull, n_inv, o);
        n_self += __shfl_down_sync(kFull, n_self, o);
        n_dup += __shfl_down_sync(kFull, n_dup, o);
    }
    if (lane == 0 && (n_inv | n_self | n_dup))
    {
        atomicAdd(p.counters + 0, n_inv);
        atomicAdd(p.counters + 1, n_self);
        atomicAdd(p.counters + 2, n_dup);
    }
}

// Copy each point's row from its scratch slot to its CSR position.
__global__ void __launch_bounds__(256) stitched_compact_kernel(uint32_t N, const uint32_t *pm_off, uint32_t r_small,
                                                               const uint32_t *rows, const uint32_t *row_off,
                                                               uint32_t *out)
{
    const int lane = threadIdx.x & 31;
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    for (uint32_t g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < N; g += warps)
    {
        const uint32_t *src = rows + (uint64_t)pm_off[g] * r_small;
        const uint32_t o = row_off[g], n = row_off[g + 1] - o;
        for (uint32_t k = lane; k < n; k += 32)
            out[o + k] = src[k];
    }
}

struct LabelPlan
{
    std::vector<uint32_t> order; // labels, largest first (ties by label id)
    uint64_t M = 0;
};

int validate_labels(uint32_t N, uint32_t num_labels, const uint64_t *label_offsets, const uint32_t *label_points)
{
    if (!label_offsets || (num_labels && !label_points))
        return fail(-1, "[GPU stitched] null label arrays");
    if (label_offsets[0] != 0)
        return fail(-1, "[GPU stitched] label_offsets[0] must be 0");
    for (uint32_t l = 0; l < num_labels; ++l)
        if (label_offsets[l + 1] < label_offsets[l])
            return fail(-1, "[GPU stitched] label_offsets must be non-decreasing (label %u)", l);
    const uint64_t M = label_offsets[num_labels];
    if (M >= 0xFFFFFFFFull)
        return fail(-1, "[GPU stitched] %llu label memberships exceed this build's 32-bit membership ids",
                    (unsigned long long)M);
    for (uint64_t m = 0; m < M; ++m)
        if (label_points[m] >= N)
            return fail(-1, "[GPU stitched] label point %u out of range (N=%u)", label_points[m], N);
    return 0;
}

struct Worker
{
    int rc = 0;
    std::string err;
    double busy = 0, max_label = 0, search_kernel = 0;
    uint64_t search_evals = 0, expansions = 0;
};

// Builds every selected label's graph into the label-major arrays.
int build_label_graphs(int dtype, const uint8_t *d_seg, uint64_t stride, uint32_t dim, uint32_t num_labels,
                       const uint64_t *label_offsets, const uint8_t *label_mask, uint32_t r_small, uint32_t l_small,
                       uint32_t C, uint32_t steps, const DanceVamanaParams &prm, uint32_t streams,
                       uint32_t *d_lgraph, uint32_t *d_ldeg, uint32_t *label_medoids_local, DanceStitchedStats *st)
{
    std::vector<uint32_t> order;
    for (uint32_t l = 0; l < num_labels; ++l)
        if (label_offsets[l + 1] > label_offsets[l] && (!label_mask || label_mask[l]))
            order.push_back(l);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        return label_offsets[a + 1] - label_offsets[a] > label_offsets[b + 1] - label_offsets[b];
    });
    if (order.empty())
        return 0;
    int dev = 0;
    DANCE_CUDA(cudaGetDevice(&dev));
    DANCE_CUDA(cudaDeviceSynchronize()); // the label store is complete before the workers start
    const uint32_t nthreads = std::max<uint32_t>(1, std::min<uint32_t>(streams, (uint32_t)order.size()));
    std::atomic<size_t> next{0};
    std::vector<Worker> workers(nthreads);
    std::vector<std::thread> pool;
    const double t0 = wall();
    for (uint32_t t = 0; t < nthreads; ++t)
    {
        pool.emplace_back([&, t]() {
            Worker &w = workers[t];
            auto bail = [&](int rc) {
                w.rc = rc;
                w.err = g_err;
            };
            if (cudaSetDevice(dev) != cudaSuccess)
                return bail(fail(-2, "[GPU stitched] cudaSetDevice failed in a label worker"));
            cudaStream_t s = nullptr;
            if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
                return bail(fail(-2, "[GPU stitched] stream creation failed"));
            DanceWorkspace ws;
            bool reserved = false;
            for (size_t k = next.fetch_add(1); k < order.size() && w.rc == 0; k = next.fetch_add(1))
            {
                const uint32_t l = order[k];
                const uint64_t off = label_offsets[l];
                const uint32_t n = (uint32_t)(label_offsets[l + 1] - off);
                if (!reserved)
                {
                    // Labels arrive largest first, so the first reservation
                    // is this worker's largest; its one-time zeroing runs on
                    // the legacy stream and is waited for here.
                    int rc = ws.reserve(n, r_small, l_small, C, steps, 0xFFFFFFFFu, false);
                    if (rc || cudaDeviceSynchronize() != cudaSuccess)
                    {
                        bail(rc ? rc : fail(-2, "[GPU stitched] workspace set-up failed"));
                        break;
                    }
                    reserved = true;
                }
                const double lt0 = wall();
                uint32_t med = 0;
                StageTimes tm;
                uint64_t ctr[8] = {0};
                int rc = build_resident_impl(dtype, d_seg + off * stride, stride, n, dim, r_small, l_small, C, steps,
                                             prm, ws, d_lgraph + off * r_small, d_ldeg + off, nullptr, &med, s,
                                             &tm, ctr);
                if (rc)
                {
                    bail(rc);
                    break;
                }
                const double dt = wall() - lt0;
                w.busy += dt;
                w.max_label = std::max(w.max_label, dt);
                w.search_kernel += tm.search_kernel;
                w.search_evals += ctr[0];
                w.expansions += ctr[1];
                label_medoids_local[l] = med < n ? med : 0u;
            }
            cudaStreamDestroy(s);
        });
    }
    for (auto &th : pool)
        th.join();
    const double wall_s = wall() - t0;
    for (auto &w : workers)
        if (w.rc)
            return fail(w.rc, "%s", w.err.c_str());
    if (st)
    {
        st->label_build_wall_seconds += wall_s;
        for (auto &w : workers)
        {
            st->per_label_gpu_build_sum_seconds += w.busy;
            st->per_label_gpu_build_max_seconds = std::max(st->per_label_gpu_build_max_seconds, w.max_label);
            st->search_kernel_seconds += w.search_kernel;
            st->search_evals += w.search_evals;
            st->search_expansions += w.expansions;
        }
        st->streams = nthreads;
        size_t fr = 0, tot = 0;
        if (cudaMemGetInfo(&fr, &tot) == cudaSuccess && tot)
            st->peak_gpu_mem_gb = std::max(st->peak_gpu_mem_gb, (double)(tot - fr) / (1024.0 * 1024.0 * 1024.0));
    }
    return 0;
}

void label_size_stats(uint32_t num_labels, const uint64_t *label_offsets, DanceStitchedStats *st)
{
    uint64_t mn = UINT64_MAX, mx = 0, sum = 0;
    for (uint32_t l = 0; l < num_labels; ++l)
    {
        const uint64_t n = label_offsets[l + 1] - label_offsets[l];
        if (!n)
            continue;
        mn = std::min(mn, n);
        mx = std::max(mx, n);
        sum += n;
    }
    st->num_labels = num_labels;
    st->npts_per_label_min = mn == UINT64_MAX ? 0u : (uint32_t)mn;
    st->npts_per_label_max = (uint32_t)mx;
    st->npts_per_label_mean = num_labels ? (double)sum / num_labels : 0.0;
    st->total_label_memberships = sum;
}

int remap_impl(uint32_t N, uint32_t num_labels, const uint64_t *label_offsets, const uint32_t *label_points,
               const uint32_t *d_label_points, const uint32_t *d_lgraph, const uint32_t *d_ldeg, uint32_t r_small,
               uint32_t r_out, uint64_t *row_offsets, uint32_t *row_ids, uint64_t capacity, DanceStitchedStats *st,
               cudaStream_t s)
{
    const uint64_t M = label_offsets[num_labels];
    // Point -> membership CSR on the host, memberships ascending per point
    // (membership order is label order).
    std::vector<uint32_t> pm_off((size_t)N + 1, 0), pm_list(M), mem_label(M);
    for (uint64_t m = 0; m < M; ++m)
        ++pm_off[label_points[m] + 1];
    for (uint32_t g = 0; g < N; ++g)
        pm_off[g + 1] += pm_off[g];
    {
        std::vector<uint32_t> cur(pm_off.begin(), pm_off.end() - 1);
        for (uint32_t l = 0; l < num_labels; ++l)
            for (uint64_t m = label_offsets[l]; m < label_offsets[l + 1]; ++m)
            {
                mem_label[m] = l;
                pm_list[cur[label_points[m]]++] = (uint32_t)m;
            }
    }
    DevBuf d_pm_off, d_pm_list, d_mem_label, d_label_off, d_rows, d_size, d_off, d_tiles, d_out, d_ctr;
    const uint32_t ntiles = (N + kScanTile - 1) / kScanTile;
    DANCE_CUDA(d_pm_off.ensure(((uint64_t)N + 1) * 4));
    DANCE_CUDA(d_pm_list.ensure(std::max<uint64_t>(M, 1) * 4));
    DANCE_CUDA(d_mem_label.ensure(std::max<uint64_t>(M, 1) * 4));
    DANCE_CUDA(d_label_off.ensure(((uint64_t)num_labels + 1) * 8));
    DANCE_CUDA(d_rows.ensure(std::max<uint64_t>(M * r_small, 1) * 4));
    DANCE_CUDA(d_size.ensure((uint64_t)N * 4));
    DANCE_CUDA(d_off.ensure(((uint64_t)N + 1) * 4));
    DANCE_CUDA(d_tiles.ensure(((uint64_t)ntiles + 1) * 4));
    DANCE_CUDA(d_ctr.ensure(32));
    DANCE_CUDA(cudaMemcpyAsync(d_pm_off.p, pm_off.data(), ((uint64_t)N + 1) * 4, cudaMemcpyHostToDevice, s));
    if (M)
    {
        DANCE_CUDA(cudaMemcpyAsync(d_pm_list.p, pm_list.data(), M * 4, cudaMemcpyHostToDevice, s));
        DANCE_CUDA(cudaMemcpyAsync(d_mem_label.p, mem_label.data(), M * 4, cudaMemcpyHostToDevice, s));
    }
    DANCE_CUDA(cudaMemcpyAsync(d_label_off.p, label_offsets, ((uint64_t)num_labels + 1) * 8, cudaMemcpyHostToDevice,
                               s));
    DANCE_CUDA(cudaMemsetAsync(d_ctr.p, 0, 32, s));
    RemapParams p{};
    p.N = N;
    p.pm_off = d_pm_off.as<uint32_t>();
    p.pm_list = d_pm_list.as<uint32_t>();
    p.mem_label = d_mem_label.as<uint32_t>();
    p.label_off = d_label_off.as<uint64_t>();
    p.label_pts = d_label_points;
    p.lgraph = d_lgraph;
    p.ldeg = d_ldeg;
    p.r_small = r_small;
    p.r_out = r_out;
    p.rows = d_rows.as<uint32_t>();
    p.row_size = d_size.as<uint32_t>();
    p.counters = d_ctr.as<unsigned long long>();
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>(((uint64_t)N + 7) / 8, sm_count() * 8ull));
    stitched_remap_kernel<<<grid, 256, 0, s>>>(p);
    DANCE_LAUNCHED();
    scan_tile_sums_kernel<<<ntiles, kScanThreads, 0, s>>>(d_size.as<uint32_t>(), N, d_tiles.as<uint32_t>());
    DANCE_LAUNCHED();
    scan_tile_offsets_kernel<<<1, kScanThreads, 0, s>>>(d_tiles.as<uint32_t>(), ntiles);
    DANCE_LAUNCHED();
    scan_apply_kernel<<<ntiles, kScanThreads, 0, s>>>(d_size.as<uint32_t>(), N, d_tiles.as<uint32_t>(),
                                                      d_off.as<uint32_t>(), nullptr);
    DANCE_LAUNCHED();
    std::vector<uint32_t> off32((size_t)N + 1);
    unsigned long long ctr[4] = {0, 0, 0, 0};
    DANCE_CUDA(cudaMemcpyAsync(off32.data(), d_off.p, ((uint64_t)N + 1) * 4, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaMemcpyAsync(ctr, d_ctr.p, 24, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    const uint64_t E = off32[N];
    if (E > capacity)
        return fail(-3, "[GPU stitched] output holds %llu edges, row_ids capacity is %llu", (unsigned long long)E,
                    (unsigned long long)capacity);
    DANCE_CUDA(d_out.ensure(std::max<uint64_t>(E, 1) * 4));
    stitched_compact_kernel<<<grid, 256, 0, s>>>(N, d_pm_off.as<uint32_t>(), r_small, d_rows.as<uint32_t>(),
                                                 d_off.as<uint32_t>(), d_out.as<uint32_t>());
    DANCE_LAUNCHED();
    if (E)
        DANCE_CUDA(cudaMemcpyAsync(row_ids, d_out.p, E * 4, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    uint32_t maxdeg = 0;
    for (uint32_t g = 0; g <= N; ++g)
    {
        row_offsets[g] = off32[g];
        if (g < N)
            maxdeg = std::max(maxdeg, off32[g + 1] - off32[g]);
    }
    if (st)
    {
        st->remap_invalid_local_ids = ctr[0];
        st->remap_self_loops = ctr[1];
        st->remap_duplicate_edges = ctr[2];
        st->output_edges = E;
        st->max_degree = maxdeg;
        st->processed_label_memberships = M;
    }
    return 0;
}

int check_stitched_params(uint32_t r_small, uint32_t l_small, uint32_t C, uint32_t steps)
{
    if (r_small == 0 || l_small == 0 || C == 0 || steps == 0)
        return fail(-1, "[GPU stitched] invalid parameters: Rsmall=%u Lsmall=%u C=%u steps=%u", r_small, l_small, C,
                    steps);
    if (C < r_small)
        return fail(-1, "[GPU stitched] invalid parameters: C=%u must be >= Rsmall=%u", C, r_small);
    return 0;
}

} // namespace
} // namespace dance

using namespace dance;

extern "C" {

int dance_stitched_label_graphs(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim,
                                uint32_t num_labels, const uint64_t *label_offsets, const uint32_t *label_points,
                                const uint8_t *label_mask, uint32_t r_small, uint32_t l_small, uint32_t C,
                                uint32_t steps, const DanceVamanaParams *params, uint32_t streams,
                                uint32_t *d_local_graph, uint32_t *d_local_degree, uint32_t *label_medoids_local,
                                DanceStitchedStats *stats)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (!rc)
        rc = check_stitched_params(r_small, l_small, C, steps);
    if (!rc)
        rc = validate_labels(N, num_labels, label_offsets, label_points);
    if (rc)
        return rc;
    if (!d_local_graph || !d_local_degree || !label_medoids_local)
        return fail(-1, "[GPU stitched] null output pointer");
    DanceVamanaParams prm;
    if (params)
        prm = *params;
    else
        dance_vamana_default_params(&prm);
    const uint64_t M = label_offsets[num_labels];
    if (stats)
        std::memset(stats, 0, sizeof(*stats));
    const double t0 = wall();
    DevBuf d_pts, d_seg;
    DANCE_CUDA(d_pts.ensure(std::max<uint64_t>(M, 1) * 4));
    DANCE_CUDA(d_seg.ensure(std::max<uint64_t>(M, 1) * stride));
    if (M)
    {
        DANCE_CUDA(cudaMemcpy(d_pts.p, label_points, M * 4, cudaMemcpyHostToDevice));
        const int grid = (int)std::min<uint64_t>((M + 7) / 8, (uint64_t)sm_count() * 16);
        gather_label_rows_kernel<<<grid, 256>>>(reinterpret_cast<const uint8_t *>(d_data), stride,
                                                 (uint32_t)stride, 0, dim, d_pts.as<uint32_t>(), M,
                                                 d_seg.as<uint8_t>(), stride);
        DANCE_LAUNCHED();
    }
    if (stats)
    {
        stats->label_data_materialization_seconds = wall() - t0;
        label_size_stats(num_labels, label_offsets, stats);
    }
    rc = build_label_graphs(dtype, d_seg.as<uint8_t>(), stride, dim, num_labels, label_offsets, label_mask, r_small,
                            l_small, C, steps, prm, streams, d_local_graph, d_local_degree, label_medoids_local,
                            stats);
    if (stats)
        stats->total_seconds = wall() - t0;
    return rc;
}

int dance_stitched_remap(uint32_t N, uint32_t num_labels, const uint64_t *label_offsets,
                         const uint32_t *label_points, const uint32_t *d_local_graph,
                         const uint32_t *d_local_degree, uint32_t r_small, uint32_t r_out, uint64_t *row_offsets,
                         uint32_t *row_ids, uint64_t row_ids_capacity, DanceStitchedStats *stats, void *stream)
{
    if (N == 0 || r_small == 0)
        return fail(-1, "[GPU stitched] invalid parameters: N=%u Rsmall=%u", N, r_small);
    int rc = validate_labels(N, num_labels, label_offsets, label_points);
    if (rc)
        return rc;
    if (!row_offsets || (!row_ids && row_ids_capacity) || !d_local_graph || !d_local_degree)
        return fail(-1, "[GPU stitched] null pointer");
    if ((uint64_t)label_offsets[num_labels] * r_small >= 0xFFFFFFFFull)
        return fail(-1, "[GPU stitched] memberships x Rsmall exceeds this build's 32-bit row offsets");
    if (r_out < r_small)
        r_out = r_small; // the reference app raises Rstitched to Rsmall (:86-87)
    const double t0 = wall();
    const uint64_t M = label_offsets[num_labels];
    DevBuf d_pts;
    cudaStream_t s = as_stream(stream);
    DANCE_CUDA(d_pts.ensure(std::max<uint64_t>(M, 1) * 4));
    if (M)
        DANCE_CUDA(cudaMemcpyAsync(d_pts.p, label_points, M * 4, cudaMemcpyHostToDevice, s));
    rc = remap_impl(N, num_labels, label_offsets, label_points, d_pts.as<uint32_t>(), d_local_graph, d_local_degree,
                    r_small, r_out, row_offsets, row_ids, row_ids_capacity, stats, s);
    if (!rc && stats)
        stats->local_to_global_remap_seconds = wall() - t0;
    return rc;
}

int dance_stitched_global_prune(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim,
                                const uint64_t *d_row_offsets, const uint32_t *d_row_ids,
                                const uint32_t *d_point_label_offsets, const uint32_t *d_point_labels,
                                uint32_t range, uint32_t max_candidates, float alpha, uint32_t *d_out_rows,
                                uint32_t *d_out_degree, uint64_t *pruned_rows_out, void *stream)
{
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    if (!d_row_offsets || !d_row_ids || !d_out_rows || !d_out_degree || range == 0 || max_candidates == 0 ||
        !(alpha >= 1.0f) || (!d_point_label_offsets) != (!d_point_labels))
        return fail(-1, "[GPU stitched prune] invalid arguments");
    cudaStream_t s = as_stream(stream);
    DevBuf scratch;
    DANCE_CUDA(scratch.ensure(16));
    uint32_t *d_max = scratch.as<uint32_t>();
    unsigned long long *d_pruned = reinterpret_cast<unsigned long long *>(scratch.as<uint8_t>() + 8);
    DANCE_CUDA(cudaMemsetAsync(scratch.p, 0, 16, s));
    csr_max_degree_kernel<<<std::max<int>(1, std::min<int>((int)((N + 255) / 256), sm_count() * 8)), 256, 0, s>>>(
        d_row_offsets, N, d_max);
    DANCE_LAUNCHED();
    uint32_t maxdeg = 0;
    DANCE_CUDA(cudaMemcpyAsync(&maxdeg, d_max, 4, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    if (maxdeg > kStitchedPruneMaxDegree)
        return fail(-1, "[GPU stitched prune] a row has %u neighbours; this build prunes rows of at most %u", maxdeg,
                    kStitchedPruneMaxDegree);
    StitchedPruneParams pp{};
    pp.st = make_view(d_data, stride, N, dim, dtype);
    pp.row_off = d_row_offsets;
    pp.row_ids = d_row_ids;
    pp.lab_off = d_point_label_offsets;
    pp.labs = d_point_labels;
    pp.range = range;
    pp.maxc = max_candidates;
    pp.pcap = (uint32_t)std::max(32, next_pow2((int)std::max(maxdeg, 1u)));
    pp.alpha = alpha;
    pp.out_rows = d_out_rows;
    pp.out_deg = d_out_degree;
    pp.pruned_rows = d_pruned;
    if ((rc = dispatch<LaunchStitchedPrune>(dtype, pp.st.nchunks, pp, s)))
        return rc;
    if (pruned_rows_out)
    {
        DANCE_CUDA(cudaMemcpyAsync(pruned_rows_out, d_pruned, 8, cudaMemcpyDeviceToHost, s));
        DANCE_CUDA(cudaStreamSynchronize(s));
    }
    return 0;
}

} // extern "C"

namespace dance
{
namespace
{
// Labels largest first to the least-loaded rank (ties: lower label id, lower
// rank), the assignment stitched.lpt_assignment also uses.
std::vector<int> lpt_owner(uint32_t num_labels, const uint64_t *label_offsets, int world)
{
    std::vector<uint32_t> order(num_labels);
    std::iota(order.begin(), order.end(), 0u);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        return label_offsets[a + 1] - label_offsets[a] > label_offsets[b + 1] - label_offsets[b];
    });
    std::vector<uint64_t> load((size_t)world, 0);
    std::vector<int> owner(num_labels, 0);
    for (uint32_t l : order)
    {
        int r = 0;
        for (int k = 1; k < world; ++k)
            if (load[(size_t)k] < load[(size_t)r])
                r = k;
        owner[l] = r;
        load[(size_t)r] += label_offsets[l + 1] - label_offsets[l];
    }
    return owner;
}

// Sends every label's local graph, degrees (label-major segments) and medoid
// from its owner to rank 0: grouped ncclSend/ncclRecv per label segment, and
// a sum-reduce of the medoid array (zero where a rank does not own the label).
int gather_label_graphs(DanceComm *c, uint32_t num_labels, const uint64_t *label_offsets, const std::vector<int> &owner,
                        uint32_t r_small, uint32_t *d_lgraph, uint32_t *d_ldeg, uint32_t *d_med, cudaStream_t s)
{
    DANCE_NCCL(ncclGroupStart());
    for (uint32_t l = 0; l < num_labels; ++l)
    {
        const uint64_t a = label_offsets[l], n = label_offsets[l + 1] - a;
        const int o = owner[l];
        if (n == 0 || o == 0)
            continue;
        if (c->rank == o)
        {
            DANCE_NCCL(ncclSend(d_lgraph + a * r_small, n * r_small, ncclUint32, 0, c->comm, s));
            DANCE_NCCL(ncclSend(d_ldeg + a, n, ncclUint32, 0, c->comm, s));
        }
        else if (c->rank == 0)
        {
            DANCE_NCCL(ncclRecv(d_lgraph + a * r_small, n * r_small, ncclUint32, o, c->comm, s));
            DANCE_NCCL(ncclRecv(d_ldeg + a, n, ncclUint32, o, c->comm, s));
        }
    }
    DANCE_NCCL(ncclGroupEnd());
    int rc = nccl_settle(c, deadline_of(c));
    if (rc)
        return rc;
    DANCE_NCCL(ncclReduce(d_med, d_med, num_labels, ncclUint32, ncclSum, 0, c->comm, s));
    if ((rc = nccl_settle(c, deadline_of(c))))
        return rc;
    return stream_wait(c, s, deadline_of(c));
}

// The stitched build, on one GPU (comm == nullptr) or label-parallel over the
// communicator's ranks (outputs written on rank 0 only).
int stitched_build_impl(DanceComm *comm, int dtype, const void *h_data, uint32_t N, uint32_t dim,
                        uint32_t num_labels, const uint64_t *label_offsets, const uint32_t *label_points,
                        uint32_t r_small, uint32_t l_small, uint32_t r_out, uint32_t C, uint32_t steps,
                        const DanceVamanaParams *params, uint32_t streams, uint64_t *row_offsets, uint32_t *row_ids,
                        uint64_t row_ids_capacity, uint32_t *label_medoids, DanceStitchedStats *stats)
{
    DanceStitchedStats local_stats;
    DanceStitchedStats *st = stats ? stats : &local_stats;
    std::memset(st, 0, sizeof(*st));
    const double t0 = wall();
    if (dtype != kU8 && dtype != kF32)
        return fail(-1, "[GPU stitched] supports uint8 and float input (dtype %d)", dtype);
    if (!h_data || N == 0 || dim == 0)
        return fail(-1, "[GPU stitched] null data or empty store (N=%u dim=%u)", N, dim);
    int rc = check_stitched_params(r_small, l_small, C, steps);
    if (!rc)
        rc = validate_labels(N, num_labels, label_offsets, label_points);
    if (rc)
        return rc;
    const bool root = !comm || comm->rank == 0;
    if (root && (!row_offsets || !label_medoids || (!row_ids && row_ids_capacity)))
        return fail(-1, "[GPU stitched] null output pointer");
    if (comm && comm->aborted)
        return fail(-1, "[GPU stitched] communicator aborted");
    if (r_out < r_small)
        r_out = r_small;
    const uint64_t M = label_offsets[num_labels];
    if (M * r_small >= 0xFFFFFFFFull)
        return fail(-1, "[GPU stitched] memberships x Rsmall exceeds this build's 32-bit row offsets");
    DanceVamanaParams prm;
    if (params)
        prm = *params;
    else
        dance_vamana_default_params(&prm);

    const int store_dtype = (dtype == kF32 && float16_build_enabled()) ? kF16 : dtype;
    const int in_es = elem_size(dtype), st_es = elem_size(store_dtype);
    const uint64_t in_row = (uint64_t)dim * in_es;
    const uint64_t stride = ((uint64_t)dim * st_es + 15u) & ~15ull;
    if (store_dtype == kF16 && (dim & 1u))
        return fail(-1, "[GPU stitched] fp16 storage needs an even dimension (dim=%u)", dim);

    // Vectors up once, then gathered label-major on the device.
    DevBuf d_in, d_pts, d_seg, d_lgraph, d_ldeg;
    cudaStream_t s = 0;
    DANCE_CUDA(d_in.ensure((uint64_t)N * in_row));
    DANCE_CUDA(d_pts.ensure(std::max<uint64_t>(M, 1) * 4));
    DANCE_CUDA(d_seg.ensure(std::max<uint64_t>(M, 1) * stride));
    DANCE_CUDA(d_lgraph.ensure(std::max<uint64_t>(M * r_small, 1) * 4));
    DANCE_CUDA(d_ldeg.ensure(std::max<uint64_t>(M, 1) * 4));
    DANCE_CUDA(cudaMemcpyAsync(d_in.p, h_data, (uint64_t)N * in_row, cudaMemcpyHostToDevice, s));
    if (M)
    {
        DANCE_CUDA(cudaMemcpyAsync(d_pts.p, label_points, M * 4, cudaMemcpyHostToDevice, s));
        const int grid = (int)std::min<uint64_t>((M + 7) / 8, (uint64_t)sm_count() * 16);
        gather_label_rows_kernel<<<grid, 256, 0, s>>>(d_in.as<uint8_t>(), in_row, (uint32_t)in_row,
                                                        store_dtype != dtype, dim, d_pts.as<uint32_t>(), M,
                                                        d_seg.as<uint8_t>(), stride);
        DANCE_LAUNCHED();
    }
    DANCE_CUDA(cudaStreamSynchronize(s));
    d_in.release();
    st->label_data_materialization_seconds = wall() - t0;
    label_size_stats(num_labels, label_offsets, st);

    std::vector<uint32_t> med_local(num_labels, 0);
    std::vector<uint8_t> mask;
    std::vector<int> owner;
    if (comm)
    {
        owner = lpt_owner(num_labels, label_offsets, comm->world);
        mask.resize(num_labels);
        for (uint32_t l = 0; l < num_labels; ++l)
            mask[l] = owner[l] == comm->rank;
    }
    rc = build_label_graphs(store_dtype, d_seg.as<uint8_t>(), stride, dim, num_labels, label_offsets,
                            comm ? mask.data() : nullptr, r_small, l_small, C, steps, prm, streams ? streams : 4u,
                            d_lgraph.as<uint32_t>(), d_ldeg.as<uint32_t>(), med_local.data(), st);
    if (rc)
        return rc;
    d_seg.release();
    if (comm)
    {
        DevBuf d_med;
        DANCE_CUDA(d_med.ensure(std::max<uint64_t>(num_labels, 1) * 4));
        for (uint32_t l = 0; l < num_labels; ++l)
            if (owner[l] != comm->rank)
                med_local[l] = 0;
        DANCE_CUDA(cudaMemcpyAsync(d_med.p, med_local.data(), (uint64_t)num_labels * 4, cudaMemcpyHostToDevice, s));
        const double xt0 = wall();
        if ((rc = gather_label_graphs(comm, num_labels, label_offsets, owner, r_small, d_lgraph.as<uint32_t>(),
                                      d_ldeg.as<uint32_t>(), d_med.as<uint32_t>(), s)))
            return rc;
        DANCE_CUDA(cudaMemcpy(med_local.data(), d_med.p, (uint64_t)num_labels * 4, cudaMemcpyDeviceToHost));
        st->label_graph_exchange_seconds = wall() - xt0;
        if (!root)
        {
            st->total_seconds = wall() - t0;
            return 0;
        }
    }
    for (uint32_t l = 0; l < num_labels; ++l)
    {
        const uint64_t n = label_offsets[l + 1] - label_offsets[l];
        label_medoids[l] = n ? label_points[label_offsets[l] + (med_local[l] < n ? med_local[l] : 0u)] : 0u;
    }
    const double rt0 = wall();
    rc = remap_impl(N, num_labels, label_offsets, label_points, d_pts.as<uint32_t>(), d_lgraph.as<uint32_t>(),
                    d_ldeg.as<uint32_t>(), r_small, r_out, row_offsets, row_ids, row_ids_capacity, st, s);
    if (rc)
        return rc;
    st->local_to_global_remap_seconds = wall() - rt0;
    st->total_seconds = wall() - t0;
    return 0;
}
} // namespace
} // namespace dance

extern "C" {

int dance_stitched_build(int dtype, const void *h_data, uint32_t N, uint32_t dim, uint32_t num_labels,
                         const uint64_t *label_offsets, const uint32_t *label_points, uint32_t r_small,
                         uint32_t l_small, uint32_t r_out, uint32_t C, uint32_t steps,
                         const DanceVamanaParams *params, uint32_t streams, uint64_t *row_offsets, uint32_t *row_ids,
                         uint64_t row_ids_capacity, uint32_t *label_medoids, DanceStitchedStats *stats)
{
    return stitched_build_impl(nullptr, dtype, h_data, N, dim, num_labels, label_offsets, label_points, r_small,
                               l_small, r_out, C, steps, params, streams, row_offsets, row_ids, row_ids_capacity,
                               label_medoids, stats);
}

int dance_stitched_build_sharded(DanceComm *comm, int dtype, const void *h_data, uint32_t N, uint32_t dim,
                                 uint32_t num_labels, const uint64_t *label_offsets, const uint32_t *label_points,
                                 uint32_t r_small, uint32_t l_small, uint32_t r_out, uint32_t C, uint32_t steps,
                                 const DanceVamanaParams *params, uint32_t streams, uint64_t *row_offsets,
                                 uint32_t *row_ids, uint64_t row_ids_capacity, uint32_t *label_medoids,
                                 DanceStitchedStats *stats)
{
    if (!comm)
        return fail(-1, "[GPU stitched] null communicator");
    return stitched_build_impl(comm, dtype, h_data, N, dim, num_labels, label_offsets, label_points, r_small,
                               l_small, r_out, C, steps, params, streams, row_offsets, row_ids, row_ids_capacity,
                               label_medoids, stats);
}

} // extern "C"
