// filtered.cu -- host driver and C ABI of GPU-FilteredVamana.
//
// Replaces gpu_vamana_filtered_build_uint8/_float of the reference
// (src/gpu_vamana_filtered.cu:6511-7066 with the canonical path
// canonical_round0_from_host_backbone_typed :5663-6483).  The plumbing is the
// B200 one: the whole build runs on one stream from a workspace allocated
// once (the reference allocates and frees per round and synchronises after
// every kernel); the only host read-back inside a round is the number of
// rows the reverse repair touches.
//
// One deliberate difference from the reference, in the reverse repair: the
// reference's candidate fill (:5071-5105) also writes the forward rows of
// rows that have no reverse source, at the start of the next row's list, so
// that row's list depends on which of the concurrent stores lands last.
// Here every touched row's list is exactly its forward row followed by its
// new reverse sources.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/dance_b200.h"
#include "../../include/gpu_vamana_filtered.h"
#include "filtered_kernels.cuh"
#include "host_common.cuh"

namespace dance
{
namespace
{

double fwall()
{
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

struct FilteredSetup
{
    uint32_t N, R, L, FL, C, STEPS;
    float alpha;
    uint32_t T, num_labels, universal, global_start;
    uint32_t task_pool, task_keep, union_pool, union_keep;
};

FilteredSetup make_setup(uint32_t N, uint32_t R, uint32_t L, uint32_t FL, uint32_t C, uint32_t STEPS, float alpha,
                         uint32_t T, uint32_t num_labels, uint32_t universal, uint32_t global_start)
{
    FilteredSetup s{};
    s.N = N;
    s.R = R;
    s.L = L;
    s.FL = FL;
    s.C = C;
    s.STEPS = STEPS;
    s.alpha = alpha;
    s.T = T;
    s.num_labels = num_labels;
    s.universal = universal;
    s.global_start = global_start;
    // per-label pool min(FilteredL, 32) keeping min(pool, 8); union pool
    // min(64, FilteredL) keeping min(R, L) (ref :5681-5688)
    s.task_pool = std::min(FL, 32u);
    s.task_keep = std::min(s.task_pool, 8u);
    s.union_pool = std::min(64u, FL);
    s.union_keep = std::min(R, L);
    return s;
}

struct FilteredWorkspace
{
    DevBuf off, lab, lpo, lp, starts, task_rows, label_bits;
    DevBuf ga, da, gb, db;
    DevBuf task_ids, task_d, union_ids, union_d;
    DevBuf work_ids, work_d, work_deg;
    DevBuf rev_cnt, rev_off, rev_cur, rev, tiles, cand_cnt, cand_off, cand_tiles;
    DevBuf cand_ids, cand_d, removed, touched, touched_n, counters;

    int reserve(const FilteredSetup &s)
    {
        const uint64_t N = s.N, NR = N * s.R;
        const uint32_t ntiles = (s.N + kScanTile - 1) / kScanTile + 1;
        DANCE_CUDA(task_rows.ensure(std::max<uint64_t>(s.T, 1) * 4));
        DANCE_CUDA(ga.ensure(NR * 4));
        DANCE_CUDA(da.ensure(N * 4));
        DANCE_CUDA(gb.ensure(NR * 4));
        DANCE_CUDA(db.ensure(N * 4));
        DANCE_CUDA(task_ids.ensure(std::max<uint64_t>(s.T, 1) * s.task_keep * 4));
        DANCE_CUDA(task_d.ensure(std::max<uint64_t>(s.T, 1) * s.task_keep * 4));
        DANCE_CUDA(union_ids.ensure(std::max<uint64_t>(N * s.union_keep, 1) * 4));
        DANCE_CUDA(union_d.ensure(std::max<uint64_t>(N * s.union_keep, 1) * 4));
        DANCE_CUDA(work_ids.ensure(N * s.C * 4));
        DANCE_CUDA(work_d.ensure(N * s.C * 4));
        DANCE_CUDA(work_deg.ensure(N * 4));
        DANCE_CUDA(rev_cnt.ensure(N * 4));
        DANCE_CUDA(rev_off.ensure((N + 1) * 4));
        DANCE_CUDA(rev_cur.ensure(N * 4));
        DANCE_CUDA(rev.ensure(std::max<uint64_t>(NR, 1) * 4));
        DANCE_CUDA(tiles.ensure((uint64_t)ntiles * 4));
        DANCE_CUDA(cand_cnt.ensure(N * 4));
        DANCE_CUDA(cand_off.ensure((N + 1) * 4));
        DANCE_CUDA(cand_tiles.ensure((uint64_t)ntiles * 4));
        // a touched row's list is its forward row plus new reverse sources: <= 2 N R in all
        DANCE_CUDA(cand_ids.ensure(std::max<uint64_t>(2 * NR, 1) * 4));
        DANCE_CUDA(cand_d.ensure(std::max<uint64_t>(2 * NR, 1) * 4));
        DANCE_CUDA(removed.ensure(std::max<uint64_t>(2 * NR, 1)));
        DANCE_CUDA(touched.ensure(N * 4));
        DANCE_CUDA(touched_n.ensure(16));
        DANCE_CUDA(counters.ensure(16 * 8));
        return 0;
    }
};

// Largest label-membership bitmap (num_labels x N bits) kept on the device;
// larger vocabularies test membership through the points' label lists.
constexpr uint64_t kLabelBitsBudget = 1ull << 30;

// Labels on the device; the label -> points postings are built on the host
// (ascending points, as the reference's h_label_points :5762-5773).
int upload_labels(FilteredWorkspace &ws, uint32_t N, const uint32_t *h_off, const uint32_t *h_lab,
                  const uint32_t *h_starts, uint32_t num_labels, fl::Labels &L, cudaStream_t s)
{
    const uint32_t T = h_off[N];
    std::vector<uint32_t> lpo((size_t)num_labels + 1, 0);
    for (uint32_t i = 0; i < T; ++i)
        ++lpo[h_lab[i] + 1];
    for (uint32_t l = 0; l < num_labels; ++l)
        lpo[l + 1] += lpo[l];
    std::vector<uint32_t> lp(std::max<uint32_t>(lpo[num_labels], 1)), cur(lpo.begin(), lpo.end() - 1);
    for (uint32_t p = 0; p < N; ++p)
        for (uint32_t i = h_off[p]; i < h_off[p + 1]; ++i)
            lp[cur[h_lab[i]]++] = p;
    DANCE_CUDA(ws.off.ensure(((uint64_t)N + 1) * 4));
    DANCE_CUDA(ws.lab.ensure(std::max<uint64_t>(T, 1) * 4));
    DANCE_CUDA(ws.lpo.ensure(((uint64_t)num_labels + 1) * 4));
    DANCE_CUDA(ws.lp.ensure((uint64_t)lp.size() * 4));
    DANCE_CUDA(ws.starts.ensure(std::max<uint64_t>(num_labels, 1) * 4));
    DANCE_CUDA(cudaMemcpyAsync(ws.off.p, h_off, ((uint64_t)N + 1) * 4, cudaMemcpyHostToDevice, s));
    if (T)
        DANCE_CUDA(cudaMemcpyAsync(ws.lab.p, h_lab, (uint64_t)T * 4, cudaMemcpyHostToDevice, s));
    DANCE_CUDA(cudaMemcpyAsync(ws.lpo.p, lpo.data(), lpo.size() * 4, cudaMemcpyHostToDevice, s));
    DANCE_CUDA(cudaMemcpyAsync(ws.lp.p, lp.data(), lp.size() * 4, cudaMemcpyHostToDevice, s));
    if (num_labels)
        DANCE_CUDA(cudaMemcpyAsync(ws.starts.p, h_starts, (uint64_t)num_labels * 4, cudaMemcpyHostToDevice, s));
    DANCE_CUDA(cudaStreamSynchronize(s)); // the host vectors above go out of scope
    L.off = ws.off.as<uint32_t>();
    L.lab = ws.lab.as<uint32_t>();
    L.lpo = ws.lpo.as<uint32_t>();
    L.lp = ws.lp.as<uint32_t>();
    L.starts = ws.starts.as<uint32_t>();
    L.num_labels = num_labels;
    // membership bitmaps, when they take at most kLabelBitsBudget bytes
    const uint64_t words = ((uint64_t)N + 31) / 32;
    const uint64_t bytes = words * 4 * (uint64_t)num_labels;
    L.bits = nullptr;
    L.bit_words = words;
    if (num_labels && bytes <= kLabelBitsBudget)
    {
        DANCE_CUDA(ws.label_bits.ensure(bytes));
        DANCE_CUDA(cudaMemsetAsync(ws.label_bits.p, 0, bytes, s));
        const int grid = (int)std::min<uint64_t>(((uint64_t)N + 255) / 256, (uint64_t)sm_count() * 8);
        fl::fl_label_bits_kernel<<<grid, 256, 0, s>>>(N, L.off, L.lab, words, ws.label_bits.as<uint32_t>());
        DANCE_LAUNCHED();
        L.bits = ws.label_bits.as<uint32_t>();
    }
    return 0;
}

int validate_labels(uint32_t N, const uint32_t *off, const uint32_t *lab, uint32_t num_labels)
{
    if (off[0] != 0)
        return fail(-1, "[gpu_vamana_filtered] point_label_offsets[0] must be 0");
    for (uint32_t p = 0; p < N; ++p)
    {
        if (off[p + 1] < off[p])
            return fail(-1, "[gpu_vamana_filtered] point_label_offsets decrease at point %u", p);
        for (uint32_t i = off[p]; i < off[p + 1]; ++i)
        {
            if (lab[i] >= num_labels)
                return fail(-1, "[gpu_vamana_filtered] point %u has label %u >= num_labels %u", p, lab[i],
                            num_labels);
            if (i > off[p] && lab[i] <= lab[i - 1])
                return fail(-1, "[gpu_vamana_filtered] labels of point %u are not strictly increasing", p);
        }
    }
    return 0;
}

// Copies of one round's intermediates (parity tests); any pointer may be null.
struct RoundTaps
{
    uint32_t *task_ids;
    float *task_d;
    uint32_t *union_ids;
    float *union_d;
    uint32_t *work_ids;
    float *work_d;
    uint32_t *work_deg;
    uint32_t *fwd_graph;
    uint32_t *fwd_degree;
};

struct RoundTimes
{
    double task = 0, union_search = 0, merge = 0, fwd_prune = 0, csr = 0, rev_prune = 0;
    uint64_t reverse_edges = 0, touched = 0;
};

inline int grid_for(const void *kernel, int threads, size_t smem, uint64_t warps)
{
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    per_sm = std::max(per_sm, 1);
    const uint64_t need = (warps + threads / 32 - 1) / (threads / 32);
    return (int)std::max<uint64_t>(1, std::min<uint64_t>(need, (uint64_t)per_sm * sm_count()));
}

inline int scan_counts(const uint32_t *cnt, uint32_t n, uint32_t *tiles, uint32_t *offsets, uint32_t *cursor,
                       cudaStream_t s)
{
    const uint32_t ntiles = (n + kScanTile - 1) / kScanTile;
    scan_tile_sums_kernel<<<ntiles, kScanThreads, 0, s>>>(cnt, n, tiles);
    DANCE_LAUNCHED();
    scan_tile_offsets_kernel<<<1, kScanThreads, 0, s>>>(tiles, ntiles);
    DANCE_LAUNCHED();
    scan_apply_kernel<<<ntiles, kScanThreads, 0, s>>>(cnt, n, tiles, offsets, cursor);
    DANCE_LAUNCHED();
    return 0;
}

struct Evs
{
    cudaEvent_t e[7] = {};
    ~Evs()
    {
        for (auto x : e)
            if (x)
                cudaEventDestroy(x);
    }
    int create()
    {
        for (auto &x : e)
            DANCE_CUDA(cudaEventCreate(&x));
        return 0;
    }
};

double ev_sec(cudaEvent_t a, cudaEvent_t b)
{
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    return ms * 1e-3;
}

// One canonical round: (ga, da) -> (gb, db).
template <int DT, int CPL>
struct LaunchFilteredRound
{
    static int run(const StoreView &st, const fl::Labels &L, const FilteredSetup &s, FilteredWorkspace &ws,
                   const uint32_t *ga, const uint32_t *da, uint32_t *gb, uint32_t *db, const RoundTaps *taps,
                   RoundTimes *tm, cudaStream_t strm)
    {
        unsigned long long *ctr = ws.counters.as<unsigned long long>();
        Evs ev;
        if (tm)
        {
            const int rc = ev.create();
            if (rc)
                return rc;
        }
        auto mark = [&](int i) -> cudaError_t { return tm ? cudaEventRecord(ev.e[i], strm) : cudaSuccess; };
        DANCE_CUDA(mark(0));
        if (s.T)
        {
            fl::TaskParams tp{};
            tp.st = st;
            tp.L = L;
            tp.R = s.R;
            tp.pool_cap = s.task_pool;
            tp.keep = s.task_keep;
            tp.steps = s.STEPS;
            tp.graph = ga;
            tp.degree = da;
            tp.task_rows = ws.task_rows.as<uint32_t>();
            tp.T = s.T;
            tp.out_ids = ws.task_ids.as<uint32_t>();
            tp.out_d = ws.task_d.as<float>();
            tp.counters = ctr + 0;
            auto k = fl::fl_task_search_kernel<DT, CPL>;
            k<<<grid_for((const void *)k, fl::kThreads, 0, s.T), fl::kThreads, 0, strm>>>(tp);
            DANCE_LAUNCHED();
        }
        DANCE_CUDA(mark(1));
        {
            fl::UnionParams up{};
            up.st = st;
            up.L = L;
            up.R = s.R;
            up.pool_cap = s.union_pool;
            up.keep = s.union_keep;
            up.steps = s.STEPS;
            up.global_start = s.global_start;
            up.graph = ga;
            up.degree = da;
            up.out_ids = ws.union_ids.as<uint32_t>();
            up.out_d = ws.union_d.as<float>();
            up.counters = ctr + 2;
            auto k = fl::fl_union_search_kernel<DT, CPL>;
            k<<<grid_for((const void *)k, fl::kThreads, 0, s.N), fl::kThreads, 0, strm>>>(up);
            DANCE_LAUNCHED();
        }
        DANCE_CUDA(mark(2));
        {
            fl::MergeParams mp{};
            mp.st = st;
            mp.L = L;
            mp.R = s.R;
            mp.C = s.C;
            mp.task_keep = s.task_keep;
            mp.union_keep = s.union_keep;
            mp.graph = ga;
            mp.degree = da;
            mp.task_ids = ws.task_ids.as<uint32_t>();
            mp.task_d = ws.task_d.as<float>();
            mp.union_ids = ws.union_ids.as<uint32_t>();
            mp.union_d = ws.union_d.as<float>();
            mp.work_ids = ws.work_ids.as<uint32_t>();
            mp.work_d = ws.work_d.as<float>();
            mp.work_deg = ws.work_deg.as<uint32_t>();
            mp.counters = ctr + 4;
            auto k = fl::fl_merge_kernel<DT, CPL>;
            k<<<grid_for((const void *)k, fl::kThreads, 0, s.N), fl::kThreads, 0, strm>>>(mp);
            DANCE_LAUNCHED();
        }
        DANCE_CUDA(mark(3));
        fl::PruneParams pp{};
        pp.st = st;
        pp.L = L;
        pp.R = s.R;
        pp.alpha = s.alpha;
        pp.counters = ctr + 5;
        {
            pp.list_ids = ws.work_ids.as<uint32_t>();
            pp.list_d = ws.work_d.as<float>();
            pp.list_off = nullptr;
            pp.width = s.C;
            pp.list_n = ws.work_deg.as<uint32_t>();
            pp.rows = nullptr;
            pp.nrows = s.N;
            pp.max_len = fl::kShortList; // >= C: every work row fits
            pp.graph = gb;
            pp.degree = db;
            auto k = fl::fl_prune_kernel<DT, CPL>;
            k<<<grid_for((const void *)k, fl::kThreads, 0, s.N), fl::kThreads, 0, strm>>>(pp);
            DANCE_LAUNCHED();
        }
        DANCE_CUDA(mark(4));
        if (taps)
        {
            auto cp = [&](void *dst, const void *src, uint64_t bytes) -> cudaError_t {
                return dst && bytes ? cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, strm) : cudaSuccess;
            };
            DANCE_CUDA(cp(taps->task_ids, ws.task_ids.p, (uint64_t)s.T * s.task_keep * 4));
            DANCE_CUDA(cp(taps->task_d, ws.task_d.p, (uint64_t)s.T * s.task_keep * 4));
            DANCE_CUDA(cp(taps->union_ids, ws.union_ids.p, (uint64_t)s.N * s.union_keep * 4));
            DANCE_CUDA(cp(taps->union_d, ws.union_d.p, (uint64_t)s.N * s.union_keep * 4));
            DANCE_CUDA(cp(taps->work_ids, ws.work_ids.p, (uint64_t)s.N * s.C * 4));
            DANCE_CUDA(cp(taps->work_d, ws.work_d.p, (uint64_t)s.N * s.C * 4));
            DANCE_CUDA(cp(taps->work_deg, ws.work_deg.p, (uint64_t)s.N * 4));
            DANCE_CUDA(cp(taps->fwd_graph, gb, (uint64_t)s.N * s.R * 4));
            DANCE_CUDA(cp(taps->fwd_degree, db, (uint64_t)s.N * 4));
        }
        // exact CSR reverse repair of the forward-pruned graph
        const uint64_t NR = (uint64_t)s.N * s.R;
        const int eg = (int)std::max<uint64_t>(1, std::min<uint64_t>((NR + 255) / 256, sm_count() * 32ull));
        DANCE_CUDA(cudaMemsetAsync(ws.rev_cnt.p, 0, (uint64_t)s.N * 4, strm));
        fl::fl_rev_count_kernel<<<eg, 256, 0, strm>>>(gb, db, s.N, s.R, ws.rev_cnt.as<uint32_t>());
        DANCE_LAUNCHED();
        int rc = scan_counts(ws.rev_cnt.as<uint32_t>(), s.N, ws.tiles.as<uint32_t>(), ws.rev_off.as<uint32_t>(),
                             ws.rev_cur.as<uint32_t>(), strm);
        if (rc)
            return rc;
        fl::fl_rev_fill_kernel<<<eg, 256, 0, strm>>>(gb, db, s.N, s.R, ws.rev_cur.as<uint32_t>(),
                                                      ws.rev.as<uint32_t>());
        DANCE_LAUNCHED();
        const int lg = grid_for((const void *)fl::fl_rev_list_kernel, fl::kThreads, 0, s.N);
        fl::fl_rev_list_kernel<<<lg, fl::kThreads, 0, strm>>>(gb, db, s.N, s.R, ws.rev_off.as<uint32_t>(),
                                                               ws.rev.as<uint32_t>(), ws.cand_cnt.as<uint32_t>(),
                                                               nullptr, nullptr, nullptr, nullptr, 0);
        DANCE_LAUNCHED();
        rc = scan_counts(ws.cand_cnt.as<uint32_t>(), s.N, ws.cand_tiles.as<uint32_t>(), ws.cand_off.as<uint32_t>(),
                         nullptr, strm);
        if (rc)
            return rc;
        DANCE_CUDA(cudaMemsetAsync(ws.touched_n.p, 0, 4, strm));
        fl::fl_rev_list_kernel<<<lg, fl::kThreads, 0, strm>>>(
            gb, db, s.N, s.R, ws.rev_off.as<uint32_t>(), ws.rev.as<uint32_t>(), ws.cand_cnt.as<uint32_t>(),
            ws.cand_off.as<uint32_t>(), ws.cand_ids.as<uint32_t>(), ws.touched.as<uint32_t>(),
            ws.touched_n.as<uint32_t>(), 1);
        DANCE_LAUNCHED();
        uint32_t touched = 0, proposals = 0;
        DANCE_CUDA(cudaMemcpyAsync(&touched, ws.touched_n.p, 4, cudaMemcpyDeviceToHost, strm));
        DANCE_CUDA(cudaMemcpyAsync(&proposals, ws.rev_off.as<uint32_t>() + s.N, 4, cudaMemcpyDeviceToHost, strm));
        DANCE_CUDA(cudaStreamSynchronize(strm));
        DANCE_CUDA(mark(5));
        if (touched)
        {
            auto kd = fl::fl_list_dist_kernel<DT, CPL>;
            kd<<<grid_for((const void *)kd, fl::kThreads, 0, touched), fl::kThreads, 0, strm>>>(
                st, ws.touched.as<uint32_t>(), touched, ws.cand_off.as<uint32_t>(), ws.cand_ids.as<uint32_t>(),
                ws.cand_d.as<float>(), ctr + 6);
            DANCE_LAUNCHED();
            pp.list_ids = ws.cand_ids.as<uint32_t>();
            pp.list_d = ws.cand_d.as<float>();
            pp.list_off = ws.cand_off.as<uint32_t>();
            pp.list_n = nullptr;
            pp.rows = ws.touched.as<uint32_t>();
            pp.nrows = touched;
            pp.max_len = fl::kShortList;
            pp.removed = ws.removed.as<uint8_t>();
            auto k = fl::fl_prune_kernel<DT, CPL>;
            k<<<grid_for((const void *)k, fl::kThreads, 0, touched), fl::kThreads, 0, strm>>>(pp);
            DANCE_LAUNCHED();
            auto kl = fl::fl_prune_long_kernel<DT, CPL>;
            kl<<<(int)std::min<uint32_t>(touched, (uint32_t)sm_count() * 4), 256, 0, strm>>>(pp);
            DANCE_LAUNCHED();
        }
        DANCE_CUDA(mark(6));
        if (tm)
        {
            DANCE_CUDA(cudaStreamSynchronize(strm));
            tm->task += ev_sec(ev.e[0], ev.e[1]);
            tm->union_search += ev_sec(ev.e[1], ev.e[2]);
            tm->merge += ev_sec(ev.e[2], ev.e[3]);
            tm->fwd_prune += ev_sec(ev.e[3], ev.e[4]);
            tm->csr += ev_sec(ev.e[4], ev.e[5]);
            tm->rev_prune += ev_sec(ev.e[5], ev.e[6]);
            tm->reverse_edges += proposals;
            tm->touched += touched;
        }
        return 0;
    }
};

int check_filtered_args(uint32_t N, uint32_t dim, uint32_t R, uint32_t L, uint32_t C)
{
    if (N == 0 || dim == 0 || R == 0 || L == 0 || C < R)
        return fail(-1, "[gpu_vamana_filtered] invalid parameters N=%u dim=%u R=%u L=%u C=%u", N, dim, R, L, C);
    if (R > fl::kMaxR)
        return fail(-1, "[gpu_vamana_filtered] R=%u exceeds the %u supported by this build", R, fl::kMaxR);
    return 0;
}

// The whole canonical build on a resident store (dtype kU8 or kF16).
int filtered_build_impl(int dtype, const void *d_store, uint64_t stride, uint32_t N, uint32_t dim,
                        const FilteredSetup &s0, const uint32_t *h_off, const uint32_t *h_lab,
                        const uint32_t *h_starts, const uint32_t *d_init_graph, const uint32_t *d_init_degree,
                        uint32_t rounds, uint32_t *d_graph_out, uint32_t *d_degree_out, const RoundTaps *taps,
                        GPUFilteredVamanaStats *stats, cudaStream_t strm)
{
    if (dtype != kU8 && dtype != kF16)
        return fail(-1, "[gpu_vamana_filtered] searches run on uint8 or fp16 storage (dtype %d)", dtype);
    int rc = check_store(dtype, d_store, stride, N, dim);
    if (rc)
        return rc;
    if (s0.C > fl::kMaxC || s0.C < s0.R)
        return fail(-1, "[gpu_vamana_filtered] work width %u must be in [R, %u]", s0.C, fl::kMaxC);
    rc = validate_labels(N, h_off, h_lab, s0.num_labels);
    if (rc)
        return rc;
    FilteredSetup s = s0;
    s.T = h_off[N];
    const double t0 = fwall();
    FilteredWorkspace ws;
    rc = ws.reserve(s);
    if (rc)
        return rc;
    fl::Labels L{};
    rc = upload_labels(ws, N, h_off, h_lab, h_starts, s.num_labels, L, strm);
    if (rc)
        return rc;
    L.universal = s.universal;
    if (stats)
        stats->label_h2d_seconds = fwall() - t0;
    const StoreView st = make_view(d_store, stride, N, dim, dtype);
    const int bg = (int)std::max<uint64_t>(1, std::min<uint64_t>(((uint64_t)N + 255) / 256, sm_count() * 16ull));
    const double tt = fwall();
    fl::fl_task_rows_kernel<<<bg, 256, 0, strm>>>(N, ws.off.as<uint32_t>(), ws.task_rows.as<uint32_t>());
    DANCE_LAUNCHED();
    uint32_t *ga = ws.ga.as<uint32_t>(), *da = ws.da.as<uint32_t>();
    uint32_t *gb = ws.gb.as<uint32_t>(), *db = ws.db.as<uint32_t>();
    if (d_init_graph)
    {
        DANCE_CUDA(cudaMemcpyAsync(ga, d_init_graph, (uint64_t)N * s.R * 4, cudaMemcpyDeviceToDevice, strm));
        DANCE_CUDA(cudaMemcpyAsync(da, d_init_degree, (uint64_t)N * 4, cudaMemcpyDeviceToDevice, strm));
    }
    else
    {
        // deterministic random graph, degree min(16, R), seed 42 (ref :6988-6996)
        fl::fl_random_graph_kernel<<<bg, 256, 0, strm>>>(N, s.R, 16u, 42u, ga, da);
        DANCE_LAUNCHED();
    }
    DANCE_CUDA(cudaMemsetAsync(ws.counters.p, 0, 16 * 8, strm));
    DANCE_CUDA(cudaStreamSynchronize(strm));
    if (stats)
        stats->task_generation_seconds = fwall() - tt;
    RoundTimes tm;
    for (uint32_t r = 0; r < rounds; ++r)
    {
        const RoundTaps *t = r == 0 ? taps : nullptr;
        RoundTimes *tp = stats ? &tm : nullptr;
        rc = dtype == kU8
                 ? dispatch_cpl<LaunchFilteredRound, kU8>(st.nchunks, st, L, s, ws, ga, da, gb, db, t, tp, strm)
                 : dispatch_cpl<LaunchFilteredRound, kF16>(st.nchunks, st, L, s, ws, ga, da, gb, db, t, tp, strm);
        if (rc)
            return rc;
        std::swap(ga, gb);
        std::swap(da, db);
    }
    DANCE_CUDA(cudaMemcpyAsync(d_graph_out, ga, (uint64_t)N * s.R * 4, cudaMemcpyDeviceToDevice, strm));
    DANCE_CUDA(cudaMemcpyAsync(d_degree_out, da, (uint64_t)N * 4, cudaMemcpyDeviceToDevice, strm));
    unsigned long long ctr[16] = {0};
    DANCE_CUDA(cudaMemcpyAsync(ctr, ws.counters.p, sizeof(ctr), cudaMemcpyDeviceToHost, strm));
    DANCE_CUDA(cudaStreamSynchronize(strm));
    if (stats)
    {
        stats->filtered_search_seconds = tm.task;
        stats->ordinary_search_seconds = tm.union_search;
        stats->merge_seconds = tm.merge;
        stats->forward_prune_seconds = tm.fwd_prune;
        stats->csr_reverse_seconds = tm.csr;
        stats->reverse_prune_seconds = tm.rev_prune;
        stats->filtered_search_distance_count = ctr[0];
        stats->unfiltered_search_distance_count = ctr[2];
        stats->reverse_edges = tm.reverse_edges;
        stats->reverse_touched_rows = tm.touched;
        stats->final_prune_rows = N;
        stats->semantic_stage = 6; // label_sync (ref GPU_FILTERED_STAGE_LABEL_SYNC)
        stats->semantic_complete = 1;
        size_t fr = 0, tot = 0;
        if (cudaMemGetInfo(&fr, &tot) == cudaSuccess)
            stats->peak_gpu_mem_gb = std::max(stats->peak_gpu_mem_gb, (double)(tot - fr) / (1024.0 * 1024.0 * 1024.0));
    }
    return 0;
}

__global__ void f32_to_f16_padded(const float *src, uint32_t dim, __half *dst, uint64_t dst_stride_elems, uint64_t n)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint64_t r = i / dim, c = i % dim;
        dst[r * dst_stride_elems + c] = __float2half_rn(src[i]);
    }
}

GPUFilteredVamanaStats g_last_filtered;

uint32_t env_u32_clamped(const char *name, uint32_t def, uint32_t lo, uint32_t hi)
{
    const char *e = std::getenv(name);
    if (!e || !*e)
        return def;
    long v = std::atol(e);
    if (v < (long)lo)
        v = lo;
    if (v > (long)hi)
        v = hi;
    return (uint32_t)v;
}

// Reference C ABI (host in, host out).
int filtered_host_build(int in_dtype, const void *h_data, uint32_t N, uint32_t dim, uint32_t R, uint32_t L,
                        uint32_t FL, uint32_t C, uint32_t STEPS, float alpha, const uint32_t *h_off,
                        const uint32_t *h_lab, uint32_t total_labels, const uint32_t *h_starts, uint32_t num_labels,
                        uint32_t universal, uint32_t global_start, uint32_t *h_graph, uint32_t *h_degree)
{
    std::memset(&g_last_filtered, 0, sizeof(g_last_filtered));
    g_last_filtered.semantic_stage = 6;
    const double t0 = fwall();
    if (!h_data || !h_graph || !h_degree || !h_off || !h_lab || !h_starts)
        return fail(-1, "[gpu_vamana_filtered] null input pointer.");
    int rc = check_filtered_args(N, dim, R, L, C);
    if (rc)
        return rc;
    if (h_off[N] != total_labels)
        return fail(-1, "[gpu_vamana_filtered] point_label_offsets[N]=%u != total_label_count=%u", h_off[N],
                    total_labels);
    rc = validate_labels(N, h_off, h_lab, num_labels);
    if (rc)
        return rc;
    // work width: min(C, 128) (DISKANN_GPU_FILTERED_WORK_C within [R, C]); the
    // reverse repair needs room for 2R per row (ref :6563-6567, :5839-5843)
    uint32_t work_C = env_u32_clamped("DISKANN_GPU_FILTERED_WORK_C", std::min(C, 128u), R, C);
    if (work_C > fl::kMaxC)
        work_C = fl::kMaxC;
    if ((uint64_t)work_C < 2ull * R)
    {
        fail(1, "[gpu_vamana_filtered] GPU work capacity cannot hold exact reverse CSR");
        return 1;
    }
    const int store_dtype = in_dtype == kF32 ? kF16 : kU8;
    const uint64_t in_row = (uint64_t)dim * elem_size(in_dtype);
    const uint64_t stride = ((uint64_t)dim * elem_size(store_dtype) + 15u) & ~15ull;
    if (store_dtype == kF16 && (dim & 1u))
        return fail(-1, "[gpu_vamana_filtered] fp16 search storage needs an even dimension (dim=%u)", dim);
    cudaStream_t s = 0;
    DevBuf input, store, graph, degree, init_g, init_d;
    DANCE_CUDA(input.ensure((uint64_t)N * in_row));
    DANCE_CUDA(cudaMemcpy(input.p, h_data, (uint64_t)N * in_row, cudaMemcpyHostToDevice));
    const void *d_store = input.p;
    if (store_dtype == kF16)
    {
        DANCE_CUDA(store.ensure((uint64_t)N * stride));
        DANCE_CUDA(cudaMemsetAsync(store.p, 0, (uint64_t)N * stride, s));
        const uint64_t n = (uint64_t)N * dim;
        const int grid = (int)std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count() * 32);
        f32_to_f16_padded<<<grid, 256, 0, s>>>(input.as<float>(), dim, store.as<__half>(), stride / 2, n);
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
    DANCE_CUDA(graph.ensure((uint64_t)N * R * 4));
    DANCE_CUDA(degree.ensure((uint64_t)N * 4));
    // optional vnew2 backbone instead of the random graph (ref :6986-7005)
    const char *handoff = std::getenv("DISKANN_GPU_FILTERED_HANDOFF");
    const bool random_init = !handoff || std::atoi(handoff) != 0;
    const double tg = fwall();
    if (!random_init)
    {
        const uint32_t backbone_C = env_u32_clamped("DISKANN_GPU_FILTERED_BACKBONE_C", std::min(C, 96u), R, C);
        const int bdt = (in_dtype == kF32 && !float16_build_enabled()) ? kF32 : store_dtype;
        const void *bstore = d_store;
        uint64_t bstride = stride;
        DevBuf b32;
        if (bdt == kF32)
        {
            bstride = ((uint64_t)dim * 4 + 15u) & ~15ull;
            DANCE_CUDA(b32.ensure((uint64_t)N * bstride));
            DANCE_CUDA(cudaMemsetAsync(b32.p, 0, (uint64_t)N * bstride, s));
            DANCE_CUDA(cudaMemcpy2DAsync(b32.p, bstride, input.p, in_row, in_row, N, cudaMemcpyDeviceToDevice, s));
            bstore = b32.p;
        }
        DanceVamanaParams prm;
        dance_vamana_default_params(&prm);
        DanceWorkspace bws;
        rc = bws.reserve(N, R, L, backbone_C, std::min(STEPS, L));
        if (rc)
            return rc;
        DANCE_CUDA(init_g.ensure((uint64_t)N * R * 4));
        DANCE_CUDA(init_d.ensure((uint64_t)N * 4));
        StageTimes bt;
        uint64_t bc[8] = {0};
        rc = build_resident_impl(bdt, bstore, bstride, N, dim, R, L, backbone_C, STEPS, prm, bws,
                                 init_g.as<uint32_t>(), init_d.as<uint32_t>(), nullptr, nullptr, s, &bt, bc);
        if (rc)
            return rc;
        g_last_filtered.backbone_seconds = fwall() - tg;
    }
    if (d_store != input.p)
        input.release();
    g_last_filtered.graph_build_seconds = fwall() - tg;
    const FilteredSetup su = make_setup(N, R, L, FL, work_C, STEPS, alpha, total_labels, num_labels, universal,
                                        global_start);
    rc = filtered_build_impl(store_dtype, d_store, stride, N, dim, su, h_off, h_lab, h_starts,
                             random_init ? nullptr : init_g.as<uint32_t>(),
                             random_init ? nullptr : init_d.as<uint32_t>(), 3, graph.as<uint32_t>(),
                             degree.as<uint32_t>(), nullptr, &g_last_filtered, s);
    if (rc)
        return rc;
    const double td = fwall();
    DANCE_CUDA(cudaMemcpy(h_graph, graph.p, (uint64_t)N * R * 4, cudaMemcpyDeviceToHost));
    DANCE_CUDA(cudaMemcpy(h_degree, degree.p, (uint64_t)N * 4, cudaMemcpyDeviceToHost));
    g_last_filtered.d2h_seconds = fwall() - td;
    uint64_t edges = 0;
    uint32_t mn = UINT32_MAX, mx = 0, invalid = 0, self = 0;
    for (uint32_t p = 0; p < N; ++p)
    {
        const uint32_t d = std::min(h_degree[p], R);
        edges += d;
        mn = std::min(mn, d);
        mx = std::max(mx, d);
        for (uint32_t i = 0; i < d; ++i)
        {
            const uint32_t v = h_graph[(uint64_t)p * R + i];
            invalid += v >= N;
            self += v == p;
        }
    }
    g_last_filtered.out_degree_min = mn;
    g_last_filtered.out_degree_max = mx;
    g_last_filtered.out_degree_avg = (double)edges / N;
    g_last_filtered.prune_output_degree_avg = (double)edges / N;
    g_last_filtered.invalid_neighbor_count = invalid;
    g_last_filtered.self_loop_count = self;
    g_last_filtered.gpu_build_seconds = fwall() - t0;
    return 0;
}

} // namespace
} // namespace dance

using namespace dance;

extern "C" {

int gpu_vamana_filtered_build_uint8(const uint8_t *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                                    uint32_t filtered_L, uint32_t C, uint32_t STEPS, float alpha,
                                    const uint32_t *point_label_offsets, const uint32_t *point_labels,
                                    uint32_t total_label_count, const uint32_t *label_to_start_id,
                                    uint32_t num_labels, uint32_t universal_label_id, uint32_t global_start_id,
                                    const uint32_t *, const uint32_t *, uint32_t, uint32_t *h_graph,
                                    uint32_t *h_degree)
{
    const int rc = filtered_host_build(kU8, h_data, num_points, dim, R, L, filtered_L, C, STEPS, alpha,
                                       point_label_offsets, point_labels, total_label_count, label_to_start_id,
                                       num_labels, universal_label_id, global_start_id, h_graph, h_degree);
    return rc == 0 ? 0 : (rc == 1 ? 1 : -1);
}

int gpu_vamana_filtered_build_float(const float *h_data, uint32_t num_points, uint32_t dim, uint32_t R, uint32_t L,
                                    uint32_t filtered_L, uint32_t C, uint32_t STEPS, float alpha,
                                    const uint32_t *point_label_offsets, const uint32_t *point_labels,
                                    uint32_t total_label_count, const uint32_t *label_to_start_id,
                                    uint32_t num_labels, uint32_t universal_label_id, uint32_t global_start_id,
                                    const uint32_t *, const uint32_t *, uint32_t, uint32_t *h_graph,
                                    uint32_t *h_degree)
{
    const int rc = filtered_host_build(kF32, h_data, num_points, dim, R, L, filtered_L, C, STEPS, alpha,
                                       point_label_offsets, point_labels, total_label_count, label_to_start_id,
                                       num_labels, universal_label_id, global_start_id, h_graph, h_degree);
    return rc == 0 ? 0 : (rc == 1 ? 1 : -1);
}

void gpu_vamana_filtered_get_last_stats(GPUFilteredVamanaStats *stats)
{
    if (stats)
        *stats = g_last_filtered;
}

int dance_filtered_random_graph(uint32_t num_points, uint32_t R, uint32_t initial_degree, uint32_t seed,
                                uint32_t *d_graph, uint32_t *d_degree, void *stream)
{
    if (num_points == 0 || R == 0 || !d_graph || !d_degree)
        return fail(-1, "invalid random graph arguments");
    const int bg = (int)std::max<uint64_t>(1, std::min<uint64_t>(((uint64_t)num_points + 255) / 256,
                                                                 (uint64_t)sm_count() * 16));
    fl::fl_random_graph_kernel<<<bg, 256, 0, as_stream(stream)>>>(num_points, R, initial_degree, seed, d_graph,
                                                                   d_degree);
    DANCE_LAUNCHED();
    return 0;
}

int dance_filtered_build_resident(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points,
                                  uint32_t dim, uint32_t R, uint32_t L, uint32_t filtered_L, uint32_t work_C,
                                  uint32_t STEPS, float alpha, const uint32_t *point_label_offsets,
                                  const uint32_t *point_labels, const uint32_t *label_to_start_id,
                                  uint32_t num_labels, uint32_t universal_label_id, uint32_t global_start_id,
                                  const uint32_t *d_init_graph, const uint32_t *d_init_degree, uint32_t rounds,
                                  uint32_t *d_graph, uint32_t *d_degree, GPUFilteredVamanaStats *stats,
                                  void *stream)
{
    if (!point_label_offsets || !point_labels || !label_to_start_id || !d_graph || !d_degree)
        return fail(-1, "[gpu_vamana_filtered] null pointer");
    int rc = check_filtered_args(num_points, dim, R, L, work_C);
    if (rc)
        return rc;
    if ((uint64_t)work_C < 2ull * R)
        return fail(1, "[gpu_vamana_filtered] work width %u below 2R", work_C);
    if (stats)
        std::memset(stats, 0, sizeof(*stats));
    const FilteredSetup su = make_setup(num_points, R, L, filtered_L, work_C, STEPS, alpha,
                                        point_label_offsets[num_points], num_labels, universal_label_id,
                                        global_start_id);
    return filtered_build_impl(dtype, d_data, row_stride_bytes, num_points, dim, su, point_label_offsets,
                               point_labels, label_to_start_id, d_init_graph, d_init_degree, rounds, d_graph,
                               d_degree, nullptr, stats, as_stream(stream));
}

int dance_filtered_stage_round(int dtype, const void *d_data, uint64_t row_stride_bytes, uint32_t num_points,
                               uint32_t dim, uint32_t R, uint32_t L, uint32_t filtered_L, uint32_t work_C,
                               uint32_t STEPS, float alpha, const uint32_t *point_label_offsets,
                               const uint32_t *point_labels, const uint32_t *label_to_start_id, uint32_t num_labels,
                               uint32_t universal_label_id, uint32_t global_start_id, const uint32_t *d_graph_in,
                               const uint32_t *d_degree_in, uint32_t *d_task_ids, float *d_task_dists,
                               uint32_t *d_union_ids, float *d_union_dists, uint32_t *d_work_ids,
                               float *d_work_dists, uint32_t *d_work_degree, uint32_t *d_forward_graph,
                               uint32_t *d_forward_degree, uint32_t *d_graph_out, uint32_t *d_degree_out,
                               void *stream)
{
    if (!d_graph_in || !d_degree_in || !point_label_offsets || !point_labels || !label_to_start_id ||
        !d_graph_out || !d_degree_out)
        return fail(-1, "[gpu_vamana_filtered] stage round needs an input graph, labels and outputs");
    RoundTaps taps{d_task_ids, d_task_dists, d_union_ids, d_union_dists, d_work_ids, d_work_dists, d_work_degree,
                   d_forward_graph, d_forward_degree};
    int rc = check_filtered_args(num_points, dim, R, L, work_C);
    if (rc)
        return rc;
    if ((uint64_t)work_C < 2ull * R)
        return fail(1, "[gpu_vamana_filtered] work width %u below 2R", work_C);
    const FilteredSetup su = make_setup(num_points, R, L, filtered_L, work_C, STEPS, alpha,
                                        point_label_offsets[num_points], num_labels, universal_label_id,
                                        global_start_id);
    return filtered_build_impl(dtype, d_data, row_stride_bytes, num_points, dim, su, point_label_offsets,
                               point_labels, label_to_start_id, d_graph_in, d_degree_in, 1, d_graph_out,
                               d_degree_out, &taps, nullptr, as_stream(stream));
}

} // extern "C"
