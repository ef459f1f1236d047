// vamana_kernels.cuh -- sm_100a kernels of the standard (vnew2) Vamana build.
//
// One round of the build (reference src/gpu_vamana_vnew2.cu:2517-2637) is
//   search_kernel      batched GreedySearch of every vertex on the frozen
//                      graph; records the expansion sequence  (ref :1119-1439)
//   replay_kernel      online RobustInsert of that sequence into C-wide
//                      work rows, pair distances from a shared-memory
//                      vector cache                            (ref :759-877)
//   rev_count/scan/fill  exact CSR of the reverse edges        (ref :1604-1661)
//   merge_kernel (+ heavy_merge_kernel)  reverse-edge merge in ascending
//                      source order                            (ref :1722-1814)
//   prune_kernel       RobustPrune(alpha) + last-round fill    (ref :1893-2147)
// plus medoid_score/medoid_argmin (ref :1032-1064, :2445-2479) and
// init_graph (ref :1066-1117).
//
// Layout in HBM: vectors row-major with a 16-byte-multiple stride; graph
// rows R-wide (ids uint32, INVALID-padded) with an aligned distance row
// (float, FLT_MAX-padded); work rows C-wide; expansion lists exp_stride-wide.
#pragma once

#include "dance_common.cuh"

namespace dance
{

constexpr int kWarpsPerBlock = 4;
constexpr int kMaxL = 256; // search pool capacity limit (8 entries per lane)
// Resident blocks per SM the search kernels are compiled for (caps their
// registers; the kernels are latency-bound and gain from more resident warps).
#ifndef DANCE_SEARCH_MIN_BLOCKS
#define DANCE_SEARCH_MIN_BLOCKS 8
#endif
// Default log2 size of the build search's per-warp visited table (shared
// memory; a lost entry only costs a repeated distance evaluation).
#ifndef DANCE_VISITED_LOG2
#define DANCE_VISITED_LOG2 10
#endif
constexpr int kBlockThreads = kWarpsPerBlock * 32;

struct StoreView
{
    const uint8_t *data;
    uint64_t stride;  // bytes between rows (multiple of 16)
    uint32_t nchunks; // 16-byte chunks per row that hold data
    uint32_t N;
};

__device__ __forceinline__ int warp_id_in_block() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ uint32_t visited_slot(uint32_t id, uint32_t log2h)
{
    return (id * 2654435761u) >> (32u - log2h);
}

// Per-warp scratch of the search kernels.
struct SearchSmem
{
    uint64_t *pk;   // pool keys (Lcap), sorted ascending
    uint8_t *pf;    // expanded flags aligned with the keys
    uint32_t Lcap;
    uint32_t *bid;  // batch ids (64)
    float *bd;      // batch distances (64)
    uint64_t *bkey; // survivor keys (64), sorted before the merge
    uint32_t *bins; // survivors' insertion points in the pool (64)
    uint32_t *vis;  // visited table (1 << log2h ids)
};

__host__ __device__ __forceinline__ uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }

__host__ __device__ __forceinline__ uint32_t search_smem_per_warp(uint32_t Lcap, uint32_t log2h)
{
    return align16(8u * Lcap) + align16(Lcap) + 256u + 256u + 512u + 256u + align16(4u << log2h);
}

__device__ __forceinline__ SearchSmem carve_search_smem(uint8_t *base, uint32_t Lcap, uint32_t log2h)
{
    SearchSmem s;
    uint8_t *p = base;
    s.Lcap = Lcap;
    s.pk = reinterpret_cast<uint64_t *>(p);
    p += align16(8u * Lcap);
    s.pf = p;
    p += align16(Lcap);
    s.bid = reinterpret_cast<uint32_t *>(p);
    p += 256;
    s.bd = reinterpret_cast<float *>(p);
    p += 256;
    s.bkey = reinterpret_cast<uint64_t *>(p);
    p += 512;
    s.bins = reinterpret_cast<uint32_t *>(p);
    p += 256;
    s.vis = reinterpret_cast<uint32_t *>(p);
    return s;
}

// Warp-uniform pool state (identical in every lane).
struct PoolState
{
    int P;   // entries in the pool
    int L;   // capacity
    int lb;  // every entry below lb is expanded
};

// Number of elements of sorted a[0..n) that are <= x.
__device__ __forceinline__ int upper_bound_u32(const uint32_t *a, int n, uint32_t x)
{
    int lo = 0, hi = n;
    while (lo < hi)
    {
        const int mid = (lo + hi) >> 1;
        if (a[mid] <= x)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// Merges m2 sorted, distinct survivor keys sm.bkey[0..m2) (whose pool
// insertion points are sm.bins[0..m2), ascending) into the pool in place.
// Entries below the first insertion point stay; the rest move up by the
// number of survivors inserted at or below them, 32 at a time from the top
// (a chunk is read whole before it is written, and nothing lands below it).
__device__ __forceinline__ void pool_merge(const SearchSmem &sm, PoolState &ps, int m2, int lane)
{
    uint64_t *pk = sm.pk;
    uint8_t *pf = sm.pf;
    const int lo = (int)sm.bins[0];
    uint32_t b[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        b[j] = (m2 <= 8 && j < m2) ? sm.bins[j] : 0xFFFFFFFFu;
    if (ps.P > lo)
    {
        for (int c0 = lo + ((ps.P - 1 - lo) & ~31); c0 >= lo; c0 -= 32)
        {
            const int i = c0 + lane;
            int np = ps.L;
            uint64_t key = 0;
            uint8_t flag = 0;
            if (i < ps.P)
            {
                int shift;
                if (m2 <= 8)
                {
                    shift = 0;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        shift += b[j] <= (uint32_t)i;
                }
                else
                    shift = upper_bound_u32(sm.bins, m2, (uint32_t)i);
                np = i + shift;
                key = pk[i];
                flag = pf[i];
            }
            __syncwarp();
            if (np < ps.L)
            {
                pk[np] = key;
                pf[np] = flag;
            }
            __syncwarp();
        }
    }
    for (int j = lane; j < m2; j += 32)
    {
        const int np = j + (int)sm.bins[j];
        if (np < ps.L)
        {
            pk[np] = sm.bkey[j];
            pf[np] = 0;
        }
    }
    __syncwarp();
    ps.lb = min(ps.lb, lo);
    ps.P = min(ps.P + m2, ps.L);
}

// Inserts up to 64 candidates (two per lane; kInvalid = none) into the pool.
// Candidates already in the visited table are skipped (they were evaluated
// before, so re-inserting them could not change the pool); the rest are
// evaluated (unless their distance is given) and keyed by (distance, id).
// Keys not below the pool's largest key when the pool is full are dropped;
// the survivors are deduplicated, checked against the pool (the visited
// table may have forgotten an id that is still pooled), sorted and merged
// so the pool keeps the L smallest keys.  Returns the distances evaluated.
template <int DT, int CPL>
__device__ __forceinline__ int pool_insert_batch(const SearchSmem &sm, PoolState &ps, uint32_t log2h,
                                                 const StoreView &st, const uint4 (&q)[CPL], uint32_t id0,
                                                 uint32_t id1, float d0, float d1, bool have_dist, int lane)
{
    bool ok0 = id0 != kInvalid;
    bool ok1 = id1 != kInvalid;
    if (ok0)
    {
        const uint32_t s = visited_slot(id0, log2h);
        if (sm.vis[s] == id0)
            ok0 = false;
        else
            sm.vis[s] = id0;
    }
    if (ok1)
    {
        const uint32_t s = visited_slot(id1, log2h);
        if (sm.vis[s] == id1)
            ok1 = false;
        else
            sm.vis[s] = id1;
    }
    const unsigned b0 = __ballot_sync(kFull, ok0);
    const unsigned b1 = __ballot_sync(kFull, ok1);
    const int m = __popc(b0) + __popc(b1);
    if (m == 0)
        return 0;
    const unsigned lt = (1u << lane) - 1u;
    if (ok0)
    {
        const int pos = __popc(b0 & lt);
        sm.bid[pos] = id0;
        sm.bd[pos] = d0;
    }
    if (ok1)
    {
        const int pos = __popc(b0) + __popc(b1 & lt);
        sm.bid[pos] = id1;
        sm.bd[pos] = d1;
    }
    __syncwarp();
    if (!have_dist)
    {
        eval_candidates<DT, CPL>(st.data, st.stride, st.nchunks, q, sm.bid, sm.bd, m, lane);
        __syncwarp();
    }
    const uint64_t *pool = sm.pk;
    const uint64_t maxk = (ps.P >= ps.L) ? pool[ps.L - 1] : kKeyMax;
    const int e0 = lane, e1 = lane + 32;
    uint64_t k0 = e0 < m ? make_key(sm.bd[e0], sm.bid[e0]) : kKeyMax;
    uint64_t k1 = e1 < m ? make_key(sm.bd[e1], sm.bid[e1]) : kKeyMax;
    if (k0 >= maxk)
        k0 = kKeyMax;
    if (k1 >= maxk)
        k1 = kKeyMax;
    const unsigned s0 = __ballot_sync(kFull, k0 != kKeyMax);
    const unsigned s1 = __ballot_sync(kFull, k1 != kKeyMax);
    const int k = __popc(s0) + __popc(s1);
    if (k == 0)
        return m;
    int m2;
    if (k <= 32)
    {
        // compact the survivors, then rank them by broadcast comparisons
        __syncwarp();
        if (k0 != kKeyMax)
            sm.bkey[__popc(s0 & lt)] = k0;
        if (k1 != kKeyMax)
            sm.bkey[__popc(s0) + __popc(s1 & lt)] = k1;
        __syncwarp();
        const uint64_t key = lane < k ? sm.bkey[lane] : kKeyMax;
        // a copy of the key in an earlier lane (only survivors hold finite keys)
        const bool dup = (__match_any_sync(kFull, key) & lt) != 0u;
        bool keep = lane < k && !dup;
        uint32_t ins = 0;
        if (keep)
        {
            const int p = lower_bound_u64(pool, ps.P, key);
            keep = !(p < ps.P && pool[p] == key);
            ins = (uint32_t)p;
        }
        const unsigned km = __ballot_sync(kFull, keep);
        m2 = __popc(km);
        if (m2 == 0)
            return m;
        int rank = 0;
#pragma unroll 4
        for (int i = 0; i < k; ++i)
            rank += ((km >> i) & 1u) && (sm.bkey[i] < key);
        __syncwarp();
        if (keep)
        {
            sm.bkey[rank] = key;
            sm.bins[rank] = ins;
        }
        __syncwarp();
    }
    else
    {
        // many survivors (early in the search): full bitonic sort
        uint64_t a = k0, b = k1;
        // warp_sort64 wants element 2*lane+s; the layout of the inputs is irrelevant
        warp_sort64(a, b, lane);
        const uint64_t prev0 = __shfl_up_sync(kFull, b, 1);
        bool keep0 = a != kKeyMax && !(lane > 0 && prev0 == a);
        bool keep1 = b != kKeyMax && b != a;
        uint32_t ins0 = 0, ins1 = 0;
        if (keep0)
        {
            const int p = lower_bound_u64(pool, ps.P, a);
            keep0 = !(p < ps.P && pool[p] == a);
            ins0 = (uint32_t)p;
        }
        if (keep1)
        {
            const int p = lower_bound_u64(pool, ps.P, b);
            keep1 = !(p < ps.P && pool[p] == b);
            ins1 = (uint32_t)p;
        }
        const unsigned c0 = __ballot_sync(kFull, keep0);
        const unsigned c1 = __ballot_sync(kFull, keep1);
        m2 = __popc(c0) + __popc(c1);
        if (m2 == 0)
            return m;
        const int before = __popc(c0 & lt) + __popc(c1 & lt);
        __syncwarp();
        if (keep0)
        {
            sm.bkey[before] = a;
            sm.bins[before] = ins0;
        }
        if (keep1)
        {
            const int j = before + (keep0 ? 1 : 0);
            sm.bkey[j] = b;
            sm.bins[j] = ins1;
        }
        __syncwarp();
    }
    pool_merge(sm, ps, m2, lane);
    return m;
}

// Index of the first unexpanded pool entry (smallest key), -1 if none;
// scanning starts at ps.lb, below which everything is expanded.
__device__ __forceinline__ int pool_select(const SearchSmem &sm, PoolState &ps, int lane)
{
    for (int base = ps.lb; base < ps.P; base += 32)
    {
        const int i = base + lane;
        const bool u = i < ps.P && sm.pf[i] == 0;
        const unsigned m = __ballot_sync(kFull, u);
        if (m)
        {
            const int sel = base + __ffs(m) - 1;
            ps.lb = sel + 1;
            return sel;
        }
    }
    ps.lb = ps.P;
    return -1;
}

__device__ __forceinline__ void clear_visited(uint32_t *vis, uint32_t log2h, int lane)
{
    uint4 *v4 = reinterpret_cast<uint4 *>(vis);
    const uint32_t n4 = (1u << log2h) >> 2;
    const uint4 inv = make_uint4(kInvalid, kInvalid, kInvalid, kInvalid);
    for (uint32_t i = lane; i < n4; i += 32)
        v4[i] = inv;
    __syncwarp();
}

// ====================================================================== medoid
template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads) medoid_score_kernel(StoreView st, uint32_t nc, uint32_t ns,
                                                                     float *scores, uint32_t *cand_ids)
{
    const int lane = lane_id();
    const uint32_t w = blockIdx.x * kWarpsPerBlock + warp_id_in_block();
    if (w >= nc)
        return;
    const int g = lane >> 3, gl = lane & 7;
    const uint32_t cand = hash_u32(w * 9973u + 17u) % st.N;
    uint4 q[CPL];
    load_frag<CPL>(q, st.data + (uint64_t)cand * st.stride, st.nchunks, gl);
    constexpr int U = Unroll<CPL>::value;
    float sum = 0.0f;
    for (uint32_t base = 0; base < ns; base += 4 * U)
    {
        uint4 buf[U][CPL];
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const uint32_t idx = base + 4 * u + g;
            if (idx < ns)
            {
                const uint32_t smp = hash_u32(idx * 10007u + 131u) % st.N;
                load_frag<CPL>(buf[u], st.data + (uint64_t)smp * st.stride, st.nchunks, gl);
            }
            else
            {
#pragma unroll
                for (int t = 0; t < CPL; ++t)
                    buf[u][t] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const float d = GroupDist<DT, CPL>::eval(q, buf[u], st.nchunks, gl);
#pragma unroll
            for (int gg = 0; gg < 4; ++gg)
            {
                const float dg = __shfl_sync(kFull, d, 8 * gg);
                const uint32_t idx = base + 4 * u + gg;
                if (lane == 0 && idx < ns)
                {
                    const uint32_t smp = hash_u32(idx * 10007u + 131u) % st.N;
                    if (smp != cand)
                        sum = __fadd_rn(sum, dg);
                }
            }
        }
    }
    if (lane == 0)
    {
        scores[w] = __fdiv_rn(sum, (float)ns);
        cand_ids[w] = cand;
    }
}

// Lowest score, first candidate on ties; entry 0 if no finite score.
static __global__ void __launch_bounds__(1024) medoid_argmin_kernel(const float *scores, const uint32_t *cand_ids,
                                                             uint32_t nc, uint32_t *medoid)
{
    __shared__ float s_v[32];
    __shared__ int s_i[32];
    float best = FLT_MAX;
    int bi = -1;
    for (uint32_t i = threadIdx.x; i < nc; i += blockDim.x)
    {
        const float v = scores[i];
        if (v < best)
        {
            best = v;
            bi = (int)i;
        }
    }
    for (int off = 16; off > 0; off >>= 1)
    {
        const float ov = __shfl_down_sync(kFull, best, off);
        const int oi = __shfl_down_sync(kFull, bi, off);
        if (oi >= 0 && (ov < best || (ov == best && (bi < 0 || oi < bi))))
        {
            best = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0)
    {
        s_v[threadIdx.x >> 5] = best;
        s_i[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0)
    {
        float b = FLT_MAX;
        int idx = -1;
        for (int w = 0; w < (int)((blockDim.x + 31) >> 5); ++w)
        {
            if (s_i[w] >= 0 && (s_v[w] < b || (s_v[w] == b && (idx < 0 || s_i[w] < idx))))
            {
                b = s_v[w];
                idx = s_i[w];
            }
        }
        *medoid = idx >= 0 ? cand_ids[idx] : 0u;
    }
}

// ====================================================================== init
template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads) init_graph_kernel(StoreView st, uint32_t R, uint32_t *cur_ids,
                                                                   float *cur_dists, uint32_t *degree, uint32_t v0,
                                                                   uint32_t v1, uint32_t lrow0)
{
    const int lane = lane_id();
    const int g = lane >> 3, gl = lane & 7;
    constexpr int U = Unroll<CPL>::value;
    for (uint32_t v = v0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < v1;
         v += gridDim.x * kWarpsPerBlock)
    {
        uint4 q[CPL];
        load_frag<CPL>(q, st.data + (uint64_t)v * st.stride, st.nchunks, gl);
        for (uint32_t base = 0; base < R; base += 4 * U)
        {
            uint4 buf[U][CPL];
            uint32_t nb[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
            {
                const uint32_t idx = base + 4 * u + g;
                nb[u] = kInvalid;
                if (idx < R)
                {
                    nb[u] = det_neighbor(v, idx, st.N);
                    if (st.N <= 1 || nb[u] >= st.N || nb[u] == v)
                        nb[u] = kInvalid;
                }
                if (nb[u] != kInvalid)
                    load_frag<CPL>(buf[u], st.data + (uint64_t)nb[u] * st.stride, st.nchunks, gl);
                else
                {
#pragma unroll
                    for (int t = 0; t < CPL; ++t)
                        buf[u][t] = make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
            {
                const uint32_t idx = base + 4 * u + g;
                const float d = GroupDist<DT, CPL>::eval(q, buf[u], st.nchunks, gl);
                if (idx < R && gl == 0)
                {
                    cur_ids[(uint64_t)v * R + idx] = nb[u];
                    cur_dists[(uint64_t)(v - lrow0) * R + idx] = nb[u] != kInvalid ? d : FLT_MAX;
                }
            }
        }
        if (lane == 0)
            degree[v] = st.N > 1 ? R : 0u;
    }
}

// ====================================================================== search
struct SearchParams
{
    StoreView st;
    uint32_t R, L, Lcap, steps, seeds, log2h;
    uint32_t entry;            // used when entry_ptr == nullptr
    const uint32_t *entry_ptr; // device scalar (medoid), optional
    const uint32_t *cur_ids;
    const float *cur_dists;
    const uint32_t *degree;
    uint32_t *exp_ids;
    float *exp_dists;
    uint32_t *exp_count;
    uint32_t exp_stride;
    uint32_t v0, v1;
    uint32_t lrow0; // first vertex of the per-rank arrays (own distance rows, expansion lists)
    unsigned long long *counters; // [0] distance evaluations, [1] expansions
};

template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads, DANCE_SEARCH_MIN_BLOCKS) search_kernel(SearchParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const int gl = lane & 7;
    const uint32_t per_warp = search_smem_per_warp(p.Lcap, p.log2h);
    const SearchSmem sm = carve_search_smem(smem_raw + warp_id_in_block() * per_warp, p.Lcap, p.log2h);
    const StoreView &st = p.st;
    const uint32_t N = st.N;
    const uint32_t entry = p.entry_ptr ? *p.entry_ptr : p.entry;
    unsigned long long evals = 0, expansions = 0;

    for (uint32_t v = p.v0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < p.v1;
         v += gridDim.x * kWarpsPerBlock)
    {
        uint4 q[CPL];
        load_frag<CPL>(q, st.data + (uint64_t)v * st.stride, st.nchunks, gl);
        clear_visited(sm.vis, p.log2h, lane);
        PoolState ps{0, (int)p.L, 0};

        // Seeds: entry point and hash seeds (distances computed) ...
        uint32_t sid = kInvalid;
        if (lane == 0)
        {
            if (entry < N && entry != v)
                sid = entry;
        }
        else if ((uint32_t)lane <= p.seeds)
        {
            const uint32_t s = det_neighbor(v, (uint32_t)(lane - 1) + 1024u, N);
            if (s < N && s != v)
                sid = s;
        }
        evals += pool_insert_batch<DT, CPL>(sm, ps, p.log2h, st, q, sid, kInvalid, 0.0f, 0.0f, false, lane);
        // ... then the vertex's own neighbours with their stored distances.
        const uint32_t deg_self = min(p.degree[v], p.R);
        for (uint32_t b = 0; b < deg_self; b += 64)
        {
            const uint32_t i0 = b + lane, i1 = b + 32 + lane;
            uint32_t a0 = kInvalid, a1 = kInvalid;
            float f0 = FLT_MAX, f1 = FLT_MAX;
            if (i0 < deg_self)
            {
                a0 = p.cur_ids[(uint64_t)v * p.R + i0];
                if (a0 < N && a0 != v)
                    f0 = p.cur_dists[(uint64_t)(v - p.lrow0) * p.R + i0];
                else
                    a0 = kInvalid;
            }
            if (i1 < deg_self)
            {
                a1 = p.cur_ids[(uint64_t)v * p.R + i1];
                if (a1 < N && a1 != v)
                    f1 = p.cur_dists[(uint64_t)(v - p.lrow0) * p.R + i1];
                else
                    a1 = kInvalid;
            }
            pool_insert_batch<DT, CPL>(sm, ps, p.log2h, st, q, a0, a1, f0, f1, true, lane);
        }

        uint32_t nexp = 0;
        for (uint32_t step = 0; step < p.steps; ++step)
        {
            const int sel = pool_select(sm, ps, lane);
            if (sel < 0)
                break;
            const uint64_t key = sm.pk[sel];
            const uint32_t x = key_id(key);
            if (lane == 0)
            {
                sm.pf[sel] = 1;
                p.exp_ids[(uint64_t)(v - p.lrow0) * p.exp_stride + step] = x;
                p.exp_dists[(uint64_t)(v - p.lrow0) * p.exp_stride + step] = key_dist(key);
            }
            __syncwarp();
            ++nexp;
            const uint32_t degx = min(p.degree[x], p.R);
            const uint32_t *row = p.cur_ids + (uint64_t)x * p.R;
            for (uint32_t b = 0; b < p.R; b += 64)
            {
                const uint32_t i0 = b + lane, i1 = b + 32 + lane;
                uint32_t a0 = i0 < degx ? row[i0] : kInvalid;
                uint32_t a1 = i1 < degx ? row[i1] : kInvalid;
                if (a0 >= N || a0 == v)
                    a0 = kInvalid;
                if (a1 >= N || a1 == v)
                    a1 = kInvalid;
                evals += pool_insert_batch<DT, CPL>(sm, ps, p.log2h, st, q, a0, a1, 0.0f, 0.0f, false, lane);
            }
        }
        if (lane == 0)
            p.exp_count[v - p.lrow0] = nexp;
        expansions += nexp;
    }
    if (lane == 0 && p.counters)
    {
        atomicAdd(&p.counters[0], evals);
        atomicAdd(&p.counters[1], expansions);
    }
}

// Query search (recall harness): best-first from `start` until every pool
// entry is expanded; the first K pool keys are the result.
struct QueryParams
{
    StoreView st;
    const uint8_t *queries;
    uint64_t qstride;
    uint32_t nq;
    const uint32_t *graph;
    uint32_t R, L, Lcap, K, log2h, start;
    uint32_t *out_ids;
    float *out_dists;
    // label-filtered search (all optional): only points carrying the
    // query's label are visited, from the query's own start point
    const uint32_t *label_off, *labels; // point label CSR, labels ascending per point
    const uint32_t *query_label;       // nq
    const uint32_t *query_start;       // nq
};

// Point p carries label l (labels of a point ascend).
__device__ __forceinline__ bool point_has_label(const uint32_t *off, const uint32_t *lab, uint32_t p, uint32_t l)
{
    const uint32_t e = off[p + 1];
    for (uint32_t i = off[p]; i < e; ++i)
        if (lab[i] >= l)
            return lab[i] == l;
    return false;
}

template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads, DANCE_SEARCH_MIN_BLOCKS) query_search_kernel(QueryParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const int gl = lane & 7;
    const uint32_t per_warp = search_smem_per_warp(p.Lcap, p.log2h);
    const SearchSmem sm = carve_search_smem(smem_raw + warp_id_in_block() * per_warp, p.Lcap, p.log2h);
    const uint32_t N = p.st.N;
    for (uint32_t qi = blockIdx.x * kWarpsPerBlock + warp_id_in_block(); qi < p.nq; qi += gridDim.x * kWarpsPerBlock)
    {
        uint4 q[CPL];
        load_frag<CPL>(q, p.queries + (uint64_t)qi * p.qstride, p.st.nchunks, gl);
        clear_visited(sm.vis, p.log2h, lane);
        PoolState ps{0, (int)p.L, 0};
        const uint32_t start = p.query_start ? p.query_start[qi] : p.start;
        const uint32_t qlabel = p.query_label ? p.query_label[qi] : kInvalid;
        const uint32_t s0 = (lane == 0 && start < N) ? start : kInvalid;
        pool_insert_batch<DT, CPL>(sm, ps, p.log2h, p.st, q, s0, kInvalid, 0.0f, 0.0f, false, lane);
        while (true)
        {
            const int sel = pool_select(sm, ps, lane);
            if (sel < 0)
                break;
            const uint32_t x = key_id(sm.pk[sel]);
            if (lane == 0)
                sm.pf[sel] = 1;
            __syncwarp();
            const uint32_t *row = p.graph + (uint64_t)x * p.R;
            for (uint32_t b = 0; b < p.R; b += 64)
            {
                const uint32_t i0 = b + lane, i1 = b + 32 + lane;
                uint32_t a0 = i0 < p.R ? row[i0] : kInvalid;
                uint32_t a1 = i1 < p.R ? row[i1] : kInvalid;
                if (a0 >= N || (p.query_label && !point_has_label(p.label_off, p.labels, a0, qlabel)))
                    a0 = kInvalid;
                if (a1 >= N || (p.query_label && !point_has_label(p.label_off, p.labels, a1, qlabel)))
                    a1 = kInvalid;
                pool_insert_batch<DT, CPL>(sm, ps, p.log2h, p.st, q, a0, a1, 0.0f, 0.0f, false, lane);
            }
        }
        for (uint32_t k = lane; k < p.K; k += 32)
        {
            const bool have = (int)k < ps.P;
            const uint64_t key = have ? sm.pk[k] : kKeyMax;
            p.out_ids[(uint64_t)qi * p.K + k] = have ? key_id(key) : kInvalid;
            p.out_dists[(uint64_t)qi * p.K + k] = have ? key_dist(key) : FLT_MAX;
        }
        __syncwarp();
    }
}

// ====================================================================== replay
struct ReplayParams
{
    StoreView st;
    uint32_t R, C;
    float alpha;
    const uint32_t *cur_ids;
    const float *cur_dists;
    const uint32_t *degree;
    const uint32_t *exp_ids;
    const float *exp_dists;
    const uint32_t *exp_count;
    uint32_t exp_stride;
    uint32_t *work_ids;
    float *work_dists;
    uint32_t *work_deg;
    uint32_t v0, v1;
    uint32_t lrow0;       // first vertex of the per-rank arrays
    uint32_t row_bytes;   // nchunks * 16
    uint32_t cache_rows;  // R + exp_stride
    uint32_t per_warp;    // smem bytes per warp
    unsigned long long *counters; // [2] pair evaluations
    uint32_t *masks;              // uint8 tensor-core replay: OCC/VIC masks of mask_vertices vertices
    uint32_t mask_vertices;       // (0: the pair-by-pair replay_kernel)
};

// Per-warp scratch of replay_kernel: the vector cache (initial neighbours,
// then the expanded nodes in order; before the gather it holds the initial
// sort keys when they are sorted in shared memory), the squared norms of the
// cached rows (uint8 rows of at most 128 bytes), the work row by slot (ids,
// distances), the kept slots in order (distance, cache row, slot) and the
// expansion list.
struct ReplayLayout
{
    uint32_t norms, wid, wd, od, ou, os, xid, xdd, bytes;
    __host__ __device__ ReplayLayout(uint32_t C, uint32_t cache_rows, uint32_t row_bytes, uint32_t exp_stride)
    {
        const uint32_t Cp = C <= 32 ? 32u : (uint32_t)next_pow2((int)C);
        const uint32_t cache_bytes = cache_rows * row_bytes;
        uint32_t o = align16(cache_bytes > 8u * Cp ? cache_bytes : 8u * Cp);
        norms = o;
        o += align16(4u * cache_rows);
        wid = o;
        o += align16(4u * C);
        wd = o;
        o += align16(4u * C);
        od = o;
        o += align16(4u * C);
        ou = o;
        o += align16(2u * C);
        os = o;
        o += align16(2u * C);
        xid = o;
        o += align16(4u * exp_stride);
        xdd = o;
        o += align16(4u * exp_stride);
        bytes = o;
    }
};

__host__ __device__ __forceinline__ uint32_t replay_smem_per_warp(uint32_t C, uint32_t cache_rows, uint32_t row_bytes,
                                                                  uint32_t exp_stride)
{
    return ReplayLayout(C, cache_rows, row_bytes, exp_stride).bytes;
}

// Warp argmax over (value, slot) pairs: larger value wins, lower slot on ties.
__device__ __forceinline__ void warp_argmax_lowslot(float &v, int &s)
{
    for (int off = 16; off > 0; off >>= 1)
    {
        const float ov = __shfl_down_sync(kFull, v, off);
        const int os = __shfl_down_sync(kFull, s, off);
        if (os >= 0 && (s < 0 || ov > v || (ov == v && os < s)))
        {
            v = ov;
            s = os;
        }
    }
    v = __shfl_sync(kFull, v, 0);
    s = __shfl_sync(kFull, s, 0);
}

// Copies `count` rows (row k from vector id idf(k)) into the cache (row k,
// row_bytes apart) with 8-lane groups, loading Unroll<CPL> rows per group
// before storing any, so that the loads overlap.
template <int CPL, class IdFn>
__device__ __forceinline__ void gather_rows_batched(const uint8_t *__restrict__ data, uint64_t stride,
                                                    uint32_t nchunks, int count, uint8_t *cache, uint32_t row_bytes,
                                                    int lane, IdFn idf)
{
    constexpr int U = Unroll<CPL>::value;
    const int g = lane >> 3, gl = lane & 7;
    for (int r0 = 0; r0 < count; r0 += 4 * U)
    {
        uint4 buf[U][CPL];
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const int r = r0 + 4 * u + g;
            if (r < count)
            {
                const uint4 *src = reinterpret_cast<const uint4 *>(data + (uint64_t)idf(r) * stride);
#pragma unroll
                for (int t = 0; t < CPL; ++t)
                {
                    const uint32_t c = (uint32_t)(gl + 8 * t);
                    if (c < nchunks)
                        buf[u][t] = ldg_chunk(src + c);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const int r = r0 + 4 * u + g;
            if (r < count)
            {
                uint4 *dst = reinterpret_cast<uint4 *>(cache + (uint32_t)r * row_bytes);
#pragma unroll
                for (int t = 0; t < CPL; ++t)
                {
                    const uint32_t c = (uint32_t)(gl + 8 * t);
                    if (c < nchunks)
                        dst[c] = buf[u][t];
                }
            }
        }
    }
}

// Same copy through cp.async (global -> shared without registers): every
// row's chunks are in flight at once.  The caller waits with
// gather_rows_async_wait() before reading the rows.
template <int CPL, class IdFn>
__device__ __forceinline__ void gather_rows_async(const uint8_t *__restrict__ data, uint64_t stride, uint32_t nchunks,
                                                  int count, uint8_t *cache, uint32_t row_bytes, int lane, IdFn idf)
{
    const int g = lane >> 3, gl = lane & 7;
    for (int r = g; r < count; r += 4)
    {
        const uint8_t *src = data + (uint64_t)idf(r) * stride;
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(cache + (uint32_t)r * row_bytes);
#pragma unroll
        for (int t = 0; t < CPL; ++t)
        {
            const uint32_t c = (uint32_t)(gl + 8 * t);
            if (c < nchunks)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst + 16u * c), "l"(src + 16u * c)
                             : "memory");
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

__device__ __forceinline__ void gather_rows_async_wait()
{
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncwarp();
}

// Order key of a work-row slot: descending distance, then ascending slot --
// the reference's preference for the victim and the worst entry
// (src/gpu_vamana_vnew2.cu:816-846, strict '>' scans in slot order).
__device__ __forceinline__ uint64_t order_key(float d, uint32_t slot)
{
    return ((uint64_t)(~__float_as_uint(d)) << 32) | slot;
}

// Pair distances of the replay: x (one cached row) against up to kPairs
// cached rows per warp pass.  uint8 rows of at most 128 bytes use four lanes
// per pair (eight pairs a pass; the two 16-byte chunks of a lane are read in
// an order that keeps each 8-lane phase on distinct banks) and the cached
// squared norms: d = |x|^2 + |y|^2 - 2<x,y>, exact in integers.  The other
// types use the 8-lane groups of GroupDist, whose summation order is the
// reference's.
template <int DT, int CPL>
struct ReplayPairs
{
    static constexpr bool kQuad = (DT == kU8 && CPL == 1);
    static constexpr bool kFQuad = (DT != kU8 && CPL <= 4); // float / half: QuadDist
    static constexpr int kPairs = (kQuad || kFQuad) ? 8 : 4;
    static constexpr int kLanes = 32 / kPairs;
    static constexpr int kT = kQuad ? 2 : (kFQuad ? 2 * CPL : CPL);
    uint4 xf[kT];
    uint32_t nx;
    int pidx, sl;
    uint32_t c0, c1;

    __device__ __forceinline__ ReplayPairs(int lane)
    {
        pidx = lane / kLanes;
        sl = lane % kLanes;
        c0 = (uint32_t)sl + 4u * (uint32_t)(pidx & 1);
        c1 = c0 ^ 4u;
        nx = 0;
    }
    __device__ __forceinline__ void load_x(const uint8_t *row, uint32_t nchunks, uint32_t norm)
    {
        if constexpr (kQuad)
        {
            const uint4 *r = reinterpret_cast<const uint4 *>(row);
            xf[0] = c0 < nchunks ? r[c0] : make_uint4(0u, 0u, 0u, 0u);
            xf[1] = c1 < nchunks ? r[c1] : make_uint4(0u, 0u, 0u, 0u);
            nx = norm;
        }
        else if constexpr (kFQuad)
        {
            const uint4 *r = reinterpret_cast<const uint4 *>(row);
#pragma unroll
            for (int t = 0; t < kT; ++t)
            {
                const uint32_t c = (uint32_t)sl + 4u * (uint32_t)t;
                xf[t] = c < nchunks ? r[c] : make_uint4(0u, 0u, 0u, 0u);
            }
        }
        else
            load_frag_smem<CPL>(xf, row, nchunks, sl);
    }
    // d(x, row) for the row in cache slot u; every lane of the pair ends with
    // the value.
    __device__ __forceinline__ float dist(const uint8_t *row, uint32_t nchunks, const uint32_t *norms,
                                          uint32_t u) const
    {
        if constexpr (kQuad)
        {
            const uint4 *r = reinterpret_cast<const uint4 *>(row);
            uint32_t a0 = 0, a1 = 0;
            if (c0 < nchunks)
            {
                const uint4 y = r[c0];
                a0 = __dp4a(xf[0].x, y.x, a0);
                a0 = __dp4a(xf[0].y, y.y, a0);
                a0 = __dp4a(xf[0].z, y.z, a0);
                a0 = __dp4a(xf[0].w, y.w, a0);
            }
            if (c1 < nchunks)
            {
                const uint4 y = r[c1];
                a1 = __dp4a(xf[1].x, y.x, a1);
                a1 = __dp4a(xf[1].y, y.y, a1);
                a1 = __dp4a(xf[1].z, y.z, a1);
                a1 = __dp4a(xf[1].w, y.w, a1);
            }
            uint32_t dot = a0 + a1;
            dot += __shfl_xor_sync(kFull, dot, 1);
            dot += __shfl_xor_sync(kFull, dot, 2);
            return (float)(int32_t)(nx + norms[u] - 2u * dot);
        }
        else if constexpr (kFQuad)
            return QuadDist<DT, kT>::eval(xf, row, nchunks, sl);
        else
        {
            uint4 c[CPL];
            load_frag_smem<CPL>(c, row, nchunks, sl);
            return GroupDist<DT, CPL>::eval(xf, c, nchunks, sl);
        }
    }
};

// Squared norms of cache rows [0, n) of at most 128 bytes (8 chunks), one
// row per lane, chunk order rotated by lane so a warp load touches every
// bank group.
__device__ __forceinline__ void cache_row_norms(const uint8_t *cache, uint32_t row_bytes, uint32_t nchunks,
                                                uint32_t n, uint32_t *norms, int lane)
{
    for (uint32_t r = lane; r < n; r += 32)
    {
        const uint4 *row = reinterpret_cast<const uint4 *>(cache + r * row_bytes);
        uint32_t a0 = 0, a1 = 0;
#pragma unroll
        for (uint32_t c8 = 0; c8 < 8; ++c8)
        {
            const uint32_t c = (c8 + (uint32_t)lane) & 7u;
            if (c < nchunks)
            {
                const uint4 y = row[c];
                a0 = __dp4a(y.x, y.x, a0);
                a1 = __dp4a(y.y, y.y, a1);
                a0 = __dp4a(y.z, y.z, a0);
                a1 = __dp4a(y.w, y.w, a1);
            }
        }
        norms[r] = a0 + a1;
    }
}

// Online RobustInsert replay (reference dynamic_robust_insert_C_warp,
// src/gpu_vamana_vnew2.cu:759-877) of each vertex's recorded expansion
// sequence into its C-wide work row.  One warp per vertex; the row's
// vectors (initial neighbours and expanded nodes) are cached in shared
// memory, and the kept slots are held in order of order_key (distance
// descending, slot ascending) as parallel arrays (distance, cache row,
// slot), so
//  - occlusion is tested from the nearest kept neighbour outwards and stops
//    at the first occluder,
//  - the victim is the first qualifying slot from the far end,
//  - the worst slot is position 0,
// and an insertion moves only the positions between its old and new place.
// Initial order of a replay row: keys of the valid slots sorted, written as
// the ordered arrays (distance, cache row = slot, slot); returns their
// number.  NPL = Cp / 32 keys per lane sorted in registers, or NPL = 0: Cp
// keys sorted in shared memory (okeys).
template <int NPL>
__device__ __forceinline__ int replay_initial_order(const ReplayParams &p, uint32_t v, uint64_t lv, uint32_t Cp,
                                                    uint32_t deg_self, uint32_t *wid, float *wd, float *od,
                                                    uint16_t *ou, uint16_t *os, uint64_t *okeys, int lane)
{
    const uint32_t C = p.C, N = p.st.N;
    int nv = 0;
    if constexpr (NPL > 0)
    {
        uint64_t k[NPL];
#pragma unroll
        for (int t = 0; t < NPL; ++t)
        {
            const uint32_t i = (uint32_t)(lane * NPL + t);
            uint32_t nb = kInvalid;
            float d = FLT_MAX;
            uint64_t ok = kKeyMax;
            if (i < deg_self)
            {
                nb = p.cur_ids[(uint64_t)v * p.R + i];
                if (nb < N && nb != v)
                {
                    d = p.cur_dists[lv * p.R + i];
                    ok = order_key(d, i);
                }
                else
                    nb = kInvalid;
            }
            if (i < C)
            {
                wid[i] = nb;
                wd[i] = d;
            }
            k[t] = ok;
        }
        __syncwarp();
        warp_sort_blocked<NPL>(k, lane);
#pragma unroll
        for (int t = 0; t < NPL; ++t)
        {
            const uint32_t e = (uint32_t)(lane * NPL + t);
            const bool valid = k[t] != kKeyMax;
            if (valid)
            {
                const uint32_t slot = (uint32_t)(k[t] & 0xFFFFu);
                od[e] = wd[slot];
                ou[e] = (uint16_t)slot;
                os[e] = (uint16_t)slot;
            }
            nv += __popc(__ballot_sync(kFull, valid));
        }
    }
    else
    {
        for (uint32_t i = lane; i < Cp; i += 32)
        {
            uint32_t nb = kInvalid;
            float d = FLT_MAX;
            uint64_t ok = kKeyMax;
            if (i < deg_self)
            {
                nb = p.cur_ids[(uint64_t)v * p.R + i];
                if (nb < N && nb != v)
                {
                    d = p.cur_dists[lv * p.R + i];
                    ok = order_key(d, i);
                }
                else
                    nb = kInvalid;
            }
            if (i < C)
            {
                wid[i] = nb;
                wd[i] = d;
            }
            okeys[i] = ok;
        }
        __syncwarp();
        warp_sort_smem_u64(okeys, (int)Cp, lane);
        for (uint32_t b = 0; b < Cp; b += 32)
        {
            const uint64_t k = okeys[b + lane];
            const bool valid = k != kKeyMax;
            nv += __popc(__ballot_sync(kFull, valid));
            if (valid)
            {
                const uint32_t slot = (uint32_t)(k & 0xFFFFu);
                od[b + lane] = wd[slot];
                ou[b + lane] = (uint16_t)slot;
                os[b + lane] = (uint16_t)slot;
            }
        }
    }
    return nv;
}

// Online RobustInsert replay (reference dynamic_robust_insert_C_warp,
// src/gpu_vamana_vnew2.cu:759-877) of each vertex's recorded expansion
// sequence into its C-wide work row.  One warp per vertex; the row's
// vectors (initial neighbours and expanded nodes) are cached in shared
// memory, and the kept slots are held in order of order_key (distance
// descending, slot ascending) as parallel arrays (distance, cache row,
// slot), so
//  - occlusion is tested from the nearest kept neighbour outwards and stops
//    at the first occluder,
//  - the victim is the first qualifying slot from the far end,
//  - the worst slot is position 0,
// and an insertion moves only the positions between its old and new place.
template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads, CPL <= 2 ? 3 : 1) replay_kernel(ReplayParams p)
{
    using Pairs = ReplayPairs<DT, CPL>;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const uint32_t C = p.C;
    const uint32_t Cp = C <= 32 ? 32u : (uint32_t)next_pow2((int)C);
    const ReplayLayout lay(C, p.cache_rows, p.row_bytes, p.exp_stride);
    uint8_t *base = smem_raw + warp_id_in_block() * p.per_warp;
    uint8_t *cache = base;
    uint32_t *norms = reinterpret_cast<uint32_t *>(base + lay.norms);
    uint32_t *wid = reinterpret_cast<uint32_t *>(base + lay.wid);
    float *wd = reinterpret_cast<float *>(base + lay.wd);
    float *od = reinterpret_cast<float *>(base + lay.od);
    uint16_t *ou = reinterpret_cast<uint16_t *>(base + lay.ou);
    uint16_t *os = reinterpret_cast<uint16_t *>(base + lay.os);
    uint32_t *xid = reinterpret_cast<uint32_t *>(base + lay.xid);
    float *xdd = reinterpret_cast<float *>(base + lay.xdd);
    uint64_t *okeys = reinterpret_cast<uint64_t *>(base); // initial sort (NPL = 0), before the gather
    const uint32_t N = p.st.N;
    const uint32_t nch = p.st.nchunks;
    const float alpha = p.alpha;
    Pairs pe(lane);
    unsigned long long pairs = 0;

    for (uint32_t v = p.v0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < p.v1;
         v += gridDim.x * kWarpsPerBlock)
    {
        const uint64_t lv = v - p.lrow0;
        const uint32_t deg_self = min(p.degree[v], p.R);
        const uint32_t cnt = min(p.exp_count[lv], p.exp_stride);
        for (uint32_t k = lane; k < cnt; k += 32)
        {
            xid[k] = p.exp_ids[lv * p.exp_stride + k];
            xdd[k] = p.exp_dists[lv * p.exp_stride + k];
        }
        int nv;
        if (Cp == 32)
            nv = replay_initial_order<1>(p, v, lv, Cp, deg_self, wid, wd, od, ou, os, okeys, lane);
        else if (Cp == 64)
            nv = replay_initial_order<2>(p, v, lv, Cp, deg_self, wid, wd, od, ou, os, okeys, lane);
        else if (Cp == 128)
            nv = replay_initial_order<4>(p, v, lv, Cp, deg_self, wid, wd, od, ou, os, okeys, lane);
        else
            nv = replay_initial_order<0>(p, v, lv, Cp, deg_self, wid, wd, od, ou, os, okeys, lane);
        __syncwarp(); // the sort keys are read and xid is complete: the cache may be filled
        // cache rows: slot i < deg_self (the row's id, v for an invalid one),
        // then expansion k at row R + k
        const uint32_t *own = p.cur_ids + (uint64_t)v * p.R;
        gather_rows_async<CPL>(p.st.data, p.st.stride, nch, (int)deg_self, cache, p.row_bytes, lane,
                               [&](int r) -> uint32_t {
                                   const uint32_t id = own[r];
                                   return id < N ? id : v;
                               });
        gather_rows_async<CPL>(p.st.data, p.st.stride, nch, (int)cnt, cache + p.R * p.row_bytes, p.row_bytes, lane,
                               [&](int r) -> uint32_t {
                                   const uint32_t id = xid[r];
                                   return id < N ? id : v;
                               });
        gather_rows_async_wait();
        if constexpr (Pairs::kQuad)
        {
            cache_row_norms(cache, p.row_bytes, nch, deg_self, norms, lane);
            cache_row_norms(cache + p.R * p.row_bytes, p.row_bytes, nch, cnt, norms + p.R, lane);
            __syncwarp();
        }
        uint32_t wdeg = deg_self;

        for (uint32_t k = 0; k < cnt; ++k)
        {
            const uint32_t x = xid[k];
            const float dx = xdd[k];
            if (x >= N || x == v)
                continue;
            const uint32_t deg = min(wdeg, C);
            // x's row is read while the row is scanned (unused if x is present)
            pe.load_x(cache + (p.R + k) * p.row_bytes, nch, Pairs::kQuad ? norms[p.R + k] : 0u);
            // already in the row?  and ngt: positions [0, ngt) have d(v,y) > d(v,x)
            bool present = false;
            int ngt = 0;
            if (C <= 128)
            {
#pragma unroll
                for (uint32_t r = 0; r < 4; ++r)
                {
                    const uint32_t i = 32u * r + lane;
                    const uint32_t w = i < deg ? wid[i] : kInvalid;
                    const float o = (int)i < nv ? od[i] : 0.0f;
                    present |= i < deg && w == x;
                    ngt += __popc(__ballot_sync(kFull, (int)i < nv && o > dx));
                }
            }
            else
            {
                for (uint32_t b = 0; b < deg; b += 32)
                {
                    const uint32_t i = b + lane;
                    present |= i < deg && wid[i] == x;
                    ngt += __popc(__ballot_sync(kFull, (int)i < nv && od[i] > dx));
                }
            }
            if (__any_sync(kFull, present))
                continue;
            // occlusion: nearest kept neighbours first
            bool occluded = false;
            for (int b = nv - 1; b >= ngt; b -= Pairs::kPairs)
            {
                const int j = b - pe.pidx;
                const bool act = j >= ngt;
                const uint32_t u = act ? ou[j] : 0u;
                const float d = pe.dist(cache + u * p.row_bytes, nch, norms, u);
                if (lane == 0)
                    pairs += (unsigned long long)min(Pairs::kPairs, b - ngt + 1);
                if (__any_sync(kFull, act && pe.sl == 0 && __fmul_rn(alpha, d) <= dx))
                {
                    occluded = true;
                    break;
                }
            }
            if (occluded)
                continue;
            // victim: the first position from the far end with alpha*d(x,y) <= d(v,y)
            int vj = -1;
            for (int b = 0; b < ngt; b += Pairs::kPairs)
            {
                const int j = b + pe.pidx;
                const bool act = j < ngt;
                const uint32_t u = act ? ou[j] : 0u;
                const float dy = act ? od[j] : 0.0f;
                const float d = pe.dist(cache + u * p.row_bytes, nch, norms, u);
                if (lane == 0)
                    pairs += (unsigned long long)min(Pairs::kPairs, ngt - b);
                const unsigned hit = __ballot_sync(kFull, act && pe.sl == 0 && __fmul_rn(alpha, d) <= dy);
                if (hit)
                {
                    vj = b + (__ffs(hit) - 1) / Pairs::kLanes;
                    break;
                }
            }
            int slot = -1, pr = -1;
            if (vj >= 0)
            {
                slot = os[vj];
                pr = vj;
            }
            else if (deg < C)
            {
                slot = (int)deg;
                wdeg = deg + 1;
            }
            else if (nv > 0 && dx < od[0])
            {
                slot = os[0];
                pr = 0;
            }
            if (slot < 0)
                continue;
            // new position of the slot among the others
            const uint64_t kn = order_key(dx, (uint32_t)slot);
            int pn = 0;
            if (C <= 128)
            {
#pragma unroll
                for (int r = 0; r < 4; ++r)
                {
                    const int j = 32 * r + lane;
                    const bool in = j < nv && j != pr;
                    const uint64_t kj = in ? order_key(od[j], os[j]) : kKeyMax;
                    pn += __popc(__ballot_sync(kFull, in && kj < kn));
                }
            }
            else
            {
                for (int b = 0; b < nv; b += 32)
                {
                    const int j = b + lane;
                    pn += __popc(__ballot_sync(kFull, j < nv && j != pr && order_key(od[j], os[j]) < kn));
                }
            }
            if (pr >= 0)
            {
                // replaced entry moves from pr to pn >= pr: positions (pr, pn] move down one
                for (int c0 = pr; c0 < pn; c0 += 32)
                {
                    const int i = c0 + lane;
                    float dd = 0.0f;
                    uint16_t uu = 0, ss = 0;
                    if (i < pn)
                    {
                        dd = od[i + 1];
                        uu = ou[i + 1];
                        ss = os[i + 1];
                    }
                    __syncwarp();
                    if (i < pn)
                    {
                        od[i] = dd;
                        ou[i] = uu;
                        os[i] = ss;
                    }
                    __syncwarp();
                }
            }
            else
            {
                // appended entry: positions [pn, nv) move up one, from the top
                if (nv > pn)
                {
                    for (int c0 = pn + ((nv - 1 - pn) & ~31); c0 >= pn; c0 -= 32)
                    {
                        const int i = c0 + lane;
                        float dd = 0.0f;
                        uint16_t uu = 0, ss = 0;
                        if (i < nv)
                        {
                            dd = od[i];
                            uu = ou[i];
                            ss = os[i];
                        }
                        __syncwarp();
                        if (i < nv)
                        {
                            od[i + 1] = dd;
                            ou[i + 1] = uu;
                            os[i + 1] = ss;
                        }
                        __syncwarp();
                    }
                }
                ++nv;
            }
            if (lane == 0)
            {
                od[pn] = dx;
                ou[pn] = (uint16_t)(p.R + k);
                os[pn] = (uint16_t)slot;
                wid[slot] = x;
                wd[slot] = dx;
            }
            __syncwarp();
        }
        for (uint32_t i = lane; i < C; i += 32)
        {
            p.work_ids[lv * C + i] = wid[i];
            p.work_dists[lv * C + i] = wd[i];
        }
        if (lane == 0)
            p.work_deg[lv] = wdeg;
        __syncwarp();
    }
    if (lane == 0 && p.counters)
        atomicAdd(&p.counters[2], pairs);
}

// ====================================================================== reverse CSR
// Reverse edges: source rows [s0, s1) of an edge table (row stride
// src_stride, first min(src_deg, R) slots), kept when the target lies in
// [t0, t1); counts and cursors are indexed by target - t0.
static __global__ void rev_count_kernel(const uint32_t *src_ids, uint64_t src_stride, const uint32_t *src_deg, uint32_t N,
                                 uint32_t R, uint32_t s0, uint32_t s1, uint32_t t0, uint32_t t1, uint32_t *cnt)
{
    const uint64_t total = (uint64_t)(s1 - s0) * R;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t src = s0 + (uint32_t)(i / R);
        const uint32_t slot = (uint32_t)(i % R);
        if (slot < min(src_deg[src - s0], R))
        {
            const uint32_t t = src_ids[(uint64_t)(src - s0) * src_stride + slot];
            if (t < N && t != src && t >= t0 && t < t1)
                atomicAdd(&cnt[t - t0], 1u);
        }
    }
}

static __global__ void rev_fill_kernel(const uint32_t *src_ids, uint64_t src_stride, const uint32_t *src_deg, uint32_t N,
                                uint32_t R, uint32_t s0, uint32_t s1, uint32_t t0, uint32_t t1, uint32_t *cursor,
                                uint32_t *rev)
{
    const uint64_t total = (uint64_t)(s1 - s0) * R;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t src = s0 + (uint32_t)(i / R);
        const uint32_t slot = (uint32_t)(i % R);
        if (slot < min(src_deg[src - s0], R))
        {
            const uint32_t t = src_ids[(uint64_t)(src - s0) * src_stride + slot];
            if (t < N && t != src && t >= t0 && t < t1)
                rev[atomicAdd(&cursor[t - t0], 1u)] = src;
        }
    }
}

// Copies the first R slots of the local work rows (and their degrees) into
// rows [v0, v1) of an R-wide edge table, for the all-gather of edge deltas.
static __global__ void pack_work_rows_kernel(const uint32_t *work_ids, const uint32_t *work_deg, uint32_t C, uint32_t R,
                                      uint32_t v0, uint32_t v1, uint32_t *table, uint32_t *table_deg)
{
    const uint64_t total = (uint64_t)(v1 - v0) * R;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint64_t lv = i / R;
        const uint32_t slot = (uint32_t)(i % R);
        table[(v0 + lv) * R + slot] = work_ids[lv * C + slot];
        if (slot == 0)
            table_deg[v0 + lv] = work_deg[lv];
    }
}

// Exclusive scan of n uint32 counts into offsets[0..n] (offsets[n] = total),
// three passes over tiles of kScanTile elements.
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *s_warp, uint32_t &total)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint32_t x = v;
    for (int off = 1; off < 32; off <<= 1)
    {
        const uint32_t y = __shfl_up_sync(kFull, x, off);
        if (lane >= off)
            x += y;
    }
    if (lane == 31)
        s_warp[w] = x;
    __syncthreads();
    if (w == 0)
    {
        uint32_t s = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0u;
        for (int off = 1; off < 32; off <<= 1)
        {
            const uint32_t y = __shfl_up_sync(kFull, s, off);
            if (lane >= off)
                s += y;
        }
        s_warp[lane] = s;
    }
    __syncthreads();
    total = s_warp[31];
    const uint32_t before = w > 0 ? s_warp[w - 1] : 0u;
    __syncthreads();
    return before + x - v;
}

static __global__ void __launch_bounds__(kScanThreads) scan_tile_sums_kernel(const uint32_t *in, uint32_t n,
                                                                      uint32_t *tile_sums)
{
    __shared__ uint32_t s_warp[32];
    const uint64_t base = (uint64_t)blockIdx.x * kScanTile + threadIdx.x * kScanItems;
    uint32_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
        if (base + k < n)
            s += in[base + k];
    uint32_t total;
    block_exclusive_scan(s, s_warp, total);
    if (threadIdx.x == 0)
        tile_sums[blockIdx.x] = total;
}

static __global__ void __launch_bounds__(kScanThreads) scan_tile_offsets_kernel(uint32_t *tile_sums, uint32_t ntiles)
{
    __shared__ uint32_t s_warp[32];
    uint32_t carry = 0;
    for (uint32_t b = 0; b < ntiles; b += kScanThreads)
    {
        const uint32_t i = b + threadIdx.x;
        const uint32_t v = i < ntiles ? tile_sums[i] : 0u;
        uint32_t total;
        const uint32_t ex = block_exclusive_scan(v, s_warp, total);
        if (i < ntiles)
            tile_sums[i] = carry + ex;
        carry += total;
        __syncthreads();
    }
}

static __global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const uint32_t *in, uint32_t n,
                                                                  const uint32_t *tile_offsets, uint32_t *out,
                                                                  uint32_t *cursor)
{
    __shared__ uint32_t s_warp[32];
    const uint64_t base = (uint64_t)blockIdx.x * kScanTile + threadIdx.x * kScanItems;
    uint32_t vals[kScanItems];
    uint32_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
    {
        vals[k] = base + k < n ? in[base + k] : 0u;
        s += vals[k];
    }
    uint32_t total;
    uint32_t ex = block_exclusive_scan(s, s_warp, total) + tile_offsets[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
    {
        if (base + k < n)
        {
            out[base + k] = ex;
            if (cursor)
                cursor[base + k] = ex;
        }
        ex += vals[k];
        if (base + k + 1 == n)
            out[n] = ex;
    }
}

// ====================================================================== reverse merge
struct MergeParams
{
    StoreView st;
    uint32_t C;
    uint32_t *work_ids;
    float *work_dists;
    uint32_t *work_deg;
    const uint32_t *offsets;
    uint32_t *rev; // sorted in place per target by the merge kernels
    uint32_t heavy_cap, heavy_threshold, heavy_sample;
    uint32_t *heavy_list;
    uint32_t *heavy_count;
    uint32_t *huge_list;
    uint32_t *huge_count;
    uint32_t *huge_scratch; // (N+1)/2 words of 16-bit counters per huge-kernel block, all zero
    uint32_t Cp;            // next_pow2(C), >= 32
    uint32_t t0, t1;    // targets handled; offsets[] and the work rows are indexed by t - t0
    uint32_t sort_cap;  // light kernel: segments up to this length
    uint32_t per_warp;  // light kernel smem bytes per warp
    unsigned long long *counters; // [3] reverse distance evaluations
};

constexpr uint32_t kMergeSortCap = 512;
constexpr uint32_t kHeavySortCap = 16384;

__host__ __device__ __forceinline__ uint32_t merge_smem_per_warp(uint32_t C, uint32_t Cp, uint32_t sort_cap)
{
    return align16(4u * sort_cap) + align16(4u * C) + align16(4u * C) + align16(4u * Cp) + 256u + 256u;
}

// ---------------------------------------------------------------- merge core
// The reference merge (src/gpu_vamana_vnew2.cu:1722-1814) walks a target's
// reverse sources in order: a source already in the row is skipped, the
// others are appended while the row has fewer than C entries, then each
// replaces the worst entry (largest distance, lowest slot on ties) when it is
// strictly closer.  Here the sources are in ascending id order.  A source
// that was in the row as the search left it, or repeats the previous source,
// is a no-op in that loop (present, or evicted earlier as the worst and so
// not closer than the current worst), so the "new" sources are filtered in
// parallel first; the sequential part then only compares each new source's
// distance with the cached worst and recomputes the worst after a
// replacement.

struct MergeState
{
    uint32_t deg; // entries in the row (warp-uniform)
    float wv;     // current worst distance, valid when ws >= 0
    int ws;       // its slot, -1 = not computed yet
};

__device__ __forceinline__ void merge_recompute_worst(const float *wd, uint32_t C, MergeState &ms, int lane)
{
    float w = -FLT_MAX;
    int s = -1;
    for (uint32_t i = lane; i < C; i += 32)
        if (wd[i] > w)
        {
            w = wd[i];
            s = (int)i;
        }
    warp_argmax_lowslot(w, s);
    ms.wv = w;
    ms.ws = s;
}

// Applies m new sources (nl/nd, ascending source order) to the row; one warp.
__device__ __forceinline__ void merge_apply(uint32_t *wid, float *wd, uint32_t C, const uint32_t *nl, const float *nd,
                                            int m, MergeState &ms, int lane)
{
    int j = 0;
    if (ms.deg < C)
    {
        const int take = min(m, (int)(C - ms.deg));
        for (int k = lane; k < take; k += 32)
        {
            wid[ms.deg + k] = nl[k];
            wd[ms.deg + k] = nd[k];
        }
        ms.deg += (uint32_t)take;
        j = take;
        __syncwarp();
    }
    if (j >= m)
        return;
    if (ms.ws < 0)
        merge_recompute_worst(wd, C, ms, lane);
    while (j < m)
    {
        int k = -1;
        for (int b = j; b < m; b += 32)
        {
            const int idx = b + lane;
            const unsigned hit = __ballot_sync(kFull, idx < m && nd[idx] < ms.wv);
            if (hit)
            {
                k = b + __ffs(hit) - 1;
                break;
            }
        }
        if (k < 0)
            break;
        if (ms.ws < 0)
            break; // no slot (C == 0 cannot happen; kept for safety)
        if (lane == 0)
        {
            wid[ms.ws] = nl[k];
            wd[ms.ws] = nd[k];
        }
        __syncwarp();
        merge_recompute_worst(wd, C, ms, lane);
        j = k + 1;
    }
}

// Binary search in the sorted initial row ids.
__device__ __forceinline__ bool sorted_contains(const uint32_t *a, int n, uint32_t x)
{
    int lo = 0, hi = n;
    while (lo < hi)
    {
        const int mid = (lo + hi) >> 1;
        if (a[mid] < x)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo < n && a[lo] == x;
}

// Position in the (optionally heavy-cap sampled) processing list -> index
// into the sorted source array (reference :1743-1760).
__device__ __forceinline__ uint32_t merge_list_index(uint32_t k, uint32_t n, uint32_t count, bool sampled)
{
    return sampled ? (uint32_t)(((uint64_t)k * n) / count) : k;
}

__device__ __forceinline__ void merge_list_size(const MergeParams &p, uint32_t n, uint32_t &count, bool &sampled)
{
    count = n;
    sampled = false;
    if (p.heavy_cap && n > p.heavy_threshold)
    {
        count = min(p.heavy_sample, n);
        if (count == 0)
            count = 1;
        sampled = count < n;
    }
}

__device__ __forceinline__ bool merge_is_new(const MergeParams &p, uint32_t t, const uint32_t *srcs, uint32_t n,
                                             uint32_t count, bool sampled, uint32_t k, const uint32_t *rsorted,
                                             int deg0, uint32_t &s)
{
    s = srcs[merge_list_index(k, n, count, sampled)];
    if (s >= p.st.N || s == t)
        return false;
    if (k > 0 && srcs[merge_list_index(k - 1, n, count, sampled)] == s)
        return false;
    return !sorted_contains(rsorted, deg0, s);
}

// Loads the row of target t into smem (wid/wd) plus a sorted copy of its
// first deg0 ids (rsorted, Cp >= C entries); one warp.
__device__ __forceinline__ uint32_t merge_load_row(const MergeParams &p, uint32_t t, uint32_t *wid, float *wd,
                                                   uint32_t *rsorted, uint32_t Cp, int lane)
{
    const uint32_t C = p.C;
    const uint64_t lt = t - p.t0;
    const uint32_t deg0 = min(p.work_deg[lt], C);
    for (uint32_t i = lane; i < Cp; i += 32)
    {
        if (i < C)
        {
            wid[i] = p.work_ids[lt * C + i];
            wd[i] = p.work_dists[lt * C + i];
        }
        rsorted[i] = i < deg0 ? p.work_ids[lt * C + i] : kInvalid;
    }
    __syncwarp();
    warp_sort_u32(rsorted, (int)Cp, lane);
    return deg0;
}

__device__ __forceinline__ void merge_store_row(const MergeParams &p, uint32_t t, const uint32_t *wid, const float *wd,
                                                uint32_t deg, int lane)
{
    const uint32_t C = p.C;
    const uint64_t lt = t - p.t0;
    for (uint32_t i = lane; i < C; i += 32)
    {
        p.work_ids[lt * C + i] = wid[i];
        p.work_dists[lt * C + i] = wd[i];
    }
    if (lane == 0)
        p.work_deg[lt] = deg;
    __syncwarp();
}

// Whole merge of one target by one warp (sources sorted in srcs[0..n)).
template <int DT, int CPL>
__device__ void merge_target_warp(const MergeParams &p, uint32_t t, const uint32_t *srcs, uint32_t n, uint32_t *wid,
                                  float *wd, uint32_t *rsorted, uint32_t *nl, float *nd, int lane,
                                  unsigned long long &evals)
{
    const int gl = lane & 7;
    const uint32_t deg0 = merge_load_row(p, t, wid, wd, rsorted, p.Cp, lane);
    uint32_t count;
    bool sampled;
    merge_list_size(p, n, count, sampled);
    uint4 q[CPL];
    load_frag<CPL>(q, p.st.data + (uint64_t)t * p.st.stride, p.st.nchunks, gl);
    MergeState ms{deg0, -FLT_MAX, -1};
    for (uint32_t b = 0; b < count; b += 64)
    {
        int m = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h)
        {
            const uint32_t k = b + h * 32 + lane;
            uint32_t s = kInvalid;
            const bool keep = k < count && merge_is_new(p, t, srcs, n, count, sampled, k, rsorted, (int)deg0, s);
            const unsigned bm = __ballot_sync(kFull, keep);
            if (keep)
                nl[m + __popc(bm & ((1u << lane) - 1u))] = s;
            m += __popc(bm);
        }
        __syncwarp();
        if (m == 0)
            continue;
        eval_candidates<DT, CPL>(p.st.data, p.st.stride, p.st.nchunks, q, nl, nd, m, lane);
        __syncwarp();
        evals += (lane == 0) ? (unsigned long long)m : 0ull;
        merge_apply(wid, wd, p.C, nl, nd, m, ms, lane);
    }
    merge_store_row(p, t, wid, wd, ms.deg, lane);
}

// Whole merge of one target by a block of kMergeBlock threads: the filter
// and the distance evaluations of each chunk of kMergeChunk sources are
// spread over all warps, warp 0 applies them in order.
constexpr int kMergeBlock = 256;
constexpr int kMergeChunk = 1024;

template <int DT, int CPL>
__device__ void merge_target_block(const MergeParams &p, uint32_t t, const uint32_t *srcs, uint32_t n, uint32_t *wid,
                                   float *wd, uint32_t *rsorted, uint32_t *nl, float *nd, int *wcount,
                                   MergeState &ms, unsigned long long &evals)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    constexpr int W = kMergeBlock / 32;
    constexpr int PER_WARP = kMergeChunk / W;
    const int gl = lane & 7;
    uint32_t deg0 = 0;
    if (w == 0)
    {
        deg0 = merge_load_row(p, t, wid, wd, rsorted, p.Cp, lane);
        if (lane == 0)
        {
            ms.deg = deg0;
            ms.ws = -1;
            ms.wv = -FLT_MAX;
        }
    }
    __syncthreads();
    deg0 = ms.deg;
    uint32_t count;
    bool sampled;
    merge_list_size(p, n, count, sampled);
    uint4 q[CPL];
    load_frag<CPL>(q, p.st.data + (uint64_t)t * p.st.stride, p.st.nchunks, gl);
    for (uint32_t b = 0; b < count; b += kMergeChunk)
    {
        // filter: warp w takes positions [b + w*PER_WARP, b + (w+1)*PER_WARP)
        int m = 0;
        uint32_t mine[PER_WARP / 32];
#pragma unroll
        for (int h = 0; h < PER_WARP / 32; ++h)
        {
            const uint32_t k = b + w * PER_WARP + h * 32 + lane;
            uint32_t s = kInvalid;
            const bool keep = k < count && merge_is_new(p, t, srcs, n, count, sampled, k, rsorted, (int)deg0, s);
            mine[h] = keep ? s : kInvalid;
            m += __popc(__ballot_sync(kFull, keep));
        }
        if (lane == 0)
            wcount[w] = m;
        __syncthreads();
        int off = 0, total = 0;
        for (int i = 0; i < W; ++i)
        {
            if (i < w)
                off += wcount[i];
            total += wcount[i];
        }
#pragma unroll
        for (int h = 0; h < PER_WARP / 32; ++h)
        {
            const bool keep = mine[h] != kInvalid;
            const unsigned bm = __ballot_sync(kFull, keep);
            if (keep)
                nl[off + __popc(bm & ((1u << lane) - 1u))] = mine[h];
            off += __popc(bm);
        }
        __syncthreads();
        if (total == 0)
            continue;
        // distances: warp w evaluates entries [w*ceil, ...)
        const int per = (total + W - 1) / W;
        const int e0 = min(total, w * per), e1 = min(total, e0 + per);
        if (e1 > e0)
            eval_candidates<DT, CPL>(p.st.data, p.st.stride, p.st.nchunks, q, nl + e0, nd + e0, e1 - e0, lane);
        else
            eval_candidates<DT, CPL>(p.st.data, p.st.stride, p.st.nchunks, q, nl, nd, 0, lane);
        __syncthreads();
        if (threadIdx.x == 0)
            evals += (unsigned long long)total;
        if (w == 0)
        {
            MergeState st = ms;
            merge_apply(wid, wd, p.C, nl, nd, total, st, lane);
            if (lane == 0)
                ms = st;
        }
        __syncthreads();
    }
    if (w == 0)
        merge_store_row(p, t, wid, wd, ms.deg, lane);
    __syncthreads();
}

template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads) merge_kernel(MergeParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    uint8_t *b = smem_raw + warp_id_in_block() * p.per_warp;
    uint32_t *buf = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * p.sort_cap);
    uint32_t *wid = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * p.C);
    float *wd = reinterpret_cast<float *>(b);
    b += align16(4u * p.C);
    uint32_t *rsorted = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * p.Cp);
    uint32_t *nl = reinterpret_cast<uint32_t *>(b);
    b += 256;
    float *nd = reinterpret_cast<float *>(b);
    unsigned long long evals = 0;
    for (uint32_t t = p.t0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); t < p.t1;
         t += gridDim.x * kWarpsPerBlock)
    {
        const uint32_t beg = p.offsets[t - p.t0], end = p.offsets[t - p.t0 + 1];
        const uint32_t n = end - beg;
        if (n == 0)
            continue;
        if (n > p.sort_cap)
        {
            if (lane == 0)
                p.heavy_list[atomicAdd(p.heavy_count, 1u)] = t;
            continue;
        }
        const int n2 = max(32, next_pow2((int)n));
        for (int i = lane; i < n2; i += 32)
            buf[i] = (uint32_t)i < n ? p.rev[beg + i] : kInvalid;
        __syncwarp();
        warp_sort_u32(buf, n2, lane);
        merge_target_warp<DT, CPL>(p, t, buf, n, wid, wd, rsorted, nl, nd, lane, evals);
    }
    if (lane == 0 && p.counters)
        atomicAdd(&p.counters[3], evals);
}

__host__ __device__ __forceinline__ uint32_t block_merge_smem_bytes(uint32_t C, uint32_t Cp)
{
    return align16(4u * C) * 2 + align16(4u * Cp) + 8u * kMergeChunk + 64u + 32u;
}

// Carves the block-merge scratch after the sort buffer.
struct BlockMergeSmem
{
    uint32_t *wid, *rsorted, *nl;
    float *wd, *nd;
    int *wcount;
    MergeState *ms;
};

__device__ __forceinline__ BlockMergeSmem carve_block_merge(uint8_t *b, uint32_t C, uint32_t Cp)
{
    BlockMergeSmem m;
    m.wid = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * C);
    m.wd = reinterpret_cast<float *>(b);
    b += align16(4u * C);
    m.rsorted = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * Cp);
    m.nl = reinterpret_cast<uint32_t *>(b);
    b += 4u * kMergeChunk;
    m.nd = reinterpret_cast<float *>(b);
    b += 4u * kMergeChunk;
    m.wcount = reinterpret_cast<int *>(b);
    b += 64u;
    m.ms = reinterpret_cast<MergeState *>(b);
    return m;
}

// Heavy targets (sort_cap < n <= kHeavySortCap sources): one block per
// target, sources sorted in shared memory by the whole block.  Longer
// segments are handed to huge_merge_kernel.
template <int DT, int CPL>
__global__ void __launch_bounds__(kMergeBlock) heavy_merge_kernel(MergeParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint32_t *sbuf = reinterpret_cast<uint32_t *>(smem_raw);
    BlockMergeSmem sm = carve_block_merge(smem_raw + 4u * kHeavySortCap, p.C, p.Cp);
    const uint32_t nheavy = *p.heavy_count;
    unsigned long long evals = 0;
    for (uint32_t h = blockIdx.x; h < nheavy; h += gridDim.x)
    {
        const uint32_t t = p.heavy_list[h];
        const uint32_t beg = p.offsets[t - p.t0], end = p.offsets[t - p.t0 + 1];
        const uint32_t n = end - beg;
        if (n > kHeavySortCap)
        {
            if (threadIdx.x == 0)
                p.huge_list[atomicAdd(p.huge_count, 1u)] = t;
            continue;
        }
        const uint32_t n2 = (uint32_t)next_pow2((int)n);
        for (uint32_t i = threadIdx.x; i < n2; i += blockDim.x)
            sbuf[i] = i < n ? p.rev[beg + i] : kInvalid;
        __syncthreads();
        for (uint32_t size = 2; size <= n2; size <<= 1)
            for (uint32_t j = size >> 1; j > 0; j >>= 1)
            {
                for (uint32_t i = threadIdx.x; i < n2; i += blockDim.x)
                {
                    const uint32_t l = i ^ j;
                    if (l > i)
                    {
                        const uint32_t x = sbuf[i], y = sbuf[l];
                        const bool asc = (i & size) == 0;
                        if (asc ? (x > y) : (x < y))
                        {
                            sbuf[i] = y;
                            sbuf[l] = x;
                        }
                    }
                }
                __syncthreads();
            }
        merge_target_block<DT, CPL>(p, t, sbuf, n, sm.wid, sm.wd, sm.rsorted, sm.nl, sm.nd, sm.wcount, *sm.ms,
                                    evals);
    }
    if (threadIdx.x == 0 && p.counters)
        atomicAdd(&p.counters[3], evals);
}

// Huge targets (more than kHeavySortCap sources, e.g. the medoid in the
// first round, which enters almost every row): the segment is put in
// ascending order in place and merged by the block.  Unless the heavy cap
// samples the segment, repeated sources are no-ops of the merge, so the
// segment is reduced to its distinct sources through a bitmap over source
// ids (N/32 words, a tenth of a pass over the counters below); a sampled
// segment keeps its repeats through a counting sort with 16-bit counters.
// Both live in this block's slice of huge_scratch, kept all-zero between
// uses.
template <int DT, int CPL>
__global__ void __launch_bounds__(kMergeBlock) huge_merge_kernel(MergeParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ uint32_t s_warp[32];
    BlockMergeSmem sm = carve_block_merge(smem_raw, p.C, p.Cp);
    const uint32_t nhuge = *p.huge_count;
    const uint32_t words = (p.st.N + 1u) / 2u;
    const uint32_t bwords = (p.st.N + 31u) / 32u;
    uint32_t *cnt = p.huge_scratch + (uint64_t)blockIdx.x * words;
    unsigned long long evals = 0;
    for (uint32_t h = blockIdx.x; h < nhuge; h += gridDim.x)
    {
        const uint32_t t = p.huge_list[h];
        const uint32_t beg = p.offsets[t - p.t0], end = p.offsets[t - p.t0 + 1];
        uint32_t n = end - beg;
        uint32_t *seg = p.rev + beg;
        uint32_t count;
        bool sampled;
        merge_list_size(p, n, count, sampled);
        if (!sampled)
        {
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
            {
                const uint32_t s = seg[i];
                atomicOr(&cnt[s >> 5], 1u << (s & 31u));
            }
            __syncthreads();
            uint32_t base = 0;
            for (uint32_t w0 = 0; w0 < bwords; w0 += blockDim.x)
            {
                const uint32_t wi = w0 + threadIdx.x;
                const uint32_t v = wi < bwords ? cnt[wi] : 0u;
                uint32_t total;
                uint32_t o = block_exclusive_scan(__popc(v), s_warp, total) + base;
                for (uint32_t r = v; r; r &= r - 1u)
                    seg[o++] = 32u * wi + (uint32_t)(__ffs(r) - 1);
                if (v)
                    cnt[wi] = 0u;
                base += total;
                __syncthreads();
            }
            n = base;
        }
        else
        {
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
            {
                const uint32_t s = seg[i];
                atomicAdd(&cnt[s >> 1], 1u << ((s & 1u) * 16u));
            }
            __syncthreads();
            uint32_t base = 0;
            for (uint32_t w0 = 0; w0 < words; w0 += blockDim.x)
            {
                const uint32_t wi = w0 + threadIdx.x;
                const uint32_t v = wi < words ? cnt[wi] : 0u;
                const uint32_t c0 = v & 0xFFFFu, c1 = v >> 16;
                uint32_t total;
                const uint32_t ex = block_exclusive_scan(c0 + c1, s_warp, total) + base;
                for (uint32_t r = 0; r < c0; ++r)
                    seg[ex + r] = 2u * wi;
                for (uint32_t r = 0; r < c1; ++r)
                    seg[ex + c0 + r] = 2u * wi + 1u;
                if (v)
                    cnt[wi] = 0u;
                base += total;
                __syncthreads();
            }
        }
        __syncthreads();
        merge_target_block<DT, CPL>(p, t, seg, n, sm.wid, sm.wd, sm.rsorted, sm.nl, sm.nd, sm.wcount, *sm.ms, evals);
    }
    if (threadIdx.x == 0 && p.counters)
        atomicAdd(&p.counters[3], evals);
}

// ====================================================================== prune
struct PruneParams
{
    StoreView st;
    uint32_t R, C, Cp; // Cp = next_pow2(C), >= 32
    float alpha;
    uint32_t min_degree;
    const uint32_t *work_ids;
    const float *work_dists;
    const uint32_t *work_deg;
    uint32_t *cur_ids;
    float *cur_dists;
    uint32_t *degree;
    uint32_t v0, v1;
    uint32_t lrow0; // first vertex of the per-rank arrays (work rows, own distance rows)
    uint32_t row_bytes;
    uint32_t per_warp;
    unsigned long long *counters; // [4] pair evaluations
};

__host__ __device__ __forceinline__ uint32_t prune_smem_per_warp(uint32_t C, uint32_t Cp, uint32_t R,
                                                                 uint32_t row_bytes)
{
    return C * row_bytes + align16(8u * Cp) + align16(4u * C) + align16(4u * C) + align16(C) + align16(2u * C) +
           align16(4u * C) + align16(4u * R) + align16(4u * R);  // cache, keys, cid, cd, state, lst, rid, oid, od
}

template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads) prune_kernel(PruneParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const int g = lane >> 3, gl = lane & 7;
    uint8_t *b = smem_raw + warp_id_in_block() * p.per_warp;
    uint8_t *cache = b;
    b += p.C * p.row_bytes;
    uint64_t *keys = reinterpret_cast<uint64_t *>(b);
    b += align16(8u * p.Cp);
    uint32_t *cid = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * p.C);
    float *cd = reinterpret_cast<float *>(b);
    b += align16(4u * p.C);
    uint8_t *state = b; // 0 open, 1 occluded, 2 selected
    b += align16(p.C);
    uint16_t *lst = reinterpret_cast<uint16_t *>(b);
    b += align16(2u * p.C);
    uint32_t *rid = reinterpret_cast<uint32_t *>(b); // row ids by slot
    b += align16(4u * p.C);
    uint32_t *oid = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * p.R);
    float *od = reinterpret_cast<float *>(b);
    const uint32_t N = p.st.N;
    const uint32_t C = p.C;
    unsigned long long pairs = 0;

    for (uint32_t v = p.v0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < p.v1;
         v += gridDim.x * kWarpsPerBlock)
    {
        const uint64_t lv = v - p.lrow0;
        const uint32_t deg = min(p.work_deg[lv], C);
        // Candidates ordered by (distance, slot): the reference's selection order.
        for (uint32_t i = lane; i < p.Cp; i += 32)
        {
            uint64_t key = kKeyMax;
            if (i < deg)
            {
                const uint32_t id = p.work_ids[lv * C + i];
                const float d = p.work_dists[lv * C + i];
                rid[i] = id;
                if (id < N && id != v && d < FLT_MAX)
                    key = ((uint64_t)__float_as_uint(d) << 32) | i;
            }
            keys[i] = key;
        }
        __syncwarp();
        warp_sort_smem_u64(keys, (int)p.Cp, lane);
        // Keep the first occurrence of every id (a selected id removes its
        // copies; an occluded one has occluded copies).
        int m = 0;
        for (uint32_t bb = 0; bb < C; bb += 32)
        {
            const uint32_t j = bb + lane;
            bool keep = false;
            uint32_t id = kInvalid;
            float d = FLT_MAX;
            if (j < C && keys[j] != kKeyMax)
            {
                const uint32_t slot = (uint32_t)(keys[j] & 0xFFFFFFFFu);
                id = rid[slot];
                d = __uint_as_float((uint32_t)(keys[j] >> 32));
                keep = true;
                for (uint32_t jj = 0; jj < j; ++jj)
                {
                    if (rid[(uint32_t)(keys[jj] & 0xFFFFFFFFu)] == id)
                    {
                        keep = false;
                        break;
                    }
                }
            }
            const unsigned bm = __ballot_sync(kFull, keep);
            if (keep)
            {
                const int pos = m + __popc(bm & ((1u << lane) - 1u));
                cid[pos] = id;
                cd[pos] = d;
                state[pos] = 0;
            }
            m += __popc(bm);
        }
        __syncwarp();
        gather_rows_batched<CPL>(p.st.data, p.st.stride, p.st.nchunks, m, cache, p.row_bytes, lane,
                                 [&](int r) -> uint32_t { return cid[r]; });
        __syncwarp();
        uint32_t out = 0;
        for (int j = 0; j < m; ++j)
        {
            if (state[j] != 0)
                continue;
            const float seld = cd[j];
            if (lane == 0)
            {
                state[j] = 2;
                oid[out] = cid[j];
                od[out] = seld;
            }
            ++out;
            __syncwarp();
            if (out >= p.R)
                break;
            int nq = 0;
            for (int bb = j + 1; bb < m; bb += 32)
            {
                const int qq = bb + lane;
                const bool in = qq < m && state[qq] == 0;
                const unsigned bm = __ballot_sync(kFull, in);
                if (in)
                    lst[nq + __popc(bm & ((1u << lane) - 1u))] = (uint16_t)qq;
                nq += __popc(bm);
            }
            __syncwarp();
            if (nq == 0)
                continue;
            uint4 sf[CPL];
            load_frag_smem<CPL>(sf, cache + (uint32_t)j * p.row_bytes, p.st.nchunks, gl);
            for (int bb = 0; bb < nq; bb += 4)
            {
                const int idx = bb + g;
                uint4 c[CPL];
                if (idx < nq)
                    load_frag_smem<CPL>(c, cache + (uint32_t)lst[idx] * p.row_bytes, p.st.nchunks, gl);
                else
                {
#pragma unroll
                    for (int t = 0; t < CPL; ++t)
                        c[t] = make_uint4(0u, 0u, 0u, 0u);
                }
                const float d = GroupDist<DT, CPL>::eval(sf, c, p.st.nchunks, gl);
                if (idx < nq && gl == 0)
                {
                    const int qq = lst[idx];
                    const float dq = cd[qq];
                    if (seld <= dq && __fmul_rn(p.alpha, d) <= dq)
                        state[qq] = 1;
                }
            }
            if (lane == 0)
                pairs += (unsigned long long)nq;
            __syncwarp();
        }
        // Last-round fill: nearest unselected candidates, ignoring occlusion.
        const uint32_t min_deg = min(p.min_degree, p.R);
        if (out < min_deg)
        {
            for (int j = 0; j < m && out < min_deg; ++j)
            {
                if (state[j] == 2)
                    continue;
                if (lane == 0)
                {
                    oid[out] = cid[j];
                    od[out] = cd[j];
                }
                ++out;
            }
            __syncwarp();
        }
        for (uint32_t i = lane; i < p.R; i += 32)
        {
            p.cur_ids[(uint64_t)v * p.R + i] = i < out ? oid[i] : kInvalid;
            p.cur_dists[lv * p.R + i] = i < out ? od[i] : FLT_MAX;
        }
        if (lane == 0)
            p.degree[v] = out;
        __syncwarp();
    }
    if (lane == 0 && p.counters)
        atomicAdd(&p.counters[4], pairs);
}

} // namespace dance
