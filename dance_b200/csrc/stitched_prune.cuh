// stitched_prune.cuh -- label-aware global prune of a stitched union graph.
//
// When rows carry more than one label (or Rsmall > Rstitched) the reference
// stitched app hands the union graph to DiskANN's CPU prune
// (apps/utils/gpu_stitched_vamana_index.cpp:353-372: Index::load,
// prune_all_neighbors(Rstitched, 750, alpha), save).  That prune, with the
// two changes the DANCE integration patch makes to it, is restated here as a
// GPU kernel, one warp per row:
//  * a row with at most `range` neighbours is left as it is;
//  * otherwise the pool is the row's distinct neighbours other than the row
//    itself with their distance to it, ordered by (distance, id);
//  * when the row has labels and the pool is longer than `range`, the pool
//    is first cut to a label-balanced shortlist (patch lines 20055-20100):
//    for every label of the row its first max(1, range / #labels) carriers
//    in pool order, then further pool entries in order until `range` are
//    kept;
//  * the kept entries, at most max_candidates of them, go through DiskANN's
//    occlusion loop: passes with a = 1, 1.2, 1.44, ... while a <= alpha; an
//    entry whose occlusion factor is <= a is selected (the row's own id is
//    never output), and selecting s raises the factor of every later entry x
//    whose factor is <= alpha to max(factor, d(row, x) / d(s, x)) -- to
//    FLT_MAX when d(s, x) = 0 -- but only when s carries every label that
//    the row and x have in common (the FilteredRobustPrune rule of patch
//    lines 20009-20047); at most `range` entries are selected.
// Distances are this library's warp arithmetic (GroupDist), the same as the
// builder's, so the oracle restatement reproduces the output bit for bit.
#pragma once

#include "vamana_kernels.cuh"

namespace dance
{

constexpr uint32_t kStitchedPruneMaxDegree = 2048; // pool rows of one warp in shared memory

struct StitchedPruneParams
{
    StoreView st;
    const uint64_t *row_off; // N + 1
    const uint32_t *row_ids;
    const uint32_t *lab_off; // point label CSR (N + 1), labels ascending per point; may be null (no labels)
    const uint32_t *labs;
    uint32_t range, maxc, pcap;
    float alpha;
    uint32_t *out_rows; // N x range, INVALID padded
    uint32_t *out_deg;  // N
    unsigned long long *pruned_rows;
};

__host__ __device__ __forceinline__ uint32_t stitched_prune_smem_per_warp(uint32_t pcap)
{
    return pcap * 8u + pcap * 4u + align16(pcap);
}

// Point p carries label l (labels of a point ascend).
__device__ __forceinline__ bool sp_has_label(const uint32_t *off, const uint32_t *lab, uint32_t p, uint32_t l)
{
    uint32_t lo = off[p], hi = off[p + 1];
    while (lo < hi)
    {
        const uint32_t mid = (lo + hi) >> 1;
        const uint32_t x = lab[mid];
        if (x == l)
            return true;
        if (x < l)
            lo = mid + 1;
        else
            hi = mid;
    }
    return false;
}

// s carries every label that t and x have in common.
__device__ __forceinline__ bool sp_covers(const uint32_t *off, const uint32_t *lab, uint32_t t, uint32_t s,
                                          uint32_t x)
{
    uint32_t i = off[t], ie = off[t + 1], j = off[x], je = off[x + 1];
    while (i < ie && j < je)
    {
        const uint32_t a = lab[i], b = lab[j];
        if (a < b)
            ++i;
        else if (b < a)
            ++j;
        else
        {
            if (!sp_has_label(off, lab, s, a))
                return false;
            ++i;
            ++j;
        }
    }
    return true;
}

template <int DT, int CPL>
__global__ void __launch_bounds__(kBlockThreads) stitched_prune_kernel(StitchedPruneParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const int g = lane >> 3, gl = lane & 7;
    const unsigned lt = (1u << lane) - 1u;
    uint8_t *base = smem_raw + warp_id_in_block() * stitched_prune_smem_per_warp(p.pcap);
    uint64_t *keys = reinterpret_cast<uint64_t *>(base);             // pcap
    float *occ = reinterpret_cast<float *>(base + 8u * p.pcap);      // pcap
    uint8_t *mark = base + 12u * p.pcap;                             // pcap
    const StoreView &st = p.st;
    const uint32_t N = st.N;
    const bool have_labels = p.lab_off != nullptr;
    unsigned long long pruned = 0;

    for (uint32_t v = blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < N; v += gridDim.x * kWarpsPerBlock)
    {
        const uint64_t b0 = p.row_off[v];
        const uint32_t deg = (uint32_t)(p.row_off[v + 1] - b0);
        uint32_t *out = p.out_rows + (uint64_t)v * p.range;
        if (deg <= p.range)
        {
            for (uint32_t i = lane; i < p.range; i += 32)
                out[i] = i < deg ? p.row_ids[b0 + i] : kInvalid;
            if (lane == 0)
                p.out_deg[v] = deg;
            continue;
        }
        ++pruned;
        // ---- pool: (distance, id) keys of the distinct neighbours other than v
        uint4 q[CPL];
        load_frag<CPL>(q, st.data + (uint64_t)v * st.stride, st.nchunks, gl);
        const int n2 = max(32, next_pow2((int)deg));
        for (int base_i = 0; base_i < n2; base_i += 32)
        {
            const int i = base_i + lane;
            const uint32_t id = i < (int)deg ? p.row_ids[b0 + i] : kInvalid;
            keys[i] = (id < N && id != v) ? (uint64_t)id : kKeyMax; // id only for now
        }
        __syncwarp();
        for (int i0 = 0; i0 < (int)deg; i0 += 4)
        {
            const int i = i0 + g;
            const uint64_t k = i < (int)deg ? keys[i] : kKeyMax;
            uint4 c[CPL];
            if (k != kKeyMax)
                load_frag<CPL>(c, st.data + k * st.stride, st.nchunks, gl);
            else
            {
#pragma unroll
                for (int t = 0; t < CPL; ++t)
                    c[t] = make_uint4(0u, 0u, 0u, 0u);
            }
            const float d = GroupDist<DT, CPL>::eval(q, c, st.nchunks, gl);
            __syncwarp();
            if (gl == 0 && k != kKeyMax)
                keys[i] = make_key(d, (uint32_t)k);
            __syncwarp();
        }
        warp_sort_smem_u64(keys, n2, lane);
        // distinct keys (a repeated id has the same distance, so copies are adjacent)
        int P = 0;
        for (int base_i = 0; base_i < n2; base_i += 32)
        {
            const int i = base_i + lane;
            const uint64_t k = keys[i];
            const bool keep = k != kKeyMax && (i == 0 || keys[i - 1] != k);
            const unsigned m = __ballot_sync(kFull, keep);
            __syncwarp();
            if (keep)
                keys[P + __popc(m & lt)] = k; // P + rank <= i: never overwrites an unread key
            P += __popc(m);
            __syncwarp();
        }
        // ---- label-balanced shortlist
        const uint32_t nlab = have_labels ? p.lab_off[v + 1] - p.lab_off[v] : 0u;
        if (nlab > 0 && P > (int)p.range)
        {
            for (int i = lane; i < P; i += 32)
                mark[i] = 0;
            __syncwarp();
            const uint32_t quota = max(1u, p.range / nlab);
            for (uint32_t li = 0; li < nlab; ++li)
            {
                const uint32_t l = p.labs[p.lab_off[v] + li];
                uint32_t seen = 0;
                for (int base_i = 0; base_i < P && seen < quota; base_i += 32)
                {
                    const int i = base_i + lane;
                    const bool carrier = i < P && sp_has_label(p.lab_off, p.labs, key_id(keys[i]), l);
                    const unsigned m = __ballot_sync(kFull, carrier);
                    if (carrier && seen + (uint32_t)__popc(m & lt) < quota)
                        mark[i] = 1;
                    seen += (uint32_t)__popc(m);
                }
                __syncwarp();
            }
            int kept = 0;
            for (int base_i = 0; base_i < P; base_i += 32)
            {
                const int i = base_i + lane;
                kept += __popc(__ballot_sync(kFull, i < P && mark[i]));
            }
            for (int base_i = 0; base_i < P && kept < (int)p.range; base_i += 32)
            {
                const int i = base_i + lane;
                const bool free_i = i < P && !mark[i];
                const unsigned m = __ballot_sync(kFull, free_i);
                if (free_i && kept + __popc(m & lt) < (int)p.range)
                    mark[i] = 1;
                kept += min(__popc(m), (int)p.range - kept);
            }
            __syncwarp();
            int P2 = 0;
            for (int base_i = 0; base_i < P; base_i += 32)
            {
                const int i = base_i + lane;
                const bool keep = i < P && mark[i];
                const uint64_t k = keep ? keys[i] : 0ull;
                const unsigned m = __ballot_sync(kFull, keep);
                __syncwarp();
                if (keep)
                    keys[P2 + __popc(m & lt)] = k;
                P2 += __popc(m);
                __syncwarp();
            }
            P = P2;
        }
        P = min(P, (int)p.maxc);
        // ---- occlusion passes
        for (int i = lane; i < P; i += 32)
            occ[i] = 0.0f;
        __syncwarp();
        uint32_t nres = 0;
        float cur = 1.0f;
        while (cur <= p.alpha && nres < p.range)
        {
            for (int i = 0; i < P && nres < p.range; ++i)
            {
                if (occ[i] > cur)
                    continue;
                const uint64_t ki = keys[i];
                const uint32_t s = key_id(ki);
                __syncwarp();
                if (lane == 0)
                    occ[i] = FLT_MAX;
                if (s != v)
                {
                    if (lane == 0)
                        out[nres] = s;
                    ++nres;
                }
                __syncwarp();
                uint4 sf[CPL];
                load_frag<CPL>(sf, st.data + (uint64_t)s * st.stride, st.nchunks, gl);
                for (int j0 = i + 1; j0 < P; j0 += 32)
                {
                    const int j = j0 + lane;
                    bool need = j < P && occ[j] <= p.alpha;
                    if (need && have_labels)
                        need = sp_covers(p.lab_off, p.labs, v, s, key_id(keys[j]));
                    const unsigned m = __ballot_sync(kFull, need);
                    // the needed entries of this chunk, four pair distances per pass
                    for (int r = 0; r < __popc(m); r += 4)
                    {
                        const int t = r + g;
                        const int jj = t < __popc(m) ? j0 + (int)__fns(m, 0u, t + 1) : -1;
                        uint4 c[CPL];
                        if (jj >= 0)
                            load_frag<CPL>(c, st.data + (uint64_t)key_id(keys[jj]) * st.stride, st.nchunks, gl);
                        else
                        {
#pragma unroll
                            for (int z = 0; z < CPL; ++z)
                                c[z] = make_uint4(0u, 0u, 0u, 0u);
                        }
                        const float djk = GroupDist<DT, CPL>::eval(sf, c, st.nchunks, gl);
                        if (jj >= 0 && gl == 0)
                        {
                            const float dj = key_dist(keys[jj]);
                            occ[jj] = djk == 0.0f ? FLT_MAX : fmaxf(occ[jj], __fdiv_rn(dj, djk));
                        }
                    }
                    __syncwarp();
                }
            }
            cur = __fmul_rn(cur, 1.2f);
        }
        for (uint32_t i = nres + lane; i < p.range; i += 32)
            out[i] = kInvalid;
        if (lane == 0)
            p.out_deg[v] = nres;
        __syncwarp();
    }
    if (lane == 0 && p.pruned_rows && pruned)
        atomicAdd(p.pruned_rows, pruned);
}

// Largest row degree of a CSR graph.
static __global__ void csr_max_degree_kernel(const uint64_t *row_off, uint32_t N, uint32_t *out)
{
    uint32_t m = 0;
    for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < N; v += gridDim.x * blockDim.x)
        m = max(m, (uint32_t)(row_off[v + 1] - row_off[v]));
    for (int o = 16; o; o >>= 1)
        m = max(m, __shfl_xor_sync(kFull, m, o));
    if ((threadIdx.x & 31) == 0 && m)
        atomicMax(out, m);
}

template <int DT, int CPL>
struct LaunchStitchedPrune
{
    static int run(const StitchedPruneParams &p, cudaStream_t s)
    {
        const size_t smem = (size_t)kWarpsPerBlock * stitched_prune_smem_per_warp(p.pcap);
        auto k = stitched_prune_kernel<DT, CPL>;
        DANCE_CUDA(allow_smem(k, smem));
        int per_sm = 0;
        DANCE_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kBlockThreads, smem));
        const uint64_t need = (p.st.N + kWarpsPerBlock - 1) / kWarpsPerBlock;
        const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>(need, (uint64_t)std::max(per_sm, 1) *
                                                                                  sm_count()));
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }
};

} // namespace dance
