// prune_quad.cuh -- RobustPrune for float and half vectors, eight pairs per
// warp pass, with the four-lane pair distance QuadDist (dance_common.cuh).
#pragma once

#include "gram_u8.cuh"

namespace dance
{

struct QuadPruneLayout
{
    uint32_t cid, cd, kill, bytes;
    __host__ __device__ QuadPruneLayout(uint32_t C, uint32_t row_bytes)
    {
        const uint32_t Cp = C <= 32 ? 32u : (uint32_t)next_pow2((int)C);
        const uint32_t staging = align16(4u * C) + 8u * Cp;
        const uint32_t cache = C * row_bytes;
        uint32_t o = align16(cache > staging ? cache : staging);
        cid = o;
        o += align16(4u * C);
        cd = o;
        o += align16(4u * C);
        kill = o;
        o += 16u;
        bytes = o;
    }
};

// prune_kernel (reference final_prune_kernel_shared,
// src/gpu_vamana_vnew2.cu:1893-2147) for float and half rows of up to
// 8 T chunks and work rows of up to 128 candidates.  Candidates in
// (distance, slot) order with the first occurrence of each id (copies of an
// id carry the same distance bits, the distance being a fixed function of
// the vertex and the id, so only a run of equal distances is searched); the
// live and selected sets are four words held by every lane.  A selection
// evaluates its row against every live candidate after it, eight pairs a
// pass; the candidates it occludes leave the live set at the end of the
// selection, as in the reference, which tests them all against the same
// selected row.
template <int DT, int T>
__global__ void __launch_bounds__(kBlockThreads) prune_quad_kernel(PruneParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const uint32_t lt = (1u << lane) - 1u;
    const int pidx = lane >> 2, sl = lane & 3;
    const uint32_t C = p.C;
    const uint32_t Cp = C <= 32 ? 32u : (uint32_t)next_pow2((int)C);
    const QuadPruneLayout lay(C, p.row_bytes);
    const uint32_t nch = p.st.nchunks;
    uint8_t *b = smem_raw + warp_id_in_block() * p.per_warp;
    uint8_t *cache = b;
    uint32_t *rid = reinterpret_cast<uint32_t *>(b);
    uint32_t *sd = reinterpret_cast<uint32_t *>(b + align16(4u * C));
    uint32_t *sid = sd + Cp;
    uint32_t *cid = reinterpret_cast<uint32_t *>(b + lay.cid);
    float *cd = reinterpret_cast<float *>(b + lay.cd);
    uint32_t *kill = reinterpret_cast<uint32_t *>(b + lay.kill);
    const float alpha = p.alpha;
    unsigned long long pairs = 0;

    for (uint32_t v = p.v0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < p.v1;
         v += gridDim.x * kWarpsPerBlock)
    {
        const uint64_t lv = v - p.lrow0;
        int nvalid;
        if (Cp == 32)
            nvalid = prune_sorted_list<1>(p, v, lv, Cp, rid, sd, sid, nullptr, lane);
        else if (Cp == 64)
            nvalid = prune_sorted_list<2>(p, v, lv, Cp, rid, sd, sid, nullptr, lane);
        else
            nvalid = prune_sorted_list<4>(p, v, lv, Cp, rid, sd, sid, nullptr, lane);
        // first occurrence of every id, searched within its equal-distance run
        const int nb = (nvalid + 31) >> 5;
        uint32_t keepbits = 0;
        for (int bb = 0; bb < nb; ++bb)
        {
            const int e = bb * 32 + lane;
            const bool valid = e < nvalid;
            const uint32_t db = valid ? sd[e] : 0u;
            const uint32_t id = valid ? sid[e] : 0u;
            bool dup = false, run = valid;
            for (int t = 1; __any_sync(kFull, run); ++t)
            {
                if (run)
                {
                    const int f = e - t;
                    if (f < 0 || sd[f] != db)
                        run = false;
                    else if (sid[f] == id)
                    {
                        dup = true;
                        run = false;
                    }
                }
            }
            if (valid && !dup)
                keepbits |= 1u << bb;
        }
        uint32_t m = 0;
        for (int bb = 0; bb < nb; ++bb)
        {
            const int e = bb * 32 + lane;
            const bool keep = (keepbits >> bb) & 1u;
            const unsigned bm = __ballot_sync(kFull, keep);
            if (keep)
            {
                const uint32_t pos = m + __popc(bm & lt);
                cid[pos] = sid[e];
                cd[pos] = __uint_as_float(sd[e]);
            }
            m += __popc(bm);
        }
        __syncwarp();
        gather_rows_async<(T + 1) / 2>(p.st.data, p.st.stride, nch, (int)m, cache, p.row_bytes, lane,
                                       [&](int r) -> uint32_t { return cid[r]; });
        if (lane < 4)
            kill[lane] = 0u;
        gather_rows_async_wait();
        // greedy selection over uniform bit sets
        uint32_t live[4], selw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int w = 0; w < 4; ++w)
        {
            const uint32_t lo = 32u * (uint32_t)w;
            live[w] = m >= lo + 32u ? 0xFFFFFFFFu : (m > lo ? ((1u << (m - lo)) - 1u) : 0u);
        }
        const uint32_t valid_w[4] = {live[0], live[1], live[2], live[3]};
        uint32_t out = 0;
        while (out < p.R)
        {
            int j = -1;
#pragma unroll
            for (int w = 3; w >= 0; --w)
                if (live[w])
                    j = 32 * w + __ffs(live[w]) - 1;
            if (j < 0)
                break;
#pragma unroll
            for (int w = 0; w < 4; ++w)
            {
                if (w == (j >> 5))
                {
                    live[w] &= ~(1u << (j & 31));
                    selw[w] |= 1u << (j & 31);
                }
            }
            if (++out >= p.R)
                break;
            // every live candidate after j is tested against j (all of them are after j)
            int cnt[4], nq = 0;
#pragma unroll
            for (int w = 0; w < 4; ++w)
            {
                cnt[w] = __popc(live[w]);
                nq += cnt[w];
            }
            if (nq == 0)
                continue;
            uint4 xf[T];
            {
                const uint4 *xr = reinterpret_cast<const uint4 *>(cache + (uint32_t)j * p.row_bytes);
#pragma unroll
                for (int t = 0; t < T; ++t)
                {
                    const uint32_t c = (uint32_t)(sl + 4 * t);
                    xf[t] = c < nch ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
                }
            }
            const float seld = cd[j];
            for (int base = 0; base < nq; base += 8)
            {
                int r = base + pidx;
                const bool act = r < nq;
                int w = 0;
                uint32_t word = live[0];
#pragma unroll
                for (int ww = 0; ww < 3; ++ww)
                {
                    const bool past = r >= cnt[ww] && w == ww;
                    r -= past ? cnt[ww] : 0;
                    w += past ? 1 : 0;
                }
                word = w == 0 ? live[0] : (w == 1 ? live[1] : (w == 2 ? live[2] : live[3]));
                const int q = act ? 32 * w + nth_set_bit(word, r) : j;
                const float d = QuadDist<DT, T>::eval(xf, cache + (uint32_t)q * p.row_bytes, nch, sl);
                const float dq = cd[q];
                if (act && sl == 0 && seld <= dq && __fmul_rn(alpha, d) <= dq)
                    atomicOr(&kill[q >> 5], 1u << (q & 31));
            }
            pairs += (unsigned long long)nq;
            __syncwarp();
#pragma unroll
            for (int w = 0; w < 4; ++w)
                live[w] &= ~kill[w];
            __syncwarp();
            if (lane < 4)
                kill[lane] = 0u;
            __syncwarp();
        }
        // last-round fill: the nearest unselected candidates, ignoring occlusion
        const uint32_t min_deg = min(p.min_degree, p.R);
        uint32_t fillw[4] = {0u, 0u, 0u, 0u};
        uint32_t nfill = 0;
        if (out < min_deg)
        {
            uint32_t need = min_deg - out;
#pragma unroll
            for (int w = 0; w < 4; ++w)
            {
                uint32_t u = valid_w[w] & ~selw[w];
                while (need && u)
                {
                    fillw[w] |= u & (0u - u);
                    u &= u - 1u;
                    --need;
                    ++nfill;
                }
            }
        }
        // output: selected in order, then the fill
        uint32_t spre = 0, fpre = 0;
#pragma unroll
        for (int w = 0; w < 4; ++w)
        {
            const uint32_t j = 32u * (uint32_t)w + (uint32_t)lane;
            const uint32_t bit = 1u << lane;
            uint32_t pos = kInvalid;
            if (selw[w] & bit)
                pos = spre + __popc(selw[w] & lt);
            else if (fillw[w] & bit)
                pos = out + fpre + __popc(fillw[w] & lt);
            if (pos != kInvalid)
            {
                p.cur_ids[(uint64_t)v * p.R + pos] = cid[j];
                p.cur_dists[lv * p.R + pos] = cd[j];
            }
            spre += __popc(selw[w]);
            fpre += __popc(fillw[w]);
        }
        const uint32_t total = out + nfill;
        for (uint32_t i = total + lane; i < p.R; i += 32)
        {
            p.cur_ids[(uint64_t)v * p.R + i] = kInvalid;
            p.cur_dists[lv * p.R + i] = FLT_MAX;
        }
        if (lane == 0)
            p.degree[v] = total;
        __syncwarp();
    }
    if (lane == 0 && p.counters)
        atomicAdd(&p.counters[4], pairs);
}

} // namespace dance
