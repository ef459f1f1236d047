// gram_u8.cuh -- uint8 RobustPrune from tensor-core pair predicates.
//
// For uint8 vectors the squared distance is an exact integer,
//   d(a, b) = |a|^2 + |b|^2 - 2 <a, b>,
// so the prune's candidate-candidate block (C x C x dim, the one dense
// contraction of the build) is one integer Gram matrix of the vertex's
// candidates, computed on the tensor cores with mma.sync m16n8k32
// (u8 x u8 -> s32, exact) and converted to float exactly as the reference
// converts its integer sum.  Each occlusion rule is evaluated once per pair
// and stored as a bit; a selection then clears the candidates it occludes
// with one AND per 32 of them.  The decisions are prune_kernel's.
//
// (The same predicates for the online-insert replay cost more than they
// save: the replay's sequential rule touches about 600 of the 8192 pairs a
// vertex's 128 cached vectors form, so it keeps evaluating them lazily.)
#pragma once

#include "vamana_kernels.cuh"

namespace dance
{

// D += A (16 x 32 u8, row) * B (32 x 8 u8, col), s32 accumulate (PTX ISA mma.m16n8k32).
__device__ __forceinline__ void mma_u8_16x8x32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

// Cache row stride of the Gram kernels: rows padded to a multiple of 32
// bytes (the MMA's K step) plus 16 bytes, so that the eight rows an MMA
// fragment load touches fall into eight different bank groups.
__host__ __device__ __forceinline__ uint32_t gram_kbytes(uint32_t row_bytes) { return (row_bytes + 31u) & ~31u; }
__host__ __device__ __forceinline__ uint32_t gram_stride(uint32_t row_bytes) { return gram_kbytes(row_bytes) + 16u; }

// Zero the K padding [row_bytes, kbytes) of cache rows [0, n).
__device__ __forceinline__ void gram_zero_pad(uint8_t *cache, uint32_t S, uint32_t row_bytes, uint32_t n, int lane)
{
    if (gram_kbytes(row_bytes) == row_bytes)
        return;
    for (uint32_t r = lane; r < n; r += 32)
        *reinterpret_cast<uint4 *>(cache + r * S + row_bytes) = make_uint4(0u, 0u, 0u, 0u);
}

// Squared norms of cache rows [0, n) (exact).
__device__ __forceinline__ void gram_norms(const uint8_t *cache, uint32_t S, uint32_t kbytes, uint32_t n,
                                           uint32_t *norms, int lane)
{
    for (uint32_t r = lane; r < n; r += 32)
    {
        const uint8_t *row = cache + r * S;
        uint32_t acc = 0;
        for (uint32_t i = 0; i < kbytes; i += 4)
        {
            const uint32_t w = lds32(row + i);
            acc = __dp4a(w, w, acc);
        }
        norms[r] = acc;
    }
}

// For cache rows 0 .. m (each both a row and a column of the Gram matrix),
// calls pred(row, col, dist) -> bool for every pair with col > row and
// stores the result as natural-order bit masks: row j's word w holds
// columns 32w .. 32w+31, W words per row, bits at or below the diagonal 0.
// All lanes call.  The 16-row MMA tiles read rows up to round_up(m, 16) and
// the 8-column tiles up to round_up(m, 32): those must lie inside the cache.
template <class Pred>
__device__ __forceinline__ void gram_upper_masks(const uint8_t *cache, uint32_t S, uint32_t kbytes,
                                                 const uint32_t *norms, uint32_t m, uint32_t W, uint32_t *mask,
                                                 Pred pred, int lane)
{
    const uint32_t gq = (uint32_t)lane >> 2, tq = (uint32_t)lane & 3u;
    const uint32_t words = (m + 31u) >> 5;
    for (uint32_t mt = 0; mt < m; mt += 16)
    {
        const uint32_t rg = mt + gq, rh = mt + gq + 8; // this lane's rows (MMA fragment layout)
        const uint8_t *pa = cache + rg * S + 4u * tq;
        const uint8_t *ph = cache + rh * S + 4u * tq;
        const bool vg = rg < m, vh = rh < m;
        const uint32_t ng = vg ? norms[rg] : 0u, nh = vh ? norms[rh] : 0u;
        for (uint32_t w = 0; w < words; ++w)
        {
            uint32_t bg = 0, bh = 0;
            for (uint32_t jj = 0; jj < 4; ++jj)
            {
                const uint32_t c0 = w * 32u + jj * 8u; // first column of this 8-column tile
                if (c0 >= m)
                    break;
                if (c0 + 7u <= mt) // every column of the tile <= every row of the tile
                    continue;
                int acc[4] = {0, 0, 0, 0};
                const uint8_t *pb = cache + (c0 + gq) * S + 4u * tq;
                for (uint32_t o = 0; o < kbytes; o += 32)
                    mma_u8_16x8x32(acc, lds32(pa + o), lds32(ph + o), lds32(pa + o + 16), lds32(ph + o + 16),
                                   lds32(pb + o), lds32(pb + o + 16));
#pragma unroll
                for (uint32_t e = 0; e < 2; ++e)
                {
                    const uint32_t col = c0 + 2u * tq + e; // acc[e]: (rg, col), acc[2+e]: (rh, col)
                    if (col >= m)
                        continue;
                    const uint32_t bit = 1u << (jj * 8u + 2u * tq + e);
                    const uint32_t nc = norms[col];
                    if (vg && col > rg && pred(rg, col, (float)(int32_t)(ng + nc - 2u * (uint32_t)acc[e])))
                        bg |= bit;
                    if (vh && col > rh && pred(rh, col, (float)(int32_t)(nh + nc - 2u * (uint32_t)acc[2 + e])))
                        bh |= bit;
                }
            }
            bg |= __shfl_xor_sync(kFull, bg, 1);
            bg |= __shfl_xor_sync(kFull, bg, 2);
            bh |= __shfl_xor_sync(kFull, bh, 1);
            bh |= __shfl_xor_sync(kFull, bh, 2);
            if (tq == 0)
            {
                if (vg)
                    mask[rg * W + w] = bg;
                if (vh)
                    mask[rh * W + w] = bh;
            }
        }
    }
}

__device__ __forceinline__ bool mask_bit(const uint32_t *row, uint32_t c) { return (row[c >> 5] >> (c & 31u)) & 1u; }

__host__ __device__ __forceinline__ uint32_t gram_prune_rows(uint32_t C) { return (C + 31u) & ~31u; }

__host__ __device__ __forceinline__ uint32_t gram_prune_smem_per_warp(uint32_t C, uint32_t Cp, uint32_t R,
                                                                    uint32_t row_bytes)
{
    const uint32_t rows = gram_prune_rows(C), W = rows / 32u;
    return rows * gram_stride(row_bytes) + align16(8u * Cp) + align16(4u * C) + align16(4u * C) +
           align16(4u * C) + align16(4u * rows) + align16(4u * C * W) + 2u * align16(4u * W) + align16(4u * R) +
           align16(4u * R); // cache, keys, rid, cid, cd, norms, occlusion masks, live, selected, oid, od
}

// prune_kernel (reference final_prune_kernel_shared,
// src/gpu_vamana_vnew2.cu:1893-2147) for uint8 vectors: bit occ[j][q] =
// d(v,j) <= d(v,q) and alpha*d(j,q) <= d(v,q) for q after j in selection
// order; a selection clears its occluded candidates with one AND per word.
template <int CPL>
__global__ void __launch_bounds__(kBlockThreads) prune_gram_kernel(PruneParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const uint32_t C = p.C;
    const uint32_t rows = gram_prune_rows(C), W = rows / 32u;
    const uint32_t Sg = gram_stride(p.row_bytes), kbytes = gram_kbytes(p.row_bytes);
    uint8_t *b = smem_raw + warp_id_in_block() * p.per_warp;
    uint8_t *cache = b;
    b += rows * Sg;
    uint64_t *keys = reinterpret_cast<uint64_t *>(b);
    b += align16(8u * p.Cp);
    uint32_t *rid = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * C);
    uint32_t *cid = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * C);
    float *cd = reinterpret_cast<float *>(b);
    b += align16(4u * C);
    uint32_t *norms = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * rows);
    uint32_t *occ = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * C * W);
    uint32_t *live = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * W);
    uint32_t *sel = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * W);
    uint32_t *oid = reinterpret_cast<uint32_t *>(b);
    b += align16(4u * p.R);
    float *od = reinterpret_cast<float *>(b);
    const uint32_t N = p.st.N;
    const float alpha = p.alpha;
    unsigned long long pairs = 0;

    for (uint32_t v = p.v0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < p.v1;
         v += gridDim.x * kWarpsPerBlock)
    {
        const uint64_t lv = v - p.lrow0;
        const uint32_t deg = min(p.work_deg[lv], C);
        // candidates ordered by (distance, slot): the reference's selection order
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
        // first occurrence of every id
        uint32_t m = 0;
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
                const uint32_t pos = m + __popc(bm & ((1u << lane) - 1u));
                cid[pos] = id;
                cd[pos] = d;
            }
            m += __popc(bm);
        }
        __syncwarp();
        gather_rows_grouped<CPL>(p.st.data, p.st.stride, p.st.nchunks, cid, (int)m, cache, Sg, lane);
        gram_zero_pad(cache, Sg, p.row_bytes, m, lane);
        __syncwarp();
        gram_norms(cache, Sg, kbytes, m, norms, lane);
        __syncwarp();
        if (m)
            gram_upper_masks(cache, Sg, kbytes, norms, m, W, occ,
                             [&](uint32_t j, uint32_t q2, float d) -> bool {
                                 return cd[j] <= cd[q2] && __fmul_rn(alpha, d) <= cd[q2];
                             },
                             lane);
        for (uint32_t w = lane; w < W; w += 32)
        {
            const uint32_t lo = w * 32u;
            live[w] = m >= lo + 32u ? 0xFFFFFFFFu : (m > lo ? ((1u << (m - lo)) - 1u) : 0u);
            sel[w] = 0;
        }
        __syncwarp();
        uint32_t out = 0;
        while (out < p.R)
        {
            // next live candidate in selection order
            int j = -1;
            for (uint32_t w0 = 0; w0 < W && j < 0; w0 += 32)
            {
                const uint32_t w = w0 + lane;
                const uint32_t word = w < W ? live[w] : 0u;
                const unsigned nz = __ballot_sync(kFull, word != 0u);
                if (nz)
                {
                    const int l = __ffs(nz) - 1;
                    const uint32_t wv = __shfl_sync(kFull, word, l);
                    j = (int)((w0 + l) * 32u) + __ffs(wv) - 1;
                }
            }
            if (j < 0)
                break;
            if (lane == 0)
            {
                oid[out] = cid[j];
                od[out] = cd[j];
                live[j >> 5] &= ~(1u << (j & 31));
                sel[j >> 5] |= 1u << (j & 31);
            }
            ++out;
            __syncwarp();
            if (out >= p.R)
                break;
            // the open candidates after j are the pairs the reference evaluates
            uint32_t open = 0;
            for (uint32_t w = lane; w < W; w += 32)
            {
                open += __popc(live[w]);
                live[w] &= ~occ[(uint32_t)j * W + w];
            }
            open = __reduce_add_sync(kFull, open);
            if (lane == 0)
                pairs += (unsigned long long)open;
            __syncwarp();
        }
        // last-round fill: nearest unselected candidates, ignoring occlusion
        const uint32_t min_deg = min(p.min_degree, p.R);
        for (uint32_t bb = 0; bb < m && out < min_deg; bb += 32)
        {
            const uint32_t j = bb + lane;
            const bool free_ = j < m && !mask_bit(sel, j);
            const unsigned bm = __ballot_sync(kFull, free_);
            const uint32_t rank = __popc(bm & ((1u << lane) - 1u));
            if (free_ && out + rank < min_deg)
            {
                oid[out + rank] = cid[j];
                od[out + rank] = cd[j];
            }
            out = min(min_deg, out + (uint32_t)__popc(bm));
        }
        __syncwarp();
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
