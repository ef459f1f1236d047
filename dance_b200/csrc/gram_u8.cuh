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

// Rows of the prune's vector cache: the 16-row MMA tiles and 8-column tiles
// of gram_prune_masks read rows up to round_up(m, 16) <= round_up(C, 16).
__host__ __device__ __forceinline__ uint32_t gram_prune_rows(uint32_t C) { return (C + 15u) & ~15u; }

// Per-warp scratch of prune_gram_kernel.  Before the gather the cache holds
// the slot -> id map and the sorted candidate list (distance bits, id).
struct GramPruneLayout
{
    uint32_t rows, W, cid, cd, norms, occ, bytes, staging;
    __host__ __device__ GramPruneLayout(uint32_t C, uint32_t row_bytes)
    {
        const uint32_t Cp = C <= 32 ? 32u : (uint32_t)next_pow2((int)C);
        rows = gram_prune_rows(C);
        W = (C + 31u) / 32u;
        uint32_t o = rows * gram_stride(row_bytes);
        // rid (C) + sorted distance bits (Cp) + sorted ids (Cp), and for
        // Cp > 128 the 64-bit sort keys (Cp) as well
        staging = align16(4u * C) + 8u * Cp + (Cp > 128u ? 8u * Cp : 0u);
        cid = o;
        o += align16(4u * rows);
        cd = o;
        o += align16(4u * rows);
        norms = o;
        o += align16(4u * rows);
        occ = o;
        o += align16(4u * rows * W);
        bytes = o;
    }
};

// Candidate list of vertex v in the reference's selection order: work-row
// slots with a valid id (not v) and a finite distance, sorted by (distance,
// slot), written as sd[e] (distance bits) and sid[e] (id).  Returns their
// number.  NPL = Cp / 32 keys per lane are sorted in registers; NPL = 0 sorts
// Cp keys in shared memory.
template <int NPL>
__device__ __forceinline__ int prune_sorted_list(const PruneParams &p, uint32_t v, uint64_t lv, uint32_t Cp,
                                                 uint32_t *rid, uint32_t *sd, uint32_t *sid, uint64_t *skeys,
                                                 int lane)
{
    const uint32_t C = p.C, N = p.st.N;
    const uint32_t deg = min(p.work_deg[lv], C);
    int nvalid = 0;
    if constexpr (NPL > 0)
    {
        uint64_t k[NPL];
#pragma unroll
        for (int s = 0; s < NPL; ++s)
        {
            const uint32_t i = (uint32_t)(lane * NPL + s);
            uint64_t key = kKeyMax;
            if (i < deg)
            {
                const uint32_t id = p.work_ids[lv * C + i];
                const float d = p.work_dists[lv * C + i];
                rid[i] = id;
                if (id < N && id != v && d < FLT_MAX)
                    key = ((uint64_t)__float_as_uint(d) << 32) | i;
            }
            k[s] = key;
        }
        __syncwarp();
        warp_sort_blocked<NPL>(k, lane);
#pragma unroll
        for (int s = 0; s < NPL; ++s)
        {
            const uint32_t e = (uint32_t)(lane * NPL + s);
            const bool valid = k[s] != kKeyMax;
            if (valid)
            {
                sd[e] = (uint32_t)(k[s] >> 32);
                sid[e] = rid[(uint32_t)(k[s] & 0xFFFFFFFFu)];
            }
            nvalid += __popc(__ballot_sync(kFull, valid));
        }
    }
    else
    {
        for (uint32_t i = lane; i < Cp; i += 32)
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
            skeys[i] = key;
        }
        __syncwarp();
        warp_sort_smem_u64(skeys, (int)Cp, lane);
        for (uint32_t e = lane; e < Cp; e += 32)
        {
            const uint64_t key = skeys[e];
            const bool valid = key != kKeyMax;
            if (valid)
            {
                sd[e] = (uint32_t)(key >> 32);
                sid[e] = rid[(uint32_t)(key & 0xFFFFFFFFu)];
            }
            nvalid += __popc(__ballot_sync(kFull, valid));
        }
    }
    __syncwarp();
    return nvalid;
}

// Occlusion bit masks from the Gram matrix of cache rows 0 .. m: bit q of row
// j (row stride W words) is alpha * d(j, q) <= cd[q].  Only bits q > j, q < m
// are meaningful (the selection never reads the others); words entirely
// below a row tile are not written.  HOIST keeps the tile's A fragments in
// registers (rows of at most 128 bytes).
template <bool HOIST>
__device__ __forceinline__ void gram_prune_masks(const uint8_t *cache, uint32_t S, uint32_t kbytes,
                                                 const uint32_t *norms, const float *cd, uint32_t m, uint32_t W,
                                                 uint32_t *occ, float alpha, int lane)
{
    const uint32_t gq = (uint32_t)lane >> 2, tq = (uint32_t)lane & 3u;
    const uint32_t words = (m + 31u) >> 5;
    for (uint32_t mt = 0; mt < m; mt += 16)
    {
        const uint32_t rg = mt + gq, rh = mt + gq + 8;
        const uint8_t *pa = cache + rg * S + 4u * tq;
        const uint8_t *ph = cache + rh * S + 4u * tq;
        const uint32_t ng = norms[rg], nh = norms[rh];
        uint32_t af[4][4];
        if constexpr (HOIST)
        {
#pragma unroll
            for (int o4 = 0; o4 < 4; ++o4)
            {
                const uint32_t o = 32u * (uint32_t)o4;
                const bool in = o < kbytes;
                af[o4][0] = in ? lds32(pa + o) : 0u;
                af[o4][1] = in ? lds32(ph + o) : 0u;
                af[o4][2] = in ? lds32(pa + o + 16) : 0u;
                af[o4][3] = in ? lds32(ph + o + 16) : 0u;
            }
        }
        for (uint32_t w = mt >> 5; w < words; ++w)
        {
            uint32_t bg = 0, bh = 0;
            for (uint32_t jj = 0; jj < 4; ++jj)
            {
                const uint32_t c0 = w * 32u + jj * 8u;
                if (c0 >= m)
                    break;
                if (c0 + 7u <= mt)
                    continue;
                int acc[4] = {0, 0, 0, 0};
                const uint8_t *pb = cache + (c0 + gq) * S + 4u * tq;
                if constexpr (HOIST)
                {
#pragma unroll
                    for (int o4 = 0; o4 < 4; ++o4)
                    {
                        const uint32_t o = 32u * (uint32_t)o4;
                        if (o < kbytes)
                            mma_u8_16x8x32(acc, af[o4][0], af[o4][1], af[o4][2], af[o4][3], lds32(pb + o),
                                           lds32(pb + o + 16));
                    }
                }
                else
                {
                    for (uint32_t o = 0; o < kbytes; o += 32)
                        mma_u8_16x8x32(acc, lds32(pa + o), lds32(ph + o), lds32(pa + o + 16), lds32(ph + o + 16),
                                       lds32(pb + o), lds32(pb + o + 16));
                }
#pragma unroll
                for (uint32_t e = 0; e < 2; ++e)
                {
                    const uint32_t col = c0 + 2u * tq + e; // acc[e]: (rg, col), acc[2+e]: (rh, col)
                    const uint32_t bit = 1u << (jj * 8u + 2u * tq + e);
                    const uint32_t nc = norms[col];
                    const float lim = cd[col];
                    if (__fmul_rn(alpha, (float)(int32_t)(ng + nc - 2u * (uint32_t)acc[e])) <= lim)
                        bg |= bit;
                    if (__fmul_rn(alpha, (float)(int32_t)(nh + nc - 2u * (uint32_t)acc[2 + e])) <= lim)
                        bh |= bit;
                }
            }
            bg |= __shfl_xor_sync(kFull, bg, 1);
            bg |= __shfl_xor_sync(kFull, bg, 2);
            bh |= __shfl_xor_sync(kFull, bh, 1);
            bh |= __shfl_xor_sync(kFull, bh, 2);
            if (tq == 0)
            {
                occ[rg * W + w] = bg;
                occ[rh * W + w] = bh;
            }
        }
    }
}

__host__ __device__ __forceinline__ uint32_t gram_prune_smem_per_warp(uint32_t C, uint32_t row_bytes)
{
    return GramPruneLayout(C, row_bytes).bytes;
}

// prune_kernel (reference final_prune_kernel_shared,
// src/gpu_vamana_vnew2.cu:1893-2147) for uint8 vectors.  Candidates in
// (distance, slot) order, first occurrence of each id kept; bit q of row j
// is alpha*d(j,q) <= d(v,q) for q after j (d(v,j) <= d(v,q) holds by the
// order), so the greedy selection is: take the lowest live candidate, clear
// its row's bits from the live set.  The live and selected sets sit in
// registers, word w in lane w.  The selection order is ascending, so the
// output is the selected candidates in order followed by the last-round
// fill (the nearest unselected ones).
template <int CPL>
__global__ void __launch_bounds__(kBlockThreads, 4) prune_gram_kernel(PruneParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id();
    const uint32_t lt = (1u << lane) - 1u;
    const uint32_t C = p.C;
    const uint32_t Cp = C <= 32 ? 32u : (uint32_t)next_pow2((int)C);
    const GramPruneLayout lay(C, p.row_bytes);
    const uint32_t Sg = gram_stride(p.row_bytes), kbytes = gram_kbytes(p.row_bytes);
    uint8_t *b = smem_raw + warp_id_in_block() * p.per_warp;
    uint8_t *cache = b;
    uint32_t *rid = reinterpret_cast<uint32_t *>(b);
    uint32_t *sd = reinterpret_cast<uint32_t *>(b + align16(4u * C));
    uint32_t *sid = sd + Cp;
    uint64_t *skeys = reinterpret_cast<uint64_t *>(sid + Cp);
    uint32_t *cid = reinterpret_cast<uint32_t *>(b + lay.cid);
    float *cd = reinterpret_cast<float *>(b + lay.cd);
    uint32_t *norms = reinterpret_cast<uint32_t *>(b + lay.norms);
    uint32_t *occ = reinterpret_cast<uint32_t *>(b + lay.occ);
    const float alpha = p.alpha;
    unsigned long long pairs = 0;

    for (uint32_t v = p.v0 + blockIdx.x * kWarpsPerBlock + warp_id_in_block(); v < p.v1;
         v += gridDim.x * kWarpsPerBlock)
    {
        const uint64_t lv = v - p.lrow0;
        int nvalid;
        if (Cp == 32)
            nvalid = prune_sorted_list<1>(p, v, lv, Cp, rid, sd, sid, skeys, lane);
        else if (Cp == 64)
            nvalid = prune_sorted_list<2>(p, v, lv, Cp, rid, sd, sid, skeys, lane);
        else if (Cp == 128)
            nvalid = prune_sorted_list<4>(p, v, lv, Cp, rid, sd, sid, skeys, lane);
        else
            nvalid = prune_sorted_list<0>(p, v, lv, Cp, rid, sd, sid, skeys, lane);
        // first occurrence of every id: copies of an id share its distance
        // (exact integer arithmetic), so they sit in one run of equal
        // distances and only that run is searched
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
        gather_rows_async<CPL>(p.st.data, p.st.stride, p.st.nchunks, (int)m, cache, Sg, lane,
                               [&](int r) -> uint32_t { return cid[r]; });
        gram_zero_pad(cache, Sg, p.row_bytes, m, lane);
        gather_rows_async_wait();
        gram_norms(cache, Sg, kbytes, m, norms, lane);
        __syncwarp();
        gram_prune_masks<CPL == 1>(cache, Sg, kbytes, norms, cd, m, lay.W, occ, alpha, lane);
        __syncwarp();
        pairs += (unsigned long long)m * (m - (m > 0 ? 1u : 0u)) / 2u;
        // greedy selection
        const uint32_t words = (m + 31u) >> 5;
        uint32_t live = 0;
        if ((uint32_t)lane < words)
        {
            const uint32_t lo = 32u * (uint32_t)lane;
            live = m >= lo + 32u ? 0xFFFFFFFFu : ((1u << (m - lo)) - 1u);
        }
        const uint32_t valid_w = live;
        uint32_t selw = 0, out = 0;
        while (out < p.R)
        {
            const unsigned nz = __ballot_sync(kFull, live != 0u);
            if (!nz)
                break;
            const int l = __ffs(nz) - 1;
            const uint32_t wv = __shfl_sync(kFull, live, l);
            const uint32_t j = 32u * (uint32_t)l + (uint32_t)(__ffs(wv) - 1);
            if (lane == l)
            {
                const uint32_t bit = 1u << (j & 31u);
                live &= ~bit;
                selw |= bit;
            }
            if (++out >= p.R)
                break;
            if ((uint32_t)lane < words)
                live &= ~occ[j * lay.W + (uint32_t)lane];
        }
        // last-round fill: the nearest unselected candidates, ignoring occlusion
        const uint32_t min_deg = min(p.min_degree, p.R);
        uint32_t fillw = 0;
        if (out < min_deg)
        {
            const uint32_t unsel = valid_w & ~selw;
            const uint32_t cnt = __popc(unsel);
            uint32_t incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1)
            {
                const uint32_t t = __shfl_up_sync(kFull, incl, o);
                if (lane >= o)
                    incl += t;
            }
            const uint32_t need = min_deg - out, before = incl - cnt;
            uint32_t take = need > before ? min(need - before, cnt) : 0u;
            uint32_t u = unsel;
            while (take--)
            {
                fillw |= u & (0u - u);
                u &= u - 1u;
            }
        }
        // output: selected in order, then the fill
        uint32_t spre = __popc(selw), fpre = __popc(fillw);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
        {
            const uint32_t ts = __shfl_up_sync(kFull, spre, o);
            const uint32_t tf = __shfl_up_sync(kFull, fpre, o);
            if (lane >= o)
            {
                spre += ts;
                fpre += tf;
            }
        }
        const uint32_t nsel = __shfl_sync(kFull, spre, 31);
        const uint32_t total = nsel + __shfl_sync(kFull, fpre, 31);
        spre -= __popc(selw);
        fpre -= __popc(fillw);
        for (uint32_t w = 0; w < words; ++w)
        {
            const uint32_t sw = __shfl_sync(kFull, selw, (int)w);
            const uint32_t fw = __shfl_sync(kFull, fillw, (int)w);
            const uint32_t sp = __shfl_sync(kFull, spre, (int)w);
            const uint32_t fp = __shfl_sync(kFull, fpre, (int)w);
            const uint32_t bit = 1u << lane;
            uint32_t pos = kInvalid;
            if (sw & bit)
                pos = sp + __popc(sw & lt);
            else if (fw & bit)
                pos = nsel + fp + __popc(fw & lt);
            if (pos != kInvalid)
            {
                const uint32_t j = 32u * w + (uint32_t)lane;
                p.cur_ids[(uint64_t)v * p.R + pos] = cid[j];
                p.cur_dists[lv * p.R + pos] = cd[j];
            }
        }
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
