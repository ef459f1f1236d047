// dance_common.cuh -- device building blocks shared by the Vamana kernels.
//
// Distance groups.  A warp is split into four groups of eight lanes; a group
// evaluates one squared L2 distance.  Vectors are read as 16-byte chunks
// (row stride is a multiple of 16 bytes, padding bytes are zero); lane gl of
// a group owns chunks gl, gl+8, gl+16, ... (CPL chunks per lane, a template
// constant), so one group load instruction moves 128 contiguous bytes and a
// warp instruction serves four candidates at once.
//
// The arithmetic reproduces the reference's warp distance
// (src/gpu_vamana_vnew2.cu:268-290 for uint8, :336-362 for float,
// :391-418 for half): 32 "virtual lane" partial sums over the reference's
// lane-strided elements, then its shfl_down tree 16,8,4,2,1.  Each group lane
// carries the partials of four virtual lanes and the tree levels map onto
// in-lane adds and xor shuffles inside the group, so the result is bitwise
// the value the reference warp computes (uint8 is an exact integer anyway).
#pragma once

#include <cfloat>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace dance
{

constexpr uint32_t kInvalid = 0xFFFFFFFFu;
constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr uint64_t kKeyMax = ~0ull;

enum DType : int
{
    kU8 = 0,
    kF16 = 1,
    kF32 = 2
};

// Hash used for the initial graph and the per-vertex search seeds
// (reference src/gpu_vamana_vnew2.cu:169-191).
__host__ __device__ __forceinline__ uint32_t hash_u32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__host__ __device__ __forceinline__ uint32_t det_neighbor(uint32_t node, uint32_t k, uint32_t N)
{
    if (N <= 1)
        return kInvalid;
    uint32_t v = hash_u32(node * 0x9e3779b1u + k * 0x85ebca6bu + 17u) % N;
    if (v == node)
        v = (v + 1u) % N;
    return v;
}

// Total order used by the search pool: distance first, then id.  Distances
// are non-negative, so their IEEE bit patterns order like the values.
__device__ __forceinline__ uint64_t make_key(float d, uint32_t id)
{
    return ((uint64_t)__float_as_uint(d) << 32) | (uint64_t)id;
}
__device__ __forceinline__ float key_dist(uint64_t k) { return __uint_as_float((uint32_t)(k >> 32)); }
__device__ __forceinline__ uint32_t key_id(uint64_t k) { return (uint32_t)(k & 0xFFFFFFFFull); }

__device__ __forceinline__ uint4 ldg_chunk(const uint4 *p) { return __ldg(p); }

// ------------------------------------------------------------------ group distance
template <int DT, int CPL>
struct GroupDist;

template <int CPL>
struct GroupDist<kF32, CPL>
{
    __device__ __forceinline__ static float eval(const uint4 (&q)[CPL], const uint4 (&c)[CPL], uint32_t nchunks, int gl)
    {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int t = 0; t < CPL; ++t)
        {
            if ((uint32_t)(gl + 8 * t) < nchunks)
            {
                const float4 a = *reinterpret_cast<const float4 *>(&q[t]);
                const float4 b = *reinterpret_cast<const float4 *>(&c[t]);
                const float d0 = __fsub_rn(a.x, b.x);
                const float d1 = __fsub_rn(a.y, b.y);
                const float d2 = __fsub_rn(a.z, b.z);
                const float d3 = __fsub_rn(a.w, b.w);
                float p = __fmul_rn(d1, d1);
                p = __fmaf_rn(d0, d0, p);
                p = __fmaf_rn(d2, d2, p);
                p = __fmaf_rn(d3, d3, p);
                acc[t & 3] = __fadd_rn(acc[t & 3], p);
            }
        }
        // virtual lanes gl+8u (u = 0..3): levels 16 and 8 are in-lane.
        float r = __fadd_rn(__fadd_rn(acc[0], acc[2]), __fadd_rn(acc[1], acc[3]));
        r = __fadd_rn(r, __shfl_xor_sync(kFull, r, 4));
        r = __fadd_rn(r, __shfl_xor_sync(kFull, r, 2));
        r = __fadd_rn(r, __shfl_xor_sync(kFull, r, 1));
        return r;
    }
};

template <int CPL>
struct GroupDist<kF16, CPL>
{
    __device__ __forceinline__ static float eval(const uint4 (&q)[CPL], const uint4 (&c)[CPL], uint32_t nchunks, int gl)
    {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int t = 0; t < CPL; ++t)
        {
            if ((uint32_t)(gl + 8 * t) < nchunks)
            {
                const __half2 *a = reinterpret_cast<const __half2 *>(&q[t]);
                const __half2 *b = reinterpret_cast<const __half2 *>(&c[t]);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                {
                    const __half2 df = __hsub2(a[i], b[i]);
                    const __half2 pr = __hmul2(df, df);
                    const float2 f = __half22float2(pr);
                    acc[i] = __fadd_rn(acc[i], __fadd_rn(f.x, f.y));
                }
            }
        }
        // virtual lanes 4*gl+i: levels 16,8,4 are xor 4,2,1; levels 2,1 in-lane.
#pragma unroll
        for (int i = 0; i < 4; ++i)
            acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(kFull, acc[i], 4));
#pragma unroll
        for (int i = 0; i < 4; ++i)
            acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(kFull, acc[i], 2));
#pragma unroll
        for (int i = 0; i < 4; ++i)
            acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(kFull, acc[i], 1));
        return __fadd_rn(__fadd_rn(acc[0], acc[2]), __fadd_rn(acc[1], acc[3]));
    }
};

template <int CPL>
struct GroupDist<kU8, CPL>
{
    __device__ __forceinline__ static float eval(const uint4 (&q)[CPL], const uint4 (&c)[CPL], uint32_t nchunks, int gl)
    {
        uint32_t acc = 0;
#pragma unroll
        for (int t = 0; t < CPL; ++t)
        {
            if ((uint32_t)(gl + 8 * t) < nchunks)
            {
                uint32_t ad = __vabsdiffu4(q[t].x, c[t].x);
                acc = __dp4a(ad, ad, acc);
                ad = __vabsdiffu4(q[t].y, c[t].y);
                acc = __dp4a(ad, ad, acc);
                ad = __vabsdiffu4(q[t].z, c[t].z);
                acc = __dp4a(ad, ad, acc);
                ad = __vabsdiffu4(q[t].w, c[t].w);
                acc = __dp4a(ad, ad, acc);
            }
        }
        acc += __shfl_xor_sync(kFull, acc, 4);
        acc += __shfl_xor_sync(kFull, acc, 2);
        acc += __shfl_xor_sync(kFull, acc, 1);
        return (float)(int32_t)acc;
    }
};

// Four-lane pair distance: the reference's warp arithmetic (virtual lanes
// over 16-byte chunks and the shfl_down tree 16,8,4,2,1) evaluated by four
// lanes instead of GroupDist's eight, so a warp pass covers eight pairs.
// Lane sl holds chunks sl, sl+4, sl+8, ... (x[t] is chunk sl + 4t of the
// first row).  For half, chunk c feeds virtual lanes 4 (c mod 8) + i, so a
// lane's even chunks feed 4 sl + i and its odd ones 4 sl + 16 + i: tree
// level 16 is in-lane, 8 and 4 are xor 2 and xor 1, 2 and 1 in-lane again.
// For float, chunk c feeds virtual lane c mod 32 = sl + 4 (t mod 8): levels
// 16, 8 and 4 are in-lane, 2 and 1 are xor 2 and xor 1.  Each virtual lane
// adds its chunks in ascending order, as the reference lane does, so the
// results are GroupDist's bit for bit.
template <int DT, int T>
struct QuadDist;

template <int T>
struct QuadDist<kF16, T>
{
    __device__ __forceinline__ static float eval(const uint4 (&x)[T], const uint8_t *row, uint32_t nchunks, int sl)
    {
        const uint4 *r = reinterpret_cast<const uint4 *>(row);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int t = 0; t < T; ++t)
        {
            const uint32_t c = (uint32_t)(sl + 4 * t);
            if (c < nchunks)
            {
                const uint4 y = r[c];
                const __half2 *a = reinterpret_cast<const __half2 *>(&x[t]);
                const __half2 *b = reinterpret_cast<const __half2 *>(&y);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                {
                    const __half2 df = __hsub2(a[i], b[i]);
                    const __half2 pr = __hmul2(df, df);
                    const float2 f = __half22float2(pr);
                    acc[(t & 1) * 4 + i] = __fadd_rn(acc[(t & 1) * 4 + i], __fadd_rn(f.x, f.y));
                }
            }
        }
        float s[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            s[i] = __fadd_rn(acc[i], acc[4 + i]); // level 16
#pragma unroll
        for (int i = 0; i < 4; ++i)
            s[i] = __fadd_rn(s[i], __shfl_xor_sync(kFull, s[i], 2)); // level 8
#pragma unroll
        for (int i = 0; i < 4; ++i)
            s[i] = __fadd_rn(s[i], __shfl_xor_sync(kFull, s[i], 1)); // level 4
        return __fadd_rn(__fadd_rn(s[0], s[2]), __fadd_rn(s[1], s[3])); // levels 2, 1
    }
};

template <int T>
struct QuadDist<kF32, T>
{
    __device__ __forceinline__ static float eval(const uint4 (&x)[T], const uint8_t *row, uint32_t nchunks, int sl)
    {
        const uint4 *r = reinterpret_cast<const uint4 *>(row);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int t = 0; t < T; ++t)
        {
            const uint32_t c = (uint32_t)(sl + 4 * t);
            if (c < nchunks)
            {
                const uint4 yv = r[c];
                const float4 a = *reinterpret_cast<const float4 *>(&x[t]);
                const float4 b = *reinterpret_cast<const float4 *>(&yv);
                const float d0 = __fsub_rn(a.x, b.x);
                const float d1 = __fsub_rn(a.y, b.y);
                const float d2 = __fsub_rn(a.z, b.z);
                const float d3 = __fsub_rn(a.w, b.w);
                float p = __fmul_rn(d1, d1);
                p = __fmaf_rn(d0, d0, p);
                p = __fmaf_rn(d2, d2, p);
                p = __fmaf_rn(d3, d3, p);
                acc[t & 7] = __fadd_rn(acc[t & 7], p);
            }
        }
        // virtual lane sl + 4u is acc[u]
        const float b0 = __fadd_rn(acc[0], acc[4]), b1 = __fadd_rn(acc[1], acc[5]); // level 16
        const float b2 = __fadd_rn(acc[2], acc[6]), b3 = __fadd_rn(acc[3], acc[7]);
        const float c0 = __fadd_rn(b0, b2), c1 = __fadd_rn(b1, b3); // level 8
        float r1 = __fadd_rn(c0, c1);                               // level 4
        r1 = __fadd_rn(r1, __shfl_xor_sync(kFull, r1, 2));          // level 2
        r1 = __fadd_rn(r1, __shfl_xor_sync(kFull, r1, 1));          // level 1
        return r1;
    }
};

// Position of the n-th (0-based) set bit of w; n < popc(w).
__device__ __forceinline__ int nth_set_bit(uint32_t w, int n)
{
    int pos = 0;
#pragma unroll
    for (int half = 16; half > 0; half >>= 1)
    {
        const int c = __popc(w & ((1u << half) - 1u));
        const bool up = n >= c;
        n -= up ? c : 0;
        w = up ? (w >> half) : w;
        pos += up ? half : 0;
    }
    return pos;
}

// Load the fragment of `row` owned by group lane gl (zero beyond nchunks).
template <int CPL>
__device__ __forceinline__ void load_frag(uint4 (&f)[CPL], const uint8_t *row, uint32_t nchunks, int gl)
{
    const uint4 *r = reinterpret_cast<const uint4 *>(row);
#pragma unroll
    for (int t = 0; t < CPL; ++t)
    {
        const uint32_t c = (uint32_t)(gl + 8 * t);
        f[t] = c < nchunks ? ldg_chunk(r + c) : make_uint4(0u, 0u, 0u, 0u);
    }
}

// Same from shared memory (no read-only path).
template <int CPL>
__device__ __forceinline__ void load_frag_smem(uint4 (&f)[CPL], const uint8_t *row, uint32_t nchunks, int gl)
{
    const uint4 *r = reinterpret_cast<const uint4 *>(row);
#pragma unroll
    for (int t = 0; t < CPL; ++t)
    {
        const uint32_t c = (uint32_t)(gl + 8 * t);
        f[t] = c < nchunks ? r[c] : make_uint4(0u, 0u, 0u, 0u);
    }
}

// Candidates evaluated per group per pipelined pass: keeps about 48-64
// registers of loads in flight per lane.
template <int CPL>
struct Unroll
{
    static constexpr int value = (CPL <= 1) ? 8 : (CPL == 2 ? 6 : (CPL <= 4 ? 4 : 2));
};

// Distances from the query fragment q to the m candidates bid[0..m) (rows
// of the global store), written to bd[0..m).  All 32 lanes must call.
template <int DT, int CPL>
__device__ __forceinline__ void eval_candidates(const uint8_t *__restrict__ data, uint64_t stride, uint32_t nchunks,
                                                const uint4 (&q)[CPL], const uint32_t *bid, float *bd, int m,
                                                int lane)
{
    constexpr int U = Unroll<CPL>::value;
    const int g = lane >> 3;
    const int gl = lane & 7;
    if constexpr (DT == kU8 && U == 8)
    {
        // uint8, 8 candidates per group and pass: each lane accumulates
        // |q|^2 + |c|^2 - 2<q,c> over its part of every candidate (exact
        // integers, so equal to the sum of squared differences), and one
        // transposing butterfly leaves candidate gl's total in lane gl.
        uint32_t qq = 0;
#pragma unroll
        for (int t = 0; t < CPL; ++t)
        {
            qq = __dp4a(q[t].x, q[t].x, qq);
            qq = __dp4a(q[t].y, q[t].y, qq);
            qq = __dp4a(q[t].z, q[t].z, qq);
            qq = __dp4a(q[t].w, q[t].w, qq);
        }
        const bool h4 = gl & 4, h2 = gl & 2, h1 = gl & 1;
        for (int base = 0; base < m; base += 32)
        {
            uint4 buf[8][CPL];
#pragma unroll
            for (int u = 0; u < 8; ++u)
            {
                const int idx = base + 4 * u + g;
                if (idx < m)
                    load_frag<CPL>(buf[u], data + (uint64_t)bid[idx] * stride, nchunks, gl);
                else
                {
#pragma unroll
                    for (int t = 0; t < CPL; ++t)
                        buf[u][t] = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            uint32_t part[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
            {
                part[u] = 0u;
                if (base + 4 * u >= m) // no candidate of this pass row (warp-uniform)
                    continue;
                uint32_t cc = qq, qc = 0;
#pragma unroll
                for (int t = 0; t < CPL; ++t)
                {
                    cc = __dp4a(buf[u][t].x, buf[u][t].x, cc);
                    cc = __dp4a(buf[u][t].y, buf[u][t].y, cc);
                    cc = __dp4a(buf[u][t].z, buf[u][t].z, cc);
                    cc = __dp4a(buf[u][t].w, buf[u][t].w, cc);
                    qc = __dp4a(q[t].x, buf[u][t].x, qc);
                    qc = __dp4a(q[t].y, buf[u][t].y, qc);
                    qc = __dp4a(q[t].z, buf[u][t].z, qc);
                    qc = __dp4a(q[t].w, buf[u][t].w, qc);
                }
                part[u] = cc - 2u * qc;
            }
            uint32_t w4[4], w2[2];
#pragma unroll
            for (int k = 0; k < 4; ++k)
            {
                const uint32_t send = h4 ? part[k] : part[k + 4];
                const uint32_t keep = h4 ? part[k + 4] : part[k];
                w4[k] = keep + __shfl_xor_sync(kFull, send, 4);
            }
#pragma unroll
            for (int k = 0; k < 2; ++k)
            {
                const uint32_t send = h2 ? w4[k] : w4[k + 2];
                const uint32_t keep = h2 ? w4[k + 2] : w4[k];
                w2[k] = keep + __shfl_xor_sync(kFull, send, 2);
            }
            const uint32_t send = h1 ? w2[0] : w2[1];
            const uint32_t keep = h1 ? w2[1] : w2[0];
            const uint32_t tot = keep + __shfl_xor_sync(kFull, send, 1);
            const int idx = base + 4 * gl + g; // this lane's total is candidate u = gl
            if (idx < m)
                bd[idx] = (float)(int32_t)tot;
        }
    }
    else
    {
        for (int base = 0; base < m; base += 4 * U)
        {
            uint4 buf[U][CPL];
#pragma unroll
            for (int u = 0; u < U; ++u)
            {
                const int idx = base + 4 * u + g;
                if (idx < m)
                    load_frag<CPL>(buf[u], data + (uint64_t)bid[idx] * stride, nchunks, gl);
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
                const int idx = base + 4 * u + g;
                const float d = GroupDist<DT, CPL>::eval(q, buf[u], nchunks, gl);
                if (idx < m && gl == 0)
                    bd[idx] = d;
            }
        }
    }
}

// Same, candidates read from a shared-memory vector cache (row_bytes apart),
// cidx[0..m) naming the cache slots.
template <int DT, int CPL>
__device__ __forceinline__ void eval_cached(const uint8_t *cache, uint32_t row_bytes, uint32_t nchunks,
                                            const uint4 (&q)[CPL], const uint16_t *cidx, float *bd, int m, int lane)
{
    const int g = lane >> 3;
    const int gl = lane & 7;
    for (int base = 0; base < m; base += 4)
    {
        const int idx = base + g;
        uint4 c[CPL];
        if (idx < m)
            load_frag_smem<CPL>(c, cache + (uint32_t)cidx[idx] * row_bytes, nchunks, gl);
        else
        {
#pragma unroll
            for (int t = 0; t < CPL; ++t)
                c[t] = make_uint4(0u, 0u, 0u, 0u);
        }
        const float d = GroupDist<DT, CPL>::eval(q, c, nchunks, gl);
        if (idx < m && gl == 0)
            bd[idx] = d;
    }
}

// ------------------------------------------------------------------ warp sorts
// Ascending bitonic sort of 32*NPL keys held NPL per lane in blocked order
// (element lane*NPL + s in k[s]): in-lane exchanges for distances below NPL,
// xor shuffles above.
template <int NPL, class K>
__device__ __forceinline__ void warp_sort_blocked(K (&k)[NPL], int lane)
{
    constexpr int n = 32 * NPL;
#pragma unroll
    for (int size = 2; size <= n; size <<= 1)
    {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1)
        {
            if (j < NPL)
            {
#pragma unroll
                for (int s = 0; s < NPL; ++s)
                {
                    const int t = s ^ j;
                    if (t > s)
                    {
                        const bool asc = ((lane * NPL + s) & size) == 0;
                        const K a = k[s], b = k[t];
                        const bool sw = asc ? (a > b) : (a < b);
                        k[s] = sw ? b : a;
                        k[t] = sw ? a : b;
                    }
                }
            }
            else
            {
                const int lm = j / NPL;
                const bool lower = (lane & lm) == 0;
#pragma unroll
                for (int s = 0; s < NPL; ++s)
                {
                    const bool asc = ((lane * NPL + s) & size) == 0;
                    const K o = __shfl_xor_sync(kFull, k[s], lm);
                    const bool take_min = lower == asc;
                    k[s] = take_min ? (k[s] < o ? k[s] : o) : (k[s] > o ? k[s] : o);
                }
            }
        }
    }
}

// Ascending bitonic sort of 64 keys held two per lane (element 2*lane+s).
__device__ __forceinline__ void warp_sort64(uint64_t &k0, uint64_t &k1, int lane)
{
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1)
    {
        const bool asc = ((2 * lane) & size) == 0;
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1)
        {
            if (j == 1)
            {
                const bool sw = asc ? (k0 > k1) : (k0 < k1);
                if (sw)
                {
                    const uint64_t t = k0;
                    k0 = k1;
                    k1 = t;
                }
            }
            else
            {
                const int pl = j >> 1;
                const uint64_t p0 = __shfl_xor_sync(kFull, k0, pl);
                const uint64_t p1 = __shfl_xor_sync(kFull, k1, pl);
                const bool take_min = (((lane & pl) == 0) == asc);
                k0 = take_min ? (k0 < p0 ? k0 : p0) : (k0 > p0 ? k0 : p0);
                k1 = take_min ? (k1 < p1 ? k1 : p1) : (k1 > p1 ? k1 : p1);
            }
        }
    }
}

// Ascending bitonic sort of n32 (power of two, 32..4096) uint32 values in
// shared memory by one warp.
__device__ __forceinline__ void warp_sort_smem_u32(uint32_t *a, int n, int lane)
{
    for (int size = 2; size <= n; size <<= 1)
    {
        for (int j = size >> 1; j > 0; j >>= 1)
        {
            for (int i = lane; i < n; i += 32)
            {
                const int l = i ^ j;
                if (l > i)
                {
                    const uint32_t x = a[i], y = a[l];
                    const bool asc = (i & size) == 0;
                    if (asc ? (x > y) : (x < y))
                    {
                        a[i] = y;
                        a[l] = x;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// Same for uint64 keys.
__device__ __forceinline__ void warp_sort_smem_u64(uint64_t *a, int n, int lane)
{
    for (int size = 2; size <= n; size <<= 1)
    {
        for (int j = size >> 1; j > 0; j >>= 1)
        {
            for (int i = lane; i < n; i += 32)
            {
                const int l = i ^ j;
                if (l > i)
                {
                    const uint64_t x = a[i], y = a[l];
                    const bool asc = (i & size) == 0;
                    if (asc ? (x > y) : (x < y))
                    {
                        a[i] = y;
                        a[l] = x;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// Ascending sort of a[0..n) (n a power of two, 32..4096; a 16-byte
// aligned) by one warp: in registers for n <= 128, else in shared memory.
__device__ __forceinline__ void warp_sort_u32(uint32_t *a, int n, int lane)
{
    if (n > 128)
    {
        warp_sort_smem_u32(a, n, lane);
        return;
    }
    __syncwarp();
    if (n == 32)
    {
        uint32_t k[1] = {a[lane]};
        warp_sort_blocked<1>(k, lane);
        a[lane] = k[0];
    }
    else if (n == 64)
    {
        const uint2 x = reinterpret_cast<const uint2 *>(a)[lane];
        uint32_t k[2] = {x.x, x.y};
        warp_sort_blocked<2>(k, lane);
        reinterpret_cast<uint2 *>(a)[lane] = make_uint2(k[0], k[1]);
    }
    else
    {
        const uint4 x = reinterpret_cast<const uint4 *>(a)[lane];
        uint32_t k[4] = {x.x, x.y, x.z, x.w};
        warp_sort_blocked<4>(k, lane);
        reinterpret_cast<uint4 *>(a)[lane] = make_uint4(k[0], k[1], k[2], k[3]);
    }
    __syncwarp();
}

// Number of elements of sorted a[0..n) strictly less than key (n <= 256).
__device__ __forceinline__ int lower_bound_u64(const uint64_t *a, int n, uint64_t key)
{
    // fixed steps of a power-of-two search (n <= 256): no data-dependent branches
    int pos = 0;
#pragma unroll
    for (int step = 256; step > 0; step >>= 1)
        if (pos + step <= n && a[pos + step - 1] < key)
            pos += step;
    return pos;
}

__host__ __device__ __forceinline__ int next_pow2(int n)
{
    int p = 1;
    while (p < n)
        p <<= 1;
    return p;
}

} // namespace dance
