// vamana_oracle.cpp -- CPU restatement of the DANCE vnew2 Vamana build.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity oracle: it is compiled
// into oracle/liboracle.so and loaded exclusively by tests/, by
// __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference
// leg.  The product (dance_b200/libdance_b200.so) never links or calls it.
//
// It restates, sequentially and per vertex, the algorithm of the reference
// file src/gpu_vamana_vnew2.cu (paths are relative to the DANCE repository):
//   hash / deterministic_neighbor ........ :169-191
//   distance arithmetic .................. :268-290 (u8), :336-362 (f32),
//                                          :391-418 (f16)
//   approximate medoid ................... :1032-1064, host argmin :2445-2479
//   random initial graph ................. :1066-1117
//   GreedySearch + online RobustInsert ... :1119-1439, :598-734, :759-877
//   CSR reverse count / fill / merge ..... :1604-1661, :1722-1814
//   RobustPrune + final degree fill ...... :1893-2147
//   round driver ......................... :2170-2855 (alpha schedule :201-213)
//
// Canonical choices where the reference is order-dependent:
//   * search pool ties: pool_mode 0 (the product's rule) orders candidates by
//     the key (distance, id); pool_mode 1 restates the reference's unsorted
//     slot pool literally (ties -> lowest slot) and is used only to pin this
//     oracle against outputs of the reference itself;
//   * reverse CSR order: sources of each target in ascending source id (the
//     reference fills with atomics, so its order varies run to run).
// Everything else -- the online insert, reverse merge and prune decisions and
// their slot tie-breaks -- follows the reference rules exactly.
//
// Distances reproduce the reference warp arithmetic: 32 lane partial sums
// over 16-byte chunks (f32: float4 index mod 32, per chunk
// fma(dw,dw,fma(dz,dz,fma(dx,dx,dy*dy))); f16: half2 index mod 32, half
// precision diff and square, float sum of the pair), then the shfl_down tree
// 16,8,4,2,1.  u8 is the exact integer sum.  Build with -ffp-contract=off.

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/dance_b200.h"

namespace
{
constexpr uint32_t kInvalid = 0xFFFFFFFFu;

// ---------------------------------------------------------------- hashing
uint32_t hash_u32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

uint32_t det_neighbor(uint32_t node, uint32_t k, uint32_t N)
{
    if (N <= 1)
        return kInvalid;
    uint32_t v = hash_u32(node * 0x9e3779b1u + k * 0x85ebca6bu + 17u) % N;
    if (v == node)
        v = (v + 1u) % N;
    return v;
}

// ------------------------------------------------------------ binary16
// IEEE-754 binary16 with round-to-nearest-even, written from the format
// definition (1 sign, 5 exponent bits biased by 15, 10 fraction bits).
uint16_t double_to_half(double x)
{
    uint16_t sign = std::signbit(x) ? 0x8000u : 0u;
    double a = std::fabs(x);
    if (std::isnan(a))
        return 0x7E00u;
    if (a >= 65520.0)
        return sign | 0x7C00u;
    if (a < 6.103515625e-05) // 2^-14: subnormal range, unit 2^-24
    {
        double q = std::nearbyint(a * 16777216.0);
        return sign | (uint16_t)q;
    }
    int k = 0;
    double f = std::frexp(a, &k); // a = f * 2^k, f in [0.5, 1)
    int e = k - 1;
    double m = std::nearbyint((f * 2.0 - 1.0) * 1024.0);
    if (m >= 1024.0)
    {
        m = 0.0;
        e += 1;
    }
    if (e > 15)
        return sign | 0x7C00u;
    return sign | (uint16_t)((e + 15) << 10) | (uint16_t)m;
}

float half_to_float(uint16_t h)
{
    uint32_t sign = (h & 0x8000u) ? 1u : 0u;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    double v;
    if (e == 0)
        v = std::ldexp((double)m, -24);
    else if (e == 31)
        v = m ? NAN : INFINITY;
    else
        v = std::ldexp((double)(m | 0x400u), (int)e - 25);
    return (float)(sign ? -v : v);
}

// ------------------------------------------------------------ distances
struct Store
{
    int dtype;
    const uint8_t *base;
    uint64_t stride;
    uint32_t dim;
    const uint8_t *row(uint32_t i) const { return base + (uint64_t)i * stride; }
};

float tree32(float *acc)
{
    for (int off = 16; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l)
            acc[l] = acc[l] + acc[l + off];
    return acc[0];
}

float dist_f32(const float *x, const float *y, uint32_t dim)
{
    float acc[32] = {0};
    const uint32_t chunks = (dim + 3) / 4;
    for (uint32_t c = 0; c < chunks; ++c)
    {
        float d[4];
        for (int i = 0; i < 4; ++i)
        {
            uint32_t e = c * 4 + i;
            d[i] = e < dim ? x[e] - y[e] : 0.0f;
        }
        float p = d[1] * d[1];
        p = std::fma(d[0], d[0], p);
        p = std::fma(d[2], d[2], p);
        p = std::fma(d[3], d[3], p);
        acc[c & 31] = acc[c & 31] + p;
    }
    return tree32(acc);
}

// The same rounding from the bits of the double (round to nearest even on
// the 42 or more dropped significand bits); checked against double_to_half
// by oracle_half_selftest.
uint16_t double_to_half_bits(double x)
{
    uint64_t b;
    std::memcpy(&b, &x, sizeof(b));
    const uint16_t sign = (uint16_t)((b >> 48) & 0x8000u);
    const uint64_t a = b & 0x7FFFFFFFFFFFFFFFull;
    if (a > 0x7FF0000000000000ull)
        return 0x7E00u;
    const int exp = (int)(a >> 52);
    if (exp == 0)
        return sign; // zero or a double subnormal: far below half's unit 2^-24
    const int e = exp - 1023;
    if (e >= 16)
        return sign | 0x7C00u;
    const uint64_t m = (a & 0xFFFFFFFFFFFFFull) | (1ull << 52); // 53-bit significand
    if (e >= -14)
    {
        uint64_t q = m >> 42;
        const uint64_t rem = m & ((1ull << 42) - 1), halfway = 1ull << 41;
        if (rem > halfway || (rem == halfway && (q & 1u)))
            ++q;
        int eh = e;
        if (q == (1ull << 11))
        {
            q >>= 1;
            ++eh;
        }
        if (eh > 15)
            return sign | 0x7C00u;
        return sign | (uint16_t)((eh + 15) << 10) | (uint16_t)(q & 0x3FFu);
    }
    const int shift = 28 - e; // value in units of 2^-24 is m >> shift
    if (shift > 53)
        return sign; // below half the smallest subnormal
    uint64_t q = m >> shift;
    const uint64_t rem = m & ((1ull << shift) - 1), halfway = 1ull << (shift - 1);
    if (rem > halfway || (rem == halfway && (q & 1u)))
        ++q;
    return sign | (uint16_t)q; // q == 1024 is the smallest normal, bit for bit
}

// Tables over all 65536 halves: value, and the half-rounded square.
struct HalfTables
{
    float h2f[65536];
    float sq[65536];
    HalfTables()
    {
        for (uint32_t h = 0; h < 65536u; ++h)
            h2f[h] = half_to_float((uint16_t)h);
        for (uint32_t h = 0; h < 65536u; ++h)
        {
            const double d = (double)h2f[h];
            sq[h] = half_to_float(double_to_half(d * d));
        }
    }
};

const HalfTables &half_tables()
{
    static const HalfTables t;
    return t;
}

// (a - b) rounded to half, squared, rounded to half (the reference's
// __hsub2 / __hmul2 pair), returned as float.
float half_sq_diff(uint16_t a, uint16_t b)
{
    const HalfTables &t = half_tables();
    return t.sq[double_to_half_bits((double)t.h2f[a] - (double)t.h2f[b])];
}

float dist_f16(const uint16_t *x, const uint16_t *y, uint32_t dim)
{
    const HalfTables &t = half_tables();
    float acc[32] = {0};
    const uint32_t pairs = dim / 2;
    for (uint32_t h = 0; h < pairs; ++h)
    {
        float lo = half_sq_diff(x[2 * h], y[2 * h]);
        float hi = half_sq_diff(x[2 * h + 1], y[2 * h + 1]);
        acc[h & 31] = acc[h & 31] + (lo + hi);
    }
    if (dim & 1u)
    {
        float d = t.h2f[x[dim - 1]] - t.h2f[y[dim - 1]];
        acc[0] = std::fma(d, d, acc[0]);
    }
    return tree32(acc);
}

float dist_u8(const uint8_t *x, const uint8_t *y, uint32_t dim)
{
    uint64_t s = 0;
    for (uint32_t e = 0; e < dim; ++e)
    {
        int d = (int)x[e] - (int)y[e];
        s += (uint64_t)(d * d);
    }
    return (float)(int32_t)(uint32_t)s;
}

float dist(const Store &st, uint32_t a, uint32_t b)
{
    switch (st.dtype)
    {
    case DANCE_U8:
        return dist_u8(st.row(a), st.row(b), st.dim);
    case DANCE_F16:
        return dist_f16(reinterpret_cast<const uint16_t *>(st.row(a)), reinterpret_cast<const uint16_t *>(st.row(b)),
                        st.dim);
    default:
        return dist_f32(reinterpret_cast<const float *>(st.row(a)), reinterpret_cast<const float *>(st.row(b)),
                        st.dim);
    }
}

float dist_query(const Store &st, const uint8_t *q, uint32_t b)
{
    switch (st.dtype)
    {
    case DANCE_U8:
        return dist_u8(q, st.row(b), st.dim);
    case DANCE_F16:
        return dist_f16(reinterpret_cast<const uint16_t *>(q), reinterpret_cast<const uint16_t *>(st.row(b)), st.dim);
    default:
        return dist_f32(reinterpret_cast<const float *>(q), reinterpret_cast<const float *>(st.row(b)), st.dim);
    }
}

inline uint64_t make_key(float d, uint32_t id)
{
    uint32_t bits;
    std::memcpy(&bits, &d, 4);
    return ((uint64_t)bits << 32) | id;
}

// ------------------------------------------------------------ counters
std::atomic<uint64_t> g_search_evals{0};
std::atomic<uint64_t> g_search_expansions{0};
std::atomic<uint64_t> g_pair_evals{0};
std::atomic<uint64_t> g_reverse_evals{0};
std::atomic<uint64_t> g_reverse_edges{0};
std::atomic<uint64_t> g_seed_mismatch{0};

// ------------------------------------------------------------ visited set
// Per-thread epoch-tagged array over all ids: exact membership.
struct Visited
{
    std::vector<uint32_t> tag;
    uint32_t epoch = 0;
    void reset(uint32_t N)
    {
        if (tag.size() < N)
            tag.assign(N, 0);
        if (++epoch == 0)
        {
            std::fill(tag.begin(), tag.end(), 0);
            epoch = 1;
        }
    }
    bool test_and_set(uint32_t id)
    {
        if (tag[id] == epoch)
            return true;
        tag[id] = epoch;
        return false;
    }
};

// ------------------------------------------------------------ search pools
// pool_mode 0: candidates ordered by key (distance, id); the pool holds the
// L smallest keys seen; expansion takes the smallest unexpanded key.
struct KeyPool
{
    uint32_t L;
    std::vector<uint64_t> keys;
    std::vector<uint8_t> expanded;
    explicit KeyPool(uint32_t L_) : L(L_) {}
    void insert(uint32_t id, float d)
    {
        uint64_t k = make_key(d, id);
        if (!keys.empty() && keys.size() >= L && k >= keys.back())
            return;
        auto it = std::lower_bound(keys.begin(), keys.end(), k);
        size_t pos = (size_t)(it - keys.begin());
        if (it != keys.end() && *it == k)
            return;
        keys.insert(it, k);
        expanded.insert(expanded.begin() + (ptrdiff_t)pos, 0);
        if (keys.size() > L)
        {
            keys.pop_back();
            expanded.pop_back();
        }
    }
    bool next(uint32_t &id, float &d)
    {
        for (size_t i = 0; i < keys.size(); ++i)
            if (!expanded[i])
            {
                expanded[i] = 1;
                id = (uint32_t)(keys[i] & 0xFFFFFFFFu);
                uint32_t bits = (uint32_t)(keys[i] >> 32);
                std::memcpy(&d, &bits, 4);
                return true;
            }
        return false;
    }
};

// pool_mode 1: literal restatement of the reference slot pool
// (insert_top_l_state_warp :598-692, select_next_unexpanded_size_warp :694-734).
struct SlotPool
{
    uint32_t L;
    std::vector<uint32_t> ids;
    std::vector<float> d;
    std::vector<uint8_t> exp;
    uint32_t size = 0;
    int max_pos = -1;
    float max_d = -FLT_MAX;
    explicit SlotPool(uint32_t L_) : L(L_), ids(L_, kInvalid), d(L_, FLT_MAX), exp(L_, 0) {}
    void recompute_max()
    {
        max_pos = -1;
        max_d = -FLT_MAX;
        for (uint32_t p = 0; p < size; ++p)
            if (ids[p] != kInvalid && d[p] > max_d)
            {
                max_d = d[p];
                max_pos = (int)p;
            }
    }
    void insert(uint32_t id, float dist)
    {
        if (id == kInvalid)
            return;
        if (size >= L && max_pos >= 0 && dist >= max_d)
            return;
        for (uint32_t p = 0; p < size; ++p)
            if (ids[p] == id)
            {
                if (dist < d[p])
                {
                    d[p] = dist;
                    exp[p] = 0;
                    if ((int)p == max_pos)
                        recompute_max();
                }
                return;
            }
        if (size < L)
        {
            ids[size] = id;
            d[size] = dist;
            exp[size] = 0;
            if (max_pos < 0 || dist > max_d)
            {
                max_pos = (int)size;
                max_d = dist;
            }
            ++size;
            return;
        }
        if (max_pos >= 0 && dist < max_d)
        {
            ids[max_pos] = id;
            d[max_pos] = dist;
            exp[max_pos] = 0;
            recompute_max();
        }
    }
    bool next(uint32_t &id, float &dist)
    {
        int best = -1;
        float bd = FLT_MAX;
        for (uint32_t p = 0; p < size; ++p)
            if (ids[p] != kInvalid && !exp[p] && d[p] < bd)
            {
                bd = d[p];
                best = (int)p;
            }
        if (best < 0)
            return false;
        exp[best] = 1;
        id = ids[best];
        dist = d[best];
        return true;
    }
};

struct Graph
{
    uint32_t N, R, C;
    std::vector<uint32_t> cur_ids;   // N x R
    std::vector<float> cur_dists;    // N x R
    std::vector<uint32_t> degree;    // N
    std::vector<uint32_t> work_ids;  // N x C
    std::vector<float> work_dists;   // N x C
    std::vector<uint32_t> work_deg;  // N
};

// GreedySearch of vertex v on the frozen graph; returns the expansion
// sequence (reference :1166-1423 without the inline insert).
template <class Pool>
void search_vertex(const Store &st, uint32_t N, uint32_t R, uint32_t L, uint32_t max_steps, uint32_t entry,
                   uint32_t seeds, const uint32_t *cur_ids, const float *cur_dists, const uint32_t *degree,
                   uint32_t v, Visited &vis, std::vector<uint32_t> &exp_ids, std::vector<float> &exp_d)
{
    Pool pool(L);
    vis.reset(N);
    exp_ids.clear();
    exp_d.clear();
    uint64_t evals = 0;
    vis.test_and_set(v);
    if (entry < N && entry != v)
    {
        if (!vis.test_and_set(entry))
        {
            pool.insert(entry, dist(st, v, entry));
            ++evals;
        }
    }
    uint32_t deg_self = std::min(degree[v], R);
    for (uint32_t i = 0; i < deg_self; ++i)
    {
        uint32_t nb = cur_ids[(size_t)v * R + i];
        if (nb == kInvalid || nb >= N || nb == v)
            continue;
        float d = cur_dists[(size_t)v * R + i];
        if (vis.test_and_set(nb))
        {
            // Already evaluated (the entry point): the stored distance must
            // equal the computed one for the skip to be exact.
            if (nb == entry && d != dist(st, v, nb))
                g_seed_mismatch.fetch_add(1, std::memory_order_relaxed);
            continue;
        }
        pool.insert(nb, d);
    }
    for (uint32_t k = 0; k < seeds; ++k)
    {
        uint32_t s = det_neighbor(v, k + 1024u, N);
        if (s == kInvalid || s >= N || s == v)
            continue;
        if (vis.test_and_set(s))
            continue;
        pool.insert(s, dist(st, v, s));
        ++evals;
    }
    for (uint32_t step = 0; step < max_steps; ++step)
    {
        uint32_t x;
        float dx;
        if (!pool.next(x, dx))
            break;
        if (x == kInvalid || x >= N)
            break;
        exp_ids.push_back(x);
        exp_d.push_back(dx);
        uint32_t deg = std::min(degree[x], R);
        for (uint32_t p = 0; p < deg; ++p)
        {
            uint32_t c = cur_ids[(size_t)x * R + p];
            if (c == kInvalid || c >= N || c == v)
                continue;
            if (vis.test_and_set(c))
                continue;
            pool.insert(c, dist(st, v, c));
            ++evals;
        }
    }
    g_search_evals.fetch_add(evals, std::memory_order_relaxed);
    g_search_expansions.fetch_add(exp_ids.size(), std::memory_order_relaxed);
}

// Work row initialisation (reference :1175-1204).
void init_work_row(uint32_t N, uint32_t R, uint32_t C, const uint32_t *cur_ids, const float *cur_dists,
                   const uint32_t *degree, uint32_t v, uint32_t *wid, float *wd, uint32_t &wdeg)
{
    uint32_t deg_self = std::min(degree[v], R);
    for (uint32_t i = 0; i < C; ++i)
    {
        uint32_t nb = kInvalid;
        float d = FLT_MAX;
        if (i < deg_self)
        {
            nb = cur_ids[(size_t)v * R + i];
            if (nb != kInvalid && nb < N && nb != v)
                d = cur_dists[(size_t)v * R + i];
            else
                nb = kInvalid;
        }
        wid[i] = nb;
        wd[i] = d;
    }
    wdeg = deg_self;
}

// Online RobustInsert of x into v's C-wide work row
// (dynamic_robust_insert_C_warp, reference :759-877).
void robust_insert(const Store &st, uint32_t N, uint32_t C, uint32_t v, uint32_t x, float d_px, float alpha,
                   uint32_t *row, float *drow, uint32_t &wdeg, uint64_t &pairs)
{
    if (x == kInvalid || x >= N || x == v)
        return;
    uint32_t deg = std::min(wdeg, C);
    for (uint32_t i = 0; i < deg; ++i)
        if (row[i] == x)
            return;
    for (uint32_t i = 0; i < deg; ++i)
    {
        uint32_t y = row[i];
        if (y == kInvalid || y >= N || y == v)
            continue;
        if (drow[i] <= d_px)
        {
            float d_yx = dist(st, y, x);
            ++pairs;
            if (alpha * d_yx <= d_px)
                return; // occluded
        }
    }
    int worst_pos = -1, victim_pos = -1;
    float worst = -FLT_MAX, victim = -FLT_MAX;
    for (uint32_t i = 0; i < deg; ++i)
    {
        uint32_t y = row[i];
        if (y == kInvalid || y >= N || y == v)
            continue;
        float d_py = drow[i];
        if (d_py > worst)
        {
            worst = d_py;
            worst_pos = (int)i;
        }
        if (d_py > d_px)
        {
            float d_xy = dist(st, x, y);
            ++pairs;
            if (alpha * d_xy <= d_py && d_py > victim)
            {
                victim = d_py;
                victim_pos = (int)i;
            }
        }
    }
    if (victim_pos >= 0)
    {
        row[victim_pos] = x;
        drow[victim_pos] = d_px;
    }
    else if (deg < C)
    {
        row[deg] = x;
        drow[deg] = d_px;
        wdeg = deg + 1;
    }
    else if (worst_pos >= 0 && d_px < worst)
    {
        row[worst_pos] = x;
        drow[worst_pos] = d_px;
    }
}

// Reverse merge of target t (reverse_merge_csr_kernel, reference :1722-1814)
// over its sources in CSR order.
void reverse_merge_target(const Store &st, uint32_t N, uint32_t C, uint32_t t, const uint32_t *srcs, uint32_t indeg,
                          const DanceVamanaParams &p, uint32_t *row, float *drow, uint32_t &wdeg, uint64_t &evals)
{
    uint32_t deg = std::min(wdeg, C);
    uint32_t count = indeg;
    bool sampled = false;
    if (p.reverse_heavy_cap && indeg > p.reverse_heavy_threshold)
    {
        count = std::min(p.reverse_heavy_sample, indeg);
        if (count == 0)
            count = 1;
        sampled = count < indeg;
    }
    for (uint32_t k = 0; k < count; ++k)
    {
        uint32_t i = sampled ? (uint32_t)(((uint64_t)k * indeg) / count) : k;
        uint32_t s = srcs[i];
        if (s == kInvalid || s >= N || s == t)
            continue;
        bool present = false;
        for (uint32_t j = 0; j < deg; ++j)
            if (row[j] == s)
            {
                present = true;
                break;
            }
        if (present)
            continue;
        float d = dist(st, t, s);
        ++evals;
        if (deg < C)
        {
            row[deg] = s;
            drow[deg] = d;
            ++deg;
            continue;
        }
        int wpos = -1;
        float w = -FLT_MAX;
        for (uint32_t j = 0; j < C; ++j)
            if (drow[j] > w)
            {
                w = drow[j];
                wpos = (int)j;
            }
        if (wpos >= 0 && d < w)
        {
            row[wpos] = s;
            drow[wpos] = d;
        }
    }
    wdeg = deg;
}

// RobustPrune(alpha) + optional degree fill (final_prune_kernel_shared,
// reference :1893-2147).  Writes the R-wide output row.
void prune_vertex(const Store &st, uint32_t N, uint32_t R, uint32_t C, float alpha, uint32_t min_degree, uint32_t v,
                  const uint32_t *wid, const float *wd, uint32_t wdeg, uint32_t *out_ids, float *out_d,
                  uint32_t &out_deg, uint64_t &pairs)
{
    std::vector<uint32_t> sid(C);
    std::vector<float> sd(C);
    std::vector<uint8_t> removed(C);
    uint32_t deg = std::min(wdeg, C);
    for (uint32_t i = 0; i < C; ++i)
    {
        uint32_t id = kInvalid;
        float d = FLT_MAX;
        uint8_t rm = 1;
        if (i < deg)
        {
            id = wid[i];
            d = wd[i];
            if (id != kInvalid && id < N && id != v && d < FLT_MAX)
                rm = 0;
            else
                id = kInvalid;
        }
        sid[i] = id;
        sd[i] = d;
        removed[i] = rm;
    }
    for (uint32_t i = 0; i < R; ++i)
    {
        out_ids[i] = kInvalid;
        out_d[i] = FLT_MAX;
    }
    uint32_t out = 0;
    for (uint32_t round = 0; round < R; ++round)
    {
        int best = -1;
        float bd = FLT_MAX;
        for (uint32_t i = 0; i < C; ++i)
            if (!removed[i] && sid[i] != kInvalid && sid[i] < N && sid[i] != v)
                if (sd[i] < bd || (sd[i] == bd && best < 0))
                {
                    bd = sd[i];
                    best = (int)i;
                }
        if (best < 0)
            break;
        uint32_t sel = sid[best];
        float seld = sd[best];
        out_ids[out] = sel;
        out_d[out] = seld;
        ++out;
        if (out >= R)
            break;
        for (uint32_t i = 0; i < C; ++i)
            if (!removed[i] && sid[i] == sel)
                removed[i] = 1;
        for (uint32_t q = 0; q < C; ++q)
        {
            if (removed[q] || sid[q] == kInvalid || sid[q] >= N || sid[q] == v)
                continue;
            if (seld <= sd[q])
            {
                float dq = dist(st, sel, sid[q]);
                ++pairs;
                if (alpha * dq <= sd[q])
                    removed[q] = 1;
            }
        }
    }
    if (min_degree > R)
        min_degree = R;
    while (out < min_degree)
    {
        int best = -1;
        float bd = FLT_MAX;
        for (uint32_t i = 0; i < C; ++i)
        {
            uint32_t id = sid[i];
            if (id == kInvalid || id >= N || id == v)
                continue;
            bool dup = false;
            for (uint32_t j = 0; j < out; ++j)
                if (out_ids[j] == id)
                {
                    dup = true;
                    break;
                }
            if (dup)
                continue;
            if (sd[i] < bd || (sd[i] == bd && best < 0))
            {
                bd = sd[i];
                best = (int)i;
            }
        }
        if (best < 0)
            break;
        out_ids[out] = sid[best];
        out_d[out] = sd[best];
        sid[best] = kInvalid;
        ++out;
    }
    out_deg = out;
}

void set_threads(int threads)
{
#ifdef _OPENMP
    if (threads > 0)
        omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

Store make_store(int dtype, const void *data, uint64_t stride, uint32_t dim)
{
    Store st;
    st.dtype = dtype;
    st.base = reinterpret_cast<const uint8_t *>(data);
    st.stride = stride;
    st.dim = dim;
    return st;
}

uint32_t medoid(const Store &st, uint32_t N, uint32_t nc, uint32_t ns, float *scores, uint32_t *cand_ids)
{
    nc = std::min(nc, N);
    ns = std::min(ns, N);
    if (nc == 0 || ns == 0)
        return 0;
    std::vector<float> sc(nc);
    std::vector<uint32_t> ci(nc);
#pragma omp parallel for schedule(dynamic, 8)
    for (int64_t w = 0; w < (int64_t)nc; ++w)
    {
        uint32_t cand = hash_u32((uint32_t)w * 9973u + 17u) % N;
        float sum = 0.0f;
        for (uint32_t s = 0; s < ns; ++s)
        {
            uint32_t smp = hash_u32(s * 10007u + 131u) % N;
            if (smp == cand)
                continue;
            sum = sum + dist(st, cand, smp);
        }
        sc[w] = sum / (float)ns;
        ci[w] = cand;
    }
    uint32_t best = 0;
    float bs = FLT_MAX;
    bool found = false;
    for (uint32_t w = 0; w < nc; ++w)
        if (sc[w] < bs)
        {
            bs = sc[w];
            best = ci[w];
            found = true;
        }
    if (scores)
        std::memcpy(scores, sc.data(), nc * sizeof(float));
    if (cand_ids)
        std::memcpy(cand_ids, ci.data(), nc * sizeof(uint32_t));
    return found ? best : 0;
}

void init_graph(const Store &st, Graph &g)
{
#pragma omp parallel for schedule(static)
    for (int64_t v = 0; v < (int64_t)g.N; ++v)
    {
        for (uint32_t i = 0; i < g.R; ++i)
        {
            uint32_t nb = det_neighbor((uint32_t)v, i, g.N);
            if (g.N <= 1 || nb == kInvalid || nb >= g.N || nb == (uint32_t)v)
                nb = kInvalid;
            g.cur_ids[(size_t)v * g.R + i] = nb;
            g.cur_dists[(size_t)v * g.R + i] = nb != kInvalid ? dist(st, (uint32_t)v, nb) : FLT_MAX;
        }
        g.degree[v] = g.N > 1 ? g.R : 0;
    }
}

void search_and_replay_all(const Store &st, Graph &g, uint32_t L, uint32_t steps, uint32_t entry, uint32_t seeds,
                           float alpha, int pool_mode)
{
    std::atomic<uint64_t> pairs_total{0};
#pragma omp parallel
    {
        Visited vis;
        std::vector<uint32_t> eid;
        std::vector<float> ed;
        uint64_t pairs = 0;
#pragma omp for schedule(dynamic, 64)
        for (int64_t vv = 0; vv < (int64_t)g.N; ++vv)
        {
            uint32_t v = (uint32_t)vv;
            if (pool_mode == 1)
                search_vertex<SlotPool>(st, g.N, g.R, L, steps, entry, seeds, g.cur_ids.data(), g.cur_dists.data(),
                                        g.degree.data(), v, vis, eid, ed);
            else
                search_vertex<KeyPool>(st, g.N, g.R, L, steps, entry, seeds, g.cur_ids.data(), g.cur_dists.data(),
                                       g.degree.data(), v, vis, eid, ed);
            uint32_t *wid = &g.work_ids[(size_t)v * g.C];
            float *wd = &g.work_dists[(size_t)v * g.C];
            init_work_row(g.N, g.R, g.C, g.cur_ids.data(), g.cur_dists.data(), g.degree.data(), v, wid, wd,
                          g.work_deg[v]);
            for (size_t k = 0; k < eid.size(); ++k)
                robust_insert(st, g.N, g.C, v, eid[k], ed[k], alpha, wid, wd, g.work_deg[v], pairs);
        }
        pairs_total.fetch_add(pairs);
    }
    g_pair_evals.fetch_add(pairs_total.load());
}

// Reverse CSR over the first min(deg, R) work slots, sources ascending.
void build_reverse(const Graph &g, std::vector<uint32_t> &offsets, std::vector<uint32_t> &srcs)
{
    offsets.assign((size_t)g.N + 1, 0);
    for (uint32_t s = 0; s < g.N; ++s)
    {
        uint32_t deg = std::min(g.work_deg[s], g.R);
        for (uint32_t p = 0; p < deg; ++p)
        {
            uint32_t t = g.work_ids[(size_t)s * g.C + p];
            if (t != kInvalid && t < g.N && t != s)
                offsets[(size_t)t + 1]++;
        }
    }
    for (size_t i = 0; i < g.N; ++i)
        offsets[i + 1] += offsets[i];
    srcs.assign(offsets[g.N], 0);
    std::vector<uint32_t> cursor(offsets.begin(), offsets.end() - 1);
    for (uint32_t s = 0; s < g.N; ++s)
    {
        uint32_t deg = std::min(g.work_deg[s], g.R);
        for (uint32_t p = 0; p < deg; ++p)
        {
            uint32_t t = g.work_ids[(size_t)s * g.C + p];
            if (t != kInvalid && t < g.N && t != s)
                srcs[cursor[t]++] = s;
        }
    }
}

void reverse_merge_all(const Store &st, Graph &g, const DanceVamanaParams &p, uint64_t *edges_out)
{
    std::vector<uint32_t> offsets, srcs;
    build_reverse(g, offsets, srcs);
    g_reverse_edges.fetch_add(srcs.size());
    if (edges_out)
        *edges_out = srcs.size();
    std::atomic<uint64_t> ev{0};
#pragma omp parallel
    {
        uint64_t local = 0;
#pragma omp for schedule(dynamic, 256)
        for (int64_t tt = 0; tt < (int64_t)g.N; ++tt)
        {
            uint32_t t = (uint32_t)tt;
            uint32_t b = offsets[t], e = offsets[t + 1];
            if (e == b)
                continue;
            reverse_merge_target(st, g.N, g.C, t, &srcs[b], e - b, p, &g.work_ids[(size_t)t * g.C],
                                 &g.work_dists[(size_t)t * g.C], g.work_deg[t], local);
        }
        ev.fetch_add(local);
    }
    g_reverse_evals.fetch_add(ev.load());
}

void prune_all(const Store &st, Graph &g, float alpha, uint32_t min_degree)
{
    std::atomic<uint64_t> pt{0};
#pragma omp parallel
    {
        uint64_t pairs = 0;
#pragma omp for schedule(dynamic, 64)
        for (int64_t vv = 0; vv < (int64_t)g.N; ++vv)
        {
            uint32_t v = (uint32_t)vv;
            prune_vertex(st, g.N, g.R, g.C, alpha, min_degree, v, &g.work_ids[(size_t)v * g.C],
                         &g.work_dists[(size_t)v * g.C], g.work_deg[v], &g.cur_ids[(size_t)v * g.R],
                         &g.cur_dists[(size_t)v * g.R], g.degree[v], pairs);
        }
        pt.fetch_add(pairs);
    }
    g_pair_evals.fetch_add(pt.load());
}

} // namespace

// ====================================================================== C ABI
extern "C" {

void oracle_default_params(DanceVamanaParams *p)
{
    std::memset(p, 0, sizeof(*p));
    p->iters = 4;
    p->alpha = 1.2f;
    p->init_random_seeds = 8;
    p->final_min_degree = 64;
    p->medoid_candidates = 1024;
    p->medoid_samples = 4096;
    p->coarse_warmup_iters = 2;
    p->warmup_expand_steps = 64;
    p->reverse_heavy_cap = 0;
    p->reverse_heavy_threshold = 256;
    p->reverse_heavy_sample = 256;
    p->visited_log2 = 10;
}

void oracle_reset_counters(void)
{
    g_search_evals = 0;
    g_search_expansions = 0;
    g_pair_evals = 0;
    g_reverse_evals = 0;
    g_reverse_edges = 0;
    g_seed_mismatch = 0;
}

// out[0..5] = search evals, expansions, pair evals (insert + prune),
// reverse evals, reverse edges, stored/computed distance mismatches.
void oracle_get_counters(uint64_t *out)
{
    out[0] = g_search_evals;
    out[1] = g_search_expansions;
    out[2] = g_pair_evals;
    out[3] = g_reverse_evals;
    out[4] = g_reverse_edges;
    out[5] = g_seed_mismatch;
}

float oracle_distance(int dtype, const void *a, const void *b, uint32_t dim)
{
    switch (dtype)
    {
    case DANCE_U8:
        return dist_u8((const uint8_t *)a, (const uint8_t *)b, dim);
    case DANCE_F16:
        return dist_f16((const uint16_t *)a, (const uint16_t *)b, dim);
    default:
        return dist_f32((const float *)a, (const float *)b, dim);
    }
}

// float32 -> binary16 (round to nearest even) for the fp16 storage mode.
void oracle_float_to_half(const float *src, uint16_t *dst, uint64_t n)
{
    for (uint64_t i = 0; i < n; ++i)
        dst[i] = double_to_half_bits((double)src[i]);
}

// Mismatches between double_to_half_bits and the frexp definition over
// every half value, the midpoints and quarter points between neighbouring
// halves, and n_random differences of random half pairs.
uint64_t oracle_half_selftest(uint64_t n_random)
{
    const HalfTables &t = half_tables();
    uint64_t bad = 0;
    for (uint32_t h = 0; h < 0x7C00u; ++h)
    {
        const double lo = (double)t.h2f[h], hi = (double)t.h2f[h + 1];
        const double probes[5] = {lo, 0.5 * (lo + hi), 0.25 * (3 * lo + hi), 0.25 * (lo + 3 * hi), hi};
        for (double v : probes)
            for (double sgn : {1.0, -1.0})
                bad += double_to_half_bits(sgn * v) != double_to_half(sgn * v);
    }
    uint64_t st = 0x9E3779B97F4A7C15ull;
    for (uint64_t i = 0; i < n_random; ++i)
    {
        st ^= st << 13;
        st ^= st >> 7;
        st ^= st << 17;
        const uint16_t a = (uint16_t)(st & 0x7BFFu), b = (uint16_t)((st >> 16) & 0xFBFFu);
        const double d = (double)t.h2f[a] - (double)t.h2f[b];
        bad += double_to_half_bits(d) != double_to_half(d);
        bad += double_to_half_bits(d * d) != double_to_half(d * d);
    }
    return bad;
}

uint32_t oracle_hash_u32(uint32_t x) { return hash_u32(x); }

// Shard-merge rank hash (reference src/gpu_merge.cu:92-101).
uint32_t oracle_hash_edge32(uint32_t src, uint32_t dst, uint64_t seed)
{
    uint64_t x = ((uint64_t)src << 32) ^ (uint64_t)dst ^ seed;
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdULL;
    x ^= x >> 33;
    x *= 0xc4ceb9fe1a85ec53ULL;
    x ^= x >> 33;
    return (uint32_t)(x ^ (x >> 32));
}

// Merge of global edges (reference merge_shards_gpu pass 2, :586-731):
// per source, distinct destinations other than itself, ranked by
// (hash_edge32, destination), first max_degree kept.
int oracle_merge_edges(const uint32_t *src, const uint32_t *dst, uint64_t n, uint32_t nnodes, uint32_t max_degree,
                       uint64_t seed, uint32_t *out_rows, uint32_t *out_deg)
{
    std::vector<std::vector<uint32_t>> adj(nnodes);
    for (uint64_t i = 0; i < n; ++i)
        if (src[i] < nnodes && src[i] != dst[i])
            adj[src[i]].push_back(dst[i]);
    for (uint32_t v = 0; v < nnodes; ++v)
    {
        auto &a = adj[v];
        std::sort(a.begin(), a.end());
        a.erase(std::unique(a.begin(), a.end()), a.end());
        std::vector<std::pair<uint32_t, uint32_t>> k;
        for (uint32_t d : a)
            k.emplace_back(oracle_hash_edge32(v, d, seed), d);
        std::sort(k.begin(), k.end());
        const uint32_t keep = std::min<uint32_t>((uint32_t)k.size(), max_degree);
        out_deg[v] = keep;
        for (uint32_t j = 0; j < max_degree; ++j)
            out_rows[(size_t)v * max_degree + j] = j < keep ? k[j].second : kInvalid;
    }
    return 0;
}
uint32_t oracle_det_neighbor(uint32_t node, uint32_t k, uint32_t N) { return det_neighbor(node, k, N); }

uint32_t oracle_medoid(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t nc,
                       uint32_t ns, float *scores, uint32_t *cand_ids, int threads)
{
    set_threads(threads);
    Store st = make_store(dtype, data, stride, dim);
    return medoid(st, N, nc, ns, scores, cand_ids);
}

int oracle_init(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                uint32_t *cur_ids, float *cur_dists, uint32_t *degree, int threads)
{
    set_threads(threads);
    Store st = make_store(dtype, data, stride, dim);
    Graph g;
    g.N = N;
    g.R = R;
    g.C = R;
    g.cur_ids.resize((size_t)N * R);
    g.cur_dists.resize((size_t)N * R);
    g.degree.resize(N);
    init_graph(st, g);
    std::memcpy(cur_ids, g.cur_ids.data(), g.cur_ids.size() * 4);
    std::memcpy(cur_dists, g.cur_dists.data(), g.cur_dists.size() * 4);
    std::memcpy(degree, g.degree.data(), g.degree.size() * 4);
    return 0;
}

// Expansion sequences of every vertex (exp_stride slots each).
int oracle_search(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R, uint32_t L,
                  uint32_t steps, uint32_t entry, uint32_t seeds, int pool_mode, const uint32_t *cur_ids,
                  const float *cur_dists, const uint32_t *degree, uint32_t *exp_ids, float *exp_dists,
                  uint32_t *exp_count, uint32_t exp_stride, int threads)
{
    set_threads(threads);
    Store st = make_store(dtype, data, stride, dim);
    steps = std::min(steps, L);
    if (steps > exp_stride)
        return -1;
#pragma omp parallel
    {
        Visited vis;
        std::vector<uint32_t> eid;
        std::vector<float> ed;
#pragma omp for schedule(dynamic, 64)
        for (int64_t vv = 0; vv < (int64_t)N; ++vv)
        {
            uint32_t v = (uint32_t)vv;
            if (pool_mode == 1)
                search_vertex<SlotPool>(st, N, R, L, steps, entry, seeds, cur_ids, cur_dists, degree, v, vis, eid,
                                        ed);
            else
                search_vertex<KeyPool>(st, N, R, L, steps, entry, seeds, cur_ids, cur_dists, degree, v, vis, eid, ed);
            exp_count[v] = (uint32_t)eid.size();
            for (uint32_t k = 0; k < exp_stride; ++k)
            {
                exp_ids[(size_t)v * exp_stride + k] = k < eid.size() ? eid[k] : kInvalid;
                exp_dists[(size_t)v * exp_stride + k] = k < eid.size() ? ed[k] : FLT_MAX;
            }
        }
    }
    return 0;
}

int oracle_replay(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R, uint32_t C,
                  float alpha, const uint32_t *cur_ids, const float *cur_dists, const uint32_t *degree,
                  const uint32_t *exp_ids, const float *exp_dists, const uint32_t *exp_count, uint32_t exp_stride,
                  uint32_t *work_ids, float *work_dists, uint32_t *work_deg, int threads)
{
    set_threads(threads);
    Store st = make_store(dtype, data, stride, dim);
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t vv = 0; vv < (int64_t)N; ++vv)
    {
        uint32_t v = (uint32_t)vv;
        uint64_t pairs = 0;
        uint32_t *wid = &work_ids[(size_t)v * C];
        float *wd = &work_dists[(size_t)v * C];
        init_work_row(N, R, C, cur_ids, cur_dists, degree, v, wid, wd, work_deg[v]);
        for (uint32_t k = 0; k < exp_count[v]; ++k)
            robust_insert(st, N, C, v, exp_ids[(size_t)v * exp_stride + k], exp_dists[(size_t)v * exp_stride + k],
                          alpha, wid, wd, work_deg[v], pairs);
    }
    return 0;
}

int oracle_reverse_merge(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                         uint32_t C, const DanceVamanaParams *params, uint32_t *work_ids, float *work_dists,
                         uint32_t *work_deg, uint64_t *edges_out, int threads)
{
    set_threads(threads);
    Store st = make_store(dtype, data, stride, dim);
    Graph g;
    g.N = N;
    g.R = R;
    g.C = C;
    g.work_ids.assign(work_ids, work_ids + (size_t)N * C);
    g.work_dists.assign(work_dists, work_dists + (size_t)N * C);
    g.work_deg.assign(work_deg, work_deg + N);
    DanceVamanaParams p;
    if (params)
        p = *params;
    else
        oracle_default_params(&p);
    reverse_merge_all(st, g, p, edges_out);
    std::memcpy(work_ids, g.work_ids.data(), g.work_ids.size() * 4);
    std::memcpy(work_dists, g.work_dists.data(), g.work_dists.size() * 4);
    std::memcpy(work_deg, g.work_deg.data(), g.work_deg.size() * 4);
    return 0;
}

int oracle_prune(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R, uint32_t C,
                 float alpha, uint32_t min_degree, const uint32_t *work_ids, const float *work_dists,
                 const uint32_t *work_deg, uint32_t *cur_ids, float *cur_dists, uint32_t *degree, int threads)
{
    set_threads(threads);
    Store st = make_store(dtype, data, stride, dim);
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t vv = 0; vv < (int64_t)N; ++vv)
    {
        uint32_t v = (uint32_t)vv;
        uint64_t pairs = 0;
        prune_vertex(st, N, R, C, alpha, min_degree, v, &work_ids[(size_t)v * C], &work_dists[(size_t)v * C],
                     work_deg[v], &cur_ids[(size_t)v * R], &cur_dists[(size_t)v * R], degree[v], pairs);
    }
    return 0;
}

// Whole build (round driver, reference :2170-2855).
int oracle_build(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R, uint32_t L,
                 uint32_t C, uint32_t STEPS, const DanceVamanaParams *params, int pool_mode, int threads,
                 uint32_t *graph, uint32_t *degree, float *dists, uint32_t *medoid_out)
{
    if (!data || !graph || !degree || N == 0 || dim == 0 || R == 0 || L == 0 || C == 0 || STEPS == 0 || C < R)
        return -1;
    set_threads(threads);
    DanceVamanaParams p;
    if (params)
        p = *params;
    else
        oracle_default_params(&p);
    if (STEPS > L)
        STEPS = L;
    Store st = make_store(dtype, data, stride, dim);
    uint32_t entry = medoid(st, N, p.medoid_candidates, p.medoid_samples, nullptr, nullptr);
    Graph g;
    g.N = N;
    g.R = R;
    g.C = C;
    g.cur_ids.resize((size_t)N * R);
    g.cur_dists.resize((size_t)N * R);
    g.degree.resize(N);
    g.work_ids.resize((size_t)N * C);
    g.work_dists.resize((size_t)N * C);
    g.work_deg.resize(N);
    init_graph(st, g);
    for (uint32_t it = 0; it < p.iters; ++it)
    {
        float alpha = (it + 1 >= p.iters) ? p.alpha : 1.0f;
        uint32_t steps = STEPS;
        if (it < p.coarse_warmup_iters && steps > p.warmup_expand_steps)
            steps = p.warmup_expand_steps;
        search_and_replay_all(st, g, L, steps, entry, p.init_random_seeds, alpha, pool_mode);
        reverse_merge_all(st, g, p, nullptr);
        uint32_t min_degree = (it + 1 == p.iters) ? p.final_min_degree : 0;
        prune_all(st, g, alpha, min_degree);
    }
    std::memcpy(graph, g.cur_ids.data(), g.cur_ids.size() * 4);
    std::memcpy(degree, g.degree.data(), g.degree.size() * 4);
    if (dists)
        std::memcpy(dists, g.cur_dists.data(), g.cur_dists.size() * 4);
    if (medoid_out)
        *medoid_out = entry;
    return 0;
}

// DiskANN-style best-first query search (list size L, K results), pool
// ordered by (distance, id); runs until every list entry is expanded.
int oracle_search_queries(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim,
                          const uint32_t *graph, uint32_t R, uint32_t start, const void *queries, uint64_t qstride,
                          uint32_t nq, uint32_t L, uint32_t K, uint32_t *out_ids, float *out_dists, int threads)
{
    set_threads(threads);
    Store st = make_store(dtype, data, stride, dim);
    const uint8_t *qb = reinterpret_cast<const uint8_t *>(queries);
#pragma omp parallel
    {
        Visited vis;
#pragma omp for schedule(dynamic, 16)
        for (int64_t qi = 0; qi < (int64_t)nq; ++qi)
        {
            const uint8_t *q = qb + (uint64_t)qi * qstride;
            KeyPool pool(L);
            vis.reset(N);
            if (start < N)
            {
                vis.test_and_set(start);
                pool.insert(start, dist_query(st, q, start));
            }
            uint32_t x;
            float dx;
            while (pool.next(x, dx))
            {
                for (uint32_t p = 0; p < R; ++p)
                {
                    uint32_t c = graph[(size_t)x * R + p];
                    if (c == kInvalid || c >= N)
                        continue;
                    if (vis.test_and_set(c))
                        continue;
                    pool.insert(c, dist_query(st, q, c));
                }
            }
            for (uint32_t k = 0; k < K; ++k)
            {
                if (k < pool.keys.size())
                {
                    out_ids[(size_t)qi * K + k] = (uint32_t)(pool.keys[k] & 0xFFFFFFFFu);
                    uint32_t bits = (uint32_t)(pool.keys[k] >> 32);
                    float d;
                    std::memcpy(&d, &bits, 4);
                    out_dists[(size_t)qi * K + k] = d;
                }
                else
                {
                    out_ids[(size_t)qi * K + k] = kInvalid;
                    out_dists[(size_t)qi * K + k] = FLT_MAX;
                }
            }
        }
    }
    return 0;
}

} // extern "C"

// ====================================================================== GPU-FilteredVamana
// Restatement of the reference's canonical filtered builder
// (src/gpu_vamana_filtered.cu): deterministic random initial graph
// (:716-744), then three rounds of label-masked per-(row, label) search
// (:4266-4426), union-label search (:4530-4670), fixed-order merge with label
// quotas (:4672-4842), missing work distances (:4845-4871), FilteredRobustPrune
// (:4877-4994) and the exact CSR reverse repair (:4996-5230), driven as in
// canonical_round0_from_host_backbone_typed (:5663-6300).  Pools are the
// reference's unsorted slot arrays (insert_top_l_state_warp :4187-4233,
// select_next_unexpanded_size_warp :4235-4263), restated literally.
//
// One deliberate difference: a row with reverse sources gets the list (its
// forward row, then the new reverse sources).  The reference's fill kernel
// (:5071-5105) also writes the forward rows of rows WITHOUT reverse sources,
// at the start of the next row's list range, so the list of a row that
// follows such a row depends on which concurrent store lands last; those
// rows cannot be reproduced and follow the rule above instead.
namespace
{
struct LabelSets
{
    const uint32_t *off;
    const uint32_t *lab;
    uint32_t num_labels;
    uint32_t universal;
    // point_has_exact_label_device (:557-571): labels of a point ascend.
    bool has(uint32_t p, uint32_t l) const
    {
        for (uint32_t i = off[p]; i < off[p + 1]; ++i)
        {
            if (lab[i] == l)
                return true;
            if (lab[i] > l)
                break;
        }
        return false;
    }
    // has_common_label_device (:495-529) with no universal label
    bool common(uint32_t a, uint32_t b) const
    {
        uint32_t i = off[a], j = off[b];
        while (i < off[a + 1] && j < off[b + 1])
        {
            if (lab[i] == lab[j])
                return true;
            if (lab[i] < lab[j])
                ++i;
            else
                ++j;
        }
        return false;
    }
    // filtered_selected_covers_common_labels (include/filtered_label_coverage.cuh:8-45)
    bool covers(uint32_t target, uint32_t selected, uint32_t cand) const
    {
        uint32_t t = off[target], c = off[cand];
        while (t < off[target + 1] && c < off[cand + 1])
        {
            if (lab[t] < lab[c])
                ++t;
            else if (lab[c] < lab[t])
                ++c;
            else
            {
                bool found = false;
                for (uint32_t s = off[selected]; s < off[selected + 1]; ++s)
                {
                    if (lab[s] == lab[t])
                    {
                        found = true;
                        break;
                    }
                    if (lab[s] > lab[t])
                        break;
                }
                if (!found)
                    return false;
                ++t;
                ++c;
            }
        }
        return true;
    }
};

uint32_t fhash(uint32_t x) { return hash_u32(x); } // filtered_hash_u32 (:694-702) is the same finaliser

struct FSlotPool
{
    uint32_t cap, count = 0;
    std::vector<uint32_t> ids;
    std::vector<float> d;
    std::vector<uint8_t> exp;
    explicit FSlotPool(uint32_t c) : cap(c), ids(c, kInvalid), d(c, FLT_MAX), exp(c, 0) {}
    static bool greater(float da, uint32_t ia, float db, uint32_t ib) { return da > db || (da == db && ia > ib); }
    void insert(uint32_t id, float dist)
    {
        if (id == kInvalid)
            return;
        for (uint32_t p = 0; p < count; ++p)
            if (ids[p] == id)
            {
                if (dist < d[p])
                {
                    d[p] = dist;
                    exp[p] = 0;
                }
                return;
            }
        if (count < cap)
        {
            ids[count] = id;
            d[count] = dist;
            exp[count] = 0;
            ++count;
            return;
        }
        int w = -1;
        for (uint32_t p = 0; p < count; ++p)
            if (w < 0 || greater(d[p], ids[p], d[w], ids[w]))
                w = (int)p;
        if (w >= 0 && (dist < d[w] || (dist == d[w] && id < ids[w])))
        {
            ids[w] = id;
            d[w] = dist;
            exp[w] = 0;
        }
    }
    int select() const
    {
        int b = -1;
        for (uint32_t p = 0; p < count; ++p)
            if (!exp[p] && (b < 0 || d[p] < d[b] || (d[p] == d[b] && ids[p] < ids[b])))
                b = (int)p;
        return b;
    }
};

struct FilteredCtx
{
    Store st;
    uint32_t N, R;
    LabelSets ls;
    const uint32_t *starts;
    std::vector<uint32_t> lp_off, lp; // label -> points (ascending)
    void build_postings()
    {
        lp_off.assign((size_t)ls.num_labels + 1, 0);
        for (uint32_t p = 0; p < N; ++p)
            for (uint32_t i = ls.off[p]; i < ls.off[p + 1]; ++i)
                if (ls.lab[i] < ls.num_labels)
                    ++lp_off[ls.lab[i] + 1];
        for (uint32_t l = 0; l < ls.num_labels; ++l)
            lp_off[l + 1] += lp_off[l];
        lp.assign(lp_off[ls.num_labels], kInvalid);
        std::vector<uint32_t> cur(lp_off.begin(), lp_off.end() - 1);
        for (uint32_t p = 0; p < N; ++p)
            for (uint32_t i = ls.off[p]; i < ls.off[p + 1]; ++i)
                if (ls.lab[i] < ls.num_labels)
                    lp[cur[ls.lab[i]]++] = p;
    }
};

// filtered_deterministic_random_graph_kernel (:716-744)
void filtered_random_graph(uint32_t N, uint32_t R, uint32_t initial_degree, uint32_t seed, uint32_t *graph,
                           uint32_t *degrees)
{
    const uint32_t target = std::min(std::min(R, initial_degree), N > 0 ? N - 1 : 0u);
    for (uint32_t row = 0; row < N; ++row)
    {
        uint32_t *g = graph + (size_t)row * R;
        uint32_t deg = 0, attempt = 0;
        while (deg < target && attempt < (1u << 24))
        {
            const uint32_t c = fhash(row * 0x9e3779b1u ^ seed * 0x85ebca6bu ^ attempt * 0xc2b2ae35u) % N;
            ++attempt;
            if (c == row)
                continue;
            bool dup = false;
            for (uint32_t i = 0; i < deg; ++i)
                dup |= g[i] == c;
            if (!dup)
                g[deg++] = c;
        }
        for (uint32_t i = deg; i < R; ++i)
            g[i] = kInvalid;
        degrees[row] = deg;
    }
}

// canonical_filtered_task_search (:4266-4426) for task p (row, label at
// label position p); label_seed_count 16, no posting anchor.
void task_search(const FilteredCtx &cx, uint32_t p, uint32_t row, const uint32_t *graph, const uint32_t *deg,
                 uint32_t pool_cap, uint32_t keep, uint32_t steps, uint32_t *out_ids, float *out_d)
{
    const uint32_t N = cx.N, R = cx.R;
    const uint32_t label = cx.ls.lab[p];
    for (uint32_t i = 0; i < keep; ++i)
    {
        out_ids[i] = kInvalid;
        out_d[i] = FLT_MAX;
    }
    if (row >= N || label >= cx.ls.num_labels || label == cx.ls.universal)
        return;
    FSlotPool pool(pool_cap);
    const uint32_t start = cx.starts[label];
    if (start < N && start != row)
        pool.insert(start, dist(cx.st, row, start));
    const uint32_t pb = cx.lp_off[label], pc = cx.lp_off[label + 1] - pb;
    const uint32_t nseed = std::min(16u, pc);
    for (uint32_t s = 0; s < nseed; ++s)
    {
        const uint32_t seed = cx.lp[pb + fhash(row + s * 7919u + label * 17u) % pc];
        if (seed >= N || seed == row)
            continue;
        pool.insert(seed, dist(cx.st, row, seed));
    }
    auto scan = [&](uint32_t x) {
        const uint32_t dx = std::min(deg[x], R);
        for (uint32_t j = 0; j < dx; ++j)
        {
            const uint32_t c = graph[(size_t)x * R + j];
            if (c >= N || c == row || !cx.ls.has(c, label))
                continue;
            pool.insert(c, dist(cx.st, row, c));
        }
    };
    scan(row);
    for (uint32_t step = 0; step < steps; ++step)
    {
        const int e = pool.select();
        if (e < 0)
            break;
        pool.exp[e] = 1;
        scan(pool.ids[e]);
    }
    for (uint32_t i = 0; i < keep && i < pool.count; ++i)
    {
        out_ids[i] = pool.ids[i];
        out_d[i] = pool.d[i];
    }
}

// canonical_ordinary_search (:4530-4670), label_seed_count 64, restricted
// traversal, all slots output.
void ordinary_search(const FilteredCtx &cx, uint32_t row, uint32_t global_start, const uint32_t *graph,
                     const uint32_t *deg, uint32_t pool_cap, uint32_t keep, uint32_t steps, uint32_t *out_ids,
                     float *out_d)
{
    const uint32_t N = cx.N, R = cx.R;
    const LabelSets &ls = cx.ls;
    FSlotPool pool(pool_cap);
    auto compatible = [&](uint32_t c) {
        for (uint32_t p = ls.off[row]; p < ls.off[row + 1]; ++p)
            if (ls.has(c, ls.lab[p]))
                return true;
        return false;
    };
    for (uint32_t p = ls.off[row]; p < ls.off[row + 1]; ++p)
    {
        const uint32_t label = ls.lab[p];
        if (label >= ls.num_labels)
            continue;
        const uint32_t start = cx.starts[label];
        if (start < N && start != row)
            pool.insert(start, dist(cx.st, row, start));
        const uint32_t pb = cx.lp_off[label], pc = cx.lp_off[label + 1] - pb;
        const uint32_t nseed = std::min(64u, pc);
        for (uint32_t s = 0; s < nseed; ++s)
        {
            const uint32_t seed = cx.lp[pb + fhash(row + s * 7919u + label * 17u) % pc];
            if (seed >= N || seed == row)
                continue;
            pool.insert(seed, dist(cx.st, row, seed));
        }
    }
    if (global_start < N && global_start != row && compatible(global_start))
        pool.insert(global_start, dist(cx.st, row, global_start));
    auto scan = [&](uint32_t x) {
        const uint32_t dx = std::min(deg[x], R);
        for (uint32_t j = 0; j < dx; ++j)
        {
            const uint32_t c = graph[(size_t)x * R + j];
            if (c >= N || c == row || !compatible(c))
                continue;
            pool.insert(c, dist(cx.st, row, c));
        }
    };
    scan(row);
    for (uint32_t step = 0; step < steps; ++step)
    {
        const int e = pool.select();
        if (e < 0)
            break;
        pool.exp[e] = 1;
        scan(pool.ids[e]);
    }
    for (uint32_t i = 0; i < keep; ++i)
    {
        out_ids[i] = i < pool.count ? pool.ids[i] : kInvalid;
        out_d[i] = i < pool.count ? pool.d[i] : FLT_MAX;
    }
}

// canonical_merge_candidates (:4703-4842) without the unrestricted-round
// options, then canonical_compute_work_distances (:4845-4871).
uint32_t merge_row(const FilteredCtx &cx, uint32_t row, uint32_t C, uint32_t per_label_keep, uint32_t ord_keep,
                   const uint32_t *graph, const uint32_t *deg, const uint32_t *task_ids, const float *task_d,
                   const uint32_t *ord_ids, const float *ord_d, uint32_t *w, float *wd)
{
    const uint32_t N = cx.N, R = cx.R;
    const LabelSets &ls = cx.ls;
    for (uint32_t i = 0; i < C; ++i)
    {
        w[i] = kInvalid;
        wd[i] = FLT_MAX;
    }
    uint32_t count = 0;
    auto add = [&](uint32_t c, float d) {
        if (c >= N || c == row || count >= C)
            return;
        for (uint32_t i = 0; i < count; ++i)
            if (w[i] == c)
            {
                if (d < wd[i])
                    wd[i] = d;
                return;
            }
        w[count] = c;
        wd[count] = d;
        ++count;
    };
    for (uint32_t p = ls.off[row]; p < ls.off[row + 1]; ++p)
        for (uint32_t i = 0; i < per_label_keep; ++i)
            add(task_ids[(size_t)p * per_label_keep + i], task_d[(size_t)p * per_label_keep + i]);
    const uint32_t dr = std::min(deg[row], R);
    for (uint32_t i = 0; i < dr; ++i)
    {
        const uint32_t c = graph[(size_t)row * R + i];
        if (c < N && c != row && ls.common(row, c))
            add(c, FLT_MAX);
    }
    for (uint32_t i = 0; i < ord_keep; ++i)
        add(ord_ids[i], ord_d[i]);
    const uint32_t nl = ls.off[row + 1] - ls.off[row];
    if (nl > 0 && nl <= 16)
    {
        uint32_t assigned[16] = {};
        uint32_t quota = (R + nl - 1) / nl;
        if (quota < per_label_keep)
            quota = per_label_keep;
        uint32_t kept = 0;
        for (uint32_t i = 0; i < count; ++i)
        {
            const uint32_t c = w[i];
            uint32_t bq = kInvalid, bcard = kInvalid;
            for (uint32_t q = 0; q < nl; ++q)
            {
                const uint32_t label = ls.lab[ls.off[row] + q];
                if (assigned[q] >= quota || !ls.has(c, label))
                    continue;
                const uint32_t card = cx.lp_off[label + 1] - cx.lp_off[label];
                if (bq == kInvalid || card < bcard || (card == bcard && label < ls.lab[ls.off[row] + bq]))
                {
                    bq = q;
                    bcard = card;
                }
            }
            if (bq == kInvalid)
                continue;
            w[kept] = c;
            wd[kept] = wd[i];
            ++assigned[bq];
            ++kept;
        }
        for (uint32_t i = kept; i < count; ++i)
        {
            w[i] = kInvalid;
            wd[i] = FLT_MAX;
        }
        count = kept;
    }
    for (uint32_t i = 0; i < count; ++i)
        if (wd[i] == FLT_MAX)
            wd[i] = dist(cx.st, row, w[i]);
    return count;
}

// canonical_exact_prune (:4877-4994) / canonical_exact_prune_csr (:5131-5230):
// select the least (distance, id); drop q iff the selection covers every
// label q shares with the row and 0 < alpha * d(sel, q) <= d(row, q).
uint32_t filtered_prune(const FilteredCtx &cx, uint32_t row, float alpha, const uint32_t *cand, const float *cd,
                        uint32_t n, uint32_t *out)
{
    std::vector<uint8_t> removed(n, 0);
    uint32_t sel = 0;
    while (sel < cx.R)
    {
        int b = -1;
        for (uint32_t i = 0; i < n; ++i)
        {
            if (removed[i])
                continue;
            if (b < 0 || cd[i] < cd[b] || (cd[i] == cd[b] && cand[i] < cand[b]))
                b = (int)i;
        }
        if (b < 0)
            break;
        const uint32_t best = cand[b];
        out[sel++] = best;
        removed[b] = 1;
        for (uint32_t i = 0; i < n; ++i)
        {
            if (removed[i] || !cx.ls.covers(row, best, cand[i]))
                continue;
            const float pd = dist(cx.st, best, cand[i]);
            g_pair_evals.fetch_add(1, std::memory_order_relaxed);
            if (pd > 0.0f && alpha * pd <= cd[i])
                removed[i] = 1;
        }
    }
    return sel;
}

struct FilteredCounters
{
    uint64_t tasks = 0, reverse_edges = 0, touched = 0;
};

struct RoundOut
{
    std::vector<uint32_t> *work, *work_deg, *fwd, *fwd_deg;
    std::vector<float> *work_d;
};

// One canonical round: graph_a -> graph_b (forward prune, then exact CSR reverse repair).
void filtered_round(const FilteredCtx &cx, uint32_t C, uint32_t L, uint32_t FL, uint32_t steps, float alpha,
                    uint32_t global_start, const std::vector<uint32_t> &ga, const std::vector<uint32_t> &da,
                    std::vector<uint32_t> &gb, std::vector<uint32_t> &db, int threads, FilteredCounters &fc,
                    const RoundOut *ro)
{
    const uint32_t N = cx.N, R = cx.R;
    const uint32_t plp = std::min(FL, 32u), plk = std::min(plp, 8u);
    const uint32_t ord_keep = std::min(R, L), ord_pool = std::min(64u, FL);
    const uint32_t T = cx.ls.off[N];
    std::vector<uint32_t> tids((size_t)T * plk);
    std::vector<float> td((size_t)T * plk);
#pragma omp parallel for schedule(dynamic, 64) num_threads(threads)
    for (int64_t row = 0; row < (int64_t)N; ++row)
        for (uint32_t p = cx.ls.off[row]; p < cx.ls.off[row + 1]; ++p)
            task_search(cx, p, (uint32_t)row, ga.data(), da.data(), plp, plk, steps, &tids[(size_t)p * plk],
                        &td[(size_t)p * plk]);
    fc.tasks += T;
    std::vector<uint32_t> w((size_t)N * C);
    std::vector<float> wd((size_t)N * C);
    std::vector<uint32_t> wdeg(N);
#pragma omp parallel num_threads(threads)
    {
        std::vector<uint32_t> oid(ord_keep);
        std::vector<float> od(ord_keep);
#pragma omp for schedule(dynamic, 64)
        for (int64_t row = 0; row < (int64_t)N; ++row)
        {
            ordinary_search(cx, (uint32_t)row, global_start, ga.data(), da.data(), ord_pool, ord_keep, steps,
                            oid.data(), od.data());
            wdeg[row] = merge_row(cx, (uint32_t)row, C, plk, ord_keep, ga.data(), da.data(), tids.data(), td.data(),
                                  oid.data(), od.data(), &w[(size_t)row * C], &wd[(size_t)row * C]);
        }
    }
    gb.assign((size_t)N * R, kInvalid);
    db.assign(N, 0);
#pragma omp parallel for schedule(dynamic, 64) num_threads(threads)
    for (int64_t row = 0; row < (int64_t)N; ++row)
        db[row] = filtered_prune(cx, (uint32_t)row, alpha, &w[(size_t)row * C], &wd[(size_t)row * C], wdeg[row],
                                 &gb[(size_t)row * R]);
    if (ro)
    {
        *ro->work = w;
        *ro->work_d = wd;
        *ro->work_deg = wdeg;
        *ro->fwd = gb;
        *ro->fwd_deg = db;
    }
    // exact CSR reverse repair on the forward-pruned graph
    std::vector<std::vector<uint32_t>> rev(N);
    for (uint32_t s = 0; s < N; ++s)
        for (uint32_t i = 0; i < std::min(db[s], R); ++i)
        {
            const uint32_t t = gb[(size_t)s * R + i];
            if (t < N && t != s)
                rev[t].push_back(s);
        }
    std::vector<uint32_t> fwd_b = gb, fdeg_b = db;
    uint64_t edges = 0, touched = 0;
#pragma omp parallel for schedule(dynamic, 16) num_threads(threads) reduction(+ : edges, touched)
    for (int64_t row = 0; row < (int64_t)N; ++row)
    {
        if (rev[row].empty())
            continue;
        edges += rev[row].size();
        ++touched;
        const uint32_t dr = std::min(fdeg_b[row], R);
        std::vector<uint32_t> cand(fwd_b.begin() + (size_t)row * R, fwd_b.begin() + (size_t)row * R + dr);
        for (uint32_t s : rev[row])
        {
            bool dup = s >= N || s == (uint32_t)row;
            for (uint32_t i = 0; !dup && i < dr; ++i)
                dup = fwd_b[(size_t)row * R + i] == s;
            if (!dup)
                cand.push_back(s);
        }
        std::vector<float> cd(cand.size());
        for (size_t i = 0; i < cand.size(); ++i)
            cd[i] = dist(cx.st, (uint32_t)row, cand[i]);
        uint32_t *out = &gb[(size_t)row * R];
        for (uint32_t i = 0; i < R; ++i)
            out[i] = kInvalid;
        db[row] = filtered_prune(cx, (uint32_t)row, alpha, cand.data(), cd.data(), (uint32_t)cand.size(), out);
    }
    fc.reverse_edges += edges;
    fc.touched += touched;
}

FilteredCtx make_ctx(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                     const uint32_t *offsets, const uint32_t *labels, const uint32_t *starts, uint32_t num_labels,
                     uint32_t universal)
{
    FilteredCtx cx{Store{dtype, static_cast<const uint8_t *>(data), stride, dim}, N, R,
                   LabelSets{offsets, labels, num_labels, universal}, starts, {}, {}};
    cx.build_postings();
    return cx;
}

} // namespace

extern "C" {

void oracle_filtered_random_graph(uint32_t N, uint32_t R, uint32_t initial_degree, uint32_t seed, uint32_t *graph,
                                  uint32_t *degrees)
{
    filtered_random_graph(N, R, initial_degree, seed, graph, degrees);
}

// One round from a given graph; optional work rows (N x C) and forward graph (N x R).
int oracle_filtered_round(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                          uint32_t L, uint32_t FL, uint32_t C, uint32_t STEPS, float alpha, const uint32_t *offsets,
                          const uint32_t *labels, const uint32_t *starts, uint32_t num_labels, uint32_t universal,
                          uint32_t global_start, const uint32_t *graph_in, const uint32_t *degree_in,
                          uint32_t *graph_out, uint32_t *degree_out, uint32_t *work_ids, float *work_dists,
                          uint32_t *work_deg, uint32_t *fwd_graph, uint32_t *fwd_deg, int threads)
{
    const FilteredCtx cx = make_ctx(dtype, data, stride, N, dim, R, offsets, labels, starts, num_labels, universal);
    std::vector<uint32_t> ga(graph_in, graph_in + (size_t)N * R), da(degree_in, degree_in + N), gb, db;
    FilteredCounters fc;
    std::vector<uint32_t> w, wdeg, fg, fd;
    std::vector<float> wd;
    RoundOut ro{&w, &wdeg, &fg, &fd, &wd};
    filtered_round(cx, C, L, FL, STEPS, alpha, global_start, ga, da, gb, db, threads, fc, &ro);
    std::copy(gb.begin(), gb.end(), graph_out);
    std::copy(db.begin(), db.end(), degree_out);
    if (work_ids)
    {
        std::copy(w.begin(), w.end(), work_ids);
        std::copy(wd.begin(), wd.end(), work_dists);
        std::copy(wdeg.begin(), wdeg.end(), work_deg);
    }
    if (fwd_graph)
    {
        std::copy(fg.begin(), fg.end(), fwd_graph);
        std::copy(fd.begin(), fd.end(), fwd_deg);
    }
    return 0;
}

// Whole canonical build from a given initial graph (NULL: the random graph
// of degree min(16, R), seed 42), `rounds` rounds (the reference runs 3).
// C is the work width after the reference's min(C, 128) clamp.
int oracle_filtered_build(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                          uint32_t L, uint32_t FL, uint32_t C, uint32_t STEPS, float alpha, const uint32_t *offsets,
                          const uint32_t *labels, const uint32_t *starts, uint32_t num_labels, uint32_t universal,
                          uint32_t global_start, const uint32_t *graph_in, const uint32_t *degree_in,
                          uint32_t rounds, int threads, uint32_t *graph_out, uint32_t *degree_out)
{
    const FilteredCtx cx = make_ctx(dtype, data, stride, N, dim, R, offsets, labels, starts, num_labels, universal);
    std::vector<uint32_t> ga((size_t)N * R), da(N), gb, db;
    if (graph_in)
    {
        std::copy(graph_in, graph_in + (size_t)N * R, ga.begin());
        std::copy(degree_in, degree_in + N, da.begin());
    }
    else
        filtered_random_graph(N, R, 16u, 42u, ga.data(), da.data());
    FilteredCounters fc;
    const bool trace = std::getenv("ORACLE_FILTERED_TRACE") != nullptr;
    for (uint32_t round = 0; round < rounds; ++round)
    {
        const FilteredCounters before = fc;
        filtered_round(cx, C, L, FL, STEPS, alpha, global_start, ga, da, gb, db, threads, fc, nullptr);
        if (trace)
            fprintf(stderr, "[oracle_filtered] round=%u touched=%llu reverse_proposals=%llu\n", round,
                    (unsigned long long)(fc.touched - before.touched),
                    (unsigned long long)(fc.reverse_edges - before.reverse_edges));
        std::swap(ga, gb);
        std::swap(da, db);
    }
    std::copy(ga.begin(), ga.end(), graph_out);
    std::copy(da.begin(), da.end(), degree_out);
    return 0;
}

// Task search outputs of every (row, label position) on a given graph (T x keep).
int oracle_filtered_task_search(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                                uint32_t FL, uint32_t STEPS, const uint32_t *offsets, const uint32_t *labels,
                                const uint32_t *starts, uint32_t num_labels, uint32_t universal,
                                const uint32_t *graph, const uint32_t *degree, uint32_t *out_ids, float *out_d,
                                int threads)
{
    const FilteredCtx cx = make_ctx(dtype, data, stride, N, dim, R, offsets, labels, starts, num_labels, universal);
    const uint32_t plp = std::min(FL, 32u), plk = std::min(plp, 8u);
#pragma omp parallel for schedule(dynamic, 64) num_threads(threads)
    for (int64_t row = 0; row < (int64_t)N; ++row)
        for (uint32_t p = offsets[row]; p < offsets[row + 1]; ++p)
            task_search(cx, p, (uint32_t)row, graph, degree, plp, plk, STEPS, out_ids + (size_t)p * plk,
                        out_d + (size_t)p * plk);
    return 0;
}

// Union-label search outputs of every row (N x min(R, L)).
int oracle_filtered_ordinary_search(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim,
                                    uint32_t R, uint32_t L, uint32_t FL, uint32_t STEPS, const uint32_t *offsets,
                                    const uint32_t *labels, const uint32_t *starts, uint32_t num_labels,
                                    uint32_t universal, uint32_t global_start, const uint32_t *graph,
                                    const uint32_t *degree, uint32_t *out_ids, float *out_d, int threads)
{
    const FilteredCtx cx = make_ctx(dtype, data, stride, N, dim, R, offsets, labels, starts, num_labels, universal);
    const uint32_t keep = std::min(R, L), pool = std::min(64u, FL);
#pragma omp parallel for schedule(dynamic, 64) num_threads(threads)
    for (int64_t row = 0; row < (int64_t)N; ++row)
        ordinary_search(cx, (uint32_t)row, global_start, graph, degree, pool, keep, STEPS,
                        out_ids + (size_t)row * keep, out_d + (size_t)row * keep);
    return 0;
}

// Per-row FilteredRobustPrune of candidate lists given as CSR (tests).
int oracle_filtered_prune_lists(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                                float alpha, const uint32_t *offsets, const uint32_t *labels, uint32_t num_labels,
                                const uint32_t *rows, uint32_t nrows, const uint64_t *list_off,
                                const uint32_t *list_ids, const float *list_d, uint32_t *graph_out,
                                uint32_t *degree_out)
{
    const FilteredCtx cx = make_ctx(dtype, data, stride, N, dim, R, offsets, labels, nullptr, num_labels, kInvalid);
    for (uint32_t r = 0; r < nrows; ++r)
    {
        uint32_t *out = graph_out + (size_t)r * R;
        for (uint32_t i = 0; i < R; ++i)
            out[i] = kInvalid;
        degree_out[r] = filtered_prune(cx, rows[r], alpha, list_ids + list_off[r], list_d + list_off[r],
                                       (uint32_t)(list_off[r + 1] - list_off[r]), out);
    }
    return 0;
}

} // extern "C"

// ====================================================================== stitched global prune
// DiskANN's Index::prune_all_neighbors(range, maxc, alpha) as the DANCE
// integration patch changes it, which the reference stitched app runs on
// multi-label union graphs (apps/utils/gpu_stitched_vamana_index.cpp:353-372):
// rows longer than `range` are pruned; pool = distinct neighbours other than
// the row with d(row, x), sorted by (distance, id); for a labelled row whose
// pool exceeds `range`, the label-balanced shortlist of patch lines
// 20055-20100 (per row label its first max(1, range / #labels) carriers, then
// pool order up to `range`), which the following prune re-sorts; then
// occlude_list: truncate to maxc, occlusion factors from 0, passes
// a = 1, 1.2, ... <= alpha selecting entries with factor <= a, each selection
// s raising every later entry x with factor <= alpha to
// max(factor, d(row,x) / d(s,x)) (FLT_MAX when d(s,x) = 0) when s covers the
// labels row and x share (patch lines 20009-20047).  DiskANN itself is not
// available here, so this restatement is pinned only by hand cases.
namespace
{
bool has_label(const uint32_t *off, const uint32_t *lab, uint32_t p, uint32_t l)
{
    return std::binary_search(lab + off[p], lab + off[p + 1], l);
}

bool covers(const uint32_t *off, const uint32_t *lab, uint32_t t, uint32_t s, uint32_t x)
{
    uint32_t i = off[t], ie = off[t + 1], j = off[x], je = off[x + 1];
    while (i < ie && j < je)
    {
        if (lab[i] < lab[j])
            ++i;
        else if (lab[j] < lab[i])
            ++j;
        else
        {
            if (!has_label(off, lab, s, lab[i]))
                return false;
            ++i;
            ++j;
        }
    }
    return true;
}
} // namespace

extern "C" int oracle_stitched_global_prune(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim,
                                            const uint64_t *row_off, const uint32_t *row_ids, const uint32_t *lab_off,
                                            const uint32_t *labs, uint32_t range, uint32_t maxc, float alpha,
                                            uint32_t *out_rows, uint32_t *out_deg)
{
    const Store st = make_store(dtype, data, stride, dim);
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t vv = 0; vv < (int64_t)N; ++vv)
    {
        const uint32_t v = (uint32_t)vv;
        const uint32_t deg = (uint32_t)(row_off[v + 1] - row_off[v]);
        const uint32_t *row = row_ids + row_off[v];
        uint32_t *out = out_rows + (uint64_t)v * range;
        for (uint32_t i = 0; i < range; ++i)
            out[i] = kInvalid;
        if (deg <= range)
        {
            std::copy(row, row + deg, out);
            out_deg[v] = deg;
            continue;
        }
        std::vector<uint64_t> pool;
        for (uint32_t i = 0; i < deg; ++i)
            if (row[i] < N && row[i] != v)
                pool.push_back(make_key(dist(st, v, row[i]), row[i]));
        std::sort(pool.begin(), pool.end());
        pool.erase(std::unique(pool.begin(), pool.end()), pool.end());
        const uint32_t nlab = lab_off ? lab_off[v + 1] - lab_off[v] : 0;
        if (nlab > 0 && pool.size() > range)
        {
            const uint32_t quota = std::max<uint32_t>(1, range / nlab);
            std::vector<char> kept(pool.size(), 0);
            for (uint32_t li = 0; li < nlab; ++li)
            {
                const uint32_t l = labs[lab_off[v] + li];
                uint32_t admitted = 0;
                for (size_t i = 0; i < pool.size() && admitted < quota; ++i)
                    if (has_label(lab_off, labs, (uint32_t)pool[i], l))
                    {
                        kept[i] = 1;
                        ++admitted;
                    }
            }
            size_t nk = std::count(kept.begin(), kept.end(), 1);
            for (size_t i = 0; i < pool.size() && nk < range; ++i)
                if (!kept[i])
                {
                    kept[i] = 1;
                    ++nk;
                }
            std::vector<uint64_t> shortlist;
            for (size_t i = 0; i < pool.size(); ++i)
                if (kept[i])
                    shortlist.push_back(pool[i]); // already in (distance, id) order
            pool.swap(shortlist);
        }
        if (pool.size() > maxc)
            pool.resize(maxc);
        std::vector<float> occ(pool.size(), 0.0f);
        uint32_t nres = 0;
        float cur = 1.0f;
        while (cur <= alpha && nres < range)
        {
            for (size_t i = 0; i < pool.size() && nres < range; ++i)
            {
                if (occ[i] > cur)
                    continue;
                occ[i] = FLT_MAX;
                const uint32_t s = (uint32_t)pool[i];
                if (s != v)
                    out[nres++] = s;
                for (size_t j = i + 1; j < pool.size(); ++j)
                {
                    if (occ[j] > alpha)
                        continue;
                    const uint32_t x = (uint32_t)pool[j];
                    if (lab_off && !covers(lab_off, labs, v, s, x))
                        continue;
                    const float djk = dist(st, s, x);
                    float dj;
                    const uint32_t bits = (uint32_t)(pool[j] >> 32);
                    std::memcpy(&dj, &bits, 4);
                    occ[j] = djk == 0.0f ? FLT_MAX : std::max(occ[j], dj / djk);
                }
            }
            cur *= 1.2f;
        }
        out_deg[v] = nres;
    }
    return 0;
}

// ====================================================================== entry point, label starts
// The inputs DiskANN computes before the filtered build hook (integration
// patch lines 20238-20267), restated as dance_b200/csrc/label_starts.cu
// defines them: centroid summed point by point in float, nearest point by
// squared L2 summed over dimensions in order (lowest index on ties); per
// label in ascending order, the least-chosen of num_cands hashed draws.
namespace
{
float elem_of(const Store &st, uint32_t i, uint32_t j)
{
    const uint8_t *row = st.row(i);
    switch (st.dtype)
    {
    case DANCE_U8:
        return (float)row[j];
    case DANCE_F16:
        return half_to_float(reinterpret_cast<const uint16_t *>(row)[j]);
    default:
        return reinterpret_cast<const float *>(row)[j];
    }
}

uint32_t start_draw(uint64_t seed, uint32_t label, uint32_t k)
{
    uint32_t h = hash_u32((uint32_t)seed ^ hash_u32(label * 0x9e3779b1u + 0x7f4a7c15u));
    return hash_u32(h ^ (uint32_t)(seed >> 32) ^ (k * 0x85ebca6bu + 0x165667b1u));
}
} // namespace

extern "C" uint32_t oracle_entry_point(int dtype, const void *data, uint64_t stride, uint32_t N, uint32_t dim)
{
    const Store st = make_store(dtype, data, stride, dim);
    std::vector<float> c(dim, 0.0f);
    for (uint32_t i = 0; i < N; ++i)
        for (uint32_t j = 0; j < dim; ++j)
            c[j] += elem_of(st, i, j);
    for (uint32_t j = 0; j < dim; ++j)
        c[j] /= (float)N;
    uint64_t best = ~0ull;
    for (uint32_t i = 0; i < N; ++i)
    {
        float d = 0.0f;
        for (uint32_t j = 0; j < dim; ++j)
        {
            const float diff = c[j] - elem_of(st, i, j);
            d += diff * diff;
        }
        best = std::min(best, make_key(d, i));
    }
    return (uint32_t)best;
}

extern "C" void oracle_label_starts(const uint32_t *off, const uint32_t *pts, uint32_t num_labels, uint32_t N,
                                    uint32_t num_cands, uint64_t seed, uint32_t *starts)
{
    std::vector<uint32_t> counts(N, 0);
    for (uint32_t l = 0; l < num_labels; ++l)
    {
        const uint32_t n = off[l + 1] - off[l];
        if (n == 0)
        {
            starts[l] = kInvalid;
            continue;
        }
        uint32_t best = kInvalid, best_count = 0;
        for (uint32_t k = 0; k < num_cands; ++k)
        {
            const uint32_t p = pts[off[l] + start_draw(seed, l, k) % n];
            if (best == kInvalid || counts[p] < best_count)
            {
                best = p;
                best_count = counts[p];
            }
        }
        starts[l] = best;
        counts[best] += 1;
    }
}

// ====================================================================== k-means partition
// DiskANN's partitioner as the DANCE patch drives it before the GPU shard
// loop (partition_with_ram_budget -> shard_data_into_clusters_only_ids,
// integration patch lines 20629-20688), restated sequentially as
// dance_b200/csrc/partition.cu defines it: squared L2 summed over
// dimensions in order without fused multiply-add; k-means++ with weights
// quantised to floor(w / max w * 2^31) and splitmix64 draws; Lloyd means in
// float64, summed in row order within blocks of 4096 rows, block sums in
// block order; k_base nearest centers, lower center on ties; shard id lists
// in ascending point order.
namespace
{
uint64_t part_splitmix64(uint64_t x)
{
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

uint64_t part_pivot_draw(uint64_t seed, uint32_t pivot)
{
    return part_splitmix64(seed ^ part_splitmix64(0x5deece66dull + pivot));
}

float part_sq_dist(const float *x, const float *c, uint32_t dim)
{
    float d = 0.0f;
    for (uint32_t j = 0; j < dim; ++j)
    {
        const float diff = c[j] - x[j];
        d += diff * diff;
    }
    return d;
}

const float *train_row(const float *train, uint64_t stride_bytes, uint64_t i)
{
    return reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(train) + i * stride_bytes);
}

constexpr uint64_t kPartLloydChunk = 4096;
} // namespace

extern "C" void oracle_kmeanspp_seed(const float *train, uint64_t stride, uint64_t n, uint32_t dim, uint32_t k,
                                     uint64_t seed, float *centers, uint64_t *picked)
{
    uint64_t pick = part_splitmix64(seed) % n;
    picked[0] = pick;
    std::copy(train_row(train, stride, pick), train_row(train, stride, pick) + dim, centers);
    std::vector<float> mind(n);
    std::vector<uint32_t> q(n);
    for (uint32_t p = 1; p < k; ++p)
    {
        const float *c = centers + (uint64_t)(p - 1) * dim;
        float mx = 0.0f;
        for (uint64_t i = 0; i < n; ++i)
        {
            const float d = part_sq_dist(train_row(train, stride, i), c, dim);
            mind[i] = p == 1 ? d : std::min(mind[i], d);
            mx = std::max(mx, mind[i]);
        }
        uint64_t total = 0;
        for (uint64_t i = 0; i < n; ++i)
        {
            q[i] = mx > 0.0f ? (uint32_t)((mind[i] / mx) * 2147483648.0f) : 1u;
            total += q[i];
        }
        const uint64_t r = total ? part_pivot_draw(seed, p) % total : 0;
        uint64_t run = 0;
        pick = n - 1;
        for (uint64_t i = 0; i < n; ++i)
        {
            run += q[i];
            if (run > r)
            {
                pick = i;
                break;
            }
        }
        picked[p] = pick;
        std::copy(train_row(train, stride, pick), train_row(train, stride, pick) + dim,
                  centers + (uint64_t)p * dim);
    }
}

extern "C" void oracle_partition_assign(int dtype, const void *data, uint64_t stride, uint64_t n, uint32_t dim,
                                        const float *centers, uint32_t k, uint32_t kb, uint32_t *out_ids,
                                        float *out_dists)
{
    const Store st = make_store(dtype, data, stride, dim);
    std::vector<float> x(dim);
    std::vector<std::pair<float, uint32_t>> best;
    for (uint64_t i = 0; i < n; ++i)
    {
        for (uint32_t j = 0; j < dim; ++j)
            x[j] = elem_of(st, (uint32_t)i, j);
        best.clear();
        for (uint32_t c = 0; c < k; ++c)
            best.emplace_back(part_sq_dist(x.data(), centers + (uint64_t)c * dim, dim), c);
        std::stable_sort(best.begin(), best.end(),
                         [](const std::pair<float, uint32_t> &a, const std::pair<float, uint32_t> &b) {
                             return a.first < b.first;
                         });
        for (uint32_t t = 0; t < kb; ++t)
        {
            out_ids[i * kb + t] = best[t].second;
            if (out_dists)
                out_dists[i * kb + t] = best[t].first;
        }
    }
}

extern "C" void oracle_kmeans_lloyd(const float *train, uint64_t stride, uint64_t n, uint32_t dim, uint32_t k,
                                    uint32_t iters, float *centers, uint32_t *assign_out, double *residual)
{
    std::vector<uint32_t> asg(n);
    std::vector<float> dist(n);
    const uint64_t nchunks = (n + kPartLloydChunk - 1) / kPartLloydChunk;
    std::vector<double> tot((size_t)k * dim), part((size_t)k * dim);
    std::vector<uint64_t> cnt(k);
    double resid = 0.0;
    for (uint32_t it = 0; it < iters; ++it)
    {
        oracle_partition_assign(DANCE_F32, train, stride, n, dim, centers, k, 1, asg.data(), dist.data());
        std::fill(tot.begin(), tot.end(), 0.0);
        std::fill(cnt.begin(), cnt.end(), 0);
        resid = 0.0;
        for (uint64_t b = 0; b < nchunks; ++b)
        {
            std::fill(part.begin(), part.end(), 0.0);
            double rs = 0.0;
            const uint64_t e = std::min(n, (b + 1) * kPartLloydChunk);
            for (uint64_t i = b * kPartLloydChunk; i < e; ++i)
            {
                const float *x = train_row(train, stride, i);
                const uint32_t c = asg[i];
                for (uint32_t j = 0; j < dim; ++j)
                    part[(size_t)c * dim + j] += (double)x[j];
                cnt[c] += 1;
                rs += (double)dist[i];
            }
            for (size_t t = 0; t < part.size(); ++t)
                tot[t] += part[t];
            resid += rs;
        }
        for (uint32_t c = 0; c < k; ++c)
            if (cnt[c])
                for (uint32_t j = 0; j < dim; ++j)
                    centers[(size_t)c * dim + j] = (float)(tot[(size_t)c * dim + j] / (double)cnt[c]);
    }
    if (assign_out)
        oracle_partition_assign(DANCE_F32, train, stride, n, dim, centers, k, 1, assign_out, nullptr);
    if (residual)
        *residual = resid;
}

extern "C" void oracle_partition_buckets(const uint32_t *assign, uint64_t n, uint32_t kb, uint32_t S,
                                         uint32_t *offsets, uint32_t *ids)
{
    std::vector<uint32_t> cnt(S + 1, 0);
    for (uint64_t e = 0; e < n * kb; ++e)
        if (assign[e] < S)
            cnt[assign[e] + 1] += 1;
    for (uint32_t s = 0; s < S; ++s)
        cnt[s + 1] += cnt[s];
    std::copy(cnt.begin(), cnt.end(), offsets);
    for (uint64_t e = 0; e < n * kb; ++e)
        if (assign[e] < S)
            ids[cnt[assign[e]]++] = (uint32_t)(e / kb);
}
