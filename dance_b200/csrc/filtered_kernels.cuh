// filtered_kernels.cuh -- GPU-FilteredVamana kernels for sm_100a.
//
// One canonical round of the reference's filtered builder
// (src/gpu_vamana_filtered.cu, canonical_round0_from_host_backbone_typed
// :5889-6172), restated for B200:
//   fl_task_search_kernel     label-masked GreedySearch per (row, label)   (ref :4266-4426)
//   fl_union_search_kernel    union-label GreedySearch per row             (ref :4530-4670)
//   fl_merge_kernel           fixed-order merge, label quotas, distances   (ref :4672-4871)
//   fl_prune_kernel           FilteredRobustPrune of a candidate list      (ref :4877-4994, :5131-5230)
//   fl_rev_* kernels          exact CSR reverse repair                     (ref :4996-5128)
//
// Search pools.  The reference keeps an unsorted array of at most 32 (task)
// or 64 (union) slots: a new id is appended to the next free slot, or, when
// the array is full, replaces the slot holding the largest (distance, id)
// if it is smaller; the next expansion is the smallest unexpanded
// (distance, id); the output is the first `keep` slots in slot order.  Here
// the pool is kept sorted by the key (distance, id) in registers -- one
// entry per lane (task) or two (union) -- and every entry carries the slot
// number the reference would have given it (append -> next slot, replace
// -> the evicted entry's slot), so set, expansion order and slot-ordered
// output are the reference's.  The distance of a (row, candidate) pair never
// changes, so a candidate already in the pool is skipped without changing
// the result (the reference recomputes it and finds a duplicate).
//
// Distances are GroupDist (four candidates per warp, eight lanes each),
// bit-identical to the reference's warp_l2_distance for fp16 and uint8
// storage.
#pragma once

#include "vamana_kernels.cuh"

namespace dance
{
namespace fl
{

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kMaxR = 128;      // graph width handled by the search and prune kernels
constexpr uint32_t kMaxC = 128;      // work width (the reference clamps its work C to 128)
constexpr uint32_t kShortList = 256; // reverse-repair lists pruned by one warp; longer ones by a block

struct Labels
{
    const uint32_t *off;    // N + 1: labels of point p are lab[off[p] .. off[p+1]), ascending
    const uint32_t *lab;
    const uint32_t *lpo;    // num_labels + 1: points of label l are lp[lpo[l] .. lpo[l+1]), ascending
    const uint32_t *lp;
    const uint32_t *starts; // num_labels
    uint32_t num_labels;
    uint32_t universal;
    const uint32_t *bits; // optional: label l's members as a bitmap of bit_words words, or nullptr
    uint64_t bit_words;
};

// point_has_exact_label_device (ref :557-571); with the label bitmaps one
// load instead of the point's label list.
__device__ __forceinline__ bool has_label(const Labels &L, uint32_t p, uint32_t l)
{
    if (L.bits)
        return (L.bits[(uint64_t)l * L.bit_words + (p >> 5)] >> (p & 31u)) & 1u;
    const uint32_t e = L.off[p + 1];
    for (uint32_t i = L.off[p]; i < e; ++i)
    {
        const uint32_t v = L.lab[i];
        if (v >= l)
            return v == l;
    }
    return false;
}

// Any label of the sorted list a[0..na) carried by point p.
__device__ __forceinline__ bool has_any(const Labels &L, uint32_t p, const uint32_t *a, uint32_t na)
{
    uint32_t i = L.off[p], j = 0;
    const uint32_t e = L.off[p + 1];
    while (i < e && j < na)
    {
        const uint32_t x = L.lab[i], y = a[j];
        if (x == y)
            return true;
        if (x < y)
            ++i;
        else
            ++j;
    }
    return false;
}

// filtered_selected_covers_common_labels (include/filtered_label_coverage.cuh:8-45):
// every label the row shares with the candidate is also a label of the selection.
__device__ __forceinline__ bool covers(const Labels &L, const uint32_t *rl, uint32_t nr, const uint32_t *sl,
                                       uint32_t ns, uint32_t cand)
{
    uint32_t t = 0, c = L.off[cand], s = 0;
    const uint32_t ce = L.off[cand + 1];
    while (t < nr && c < ce)
    {
        const uint32_t a = rl[t], b = L.lab[c];
        if (a < b)
            ++t;
        else if (b < a)
            ++c;
        else
        {
            while (s < ns && sl[s] < a)
                ++s;
            if (s == ns || sl[s] != a)
                return false;
            ++t;
            ++c;
        }
    }
    return true;
}

__device__ __forceinline__ uint32_t fhash(uint32_t x) { return hash_u32(x); } // ref filtered_hash_u32 :694-702

// ------------------------------------------------------------------ pools
// Sorted pool of at most 32 entries, entry i in lane i.
struct Pool32
{
    uint64_t key;  // (distance bits, id); kKeyMax when empty
    uint32_t slot; // the reference's slot of this entry
    bool exp;
    uint32_t count, cap;

    __device__ __forceinline__ void init(uint32_t c)
    {
        key = kKeyMax;
        slot = 0;
        exp = false;
        count = 0;
        cap = c;
    }
    // Per-lane membership of the lane's own id c.
    __device__ __forceinline__ bool holds(uint32_t c) const
    {
        bool present = false;
        for (uint32_t pl = 0; pl < count; ++pl)
            present |= key_id(__shfl_sync(kFull, key, pl)) == c;
        return present;
    }
    // insert_top_l_state_warp (ref :4187-4233) for an id not in the pool.
    __device__ __forceinline__ void insert(uint64_t k, int lane)
    {
        const bool valid = (uint32_t)lane < count;
        uint32_t last, nslot;
        if (count < cap)
        {
            last = count;
            nslot = count;
        }
        else
        {
            if (!(k < __shfl_sync(kFull, key, cap - 1)))
                return;
            last = cap - 1;
            nslot = __shfl_sync(kFull, slot, cap - 1);
        }
        const uint32_t pos = __popc(__ballot_sync(kFull, valid && key < k));
        const uint64_t uk = __shfl_up_sync(kFull, key, 1);
        const uint32_t us = __shfl_up_sync(kFull, slot, 1);
        const bool ue = __shfl_up_sync(kFull, exp, 1);
        if ((uint32_t)lane > pos && (uint32_t)lane <= last)
        {
            key = uk;
            slot = us;
            exp = ue;
        }
        if ((uint32_t)lane == pos)
        {
            key = k;
            slot = nslot;
            exp = false;
        }
        if (count < cap)
            ++count;
    }
    // select_next_unexpanded_size_warp (ref :4235-4263); marks it expanded.
    __device__ __forceinline__ int select(int lane)
    {
        const unsigned m = __ballot_sync(kFull, (uint32_t)lane < count && !exp);
        if (!m)
            return -1;
        const int l = __ffs(m) - 1;
        if (lane == l)
            exp = true;
        return l;
    }
};

// Sorted pool of at most 64 entries: entry i in lane i (k0) and entry 32+i in lane i (k1).
struct Pool64
{
    uint64_t k0, k1;
    uint32_t s0, s1;
    bool e0, e1;
    uint32_t count, cap;

    __device__ __forceinline__ void init(uint32_t c)
    {
        k0 = k1 = kKeyMax;
        s0 = s1 = 0;
        e0 = e1 = false;
        count = 0;
        cap = c;
    }
    __device__ __forceinline__ uint64_t key_at(uint32_t p) const
    {
        const uint64_t a = __shfl_sync(kFull, k0, p & 31), b = __shfl_sync(kFull, k1, p & 31);
        return p < 32 ? a : b;
    }
    __device__ __forceinline__ uint32_t slot_at(uint32_t p) const
    {
        const uint32_t a = __shfl_sync(kFull, s0, p & 31), b = __shfl_sync(kFull, s1, p & 31);
        return p < 32 ? a : b;
    }
    // Per-lane membership of the lane's own id c.
    __device__ __forceinline__ bool holds(uint32_t c) const
    {
        bool present = false;
        for (uint32_t pl = 0; pl < count; ++pl)
            present |= key_id(key_at(pl)) == c;
        return present;
    }
    __device__ __forceinline__ void insert(uint64_t k, int lane)
    {
        const uint32_t p0 = (uint32_t)lane, p1 = (uint32_t)lane + 32;
        uint32_t last, nslot;
        if (count < cap)
        {
            last = count;
            nslot = count;
        }
        else
        {
            if (!(k < key_at(cap - 1)))
                return;
            last = cap - 1;
            nslot = slot_at(cap - 1);
        }
        const uint32_t pos = __popc(__ballot_sync(kFull, p0 < count && k0 < k)) +
                             __popc(__ballot_sync(kFull, p1 < count && k1 < k));
        const uint64_t u0 = __shfl_up_sync(kFull, k0, 1), u1 = __shfl_up_sync(kFull, k1, 1);
        const uint64_t t0 = __shfl_sync(kFull, k0, 31);
        const uint32_t v0 = __shfl_up_sync(kFull, s0, 1), v1 = __shfl_up_sync(kFull, s1, 1);
        const uint32_t ts = __shfl_sync(kFull, s0, 31);
        const bool w0 = __shfl_up_sync(kFull, e0, 1), w1 = __shfl_up_sync(kFull, e1, 1);
        const bool te = __shfl_sync(kFull, e0, 31);
        if (p1 > pos && p1 <= last)
        {
            k1 = lane == 0 ? t0 : u1;
            s1 = lane == 0 ? ts : v1;
            e1 = lane == 0 ? te : w1;
        }
        if (p0 > pos && p0 <= last)
        {
            k0 = u0;
            s0 = v0;
            e0 = w0;
        }
        if (p0 == pos)
        {
            k0 = k;
            s0 = nslot;
            e0 = false;
        }
        if (p1 == pos)
        {
            k1 = k;
            s1 = nslot;
            e1 = false;
        }
        if (count < cap)
            ++count;
    }
    __device__ __forceinline__ int select(int lane)
    {
        const unsigned m0 = __ballot_sync(kFull, (uint32_t)lane < count && !e0);
        if (m0)
        {
            const int l = __ffs(m0) - 1;
            if (lane == l)
                e0 = true;
            return l;
        }
        const unsigned m1 = __ballot_sync(kFull, (uint32_t)lane + 32 < count && !e1);
        if (!m1)
            return -1;
        const int l = __ffs(m1) - 1;
        if (lane == l)
            e1 = true;
        return 32 + l;
    }
};

// ------------------------------------------------------------------ candidate batches
struct SearchScratch
{
    uint32_t ids[kMaxR];
    float d[kMaxR];
};

// Distances for the ids listed in sc.ids[0..m), then sequential inserts in
// list order.  List entries are distinct and not in the pool.
template <int DT, int CPL, class Pool>
__device__ __forceinline__ uint32_t eval_and_insert(const StoreView &st, const uint4 (&q)[CPL], SearchScratch &sc,
                                                    uint32_t m, Pool &pool, int lane)
{
    if (m == 0)
        return 0;
    eval_candidates<DT, CPL>(st.data, st.stride, st.nchunks, q, sc.ids, sc.d, (int)m, lane);
    __syncwarp();
    for (uint32_t i = 0; i < m; ++i)
        pool.insert(make_key(sc.d[i], sc.ids[i]), lane);
    __syncwarp();
    return m;
}

// Appends the lanes' candidates flagged by `keep` (lane order) to sc.ids[m..).
__device__ __forceinline__ uint32_t push_flagged(SearchScratch &sc, uint32_t m, bool keep, uint32_t c, int lane)
{
    const unsigned b = __ballot_sync(kFull, keep);
    if (keep)
        sc.ids[m + __popc(b & ((1u << lane) - 1u))] = c;
    return m + __popc(b);
}

// Like push_flagged, but an id already in sc.ids[0..m) or flagged by an
// earlier lane is not appended again: a graph row handed in by a caller may
// repeat an id, and the reference's insert ignores the repeat.
__device__ __forceinline__ uint32_t push_unique(SearchScratch &sc, uint32_t m, bool keep, uint32_t c, int lane)
{
    bool dup = false;
    for (int o = 0; o < 32; ++o)
    {
        const uint32_t other = __shfl_sync(kFull, c, o);
        const bool other_keep = __shfl_sync(kFull, keep, o);
        dup |= o < lane && other_keep && other == c;
    }
    if (keep)
        for (uint32_t j = 0; j < m && !dup; ++j)
            dup = sc.ids[j] == c;
    return push_flagged(sc, m, keep && !dup, c, lane);
}

// True when an earlier lane (among the first `upto`) holds the same value.
__device__ __forceinline__ bool dup_of_earlier_lane(uint32_t c, int lane, int upto)
{
    bool dup = false;
    for (int o = 0; o < upto; ++o)
    {
        const uint32_t other = __shfl_sync(kFull, c, o);
        dup |= o < lane && other == c;
    }
    return dup;
}

// ------------------------------------------------------------------ task search
struct TaskParams
{
    StoreView st;
    Labels L;
    uint32_t R, pool_cap, keep, steps;
    const uint32_t *graph, *degree;
    const uint32_t *task_rows; // T
    uint32_t T;
    uint32_t *out_ids; // T x keep
    float *out_d;
    unsigned long long *counters; // [0] distance evaluations, [1] expansions
};

// canonical_filtered_task_search (ref :4266-4426), label_seed_count 16.
template <int DT, int CPL>
__global__ void __launch_bounds__(kThreads) fl_task_search_kernel(TaskParams p)
{
    __shared__ SearchScratch scratch[kWarps];
    SearchScratch &sc = scratch[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31, gl = lane & 7;
    const uint32_t N = p.st.N;
    unsigned long long evals = 0, expansions = 0;
    for (uint32_t t = blockIdx.x * kWarps + (threadIdx.x >> 5); t < p.T; t += gridDim.x * kWarps)
    {
        const uint32_t row = p.task_rows[t];
        const uint32_t label = p.L.lab[t];
        uint32_t *oi = p.out_ids + (uint64_t)t * p.keep;
        float *od = p.out_d + (uint64_t)t * p.keep;
        if (row >= N || label >= p.L.num_labels || label == p.L.universal)
        {
            for (uint32_t i = lane; i < p.keep; i += 32)
            {
                oi[i] = kInvalid;
                od[i] = FLT_MAX;
            }
            continue;
        }
        uint4 q[CPL];
        load_frag<CPL>(q, p.st.data + (uint64_t)row * p.st.stride, p.st.nchunks, gl);
        Pool32 pool;
        pool.init(p.pool_cap);
        // label start, then up to 16 hashed members of the label's posting list
        const uint32_t start = p.L.starts[label];
        const bool start_ok = start < N && start != row;
        const uint32_t pb = p.L.lpo[label], pc = p.L.lpo[label + 1] - pb;
        const uint32_t nseed = min(16u, pc);
        uint32_t m = push_flagged(sc, 0, lane == 0 && start_ok, start, lane);
        {
            uint32_t s = kInvalid;
            if ((uint32_t)lane < nseed)
                s = p.L.lp[pb + fhash(row + (uint32_t)lane * 7919u + label * 17u) % pc];
            // every lane takes part in the shuffles: no short-circuit around them
            const bool earlier = dup_of_earlier_lane(s, lane, 16);
            const bool dup = (start_ok && s == start) || earlier;
            m = push_flagged(sc, m, (uint32_t)lane < nseed && s < N && s != row && !dup, s, lane);
        }
        __syncwarp();
        evals += eval_and_insert<DT, CPL>(p.st, q, sc, m, pool, lane);
        // the row's own neighbours carrying the label, then one scan per expansion
        uint32_t x = row;
        for (uint32_t step = 0;; ++step)
        {
            const uint32_t dx = min(p.degree[x], p.R);
            m = 0;
            for (uint32_t b = 0; b < dx; b += 32)
            {
                const uint32_t j = b + lane;
                const uint32_t c = j < dx ? p.graph[(uint64_t)x * p.R + j] : kInvalid;
                const bool ok = c < N && c != row && has_label(p.L, c, label);
                const bool present = pool.holds(c);
                m = push_unique(sc, m, ok && !present, c, lane);
            }
            __syncwarp();
            evals += eval_and_insert<DT, CPL>(p.st, q, sc, m, pool, lane);
            if (step >= p.steps)
                break;
            const int e = pool.select(lane);
            if (e < 0)
                break;
            ++expansions;
            x = key_id(__shfl_sync(kFull, pool.key, e));
        }
        if ((uint32_t)lane < pool.count && pool.slot < p.keep)
        {
            oi[pool.slot] = key_id(pool.key);
            od[pool.slot] = key_dist(pool.key);
        }
        for (uint32_t i = pool.count + lane; i < p.keep; i += 32)
        {
            oi[i] = kInvalid;
            od[i] = FLT_MAX;
        }
    }
    if (lane == 0 && p.counters)
    {
        atomicAdd(p.counters + 0, evals);
        atomicAdd(p.counters + 1, expansions);
    }
}

// ------------------------------------------------------------------ union search
struct UnionParams
{
    StoreView st;
    Labels L;
    uint32_t R, pool_cap, keep, steps, global_start;
    const uint32_t *graph, *degree;
    uint32_t *out_ids; // N x keep
    float *out_d;
    unsigned long long *counters;
};

constexpr uint32_t kRowLabelCache = 64;

// canonical_ordinary_search (ref :4530-4670), label_seed_count 64,
// traversal restricted to points sharing a label with the row.
template <int DT, int CPL>
__global__ void __launch_bounds__(kThreads) fl_union_search_kernel(UnionParams p)
{
    __shared__ SearchScratch scratch[kWarps];
    __shared__ uint32_t row_labels[kWarps][kRowLabelCache];
    SearchScratch &sc = scratch[threadIdx.x >> 5];
    uint32_t *rl_cache = row_labels[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31, gl = lane & 7;
    const uint32_t N = p.st.N;
    unsigned long long evals = 0, expansions = 0;
    for (uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < N; row += gridDim.x * kWarps)
    {
        const uint32_t lb = p.L.off[row], nl = p.L.off[row + 1] - lb;
        const uint32_t *rl = p.L.lab + lb;
        __syncwarp();
        if (nl <= kRowLabelCache)
        {
            for (uint32_t i = lane; i < nl; i += 32)
                rl_cache[i] = rl[i];
            __syncwarp();
            rl = rl_cache;
        }
        uint4 q[CPL];
        load_frag<CPL>(q, p.st.data + (uint64_t)row * p.st.stride, p.st.nchunks, gl);
        Pool64 pool;
        pool.init(p.pool_cap);
        // per row label: its start, then up to 64 hashed posting-list members
        for (uint32_t li = 0; li < nl; ++li)
        {
            const uint32_t label = rl[li];
            if (label >= p.L.num_labels)
                continue;
            const uint32_t start = p.L.starts[label];
            {
                const bool present = pool.holds(start);
            const bool ok = start < N && start != row && !present;
                uint32_t m = push_flagged(sc, 0, lane == 0 && ok, start, lane);
                __syncwarp();
                evals += eval_and_insert<DT, CPL>(p.st, q, sc, m, pool, lane);
            }
            const uint32_t pb = p.L.lpo[label], pc = p.L.lpo[label + 1] - pb;
            const uint32_t nseed = min(64u, pc);
            for (uint32_t b = 0; b < nseed; b += 32)
            {
                const uint32_t sidx = b + lane;
                uint32_t s = kInvalid;
                if (sidx < nseed)
                    s = p.L.lp[pb + fhash(row + sidx * 7919u + label * 17u) % pc];
                // every lane takes part in the shuffles: no short-circuit around them
                const bool earlier = dup_of_earlier_lane(s, lane, 32);
                const bool present = pool.holds(s);
                const bool ok = sidx < nseed && s < N && s != row && !earlier && !present;
                uint32_t m = push_flagged(sc, 0, ok, s, lane);
                __syncwarp();
                evals += eval_and_insert<DT, CPL>(p.st, q, sc, m, pool, lane);
            }
        }
        {
            const uint32_t g = p.global_start;
            const bool present = pool.holds(g);
            const bool ok = g < N && g != row && has_any(p.L, g, rl, nl) && !present;
            uint32_t m = push_flagged(sc, 0, lane == 0 && ok, g, lane);
            __syncwarp();
            evals += eval_and_insert<DT, CPL>(p.st, q, sc, m, pool, lane);
        }
        uint32_t x = row;
        for (uint32_t step = 0;; ++step)
        {
            const uint32_t dx = min(p.degree[x], p.R);
            uint32_t m = 0;
            for (uint32_t b = 0; b < dx; b += 32)
            {
                const uint32_t j = b + lane;
                const uint32_t c = j < dx ? p.graph[(uint64_t)x * p.R + j] : kInvalid;
                const bool present = pool.holds(c);
                const bool ok = c < N && c != row && !present && has_any(p.L, c, rl, nl);
                m = push_unique(sc, m, ok, c, lane);
            }
            __syncwarp();
            evals += eval_and_insert<DT, CPL>(p.st, q, sc, m, pool, lane);
            if (step >= p.steps)
                break;
            const int e = pool.select(lane);
            if (e < 0)
                break;
            ++expansions;
            x = key_id(pool.key_at((uint32_t)e));
        }
        uint32_t *oi = p.out_ids + (uint64_t)row * p.keep;
        float *od = p.out_d + (uint64_t)row * p.keep;
        if ((uint32_t)lane < pool.count && pool.s0 < p.keep)
        {
            oi[pool.s0] = key_id(pool.k0);
            od[pool.s0] = key_dist(pool.k0);
        }
        if ((uint32_t)lane + 32 < pool.count && pool.s1 < p.keep)
        {
            oi[pool.s1] = key_id(pool.k1);
            od[pool.s1] = key_dist(pool.k1);
        }
        for (uint32_t i = pool.count + lane; i < p.keep; i += 32)
        {
            oi[i] = kInvalid;
            od[i] = FLT_MAX;
        }
        __syncwarp();
    }
    if (lane == 0 && p.counters)
    {
        atomicAdd(p.counters + 0, evals);
        atomicAdd(p.counters + 1, expansions);
    }
}

// ------------------------------------------------------------------ merge
struct MergeParams
{
    StoreView st;
    Labels L;
    uint32_t R, C, task_keep, union_keep;
    const uint32_t *graph, *degree;
    const uint32_t *task_ids; // T x task_keep (row's label positions)
    const float *task_d;
    const uint32_t *union_ids; // N x union_keep
    const float *union_d;
    uint32_t *work_ids; // N x C
    float *work_d;
    uint32_t *work_deg;
    unsigned long long *counters; // [0] work distance evaluations
};

struct MergeScratch
{
    uint32_t ids[kMaxC];
    float d[kMaxC];
    uint16_t mask[kMaxC];
    uint32_t need[kMaxC];
    float nd[kMaxC];
};

// Appends one batch of up to 32 candidates (lane order) with the
// reference's canonical_merge_one_warp rule (ref :4672-4701): invalid ids,
// the row itself and anything after the row is full are ignored; a repeated
// id keeps its first position and the smaller distance.
__device__ __forceinline__ void merge_batch(MergeScratch &w, uint32_t &count, uint32_t C, uint32_t row, uint32_t N,
                                            uint32_t c, float d, bool active, int lane)
{
    const bool valid = active && c < N && c != row;
    int first = -1; // position of an equal id already in the row
    if (valid)
        for (uint32_t k = 0; k < count && first < 0; ++k)
            if (w.ids[k] == c)
                first = (int)k;
    int prev_lane = -1; // earliest lane of this batch with the same id
    for (int o = 0; o < 32; ++o)
    {
        const uint32_t other = __shfl_sync(kFull, c, o);
        const bool ov = __shfl_sync(kFull, valid, o);
        if (o < lane && ov && other == c && prev_lane < 0)
            prev_lane = o;
    }
    const bool is_new = valid && first < 0 && prev_lane < 0;
    const unsigned nb = __ballot_sync(kFull, is_new);
    const uint32_t before = __popc(nb & ((1u << lane) - 1u));
    const bool processed = valid && count + before < C;
    const uint32_t my_pos = count + before;
    const uint32_t prev_pos = __shfl_sync(kFull, my_pos, prev_lane < 0 ? 0 : prev_lane);
    if (processed && is_new)
    {
        w.ids[my_pos] = c;
        w.d[my_pos] = d;
    }
    __syncwarp();
    // a repeated id keeps the smaller distance; searches report the same
    // distance for a pair and an own neighbour reports none, so any real
    // distance is the one
    if (processed && !is_new && d != FLT_MAX)
        w.d[first >= 0 ? (uint32_t)first : prev_pos] = d;
    __syncwarp();
    count = min(C, count + (uint32_t)__popc(nb));
}

// canonical_merge_candidates + canonical_compute_work_distances (ref :4703-4871).
template <int DT, int CPL>
__global__ void __launch_bounds__(kThreads) fl_merge_kernel(MergeParams p)
{
    __shared__ MergeScratch scratch[kWarps];
    MergeScratch &w = scratch[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31, gl = lane & 7;
    const uint32_t N = p.st.N;
    unsigned long long evals = 0;
    for (uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < N; row += gridDim.x * kWarps)
    {
        const uint32_t lb = p.L.off[row], nl = p.L.off[row + 1] - lb;
        uint32_t count = 0;
        // per-label task outputs, in label position order
        for (uint32_t li = 0; li < nl; ++li)
            for (uint32_t b = 0; b < p.task_keep; b += 32)
            {
                const uint32_t i = b + lane;
                const bool act = i < p.task_keep;
                const uint64_t o = (uint64_t)(lb + li) * p.task_keep + i;
                merge_batch(w, count, p.C, row, N, act ? p.task_ids[o] : kInvalid, act ? p.task_d[o] : FLT_MAX,
                            act, lane);
            }
        // own neighbours sharing a label with the row
        const uint32_t dr = min(p.degree[row], p.R);
        for (uint32_t b = 0; b < dr; b += 32)
        {
            const uint32_t j = b + lane;
            const uint32_t c = j < dr ? p.graph[(uint64_t)row * p.R + j] : kInvalid;
            const bool act = j < dr && c < N && c != row && has_any(p.L, c, p.L.lab + lb, nl);
            merge_batch(w, count, p.C, row, N, c, FLT_MAX, act, lane);
        }
        // union search outputs
        for (uint32_t b = 0; b < p.union_keep; b += 32)
        {
            const uint32_t i = b + lane;
            const bool act = i < p.union_keep;
            const uint64_t o = (uint64_t)row * p.union_keep + i;
            merge_batch(w, count, p.C, row, N, act ? p.union_ids[o] : kInvalid, act ? p.union_d[o] : FLT_MAX, act,
                        lane);
        }
        // label quotas (rows with 1..16 labels): each entry, in order, is
        // charged to its rarest row label (then lowest id) with room left;
        // entries with no such label are dropped
        if (nl > 0 && nl <= 16)
        {
            for (uint32_t k = lane; k < count; k += 32)
            {
                uint16_t m = 0;
                for (uint32_t q2 = 0; q2 < nl; ++q2)
                    if (has_label(p.L, w.ids[k], p.L.lab[lb + q2]))
                        m |= (uint16_t)(1u << q2);
                w.mask[k] = m;
            }
            __syncwarp();
            if (lane == 0)
            {
                uint32_t order[16], assigned[16];
                for (uint32_t q2 = 0; q2 < nl; ++q2)
                {
                    order[q2] = q2;
                    assigned[q2] = 0;
                }
                // preference: smaller label cardinality, then smaller label id
                for (uint32_t a = 1; a < nl; ++a)
                {
                    const uint32_t v = order[a];
                    const uint32_t lv = p.L.lab[lb + v], cv = p.L.lpo[lv + 1] - p.L.lpo[lv];
                    uint32_t b2 = a;
                    while (b2 > 0)
                    {
                        const uint32_t u = order[b2 - 1];
                        const uint32_t lu = p.L.lab[lb + u], cu = p.L.lpo[lu + 1] - p.L.lpo[lu];
                        if (cu < cv || (cu == cv && lu < lv))
                            break;
                        order[b2] = u;
                        --b2;
                    }
                    order[b2] = v;
                }
                uint32_t quota = (p.R + nl - 1) / nl;
                if (quota < p.task_keep)
                    quota = p.task_keep;
                uint32_t kept = 0;
                for (uint32_t k = 0; k < count; ++k)
                {
                    const uint32_t m = w.mask[k];
                    int pick = -1;
                    for (uint32_t a = 0; a < nl && pick < 0; ++a)
                        if (((m >> order[a]) & 1u) && assigned[order[a]] < quota)
                            pick = (int)order[a];
                    if (pick < 0)
                        continue;
                    ++assigned[pick];
                    w.ids[kept] = w.ids[k];
                    w.d[kept] = w.d[k];
                    ++kept;
                }
                w.need[0] = kept; // hand the count to the warp
            }
            __syncwarp();
            count = w.need[0];
            __syncwarp();
        }
        // distances of entries that arrived without one
        uint4 q[CPL];
        load_frag<CPL>(q, p.st.data + (uint64_t)row * p.st.stride, p.st.nchunks, gl);
        uint32_t m = 0;
        for (uint32_t b = 0; b < count; b += 32)
        {
            const uint32_t k = b + lane;
            const bool needs = k < count && w.d[k] == FLT_MAX;
            const unsigned nb = __ballot_sync(kFull, needs);
            if (needs)
                w.need[m + __popc(nb & ((1u << lane) - 1u))] = k;
            m += __popc(nb);
        }
        __syncwarp();
        if (m)
        {
            // the ids to evaluate go into nd; their distances come back in place
            for (uint32_t i = lane; i < m; i += 32)
                w.nd[i] = __uint_as_float(w.ids[w.need[i]]);
            __syncwarp();
            eval_candidates<DT, CPL>(p.st.data, p.st.stride, p.st.nchunks, q,
                                     reinterpret_cast<const uint32_t *>(w.nd), w.nd, (int)m, lane);
            __syncwarp();
            for (uint32_t i = lane; i < m; i += 32)
                w.d[w.need[i]] = w.nd[i];
            evals += m;
        }
        __syncwarp();
        uint32_t *wi = p.work_ids + (uint64_t)row * p.C;
        float *wd = p.work_d + (uint64_t)row * p.C;
        for (uint32_t k = lane; k < p.C; k += 32)
        {
            wi[k] = k < count ? w.ids[k] : kInvalid;
            wd[k] = k < count ? w.d[k] : FLT_MAX;
        }
        if (lane == 0)
            p.work_deg[row] = count;
        __syncwarp();
    }
    if (lane == 0 && p.counters)
        atomicAdd(p.counters, evals);
}

// ------------------------------------------------------------------ prune
struct PruneParams
{
    StoreView st;
    Labels L;
    uint32_t R;
    float alpha;
    // candidate lists: CSR (list_off, N + 1 entries) or fixed-width rows
    // (width, per-row length list_n)
    const uint32_t *list_ids;
    const float *list_d;
    const uint32_t *list_off;
    uint32_t width;
    const uint32_t *list_n;
    const uint32_t *rows; // rows to prune (nullptr: all N)
    uint32_t nrows;
    uint32_t max_len; // the warp kernel prunes lists up to this length, the block kernel longer ones
    uint32_t *graph;  // N x R output rows (INVALID padded)
    uint32_t *degree;
    uint8_t *removed;             // block kernel: one flag per list entry
    unsigned long long *counters; // [0] pair distance evaluations
};

struct PruneScratch
{
    uint32_t ids[kShortList];
    float d[kShortList];
    uint32_t cover[kShortList];
    float pd[kShortList];
    uint32_t sel_labels[64];
    uint32_t killw[kShortList / 32]; // entries a selection occludes, bit lane of word i = entry 32 i + lane
    uint32_t cmask[kShortList];      // per entry: bit t = it carries the row's label t (rows of <= 32 labels)
};

// Bit t set when the candidate carries the row's label rl[t] (nr <= 32).
__device__ __forceinline__ uint32_t row_label_mask(const Labels &L, const uint32_t *rl, uint32_t nr, uint32_t cand)
{
    uint32_t t = 0, c = L.off[cand], m = 0;
    const uint32_t ce = L.off[cand + 1];
    while (t < nr && c < ce)
    {
        const uint32_t a = rl[t], b = L.lab[c];
        if (a < b)
            ++t;
        else if (b < a)
            ++c;
        else
        {
            m |= 1u << t;
            ++t;
            ++c;
        }
    }
    return m;
}

__device__ __forceinline__ void row_list(const PruneParams &p, uint32_t row, uint32_t &begin, uint32_t &n)
{
    if (p.list_off)
    {
        begin = p.list_off[row];
        n = p.list_off[row + 1] - begin;
    }
    else
    {
        begin = row * p.width;
        n = min(p.list_n[row], p.width);
    }
}

// canonical_exact_prune / canonical_exact_prune_csr (ref :4877-4994,
// :5131-5230): repeatedly select the least (distance, id) not removed; a
// remaining q is removed iff the selection covers every label q shares with
// the row and 0 < alpha * d(sel, q) <= d(row, q).  One warp per row, list in
// shared memory, liveness as one bit per entry in the owning lane.
template <int DT, int CPL>
__global__ void __launch_bounds__(kThreads) fl_prune_kernel(PruneParams p)
{
    __shared__ PruneScratch scratch[kWarps];
    PruneScratch &w = scratch[threadIdx.x >> 5];
    const int lane = threadIdx.x & 31, gl = lane & 7;
    unsigned long long evals = 0;
    const uint32_t count = p.rows ? p.nrows : p.st.N;
    if ((uint32_t)lane < kShortList / 32)
        w.killw[lane] = 0u;
    __syncwarp();
    for (uint32_t r = blockIdx.x * kWarps + (threadIdx.x >> 5); r < count; r += gridDim.x * kWarps)
    {
        const uint32_t row = p.rows ? p.rows[r] : r;
        uint32_t begin, n;
        row_list(p, row, begin, n);
        if (n > p.max_len)
            continue;
        const uint32_t lb = p.L.off[row], nl = p.L.off[row + 1] - lb;
        const uint32_t *rl = p.L.lab + lb;
        // rows of up to 32 labels: coverage by a selection becomes a mask test,
        // (labels shared by row and entry) subset of (row labels the selection carries)
        const bool masks = nl <= 32;
        for (uint32_t k = lane; k < n; k += 32)
        {
            const uint32_t id = p.list_ids[begin + k];
            w.ids[k] = id;
            w.d[k] = p.list_d[begin + k];
            if (masks)
                w.cmask[k] = id < p.st.N ? row_label_mask(p.L, rl, nl, id) : 0u;
        }
        __syncwarp();
        uint32_t *out = p.graph + (uint64_t)row * p.R;
        uint32_t sel = 0;
        uint32_t live = 0; // bit i: entry k = 32 i + lane is live
        for (uint32_t i = 0; i * 32 + lane < n; ++i)
            live |= 1u << i;
        while (sel < p.R)
        {
            uint64_t best = kKeyMax;
            uint32_t bk = kInvalid;
            for (uint32_t i = 0; i * 32 + lane < n; ++i)
                if ((live >> i) & 1u)
                {
                    const uint32_t k = i * 32 + lane;
                    const uint64_t key = make_key(w.d[k], w.ids[k]);
                    if (key < best)
                    {
                        best = key;
                        bk = k;
                    }
                }
            for (int o = 16; o > 0; o >>= 1)
            {
                const uint64_t ob = __shfl_xor_sync(kFull, best, o);
                const uint32_t ok = __shfl_xor_sync(kFull, bk, o);
                if (ob < best)
                {
                    best = ob;
                    bk = ok;
                }
            }
            if (best == kKeyMax)
                break;
            const uint32_t bid = key_id(best);
            if (lane == 0)
                out[sel] = bid;
            ++sel;
            if ((bk & 31u) == (uint32_t)lane)
                live &= ~(1u << (bk >> 5));
            // labels of the selection
            const uint32_t sb = p.L.off[bid], ns = p.L.off[bid + 1] - sb;
            const uint32_t *sl = p.L.lab + sb;
            if (ns <= 64)
            {
                for (uint32_t i = lane; i < ns; i += 32)
                    w.sel_labels[i] = sl[i];
                __syncwarp();
                sl = w.sel_labels;
            }
            // live entries whose shared labels the selection covers
            uint32_t smask = 0;
            if (masks)
            {
                bool has = false;
                if ((uint32_t)lane < nl)
                {
                    const uint32_t a = rl[lane];
                    for (uint32_t s2 = 0; s2 < ns && !has; ++s2)
                        has = sl[s2] == a;
                }
                smask = __ballot_sync(kFull, has);
            }
            uint32_t m = 0;
            for (uint32_t i = 0; i * 32 < n; ++i)
            {
                const uint32_t k = i * 32 + lane;
                const bool cand = k < n && ((live >> i) & 1u) &&
                                  (masks ? (w.cmask[k] & ~smask) == 0u : covers(p.L, rl, nl, sl, ns, w.ids[k]));
                const unsigned cb = __ballot_sync(kFull, cand);
                if (cand)
                    w.cover[m + __popc(cb & ((1u << lane) - 1u))] = k;
                m += __popc(cb);
            }
            __syncwarp();
            if (m)
            {
                uint4 q[CPL];
                load_frag<CPL>(q, p.st.data + (uint64_t)bid * p.st.stride, p.st.nchunks, gl);
                // the covered ids go into pd; d(selection, id) comes back in place
                for (uint32_t i = lane; i < m; i += 32)
                    w.pd[i] = __uint_as_float(w.ids[w.cover[i]]);
                __syncwarp();
                eval_candidates<DT, CPL>(p.st.data, p.st.stride, p.st.nchunks, q,
                                         reinterpret_cast<const uint32_t *>(w.pd), w.pd, (int)m, lane);
                __syncwarp();
                evals += m;
                // occluded entries leave the live set (order-free: only removals)
                for (uint32_t i = lane; i < m; i += 32)
                {
                    const uint32_t k = w.cover[i];
                    const float pd = w.pd[i];
                    if (pd > 0.0f && __fmul_rn(p.alpha, pd) <= w.d[k])
                        atomicOr(&w.killw[k >> 5], 1u << (k & 31u));
                }
                __syncwarp();
                for (uint32_t i = 0; i * 32 < n; ++i)
                    if ((w.killw[i] >> lane) & 1u)
                        live &= ~(1u << i);
                __syncwarp();
                if ((uint32_t)lane < kShortList / 32)
                    w.killw[lane] = 0u;
            }
            __syncwarp();
        }
        for (uint32_t i = sel + lane; i < p.R; i += 32)
            out[i] = kInvalid;
        if (lane == 0)
            p.degree[row] = sel;
        __syncwarp();
    }
    if (lane == 0 && p.counters)
        atomicAdd(p.counters, evals);
}

// Block-per-row variant for lists longer than max_len (hub rows of the
// reverse repair): entries stay in global memory with a removed flag each.
template <int DT, int CPL>
__global__ void __launch_bounds__(256) fl_prune_long_kernel(PruneParams p)
{
    __shared__ uint64_t s_best[8];
    __shared__ uint32_t s_bk[8];
    __shared__ uint32_t s_cover[8][64];
    __shared__ float s_pd[8][64];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, gl = lane & 7;
    unsigned long long evals = 0;
    for (uint32_t r = blockIdx.x; r < p.nrows; r += gridDim.x)
    {
        const uint32_t row = p.rows[r];
        uint32_t begin, n;
        row_list(p, row, begin, n);
        if (n <= p.max_len)
            continue;
        const uint32_t lb = p.L.off[row], nl = p.L.off[row + 1] - lb;
        const uint32_t *rl = p.L.lab + lb;
        const uint32_t *ids = p.list_ids + begin;
        const float *dd = p.list_d + begin;
        uint8_t *rem = p.removed + begin;
        for (uint32_t k = threadIdx.x; k < n; k += blockDim.x)
            rem[k] = 0;
        __syncthreads();
        uint32_t *out = p.graph + (uint64_t)row * p.R;
        uint32_t sel = 0;
        while (sel < p.R)
        {
            uint64_t best = kKeyMax;
            uint32_t bk = kInvalid;
            for (uint32_t k = threadIdx.x; k < n; k += blockDim.x)
                if (!rem[k])
                {
                    const uint64_t key = make_key(dd[k], ids[k]);
                    if (key < best)
                    {
                        best = key;
                        bk = k;
                    }
                }
            for (int o = 16; o > 0; o >>= 1)
            {
                const uint64_t ob = __shfl_xor_sync(kFull, best, o);
                const uint32_t ok = __shfl_xor_sync(kFull, bk, o);
                if (ob < best)
                {
                    best = ob;
                    bk = ok;
                }
            }
            if (lane == 0)
            {
                s_best[wid] = best;
                s_bk[wid] = bk;
            }
            __syncthreads();
            best = s_best[0];
            bk = s_bk[0];
            for (int i = 1; i < 8; ++i)
                if (s_best[i] < best)
                {
                    best = s_best[i];
                    bk = s_bk[i];
                }
            __syncthreads();
            if (best == kKeyMax)
                break;
            const uint32_t bid = key_id(best);
            if (threadIdx.x == 0)
            {
                out[sel] = bid;
                rem[bk] = 1;
            }
            ++sel;
            __syncthreads();
            const uint32_t sb = p.L.off[bid], ns = p.L.off[bid + 1] - sb;
            const uint32_t *sl = p.L.lab + sb;
            uint4 q[CPL];
            load_frag<CPL>(q, p.st.data + (uint64_t)bid * p.st.stride, p.st.nchunks, gl);
            // each warp walks its own 64-entry chunks of the list
            for (uint32_t base = wid * 64; base < n; base += 8 * 64)
            {
                uint32_t m = 0;
                for (uint32_t b = 0; b < 64; b += 32)
                {
                    const uint32_t k = base + b + lane;
                    const bool cand = k < n && !rem[k] && covers(p.L, rl, nl, sl, ns, ids[k]);
                    const unsigned cb = __ballot_sync(kFull, cand);
                    if (cand)
                        s_cover[wid][m + __popc(cb & ((1u << lane) - 1u))] = k;
                    m += __popc(cb);
                }
                __syncwarp();
                if (m)
                {
                    for (uint32_t i = lane; i < m; i += 32)
                        s_pd[wid][i] = __uint_as_float(ids[s_cover[wid][i]]);
                    __syncwarp();
                    eval_candidates<DT, CPL>(p.st.data, p.st.stride, p.st.nchunks, q,
                                             reinterpret_cast<const uint32_t *>(s_pd[wid]), s_pd[wid], (int)m, lane);
                    __syncwarp();
                    evals += m;
                    for (uint32_t i = lane; i < m; i += 32)
                    {
                        const uint32_t k = s_cover[wid][i];
                        const float pd = s_pd[wid][i];
                        if (pd > 0.0f && __fmul_rn(p.alpha, pd) <= dd[k])
                            rem[k] = 1;
                    }
                }
                __syncwarp();
            }
            __syncthreads();
        }
        for (uint32_t i = sel + threadIdx.x; i < p.R; i += blockDim.x)
            out[i] = kInvalid;
        if (threadIdx.x == 0)
            p.degree[row] = sel;
        __syncthreads();
    }
    if (lane == 0 && p.counters)
        atomicAdd(p.counters, evals);
}

// ------------------------------------------------------------------ reverse repair
// Reverse edges of the forward-pruned graph: target t gets source s for
// every s -> t (t valid, t != s).  Order within a target is irrelevant: the
// prune's result does not depend on list order.
static __global__ void fl_rev_count_kernel(const uint32_t *graph, const uint32_t *degree, uint32_t N, uint32_t R,
                                           uint32_t *cnt)
{
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < (uint64_t)N * R;
         e += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t s = (uint32_t)(e / R), i = (uint32_t)(e % R);
        if (i >= min(degree[s], R))
            continue;
        const uint32_t t = graph[e];
        if (t < N && t != s)
            atomicAdd(cnt + t, 1u);
    }
}

static __global__ void fl_rev_fill_kernel(const uint32_t *graph, const uint32_t *degree, uint32_t N, uint32_t R,
                                          uint32_t *cursor, uint32_t *rev)
{
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < (uint64_t)N * R;
         e += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t s = (uint32_t)(e / R), i = (uint32_t)(e % R);
        if (i >= min(degree[s], R))
            continue;
        const uint32_t t = graph[e];
        if (t < N && t != s)
            rev[atomicAdd(cursor + t, 1u)] = s;
    }
}

// canonical_reverse_candidate_count / _fill (ref :5038-5105): a row with
// reverse sources gets the list (its forward row, then its reverse sources
// not already in the forward row); a row without keeps its forward row.
// pass 0 counts into cand_cnt (0 for rows without sources), pass 1 fills
// and lists the touched rows.
static __global__ void __launch_bounds__(kThreads) fl_rev_list_kernel(const uint32_t *graph, const uint32_t *degree,
                                                                       uint32_t N, uint32_t R, const uint32_t *rev_off,
                                                                       const uint32_t *rev, uint32_t *cand_cnt,
                                                                       const uint32_t *cand_off, uint32_t *cand_ids,
                                                                       uint32_t *touched_rows, uint32_t *touched_n,
                                                                       int pass)
{
    const int lane = threadIdx.x & 31;
    for (uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < N; row += gridDim.x * kWarps)
    {
        const uint32_t b = rev_off[row], e = rev_off[row + 1];
        if (b == e)
        {
            if (pass == 0 && lane == 0)
                cand_cnt[row] = 0;
            continue;
        }
        const uint32_t dr = min(degree[row], R);
        const uint32_t *fr = graph + (uint64_t)row * R;
        const uint32_t out = pass ? cand_off[row] : 0;
        if (pass)
            for (uint32_t i = lane; i < dr; i += 32)
                cand_ids[out + i] = fr[i];
        uint32_t m = dr;
        for (uint32_t k0 = b; k0 < e; k0 += 32)
        {
            const uint32_t k = k0 + lane;
            const uint32_t s = k < e ? rev[k] : kInvalid;
            bool keep = k < e && s < N && s != row;
            for (uint32_t i = 0; keep && i < dr; ++i)
                keep = fr[i] != s;
            const unsigned kb = __ballot_sync(kFull, keep);
            if (pass && keep)
                cand_ids[out + m + __popc(kb & ((1u << lane) - 1u))] = s;
            m += __popc(kb);
        }
        if (lane == 0)
        {
            if (pass == 0)
                cand_cnt[row] = m;
            else
                touched_rows[atomicAdd(touched_n, 1u)] = row;
        }
    }
}

// d(row, candidate) for every entry of the touched rows' lists.
template <int DT, int CPL>
__global__ void __launch_bounds__(kThreads) fl_list_dist_kernel(StoreView st, const uint32_t *rows, uint32_t nrows,
                                                                 const uint32_t *off, const uint32_t *ids, float *d,
                                                                 unsigned long long *counters)
{
    const int lane = threadIdx.x & 31, gl = lane & 7;
    unsigned long long evals = 0;
    for (uint32_t r = blockIdx.x * kWarps + (threadIdx.x >> 5); r < nrows; r += gridDim.x * kWarps)
    {
        const uint32_t row = rows[r];
        uint4 q[CPL];
        load_frag<CPL>(q, st.data + (uint64_t)row * st.stride, st.nchunks, gl);
        const uint32_t b = off[row], n = off[row + 1] - b;
        eval_candidates<DT, CPL>(st.data, st.stride, st.nchunks, q, ids + b, d + b, (int)n, lane);
        evals += n;
    }
    if (lane == 0 && counters)
        atomicAdd(counters, evals);
}

// filtered_deterministic_random_graph_kernel semantics (ref :716-744):
// min(R, initial_degree, N - 1) distinct hashed neighbours per row.
static __global__ void fl_random_graph_kernel(uint32_t N, uint32_t R, uint32_t initial_degree, uint32_t seed,
                                              uint32_t *graph, uint32_t *degree)
{
    for (uint32_t row = blockIdx.x * blockDim.x + threadIdx.x; row < N; row += gridDim.x * blockDim.x)
    {
        const uint32_t target = min(min(R, initial_degree), N > 0 ? N - 1 : 0u);
        uint32_t *g = graph + (uint64_t)row * R;
        uint32_t deg = 0, attempt = 0;
        // the hash over attempts reaches every residue long before this bound
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
        degree[row] = deg;
    }
}

// task_rows[p] = the point whose label position p is (ref canonical_make_task_rows :4139-4146).
// Label membership bitmaps: bit p of label l's bitmap for every (p, l) pair.
static __global__ void fl_label_bits_kernel(uint32_t N, const uint32_t *off, const uint32_t *lab,
                                            uint64_t bit_words, uint32_t *bits)
{
    for (uint32_t p = blockIdx.x * blockDim.x + threadIdx.x; p < N; p += gridDim.x * blockDim.x)
        for (uint32_t i = off[p]; i < off[p + 1]; ++i)
            atomicOr(&bits[(uint64_t)lab[i] * bit_words + (p >> 5)], 1u << (p & 31u));
}

static __global__ void fl_task_rows_kernel(uint32_t N, const uint32_t *off, uint32_t *task_rows)
{
    for (uint32_t row = blockIdx.x * blockDim.x + threadIdx.x; row < N; row += gridDim.x * blockDim.x)
        for (uint32_t p = off[row]; p < off[row + 1]; ++p)
            task_rows[p] = row;
}

} // namespace fl
} // namespace dance
