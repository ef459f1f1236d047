// partition.cu -- the GPU half of the sharded disk-index pipeline: k-means
// partitioning of the base set into overlapping shards.
//
// The DANCE patch drives DiskANN's partitioner (partition_with_ram_budget
// and shard_data_into_clusters_only_ids, integration patch lines
// 20629-20688) before its GPU shard-build loop (lines 3270-3600) and the
// shard merge.  DiskANN is not part of the reference repository, so the
// partitioner is restated here from its published algorithm:
//
//  * k-means++ seeding on a training sample: the first pivot is a drawn
//    point, every further pivot is drawn with probability proportional to
//    the squared distance to the nearest pivot so far.  The weights are
//    quantised to 31-bit integers (w / max w * 2^31, rounded toward zero) so
//    that their prefix sums are exact and the draw is reproducible; a draw
//    is splitmix64(seed, pivot) modulo the total.
//  * Lloyd iterations: every training vector goes to its nearest center;
//    every center becomes the mean of its members.  Members are summed in
//    float64 in vector order inside chunks of kLloydChunk vectors, the chunk
//    sums in chunk order, then divided by the member count and rounded to
//    float; a center without members keeps its place.
//  * assignment: every base point goes to its k_base nearest centers (the
//    shards it is copied into), nearest first, the lower center on ties.
//  * shard id lists: per shard the ids of its points in ascending order
//    (a stable counting sort of the (point, choice) pairs by shard).
//
// Distances are squared L2 in float: per dimension in order, the
// difference, its square and the running sum, each rounded (no fused
// multiply-add), so a CPU restatement reproduces them bit for bit.
// DiskANN computes the same quantity through a GEMM expansion
// (|x|^2 + |c|^2 - 2<x,c>) and draws with std::random_device, so its shards
// are not reproducible run to run; parity with it is not pinned.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <vector>

#include "../../include/dance_b200.h"
#include "host_common.cuh"

namespace dance
{
namespace
{

constexpr uint32_t kLloydChunk = 4096;  // training vectors per partial-sum block
constexpr uint32_t kBucketTile = 4096;  // (point, choice) pairs per warp tile
constexpr uint32_t kMaxKBase = 8;
constexpr uint32_t kMaxShards = 8192;
constexpr uint32_t kMaxAccum = 24576;   // k * dim float64 accumulators in shared memory
constexpr size_t kSmemCap = 200 * 1024; // dynamic shared memory a block may ask for

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x)
{
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

__host__ __device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

__host__ __device__ __forceinline__ uint64_t pivot_draw(uint64_t seed, uint32_t pivot)
{
    return splitmix64(seed ^ splitmix64(0x5deece66dull + pivot));
}

template <typename T>
__device__ __forceinline__ float load_elem(const uint8_t *row, uint32_t j)
{
    return (float)reinterpret_cast<const T *>(row)[j];
}

template <>
__device__ __forceinline__ float load_elem<__half>(const uint8_t *row, uint32_t j)
{
    return __half2float(reinterpret_cast<const __half *>(row)[j]);
}

// Squared L2 between a staged row and a center, dimension by dimension.
__device__ __forceinline__ float sq_dist(const float *x, const float *c, uint32_t dim)
{
    float d = 0.0f;
    for (uint32_t j = 0; j < dim; ++j)
    {
        const float diff = __fsub_rn(c[j], x[j]);
        d = __fadd_rn(d, __fmul_rn(diff, diff));
    }
    return d;
}

// Row stride (floats) of the per-warp staging tile: at least dim, and 4 mod
// 32 so that the 32 lanes of a warp reading their own rows at the same
// column fall in different banks.
__host__ __device__ __forceinline__ uint32_t stage_stride(uint32_t dim)
{
    uint32_t s = (dim + 3u) & ~3u;
    while (s % 32u != 4u)
        s += 4u;
    return s;
}

// Every point's kb nearest centers (ascending (distance, center)).  Each warp
// stages 32 rows in shared memory (coalesced reads, converted to float),
// then every lane scans the centers for its own row.
template <typename T>
__global__ void assign_kernel(const uint8_t *__restrict__ data, uint64_t stride, uint64_t n, uint32_t dim,
                              const float *__restrict__ centers, uint32_t k, uint32_t kb, uint32_t *out_ids,
                              float *out_dists)
{
    extern __shared__ __align__(16) float smem_f[];
    const uint32_t rs = stage_stride(dim);
    const uint32_t kd = (k * dim + 3u) & ~3u;
    float *cs = smem_f;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    float *rows = smem_f + kd + (uint32_t)warp * 32u * rs;
    for (uint32_t i = threadIdx.x; i < k * dim; i += blockDim.x)
        cs[i] = centers[i];
    __syncthreads();
    for (uint64_t base = ((uint64_t)blockIdx.x * wpb + warp) * 32u; base < n; base += (uint64_t)gridDim.x * wpb * 32u)
    {
        const uint32_t nr = (uint32_t)umin64(32u, n - base);
        for (uint32_t r = 0; r < nr; ++r)
        {
            const uint8_t *row = data + (base + r) * stride;
            for (uint32_t j = lane; j < dim; j += 32)
                rows[r * rs + j] = load_elem<T>(row, j);
        }
        __syncwarp();
        if ((uint32_t)lane < nr)
        {
            float bd[kMaxKBase];
            uint32_t bi[kMaxKBase];
#pragma unroll
            for (uint32_t t = 0; t < kMaxKBase; ++t)
            {
                bd[t] = FLT_MAX;
                bi[t] = kInvalid;
            }
            const float *x = rows + (uint32_t)lane * rs;
            for (uint32_t c = 0; c < k; ++c)
            {
                float d = sq_dist(x, cs + c * dim, dim);
                uint32_t ci = c;
                // insertion into the sorted kb-list: the first slot that is
                // empty or holds a strictly larger distance (centers come in
                // ascending order, so the earlier center stays first on ties),
                // then every later entry moves down one slot
                bool moving = false;
#pragma unroll
                for (uint32_t t = 0; t < kMaxKBase; ++t)
                {
                    if (t < kb && (moving || bi[t] == kInvalid || d < bd[t]))
                    {
                        const float td = bd[t];
                        const uint32_t ti = bi[t];
                        bd[t] = d;
                        bi[t] = ci;
                        d = td;
                        ci = ti;
                        moving = true;
                    }
                }
            }
            const uint64_t p = base + (uint32_t)lane;
#pragma unroll
            for (uint32_t t = 0; t < kMaxKBase; ++t)
                if (t < kb)
                {
                    out_ids[p * kb + t] = bi[t];
                    if (out_dists)
                        out_dists[p * kb + t] = bd[t];
                }
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------- k-means++
// mind[i] = min(mind[i], d(x_i, center)) (or = when first).
__global__ void kpp_update_kernel(const uint8_t *__restrict__ train, uint64_t stride, uint64_t n, uint32_t dim,
                                  const float *__restrict__ center, int first, float *mind, unsigned *maxbits)
{
    extern __shared__ __align__(16) float c_s[];
    for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x)
        c_s[j] = center[j];
    __syncthreads();
    unsigned mx = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const float *x = reinterpret_cast<const float *>(train + i * stride);
        const float d = sq_dist(x, c_s, dim);
        const float m = first ? d : fminf(mind[i], d);
        mind[i] = m;
        mx = max(mx, __float_as_uint(m)); // non-negative floats order as their bits
    }
    for (int o = 16; o; o >>= 1)
        mx = max(mx, __shfl_xor_sync(kFull, mx, o));
    if ((threadIdx.x & 31) == 0)
        atomicMax(maxbits, mx);
}

constexpr uint32_t kWeightTile = 4096;

// Quantised weights q_i = floor(mind_i / max * 2^31) and their per-tile
// sums (uint64, exact).
__global__ void kpp_weights_kernel(const float *mind, uint64_t n, const unsigned *maxbits, uint32_t *q,
                                   unsigned long long *tile_sums)
{
    __shared__ unsigned long long s[32];
    const float mx = __uint_as_float(*maxbits);
    const uint64_t base = (uint64_t)blockIdx.x * kWeightTile;
    unsigned long long acc = 0;
    for (uint32_t t = threadIdx.x; t < kWeightTile; t += blockDim.x)
    {
        const uint64_t i = base + t;
        if (i >= n)
            break;
        uint32_t w = 1u;
        if (mx > 0.0f)
            w = __float2uint_rz(__fmul_rn(__fdiv_rn(mind[i], mx), 2147483648.0f));
        q[i] = w;
        acc += w;
    }
    for (int o = 16; o; o >>= 1)
        acc += __shfl_xor_sync(kFull, acc, o);
    if ((threadIdx.x & 31) == 0)
        s[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0)
    {
        unsigned long long t = 0;
        for (uint32_t w = 0; w < blockDim.x / 32; ++w)
            t += s[w];
        tile_sums[blockIdx.x] = t;
    }
}

// One block: finds the tile whose running sum passes r, then the point in it
// (the smallest i with q_0 + ... + q_i > r), and copies that row to `center`.
__global__ void kpp_pick_kernel(const uint32_t *q, uint64_t n, const unsigned long long *tile_sums, uint32_t ntiles,
                                uint64_t seed, uint32_t pivot, const uint8_t *train, uint64_t stride, uint32_t dim,
                                float *center, uint64_t *picked)
{
    __shared__ uint64_t s_pick;
    if (threadIdx.x == 0)
    {
        unsigned long long total = 0;
        for (uint32_t t = 0; t < ntiles; ++t)
            total += tile_sums[t];
        const unsigned long long r = total ? pivot_draw(seed, pivot) % total : 0ull;
        unsigned long long run = 0;
        uint32_t tile = 0;
        for (; tile + 1 < ntiles; ++tile)
        {
            if (run + tile_sums[tile] > r)
                break;
            run += tile_sums[tile];
        }
        const uint64_t end = umin64(n, (uint64_t)(tile + 1) * kWeightTile);
        uint64_t pick = end - 1;
        for (uint64_t i = (uint64_t)tile * kWeightTile; i < end; ++i)
        {
            run += q[i];
            if (run > r)
            {
                pick = i;
                break;
            }
        }
        s_pick = pick;
        picked[pivot] = pick;
    }
    __syncthreads();
    const float *x = reinterpret_cast<const float *>(train + s_pick * stride);
    for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x)
        center[j] = x[j];
}

__global__ void copy_row_kernel(const uint8_t *train, uint64_t stride, uint64_t row, uint32_t dim, float *center,
                                uint64_t *picked)
{
    if (threadIdx.x == 0)
        picked[0] = row;
    const float *x = reinterpret_cast<const float *>(train + row * stride);
    for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x)
        center[j] = x[j];
}

// ---------------------------------------------------------------- Lloyd
// Per chunk of kLloydChunk vectors: member sums per (center, dimension) in
// vector order (float64), member counts, and the chunk's distance sum.
__global__ void lloyd_partial_kernel(const uint8_t *__restrict__ train, uint64_t stride, uint64_t n, uint32_t dim,
                                     uint32_t k, const uint32_t *assign, const float *dist, double *partial,
                                     uint32_t *counts, double *resid)
{
    extern __shared__ __align__(16) double acc[];
    const uint32_t kd = k * dim;
    for (uint32_t i = threadIdx.x; i < kd; i += blockDim.x)
        acc[i] = 0.0;
    uint32_t *cnt = reinterpret_cast<uint32_t *>(acc + kd);
    for (uint32_t i = threadIdx.x; i < k; i += blockDim.x)
        cnt[i] = 0;
    __syncthreads();
    const uint64_t b0 = (uint64_t)blockIdx.x * kLloydChunk;
    const uint64_t b1 = umin64(n, b0 + kLloydChunk);
    double rs = 0.0;
    for (uint64_t i = b0; i < b1; ++i)
    {
        const uint32_t c = assign[i];
        const float *x = reinterpret_cast<const float *>(train + i * stride);
        for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x)
            acc[c * dim + j] = __dadd_rn(acc[c * dim + j], (double)x[j]);
        if (threadIdx.x == 0)
        {
            cnt[c] += 1;
            rs = __dadd_rn(rs, (double)dist[i]);
        }
    }
    __syncthreads();
    double *out = partial + (uint64_t)blockIdx.x * kd;
    for (uint32_t i = threadIdx.x; i < kd; i += blockDim.x)
        out[i] = acc[i];
    for (uint32_t i = threadIdx.x; i < k; i += blockDim.x)
        counts[(uint64_t)blockIdx.x * k + i] = cnt[i];
    if (threadIdx.x == 0)
        resid[blockIdx.x] = rs;
}

// One thread per (center, dimension): chunk sums in chunk order, then the mean.
__global__ void lloyd_reduce_kernel(const double *partial, const uint32_t *counts, uint32_t nchunks, uint32_t k,
                                    uint32_t dim, float *centers, const double *resid, double *resid_total)
{
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e == 0 && resid_total)
    {
        double t = 0.0;
        for (uint32_t b = 0; b < nchunks; ++b)
            t = __dadd_rn(t, resid[b]);
        *resid_total = t;
    }
    if (e >= k * dim)
        return;
    const uint32_t c = e / dim;
    double s = 0.0;
    uint64_t m = 0;
    for (uint32_t b = 0; b < nchunks; ++b)
    {
        s = __dadd_rn(s, partial[(uint64_t)b * k * dim + e]);
        m += counts[(uint64_t)b * k + c];
    }
    if (m)
        centers[e] = __double2float_rn(__ddiv_rn(s, (double)m));
}

// ---------------------------------------------------------------- shard id lists
// hist[s * ntiles + t] = pairs of tile t that choose shard s.
__global__ void bucket_count_kernel(const uint32_t *keys, uint64_t m, uint32_t S, uint32_t ntiles, uint32_t *hist)
{
    extern __shared__ uint32_t cnt_s[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    uint32_t *cnt = cnt_s + (uint32_t)warp * S;
    const uint32_t tile = blockIdx.x * wpb + warp;
    for (uint32_t s = lane; s < S; s += 32)
        cnt[s] = 0;
    __syncwarp();
    if (tile < ntiles)
    {
        const uint64_t e0 = (uint64_t)tile * kBucketTile;
        const uint64_t e1 = umin64(m, e0 + kBucketTile);
        for (uint64_t e = e0 + lane; e < e1; e += 32)
        {
            const uint32_t key = keys[e];
            if (key < S) // a point with fewer valid choices than k_base
                atomicAdd(&cnt[key], 1u);
        }
        __syncwarp();
        for (uint32_t s = lane; s < S; s += 32)
            hist[(uint64_t)s * ntiles + tile] = cnt[s];
    }
}

// Writes every pair's point id at its shard's running position: pairs are
// taken 32 at a time in order, lanes with the same shard ranked by lane.
__global__ void bucket_fill_kernel(const uint32_t *keys, uint64_t m, uint32_t kb, uint32_t S, uint32_t ntiles,
                                   const uint32_t *off, uint32_t *ids)
{
    extern __shared__ uint32_t pos_s[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    uint32_t *pos = pos_s + (uint32_t)warp * S;
    const uint32_t tile = blockIdx.x * wpb + warp;
    if (tile >= ntiles)
        return;
    for (uint32_t s = lane; s < S; s += 32)
        pos[s] = off[(uint64_t)s * ntiles + tile];
    __syncwarp();
    const unsigned lt = (1u << lane) - 1u;
    const uint64_t e0 = (uint64_t)tile * kBucketTile;
    const uint64_t e1 = umin64(m, e0 + kBucketTile);
    for (uint64_t c = e0; c < e1; c += 32)
    {
        const uint64_t e = c + lane;
        uint32_t key = e < e1 ? keys[e] : 0xFFFFFFFFu;
        if (key >= S)
            key = 0xFFFFFFFFu;
        const bool valid = key != 0xFFFFFFFFu;
        const unsigned peers = __match_any_sync(kFull, key);
        const uint32_t rank = __popc(peers & lt);
        uint32_t base = 0;
        if (valid)
            base = pos[key];
        __syncwarp();
        if (valid)
        {
            ids[base + rank] = (uint32_t)(e / kb);
            if ((peers >> lane) == 1u) // highest lane of its group advances the cursor
                pos[key] = base + __popc(peers);
        }
        __syncwarp();
    }
}

__global__ void shard_offsets_kernel(const uint32_t *off, uint32_t S, uint32_t ntiles, uint32_t *shard_off)
{
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s <= S)
        shard_off[s] = off[(uint64_t)s * ntiles]; // off[S * ntiles] is the total
}

int check_train(const void *d_train, uint64_t stride, uint64_t n, uint32_t dim, uint32_t k)
{
    if (!d_train || n == 0 || dim == 0 || k == 0)
        return fail(-1, "[kmeans] empty training set or no centers (n=%llu dim=%u k=%u)", (unsigned long long)n,
                    dim, k);
    if (stride % 4 != 0 || stride < (uint64_t)dim * 4 || (reinterpret_cast<uintptr_t>(d_train) & 3u))
        return fail(-1, "[kmeans] training rows must be 4-byte aligned floats with stride >= dim*4");
    if ((uint64_t)k * dim * 8 + (uint64_t)k * 4 > kSmemCap)
        return fail(-1, "[kmeans] %u centers of dimension %u exceed the shared-memory accumulators (k*dim <= %u)", k,
                    dim, kMaxAccum);
    return 0;
}

template <typename T>
int assign_typed(const uint8_t *data, uint64_t stride, uint64_t n, uint32_t dim, const float *centers, uint32_t k,
                 uint32_t kb, uint32_t *out_ids, float *out_dists, cudaStream_t s)
{
    const size_t cbytes = (size_t)((k * dim + 3u) & ~3u) * 4u;
    const size_t wbytes = (size_t)32u * stage_stride(dim) * 4u;
    if (cbytes + wbytes > kSmemCap)
        return fail(-1, "[partition] %u centers of dimension %u do not fit the shared-memory tiles", k, dim);
    const int wpb = (int)std::min<size_t>(4, (kSmemCap - cbytes) / wbytes);
    const size_t smem = cbytes + (size_t)wpb * wbytes;
    DANCE_CUDA(cudaFuncSetAttribute(assign_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const uint64_t need = (n + 32u * wpb - 1) / (32u * wpb);
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>(need, (uint64_t)sm_count() * 8));
    assign_kernel<T><<<grid, wpb * 32, smem, s>>>(data, stride, n, dim, centers, k, kb, out_ids, out_dists);
    DANCE_LAUNCHED();
    return 0;
}

int assign_any(int dtype, const void *d_data, uint64_t stride, uint64_t n, uint32_t dim, const float *centers,
               uint32_t k, uint32_t kb, uint32_t *out_ids, float *out_dists, cudaStream_t s)
{
    const uint8_t *data = static_cast<const uint8_t *>(d_data);
    switch (dtype)
    {
    case DANCE_U8:
        return assign_typed<uint8_t>(data, stride, n, dim, centers, k, kb, out_ids, out_dists, s);
    case DANCE_F16:
        return assign_typed<__half>(data, stride, n, dim, centers, k, kb, out_ids, out_dists, s);
    default:
        return assign_typed<float>(data, stride, n, dim, centers, k, kb, out_ids, out_dists, s);
    }
}

} // namespace
} // namespace dance

using namespace dance;

extern "C" {

DANCE_API int dance_kmeanspp_seed(const float *d_train, uint64_t row_stride_bytes, uint64_t n, uint32_t dim,
                                  uint32_t k, uint64_t seed, float *d_centers, uint64_t *d_picked, void *stream)
{
    int rc = check_train(d_train, row_stride_bytes, n, dim, k);
    if (rc)
        return rc;
    if (!d_centers || !d_picked)
        return fail(-1, "[kmeans++] null output");
    cudaStream_t s = as_stream(stream);
    const uint8_t *train = reinterpret_cast<const uint8_t *>(d_train);
    const uint32_t ntiles = (uint32_t)((n + kWeightTile - 1) / kWeightTile);
    DevBuf mind, q, tiles, mx;
    DANCE_CUDA(mind.ensure(n * 4));
    DANCE_CUDA(q.ensure(n * 4));
    DANCE_CUDA(tiles.ensure((size_t)ntiles * 8));
    DANCE_CUDA(mx.ensure(4));
    const uint64_t first = splitmix64(seed) % n;
    copy_row_kernel<<<1, 128, 0, s>>>(train, row_stride_bytes, first, dim, d_centers, d_picked);
    DANCE_LAUNCHED();
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count() * 8));
    for (uint32_t p = 1; p < k; ++p)
    {
        DANCE_CUDA(cudaMemsetAsync(mx.p, 0, 4, s));
        kpp_update_kernel<<<grid, 256, dim * 4, s>>>(train, row_stride_bytes, n, dim,
                                                     d_centers + (uint64_t)(p - 1) * dim, p == 1, mind.as<float>(),
                                                     mx.as<unsigned>());
        DANCE_LAUNCHED();
        kpp_weights_kernel<<<ntiles, 256, 0, s>>>(mind.as<float>(), n, mx.as<unsigned>(), q.as<uint32_t>(),
                                                  tiles.as<unsigned long long>());
        DANCE_LAUNCHED();
        kpp_pick_kernel<<<1, 128, 0, s>>>(q.as<uint32_t>(), n, tiles.as<unsigned long long>(), ntiles, seed, p, train,
                                          row_stride_bytes, dim, d_centers + (uint64_t)p * dim, d_picked);
        DANCE_LAUNCHED();
    }
    DANCE_CUDA(cudaStreamSynchronize(s)); // the scratch buffers are freed on return
    return 0;
}

DANCE_API int dance_kmeans_lloyd(const float *d_train, uint64_t row_stride_bytes, uint64_t n, uint32_t dim, uint32_t k,
                                 uint32_t iters, float *d_centers, uint32_t *d_assign, double *residual_out,
                                 void *stream)
{
    int rc = check_train(d_train, row_stride_bytes, n, dim, k);
    if (rc)
        return rc;
    if (!d_centers)
        return fail(-1, "[kmeans] null centers");
    cudaStream_t s = as_stream(stream);
    const uint8_t *train = reinterpret_cast<const uint8_t *>(d_train);
    const uint32_t nchunks = (uint32_t)((n + kLloydChunk - 1) / kLloydChunk);
    DevBuf asg, dist, partial, counts, resid, rtot;
    DANCE_CUDA(asg.ensure(n * 4));
    DANCE_CUDA(dist.ensure(n * 4));
    DANCE_CUDA(partial.ensure((size_t)nchunks * k * dim * 8));
    DANCE_CUDA(counts.ensure((size_t)nchunks * k * 4));
    DANCE_CUDA(resid.ensure((size_t)nchunks * 8));
    DANCE_CUDA(rtot.ensure(8));
    DANCE_CUDA(cudaMemsetAsync(rtot.p, 0, 8, s));
    const size_t smem = (size_t)k * dim * 8 + (size_t)k * 4;
    DANCE_CUDA(cudaFuncSetAttribute(lloyd_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    for (uint32_t it = 0; it < iters; ++it)
    {
        if ((rc = assign_any(DANCE_F32, d_train, row_stride_bytes, n, dim, d_centers, k, 1, asg.as<uint32_t>(),
                             dist.as<float>(), s)))
            return rc;
        lloyd_partial_kernel<<<nchunks, 128, smem, s>>>(train, row_stride_bytes, n, dim, k, asg.as<uint32_t>(),
                                                        dist.as<float>(), partial.as<double>(),
                                                        counts.as<uint32_t>(), resid.as<double>());
        DANCE_LAUNCHED();
        lloyd_reduce_kernel<<<(k * dim + 127) / 128, 128, 0, s>>>(partial.as<double>(), counts.as<uint32_t>(),
                                                                  nchunks, k, dim, d_centers, resid.as<double>(),
                                                                  rtot.as<double>());
        DANCE_LAUNCHED();
    }
    if (d_assign)
    {
        if ((rc = assign_any(DANCE_F32, d_train, row_stride_bytes, n, dim, d_centers, k, 1, d_assign, nullptr, s)))
            return rc;
    }
    double r = 0.0;
    DANCE_CUDA(cudaMemcpyAsync(&r, rtot.p, 8, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    if (residual_out)
        *residual_out = r;
    return 0;
}

DANCE_API int dance_partition_assign(int dtype, const void *d_data, uint64_t row_stride_bytes, uint64_t num_points,
                                     uint32_t dim, const float *d_centers, uint32_t num_centers, uint32_t k_base,
                                     uint32_t *d_out_centers, float *d_out_dists, void *stream)
{
    const int es = elem_size(dtype);
    if (!es)
        return fail(-1, "[partition] unknown dtype %d", dtype);
    if (!d_data || !d_centers || !d_out_centers || num_points == 0 || dim == 0 || num_centers == 0)
        return fail(-1, "[partition] invalid arguments");
    if (k_base == 0 || k_base > kMaxKBase || k_base > num_centers)
        return fail(-1, "[partition] k_base=%u must be in [1, min(%u, centers=%u)]", k_base, kMaxKBase, num_centers);
    if (row_stride_bytes < (uint64_t)dim * es || row_stride_bytes % es != 0 ||
        (reinterpret_cast<uintptr_t>(d_data) % es) != 0)
        return fail(-1, "[partition] row stride %llu must hold dim*%d bytes and keep elements aligned",
                    (unsigned long long)row_stride_bytes, es);
    return assign_any(dtype, d_data, row_stride_bytes, num_points, dim, d_centers, num_centers, k_base, d_out_centers,
                      d_out_dists, as_stream(stream));
}

DANCE_API int dance_partition_buckets(const uint32_t *d_assign, uint64_t num_points, uint32_t k_base,
                                      uint32_t num_shards, uint32_t *d_shard_offsets, uint32_t *d_shard_ids,
                                      void *stream)
{
    if (!d_assign || !d_shard_offsets || !d_shard_ids || num_points == 0 || k_base == 0 || k_base > kMaxKBase)
        return fail(-1, "[partition] invalid bucket arguments");
    if (num_shards == 0 || num_shards > kMaxShards)
        return fail(-1, "[partition] %u shards (1..%u supported)", num_shards, kMaxShards);
    const uint64_t m = num_points * k_base;
    if (m >= 0xFFFFFFFFull)
        return fail(-1, "[partition] %llu (point, shard) pairs exceed 32-bit offsets", (unsigned long long)m);
    cudaStream_t s = as_stream(stream);
    const uint32_t ntiles = (uint32_t)((m + kBucketTile - 1) / kBucketTile);
    const uint64_t hn = (uint64_t)num_shards * ntiles;
    if (hn >= 0xFFFFFFFFull)
        return fail(-1, "[partition] histogram of %llu cells too large", (unsigned long long)hn);
    DevBuf hist, off, tiles;
    DANCE_CUDA(hist.ensure(hn * 4));
    DANCE_CUDA(off.ensure((hn + 1) * 4));
    const uint32_t stiles = (uint32_t)((hn + kScanTile - 1) / kScanTile);
    DANCE_CUDA(tiles.ensure((size_t)stiles * 4 + 4));
    const int wpb = 4;
    const size_t smem = (size_t)wpb * num_shards * 4;
    DANCE_CUDA(cudaFuncSetAttribute(bucket_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    DANCE_CUDA(cudaFuncSetAttribute(bucket_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const uint32_t grid = (ntiles + wpb - 1) / wpb;
    bucket_count_kernel<<<grid, wpb * 32, smem, s>>>(d_assign, m, num_shards, ntiles, hist.as<uint32_t>());
    DANCE_LAUNCHED();
    scan_tile_sums_kernel<<<stiles, kScanThreads, 0, s>>>(hist.as<uint32_t>(), (uint32_t)hn, tiles.as<uint32_t>());
    DANCE_LAUNCHED();
    scan_tile_offsets_kernel<<<1, kScanThreads, 0, s>>>(tiles.as<uint32_t>(), stiles);
    DANCE_LAUNCHED();
    scan_apply_kernel<<<stiles, kScanThreads, 0, s>>>(hist.as<uint32_t>(), (uint32_t)hn, tiles.as<uint32_t>(),
                                                      off.as<uint32_t>(), nullptr);
    DANCE_LAUNCHED();
    bucket_fill_kernel<<<grid, wpb * 32, smem, s>>>(d_assign, m, k_base, num_shards, ntiles, off.as<uint32_t>(),
                                                    d_shard_ids);
    DANCE_LAUNCHED();
    shard_offsets_kernel<<<(num_shards + 128) / 128, 128, 0, s>>>(off.as<uint32_t>(), num_shards, ntiles,
                                                                 d_shard_offsets);
    DANCE_LAUNCHED();
    DANCE_CUDA(cudaStreamSynchronize(s)); // the scratch buffers are freed on return
    return 0;
}

} // extern "C"
