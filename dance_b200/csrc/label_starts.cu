// label_starts.cu -- the inputs that DiskANN computes before the filtered
// build hook: the index entry point and one start point per label.
//
// The DANCE integration patch calls gpu_vamana_filtered_build_* from
// DiskANN's Index::build_filtered_index after upstream DiskANN code has set
// _start = calculate_entry_point() and filled _label_to_start_id
// (integration patch lines 20238-20267, context of the hook).  DiskANN is
// not part of the reference repository, so both are restated here from the
// published algorithm, on the GPU:
//
//  * entry point: the centroid of all points (per dimension a float sum
//    taken point by point in point order, divided by N), then the point
//    nearest to it by squared L2 (per point a float sum over dimensions in
//    order, no fused multiply-add), the lowest index among equal distances.
//    The centroid is summed in exactly that order (one thread per dimension,
//    sequentially), so the result is the sequential definition's, not a
//    reassociated parallel sum's.
//  * label starts: labels in ascending id order; each draws num_candidates
//    of its points and takes the one that has been chosen as a start the
//    fewest times so far (the first such draw on ties), then counts it.
//    DiskANN draws with rand() and walks its labels in hash-set order; here
//    draw k of label l is point hash(seed, l, k) mod |points of l|, so the
//    choice is reproducible.  An empty label gets 0xFFFFFFFF.

#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "../../include/dance_b200.h"
#include "host_common.cuh"

namespace dance
{
namespace
{

template <typename T>
__device__ __forceinline__ float elem(const uint8_t *row, uint32_t j)
{
    return (float)reinterpret_cast<const T *>(row)[j];
}

template <>
__device__ __forceinline__ float elem<__half>(const uint8_t *row, uint32_t j)
{
    return __half2float(reinterpret_cast<const __half *>(row)[j]);
}

// One thread per dimension, points summed in order.
template <typename T>
__global__ void centroid_kernel(const uint8_t *data, uint64_t stride, uint32_t N, uint32_t dim, float *center)
{
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= dim)
        return;
    float s = 0.0f;
    for (uint32_t i = 0; i < N; ++i)
        s = __fadd_rn(s, elem<T>(data + (uint64_t)i * stride, j));
    center[j] = __fdiv_rn(s, (float)N);
}

// Squared distance of every point to the centroid; the smallest (distance,
// index) key wins.
template <typename T>
__global__ void nearest_to_center_kernel(const uint8_t *data, uint64_t stride, uint32_t N, uint32_t dim,
                                         const float *center, unsigned long long *best)
{
    extern __shared__ float c_s[];
    for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x)
        c_s[j] = center[j];
    __syncthreads();
    unsigned long long mine = ~0ull;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x)
    {
        const uint8_t *row = data + (uint64_t)i * stride;
        float d = 0.0f;
        for (uint32_t j = 0; j < dim; ++j)
        {
            const float diff = __fsub_rn(c_s[j], elem<T>(row, j));
            d = __fadd_rn(d, __fmul_rn(diff, diff));
        }
        const unsigned long long k = ((unsigned long long)__float_as_uint(d) << 32) | i;
        mine = k < mine ? k : mine;
    }
    for (int o = 16; o; o >>= 1)
    {
        const unsigned long long other = __shfl_xor_sync(kFull, mine, o);
        mine = other < mine ? other : mine;
    }
    if ((threadIdx.x & 31) == 0 && mine != ~0ull)
        atomicMin(best, mine);
}

__device__ __forceinline__ uint32_t start_draw(uint64_t seed, uint32_t label, uint32_t k)
{
    uint32_t h = hash_u32((uint32_t)seed ^ hash_u32(label * 0x9e3779b1u + 0x7f4a7c15u));
    h = hash_u32(h ^ (uint32_t)(seed >> 32) ^ (k * 0x85ebca6bu + 0x165667b1u));
    return h;
}

// One warp walks the labels in order; lane k holds draw k.
__global__ void label_starts_kernel(const uint32_t *off, const uint32_t *pts, uint32_t num_labels,
                                    uint32_t num_cands, uint64_t seed, uint32_t *counts, uint32_t *starts)
{
    const int lane = threadIdx.x;
    for (uint32_t l = 0; l < num_labels; ++l)
    {
        const uint32_t a = off[l], n = off[l + 1] - a;
        if (n == 0)
        {
            if (lane == 0)
                starts[l] = kInvalid;
            __syncwarp();
            continue;
        }
        uint64_t best = ~0ull; // (count, draw index)
        for (uint32_t k0 = 0; k0 < num_cands; k0 += 32)
        {
            const uint32_t k = k0 + lane;
            if (k < num_cands)
            {
                const uint32_t p = pts[a + start_draw(seed, l, k) % n];
                const uint64_t key = ((uint64_t)counts[p] << 32) | k;
                best = key < best ? key : best;
            }
        }
        for (int o = 16; o; o >>= 1)
        {
            const uint64_t other = __shfl_xor_sync(kFull, best, o);
            best = other < best ? other : best;
        }
        if (lane == 0)
        {
            const uint32_t p = pts[a + start_draw(seed, l, (uint32_t)best) % n];
            starts[l] = p;
            counts[p] += 1;
        }
        __syncwarp();
    }
}

template <typename T>
int entry_point_typed(const uint8_t *data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t *entry_out,
                      cudaStream_t s)
{
    DevBuf buf;
    DANCE_CUDA(buf.ensure(8 + (uint64_t)dim * 4));
    unsigned long long *best = reinterpret_cast<unsigned long long *>(buf.p);
    float *center = reinterpret_cast<float *>(buf.as<uint8_t>() + 8);
    DANCE_CUDA(cudaMemsetAsync(best, 0xFF, 8, s));
    centroid_kernel<T><<<(dim + 127) / 128, 128, 0, s>>>(data, stride, N, dim, center);
    DANCE_LAUNCHED();
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((N + 255) / 256, (uint64_t)sm_count() * 8));
    nearest_to_center_kernel<T><<<grid, 256, dim * 4, s>>>(data, stride, N, dim, center, best);
    DANCE_LAUNCHED();
    unsigned long long h = 0;
    DANCE_CUDA(cudaMemcpyAsync(&h, best, 8, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    *entry_out = (uint32_t)(h & 0xFFFFFFFFull);
    return 0;
}

} // namespace
} // namespace dance

using namespace dance;

extern "C" {

DANCE_API int dance_calculate_entry_point(int dtype, const void *d_data, uint64_t row_stride_bytes,
                                          uint32_t num_points, uint32_t dim, uint32_t *entry_out, void *stream)
{
    int rc = check_store(dtype, d_data, row_stride_bytes, num_points, dim);
    if (rc)
        return rc;
    if (!entry_out || num_points == 0 || dim > 8192)
        return fail(-1, "[entry point] invalid arguments");
    const uint8_t *data = static_cast<const uint8_t *>(d_data);
    cudaStream_t s = as_stream(stream);
    switch (dtype)
    {
    case DANCE_U8:
        return entry_point_typed<uint8_t>(data, row_stride_bytes, num_points, dim, entry_out, s);
    case DANCE_F16:
        return entry_point_typed<__half>(data, row_stride_bytes, num_points, dim, entry_out, s);
    default:
        return entry_point_typed<float>(data, row_stride_bytes, num_points, dim, entry_out, s);
    }
}

DANCE_API int dance_select_label_starts(const uint32_t *d_label_offsets, const uint32_t *d_label_points,
                                        uint32_t num_labels, uint32_t num_points, uint32_t num_candidates,
                                        uint64_t seed, uint32_t *d_starts, void *stream)
{
    if (!d_label_offsets || !d_starts || (!d_label_points && num_labels) || num_candidates == 0 || num_points == 0)
        return fail(-1, "[label starts] invalid arguments");
    if (num_labels == 0)
        return 0;
    cudaStream_t s = as_stream(stream);
    DevBuf counts;
    DANCE_CUDA(counts.ensure((uint64_t)num_points * 4));
    DANCE_CUDA(cudaMemsetAsync(counts.p, 0, (uint64_t)num_points * 4, s));
    label_starts_kernel<<<1, 32, 0, s>>>(d_label_offsets, d_label_points, num_labels, num_candidates, seed,
                                         counts.as<uint32_t>(), d_starts);
    DANCE_LAUNCHED();
    DANCE_CUDA(cudaStreamSynchronize(s)); // the counts buffer is freed on return
    return 0;
}

} // extern "C"
