// gpu_merge.cu -- merge of overlapping shard graphs into one DiskANN graph.
//
// Replaces diskann::merge_shards_gpu of the reference (src/gpu_merge.cu:351-871,
// declared in include/gpu_merge.h:13) with the same files, semantics and
// return codes:
//   * shard i's graph is <vamana_prefix>i<vamana_suffix> (DiskANN graph
//     layout, frozen points must be 0) and its id map
//     <idmaps_prefix>i<idmaps_suffix> (u32 n, u32 1, n global ids);
//   * every edge is remapped to global ids, self loops are dropped, and for
//     each source the distinct destinations are ranked by
//     hash_edge32(src, dst, seed) (ties by destination, as the reference's
//     stable key sort over (src, dst)-sorted unique edges gives) and the
//     first max_degree kept (reference :103-160, :586-589, :677-731);
//   * the medoids file is u32 nshards, u32 1, then each shard's medoid as a
//     global id; the merged graph's start is the last shard's medoid
//     (:551-569).
// The B200 path: sources are processed in ranges ("buckets") sized to the
// device memory; per bucket the edges are put into a CSR by source with a
// count / scan / fill, and one warp per source (one block for long
// segments) sorts, deduplicates, ranks and truncates its segment in shared
// memory -- no device-wide sort.  DISKANN_GPU_MERGE_DEVICES (comma list)
// spreads buckets over several GPUs, one host thread each, like the
// reference's round-robin (:643-650).

#include <cuda.h> // CUcontext / CUresult types for the context id lookup
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "../../include/gpu_merge.h"
#include "host_common.cuh"

namespace dance
{

__host__ __device__ __forceinline__ uint32_t hash_edge32(uint32_t src, uint32_t dst, uint64_t seed)
{
    uint64_t x = ((uint64_t)src << 32) ^ (uint64_t)dst ^ seed;
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdULL;
    x ^= x >> 33;
    x *= 0xc4ceb9fe1a85ec53ULL;
    x ^= x >> 33;
    return (uint32_t)(x ^ (x >> 32));
}

static __global__ void mrg_count_kernel(const uint32_t *src, uint64_t n, uint32_t begin, uint32_t count,
                                        uint32_t *cnt)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t s = src[i] - begin;
        if (s < count)
            atomicAdd(&cnt[s], 1u);
    }
}

static __global__ void mrg_fill_kernel(const uint32_t *src, const uint32_t *dst, uint64_t n, uint32_t begin,
                                       uint32_t count, uint32_t *cursor, uint32_t *seg)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t s = src[i] - begin;
        if (s < count)
            seg[atomicAdd(&cursor[s], 1u)] = dst[i];
    }
}

constexpr uint32_t kMergeWarpCap = 512;   // segment length handled by one warp
constexpr uint32_t kMergeBlockCap = 16384; // segment length handled by one block

// Sorted, distinct destinations ranked by (hash, dst); keeps the first
// max_degree.  a[0..n2) in shared memory holds the segment padded with
// UINT32_MAX; keys is a scratch of n2 uint64.  Warp version.
__device__ void mrg_select_warp(uint32_t src, uint32_t *a, uint64_t *keys, int n, int n2, uint32_t max_degree,
                                uint64_t seed, uint32_t *out_row, uint32_t *out_deg, int lane)
{
    warp_sort_smem_u32(a, n2, lane);
    int u = 0;
    for (int b = 0; b < n2; b += 32)
    {
        const int i = b + lane;
        const bool first = i < n && (i == 0 || a[i - 1] != a[i]);
        const unsigned bm = __ballot_sync(kFull, first);
        if (first)
        {
            const uint32_t d = a[i];
            keys[u + __popc(bm & ((1u << lane) - 1u))] = ((uint64_t)hash_edge32(src, d, seed) << 32) | d;
        }
        u += __popc(bm);
    }
    __syncwarp();
    const int u2 = max(32, next_pow2(u));
    for (int i = u + lane; i < u2; i += 32)
        keys[i] = kKeyMax;
    __syncwarp();
    warp_sort_smem_u64(keys, u2, lane);
    const uint32_t keep = min((uint32_t)u, max_degree);
    for (uint32_t i = lane; i < keep; i += 32)
        out_row[i] = (uint32_t)(keys[i] & 0xFFFFFFFFu);
    if (lane == 0)
        *out_deg = keep;
    __syncwarp();
}

struct MergeSelectParams
{
    const uint32_t *offsets; // count + 1
    const uint32_t *seg;
    uint32_t begin, count, max_degree;
    uint64_t seed;
    uint32_t *out_neighbors; // count x max_degree
    uint32_t *out_degrees;   // count
    uint32_t *long_list;     // sources whose segment exceeds kMergeWarpCap
    uint32_t *long_count;
    uint32_t *error;         // set when a segment exceeds kMergeBlockCap
};

static __global__ void __launch_bounds__(128) mrg_select_kernel(MergeSelectParams p)
{
    __shared__ __align__(16) uint32_t s_a[4][kMergeWarpCap];
    __shared__ __align__(16) uint64_t s_k[4][kMergeWarpCap];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (uint32_t s = blockIdx.x * 4 + w; s < p.count; s += gridDim.x * 4)
    {
        const uint32_t beg = p.offsets[s], end = p.offsets[s + 1];
        const int n = (int)(end - beg);
        uint32_t *row = p.out_neighbors + (uint64_t)s * p.max_degree;
        if (n == 0)
        {
            if (lane == 0)
                p.out_degrees[s] = 0;
            continue;
        }
        if ((uint32_t)n > kMergeWarpCap)
        {
            if (lane == 0)
                p.long_list[atomicAdd(p.long_count, 1u)] = s;
            continue;
        }
        const int n2 = max(32, next_pow2(n));
        for (int i = lane; i < n2; i += 32)
            s_a[w][i] = i < n ? p.seg[beg + i] : kInvalid;
        __syncwarp();
        mrg_select_warp(p.begin + s, s_a[w], s_k[w], n, n2, p.max_degree, p.seed, row, &p.out_degrees[s], lane);
    }
}

// Long segments: one block each, sorted by the whole block in shared memory.
static __global__ void __launch_bounds__(256) mrg_select_long_kernel(MergeSelectParams p)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint32_t *a = reinterpret_cast<uint32_t *>(smem_raw);                         // kMergeBlockCap
    uint64_t *keys = reinterpret_cast<uint64_t *>(smem_raw + 4u * kMergeBlockCap); // kMergeBlockCap
    __shared__ int s_u;
    const uint32_t nlong = *p.long_count;
    for (uint32_t h = blockIdx.x; h < nlong; h += gridDim.x)
    {
        const uint32_t s = p.long_list[h];
        const uint32_t beg = p.offsets[s], end = p.offsets[s + 1];
        const uint32_t n = end - beg;
        if (n > kMergeBlockCap)
        {
            if (threadIdx.x == 0)
                atomicMax(p.error, n);
            continue;
        }
        const uint32_t n2 = (uint32_t)next_pow2((int)n);
        for (uint32_t i = threadIdx.x; i < n2; i += blockDim.x)
            a[i] = i < n ? p.seg[beg + i] : kInvalid;
        __syncthreads();
        for (uint32_t size = 2; size <= n2; size <<= 1)
            for (uint32_t j = size >> 1; j > 0; j >>= 1)
            {
                for (uint32_t i = threadIdx.x; i < n2; i += blockDim.x)
                {
                    const uint32_t l = i ^ j;
                    if (l > i)
                    {
                        const uint32_t x = a[i], y = a[l];
                        if (((i & size) == 0) ? (x > y) : (x < y))
                        {
                            a[i] = y;
                            a[l] = x;
                        }
                    }
                }
                __syncthreads();
            }
        // distinct destinations -> keys (block compaction by warp 0 in order)
        if (threadIdx.x < 32)
        {
            const int lane = threadIdx.x;
            int u = 0;
            for (uint32_t b = 0; b < n2; b += 32)
            {
                const uint32_t i = b + lane;
                const bool first = i < n && (i == 0 || a[i - 1] != a[i]);
                const unsigned bm = __ballot_sync(kFull, first);
                if (first)
                    keys[u + __popc(bm & ((1u << lane) - 1u))] =
                        ((uint64_t)hash_edge32(p.begin + s, a[i], p.seed) << 32) | a[i];
                u += __popc(bm);
            }
            if (lane == 0)
                s_u = u;
        }
        __syncthreads();
        const int u = s_u;
        const uint32_t u2 = (uint32_t)max(32, next_pow2(u));
        for (uint32_t i = u + threadIdx.x; i < u2; i += blockDim.x)
            keys[i] = kKeyMax;
        __syncthreads();
        for (uint32_t size = 2; size <= u2; size <<= 1)
            for (uint32_t j = size >> 1; j > 0; j >>= 1)
            {
                for (uint32_t i = threadIdx.x; i < u2; i += blockDim.x)
                {
                    const uint32_t l = i ^ j;
                    if (l > i)
                    {
                        const uint64_t x = keys[i], y = keys[l];
                        if (((i & size) == 0) ? (x > y) : (x < y))
                        {
                            keys[i] = y;
                            keys[l] = x;
                        }
                    }
                }
                __syncthreads();
            }
        const uint32_t keep = min((uint32_t)u, p.max_degree);
        uint32_t *row = p.out_neighbors + (uint64_t)s * p.max_degree;
        for (uint32_t i = threadIdx.x; i < keep; i += blockDim.x)
            row[i] = (uint32_t)(keys[i] & 0xFFFFFFFFu);
        if (threadIdx.x == 0)
            p.out_degrees[s] = keep;
        __syncthreads();
    }
}

// Device part of one bucket: edges (src, dst) already remapped and without
// self loops; sources [begin, begin + count).  Rows of out_neighbors beyond a
// source's degree are left as they are.
static int merge_bucket_device(const uint32_t *d_src, const uint32_t *d_dst, uint64_t n_edges, uint32_t begin,
                               uint32_t count, uint32_t max_degree, uint64_t seed, uint32_t *d_out_neighbors,
                               uint32_t *d_out_degrees, cudaStream_t s)
{
    if (count == 0)
        return 0;
    DevBuf cnt, off, cursor, tiles, seg, longl, misc;
    const uint32_t ntiles = (count + kScanTile - 1) / kScanTile;
    DANCE_CUDA(cnt.ensure((uint64_t)count * 4));
    DANCE_CUDA(off.ensure(((uint64_t)count + 1) * 4));
    DANCE_CUDA(cursor.ensure((uint64_t)count * 4));
    DANCE_CUDA(tiles.ensure(((uint64_t)ntiles + 1) * 4));
    DANCE_CUDA(seg.ensure(std::max<uint64_t>(n_edges, 1) * 4));
    DANCE_CUDA(longl.ensure((uint64_t)count * 4));
    DANCE_CUDA(misc.ensure(16));
    DANCE_CUDA(cudaMemsetAsync(cnt.p, 0, (uint64_t)count * 4, s));
    DANCE_CUDA(cudaMemsetAsync(misc.p, 0, 16, s));
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((n_edges + 255) / 256, sm_count() * 16ull));
    if (n_edges)
    {
        mrg_count_kernel<<<grid, 256, 0, s>>>(d_src, n_edges, begin, count, cnt.as<uint32_t>());
        DANCE_LAUNCHED();
    }
    scan_tile_sums_kernel<<<ntiles, kScanThreads, 0, s>>>(cnt.as<uint32_t>(), count, tiles.as<uint32_t>());
    DANCE_LAUNCHED();
    scan_tile_offsets_kernel<<<1, kScanThreads, 0, s>>>(tiles.as<uint32_t>(), ntiles);
    DANCE_LAUNCHED();
    scan_apply_kernel<<<ntiles, kScanThreads, 0, s>>>(cnt.as<uint32_t>(), count, tiles.as<uint32_t>(),
                                                      off.as<uint32_t>(), cursor.as<uint32_t>());
    DANCE_LAUNCHED();
    if (n_edges)
    {
        mrg_fill_kernel<<<grid, 256, 0, s>>>(d_src, d_dst, n_edges, begin, count, cursor.as<uint32_t>(),
                                             seg.as<uint32_t>());
        DANCE_LAUNCHED();
    }
    MergeSelectParams mp{};
    mp.offsets = off.as<uint32_t>();
    mp.seg = seg.as<uint32_t>();
    mp.begin = begin;
    mp.count = count;
    mp.max_degree = max_degree;
    mp.seed = seed;
    mp.out_neighbors = d_out_neighbors;
    mp.out_degrees = d_out_degrees;
    mp.long_list = longl.as<uint32_t>();
    mp.long_count = misc.as<uint32_t>();
    mp.error = misc.as<uint32_t>() + 1;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mrg_select_kernel, 128, 0);
    const int g2 = (int)std::max<uint64_t>(1, std::min<uint64_t>((count + 3) / 4, (uint64_t)std::max(per_sm, 1) *
                                                                                       sm_count()));
    mrg_select_kernel<<<g2, 128, 0, s>>>(mp);
    DANCE_LAUNCHED();
    const size_t lsmem = 12u * kMergeBlockCap;
    DANCE_CUDA(allow_smem(mrg_select_long_kernel, lsmem));
    mrg_select_long_kernel<<<sm_count(), 256, lsmem, s>>>(mp);
    DANCE_LAUNCHED();
    uint32_t err = 0;
    DANCE_CUDA(cudaMemcpyAsync(&err, mp.error, 4, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    if (err)
        return fail(-20, "a source has %u merged edges, more than the %u supported per source", err, kMergeBlockCap);
    return 0;
}

} // namespace dance

using namespace dance;

extern "C" DANCE_API int dance_merge_edges_device(const uint32_t *d_src, const uint32_t *d_dst, uint64_t n_edges,
                                                  uint32_t node_begin, uint32_t node_count, uint32_t max_degree,
                                                  uint64_t seed, uint32_t *d_out_neighbors, uint32_t *d_out_degrees,
                                                  void *stream)
{
    if ((n_edges && (!d_src || !d_dst)) || !d_out_neighbors || !d_out_degrees || max_degree == 0)
        return fail(-1, "invalid merge arguments");
    return merge_bucket_device(d_src, d_dst, n_edges, node_begin, node_count, max_degree, seed, d_out_neighbors,
                               d_out_degrees, as_stream(stream));
}

// ---------------------------------------------------------------- no-alloc variant
// dance_merge_edges_device_noalloc runs the same kernels as
// dance_merge_edges_device, but its scratch (per-source counts, offsets and
// cursors, scan tile sums, the long-segment list, two status words and the
// source-sorted edge array) lives in one fixed array in the library's device
// memory instead of buffers allocated per call.  The array holds
// kNoAllocMaxNodes sources and kNoAllocMaxEdges edges, about 4.3 MiB; larger
// requests are refused before anything is launched.
namespace dance
{
constexpr uint32_t kNoAllocMaxNodes = 16384;
constexpr uint32_t kNoAllocMaxEdges = 1u << 20;
constexpr uint32_t kNoAllocTiles = (kNoAllocMaxNodes + kScanTile - 1) / kScanTile;

constexpr uint32_t na_align(uint32_t words) { return (words + 63u) & ~63u; } // 256-byte sub-buffers
constexpr uint32_t kNaCnt = 0;
constexpr uint32_t kNaOff = kNaCnt + na_align(kNoAllocMaxNodes);
constexpr uint32_t kNaCursor = kNaOff + na_align(kNoAllocMaxNodes + 1);
constexpr uint32_t kNaTiles = kNaCursor + na_align(kNoAllocMaxNodes);
constexpr uint32_t kNaLong = kNaTiles + na_align(kNoAllocTiles + 1);
constexpr uint32_t kNaMisc = kNaLong + na_align(kNoAllocMaxNodes);
constexpr uint32_t kNaSeg = kNaMisc + na_align(4);
constexpr uint32_t kNaWords = kNaSeg + na_align(kNoAllocMaxEdges);

static __device__ __align__(256) uint32_t g_merge_noalloc_scratch[kNaWords];

// Unique id of the calling thread's current CUDA context (cuCtxGetId, reached
// through the runtime's driver entry-point table so the library needs no
// libcuda link), or 0 when there is none yet or the driver lacks the call.
static unsigned long long current_context_id()
{
    using GetCurrent = CUresult (*)(CUcontext *);
    using GetId = CUresult (*)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Address of this device's copy of the scratch array.  It is looked up with
// cudaGetSymbolAddress (which loads the module on first use) at the first
// call on a device and again whenever that device's context has changed
// since, e.g. after cudaDeviceReset: a new context loads the module afresh
// and the array moves.
static int merge_noalloc_scratch(uint32_t **out)
{
    static std::mutex mu;
    static uint32_t *addr[64] = {};
    static unsigned long long ctx_of[64] = {};
    int dev = 0;
    DANCE_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64)
        return fail(-1, "device ordinal %d out of range for the merge scratch table", dev);
    std::lock_guard<std::mutex> lock(mu);
    const unsigned long long ctx = current_context_id();
    if (!addr[dev] || ctx == 0 || ctx != ctx_of[dev])
    {
        void *p = nullptr;
        DANCE_CUDA(cudaGetSymbolAddress(&p, g_merge_noalloc_scratch));
        addr[dev] = static_cast<uint32_t *>(p);
        ctx_of[dev] = current_context_id(); // the lookup made the device's context current
    }
    *out = addr[dev];
    return 0;
}

static int merge_bucket_noalloc(const uint32_t *d_src, const uint32_t *d_dst, uint64_t n_edges, uint32_t begin,
                                uint32_t count, uint32_t max_degree, uint64_t seed, uint32_t *d_out_neighbors,
                                uint32_t *d_out_degrees, cudaStream_t s)
{
    if (count == 0)
        return 0;
    uint32_t *base = nullptr;
    int rc = merge_noalloc_scratch(&base);
    if (rc)
        return rc;
    uint32_t *cnt = base + kNaCnt, *off = base + kNaOff, *cursor = base + kNaCursor, *tiles = base + kNaTiles;
    uint32_t *longl = base + kNaLong, *misc = base + kNaMisc, *seg = base + kNaSeg;
    const uint32_t ntiles = (count + kScanTile - 1) / kScanTile;
    // The counts and the two status words (long-segment count, error) must
    // start at zero; everything else is written before it is read.
    DANCE_CUDA(cudaMemsetAsync(cnt, 0, (uint64_t)count * 4, s));
    DANCE_CUDA(cudaMemsetAsync(misc, 0, 16, s));
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((n_edges + 255) / 256, sm_count() * 16ull));
    if (n_edges)
    {
        mrg_count_kernel<<<grid, 256, 0, s>>>(d_src, n_edges, begin, count, cnt);
        DANCE_LAUNCHED();
    }
    scan_tile_sums_kernel<<<ntiles, kScanThreads, 0, s>>>(cnt, count, tiles);
    DANCE_LAUNCHED();
    scan_tile_offsets_kernel<<<1, kScanThreads, 0, s>>>(tiles, ntiles);
    DANCE_LAUNCHED();
    scan_apply_kernel<<<ntiles, kScanThreads, 0, s>>>(cnt, count, tiles, off, cursor);
    DANCE_LAUNCHED();
    if (n_edges)
    {
        mrg_fill_kernel<<<grid, 256, 0, s>>>(d_src, d_dst, n_edges, begin, count, cursor, seg);
        DANCE_LAUNCHED();
    }
    MergeSelectParams mp{};
    mp.offsets = off;
    mp.seg = seg;
    mp.begin = begin;
    mp.count = count;
    mp.max_degree = max_degree;
    mp.seed = seed;
    mp.out_neighbors = d_out_neighbors;
    mp.out_degrees = d_out_degrees;
    mp.long_list = longl;
    mp.long_count = misc;
    mp.error = misc + 1;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mrg_select_kernel, 128, 0);
    const int g2 = (int)std::max<uint64_t>(1, std::min<uint64_t>((count + 3) / 4, (uint64_t)std::max(per_sm, 1) *
                                                                                       sm_count()));
    mrg_select_kernel<<<g2, 128, 0, s>>>(mp);
    DANCE_LAUNCHED();
    const size_t lsmem = 12u * kMergeBlockCap;
    DANCE_CUDA(allow_smem(mrg_select_long_kernel, lsmem));
    mrg_select_long_kernel<<<sm_count(), 256, lsmem, s>>>(mp);
    DANCE_LAUNCHED();
    uint32_t err = 0;
    DANCE_CUDA(cudaMemcpyAsync(&err, mp.error, 4, cudaMemcpyDeviceToHost, s));
    DANCE_CUDA(cudaStreamSynchronize(s));
    if (err)
        return fail(-20, "a source has %u merged edges, more than the %u supported per source", err, kMergeBlockCap);
    return 0;
}
} // namespace dance

extern "C" DANCE_API int dance_merge_edges_device_noalloc(const uint32_t *d_src, const uint32_t *d_dst,
                                                          uint64_t n_edges, uint32_t node_begin, uint32_t node_count,
                                                          uint32_t max_degree, uint64_t seed,
                                                          uint32_t *d_out_neighbors, uint32_t *d_out_degrees,
                                                          void *stream)
{
    if ((n_edges && (!d_src || !d_dst)) || !d_out_neighbors || !d_out_degrees || max_degree == 0)
        return fail(-1, "invalid merge arguments");
    if (node_count > kNoAllocMaxNodes || n_edges > kNoAllocMaxEdges)
        return fail(-5, "no-alloc merge holds at most %u sources and %u edges (asked for %u and %llu)",
                    kNoAllocMaxNodes, kNoAllocMaxEdges, node_count, (unsigned long long)n_edges);
    return merge_bucket_noalloc(d_src, d_dst, n_edges, node_begin, node_count, max_degree, seed, d_out_neighbors,
                                d_out_degrees, as_stream(stream));
}

namespace
{
struct ShardMeta
{
    std::string graph_path, idmap_path;
    std::vector<uint32_t> idmap;
    uint32_t width = 0, medoid = 0;
    uint64_t frozen = 0;
};

bool read_idmap(const std::string &path, std::vector<uint32_t> &out)
{
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in)
        return false;
    const uint64_t size = (uint64_t)in.tellg();
    in.seekg(0);
    uint32_t n = 0, d = 0;
    in.read(reinterpret_cast<char *>(&n), 4);
    in.read(reinterpret_cast<char *>(&d), 4);
    if (!in || d != 1 || size != 8 + 4ull * n)
        return false;
    out.resize(n);
    if (n)
        in.read(reinterpret_cast<char *>(out.data()), 4ull * n);
    return (bool)in;
}

bool read_header(std::ifstream &in, uint32_t &width, uint32_t &medoid, uint64_t &frozen)
{
    uint64_t size = 0;
    in.read(reinterpret_cast<char *>(&size), 8);
    in.read(reinterpret_cast<char *>(&width), 4);
    in.read(reinterpret_cast<char *>(&medoid), 4);
    in.read(reinterpret_cast<char *>(&frozen), 8);
    return (bool)in;
}

std::vector<int> merge_devices()
{
    std::vector<int> devs;
    const char *env = std::getenv("DISKANN_GPU_MERGE_DEVICES");
    if (env && *env)
    {
        std::stringstream ss(env);
        std::string tok;
        while (std::getline(ss, tok, ','))
            if (!tok.empty())
                devs.push_back(std::atoi(tok.c_str()));
    }
    if (devs.empty())
    {
        int cur = 0;
        cudaGetDevice(&cur);
        devs.push_back(cur);
    }
    return devs;
}

uint64_t env_u64(const char *name, uint64_t dflt)
{
    const char *e = std::getenv(name);
    return (e && *e) ? std::strtoull(e, nullptr, 10) : dflt;
}
} // namespace

namespace diskann
{

DANCE_API int merge_shards_gpu(const std::string &vamana_prefix, const std::string &vamana_suffix,
                               const std::string &idmaps_prefix, const std::string &idmaps_suffix, uint64_t nshards,
                               uint32_t max_degree, const std::string &output_vamana, const std::string &medoids_file)
{
    const std::vector<int> devices = merge_devices();
    if (devices.empty() || max_degree == 0)
        return -1;
    std::vector<ShardMeta> shards(nshards);
    uint64_t nnodes = 0, est_edges = 0;
    for (uint64_t i = 0; i < nshards; ++i)
    {
        ShardMeta &s = shards[i];
        s.graph_path = vamana_prefix + std::to_string(i) + vamana_suffix;
        s.idmap_path = idmaps_prefix + std::to_string(i) + idmaps_suffix;
        if (!read_idmap(s.idmap_path, s.idmap))
            return -2;
        for (uint32_t id : s.idmap)
            nnodes = std::max<uint64_t>(nnodes, (uint64_t)id + 1);
        std::ifstream in(s.graph_path, std::ios::binary);
        if (!read_header(in, s.width, s.medoid, s.frozen) || s.frozen != 0)
            return -3;
        if (s.medoid >= s.idmap.size())
            return -4;
        est_edges += (uint64_t)s.idmap.size() * s.width;
    }
    // buckets of sources sized for the device (each edge costs ~16 B on it)
    size_t free_b = 0, total_b = 0;
    cudaSetDevice(devices[0]);
    cudaMemGetInfo(&free_b, &total_b);
    uint64_t target = free_b > (8ull << 30) ? (free_b - (8ull << 30)) / 24 : (1ull << 24);
    target = std::max<uint64_t>(target, 1ull << 20);
    target = env_u64("DISKANN_GPU_MERGE_BUCKET_EDGES", target);
    uint64_t buckets = std::max<uint64_t>(1, (est_edges + target - 1) / target);
    buckets = env_u64("DISKANN_GPU_MERGE_BUCKETS", buckets);
    buckets = std::max<uint64_t>(1, std::min<uint64_t>(buckets, std::max<uint64_t>(1, nnodes)));
    auto bucket_of = [&](uint32_t src) { return std::min<uint64_t>(((uint64_t)src * buckets) / nnodes, buckets - 1); };
    auto bucket_begin = [&](uint64_t b) { return (uint32_t)((b * nnodes + buckets - 1) / buckets); };

    // pass 1: remap and bucket the edges in host memory (each shard file is
    // read whole, then parsed row by row)
    std::vector<std::vector<uint32_t>> bsrc(buckets), bdst(buckets);
    {
        const uint64_t per = est_edges / buckets + est_edges / (8 * buckets) + 1024;
        for (uint64_t b = 0; b < buckets; ++b)
        {
            bsrc[b].reserve(per);
            bdst[b].reserve(per);
        }
    }
    std::vector<uint32_t> body;
    for (uint64_t i = 0; i < nshards; ++i)
    {
        const ShardMeta &s = shards[i];
        std::ifstream in(s.graph_path, std::ios::binary | std::ios::ate);
        const uint64_t fbytes = (uint64_t)in.tellg();
        if (fbytes < 24 || (fbytes - 24) % 4 != 0)
            return -6;
        in.seekg(24);
        body.resize((fbytes - 24) / 4);
        if (!body.empty())
            in.read(reinterpret_cast<char *>(body.data()), fbytes - 24);
        if (!in)
            return -6;
        uint64_t pos = 0;
        const uint64_t nw = body.size();
        const uint32_t nloc = (uint32_t)s.idmap.size();
        for (uint32_t ls = 0; ls < nloc; ++ls)
        {
            const uint32_t gs = s.idmap[ls];
            if (pos >= nw)
                return -6;
            const uint32_t deg = body[pos++];
            if (deg > nw - pos)
                return -6;
            const uint64_t b = bucket_of(gs);
            std::vector<uint32_t> &vs = bsrc[b], &vd = bdst[b];
            for (uint32_t j = 0; j < deg; ++j)
            {
                const uint32_t ld = body[pos + j];
                if (ld >= nloc)
                    return -7;
                const uint32_t gd = s.idmap[ld];
                if (gd == gs)
                    continue;
                vs.push_back(gs);
                vd.push_back(gd);
            }
            pos += deg;
        }
    }
    std::vector<uint32_t>().swap(body);
    // medoids file
    {
        std::ofstream mw(medoids_file, std::ios::binary);
        if (!mw)
            return -10;
        const uint32_t ns = (uint32_t)nshards, one = 1;
        mw.write(reinterpret_cast<const char *>(&ns), 4);
        mw.write(reinterpret_cast<const char *>(&one), 4);
        for (uint64_t i = 0; i < nshards; ++i)
        {
            const uint32_t g = shards[i].idmap[shards[i].medoid];
            mw.write(reinterpret_cast<const char *>(&g), 4);
        }
        if (!mw)
            return -10;
    }
    const uint32_t out_medoid = nshards ? shards[nshards - 1].idmap[shards[nshards - 1].medoid] : 0;
    std::ofstream out(output_vamana, std::ios::binary | std::ios::trunc);
    if (!out)
        return -11;
    uint64_t size = 24;
    const uint64_t zero = 0;
    out.write(reinterpret_cast<const char *>(&size), 8);
    out.write(reinterpret_cast<const char *>(&max_degree), 4);
    out.write(reinterpret_cast<const char *>(&out_medoid), 4);
    out.write(reinterpret_cast<const char *>(&zero), 8);

    // pass 2: buckets on the devices, written back in node order
    const uint64_t seed = env_u64("DISKANN_GPU_MERGE_HASH_SEED", 0x9e3779b97f4a7c15ULL);
    std::vector<std::vector<uint32_t>> rows(buckets), degs(buckets);
    std::atomic<int> status{0};
    std::atomic<uint64_t> next{0};
    auto worker = [&](int dev) {
        if (cudaSetDevice(dev) != cudaSuccess)
        {
            status = -12;
            return;
        }
        while (status == 0)
        {
            const uint64_t b = next.fetch_add(1);
            if (b >= buckets)
                break;
            const uint32_t nb0 = bucket_begin(b), nb1 = bucket_begin(b + 1);
            const uint32_t cnt = nb1 - nb0;
            const uint64_t ne = bsrc[b].size();
            DevBuf ds, dd, on, od;
            if (ds.ensure(std::max<uint64_t>(ne, 1) * 4) || dd.ensure(std::max<uint64_t>(ne, 1) * 4) ||
                on.ensure(std::max<uint64_t>((uint64_t)cnt * max_degree, 1) * 4) ||
                od.ensure(std::max<uint64_t>(cnt, 1) * 4))
            {
                status = -14;
                return;
            }
            if (ne && (cudaMemcpy(ds.p, bsrc[b].data(), ne * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                       cudaMemcpy(dd.p, bdst[b].data(), ne * 4, cudaMemcpyHostToDevice) != cudaSuccess))
            {
                status = -15;
                return;
            }
            std::vector<uint32_t>().swap(bsrc[b]);
            std::vector<uint32_t>().swap(bdst[b]);
            const int rc = merge_bucket_device(ds.as<uint32_t>(), dd.as<uint32_t>(), ne, nb0, cnt, max_degree, seed,
                                               on.as<uint32_t>(), od.as<uint32_t>(), 0);
            if (rc)
            {
                status = rc == -20 ? -19 : -16;
                return;
            }
            rows[b].resize((uint64_t)cnt * max_degree);
            degs[b].resize(cnt);
            if (cnt && (cudaMemcpy(rows[b].data(), on.p, rows[b].size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
                        cudaMemcpy(degs[b].data(), od.p, degs[b].size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess))
            {
                status = -17;
                return;
            }
        }
    };
    int saved = 0;
    cudaGetDevice(&saved);
    if (devices.size() == 1)
        worker(devices[0]);
    else
    {
        std::vector<std::thread> th;
        for (int d : devices)
            th.emplace_back(worker, d);
        for (auto &t : th)
            t.join();
    }
    cudaSetDevice(saved);
    if (status != 0)
        return status;
    std::vector<uint32_t> packed;
    for (uint64_t b = 0; b < buckets; ++b)
    {
        const uint32_t cnt = bucket_begin(b + 1) - bucket_begin(b);
        packed.clear();
        packed.reserve((uint64_t)cnt * (max_degree + 1));
        for (uint32_t l = 0; l < cnt; ++l)
        {
            const uint32_t d = degs[b][l];
            if (d > max_degree)
                return -19;
            packed.push_back(d);
            const uint32_t *r = rows[b].data() + (uint64_t)l * max_degree;
            packed.insert(packed.end(), r, r + d);
        }
        out.write(reinterpret_cast<const char *>(packed.data()), 4ull * packed.size());
        size += 4ull * packed.size();
        std::vector<uint32_t>().swap(rows[b]);
        std::vector<uint32_t>().swap(degs[b]);
    }
    out.seekp(0);
    out.write(reinterpret_cast<const char *>(&size), 8);
    out.close();
    return out ? 0 : -11;
}

} // namespace diskann

extern "C" DANCE_API int dance_merge_shards_gpu(const char *vamana_prefix, const char *vamana_suffix,
                                                const char *idmaps_prefix, const char *idmaps_suffix,
                                                uint64_t nshards, uint32_t max_degree, const char *output_vamana,
                                                const char *medoids_file)
{
    if (!vamana_prefix || !vamana_suffix || !idmaps_prefix || !idmaps_suffix || !output_vamana || !medoids_file)
        return -1;
    return diskann::merge_shards_gpu(vamana_prefix, vamana_suffix, idmaps_prefix, idmaps_suffix, nshards, max_degree,
                                     output_vamana, medoids_file);
}
