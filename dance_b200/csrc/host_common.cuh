// host_common.cuh -- host-side plumbing shared by the single-GPU build
// (vamana_build.cu) and the NCCL-sharded build (vamana_sharded.cu): error
// reporting, device buffers, dtype/width dispatch, kernel launchers, the
// per-build workspace and the reverse-CSR + merge driver.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/dance_b200.h"
#include "../../include/gpu_vamana_builder.h"
#include "../../include/gpu_vamana_config.h"
#include "vamana_kernels.cuh"
#include "gram_u8.cuh"
#include "prune_quad.cuh"
#include "replay_umma.cuh"

namespace dance
{

// ---------------------------------------------------------------- errors
extern thread_local char g_err[512];
extern std::atomic<uint64_t> g_launches;
extern thread_local DanceBuildReport g_report; // last resident or sharded build

inline int fail(int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    fprintf(stderr, "[dance_b200] %s\n", g_err);
    return code;
}

#define DANCE_CUDA(call)                                                                                        \
    do                                                                                                          \
    {                                                                                                           \
        cudaError_t e__ = (call);                                                                               \
        if (e__ != cudaSuccess)                                                                                 \
            return fail(-2, "CUDA error %s at %s:%d (%s)", cudaGetErrorString(e__), __FILE__, __LINE__, #call); \
    } while (0)

#define DANCE_LAUNCHED()                                                                                        \
    do                                                                                                          \
    {                                                                                                           \
        g_launches.fetch_add(1, std::memory_order_relaxed);                                                    \
        cudaError_t e__ = cudaGetLastError();                                                                   \
        if (e__ != cudaSuccess)                                                                                 \
            return fail(-2, "kernel launch failed: %s at %s:%d", cudaGetErrorString(e__), __FILE__, __LINE__);  \
    } while (0)

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------- device buffer
struct DevBuf
{
    void *p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    ~DevBuf() { release(); }
    void release()
    {
        if (p)
            cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    cudaError_t ensure(size_t b)
    {
        if (b <= bytes && p)
            return cudaSuccess;
        release();
        cudaError_t e = cudaMalloc(&p, b ? b : 16);
        if (e == cudaSuccess)
            bytes = b;
        return e;
    }
    template <class T>
    T *as() const
    {
        return reinterpret_cast<T *>(p);
    }
};

inline int elem_size(int dtype)
{
    switch (dtype)
    {
    case kU8:
        return 1;
    case kF16:
        return 2;
    case kF32:
        return 4;
    default:
        return 0;
    }
}

inline int sm_count()
{
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 1;
}

// One wave of resident blocks (a multiple of the SM count), or fewer when
// there is less work than that.
template <class K>
inline int wave_grid(K kernel, int threads, size_t smem, uint64_t work_warps)
{
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (per_sm < 1)
        per_sm = 1;
    const uint64_t wave = (uint64_t)per_sm * sm_count();
    const uint64_t need = (work_warps + (threads / 32) - 1) / (threads / 32);
    uint64_t g = need < wave ? need : wave;
    return (int)(g ? g : 1);
}

template <class K>
inline cudaError_t allow_smem(K kernel, size_t smem)
{
    if (smem <= 48 * 1024)
        return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

inline int max_optin_smem()
{
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return v;
}

// ---------------------------------------------------------------- CPL dispatch
// Chunks (16 bytes) per group lane; instantiated widths cover rows up to
// 1024 bytes (f32 dim <= 256, f16 <= 512, u8 <= 1024).
template <template <int, int> class F, int DT, class... A>
inline int dispatch_cpl(uint32_t nchunks, A &&...args)
{
    const uint32_t cpl = (nchunks + 7) / 8;
    if (cpl <= 1)
        return F<DT, 1>::run(args...);
    if (cpl <= 2)
        return F<DT, 2>::run(args...);
    if (cpl <= 3)
        return F<DT, 3>::run(args...);
    if (cpl <= 4)
        return F<DT, 4>::run(args...);
    if (cpl <= 8)
        return F<DT, 8>::run(args...);
    return fail(-1, "row of %u bytes exceeds the 1024-byte limit of this build", nchunks * 16);
}

template <template <int, int> class F, class... A>
inline int dispatch(int dtype, uint32_t nchunks, A &&...args)
{
    switch (dtype)
    {
    case kU8:
        return dispatch_cpl<F, kU8>(nchunks, args...);
    case kF16:
        return dispatch_cpl<F, kF16>(nchunks, args...);
    case kF32:
        return dispatch_cpl<F, kF32>(nchunks, args...);
    default:
        return fail(-1, "unknown dtype %d", dtype);
    }
}

// ---------------------------------------------------------------- launchers
template <int DT, int CPL>
struct LaunchMedoid
{
    static int run(const StoreView &st, uint32_t nc, uint32_t ns, float *scores, uint32_t *cand, uint32_t *medoid,
                   cudaStream_t s)
    {
        const int blocks = (int)((nc + kWarpsPerBlock - 1) / kWarpsPerBlock);
        medoid_score_kernel<DT, CPL><<<blocks, kBlockThreads, 0, s>>>(st, nc, ns, scores, cand);
        DANCE_LAUNCHED();
        medoid_argmin_kernel<<<1, 1024, 0, s>>>(scores, cand, nc, medoid);
        DANCE_LAUNCHED();
        return 0;
    }
};

template <int DT, int CPL>
struct LaunchInit
{
    static int run(const StoreView &st, uint32_t R, uint32_t *ids, float *dists, uint32_t *deg, uint32_t v0,
                   uint32_t v1, uint32_t lrow0, cudaStream_t s)
    {
        auto k = init_graph_kernel<DT, CPL>;
        const int grid = wave_grid(k, kBlockThreads, 0, v1 - v0);
        k<<<grid, kBlockThreads, 0, s>>>(st, R, ids, dists, deg, v0, v1, lrow0);
        DANCE_LAUNCHED();
        return 0;
    }
};

template <int DT, int CPL>
struct LaunchSearch
{
    static int run(const SearchParams &p, cudaStream_t s)
    {
        auto k = search_kernel<DT, CPL>;
        const size_t smem = (size_t)search_smem_per_warp(p.Lcap, p.log2h) * kWarpsPerBlock;
        if ((int)smem > max_optin_smem())
            return fail(-1, "search scratch %zu B exceeds shared memory (L=%u, visited 2^%u)", smem, p.L, p.log2h);
        DANCE_CUDA(allow_smem(k, smem));
        const int grid = wave_grid(k, kBlockThreads, smem, p.v1 - p.v0);
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }
};

template <int DT, int CPL>
struct LaunchQuery
{
    static int run(const QueryParams &p, cudaStream_t s)
    {
        auto k = query_search_kernel<DT, CPL>;
        const size_t smem = (size_t)search_smem_per_warp(p.Lcap, p.log2h) * kWarpsPerBlock;
        if ((int)smem > max_optin_smem())
            return fail(-1, "query scratch %zu B exceeds shared memory", smem);
        DANCE_CUDA(allow_smem(k, smem));
        const int grid = wave_grid(k, kBlockThreads, smem, p.nq);
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }
};

// uint8 replay on the tcgen05 tensor cores (replay_umma.cuh) for rows of at
// most 128 bytes, at most 128 cached rows (R + STEPS) and C <= 128; the
// same graph as replay_kernel.  DANCE_REPLAY_UMMA=0 at the call selects the
// pair-by-pair replay_kernel instead.
constexpr uint32_t kReplayMaskChunk = 1u << 20; // vertices per masks/bits pass

inline bool replay_umma_enabled()
{
    const char *e = getenv("DANCE_REPLAY_UMMA");
    return !(e && e[0] == '0');
}

inline bool replay_umma_fits(int dtype, uint32_t nchunks, uint32_t R, uint32_t S, uint32_t C)
{
    return dtype == kU8 && nchunks <= 8 && R + S <= kUmmaRows && C <= kUmmaRows && replay_umma_enabled();
}

// Mask buffer for a replay over `nverts` vertices (0 when the tensor-core
// replay does not apply), and its vertex capacity.
inline uint32_t replay_mask_vertices(int dtype, uint32_t nchunks, uint32_t R, uint32_t S, uint32_t C,
                                     uint32_t nverts)
{
    if (!replay_umma_fits(dtype, nchunks, R, S, C))
        return 0;
    // DANCE_REPLAY_MASK_CHUNK (vertices) shrinks the chunk, e.g. to test the
    // chunk loop on small inputs
    uint32_t chunk = kReplayMaskChunk;
    if (const char *e = getenv("DANCE_REPLAY_MASK_CHUNK"))
    {
        const unsigned long v = strtoul(e, nullptr, 10);
        if (v > 0 && v < chunk)
            chunk = (uint32_t)v;
    }
    return std::max(1u, std::min(nverts, chunk));
}

inline uint64_t replay_mask_bytes(uint32_t vertices, uint32_t S) { return (uint64_t)vertices * S * kMaskWords * 4u; }

inline int launch_replay_umma(ReplayParams p, cudaStream_t s)
{
    auto ka = replay_masks_kernel<1>;
    const uint32_t kch = umma_kchunks(p.st.nchunks);
    // at least 50 KB per block: at most four blocks (4 x 128 tensor-memory
    // columns) share an SM, so no allocation has to wait
    const size_t smem_a =
        std::max<size_t>((size_t)UmmaMaskLayout(p.R, p.exp_stride, kch).bytes * kWarpsPerBlock, 50u * 1024u);
    DANCE_CUDA(cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_a));
    DANCE_CUDA(cudaFuncSetAttribute(ka, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    (int)cudaSharedmemCarveoutMaxShared));
    // resident blocks per SM from the shared memory and registers they take
    // (the occupancy query does not account for the carveout set above), at
    // most four for the tensor memory
    int dev = 0, smem_sm = 0, regs_sm = 0;
    DANCE_CUDA(cudaGetDevice(&dev));
    DANCE_CUDA(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    DANCE_CUDA(cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev));
    cudaFuncAttributes fa{};
    DANCE_CUDA(cudaFuncGetAttributes(&fa, ka));
    const size_t per_block = smem_a + fa.sharedSizeBytes + 1024; // + the driver's reserve per block
    const int by_smem = (int)((size_t)smem_sm / per_block);
    const int by_regs = regs_sm / std::max(1, ((fa.numRegs + 7) / 8 * 8) * kBlockThreads);
    const uint64_t per_sm = (uint64_t)std::max(1, std::min(4, std::min(by_smem, by_regs)));
    auto kb = replay_bits_kernel;
    const size_t smem_b = (size_t)UmmaBitsLayout(p.C, p.exp_stride).bytes * kWarpsPerBlock;
    DANCE_CUDA(allow_smem(kb, smem_b));
    for (uint32_t c0 = p.v0; c0 < p.v1; c0 += p.mask_vertices)
    {
        const uint32_t c1 = c0 + std::min(p.mask_vertices, p.v1 - c0);
        const uint64_t batches = (c1 - c0 + kWarpsPerBlock - 1) / kWarpsPerBlock;
        const int grid_a = (int)std::max<uint64_t>(1, std::min<uint64_t>(batches, per_sm * sm_count()));
        ka<<<grid_a, kBlockThreads, smem_a, s>>>(p, c0, c1);
        DANCE_LAUNCHED();
        const int grid_b = wave_grid(kb, kBlockThreads, smem_b, c1 - c0);
        kb<<<grid_b, kBlockThreads, smem_b, s>>>(p, c0, c1);
        DANCE_LAUNCHED();
    }
    return 0;
}

// Reads and clears the tensor-core replay's timeout counter (after the
// stream has been synchronised).
inline int replay_umma_status()
{
    unsigned int t = 0;
    DANCE_CUDA(cudaMemcpyFromSymbol(&t, g_replay_umma_timeouts, sizeof(t)));
    if (t)
    {
        const unsigned int z = 0;
        DANCE_CUDA(cudaMemcpyToSymbol(g_replay_umma_timeouts, &z, sizeof(z)));
        return fail(-4, "tensor-core replay: %u blocks timed out waiting for the MMA", t);
    }
    return 0;
}

template <int DT, int CPL>
struct LaunchReplay
{
    static int run(ReplayParams p, cudaStream_t s)
    {
        if constexpr (DT == kU8 && CPL == 1)
        {
            if (p.masks && p.mask_vertices && replay_umma_fits(DT, p.st.nchunks, p.R, p.exp_stride, p.C))
                return launch_replay_umma(p, s);
        }
        auto k = replay_kernel<DT, CPL>;
        p.per_warp = align16(replay_smem_per_warp(p.C, p.cache_rows, p.row_bytes, p.exp_stride));
        const size_t smem = (size_t)p.per_warp * kWarpsPerBlock;
        if ((int)smem > max_optin_smem())
            return fail(-1, "replay vector cache %zu B exceeds shared memory (R+steps=%u rows of %u B)", smem,
                        p.cache_rows, p.row_bytes);
        DANCE_CUDA(allow_smem(k, smem));
        const int grid = wave_grid(k, kBlockThreads, smem, p.v1 - p.v0);
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }
};

template <int DT, int CPL>
struct LaunchMerge
{
    // huge_blocks: blocks (and scratch slices) of the huge-segment kernel
    static int run(MergeParams p, int huge_blocks, cudaStream_t s)
    {
        auto k = merge_kernel<DT, CPL>;
        p.sort_cap = kMergeSortCap;
        p.Cp = std::max<uint32_t>(32u, (uint32_t)next_pow2((int)p.C));
        p.per_warp = align16(merge_smem_per_warp(p.C, p.Cp, p.sort_cap));
        const size_t smem = (size_t)p.per_warp * kWarpsPerBlock;
        DANCE_CUDA(allow_smem(k, smem));
        const int grid = wave_grid(k, kBlockThreads, smem, p.t1 - p.t0);
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        auto hk = heavy_merge_kernel<DT, CPL>;
        const size_t hsmem = 4u * kHeavySortCap + block_merge_smem_bytes(p.C, p.Cp);
        DANCE_CUDA(allow_smem(hk, hsmem));
        hk<<<sm_count(), kMergeBlock, hsmem, s>>>(p);
        DANCE_LAUNCHED();
        auto gk = huge_merge_kernel<DT, CPL>;
        const size_t gsmem = block_merge_smem_bytes(p.C, p.Cp);
        DANCE_CUDA(allow_smem(gk, gsmem));
        gk<<<huge_blocks, kMergeBlock, gsmem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }
};

template <int DT, int CPL>
struct LaunchPrune
{
    static int run(PruneParams p, cudaStream_t s)
    {
        if constexpr (DT == kU8)
            return run_gram(p, s);
        else
        {
            if (CPL <= 4 && p.C <= 128)
                return run_quad(p, s);
        }
        auto k = prune_kernel<DT, CPL>;
        p.Cp = (uint32_t)next_pow2((int)p.C);
        if (p.Cp < 32)
            p.Cp = 32;
        p.per_warp = align16(prune_smem_per_warp(p.C, p.Cp, p.R, p.row_bytes));
        const size_t smem = (size_t)p.per_warp * kWarpsPerBlock;
        if ((int)smem > max_optin_smem())
            return fail(-1, "prune vector cache %zu B exceeds shared memory", smem);
        DANCE_CUDA(allow_smem(k, smem));
        const int grid = wave_grid(k, kBlockThreads, smem, p.v1 - p.v0);
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }

    // float / half rows of up to 32 chunks: eight pairs per pass
    static int run_quad(PruneParams p, cudaStream_t s)
    {
        auto k = prune_quad_kernel<DT, (CPL <= 4 ? 2 * CPL : 2)>;
        p.Cp = (uint32_t)next_pow2((int)p.C);
        if (p.Cp < 32)
            p.Cp = 32;
        p.per_warp = align16(QuadPruneLayout(p.C, p.row_bytes).bytes);
        const size_t smem = (size_t)p.per_warp * kWarpsPerBlock;
        if ((int)smem > max_optin_smem())
            return fail(-1, "prune vector cache %zu B exceeds shared memory", smem);
        DANCE_CUDA(allow_smem(k, smem));
        const int grid = wave_grid(k, kBlockThreads, smem, p.v1 - p.v0);
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }

    // uint8: occlusion predicates from the tensor-core Gram matrix
    static int run_gram(PruneParams p, cudaStream_t s)
    {
        auto k = prune_gram_kernel<CPL>;
        p.Cp = (uint32_t)next_pow2((int)p.C);
        if (p.Cp < 32)
            p.Cp = 32;
        const GramPruneLayout lay(p.C, p.row_bytes);
        if (lay.staging > lay.rows * gram_stride(p.row_bytes))
            return fail(-1, "prune staging %u B exceeds the vector cache", lay.staging);
        p.per_warp = align16(lay.bytes);
        const size_t smem = (size_t)p.per_warp * kWarpsPerBlock;
        if ((int)smem > max_optin_smem())
            return fail(-1, "prune vector cache %zu B exceeds shared memory", smem);
        DANCE_CUDA(allow_smem(k, smem));
        const int grid = wave_grid(k, kBlockThreads, smem, p.v1 - p.v0);
        k<<<grid, kBlockThreads, smem, s>>>(p);
        DANCE_LAUNCHED();
        return 0;
    }
};

// ---------------------------------------------------------------- validation
inline int check_store(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim)
{
    const int es = elem_size(dtype);
    if (!es)
        return fail(-1, "unknown dtype %d", dtype);
    if (!d_data || N == 0 || dim == 0)
        return fail(-1, "null data or empty store (N=%u dim=%u)", N, dim);
    if (stride % 16 != 0 || stride < (uint64_t)dim * es)
        return fail(-1, "row stride %llu must be a multiple of 16 and hold dim*%d bytes", (unsigned long long)stride,
                    es);
    if (dtype == kF16 && (dim & 1u))
        return fail(-1, "fp16 storage needs an even dimension (dim=%u)", dim);
    if ((reinterpret_cast<uintptr_t>(d_data) & 15u) != 0)
        return fail(-1, "vector store must be 16-byte aligned");
    return 0;
}

inline StoreView make_view(const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, int dtype)
{
    StoreView st;
    st.data = reinterpret_cast<const uint8_t *>(d_data);
    st.stride = stride;
    st.nchunks = (uint32_t)(((uint64_t)dim * elem_size(dtype) + 15u) / 16u);
    st.N = N;
    return st;
}

inline uint32_t lcap_of(uint32_t L) { return (L + 31u) & ~31u; }

// Float entry points store the vectors as fp16 when ENABLE_FLOAT16_BUILD is
// set at build time, or DANCE_FLOAT16_BUILD=0|1 at run time (the run-time
// variable wins), mirroring the reference's FAST profiles.
inline bool float16_build_enabled()
{
    const char *e = std::getenv("DANCE_FLOAT16_BUILD");
    if (e && *e)
        return std::atoi(e) != 0;
    return ENABLE_FLOAT16_BUILD != 0;
}

} // namespace dance

using namespace dance;

// ====================================================================== workspace
struct DanceWorkspace
{
    int device = 0;
    uint32_t N = 0, R = 0, L = 0, C = 0, S = 0, Local = 0;
    DevBuf cur_ids, cur_dists, degree;
    DevBuf work_ids, work_dists, work_deg;
    DevBuf exp_ids, exp_dists, exp_count;
    DevBuf rev_cnt, rev_off, rev_cursor, rev, tiles;
    DevBuf heavy_list, heavy_count, huge_list, huge_scratch;
    static constexpr int kHugeBlocks = 4;
    DevBuf med_scores, med_cand, medoid;
    DevBuf counters;
    DevBuf replay_masks; // uint8 tensor-core replay (one chunk of vertices)
    // sharded build: edge exchange (per-rank counts, send/receive pairs)
    DevBuf xcnt, xmat, xoff, xcur, xsend, xrecv;

    // n: vertices of the whole graph; local: vertices whose work rows,
    // expansion lists and own distance rows live here (n on one GPU, the
    // shard size when the build is sharded); graph: also allocate the N x R
    // graph and degrees (the sharded build uses the caller's buffers).
    int reserve(uint32_t n, uint32_t r, uint32_t l, uint32_t c, uint32_t s, uint32_t local = 0xFFFFFFFFu,
                bool graph = true)
    {
        if (local > n)
            local = n;
        N = n;
        R = r;
        L = l;
        C = c;
        S = s;
        Local = local;
        const uint64_t nr = (uint64_t)n * r;
        const uint64_t lr = (uint64_t)local * r, lc = (uint64_t)local * c, ls = (uint64_t)local * s;
        const uint64_t ntiles = (local + kScanTile - 1) / kScanTile + 1;
        if (graph)
        {
            DANCE_CUDA(cur_ids.ensure(nr * 4));
            DANCE_CUDA(degree.ensure((uint64_t)n * 4));
        }
        DANCE_CUDA(cur_dists.ensure(lr * 4));
        DANCE_CUDA(work_ids.ensure(lc * 4));
        DANCE_CUDA(work_dists.ensure(lc * 4));
        DANCE_CUDA(work_deg.ensure((uint64_t)local * 4));
        DANCE_CUDA(exp_ids.ensure(ls * 4));
        DANCE_CUDA(exp_dists.ensure(ls * 4));
        DANCE_CUDA(exp_count.ensure((uint64_t)local * 4));
        DANCE_CUDA(rev_cnt.ensure((uint64_t)local * 4));
        DANCE_CUDA(rev_off.ensure(((uint64_t)local + 1) * 4));
        DANCE_CUDA(rev_cursor.ensure((uint64_t)local * 4));
        // one GPU: every edge may target this GPU's vertices; sharded: the
        // exchange grows the array to the edges a round actually delivers
        DANCE_CUDA(rev.ensure((graph ? nr : lr) * 4));
        DANCE_CUDA(tiles.ensure(ntiles * 4));
        DANCE_CUDA(heavy_list.ensure((uint64_t)local * 4));
        DANCE_CUDA(heavy_count.ensure(16));
        DANCE_CUDA(huge_list.ensure((uint64_t)local * 4));
        const uint64_t huge_words = (uint64_t)kHugeBlocks * ((n + 1u) / 2u);
        if (!huge_scratch.p || huge_scratch.bytes < huge_words * 4)
        {
            DANCE_CUDA(huge_scratch.ensure(huge_words * 4));
            DANCE_CUDA(cudaMemset(huge_scratch.p, 0, huge_words * 4)); // counters stay zero between uses
        }
        DANCE_CUDA(med_scores.ensure(4096 * 4));
        DANCE_CUDA(med_cand.ensure(4096 * 4));
        DANCE_CUDA(medoid.ensure(16));
        DANCE_CUDA(counters.ensure(8 * 8));
        return 0;
    }
};

namespace dance
{

// Reverse CSR + merge.  Edges come from source rows [s0, s1) of an edge
// table (src_ids, row stride src_stride, degrees src_deg, first R slots);
// targets [t0, t1) are merged into the work rows, which are indexed by
// t - t0.  Sorting inside the merge kernels puts every target's sources in
// ascending order, so the merge is deterministic.
inline int merge_from_csr(int dtype, const StoreView &st, uint32_t C, const DanceVamanaParams &prm,
                          DanceWorkspace &ws, uint32_t *work_ids, float *work_dists, uint32_t *work_deg, uint32_t t0,
                          uint32_t t1, cudaStream_t s);

inline int reverse_merge_impl(int dtype, const StoreView &st, uint32_t R, uint32_t C, const DanceVamanaParams &prm,
                              DanceWorkspace &ws, const uint32_t *src_ids, uint64_t src_stride,
                              const uint32_t *src_deg, uint32_t s0, uint32_t s1, uint32_t *work_ids, float *work_dists,
                              uint32_t *work_deg, uint32_t t0, uint32_t t1, cudaStream_t s)
{
    const uint32_t N = st.N;
    const uint32_t nt = t1 - t0;
    DANCE_CUDA(cudaMemsetAsync(ws.rev_cnt.p, 0, (size_t)nt * 4, s));
    const uint64_t total = (uint64_t)(s1 - s0) * R;
    int grid = (int)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 16);
    if (grid < 1)
        grid = 1;
    rev_count_kernel<<<grid, 256, 0, s>>>(src_ids, src_stride, src_deg, N, R, s0, s1, t0, t1,
                                          ws.rev_cnt.as<uint32_t>());
    DANCE_LAUNCHED();
    const uint32_t ntiles = (nt + kScanTile - 1) / kScanTile;
    if (ntiles > 0)
    {
        scan_tile_sums_kernel<<<ntiles, kScanThreads, 0, s>>>(ws.rev_cnt.as<uint32_t>(), nt, ws.tiles.as<uint32_t>());
        DANCE_LAUNCHED();
        scan_tile_offsets_kernel<<<1, kScanThreads, 0, s>>>(ws.tiles.as<uint32_t>(), ntiles);
        DANCE_LAUNCHED();
        scan_apply_kernel<<<ntiles, kScanThreads, 0, s>>>(ws.rev_cnt.as<uint32_t>(), nt, ws.tiles.as<uint32_t>(),
                                                          ws.rev_off.as<uint32_t>(), ws.rev_cursor.as<uint32_t>());
        DANCE_LAUNCHED();
    }
    rev_fill_kernel<<<grid, 256, 0, s>>>(src_ids, src_stride, src_deg, N, R, s0, s1, t0, t1,
                                         ws.rev_cursor.as<uint32_t>(), ws.rev.as<uint32_t>());
    DANCE_LAUNCHED();
    return merge_from_csr(dtype, st, C, prm, ws, work_ids, work_dists, work_deg, t0, t1, s);
}

// Reverse merge of targets [t0, t1) from the CSR already in ws.rev_off /
// ws.rev (sources of target t at rev[rev_off[t - t0] .. rev_off[t - t0 + 1])).
inline int merge_from_csr(int dtype, const StoreView &st, uint32_t C, const DanceVamanaParams &prm,
                          DanceWorkspace &ws, uint32_t *work_ids, float *work_dists, uint32_t *work_deg, uint32_t t0,
                          uint32_t t1, cudaStream_t s)
{
    DANCE_CUDA(cudaMemsetAsync(ws.heavy_count.p, 0, 8, s)); // heavy and huge counts
    MergeParams mp{};
    mp.st = st;
    mp.C = C;
    mp.work_ids = work_ids;
    mp.work_dists = work_dists;
    mp.work_deg = work_deg;
    mp.offsets = ws.rev_off.as<uint32_t>();
    mp.rev = ws.rev.as<uint32_t>();
    mp.heavy_cap = prm.reverse_heavy_cap;
    mp.heavy_threshold = prm.reverse_heavy_threshold;
    mp.heavy_sample = prm.reverse_heavy_sample;
    mp.heavy_list = ws.heavy_list.as<uint32_t>();
    mp.heavy_count = ws.heavy_count.as<uint32_t>();
    mp.huge_list = ws.huge_list.as<uint32_t>();
    mp.huge_count = ws.heavy_count.as<uint32_t>() + 1;
    mp.huge_scratch = ws.huge_scratch.as<uint32_t>();
    mp.t0 = t0;
    mp.t1 = t1;
    mp.counters = ws.counters.as<unsigned long long>();
    return dispatch<LaunchMerge>(dtype, st.nchunks, mp, (int)DanceWorkspace::kHugeBlocks, s);
}

inline uint32_t steps_for_round(uint32_t it, uint32_t STEPS, const DanceVamanaParams &p)
{
    uint32_t steps = STEPS;
    if (it < p.coarse_warmup_iters && steps > p.warmup_expand_steps)
        steps = p.warmup_expand_steps;
    return steps;
}

// Device time per stage of one build (seconds), summed over rounds; the
// search stage includes the online-insert replay, as in the reference's
// search_online_insert_seconds.  search_kernel is the GreedySearch kernel
// alone, from events recorded right after each of its launches.
struct StageTimes
{
    double medoid = 0, search = 0, replay = 0, reverse = 0, prune = 0, total = 0, search_kernel = 0;
};

// The whole build on resident vectors.  graph_out/dists_out/degree_out may
// alias the workspace's own buffers.  Defined in vamana_build.cu.
int build_resident_impl(int dtype, const void *d_data, uint64_t stride, uint32_t N, uint32_t dim, uint32_t R,
                        uint32_t L, uint32_t C, uint32_t STEPS, const DanceVamanaParams &prm, DanceWorkspace &ws,
                        uint32_t *graph_out, uint32_t *degree_out, float *dists_out, uint32_t *medoid_out,
                        cudaStream_t s, StageTimes *times, uint64_t *counters_out);
} // namespace dance
