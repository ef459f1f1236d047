// replay_umma.cuh -- uint8 online-insert replay from a tensor-core Gram
// matrix (tcgen05.mma kind::i8, accumulator in tensor memory).
//
// The online RobustInsert of a vertex's expansion sequence (reference
// dynamic_robust_insert_C_warp, src/gpu_vamana_vnew2.cu:759-877; replay_kernel
// restates it pair by pair) only ever compares an expanded node x with
// vectors of the same vertex's candidate set: its initial neighbours and its
// expansions, at most 128 rows.  For uint8 vectors every pair distance is an
// exact integer, d(a, b) = |a|^2 + |b|^2 - 2 <a, b>, so the whole
// candidate-candidate block is one u8 x u8 -> s32 Gram matrix of the cached
// rows: one tcgen05.mma group (M = N = 128, K = 32 bytes per instruction)
// into tensor memory.  From it each expansion k gets two 128-bit masks over
// the cached rows (expansion k is row k, initial slot i is row S + i):
//   OCC[k]: rows y with d(v,y) <= d(v,x) and alpha*d(y,x) <= d(v,x)
//           (y occludes x), plus the rows holding x's own id (x present);
//   VIC[k]: rows y with d(v,y) > d(v,x) and alpha*d(x,y) <= d(v,y)
//           (x may replace y).
// The sequential rule then runs on bits: x is skipped if OCC[k] meets the
// kept set; otherwise it replaces the kept VIC[k] row of largest distance
// (lowest slot on ties), else is appended while the row has room, else
// replaces the worst kept row if closer -- replay_kernel's decisions.
//
// The default uint8 replay where it fits (host_common.cuh; DANCE_REPLAY_UMMA=0
// selects replay_kernel).  On the 10M uint8 build (R64 STEPS64 C80) the
// replay takes 0.85 s per build against 1.25 s for replay_kernel, graph
// bit-identical.
//
// Two kernels per chunk of vertices, so that the sequential part does not
// hold the tensor-memory block:
//   replay_masks_kernel  4 warps, one vertex per warp per batch: each warp
//     gathers its vertex's rows into shared memory in the canonical K-major
//     core-matrix layout (8 rows x 16 bytes per 128-byte core matrix, K
//     chunks 128 bytes apart); the four Grams pass through one 128-column
//     accumulator (thread 0 issues the MMAs and commits them to an
//     mbarrier, every warp reads its 32 accumulator lanes) and the lanes of
//     the expansion rows write OCC/VIC to a global mask buffer;
//   replay_bits_kernel   one warp per vertex, a few KB of shared memory:
//     the sequential insert on the masks.
// Waits on the mbarrier are bounded: on a timeout the block counts itself in
// g_replay_umma_timeouts and stops; the build then fails with status -4.
#pragma once

#include "vamana_kernels.cuh"

namespace dance
{

constexpr uint32_t kUmmaRows = 128;     // cached rows per vertex (M = N of the MMA)
constexpr uint32_t kUmmaTmemCols = 128; // s32 accumulator columns
constexpr uint32_t kUmmaWaitLimit = 1u << 24;
constexpr uint32_t kMaskWords = 8;      // OCC (4 words) + VIC (4 words) per expansion

// Blocks that gave up waiting for the tensor core (0 in a healthy run).
static __device__ unsigned int g_replay_umma_timeouts;

__host__ __device__ __forceinline__ uint32_t umma_kchunks(uint32_t nchunks) { return (nchunks + 1u) & ~1u; }

// Per-warp scratch of replay_masks_kernel: the core-matrix cache first.
struct UmmaMaskLayout
{
    uint32_t norms, dv, dup, xid, wid, bytes;
    __host__ __device__ UmmaMaskLayout(uint32_t R, uint32_t S, uint32_t kch)
    {
        uint32_t o = kUmmaRows * kch * 16u;
        norms = o;
        o += 4u * kUmmaRows;
        dv = o;
        o += 4u * kUmmaRows;
        dup = o;
        o += 16u * S;
        xid = o;
        o += align16(4u * S);
        wid = o;
        o += align16(4u * R);
        bytes = (o + 127u) & ~127u;
    }
};

// Per-warp scratch of replay_bits_kernel.
struct UmmaBitsLayout
{
    uint32_t dv, slot, wid, wd, xid, xdd, mk, bytes;
    __host__ __device__ UmmaBitsLayout(uint32_t C, uint32_t S)
    {
        uint32_t o = 0;
        dv = o;
        o += 4u * kUmmaRows;
        mk = o;
        o += 4u * kMaskWords * S;
        wid = o;
        o += align16(4u * C);
        wd = o;
        o += align16(4u * C);
        xid = o;
        o += align16(4u * S);
        xdd = o;
        o += align16(4u * S);
        slot = o;
        o += kUmmaRows;
        bytes = align16(o);
    }
};

// Byte offset of 16-byte chunk c of row r in the K-major no-swizzle layout.
__device__ __forceinline__ uint32_t umma_off(uint32_t r, uint32_t c, uint32_t kch)
{
    return (r >> 3) * (kch * 128u) + c * 128u + (r & 7u) * 16u;
}

// Shared-memory matrix descriptor (K-major, no swizzle): start address,
// leading byte offset (between the two 16-byte K chunks of one MMA), stride
// byte offset (between 8-row core-matrix groups), descriptor version 1.
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::i8: s32 accumulator, u8 A and B, both
// K-major, N = 128 (bits 17-22 hold N/8), M = 128 (bits 24-28 hold M/16).
constexpr uint32_t kUmmaIdescU8 = (2u << 4) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void umma_u8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
                 "l"(adesc), "l"(bdesc), "r"(kUmmaIdescU8), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint32_t mbar_saddr)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mbar_saddr)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t mbar_saddr, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(mbar_saddr), "r"(parity)
                 : "memory");
    return ok != 0;
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }

// 32 consecutive accumulator columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                 "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                 "[%32];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// Tensor memory for one block (one warp executes it) and its release.
__device__ __forceinline__ void tmem_alloc_cols(uint32_t *dst_smem, uint32_t cols)
{
    const uint32_t dst = (uint32_t)__cvta_generic_to_shared(dst_smem);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_free_cols(uint32_t taddr, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(cols) : "memory");
}

// OCC/VIC masks of the expansions of vertices [c0, c1) into
// masks[((v - c0) * S + k) * 8 ...].
template <int CPL>
__global__ void __launch_bounds__(kBlockThreads, 1) replay_masks_kernel(ReplayParams p, uint32_t c0, uint32_t c1)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t mbar;
    __shared__ uint32_t tmem_base_s;
    __shared__ uint32_t cnt_s[kWarpsPerBlock];
    __shared__ int abort_s;
    const int lane = lane_id(), warp = warp_id_in_block();
    const uint32_t R = p.R, S = p.exp_stride, N = p.st.N;
    const uint32_t nch = p.st.nchunks, kch = umma_kchunks(nch);
    const UmmaMaskLayout lay(R, S, kch);
    uint8_t *base = smem_raw + (uint32_t)warp * lay.bytes;
    uint8_t *cache = base;
    uint32_t *norms = reinterpret_cast<uint32_t *>(base + lay.norms);
    float *dv = reinterpret_cast<float *>(base + lay.dv);
    uint32_t *dup = reinterpret_cast<uint32_t *>(base + lay.dup);
    uint32_t *xid = reinterpret_cast<uint32_t *>(base + lay.xid);
    uint32_t *wid = reinterpret_cast<uint32_t *>(base + lay.wid);
    const uint32_t mbar_s = (uint32_t)__cvta_generic_to_shared(&mbar);
    const float alpha = p.alpha;

    if (warp == 0)
        tmem_alloc_cols(&tmem_base_s, kUmmaTmemCols);
    if (threadIdx.x == 0)
    {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(mbar_s) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        abort_s = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    uint32_t parity = 0;
    const uint32_t nbatch = (c1 - c0 + kWarpsPerBlock - 1) / kWarpsPerBlock;

    for (uint32_t bt = blockIdx.x; bt < nbatch; bt += gridDim.x)
    {
        // ---- each warp: its vertex's rows, norms, distances and duplicate-id bits
        const uint32_t v = c0 + bt * kWarpsPerBlock + (uint32_t)warp;
        uint32_t cnt = 0;
        if (v < c1)
        {
            const uint64_t lv = v - p.lrow0;
            const uint32_t deg_self = min(p.degree[v], R);
            cnt = min(p.exp_count[lv], S);
            for (uint32_t k = lane; k < cnt; k += 32)
            {
                xid[k] = p.exp_ids[lv * S + k];
                dv[k] = p.exp_dists[lv * S + k];
            }
            for (uint32_t i = lane; i < R; i += 32)
            {
                uint32_t nb = kInvalid;
                float d = FLT_MAX;
                if (i < deg_self)
                {
                    const uint32_t id = p.cur_ids[(uint64_t)v * R + i];
                    if (id < N && id != v)
                    {
                        nb = id;
                        d = p.cur_dists[lv * R + i];
                    }
                }
                wid[i] = nb;
                dv[S + i] = d;
            }
            __syncwarp();
            // rows: expansion k at row k, initial slot i at row S + i (an
            // invalid id's row is v's own; it is never kept)
            const uint32_t rows = cnt + deg_self;
            for (uint32_t e = lane; e < rows * kch; e += 32)
            {
                const uint32_t rr = e / kch, c = e - rr * kch;
                const uint32_t r = rr < cnt ? rr : S + (rr - cnt);
                uint32_t id = rr < cnt ? xid[rr] : wid[rr - cnt];
                id = id < N ? id : v;
                const uint32_t dst = (uint32_t)__cvta_generic_to_shared(cache + umma_off(r, c, kch));
                if (c < nch)
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst),
                                 "l"(p.st.data + (uint64_t)id * p.st.stride + 16u * c)
                                 : "memory");
                else
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};\n" ::"r"(dst), "r"(0u) : "memory");
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
            // x is already in the row when a kept row holds its id: the initial
            // slots and the earlier expansions with the same id
            for (uint32_t k = lane; k < cnt; k += 32)
            {
                const uint32_t x = xid[k];
                uint32_t b[4] = {0u, 0u, 0u, 0u};
                for (uint32_t i = 0; i < deg_self; ++i)
                    if (wid[i] == x)
                        b[(S + i) >> 5] |= 1u << ((S + i) & 31u);
                for (uint32_t j = 0; j < k; ++j)
                    if (xid[j] == x)
                        b[j >> 5] |= 1u << (j & 31u);
                *reinterpret_cast<uint4 *>(dup + 4u * k) = make_uint4(b[0], b[1], b[2], b[3]);
            }
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            __syncwarp();
            for (uint32_t rr = lane; rr < rows; rr += 32)
            {
                const uint32_t r = rr < cnt ? rr : S + (rr - cnt);
                uint32_t acc = 0;
                for (uint32_t c = 0; c < nch; ++c)
                {
                    const uint4 y = *reinterpret_cast<const uint4 *>(cache + umma_off(r, c, kch));
                    acc = __dp4a(y.x, y.x, acc);
                    acc = __dp4a(y.y, y.y, acc);
                    acc = __dp4a(y.z, y.z, acc);
                    acc = __dp4a(y.w, y.w, acc);
                }
                norms[r] = acc;
            }
        }
        if (lane == 0)
            cnt_s[warp] = cnt;
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        tc_fence_before();
        __syncthreads();

        // ---- the four Grams through one accumulator
        for (int w = 0; w < kWarpsPerBlock; ++w)
        {
            const uint32_t cw = cnt_s[w];
            if (cw == 0)
                continue;
            uint8_t *wb = smem_raw + (uint32_t)w * lay.bytes;
            if (threadIdx.x == 0)
            {
                tc_fence_after();
                const uint32_t a0 = (uint32_t)__cvta_generic_to_shared(wb);
                for (uint32_t ks = 0; ks < kch / 2; ++ks)
                {
                    const uint64_t d = umma_smem_desc(a0 + ks * 256u, 128u, kch * 128u);
                    umma_u8(tmem, d, d, ks > 0 ? 1u : 0u);
                }
                umma_commit(mbar_s);
            }
            bool done = false;
            for (uint32_t it = 0; it < kUmmaWaitLimit; ++it)
            {
                done = __all_sync(kFull, mbar_try_wait(mbar_s, parity));
                if (done)
                    break;
            }
            parity ^= 1u;
            if (!done)
            {
                if (lane == 0)
                    abort_s = 1;
            }
            else
            {
                tc_fence_after();
                if ((uint32_t)warp * 32u < cw)
                {
                    const uint32_t r = (uint32_t)warp * 32u + (uint32_t)lane; // this lane's expansion
                    const uint32_t *wn = reinterpret_cast<const uint32_t *>(wb + lay.norms);
                    const float *wdv = reinterpret_cast<const float *>(wb + lay.dv);
                    const uint32_t *wdup = reinterpret_cast<const uint32_t *>(wb + lay.dup);
                    const bool mine = r < cw;
                    const uint32_t nx = mine ? wn[r] : 0u;
                    const float dx = mine ? wdv[r] : 0.0f;
                    // expansion k only meets kept rows of earlier expansions
                    // (j < k) and of initial slots (S .. S + R): a column
                    // chunk of expansion rows at or beyond this warp's last
                    // expansion, or past the initial rows, stays zero
                    const uint32_t kend = min(cw, (uint32_t)warp * 32u + 32u);
                    uint32_t ob[4], vb[4];
#pragma unroll
                    for (uint32_t q = 0; q < 4; ++q)
                    {
                        ob[q] = 0u;
                        vb[q] = 0u;
                        const uint32_t c0q = 32u * q;
                        if ((c0q + 32u <= S && c0q + 1u >= kend) || c0q >= S + R)
                            continue; // warp-uniform
                        uint32_t g[32];
                        tmem_ld32(tmem + (((uint32_t)warp * 32u) << 16) + 32u * q, g);
                        uint32_t o = 0, vv = 0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                        {
                            const uint32_t u = 32u * q + (uint32_t)j;
                            const float d = (float)(int32_t)(nx + wn[u] - 2u * g[j]);
                            const float ad = __fmul_rn(alpha, d);
                            const float dy = wdv[u];
                            if (dy <= dx && ad <= dx)
                                o |= 1u << j;
                            if (dy > dx && ad <= dy)
                                vv |= 1u << j;
                        }
                        ob[q] = o;
                        vb[q] = vv;
                    }
                    if (mine)
                    {
                        const uint4 dd = *reinterpret_cast<const uint4 *>(wdup + 4u * r);
                        const uint32_t vw = c0 + bt * kWarpsPerBlock + (uint32_t)w;
                        uint4 *dst = reinterpret_cast<uint4 *>(p.masks + ((uint64_t)(vw - c0) * S + r) * kMaskWords);
                        dst[0] = make_uint4(ob[0] | dd.x, ob[1] | dd.y, ob[2] | dd.z, ob[3] | dd.w);
                        dst[1] = make_uint4(vb[0], vb[1], vb[2], vb[3]);
                    }
                }
            }
            tc_fence_before();
            __syncthreads();
            if (abort_s)
                break;
        }
        if (abort_s)
            break;
    }

    if (abort_s && threadIdx.x == 0)
        atomicAdd(&g_replay_umma_timeouts, 1u);
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
    {
        tc_fence_after();
        tmem_free_cols(tmem, kUmmaTmemCols);
    }
}

// Kept row with the smallest order_key (largest distance, lowest slot):
// keys carry the row in their low byte; kept word j sits in lane j.
__device__ __forceinline__ uint32_t umma_worst_row(uint32_t keptw, const float *dv, const uint8_t *slot_of,
                                                   int lane)
{
    uint64_t best = kKeyMax;
#pragma unroll
    for (int j = 0; j < 4; ++j)
    {
        const uint32_t w = __shfl_sync(kFull, keptw, j);
        const uint32_t r = 32u * (uint32_t)j + (uint32_t)lane;
        if ((w >> lane) & 1u)
        {
            const uint64_t k = (((uint64_t)(~__float_as_uint(dv[r]))) << 32) | ((uint64_t)slot_of[r] << 8) | r;
            best = k < best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
    {
        const uint64_t other = __shfl_xor_sync(kFull, best, o);
        best = other < best ? other : best;
    }
    return (uint32_t)(best & 0xFFu);
}

// The sequential insert of vertices [c0, c1) on their masks, one warp per
// vertex.
static __global__ void __launch_bounds__(kBlockThreads) replay_bits_kernel(ReplayParams p, uint32_t c0, uint32_t c1)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int lane = lane_id(), warp = warp_id_in_block();
    const uint32_t C = p.C, R = p.R, S = p.exp_stride, N = p.st.N;
    const UmmaBitsLayout lay(C, S);
    uint8_t *base = smem_raw + (uint32_t)warp * lay.bytes;
    float *dv = reinterpret_cast<float *>(base + lay.dv);
    uint32_t *mk = reinterpret_cast<uint32_t *>(base + lay.mk);
    uint32_t *wid = reinterpret_cast<uint32_t *>(base + lay.wid);
    float *wd = reinterpret_cast<float *>(base + lay.wd);
    uint32_t *xid = reinterpret_cast<uint32_t *>(base + lay.xid);
    float *xdd = reinterpret_cast<float *>(base + lay.xdd);
    uint8_t *slot_of = base + lay.slot;
    unsigned long long pairs = 0;

    for (uint32_t v = c0 + blockIdx.x * kWarpsPerBlock + (uint32_t)warp; v < c1; v += gridDim.x * kWarpsPerBlock)
    {
        const uint64_t lv = v - p.lrow0;
        const uint32_t deg_self = min(p.degree[v], R);
        const uint32_t cnt = min(p.exp_count[lv], S);
        for (uint32_t k = lane; k < cnt; k += 32)
        {
            const float dx = p.exp_dists[lv * S + k];
            xid[k] = p.exp_ids[lv * S + k];
            xdd[k] = dx;
            dv[k] = dx;
        }
        for (uint32_t i = lane; i < C; i += 32)
        {
            uint32_t nb = kInvalid;
            float d = FLT_MAX;
            if (i < deg_self)
            {
                const uint32_t id = p.cur_ids[(uint64_t)v * R + i];
                if (id < N && id != v)
                {
                    nb = id;
                    d = p.cur_dists[lv * R + i];
                }
            }
            wid[i] = nb;
            wd[i] = d;
            if (i < R)
            {
                dv[S + i] = d;
                slot_of[S + i] = (uint8_t)i;
            }
        }
        const uint4 *src = reinterpret_cast<const uint4 *>(p.masks + (uint64_t)(v - c0) * S * kMaskWords);
        for (uint32_t e = lane; e < 2u * cnt; e += 32)
            reinterpret_cast<uint4 *>(mk)[e] = src[e];
        __syncwarp();
        uint32_t keptw = 0; // word `lane` of the kept-row set (lanes 0..3)
        for (uint32_t i = 0; i < deg_self; ++i)
            if (wid[i] != kInvalid && (uint32_t)lane == ((S + i) >> 5))
                keptw |= 1u << ((S + i) & 31u);
        int nv = __popc(__shfl_sync(kFull, keptw, 0)) + __popc(__shfl_sync(kFull, keptw, 1)) +
                 __popc(__shfl_sync(kFull, keptw, 2)) + __popc(__shfl_sync(kFull, keptw, 3));
        uint32_t wdeg = deg_self;
        for (uint32_t k = 0; k < cnt; ++k)
        {
            const uint32_t x = xid[k];
            if (x >= N || x == v)
                continue;
            const float dx = xdd[k];
            const uint32_t deg = min(wdeg, C);
            const uint32_t ow = lane < 4 ? mk[kMaskWords * k + lane] & keptw : 0u;
            if (__any_sync(kFull, ow != 0u))
                continue;
            const uint32_t vw = lane < 4 ? mk[kMaskWords * k + 4 + lane] & keptw : 0u;
            int slot = -1, prow = -1;
            if (__any_sync(kFull, vw != 0u))
            {
                prow = (int)umma_worst_row(vw, dv, slot_of, lane);
                slot = slot_of[prow];
            }
            else if (deg < C)
            {
                slot = (int)deg;
                wdeg = deg + 1;
            }
            else if (nv > 0)
            {
                const uint32_t r0 = umma_worst_row(keptw, dv, slot_of, lane);
                if (dx < dv[r0])
                {
                    prow = (int)r0;
                    slot = slot_of[r0];
                }
            }
            if (slot < 0)
                continue;
            if (prow >= 0)
            {
                if ((uint32_t)lane == ((uint32_t)prow >> 5))
                    keptw &= ~(1u << (prow & 31));
            }
            else
                ++nv;
            if ((uint32_t)lane == (k >> 5))
                keptw |= 1u << (k & 31u);
            __syncwarp();
            if (lane == 0)
            {
                slot_of[k] = (uint8_t)slot;
                wid[slot] = x;
                wd[slot] = dx;
            }
            __syncwarp();
        }
        for (uint32_t i = lane; i < C; i += 32)
        {
            p.work_ids[lv * C + i] = wid[i];
            p.work_dists[lv * C + i] = wd[i];
        }
        if (lane == 0)
        {
            p.work_deg[lv] = wdeg;
            pairs += (unsigned long long)cnt * (cnt + deg_self);
        }
        __syncwarp();
    }
    if (lane == 0 && p.counters)
        atomicAdd(&p.counters[2], pairs);
}

} // namespace dance
