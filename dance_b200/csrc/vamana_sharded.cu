// vamana_sharded.cu -- the standard build sharded over the GPUs of one box.
//
// The reference has no multi-GPU build of one graph (its only multi-GPU
// modes are independent shard builds on host threads, integration patch
// lines 3376-3600, and round-robin merge buckets, src/gpu_merge.cu:643-650).
// Here one process per GPU owns the contiguous vertex range
// [rank*chunk, min(N, (rank+1)*chunk)), chunk = ceil(N / world); vectors and
// the current graph are replicated.  Each round:
//   search + insert replay of own vertices  (reads the replicated graph)
//   every edge of the own work rows (first R slots) goes to the rank that
//   owns its target: per-owner counts, an all-gather of the world x world
//   count matrix, grouped ncclSend/ncclRecv of (target, source) pairs
//   reverse CSR of the received edges + merge (local)
//   prune own vertices into rows [v0, v1) of the graph, ncclAllGather the
//   graph and degrees (in place) for the next round.
// Every rank runs the same kernels as the one-GPU build on the same inputs,
// so the graph is bit-identical to it.  The communicator is non-blocking:
// every wait on NCCL or on the build stream is bounded by the communicator's
// timeout, after which the communicator is aborted and -4 is returned.

#include "comm.cuh"

namespace dance
{

// Events recorded on the build stream at stage boundaries; the time between
// consecutive marks is charged to the stage of the later mark.
enum ShardStage
{
    kStMedoidInit = 0,
    kStSearch,
    kStReplay,
    kStEdgeExchange,
    kStReverse,
    kStPrune,
    kStGraphExchange,
    kStCount
};

struct StageClock
{
    std::vector<cudaEvent_t> ev;
    std::vector<int> stage;
    ~StageClock()
    {
        for (auto e : ev)
            cudaEventDestroy(e);
    }
    int mark(int st, cudaStream_t s)
    {
        cudaEvent_t e = nullptr;
        DANCE_CUDA(cudaEventCreate(&e));
        ev.push_back(e);
        stage.push_back(st);
        DANCE_CUDA(cudaEventRecord(e, s));
        return 0;
    }
    void sum(double *acc) const // acc[kStCount], seconds
    {
        for (size_t i = 1; i < ev.size(); ++i)
        {
            float ms = 0;
            if (cudaEventElapsedTime(&ms, ev[i - 1], ev[i]) == cudaSuccess)
                acc[stage[i]] += ms * 1e-3;
        }
    }
    double total() const
    {
        float ms = 0;
        if (ev.size() >= 2 && cudaEventElapsedTime(&ms, ev.front(), ev.back()) == cudaSuccess)
            return ms * 1e-3;
        return 0;
    }
};

thread_local DanceShardedReport g_sharded_report;

// In-place all-gather of rows [rank*chunk, (rank+1)*chunk) of a table with
// `width` uint32 per row.
static int allgather_rows(DanceComm *c, uint32_t *table, uint64_t chunk, uint64_t width, cudaStream_t s)
{
    const uint64_t count = chunk * width;
    DANCE_NCCL(ncclAllGather(table + (uint64_t)c->rank * count, table, count, ncclUint32, c->comm, s));
    return nccl_settle(c, deadline_of(c));
}

// ---------------------------------------------------------------- edge exchange
// Every reverse edge (s -> t) of a round goes from the rank that owns s to
// the rank that owns t, as a pair (t - owner's first vertex, s).  Edges are
// the first min(work degree, R) slots of the own work rows with t < N and
// t != s -- the edges the one-GPU reverse CSR counts.
constexpr int kMaxWorld = 64;
constexpr int kXchThreads = 256;
constexpr int kXchItems = 8; // edges per thread and tile

__device__ __forceinline__ bool xch_edge(const uint32_t *work_ids, const uint32_t *work_deg, uint32_t C, uint32_t R,
                                         uint32_t N, uint32_t v0, uint64_t e, uint32_t &src, uint32_t &t)
{
    const uint64_t lv = e / R;
    const uint32_t slot = (uint32_t)(e % R);
    src = v0 + (uint32_t)lv;
    if (slot >= min(work_deg[lv], R))
        return false;
    t = work_ids[lv * C + slot];
    return t < N && t != src;
}

static __global__ void __launch_bounds__(kXchThreads) xch_count_kernel(const uint32_t *work_ids,
                                                                       const uint32_t *work_deg, uint32_t C,
                                                                       uint32_t R, uint32_t N, uint32_t v0,
                                                                       uint32_t nloc, uint32_t chunk, int world,
                                                                       uint32_t *counts)
{
    __shared__ uint32_t sc[kMaxWorld];
    for (int i = threadIdx.x; i < world; i += blockDim.x)
        sc[i] = 0;
    __syncthreads();
    const uint64_t total = (uint64_t)nloc * R;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x)
    {
        uint32_t src, t;
        if (xch_edge(work_ids, work_deg, C, R, N, v0, e, src, t))
            atomicAdd(&sc[t / chunk], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < world; i += blockDim.x)
        if (sc[i])
            atomicAdd(&counts[i], sc[i]);
}

// Tiles of kXchThreads * kXchItems edges: positions inside the tile come from
// shared-memory counters, each tile reserves its range per owner with one
// global atomic, then every edge is written to its owner's bucket.
static __global__ void __launch_bounds__(kXchThreads) xch_fill_kernel(const uint32_t *work_ids,
                                                                      const uint32_t *work_deg, uint32_t C, uint32_t R,
                                                                      uint32_t N, uint32_t v0, uint32_t nloc,
                                                                      uint32_t chunk, int world,
                                                                      const uint32_t *send_off, uint32_t *cursor,
                                                                      uint2 *send)
{
    __shared__ uint32_t sc[kMaxWorld], sbase[kMaxWorld];
    const uint64_t total = (uint64_t)nloc * R;
    const uint64_t tile = (uint64_t)kXchThreads * kXchItems;
    for (uint64_t t0 = blockIdx.x * tile; t0 < total; t0 += (uint64_t)gridDim.x * tile)
    {
        for (int i = threadIdx.x; i < world; i += blockDim.x)
            sc[i] = 0;
        __syncthreads();
        uint32_t owner[kXchItems], pos[kXchItems], tl[kXchItems], sv[kXchItems];
#pragma unroll
        for (int k = 0; k < kXchItems; ++k)
        {
            const uint64_t e = t0 + (uint64_t)k * kXchThreads + threadIdx.x;
            uint32_t src = 0, t = 0;
            owner[k] = 0xFFFFFFFFu;
            if (e < total && xch_edge(work_ids, work_deg, C, R, N, v0, e, src, t))
            {
                owner[k] = t / chunk;
                tl[k] = t - owner[k] * chunk;
                sv[k] = src;
                pos[k] = atomicAdd(&sc[owner[k]], 1u);
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < world; i += blockDim.x)
            sbase[i] = sc[i] ? send_off[i] + atomicAdd(&cursor[i], sc[i]) : 0u;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kXchItems; ++k)
            if (owner[k] != 0xFFFFFFFFu)
                send[sbase[owner[k]] + pos[k]] = make_uint2(tl[k], sv[k]);
        __syncthreads();
    }
}

static __global__ void rev_count_pairs_kernel(const uint2 *pairs, uint64_t n, uint32_t *cnt)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        atomicAdd(&cnt[pairs[i].x], 1u);
}

static __global__ void rev_fill_pairs_kernel(const uint2 *pairs, uint64_t n, uint32_t *cursor, uint32_t *rev)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint2 p = pairs[i];
        rev[atomicAdd(&cursor[p.x], 1u)] = p.y;
    }
}

// Sends every own edge to the owner of its target and builds the reverse
// CSR of the own targets [v0, v0 + nloc) from what arrives: counts by
// owner, an all-gather of the world x world count matrix, grouped
// ncclSend/ncclRecv of (target, source) pairs, then count / scan / fill.
static int exchange_edges(DanceComm *c, DanceWorkspace &ws, uint32_t N, uint32_t R, uint32_t C, uint32_t v0,
                          uint32_t nloc, uint32_t chunk, cudaStream_t s, uint64_t &sent_bytes, uint64_t &recv_bytes)
{
    const int W = c->world, me = c->rank;
    const uint32_t *work_ids = ws.work_ids.as<uint32_t>();
    const uint32_t *work_deg = ws.work_deg.as<uint32_t>();
    DANCE_CUDA(ws.xcnt.ensure((uint64_t)W * 4));
    DANCE_CUDA(ws.xmat.ensure((uint64_t)W * W * 4));
    DANCE_CUDA(ws.xoff.ensure((uint64_t)W * 4));
    DANCE_CUDA(ws.xcur.ensure((uint64_t)W * 4));
    DANCE_CUDA(cudaMemsetAsync(ws.xcnt.p, 0, (uint64_t)W * 4, s));
    const uint64_t total = (uint64_t)nloc * R;
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((total + kXchThreads - 1) / kXchThreads,
                                                                    (uint64_t)sm_count() * 8));
    if (total)
    {
        xch_count_kernel<<<grid, kXchThreads, 0, s>>>(work_ids, work_deg, C, R, N, v0, nloc, chunk, W,
                                                      ws.xcnt.as<uint32_t>());
        DANCE_LAUNCHED();
    }
    DANCE_NCCL(ncclAllGather(ws.xcnt.as<uint32_t>(), ws.xmat.as<uint32_t>(), (size_t)W, ncclUint32, c->comm, s));
    int rc = nccl_settle(c, deadline_of(c));
    if (rc)
        return rc;
    std::vector<uint32_t> mat((size_t)W * W);
    DANCE_CUDA(cudaMemcpyAsync(mat.data(), ws.xmat.p, (uint64_t)W * W * 4, cudaMemcpyDeviceToHost, s));
    if ((rc = stream_wait(c, s, deadline_of(c))))
        return rc;
    // row r of mat: what rank r sends to each owner
    std::vector<uint32_t> send_off(W + 1, 0), recv_off(W + 1, 0);
    for (int o = 0; o < W; ++o)
        send_off[o + 1] = send_off[o] + mat[(size_t)me * W + o];
    for (int r = 0; r < W; ++r)
        recv_off[r + 1] = recv_off[r] + mat[(size_t)r * W + me];
    const uint64_t nsend = send_off[W], nrecv = recv_off[W];
    DANCE_CUDA(ws.xsend.ensure(std::max<uint64_t>(nsend, 1) * 8));
    DANCE_CUDA(ws.xrecv.ensure(std::max<uint64_t>(nrecv, 1) * 8));
    DANCE_CUDA(ws.rev.ensure(std::max<uint64_t>(nrecv, 1) * 4));
    DANCE_CUDA(cudaMemcpyAsync(ws.xoff.p, send_off.data(), (uint64_t)W * 4, cudaMemcpyHostToDevice, s));
    DANCE_CUDA(cudaMemsetAsync(ws.xcur.p, 0, (uint64_t)W * 4, s));
    uint2 *send = ws.xsend.as<uint2>(), *recv = ws.xrecv.as<uint2>();
    if (total)
    {
        const uint64_t tiles = (total + (uint64_t)kXchThreads * kXchItems - 1) / ((uint64_t)kXchThreads * kXchItems);
        xch_fill_kernel<<<(int)std::max<uint64_t>(1, std::min<uint64_t>(tiles, (uint64_t)sm_count() * 8)),
                          kXchThreads, 0, s>>>(work_ids, work_deg, C, R, N, v0, nloc, chunk, W,
                                               ws.xoff.as<uint32_t>(), ws.xcur.as<uint32_t>(), send);
        DANCE_LAUNCHED();
    }
    const uint32_t own = mat[(size_t)me * W + me];
    if (own)
        DANCE_CUDA(cudaMemcpyAsync(recv + recv_off[me], send + send_off[me], (uint64_t)own * 8,
                                   cudaMemcpyDeviceToDevice, s));
    DANCE_NCCL(ncclGroupStart());
    for (int o = 0; o < W; ++o)
    {
        if (o == me)
            continue;
        const uint32_t ns = mat[(size_t)me * W + o], nr = mat[(size_t)o * W + me];
        if (ns)
            DANCE_NCCL(ncclSend(send + send_off[o], (size_t)ns * 2, ncclUint32, o, c->comm, s));
        if (nr)
            DANCE_NCCL(ncclRecv(recv + recv_off[o], (size_t)nr * 2, ncclUint32, o, c->comm, s));
    }
    DANCE_NCCL(ncclGroupEnd());
    if ((rc = nccl_settle(c, deadline_of(c))))
        return rc;
    sent_bytes += (nsend - own) * 8 + (uint64_t)W * 4;
    recv_bytes += (nrecv - own) * 8 + (uint64_t)W * W * 4;
    // reverse CSR of the own targets from the pairs that arrived
    DANCE_CUDA(cudaMemsetAsync(ws.rev_cnt.p, 0, (uint64_t)nloc * 4, s));
    const int g2 = (int)std::max<uint64_t>(1, std::min<uint64_t>((nrecv + 255) / 256, (uint64_t)sm_count() * 16));
    if (nrecv)
    {
        rev_count_pairs_kernel<<<g2, 256, 0, s>>>(recv, nrecv, ws.rev_cnt.as<uint32_t>());
        DANCE_LAUNCHED();
    }
    const uint32_t ntiles = (nloc + kScanTile - 1) / kScanTile;
    if (ntiles > 0)
    {
        scan_tile_sums_kernel<<<ntiles, kScanThreads, 0, s>>>(ws.rev_cnt.as<uint32_t>(), nloc, ws.tiles.as<uint32_t>());
        DANCE_LAUNCHED();
        scan_tile_offsets_kernel<<<1, kScanThreads, 0, s>>>(ws.tiles.as<uint32_t>(), ntiles);
        DANCE_LAUNCHED();
        scan_apply_kernel<<<ntiles, kScanThreads, 0, s>>>(ws.rev_cnt.as<uint32_t>(), nloc, ws.tiles.as<uint32_t>(),
                                                          ws.rev_off.as<uint32_t>(), ws.rev_cursor.as<uint32_t>());
        DANCE_LAUNCHED();
    }
    if (nrecv)
    {
        rev_fill_pairs_kernel<<<g2, 256, 0, s>>>(recv, nrecv, ws.rev_cursor.as<uint32_t>(), ws.rev.as<uint32_t>());
        DANCE_LAUNCHED();
    }
    return 0;
}

} // namespace dance

extern "C" {

DANCE_API void dance_shard_range(uint32_t num_points, int world, int rank, uint32_t *v0, uint32_t *v1, uint32_t *chunk)
{
    const uint32_t ch = world > 0 ? (uint32_t)((num_points + (uint32_t)world - 1u) / (uint32_t)world) : num_points;
    uint64_t a = (uint64_t)ch * (uint32_t)rank;
    uint64_t b = a + ch;
    if (a > num_points)
        a = num_points;
    if (b > num_points)
        b = num_points;
    if (v0)
        *v0 = (uint32_t)a;
    if (v1)
        *v1 = (uint32_t)b;
    if (chunk)
        *chunk = ch;
}

DANCE_API int dance_nccl_unique_id(uint8_t *out, size_t out_bytes)
{
    if (!out || out_bytes < sizeof(ncclUniqueId))
        return fail(-1, "unique id buffer must hold %zu bytes", sizeof(ncclUniqueId));
    ncclUniqueId id;
    DANCE_NCCL(ncclGetUniqueId(&id));
    std::memcpy(out, &id, sizeof(id));
    return 0;
}

DANCE_API int dance_comm_create(int rank, int world, const uint8_t *unique_id, size_t id_bytes, double timeout_s,
                                DanceComm **out)
{
    if (!out || !unique_id || id_bytes < sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world ||
        timeout_s <= 0)
        return fail(-1, "invalid communicator arguments");
    DanceComm *c = new DanceComm();
    c->rank = rank;
    c->world = world;
    c->timeout_s = timeout_s;
    cudaGetDevice(&c->device);
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->comm, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress)
    {
        delete c;
        return fail(-3, "ncclCommInitRankConfig: %s", ncclGetErrorString(r));
    }
    int rc = nccl_settle(c, deadline_of(c));
    if (rc)
    {
        if (!c->aborted && c->comm)
            ncclCommAbort(c->comm);
        delete c;
        return rc;
    }
    *out = c;
    return 0;
}

DANCE_API void dance_comm_destroy(DanceComm *c)
{
    if (!c)
        return;
    if (c->comm && !c->aborted)
    {
        ncclCommFinalize(c->comm);
        nccl_settle(c, deadline_of(c));
        if (!c->aborted)
            ncclCommDestroy(c->comm);
    }
    delete c;
}

DANCE_API int dance_vamana_build_sharded(DanceComm *comm, int dtype, const void *d_data, uint64_t stride,
                                         uint32_t N, uint32_t dim, uint32_t R, uint32_t L, uint32_t C,
                                         uint32_t STEPS, const DanceVamanaParams *params, DanceWorkspace *ws,
                                         uint32_t *d_graph, uint32_t *d_degree, uint32_t *d_table_degree,
                                         uint32_t *medoid_out, void *stream)
{
    if (!comm || comm->aborted)
        return fail(-1, "communicator missing or aborted");
    int rc = check_store(dtype, d_data, stride, N, dim);
    if (rc)
        return rc;
    if (!d_graph || !d_degree || !d_table_degree)
        return fail(-1, "null graph buffers");
    if (comm->world > kMaxWorld)
        return fail(-1, "at most %d ranks", kMaxWorld);
    if (R == 0 || L == 0 || C == 0 || STEPS == 0 || C < R || C > 1024 || L > (uint32_t)kMaxL)
        return fail(-1, "invalid parameters: R=%u L=%u C=%u STEPS=%u", R, L, C, STEPS);
    if (STEPS > L)
        STEPS = L;
    DanceVamanaParams prm;
    if (params)
        prm = *params;
    else
        dance_vamana_default_params(&prm);
    if (prm.iters == 0 || prm.visited_log2 < 8 || prm.visited_log2 > 16)
        return fail(-1, "invalid params");
    uint32_t v0, v1, chunk;
    dance_shard_range(N, comm->world, comm->rank, &v0, &v1, &chunk);
    const uint32_t nloc = v1 - v0;
    DanceWorkspace *own = nullptr;
    if (!ws)
    {
        own = new DanceWorkspace();
        cudaGetDevice(&own->device);
        rc = own->reserve(N, R, L, C, std::min(STEPS, L), std::max<uint32_t>(chunk, 1u), false);
        if (rc)
        {
            delete own;
            return rc;
        }
        ws = own;
    }
    struct Owner
    {
        DanceWorkspace *p;
        ~Owner() { delete p; }
    } owner{own};
    if (ws->N < N || ws->Local < chunk || ws->R != R || ws->C != C || ws->S < std::min(STEPS, L))
        return fail(-1, "workspace too small for the shard");
    cudaStream_t s = as_stream(stream);
    const StoreView st = make_view(d_data, stride, N, dim, dtype);
    uint32_t *cur_ids = d_graph;   // (world * chunk) x R, replicated
    uint32_t *degree = d_degree;   // world * chunk, replicated
    (void)d_table_degree; // kept in the signature; the edge exchange no longer needs a gathered table
    float *cur_dists = ws->cur_dists.as<float>(); // own rows only
    DANCE_CUDA(cudaMemsetAsync(ws->counters.p, 0, 64, s));
    StageClock clk;
    uint64_t edge_sent = 0, edge_recv = 0, graph_recv = 0;
    const uint64_t peer_rows = (uint64_t)chunk * (uint64_t)(comm->world - 1);
    if ((rc = clk.mark(kStMedoidInit, s)))
        return rc;

    // medoid: every rank computes the same entry point
    const uint32_t nc = std::min<uint32_t>(prm.medoid_candidates, std::min<uint32_t>(N, 4096u));
    const uint32_t ns = std::min<uint32_t>(prm.medoid_samples, N);
    uint32_t *d_medoid = ws->medoid.as<uint32_t>();
    if (nc > 0 && ns > 0)
    {
        rc = dispatch<LaunchMedoid>(dtype, st.nchunks, st, nc, ns, ws->med_scores.as<float>(),
                                    ws->med_cand.as<uint32_t>(), d_medoid, s);
        if (rc)
            return rc;
    }
    else
        DANCE_CUDA(cudaMemsetAsync(d_medoid, 0, 4, s));
    if (nloc)
    {
        rc = dispatch<LaunchInit>(dtype, st.nchunks, st, R, cur_ids, cur_dists, degree, v0, v1, v0, s);
        if (rc)
            return rc;
    }
    if ((rc = allgather_rows(comm, cur_ids, chunk, R, s)) || (rc = allgather_rows(comm, degree, chunk, 1, s)))
        return rc;
    graph_recv += peer_rows * (R + 1) * 4;
    if ((rc = clk.mark(kStMedoidInit, s)))
        return rc;
    const uint32_t mask_vertices = nloc ? replay_mask_vertices(dtype, st.nchunks, R, ws->S, C, nloc) : 0u;
    if (mask_vertices)
        DANCE_CUDA(ws->replay_masks.ensure(replay_mask_bytes(mask_vertices, ws->S)));

    for (uint32_t it = 0; it < prm.iters; ++it)
    {
        const float alpha = (it + 1 >= prm.iters) ? prm.alpha : 1.0f;
        const uint32_t steps = steps_for_round(it, STEPS, prm);
        if (nloc)
        {
            SearchParams sp{};
            sp.st = st;
            sp.R = R;
            sp.L = L;
            sp.Lcap = lcap_of(L);
            sp.steps = steps;
            sp.seeds = std::min<uint32_t>(prm.init_random_seeds, 31u);
            sp.log2h = prm.visited_log2;
            sp.entry_ptr = d_medoid;
            sp.cur_ids = cur_ids;
            sp.cur_dists = cur_dists;
            sp.degree = degree;
            sp.exp_ids = ws->exp_ids.as<uint32_t>();
            sp.exp_dists = ws->exp_dists.as<float>();
            sp.exp_count = ws->exp_count.as<uint32_t>();
            sp.exp_stride = ws->S;
            sp.v0 = v0;
            sp.v1 = v1;
            sp.lrow0 = v0;
            sp.counters = ws->counters.as<unsigned long long>();
            if ((rc = dispatch<LaunchSearch>(dtype, st.nchunks, sp, s)))
                return rc;
            if ((rc = clk.mark(kStSearch, s)))
                return rc;
            ReplayParams rp{};
            rp.st = st;
            rp.R = R;
            rp.C = C;
            rp.alpha = alpha;
            rp.cur_ids = cur_ids;
            rp.cur_dists = cur_dists;
            rp.degree = degree;
            rp.exp_ids = sp.exp_ids;
            rp.exp_dists = sp.exp_dists;
            rp.exp_count = sp.exp_count;
            rp.exp_stride = ws->S;
            rp.work_ids = ws->work_ids.as<uint32_t>();
            rp.work_dists = ws->work_dists.as<float>();
            rp.work_deg = ws->work_deg.as<uint32_t>();
            rp.v0 = v0;
            rp.v1 = v1;
            rp.lrow0 = v0;
            rp.row_bytes = st.nchunks * 16;
            rp.cache_rows = R + ws->S;
            rp.counters = sp.counters;
            rp.masks = mask_vertices ? ws->replay_masks.as<uint32_t>() : nullptr;
            rp.mask_vertices = mask_vertices;
            if ((rc = dispatch<LaunchReplay>(dtype, st.nchunks, rp, s)))
                return rc;
        }
        if ((rc = clk.mark(kStReplay, s)))
            return rc;
        if ((rc = exchange_edges(comm, *ws, N, R, C, v0, nloc, chunk, s, edge_sent, edge_recv)))
            return rc;
        if ((rc = clk.mark(kStEdgeExchange, s)))
            return rc;
        if (nloc)
        {
            rc = merge_from_csr(dtype, st, C, prm, *ws, ws->work_ids.as<uint32_t>(), ws->work_dists.as<float>(),
                                ws->work_deg.as<uint32_t>(), v0, v1, s);
            if (rc)
                return rc;
            if ((rc = clk.mark(kStReverse, s)))
                return rc;
            PruneParams pp{};
            pp.st = st;
            pp.R = R;
            pp.C = C;
            pp.alpha = alpha;
            pp.min_degree = (it + 1 == prm.iters) ? prm.final_min_degree : 0u;
            pp.work_ids = ws->work_ids.as<uint32_t>();
            pp.work_dists = ws->work_dists.as<float>();
            pp.work_deg = ws->work_deg.as<uint32_t>();
            pp.cur_ids = cur_ids;
            pp.cur_dists = cur_dists;
            pp.degree = degree;
            pp.v0 = v0;
            pp.v1 = v1;
            pp.lrow0 = v0;
            pp.row_bytes = st.nchunks * 16;
            pp.counters = ws->counters.as<unsigned long long>();
            if ((rc = dispatch<LaunchPrune>(dtype, st.nchunks, pp, s)))
                return rc;
        }
        if ((rc = clk.mark(kStPrune, s)))
            return rc;
        if ((rc = allgather_rows(comm, cur_ids, chunk, R, s)) || (rc = allgather_rows(comm, degree, chunk, 1, s)))
            return rc;
        graph_recv += peer_rows * (R + 1) * 4;
        if ((rc = clk.mark(kStGraphExchange, s)))
            return rc;
        if ((rc = stream_wait(comm, s, deadline_of(comm))))
            return rc;
    }
    if (medoid_out)
        DANCE_CUDA(cudaMemcpyAsync(medoid_out, d_medoid, 4, cudaMemcpyDeviceToHost, s));
    if ((rc = clk.mark(kStGraphExchange, s)))
        return rc;
    if ((rc = stream_wait(comm, s, deadline_of(comm))))
        return rc;
    if ((rc = replay_umma_status())) // after the last collective: no rank is left waiting
        return rc;
    double acc[kStCount] = {0};
    clk.sum(acc);
    DanceShardedReport &sr = g_sharded_report;
    std::memset(&sr, 0, sizeof(sr));
    sr.medoid_init_seconds = acc[kStMedoidInit];
    sr.search_seconds = acc[kStSearch];
    sr.replay_seconds = acc[kStReplay];
    sr.edge_exchange_seconds = acc[kStEdgeExchange];
    sr.reverse_seconds = acc[kStReverse];
    sr.prune_seconds = acc[kStPrune];
    sr.graph_exchange_seconds = acc[kStGraphExchange];
    sr.total_seconds = clk.total();
    sr.edge_bytes_sent = edge_sent;
    sr.edge_bytes_received = edge_recv;
    sr.graph_bytes_received = graph_recv;
    sr.rounds = prm.iters;
    DanceBuildReport &r = g_report;
    std::memset(&r, 0, sizeof(r));
    r.total_seconds = sr.total_seconds;
    r.medoid_seconds = sr.medoid_init_seconds;
    r.search_kernel_seconds = sr.search_seconds;
    r.search_seconds = sr.search_seconds + sr.replay_seconds;
    r.replay_seconds = sr.replay_seconds;
    r.reverse_seconds = sr.edge_exchange_seconds + sr.reverse_seconds;
    r.prune_seconds = sr.prune_seconds + sr.graph_exchange_seconds;
    uint64_t ctr[8] = {0};
    DANCE_CUDA(cudaMemcpy(ctr, ws->counters.p, 64, cudaMemcpyDeviceToHost));
    r.search_evals = ctr[0];
    r.expansions = ctr[1];
    r.replay_pairs = ctr[2];
    r.reverse_evals = ctr[3];
    r.prune_pairs = ctr[4];
    return 0;
}

DANCE_API int dance_last_sharded_report(DanceShardedReport *report)
{
    if (!report)
        return fail(-1, "null report");
    *report = g_sharded_report;
    return 0;
}

DANCE_API int dance_workspace_create_sharded(uint32_t num_points, int world, uint32_t R, uint32_t L, uint32_t C,
                                             uint32_t STEPS, DanceWorkspace **out)
{
    if (!out || num_points == 0 || world < 1 || R == 0 || L == 0 || C == 0 || STEPS == 0 || C < R)
        return fail(-1, "invalid workspace shape");
    uint32_t chunk;
    dance_shard_range(num_points, world, 0, nullptr, nullptr, &chunk);
    DanceWorkspace *ws = new DanceWorkspace();
    cudaGetDevice(&ws->device);
    int rc = ws->reserve(num_points, R, L, C, std::min(STEPS, L), std::max<uint32_t>(chunk, 1u), false);
    if (rc)
    {
        delete ws;
        return rc;
    }
    *out = ws;
    return 0;
}

} // extern "C"
