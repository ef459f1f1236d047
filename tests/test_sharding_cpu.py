"""The sharded build's exchange schedule, checked on CPU with two gloo ranks.

Each rank owns [v0, v1) (dance_shard_range) and must be able to finish the
build from its own rows plus what the GPU path all-gathers each round:
the first R slots of every work row with its degree (before the reverse
merge) and every pruned graph row with its degree (after the prune).  Rows a
rank does not own are overwritten with garbage before every exchange, so a
missing exchange changes the result.  The stages are the oracle's.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
R, L, C, S, N = 16, 32, 24, 16, 1200


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _garble(a, v0, v1, rng):
    out = a.copy()
    mask = np.ones(len(a), bool)
    mask[v0:v1] = False
    if out.dtype == np.float32:
        out[mask] = rng.random(out[mask].shape).astype(np.float32)
    else:
        out[mask] = rng.integers(0, 2**31, out[mask].shape).astype(out.dtype)
    return out


def _gather_rows(a, v0, v1, chunk, world):
    """all_gather of own rows (padded to chunk) as the GPU path does."""
    pad = np.zeros((chunk,) + a.shape[1:], a.dtype)
    pad[:v1 - v0] = a[v0:v1]
    t = torch.from_numpy(pad.view(np.int32) if a.dtype == np.uint32 else pad)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    full = torch.cat(parts).numpy()
    if a.dtype == np.uint32:
        full = full.view(np.uint32)
    return full[:len(a)].copy()


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["ORACLE_THREADS"] = "2"
    import oracle
    from dance_b200 import workloads
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(100 + rank)
        x = workloads.clustered_u8(N, 32, centroids=12, seed=9).numpy()
        chunk = (N + world - 1) // world
        v0, v1 = min(N, rank * chunk), min(N, (rank + 1) * chunk)
        m, _, _ = oracle.medoid(x)
        ids, ds, deg = oracle.init(x, R)
        ids, deg = _gather_rows(_garble(ids, v0, v1, rng), v0, v1, chunk, world), \
            _gather_rows(_garble(deg, v0, v1, rng), v0, v1, chunk, world)
        ds = _garble(ds, v0, v1, rng)  # own distance rows stay local
        for it in range(4):
            alpha = np.float32(1.2) if it == 3 else np.float32(1.0)
            e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
            wid, wd, wdeg = oracle.replay(x, R, C, alpha, ids, ds, deg, *e)
            table = _gather_rows(_garble(wid[:, :R].copy(), v0, v1, rng), v0, v1, chunk, world)
            tdeg = _gather_rows(_garble(wdeg, v0, v1, rng), v0, v1, chunk, world)
            full = _garble(wid, v0, v1, rng)
            full[:, :R] = table  # sources come from the gathered table only
            fd = _garble(wd, v0, v1, rng)
            fdeg = tdeg.copy()
            fdeg[v0:v1] = wdeg[v0:v1]
            mw = oracle.reverse_merge(x, R, C, full, fd, fdeg)[:3]
            nids, nds, ndeg = oracle.prune(x, R, C, alpha, 64 if it == 3 else 0, *mw)
            ids = _gather_rows(_garble(nids, v0, v1, rng), v0, v1, chunk, world)
            deg = _gather_rows(_garble(ndeg, v0, v1, rng), v0, v1, chunk, world)
            ds = _garble(nds, v0, v1, rng)
        if rank == 0:
            g, gdeg, _, gm = oracle.build_graph(x, R, L, C, S)
            q.put(bool(np.array_equal(ids, g) and np.array_equal(deg, gdeg) and gm == m))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_sharded_schedule_matches_single_process_build():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=280)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def test_shard_ranges_cover_all_vertices(dance_lib):
    from dance_b200 import vamana
    for n, w in [(10, 3), (1, 4), (7, 8), (10_000_000, 8), (1000, 1)]:
        seen = []
        for r in range(w):
            a, b, c = vamana.shard_range(n, w, r)
            assert c == (n + w - 1) // w and a <= b and b - a <= c
            seen.extend(range(a, b)) if n < 100000 else seen.append((a, b))
        if n < 100000:
            assert seen == list(range(n))
        else:
            assert seen[0][0] == 0 and seen[-1][1] == n and all(seen[i][1] == seen[i + 1][0] for i in range(w - 1))
