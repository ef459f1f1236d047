"""Sharded disk-index pipeline: k-means partition, shard builds, merge.

The partition restates DiskANN's partitioner (integration patch lines
20629-20688), which the reference repository does not contain, so parity
with DiskANN itself is unpinned.  CPU: the oracle's restatement against an
independent numpy restatement, and the host logic of dance_b200.shards.
GPU: the four partition kernels bit-exact against the oracle, and the whole
pipeline (partition -> shard builds -> merge) against oracle shard builds
and the oracle merge.
"""
import struct

import numpy as np
import pytest

import oracle
from dance_b200 import formats, shards, workloads


def np_sq_dist(x, c):
    """Squared L2 of float32 rows x (n x d) to one center, dimension by
    dimension in float32 (each operation rounded, as the kernels do)."""
    d = np.zeros(x.shape[0], np.float32)
    for j in range(x.shape[1]):
        diff = (np.float32(c[j]) - x[:, j]).astype(np.float32)
        d = (d + diff * diff).astype(np.float32)
    return d


def np_assign(x, centers, kb):
    dist = np.stack([np_sq_dist(x, c) for c in centers], axis=1)
    order = np.argsort(dist, axis=1, kind="stable")[:, :kb]
    return order.astype(np.uint32), np.take_along_axis(dist, order, axis=1)


def np_kmeanspp(x, k, seed):
    n = x.shape[0]
    picked = [int(shards.splitmix64(np.uint64(seed)) % np.uint64(n))]
    mind = None
    for p in range(1, k):
        d = np_sq_dist(x, x[picked[-1]])
        mind = d if mind is None else np.minimum(mind, d)
        mx = np.float32(mind.max())
        q = ((mind / mx).astype(np.float32) * np.float32(2.0 ** 31)).astype(np.float32).astype(np.uint64) \
            if mx > 0 else np.ones(n, np.uint64)
        cum = np.cumsum(q, dtype=np.uint64)
        draw = shards.splitmix64(np.uint64(seed) ^ shards.splitmix64(np.uint64(0x5DEECE66D + p)))
        r = draw % cum[-1]
        picked.append(int(np.searchsorted(cum, r, side="right")))
    return x[picked].copy(), np.array(picked, np.uint64)


def np_lloyd(x, centers, iters, chunk=4096):
    c = centers.copy()
    k, dim = c.shape
    for _ in range(iters):
        asg, dist = np_assign(x, c, 1)
        asg, dist = asg[:, 0], dist[:, 0]
        tot = np.zeros((k, dim), np.float64)
        cnt = np.zeros(k, np.int64)
        resid = 0.0
        for b in range(0, len(x), chunk):
            part = np.zeros((k, dim), np.float64)
            rs = 0.0
            for i in range(b, min(len(x), b + chunk)):
                part[asg[i]] += x[i].astype(np.float64)
                cnt[asg[i]] += 1
                rs += float(dist[i])
            tot += part
            resid += rs
        for j in range(k):
            if cnt[j]:
                c[j] = (tot[j] / cnt[j]).astype(np.float32)
    return c, np_assign(x, c, 1)[0][:, 0], resid


def test_oracle_assign_matches_numpy():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((700, 12)).astype(np.float32)
    c = rng.standard_normal((9, 12)).astype(np.float32)
    c[4] = c[2]  # duplicate center: the lower index must come first
    ids, d = oracle.partition_assign(x, c, 3)
    eids, ed = np_assign(x, c, 3)
    assert np.array_equal(ids, eids)
    assert np.array_equal(d.view(np.uint32), ed.view(np.uint32))
    rows4 = np.any(ids == 4, axis=1)
    assert np.all(np.any(ids[rows4] == 2, axis=1))  # center 2 is listed wherever its copy is


def test_oracle_kmeanspp_matches_numpy():
    rng = np.random.default_rng(6)
    x = rng.standard_normal((900, 6)).astype(np.float32)
    c, picked = oracle.kmeanspp_seed(x, 7, seed=11)
    ec, ep = np_kmeanspp(x, 7, 11)
    assert np.array_equal(picked, ep)
    assert np.array_equal(c, ec)


def test_oracle_lloyd_matches_numpy():
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((5000, 5)) + rng.integers(0, 4, (5000, 1)) * 3).astype(np.float32)
    c0 = x[:6].copy()
    c, asg, resid = oracle.kmeans_lloyd(x, c0, 3)
    ec, easg, eres = np_lloyd(x, c0, 3)
    assert np.array_equal(c.view(np.uint32), ec.view(np.uint32))
    assert np.array_equal(asg, easg)
    assert resid == eres


def test_oracle_buckets_are_stable_lists():
    rng = np.random.default_rng(8)
    a = rng.integers(0, 13, (2000, 2)).astype(np.uint32)
    off, ids = oracle.partition_buckets(a, 13)
    for s in range(13):
        # a point that chose s twice appears twice, adjacent
        want = np.repeat(np.arange(len(a)), (a == s).sum(axis=1))
        assert np.array_equal(ids[off[s]:off[s + 1]], want)


def test_random_slice_is_reproducible_and_near_rate():
    a = shards.gen_random_slice_ids(200_000, 0.05, 42)
    b = shards.gen_random_slice_ids(200_000, 0.05, 42)
    c = shards.gen_random_slice_ids(200_000, 0.05, 43)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert abs(len(a) / 200_000 - 0.05) < 0.005
    assert np.all(np.diff(a) > 0)
    assert len(shards.gen_random_slice_ids(10, 1e-9, 1)) == 1
    with pytest.raises(ValueError):
        shards.gen_random_slice_ids(10, 0.0, 1)


def test_shard_build_params_follow_the_patch(monkeypatch):
    for k in ("DISKANN_GPU_SHARD_R", "DISKANN_GPU_C", "DISKANN_GPU_STEPS"):
        monkeypatch.delenv(k, raising=False)
    assert shards.shard_build_params(64, 100) == (42, 84, 20)
    assert shards.shard_build_params(32, 10) == (21, 53, 10)
    monkeypatch.setenv("DISKANN_GPU_SHARD_R", "48")
    monkeypatch.setenv("DISKANN_GPU_STEPS", "200")
    assert shards.shard_build_params(64, 100) == (48, 96, 100)
    monkeypatch.setenv("DISKANN_GPU_C", "16")
    assert shards.shard_build_params(64, 100)[1] == 48  # C never below R_shard


def test_ram_estimate_and_files(tmp_path):
    assert shards.estimate_ram_usage(2000, 100, 4, 64) > shards.estimate_ram_usage(1000, 100, 4, 64)
    assert shards.estimate_ram_usage(1000, 97, 1, 64) == shards.estimate_ram_usage(1000, 104, 1, 64)
    ids = np.array([3, 9, 11], np.uint32)
    shards.write_idmap(tmp_path / "m.bin", ids)
    assert (tmp_path / "m.bin").read_bytes()[:8] == struct.pack("<II", 3, 1)
    assert np.array_equal(shards.read_idmap(tmp_path / "m.bin"), ids)
    c = np.arange(12, dtype=np.float32).reshape(3, 4)
    shards.write_centroids(tmp_path / "c.bin", c)
    assert (tmp_path / "c.bin").read_bytes() == struct.pack("<II", 3, 4) + c.tobytes()


# ---------------------------------------------------------------- GPU
def _cuda(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("k,seed", [(5, 1), (24, 42)])
def test_kmeanspp_matches_oracle(dance_lib, k, seed):
    import torch
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((30_000, 24)) + rng.integers(0, 10, (30_000, 1))).astype(np.float32)
    t = _cuda(x)
    centers = torch.empty((k, 24), dtype=torch.float32, device="cuda")
    picked = torch.empty((k,), dtype=torch.int64, device="cuda")
    assert dance_lib.dance_kmeanspp_seed(t.data_ptr(), 96, len(x), 24, k, seed, centers.data_ptr(),
                                         picked.data_ptr(), None) == 0
    oc, op = oracle.kmeanspp_seed(x, k, seed)
    assert np.array_equal(picked.cpu().numpy().astype(np.uint64), op)
    assert np.array_equal(centers.cpu().numpy(), oc)


@pytest.mark.gpu
def test_kmeans_lloyd_matches_oracle():
    x = workloads.gaussian_mixture_f32(20_000, 32, 40, 0.3, seed=3).numpy()
    t = _cuda(x)
    c, resid = shards.kmeans_centers(t, 12, max_reps=4, seed=9)
    oc0, _ = oracle.kmeanspp_seed(x, 12, 9)
    oc, oasg, ores = oracle.kmeans_lloyd(x, oc0, 4)
    assert np.array_equal(c.cpu().numpy().view(np.uint32), oc.view(np.uint32))
    assert resid == ores
    ids, _ = shards.assign_points(t, c, 1)
    assert np.array_equal(ids.cpu().numpy()[:, 0].astype(np.uint32), oasg)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,dim,kb", [(np.uint8, 128, 2), (np.float32, 96, 3), (np.float16, 100, 1),
                                          (np.uint8, 7, 8)])
def test_partition_assign_matches_oracle(dtype, dim, kb):
    rng = np.random.default_rng(dim)
    if dtype == np.uint8:
        x = rng.integers(0, 256, (20_011, dim)).astype(np.uint8)
        c = rng.integers(0, 256, (17, dim)).astype(np.float32)
    else:
        x = rng.standard_normal((20_011, dim)).astype(dtype)
        c = rng.standard_normal((17, dim)).astype(np.float32)
    c[9] = c[3]  # equal distances: the lower center first
    ids, d = shards.assign_points(_cuda(x), _cuda(c), kb)
    oids, od = oracle.partition_assign(x, c, kb)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), oids)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), od.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("n,kb,S", [(100_000, 2, 40), (3, 1, 1), (50_000, 3, 700)])
def test_partition_buckets_match_oracle(n, kb, S):
    rng = np.random.default_rng(S)
    a = np.stack([rng.permutation(S)[:kb] for _ in range(n)]) if S >= kb else rng.integers(0, S, (n, kb))
    a = a.astype(np.int32)
    off, ids = shards.shard_lists(_cuda(a), S)
    ooff, oids = oracle.partition_buckets(a.astype(np.uint32), S)
    assert np.array_equal(off, ooff.astype(np.int64))
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), oids)


@pytest.mark.gpu
def test_sharded_pipeline_matches_oracle(tmp_path, monkeypatch):
    """Partition a u8 base into 3 overlapping shards, build them on the GPU,
    merge; every shard graph equals the oracle's build of the shard and the
    merged graph equals the oracle merge of the shard graphs."""
    for k in ("DISKANN_GPU_SHARD_R", "DISKANN_GPU_C", "DISKANN_GPU_STEPS", "DISKANN_SHARD_BUILD_PARALLELISM"):
        monkeypatch.delenv(k, raising=False)
    x = workloads.clustered_u8(6000, 32, centroids=30, seed=4).numpy()
    base = tmp_path / "base.u8bin"
    formats.write_bin(base, x)
    R, L = 36, 48
    out = tmp_path / "idx_mem.index"
    med = tmp_path / "idx_medoids.bin"
    res = shards.build_merged_vamana_index(base, "uint8", R, L, 1.0, out, med, sampling_rate=0.2, k_base=2,
                                           num_parts=3, devices=[0], seed=5, keep_tempfiles=True)
    assert res["num_parts"] == 3 and sum(res["shard_sizes"]) == 2 * len(x)
    prefix = str(out) + "_tempFiles"
    # the partition is the oracle's on the same sample
    train_ids = shards.gen_random_slice_ids(len(x), 0.2, 5)
    oc, _ = oracle.kmeanspp_seed(x[train_ids].astype(np.float32), 3, 5)
    oc, _, _ = oracle.kmeans_lloyd(x[train_ids].astype(np.float32), oc, 10)
    oa, _ = oracle.partition_assign(x, oc, 2)
    ooff, oids = oracle.partition_buckets(oa, 3)
    shard_r, C, steps = shards.shard_build_params(R, L)
    src, dst, medoids = [], [], []
    for s in range(3):
        ids = shards.read_idmap(f"{prefix}_subshard-{s}_ids_uint32.bin")
        assert np.array_equal(ids, oids[ooff[s]:ooff[s + 1]])
        g, deg, _, m = oracle.build_graph(np.ascontiguousarray(x[ids]), shard_r, L, C, steps)
        rows, width, start, _ = formats.read_graph(f"{prefix}_subshard-{s}_mem.index")
        assert width == shard_r and start == m
        for v in range(len(ids)):
            assert list(rows[v]) == list(g[v, :deg[v]])
        for v in range(len(ids)):
            for j in range(deg[v]):
                src.append(ids[v])
                dst.append(ids[g[v, j]])
        medoids.append(int(ids[m]))
    mrows, mdeg = oracle.merge_edges(np.array(src, np.uint32), np.array(dst, np.uint32), len(x), R)
    got, width, start, _ = formats.read_graph(out)
    assert width == R and start == medoids[-1]
    for v in range(len(x)):
        assert list(got[v]) == list(mrows[v, :mdeg[v]])
    assert med.read_bytes() == struct.pack("<II", 3, 1) + np.array(medoids, np.uint32).tobytes()
    g = np.full((len(x), R), 0xFFFFFFFF, np.uint32)
    deg = np.array([len(r) for r in got], np.uint32)
    for v, r in enumerate(got):
        g[v, :len(r)] = r
    audit = formats.audit_graph(g, deg, R, start)
    assert all(v == 0 for v in audit.values()), audit
