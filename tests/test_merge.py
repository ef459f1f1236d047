"""Shard merge (reference src/gpu_merge.cu merge_shards_gpu).

CPU: the oracle's rule against an independent Python restatement.
GPU: dance_merge_shards_gpu on shard files against the oracle, byte for
byte (graph file and medoids file), the device core, and the error codes.
"""
import ctypes
import struct

import numpy as np
import pytest

import oracle
from dance_b200 import formats

SEED = 0x9e3779b97f4a7c15
M64 = (1 << 64) - 1


def py_hash_edge32(src, dst, seed=SEED):
    x = ((src << 32) ^ dst ^ seed) & M64
    x ^= x >> 33
    x = (x * 0xff51afd7ed558ccd) & M64
    x ^= x >> 33
    x = (x * 0xc4ceb9fe1a85ec53) & M64
    x ^= x >> 33
    return (x ^ (x >> 32)) & 0xFFFFFFFF


def py_merge(src, dst, nnodes, max_degree):
    adj = [set() for _ in range(nnodes)]
    for s, d in zip(src.tolist(), dst.tolist()):
        if s != d:
            adj[s].add(d)
    rows = np.full((nnodes, max_degree), 0xFFFFFFFF, np.uint32)
    deg = np.zeros(nnodes, np.uint32)
    for v in range(nnodes):
        ranked = sorted(adj[v], key=lambda d: (py_hash_edge32(v, d), d))[:max_degree]
        deg[v] = len(ranked)
        rows[v, :len(ranked)] = ranked
    return rows, deg


def test_hash_edge32_known_answers(oracle_lib):
    for s, d in [(0, 0), (1, 2), (123456, 7890), (2**32 - 1, 2**32 - 1), (5, 4000000000)]:
        assert oracle_lib.oracle_hash_edge32(s, d, SEED) == py_hash_edge32(s, d)


def test_oracle_merge_rule_matches_restatement():
    rng = np.random.default_rng(0)
    n = 300
    src = rng.integers(0, n, 20000).astype(np.uint32)
    dst = rng.integers(0, n, 20000).astype(np.uint32)
    a = oracle.merge_edges(src, dst, n, 24)
    b = py_merge(src, dst, n, 24)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def make_shards(tmp_path, n=3000, nshards=3, width=16, overlap=2, seed=1):
    """Overlapping shards: every point in `overlap` random shards, random local graphs."""
    rng = np.random.default_rng(seed)
    member = [[] for _ in range(nshards)]
    for v in range(n):
        for s in rng.choice(nshards, size=overlap, replace=False):
            member[s].append(v)
    src_all, dst_all, medoids = [], [], []
    for s in range(nshards):
        ids = np.array(sorted(member[s]), np.uint32)
        k = len(ids)
        g = np.full((k, width), 0xFFFFFFFF, np.uint32)
        deg = rng.integers(0, width + 1, k).astype(np.uint32)
        for i in range(k):
            g[i, :deg[i]] = rng.integers(0, k, deg[i])
        med = int(rng.integers(0, k))
        formats.write_graph(tmp_path / f"shard{s}.idx", g, deg, med)
        with open(tmp_path / f"shard{s}_ids.bin", "wb") as f:
            f.write(struct.pack("<II", k, 1) + ids.tobytes())
        for i in range(k):
            for j in range(deg[i]):
                src_all.append(ids[i])
                dst_all.append(ids[g[i, j]])
        medoids.append(int(ids[med]))
    return np.array(src_all, np.uint32), np.array(dst_all, np.uint32), medoids


@pytest.mark.gpu
def test_merge_shards_files_match_oracle(tmp_path, dance_lib):
    n, nshards, R = 3000, 3, 24
    src, dst, medoids = make_shards(tmp_path, n, nshards)
    rows, deg = oracle.merge_edges(src, dst, n, R)
    expected = formats.encode_graph(rows, deg, medoids[-1])
    # the graph header carries max_degree = R (the requested width), not the max degree
    expected = expected[:8] + struct.pack("<I", R) + expected[12:]
    out, med = tmp_path / "merged.idx", tmp_path / "medoids.bin"
    rc = dance_lib.dance_merge_shards_gpu(str(tmp_path / "shard").encode(), b".idx",
                                          str(tmp_path / "shard").encode(), b"_ids.bin", nshards, R,
                                          str(out).encode(), str(med).encode())
    assert rc == 0
    assert out.read_bytes() == expected
    assert med.read_bytes() == struct.pack("<II", nshards, 1) + np.array(medoids, np.uint32).tobytes()


@pytest.mark.gpu
def test_merge_shards_bucketed_and_long_segments(tmp_path, dance_lib, monkeypatch):
    # many buckets, and a few sources with more than 512 merged edges
    n, R = 2000, 700
    rng = np.random.default_rng(3)
    ids = np.arange(n, dtype=np.uint32)
    g = np.full((n, 900), 0xFFFFFFFF, np.uint32)
    deg = rng.integers(0, 8, n).astype(np.uint32)
    for v in range(n):
        g[v, :deg[v]] = rng.integers(0, n, deg[v])
    for v in (5, 77):
        deg[v] = 900
        g[v] = rng.permutation(n)[:900]
    formats.write_graph(tmp_path / "s0.idx", g, deg, 0)
    with open(tmp_path / "s0_ids.bin", "wb") as f:
        f.write(struct.pack("<II", n, 1) + ids.tobytes())
    src = np.repeat(np.arange(n, dtype=np.uint32), deg.astype(np.int64))
    dst = np.concatenate([g[v, :deg[v]] for v in range(n)]).astype(np.uint32)
    rows, odeg = oracle.merge_edges(src, dst, n, R)
    monkeypatch.setenv("DISKANN_GPU_MERGE_BUCKETS", "7")
    out, med = tmp_path / "m.idx", tmp_path / "med.bin"
    rc = dance_lib.dance_merge_shards_gpu(str(tmp_path / "s").encode(), b".idx", str(tmp_path / "s").encode(),
                                          b"_ids.bin", 1, R, str(out).encode(), str(med).encode())
    assert rc == 0
    got_rows, _, start, _ = formats.read_graph(out)
    assert start == 0
    for v in range(n):
        assert list(got_rows[v]) == list(rows[v, :odeg[v]])


@pytest.mark.gpu
def test_merge_device_core(dance_lib):
    import torch
    rng = np.random.default_rng(5)
    n, R = 5000, 32
    src = rng.integers(0, n, 200000).astype(np.uint32)
    dst = rng.integers(0, n, 200000).astype(np.uint32)
    keep = src != dst
    src, dst = src[keep], dst[keep]
    rows, deg = oracle.merge_edges(src, dst, n, R)
    ds = torch.from_numpy(src.view(np.int32)).cuda()
    dd = torch.from_numpy(dst.view(np.int32)).cuda()
    on = torch.full((n, R), -1, dtype=torch.int32, device="cuda")
    od = torch.zeros(n, dtype=torch.int32, device="cuda")
    rc = dance_lib.dance_merge_edges_device(ctypes.c_void_p(ds.data_ptr()), ctypes.c_void_p(dd.data_ptr()), len(src),
                                            0, n, R, SEED, ctypes.c_void_p(on.data_ptr()),
                                            ctypes.c_void_p(od.data_ptr()), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert np.array_equal(od.cpu().numpy().view(np.uint32), deg)
    assert np.array_equal(on.cpu().numpy().view(np.uint32), rows)


@pytest.mark.gpu
def test_merge_error_codes(tmp_path, dance_lib):
    src, dst, medoids = make_shards(tmp_path, 500, 2)
    call = lambda pre, nsh=2: dance_lib.dance_merge_shards_gpu(  # noqa: E731
        str(tmp_path / pre).encode(), b".idx", str(tmp_path / "shard").encode(), b"_ids.bin", nsh, 16,
        str(tmp_path / "o.idx").encode(), str(tmp_path / "m.bin").encode())
    assert call("shard", 3) == -2  # missing id map of shard 2
    blob = bytearray((tmp_path / "shard0.idx").read_bytes())
    blob[16:24] = struct.pack("<Q", 1)  # frozen points
    (tmp_path / "bad0.idx").write_bytes(bytes(blob))
    (tmp_path / "bad1.idx").write_bytes((tmp_path / "shard1.idx").read_bytes())
    assert call("bad") == -3
    blob = bytearray((tmp_path / "shard0.idx").read_bytes())
    blob[12:16] = struct.pack("<I", 10**6)  # medoid out of range
    (tmp_path / "bad0.idx").write_bytes(bytes(blob))
    assert call("bad") == -4
    assert call("shard") == 0


# ---------------------------------------------------------------- reference goldens
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _merge_golden_cases():
    import json
    m = GOLDEN / "manifest_merge.json"
    return json.loads(m.read_text()) if m.exists() else []


def _golden_inputs(tmp_path, case):
    from tests.golden.make_golden_merge import write_shards
    recipe = dict(case["shards"])
    if "hubs" in recipe:
        recipe["hubs"] = tuple(recipe["hubs"])
    src, dst, medoids, digest = write_shards(tmp_path, **recipe)
    assert digest == case["inputs_sha256"], "regenerated shard files differ from the golden's inputs"
    z = np.load(GOLDEN / case["file"])
    return src, dst, medoids, z["graph_file"].tobytes(), z["medoids_file"].tobytes()


@pytest.mark.parametrize("case", _merge_golden_cases(), ids=lambda c: c["file"])
def test_oracle_merge_matches_reference_goldens(tmp_path, case):
    """The oracle's merge rule reproduces the files the reference's own
    merge_shards_gpu wrote (tests/golden/make_golden_merge.py), byte for byte."""
    src, dst, medoids, gfile, mfile = _golden_inputs(tmp_path, case)
    R = case["max_degree"]
    seed = int(case["env"].get("DISKANN_GPU_MERGE_HASH_SEED", SEED))
    nnodes = int(max(src.max(initial=0), dst.max(initial=0))) + 1
    keep = src != dst
    rows, deg = oracle.merge_edges(src[keep], dst[keep], nnodes, R, seed=seed)
    expected = formats.encode_graph(rows, deg, medoids[-1])
    expected = expected[:8] + struct.pack("<I", R) + expected[12:]
    assert expected == gfile
    assert mfile == struct.pack("<II", len(medoids), 1) + np.array(medoids, np.uint32).tobytes()


@pytest.mark.gpu
@pytest.mark.parametrize("case", _merge_golden_cases(), ids=lambda c: c["file"])
def test_merge_shards_gpu_matches_reference_goldens(tmp_path, case, dance_lib, monkeypatch):
    _, _, medoids, gfile, mfile = _golden_inputs(tmp_path, case)
    for k, v in case["env"].items():
        monkeypatch.setenv(k, v)
    out, med = tmp_path / "merged.idx", tmp_path / "medoids.bin"
    pre = str(tmp_path / "shard").encode()
    rc = dance_lib.dance_merge_shards_gpu(pre, b".idx", pre, b"_ids.bin", case["shards"]["nshards"],
                                          case["max_degree"], str(out).encode(), str(med).encode())
    assert rc == 0
    assert out.read_bytes() == gfile
    assert med.read_bytes() == mfile
