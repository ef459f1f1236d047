"""dance_merge_edges_device_noalloc: the shard-merge core with its scratch in
a fixed device array instead of per-call allocations.

It must give exactly what dance_merge_edges_device gives, call after call
(the second call reuses the scratch the first one left behind), and refuse
requests beyond its fixed capacity before touching the device.  The file name
sorts last so the suite also runs it after every other test.
"""
import ctypes

import numpy as np
import pytest

SEED = 0x9e3779b97f4a7c15
MAX_NODES, MAX_EDGES = 16384, 1 << 20


def _edges(rng, begin, count, n_edges, hub_edges=0):
    src = rng.integers(begin, begin + count, n_edges).astype(np.uint32)
    dst = rng.integers(0, begin + count + 1000, n_edges).astype(np.uint32)
    if hub_edges:  # one source with a long segment (the one-block path)
        src[:hub_edges] = begin + count // 2
    keep = src != dst
    return src[keep], dst[keep]


def _run(lib, fn, src, dst, begin, count, R):
    import torch
    ds = torch.from_numpy(src.view(np.int32)).cuda()
    dd = torch.from_numpy(dst.view(np.int32)).cuda()
    on = torch.full((count, R), -7, dtype=torch.int32, device="cuda")
    od = torch.full((count,), -7, dtype=torch.int32, device="cuda")
    rc = getattr(lib, fn)(ctypes.c_void_p(ds.data_ptr()), ctypes.c_void_p(dd.data_ptr()), len(src), begin, count, R,
                          SEED, ctypes.c_void_p(on.data_ptr()), ctypes.c_void_p(od.data_ptr()), None)
    torch.cuda.synchronize()
    return rc, on.cpu().numpy(), od.cpu().numpy()


@pytest.mark.gpu
def test_noalloc_merge_matches_allocating_merge_twice(dance_lib):
    rng = np.random.default_rng(2024)
    cases = [
        # (begin, count, edges, hub_edges, R): the second call is smaller, so
        # anything the first call left in the scratch would show up
        (1000, MAX_NODES, 900_000, 5000, 64),
        (37, 3000, 120_000, 700, 24),
    ]
    for begin, count, n_edges, hub, R in cases:
        src, dst = _edges(rng, begin, count, n_edges, hub)
        rc0, rows0, deg0 = _run(dance_lib, "dance_merge_edges_device", src, dst, begin, count, R)
        rc1, rows1, deg1 = _run(dance_lib, "dance_merge_edges_device_noalloc", src, dst, begin, count, R)
        assert rc0 == 0 and rc1 == 0
        assert np.array_equal(deg0, deg1)
        assert np.array_equal(rows0, rows1)
        assert deg1.max() == R  # rows filled to the cap, so the rank order is exercised


def test_noalloc_merge_refuses_oversize_requests(dance_lib):
    # Refused on argument checks alone: the (never dereferenced) pointers are
    # not touched, so this runs without a GPU.
    p = ctypes.c_void_p(256)
    fn = dance_lib.dance_merge_edges_device_noalloc
    assert fn(p, p, 10, 0, MAX_NODES + 1, 8, SEED, p, p, None) == -5
    assert fn(p, p, MAX_EDGES + 1, 0, 16, 8, SEED, p, p, None) == -5
    assert "no-alloc merge holds at most" in dance_lib.dance_last_error().decode()
