"""The online insert on occlusion/victim sets equals the pair-by-pair rule.

The uint8 replay on the tensor cores (dance_b200/csrc/replay_umma.cuh) does
not scan a vertex's kept neighbours pair by pair as the reference's
dynamic_robust_insert_C_warp (src/gpu_vamana_vnew2.cu:759-877) does: it
precomputes, for every expansion x, the set of cached rows that occlude x or
hold x's id, and the set of rows x may replace, and then runs the insert on
those sets against the kept set.  This CPU test restates that set-based rule
in Python and checks it against the oracle's restatement of the reference
rule on the same inputs (exact integer uint8 distances, float32 products),
independently of any GPU.
"""
import numpy as np
import pytest

import oracle
from dance_b200 import workloads

INVALID = 0xFFFFFFFF
FMAX = np.float32(np.finfo(np.float32).max)


def replay_on_sets(x, R, C, alpha, ids, ds, deg, eids, eds, ecnt):
    n = len(x)
    S = eids.shape[1]
    xi = x.astype(np.int64)
    alpha = np.float32(alpha)
    wid_all = np.full((n, C), INVALID, np.uint32)
    wd_all = np.full((n, C), FMAX, np.float32)
    wdeg_all = np.zeros(n, np.uint32)

    def dist(a, b):  # exact integer squared L2, as a float32
        d = xi[a] - xi[b]
        return np.float32(int((d * d).sum()))

    for v in range(n):
        deg_self = min(int(deg[v]), R)
        cnt = min(int(ecnt[v]), S)
        wid = [INVALID] * C
        wd = [FMAX] * C
        for i in range(deg_self):
            nb = int(ids[v, i])
            if nb < n and nb != v:
                wid[i] = nb
                wd[i] = np.float32(ds[v, i])
        # cached rows: ("i", slot) for initial neighbours, ("e", k) for expansions
        row_id = {("i", i): wid[i] for i in range(deg_self)}
        row_dv = {("i", i): wd[i] for i in range(deg_self)}
        slot_of = {("i", i): i for i in range(deg_self)}
        kept = {("i", i) for i in range(deg_self) if wid[i] != INVALID}
        wdeg = deg_self
        for k in range(cnt):
            xk = int(eids[v, k])
            dx = np.float32(eds[v, k])
            row_id[("e", k)] = xk
            row_dv[("e", k)] = dx
            if xk >= n or xk == v:
                continue
            d = min(wdeg, C)
            present = any(row_id[r] == xk for r in kept)
            occluded = any(row_dv[r] <= dx and alpha * dist(row_id[r], xk) <= dx for r in kept)
            if present or occluded:
                continue
            victims = [r for r in kept if row_dv[r] > dx and alpha * dist(xk, row_id[r]) <= row_dv[r]]

            def order(r):  # largest distance first, lowest slot on ties
                return (-float(row_dv[r]), slot_of[r])

            slot, gone = -1, None
            if victims:
                gone = min(victims, key=order)
                slot = slot_of[gone]
            elif d < C:
                slot = d
                wdeg = d + 1
            elif kept:
                worst = min(kept, key=order)
                if dx < row_dv[worst]:
                    gone = worst
                    slot = slot_of[worst]
            if slot < 0:
                continue
            if gone is not None:
                kept.discard(gone)
            kept.add(("e", k))
            slot_of[("e", k)] = slot
            wid[slot] = xk
            wd[slot] = dx
        wid_all[v] = wid
        wd_all[v] = wd
        wdeg_all[v] = wdeg
    return wid_all, wd_all, wdeg_all


@pytest.mark.parametrize("alpha", [1.0, 1.2])
@pytest.mark.parametrize("R,S,C", [(8, 8, 12), (12, 16, 16), (16, 12, 24)])
def test_set_based_insert_equals_pair_rule(alpha, R, S, C):
    x = workloads.clustered_u8(700, 16, centroids=12, seed=R + S).numpy()
    m, _, _ = oracle.medoid(x)
    ids, ds, deg = oracle.init(x, R)
    L = max(S, 16)
    e = oracle.search(x, R, L, S, m, 8, ids, ds, deg, S)
    want = oracle.replay(x, R, C, np.float32(alpha), ids, ds, deg, *e)
    got = replay_on_sets(x, R, C, alpha, ids, ds, deg, *e)
    assert np.array_equal(got[2], want[2])
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))
