"""Worker for the multi-GPU stitched check (launched by torchrun, one rank per GPU).

Builds the per-label graphs spread over the ranks through the C ABI
(dance_stitched_build_sharded: local graphs to rank 0 over NCCL) and, on
rank 0, compares the stitched CSR graph and the label medoids with the
one-GPU stitched build of the same data: they must be identical (the label
graphs are independent, so where a label is built cannot change it).
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        --master-port 29513 tests/stitched_sharded_check.py [N]
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from dance_b200 import stitched as S, vamana  # noqa: E402


def main():
    n = int(sys.argv[1]) if len(sys.argv) > 1 else 30000
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ok = True
    try:
        rng = np.random.default_rng(11)
        nl, dim = 24, 32
        c = rng.standard_normal((32, dim))
        x = (c[rng.integers(0, 32, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
        w = 1.0 / np.arange(1, nl + 1)
        sizes = np.maximum(1, np.floor(w / w.sum() * n)).astype(int)
        sizes[0] += n - sizes.sum()
        assign = np.repeat(np.arange(nl), sizes)
        rng.shuffle(assign)
        offs, pts = S.labels_csr(S.labels_from_assignment(assign, nl))
        args = dict(r_small=16, l_small=40, r_stitched=24, C=32, steps=24)
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.tensor(list(vamana.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = vamana.Comm(rank, world, bytes(uid.cpu().tolist()), timeout_s=60.0)
        ro, ri, med, st = S.stitched_build_sharded(comm, x, offs, pts, **args)
        torch.cuda.synchronize()
        comm.close()
        if rank == 0:
            so, si, smed, _ = S.stitched_build(x, offs, pts, **args)
            ok = (np.array_equal(ro, so) and np.array_equal(ri, si) and np.array_equal(med, smed))
            print(f"stitched x{world} vs one GPU: edges {len(ri)} vs {len(si)}, exchange "
                  f"{st['label_graph_exchange_seconds']:.3f} s, identical={ok}", flush=True)
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.broadcast(flag, 0)
        ok = bool(flag.item())
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
