"""Worker for the multi-GPU parity check (launched by torchrun, one rank per GPU).

Builds one graph sharded over the ranks and, on rank 0, compares it with the
one-GPU build of the same data: the graphs must be bit-identical.
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        --master-port 29511 tests/sharded_check.py [N]
"""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import dance_b200  # noqa: E402
from dance_b200 import vamana, workloads  # noqa: E402


def main():
    n = int(sys.argv[1]) if len(sys.argv) > 1 else 20000
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ok = True
    try:
        x = workloads.clustered_u8(n, 128, centroids=64, seed=5, device="cuda")
        store, stride = vamana.padded_store(x)
        R, L, C, S = 32, 64, 48, 32
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.tensor(list(vamana.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = vamana.Comm(rank, world, bytes(uid.cpu().tolist()), timeout_s=60.0)
        g, d, m = vamana.build_sharded(comm, store, 128, stride, R, L, C, S)
        g2, d2, m2 = vamana.build_sharded(comm, store, 128, stride, R, L, C, S)  # deterministic across calls
        torch.cuda.synchronize()
        comm.close()
        if rank == 0:
            gs, ds, _, ms = vamana.build_resident(store, 128, stride, R, L, C, S)
            ok = (m == ms and m2 == m and torch.equal(g[:n], gs) and torch.equal(d[:n], ds)
                  and torch.equal(g2, g) and torch.equal(d2, d))
            print(f"sharded x{world} vs one GPU: medoid {m} vs {ms}, identical={ok}", flush=True)
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.broadcast(flag, 0)
        ok = bool(flag.item())
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
