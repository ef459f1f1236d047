"""Worker for the sharded-build failure test (launched by torchrun, 2 ranks).

Rank 1 creates its NCCL communicator and then never takes part in the build:
it leaves between steps, with nothing of its own in flight.  Rank 0 runs
dance_vamana_build_sharded with a short communicator timeout; its first
collective cannot complete, the bounded wait runs out, the communicator is
aborted and the call must return -4 with an error message that says so,
within a few timeouts.  The ranks coordinate over a gloo group on the CPU,
not over the communicator under test.  NVLS is off (NCCL_NVLS_ENABLE=0).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29521 tests/sharded_abort_check.py
"""
import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from dance_b200 import DanceError, vamana, workloads  # noqa: E402

TIMEOUT_S = 5.0


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    uid = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        uid.copy_(torch.tensor(list(vamana.nccl_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    comm = vamana.Comm(rank, world, bytes(uid.tolist()), timeout_s=TIMEOUT_S)
    ok = True
    if rank == 0:
        n = 20000
        x = workloads.clustered_u8(n, 128, centroids=32, seed=9, device="cuda")
        store, stride = vamana.padded_store(x)
        t0 = time.perf_counter()
        err = ""
        try:
            vamana.build_sharded(comm, store, 128, stride, 32, 64, 48, 32)
        except DanceError as e:
            err = str(e)
        dt = time.perf_counter() - t0
        torch.cuda.synchronize()  # whatever was queued behind the aborted collective drains
        ok = "status -4" in err and "aborted" in err and dt < 6 * TIMEOUT_S
        print(f"rank 0: build returned after {dt:.1f} s: {err!r} ok={ok}", flush=True)
    flag = torch.tensor([1 if ok else 0])
    dist.broadcast(flag, 0)  # rank 1 waits here, outside the communicator, until rank 0 is done
    comm.close()
    dist.destroy_process_group()
    if rank == 0:
        print(f"abort_ok={bool(flag.item())}", flush=True)
    return 0 if flag.item() else 1


if __name__ == "__main__":
    sys.exit(main())
