"""One rank of the L-sharded top-k check (launched by tests/test_parallel_gpu.py with
torch.distributed.run, one process per GPU, NCCL).  Rank 0 compares the merged result with
the single-GPU top-k of the whole cache and writes OK or the mismatch to argv[1]."""

from __future__ import annotations

import datetime
import math
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from dsa_b200 import scores_topk  # noqa: E402
from dsa_b200.parallel import LShardedPlan, LShardedTopK, shard_bounds  # noqa: E402


def main() -> None:
    out_path = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        gen = torch.Generator().manual_seed(5)
        b, length, k = 8, 131072, 2048  # config 5 shape
        q = (torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16)
        w = torch.randn(b, 64, generator=gen) / 8
        keys = torch.randn(b, length, 128, generator=gen).to(torch.bfloat16)
        keys[:, 60000:70000] = keys[:, 60000:60001]  # a run of ties across a shard boundary
        start, stop = shard_bounds(length, rank, world)
        dev = torch.device("cuda", torch.cuda.current_device())
        shard = keys[:, start:stop].contiguous().to(dev)
        qd, wd = q.to(dev), w.to(dev)
        idx, val = LShardedTopK(k, sorted=True)(qd, wd, shard, start)
        plan = LShardedPlan(qd, wd, shard, k, start, sorted=True)
        peer = LShardedPlan(qd, wd, shard, k, start, sorted=True, exchange="peer")
        pidx, pval = plan.run()
        xidx, xval = peer.run()
        torch.cuda.synchronize()
        want_i, want_v = scores_topk(qd, wd, keys.to(dev), k, sorted=True,
                                     index_dtype=torch.int64)
        ok = (torch.equal(idx, want_i) and torch.equal(val, want_v)
              and torch.equal(pidx, want_i) and torch.equal(pval, want_v)
              and torch.equal(xidx, want_i) and torch.equal(xval, want_v))
        msg = "" if ok else f"step 0: {int((xidx != want_i).sum())} peer-exchange indices differ"
        # later steps: new queries in place; the peer exchange reuses both region parities
        for step in range(1, 5):
            qd.copy_((qd.float() * 0.9 + 0.1 * torch.randn(b, 64, 128, generator=gen).to(dev)
                      / math.sqrt(128)).to(torch.bfloat16))
            pidx, pval = plan.run()
            xidx, xval = peer.run()
            torch.cuda.synchronize()
            if not (torch.equal(pidx, xidx) and torch.equal(pval, xval)):
                ok, msg = False, msg or f"step {step}: peer exchange != all-gather"
        peer.close()
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(out_path, "w") as f:
                f.write("OK" if int(flag) == 1 else f"MISMATCH {msg or 'on another rank'}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
