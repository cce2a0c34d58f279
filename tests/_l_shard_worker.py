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
        idx, val = LShardedTopK(k, sorted=True)(q.to(dev), w.to(dev), shard, start)
        plan = LShardedPlan(q.to(dev), w.to(dev), shard, k, start, sorted=True)
        pidx, pval = plan.run()
        torch.cuda.synchronize()
        if rank == 0:
            want_i, want_v = scores_topk(q.to(dev), w.to(dev), keys.to(dev), k, sorted=True,
                                         index_dtype=torch.int64)
            ok = (torch.equal(idx, want_i) and torch.equal(val, want_v)
                  and torch.equal(pidx, want_i) and torch.equal(pval, want_v))
            with open(out_path, "w") as f:
                f.write("OK" if ok else f"MISMATCH {int((idx != want_i).sum())} indices")
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
