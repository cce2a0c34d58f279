"""Child process for test_graph_capture_gpu: the first ScoreTopkPlan.run of each shape is
captured into a CUDA graph with no call before it, so one-time per-process setup (kernel
attributes, the cluster-size query) happens inside the capture.  Exits non-zero on any
mismatch with separate score + stable top-k calls."""

from __future__ import annotations

import math
import sys

import torch

from dsa_b200 import score_dense, topk
from dsa_b200.indexer import ScoreTopkPlan


def main() -> int:
    dev = torch.device("cuda")
    gen = torch.Generator(device="cuda").manual_seed(5)
    for batch, length in ((1, 32768), (16, 20000), (96, 4096)):
        q = (torch.randn(batch, 64, 128, device=dev, generator=gen) / math.sqrt(128)).to(
            torch.bfloat16)
        w = torch.randn(batch, 64, device=dev, generator=gen) / 8
        keys = torch.randn(batch, length, 128, device=dev, generator=gen).to(torch.bfloat16)
        plan = ScoreTopkPlan(q, w, keys, 2048, sorted=False)
        stream = torch.cuda.Stream(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            plan.run()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
        want_i, want_v = topk(score_dense(q, w, keys), 2048, sorted=False)
        if not (torch.equal(plan.indices.to(torch.int64), want_i.to(torch.int64))
                and torch.equal(plan.values, want_v)):
            print(f"mismatch at batch {batch}, length {length}", file=sys.stderr)
            return 1
        if int(plan.key_hist.abs().sum()) != 0:
            print(f"histogram not consumed at batch {batch}", file=sys.stderr)
            return 1
        del graph
    return 0


if __name__ == "__main__":
    sys.exit(main())
