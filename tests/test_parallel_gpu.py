"""GPU parity of the L-sharded top-k: the shard-local top-k + merge equals the whole-row
top-k bit for bit, emulated in one process (any GPU count) and, with two or more GPUs, as
two NCCL ranks (config 5 shape)."""

from __future__ import annotations

import math
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()
    yield
    from dsa_b200 import device_status

    assert device_status() == 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_local_topk_and_merge_equal_whole_row(world):
    from dsa_b200 import merge_topk, scores_topk
    from dsa_b200.parallel import local_candidates, shard_bounds

    gen = torch.Generator().manual_seed(world)
    b, length, k = 4, 40000 + world, 1024
    q = (torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16).cuda()
    w = (torch.randn(b, 64, generator=gen) / 8).cuda()
    keys = torch.randn(b, length, 128, generator=gen).to(torch.bfloat16)
    keys[:, 9000:26000] = keys[:, 9000:9001]  # ties across shard boundaries
    keys = keys.cuda()
    vs, js = [], []
    for r in range(world):
        start, stop = shard_bounds(length, r, world)
        v, j = local_candidates(q, w, keys[:, start:stop], k, start)
        vs.append(v)
        js.append(j)
    idx, val = merge_topk(torch.cat(vs, 1), torch.cat(js, 1), k, sorted=True)
    want_i, want_v = scores_topk(q, w, keys, k, sorted=True)
    assert torch.equal(idx, want_i) and torch.equal(val, want_v)
    from dsa_b200 import score_dense

    s = score_dense(q, w, keys).cpu().numpy()
    np.testing.assert_array_equal(idx.cpu().numpy(), oracle.topk_rows(s, k)[0])


def test_l_sharded_plan_single_process_equals_whole_row():
    """LShardedPlan with one rank (no process group): local top-k, packing and merge."""
    from dsa_b200 import scores_topk
    from dsa_b200.parallel import LShardedPlan

    gen = torch.Generator().manual_seed(3)
    b, length, k = 3, 50000, 2048
    q = (torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16).cuda()
    w = (torch.randn(b, 64, generator=gen) / 8).cuda()
    keys = torch.randn(b, length, 128, generator=gen).to(torch.bfloat16).cuda()
    plan = LShardedPlan(q, w, keys, k, 0, sorted=True)
    for _ in range(2):
        idx, val = plan.run()
        want_i, want_v = scores_topk(q, w, keys, k, sorted=True, index_dtype=torch.int64)
        assert torch.equal(idx, want_i) and torch.equal(val, want_v)


@pytest.mark.parametrize("sorted_", [True, False])
def test_peer_exchange_single_rank_equals_allgather_every_step(sorted_):
    """The peer-memory exchange in one process (world 1: the rank publishes into and pulls
    from its own region) returns what the all-gather merge returns, over steps that reuse
    both parities of the region, with ties and a nonzero shard offset."""
    from dsa_b200.parallel import LShardedPlan

    gen = torch.Generator().manual_seed(13)
    b, length, k = 8, 20000, 2048
    q = (torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16).cuda()
    w = (torch.randn(b, 64, generator=gen) / 8).cuda()
    keys = torch.randn(b, length, 128, generator=gen).to(torch.bfloat16).cuda()
    keys[:, 5000:9000] = keys[:, 5000:5001]  # a run of tied scores
    peer = LShardedPlan(q, w, keys, k, 777, sorted=sorted_, exchange="peer")
    ref = LShardedPlan(q, w, keys, k, 777, sorted=sorted_)
    try:
        for step in range(5):
            got_i, got_v = peer.run()
            want_i, want_v = ref.run()
            assert torch.equal(got_i, want_i) and torch.equal(got_v, want_v), step
            q.copy_((q.float() * 0.9 + 0.1 * torch.randn(b, 64, 128, generator=gen).cuda()
                     / math.sqrt(128)).to(torch.bfloat16))
    finally:
        peer.close()


def test_peer_exchange_argument_errors():
    import ctypes as C

    from dsa_b200 import _capi as capi

    lib = capi.lib()
    ptr = C.c_void_p()
    handle = (C.c_uint8 * capi.TDSA_IPC_HANDLE_BYTES)()
    assert lib.tdsa_exchange_create(0, 0, 8, 2048, C.byref(ptr), handle) == capi.TDSA_ERR_INVALID
    assert lib.tdsa_exchange_create(2, 2, 8, 2048, C.byref(ptr), handle) == capi.TDSA_ERR_INVALID
    assert lib.tdsa_exchange_create(16, 0, 8, 4096, C.byref(ptr), handle) == \
        capi.TDSA_ERR_UNSUPPORTED  # 65536 candidates per row
    assert lib.tdsa_exchange_create(1, 0, 8, 2048, C.byref(ptr), handle) == capi.TDSA_OK
    try:
        out = torch.empty(8, 2048, dtype=torch.int64, device="cuda")
        vals = torch.zeros(8, 2048, device="cuda")
        idx = torch.zeros(8, 2048, dtype=torch.int32, device="cuda")
        # not connected yet
        assert lib.tdsa_exchange_topk(ptr, vals.data_ptr(), idx.data_ptr(), 2048, 0, 0,
                                      out.data_ptr(), 8, 2048, None, 0, None) == \
            capi.TDSA_ERR_INVALID
    finally:
        assert lib.tdsa_exchange_destroy(ptr) == capi.TDSA_OK


@pytest.mark.parametrize("world", [2, 3])
def test_l_sharded_exact_progressive_equals_dense_every_step(world):
    """Exact progressive top-k per shard (append-only: new keys go to the last shard) plus
    the merge equals the whole-row dense top-k at every step, with block-structured keys
    and slowly drifting queries so that shards prune blocks."""
    from dsa_b200 import merge_topk, scores_topk
    from dsa_b200.parallel import LShardedExact, shard_bounds

    gen = torch.Generator().manual_seed(50 + world)
    b, base, steps, k, bs = 2, 24576, 6, 512, 64
    total = base + steps
    # keys: a per-block level times a shared direction, so most blocks score far below
    # the hot ones and the certified bound prunes them
    level = torch.randn(b, total // bs + 1, 1, generator=gen) * 0.2
    level[:, ::37] += 3.0
    keys = (level.repeat_interleave(bs, 1)[:, :total] * torch.randn(1, 1, 128, generator=gen)
            + 0.05 * torch.randn(b, total, 128, generator=gen)).to(torch.bfloat16).cuda()
    q = torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)
    w = (torch.randn(b, 64, generator=gen) / 8).cuda()
    bounds = [shard_bounds(base, r, world) for r in range(world)]
    parts = [LShardedExact(b, (stop - start) + steps, k, start, block_size=bs, sorted=True)
             for start, stop in bounds]
    pruned = 0
    for t in range(steps):
        length = base + t
        qt = q.to(torch.bfloat16).cuda()
        vs, js = [], []
        for r, (start, stop) in enumerate(bounds):
            stop = length if r == world - 1 else stop
            fn = parts[r].init if t == 0 else parts[r].step
            idx_r, val_r = fn(qt, w, keys[:, start:stop])
            vs.append(val_r)
            js.append(idx_r.to(torch.int32))
        idx, val = merge_topk(torch.cat(vs, 1), torch.cat(js, 1), k, sorted=True)
        want_i, want_v = scores_topk(qt, w, keys[:, :length], k, sorted=True,
                                     index_dtype=torch.int64)
        assert torch.equal(idx, want_i) and torch.equal(val, want_v), t
        q = 0.995 * q + 0.005 * torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)
    for part in parts:
        pruned += sum(st["blocks_pruned"] for st in part.stats())
    assert pruned > 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_l_sharded_topk_two_nccl_ranks(tmp_path):
    out = tmp_path / "result.txt"
    worker = os.path.join(os.path.dirname(__file__), "_l_shard_worker.py")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531",
           worker, str(out)]
    subprocess.run(cmd, check=True, env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert out.read_text() == "OK"
