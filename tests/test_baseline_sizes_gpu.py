"""GPU parity at the sizes BASELINE.json states for configs 3, 4 and 5.

- Config 3: one sequence, L = 16384 growing by one key per step for 256 decode steps, AR(1)
  queries (rho 0.95), fixed weights, bf16, top-2048, blocks of 16/32/64/128.  The exact
  certified progressive top-k (``ExactProgressivePlan``) must equal dense scoring's top-k bit
  for bit at every step and block size; dense scoring's top-k must match the oracle's
  (``stable_topk`` of float32 scores) up to keys that tie the k-th score within the
  norm-wise tolerance.  The schedule it follows is the reference's replay filter
  (src/temporal_dsa/replay.py:172-222, tail rule :263-266) with the certified bound of
  certified.py:18-48.
- Config 4: one layer of the sidecar pipeline at B = 64, L = 32768, top-2048:
  ``QueryProjector`` -> ``ScoreTopkPlan`` (score with key histogram, unsorted top-k), every
  row's index set against the oracle's top-k of the oracle's scores from the kernel's own q
  and w, 8 rows' scores against float64.
- Config 5: B = 8, L = 131072, sharded along L into 1, 2, 4 and 8 emulated shards on one
  GPU (each shard's ``LShardedPlan`` local top-k with global indices, then the merge): the
  merged top-2048 equals the whole-row top-k of the oracle.

Tolerances: scores within 1e-5 norm-wise (relative to sum_h |w_h| |q_h . k|, the scale of a
score's float32 rounding); index sets may differ only in keys whose oracle score lies within
2e-5 x the row's largest norm-wise scale of the oracle's k-th score.
"""

from __future__ import annotations

import functools
import math

import numpy as np
import pytest
import torch

import oracle
from oracle import sidecar as osc
from tests._util import assert_scores_close, assert_topk_equivalent, normwise_bound

pytestmark = pytest.mark.gpu

K = 2048


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()
    yield
    from dsa_b200 import device_status

    assert device_status() == 0, "a kernel raised a device status bit"


def oracle_row(q, w, keys):
    """(oracle float32 scores, the row's tie tolerance) for one sequence."""
    ref = oracle.full_scores(q, w, keys)
    dots = np.asarray(q, np.float32) @ np.asarray(keys, np.float32).T
    scale = (np.abs(np.asarray(w, np.float32))[:, None] * np.abs(dots)).sum(axis=0)
    return ref, 2e-5 * float(scale.max())


# ----------------------------------------------------------------------------- config 3
CFG3_L0, CFG3_STEPS = 16384, 256


@functools.lru_cache(maxsize=1)
def config3_trace():
    """Seed 0, drawn in the order BASELINE lists them: q_0, w, the keys (the 16384 initial
    ones and one new key per later step), then the AR(1) innovations."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(64, 128, generator=g) / math.sqrt(128)
    w = torch.randn(64, generator=g) / math.sqrt(64)
    keys = torch.randn(CFG3_L0 + CFG3_STEPS - 1, 128, generator=g).to(torch.bfloat16)
    rho = 0.95
    qs = [q]
    for _ in range(CFG3_STEPS - 1):
        qs.append(rho * qs[-1] + math.sqrt(1 - rho * rho) *
                  torch.randn(64, 128, generator=g) / math.sqrt(128))
    return keys, torch.stack(qs).to(torch.bfloat16), w


@functools.lru_cache(maxsize=1)
def config3_dense():
    """Dense score + top-2048 (sorted) of every step on the GPU: (indices, values) [steps, k]
    and the scores of every step (host, for the oracle comparison)."""
    from dsa_b200 import score_dense, topk

    keys, qs, w = config3_trace()
    kc, wc, qc = keys.cuda().unsqueeze(0), w.cuda().unsqueeze(0), qs.cuda()
    idx, val, scores = [], [], []
    for t in range(CFG3_STEPS):
        s = score_dense(qc[t:t + 1], wc, kc[:, :CFG3_L0 + t])
        i, v = topk(s, K, sorted=True, index_dtype=torch.int32)
        idx.append(i[0])
        val.append(v[0])
        scores.append(s[0].cpu().numpy())
    return torch.stack(idx), torch.stack(val), scores


def test_config3_dense_topk_matches_oracle_every_step():
    keys, qs, w = config3_trace()
    idx, _, scores = config3_dense()
    idx = idx.cpu().numpy()
    kf, wf = keys.float().numpy(), w.numpy()
    for t in range(CFG3_STEPS):
        length = CFG3_L0 + t
        qf = qs[t].float().numpy()
        ref, tol = oracle_row(qf, wf, kf[:length])
        assert_topk_equivalent(idx[t], oracle.stable_topk(ref, K), ref, tol, msg=f"step {t}")
        # the selection itself is exact: stable_topk of the kernel's own scores
        np.testing.assert_array_equal(idx[t], oracle.stable_topk(scores[t], K),
                                      err_msg=f"step {t}")


@pytest.mark.parametrize("block_size", [16, 32, 64, 128])
def test_config3_exact_progressive_equals_dense_every_step(block_size):
    from dsa_b200.progressive_exact import ExactProgressivePlan

    keys, qs, w = config3_trace()
    want_i, want_v, _ = config3_dense()
    kc = keys.cuda().unsqueeze(0)
    qbuf = qs[0].cuda().unsqueeze(0).contiguous()
    wc = w.cuda().unsqueeze(0).contiguous()
    qc = qs.cuda()
    plan = ExactProgressivePlan(qbuf, wc, kc, K, block_size=block_size, sorted=True,
                                index_dtype=torch.int32)
    bad = []
    for t in range(CFG3_STEPS):
        qbuf[0].copy_(qc[t])
        got_i, got_v = plan.init(CFG3_L0) if t == 0 else plan.step(CFG3_L0 + t)
        if not (torch.equal(got_i[0], want_i[t]) and torch.equal(got_v[0], want_v[t])):
            bad.append(t)
    assert not bad, f"exact != dense at steps {bad[:10]} (block {block_size})"
    st = plan.stats()[0]
    assert st["steps"] == CFG3_STEPS
    assert st["keys_total"] == sum(CFG3_L0 + t for t in range(CFG3_STEPS))
    assert st["keys_scored"] <= st["keys_total"]


# ----------------------------------------------------------------------------- config 4
def test_config4_layer_pipeline_matches_oracle():
    """One config-4 layer at its full size: x [64, 2048] -> QueryProjector -> ScoreTopkPlan."""
    from dsa_b200.indexer import ScoreTopkPlan
    from dsa_b200.sidecar import QueryProjector, encode_keys

    b, length, hidden = 64, 32768, 2048
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(4)
    std = hidden ** -0.5
    wq = (torch.randn(8192, hidden, generator=g, device=dev) * std).to(torch.bfloat16)
    ww = torch.randn(64, hidden, generator=g, device=dev) * std
    wk = (torch.randn(128, hidden, generator=g, device=dev) * std).to(torch.bfloat16)
    ln_w, ln_b = torch.ones(128, device=dev), torch.zeros(128, device=dev)
    positions = torch.arange(length, device=dev)
    cache = torch.empty(b, length, 128, device=dev, dtype=torch.bfloat16)
    for r in range(b):
        h = torch.randn(length, hidden, generator=g, device=dev, dtype=torch.bfloat16)
        cache[r] = encode_keys(h, wk, ln_w, ln_b, positions)
    x = torch.randn(b, hidden, generator=g, device=dev, dtype=torch.bfloat16)
    qpos = torch.full((b,), length - 1, device=dev, dtype=torch.long)

    proj = QueryProjector(wq, ww, b)
    q, w = proj.project(x, qpos)
    plan = ScoreTopkPlan(q, w, cache, K, sorted=False)
    idx, val = plan.run()
    torch.cuda.synchronize()
    idx, val = idx.cpu().numpy(), val.cpu().numpy()
    scores = plan.scores.cpu().numpy()
    qh, wh = q.float().cpu().numpy(), w.cpu().numpy()

    # the head weights of the projection against float64 (the GEMV has no 16-bit rounding)
    _, w64 = osc.encode_queries(x.float().cpu().numpy(), wq.float().cpu().numpy(),
                                ww.cpu().numpy(), qpos.cpu().numpy())
    np.testing.assert_allclose(wh, w64, rtol=1e-4, atol=1e-6)

    for r in range(b):
        kf = cache[r].float().cpu().numpy()
        ref, tol = oracle_row(qh[r], wh[r], kf)
        want = oracle.stable_topk(ref, K)
        assert_topk_equivalent(idx[r], want, ref, tol, msg=f"row {r}")
        # unsorted output: the set in ascending index order, values of the kernel's scores
        np.testing.assert_array_equal(idx[r], np.sort(oracle.stable_topk(scores[r], K)),
                                      err_msg=f"row {r}")
        np.testing.assert_array_equal(val[r], scores[r][idx[r]])
        if r % 8 == 3:  # 8 sampled rows against float64
            exact = oracle.relu_index_score(qh[r], kf, wh[r])
            assert_scores_close(scores[r], exact, normwise_bound(qh[r], wh[r], kf), rtol=1e-5,
                                atol=1e-7, msg=f"row {r} vs float64")


# ----------------------------------------------------------------------------- config 5
CFG5_B, CFG5_L = 8, 131072


@functools.lru_cache(maxsize=1)
def config5_inputs():
    """Config 5 (config 2's distributions): q ~ N(0,1)/sqrt(128), w ~ N(0,1)/sqrt(64),
    K ~ N(0,1) bf16, and the oracle's whole-row top-k with each row's tie tolerance."""
    g = torch.Generator().manual_seed(5)
    q = (torch.randn(CFG5_B, 64, 128, generator=g) / math.sqrt(128)).to(torch.bfloat16)
    w = torch.randn(CFG5_B, 64, generator=g) / math.sqrt(64)
    keys = torch.randn(CFG5_B, CFG5_L, 128, generator=g).to(torch.bfloat16)
    refs = []
    for r in range(CFG5_B):
        ref, tol = oracle_row(q[r].float().numpy(), w[r].numpy(), keys[r].float().numpy())
        refs.append((ref, oracle.stable_topk(ref, K), tol))
    return q, w, keys, refs


@pytest.mark.parametrize("world,sorted_", [(1, True), (2, True), (4, True), (8, True),
                                           (8, False)])
def test_config5_sharded_merge_matches_oracle(world, sorted_):
    from dsa_b200 import merge_topk, score_dense
    from dsa_b200.parallel import LShardedPlan, shard_bounds

    q, w, keys, refs = config5_inputs()
    qc, wc, kc = q.cuda(), w.cuda(), keys.cuda()
    vs, js = [], []
    for r in range(world):
        start, stop = shard_bounds(CFG5_L, r, world)
        shard = kc[:, start:stop]
        # this shard's step as a rank runs it: score + local top-k, global indices
        plan = LShardedPlan(qc, wc, shard, K, start, sorted=True)
        plan.plan.run()
        vs.append(plan.plan.values.clone())
        js.append(plan.plan.indices + start)
        plan.close()
    idx, val = merge_topk(torch.cat(vs, 1), torch.cat(js, 1), K, sorted=sorted_,
                          index_dtype=torch.int64)
    idx, val = idx.cpu().numpy(), val.cpu().numpy()
    whole = score_dense(qc, wc, kc).cpu().numpy()
    want_i, want_v = oracle.topk_rows(whole, K, sorted=sorted_)
    np.testing.assert_array_equal(idx, want_i)  # bit-exact vs the whole row's selection
    np.testing.assert_array_equal(val, want_v)
    for r in range(CFG5_B):
        ref, want, tol = refs[r]
        assert_topk_equivalent(idx[r], want, ref, tol, msg=f"row {r} (world {world})")
