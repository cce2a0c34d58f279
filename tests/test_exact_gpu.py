"""GPU parity of the exact progressive path and the float64 certified helpers.

Invariant under test: at every decode step the bound-pruned top-k
equals dense scoring's top-k.  It is checked bit-exactly against the library's own dense
path (same kernels) and up to near-ties against the CPU oracle (stable_topk of float32
scores), on a scaled config-3 trace (AR(1) queries, one new key per step) for every block
size, and on a structured cache where the certified bound does prune.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from oracle import progressive_exact as opx
from tests._util import assert_topk_equivalent, normwise_bound
from tests.conftest import load_golden

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


def ar1_trace(seed, batch, l0, steps, k_scale=1.0, rho=0.95):
    g = torch.Generator().manual_seed(seed)
    keys = (torch.randn(batch, l0 + steps, 128, generator=g) * k_scale).to(torch.bfloat16)
    q = torch.randn(batch, 64, 128, generator=g) / math.sqrt(128)
    w = torch.randn(batch, 64, generator=g) / 8
    qs = [q]
    for _ in range(steps):
        qs.append(rho * qs[-1] + math.sqrt(1 - rho * rho) * torch.randn(batch, 64, 128, generator=g)
                  / math.sqrt(128))
    return keys, [x.to(torch.bfloat16) for x in qs], w


@pytest.mark.parametrize("block_size", [16, 32, 64, 128])
def test_exact_progressive_equals_dense_every_step(block_size):
    from dsa_b200 import score_dense, topk
    from dsa_b200.progressive_exact import ExactProgressiveTopK

    batch, l0, steps, k = 2, 4000, 6, 256
    keys, qs, w = ar1_trace(block_size, batch, l0, steps)
    cache = keys.cuda()
    wc = w.cuda()
    ex = ExactProgressiveTopK(batch, l0 + steps, k, block_size=block_size)
    top, val = ex.init(qs[0].cuda(), wc, cache[:, :l0])
    for step in range(steps + 1):
        length = l0 + step
        qc = qs[step].cuda()
        if step:
            top, val = ex.step(qc, wc, cache[:, :length])
        dense = score_dense(qc, wc, cache[:, :length])
        want_i, want_v = topk(dense, k, sorted=True)
        assert torch.equal(top, want_i), f"step {step}"
        assert torch.equal(val, want_v), f"step {step}"
        d = dense.cpu().numpy()
        for b in range(batch):
            qf, kf = qs[step][b].float().numpy(), keys[b, :length].float().numpy()
            ref = oracle.full_scores(qf, w[b].numpy(), kf)
            tol = 2e-5 * normwise_bound(qf, w[b].numpy(), kf).max()
            assert_topk_equivalent(top[b].cpu().numpy(), oracle.stable_topk(ref, k), ref, tol)
            np.testing.assert_array_equal(top[b].cpu().numpy(), oracle.stable_topk(d[b], k))
    st = ex.stats()
    assert st[0]["steps"] == steps + 1
    assert st[0]["keys_scored"] <= st[0]["keys_total"]


@pytest.mark.parametrize("block_size", [32, 64])
def test_exact_plan_matches_function_form(block_size):
    """ExactProgressivePlan (fixed buffers, one C call per step) returns what the function
    form returns, step for step, on a cache that grows inside its buffer."""
    from dsa_b200.progressive_exact import ExactProgressivePlan, ExactProgressiveTopK

    batch, l0, steps, k = 2, 3000, 5, 128
    keys, qs, w = ar1_trace(9 + block_size, batch, l0, steps)
    cache = keys.cuda()
    wc = w.cuda().contiguous()
    qbuf = qs[0].cuda().clone()
    plan = ExactProgressivePlan(qbuf, wc, cache, k, block_size=block_size, sorted=True,
                                index_dtype=torch.int64)
    ref = ExactProgressiveTopK(batch, l0 + steps, k, block_size=block_size)
    got_i, got_v = plan.init(l0)
    want_i, want_v = ref.init(qbuf, wc, cache[:, :l0])
    assert torch.equal(got_i, want_i) and torch.equal(got_v, want_v)
    for step in range(1, steps + 1):
        qbuf.copy_(qs[step].cuda())
        got_i, got_v = plan.step(l0 + step)
        want_i, want_v = ref.step(qbuf, wc, cache[:, :l0 + step])
        assert torch.equal(got_i, want_i) and torch.equal(got_v, want_v), step
    assert plan.stats() == ref.stats()
    with pytest.raises(ValueError):
        plan.step(l0)  # append-only


@pytest.mark.parametrize("block_size,structured,l0,batch", [
    (64, True, 32760, 3),     # crosses into a second 32768-key segment
    (64, False, 32762, 20),   # the same on a batch too large for clusters: wide one-CTA rows
    (16, True, 65530, 3),     # crosses into a third segment at block size 16
    (128, False, 70001, 3),   # three segments, i.i.d. keys, an odd score-row stride
    (32, True, 98300, 3),     # crosses into a fourth segment
])
def test_exact_long_rows_segment_histograms(block_size, structured, l0, batch):
    """Rows longer than one 32768-key top-k segment: the score waves keep one key
    histogram per segment (pruned keys counted in its -inf bin) and the top-k's first level
    starts every segment from its own; exact == dense bit for bit at every step, sorted and
    unsorted, including the steps that open a new segment."""
    from dsa_b200.indexer import ScoreTopkPlan
    from dsa_b200.progressive_exact import ExactProgressivePlan

    steps, k = 8, 2048
    g = torch.Generator().manual_seed(l0 + block_size)
    total = l0 + steps
    keys = torch.randn(batch, total, 128, generator=g)
    w = torch.randn(batch, 64, generator=g).abs() / 8 if structured else \
        torch.randn(batch, 64, generator=g) / 8
    if structured:
        nb = (total + block_size - 1) // block_size
        scale = torch.where(torch.rand(batch, nb, generator=g) < 0.25, 3.0, 0.05)
        keys *= scale.repeat_interleave(block_size, dim=1)[:, :total, None]
    cache = keys.to(torch.bfloat16).cuda()
    q = torch.randn(batch, 64, 128, generator=g) / math.sqrt(128)
    rho, innov = (0.999, 0.02) if structured else (0.95, math.sqrt(1 - 0.95 ** 2))
    qbuf = q.to(torch.bfloat16).cuda()
    wc = w.cuda()
    plans = {}
    for sorted_ in (False, True):
        plans[sorted_] = ExactProgressivePlan(qbuf, wc, cache, k, block_size=block_size,
                                              sorted=sorted_)
        plans[sorted_].init(l0)
    for t in range(1, steps + 1):
        q = rho * q + innov * torch.randn(batch, 64, 128, generator=g) / math.sqrt(128)
        qbuf.copy_(q.to(torch.bfloat16))
        length = l0 + t
        for sorted_, plan in plans.items():
            got_i, got_v = plan.step(length)
            want_i, want_v = ScoreTopkPlan(qbuf, wc, cache[:, :length], k, sorted=sorted_).run()
            assert torch.equal(got_i.long(), want_i.long()), (t, sorted_)
            assert torch.equal(got_v, want_v), (t, sorted_)
    st = plans[False].stats()
    if structured:
        assert all(s["blocks_pruned"] > 0 for s in st)


def test_exact_progressive_prunes_structured_cache_and_stays_exact():
    """Blocks of small-norm keys next to a few large ones: the bound must skip them."""
    from dsa_b200 import score_dense, topk
    from dsa_b200.progressive_exact import ExactProgressiveTopK

    g = torch.Generator().manual_seed(1)
    length, k, bs = 8192, 64, 64
    scale = torch.where(torch.rand(length // bs, generator=g) < 0.1, 3.0, 0.05)
    keys = (torch.randn(length, 128, generator=g) * scale.repeat_interleave(bs)[:, None])
    keys = keys.to(torch.bfloat16).cuda()
    q0 = torch.randn(64, 128, generator=g) / math.sqrt(128)
    w = (torch.randn(64, generator=g).abs() / 8).cuda()
    ex = ExactProgressiveTopK(1, length, k, block_size=bs)
    ex.init(q0.to(torch.bfloat16).cuda(), w, keys)
    q = q0
    for _ in range(4):
        q = 0.999 * q + 0.02 * torch.randn(64, 128, generator=g) / math.sqrt(128)
        qc = q.to(torch.bfloat16).cuda()
        top, val = ex.step(qc, w, keys)
        want_i, want_v = topk(score_dense(qc, w, keys), k)
        assert torch.equal(top, want_i) and torch.equal(val, want_v)
    st = ex.stats()[0]
    assert st["blocks_pruned"] > 0
    assert st["keys_scored"] < st["keys_total"]


def test_exact_block_decisions_match_oracle_schedule():
    """The device schedule (hot wave, tau, bound) against the oracle's restatement."""
    from dsa_b200.progressive_exact import ExactProgressiveTopK

    g = torch.Generator().manual_seed(2)
    length, k, bs = 4096, 64, 64
    scale = torch.where(torch.rand(length // bs, generator=g) < 0.15, 2.0, 0.1)
    keys = (torch.randn(length, 128, generator=g) * scale.repeat_interleave(bs)[:, None])
    keys = keys.to(torch.bfloat16)
    q0 = (torch.randn(64, 128, generator=g) / math.sqrt(128)).to(torch.bfloat16)
    q1 = (0.998 * q0.float() + 0.03 * torch.randn(64, 128, generator=g) / math.sqrt(128)
          ).to(torch.bfloat16)
    w = torch.randn(64, generator=g).abs() / 8
    ex = ExactProgressiveTopK(1, length, k, block_size=bs)
    ex.init(q0.cuda(), w.cuda(), keys.cuda())
    top, _ = ex.step(q1.cuda(), w.cuda(), keys.cuda())
    st = ex.stats()[0]
    state, _, _ = opx.exact_init(q0.float().numpy(), w.numpy(), keys.float().numpy(), k, bs)
    otop, _, ostats, _ = opx.exact_step(state, q1.float().numpy(), w.numpy(),
                                        keys.float().numpy())
    pruned_gpu = st["blocks_pruned"]  # the init step prunes nothing
    # bounds differ only by float32 round-up on the device, hot sets by near-tie top-k keys
    slack = max(1, ostats["blocks"] // 50)
    assert abs(pruned_gpu - ostats["pruned_blocks"]) <= slack
    assert abs(st["second_wave_blocks"] - ostats["wave2_blocks"]) <= slack
    assert pruned_gpu > 0
    assert set(top.cpu().tolist()) == set(otop.tolist())


def test_certified_helpers_match_reference_golden():
    from dsa_b200.certified import block_key_norms, relu_index_score, temporal_score_radius

    g = load_golden("certified")
    cu = lambda x: torch.from_numpy(np.asarray(x)).cuda()  # noqa: E731
    rep = np.repeat(g["keys"][:, 0][:, None, :], 8, axis=1)
    norms = block_key_norms(cu(rep), 7)
    np.testing.assert_allclose(norms.cpu().numpy(), g["norms"], rtol=1e-13)
    np.testing.assert_allclose(block_key_norms(cu(g["keys"]), 5).cpu().numpy(), g["norms_full"],
                               rtol=1e-13)
    rad = temporal_score_radius(cu(g["qc"]), cu(g["qp"]), cu(g["wc"]), cu(g["wp"]), norms)
    np.testing.assert_allclose(rad.cpu().numpy(), g["radius"], rtol=1e-12)
    rad = temporal_score_radius(cu(g["iq1"]), cu(g["iq0"]), cu(g["iw1"]), cu(g["iw0"]),
                                cu(g["inorms"]))
    np.testing.assert_allclose(rad.cpu().numpy(), g["iradius"], rtol=1e-12)
    prev = relu_index_score(cu(g["qp"]), cu(g["keys"][:, 0]), cu(g["wp"]))
    np.testing.assert_allclose(prev.cpu().numpy(), g["prev"], rtol=1e-12, atol=1e-13)
    c1 = load_golden("cfg1")
    from tests.conftest import cfg1_inputs

    q, w, k = cfg1_inputs()
    got = relu_index_score(q.cuda(), k.cuda(), w.cuda()).cpu().numpy()
    np.testing.assert_allclose(got, c1["relu_index_f64"], rtol=1e-11, atol=1e-12)
    with pytest.raises(ValueError):
        block_key_norms(cu(g["keys"][:, 0]), 4)
    with pytest.raises(ValueError):
        temporal_score_radius(cu(g["qc"]), cu(g["qp"][:4]), cu(g["wc"]), cu(g["wp"]), norms)


def test_topk_kth_value_output():
    """The k-th value the exact path uses as its threshold (top-k kernel side output)."""
    from dsa_b200 import topk

    rng = np.random.default_rng(4)
    for length, k in [(1000, 10), (32768, 2048), (100000, 512)]:
        s = rng.normal(size=(3, length)).astype(np.float32)
        _, val = topk(torch.from_numpy(s).cuda(), k, sorted=True)
        want = np.sort(s, axis=1)[:, ::-1][:, k - 1]
        np.testing.assert_array_equal(val[:, -1].cpu().numpy(), want)
