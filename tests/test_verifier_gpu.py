"""GPU parity of the verifier scorer and the torch-named scoring entry points.

score_head_sparse against the reference's golden outputs (verifier_scoring.py:49-92,
float32, fixed and per-query head ids) and the oracle (bf16); torch_full_scores /
torch_progressive_scores (progressive_kernel.py:45-90) against the golden scores and the
oracle's restatement of the per-block torch loop.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from tests._util import assert_scores_close, normwise_bound
from tests.conftest import bf16_from_bits, load_golden

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


def _selected_bound(q, w, k, ids):
    """Norm-wise scale of a head-sparse score: sum over the selected heads of |w||q.k|."""
    ids = np.asarray(ids)
    out = []
    for row in range(q.shape[0]):
        sel = ids if ids.ndim == 1 else ids[row]
        out.append((np.abs(w[row, sel])[:, None] * np.abs(q[row, sel] @ k.T)).sum(axis=0))
    return np.stack(out)


@pytest.mark.parametrize("which", ["fixed", "dyn"])
def test_score_head_sparse_matches_reference_golden(which):
    from dsa_b200.verifier_scoring import score_head_sparse

    g = load_golden("batched")
    q, w, k = g["q"][0], g["w"][0], g["k"][0]
    ids = g[f"ids_{which}"]
    got = score_head_sparse(torch.from_numpy(q).cuda(), torch.from_numpy(w).cuda(),
                            torch.from_numpy(k).cuda(), torch.from_numpy(ids).cuda())
    assert got.dtype == torch.float32 and got.shape == (2, 100)
    scale = _selected_bound(q, w, k, ids)
    assert_scores_close(got.cpu().numpy(), g[f"hs_{which}"], scale, rtol=1e-5, atol=1e-7)
    want = oracle.score_head_sparse(q, w, k, ids)
    assert_scores_close(got.cpu().numpy(), want, scale, rtol=1e-5, atol=1e-7)


def test_score_head_sparse_bf16_repeated_ids_and_errors():
    from dsa_b200.verifier_scoring import dynamic_head_indices, score_head_sparse

    gen = torch.Generator().manual_seed(5)
    q = (torch.randn(3, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16)
    w = torch.randn(3, 64, generator=gen) / 8
    k = torch.randn(777, 128, generator=gen).to(torch.bfloat16)
    ids = dynamic_head_indices(w, 8, "high_weight")
    ids[:, 7] = ids[:, 0]  # a repeated head counts twice
    got = score_head_sparse(q.cuda(), w.cuda(), k.cuda(), ids.cuda()).cpu().numpy()
    want = oracle.score_head_sparse(q.float().numpy(), w.numpy(), k.float().numpy(), ids.numpy())
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-3)
    with pytest.raises(ValueError):
        score_head_sparse(q.cuda(), w.cuda(), k.cuda(), ids[:2].cuda())
    with pytest.raises(ValueError):
        score_head_sparse(q[0].cuda(), w.cuda(), k.cuda(), ids.cuda())


@pytest.mark.parametrize("strategy", ["high_weight", "positive_weight"])
def test_dynamic_head_indices_stable_ties(strategy):
    from dsa_b200.verifier_scoring import dynamic_head_indices

    w = torch.tensor(np.round(np.random.default_rng(3).normal(size=(4, 64)) * 2) / 2,
                     dtype=torch.float32)
    got = dynamic_head_indices(w.cuda(), 12, strategy).cpu().numpy()
    vals = np.abs(w.numpy()) if strategy == "high_weight" else np.maximum(w.numpy(), 0)
    want = np.stack([np.lexsort((np.arange(64), -v))[:12] for v in vals])
    np.testing.assert_array_equal(got, want)
    with pytest.raises(ValueError):
        dynamic_head_indices(w, 0, strategy)
    with pytest.raises(ValueError):
        dynamic_head_indices(w, 8, "other")


def test_torch_full_scores_f32_golden():
    from dsa_b200.progressive_kernel import torch_full_scores

    g = load_golden("progressive_kernel")
    q, w, k = g["f32_q"], g["f32_w"], g["f32_L257_keys"]
    got = torch_full_scores(torch.from_numpy(q).cuda(), torch.from_numpy(w).cuda(),
                            torch.from_numpy(k).cuda()).cpu().numpy()
    assert_scores_close(got, g["f32_L257_scores"], normwise_bound(q, w, k), rtol=1e-5)


@pytest.mark.parametrize("block_size", [16, 32, 64, 128])
def test_torch_progressive_scores_matches_oracle(block_size):
    from dsa_b200.progressive_kernel import dynamic_head_ids, torch_progressive_scores

    length = 1000
    gen = torch.Generator().manual_seed(block_size)
    q = (torch.randn(64, 128, generator=gen) * 0.1).to(torch.bfloat16)
    w = torch.randn(64, generator=gen)
    k = (torch.randn(length, 128, generator=gen) * 0.1).to(torch.bfloat16)
    nb = math.ceil(length / block_size)
    direct = torch.from_numpy(np.random.default_rng(block_size).random(nb) < 0.3)
    heads = dynamic_head_ids(w)
    qf, kf = q.float().numpy(), k.float().numpy()
    _, _, probe = oracle.progressive_scores(qf, w.numpy(), kf, heads.numpy(), direct.numpy(),
                                            math.inf, block_size=block_size)
    thr = float(np.quantile(probe, 0.6))
    scores, accepted, block_max = torch_progressive_scores(
        q.cuda(), w.cuda(), k.cuda(), heads, direct.cuda(), thr, block_size=block_size)
    ws, wa, wm = oracle.progressive_scores(qf, w.numpy(), kf, heads.numpy(), direct.numpy(), thr,
                                           block_size=block_size)
    assert accepted.dtype == torch.bool
    np.testing.assert_allclose(block_max.cpu().numpy(), wm, rtol=1e-5, atol=1e-5)
    got_a = accepted.cpu().numpy()
    near = np.abs(wm.astype(np.float64) - thr) <= 1e-5 * max(1.0, abs(thr))
    assert not np.any((got_a != wa) & ~near)
    same = np.repeat(got_a == wa, block_size)[:length]
    got_s = scores.cpu().numpy()
    np.testing.assert_array_equal(np.isneginf(got_s[same]), np.isneginf(ws[same]))
    fin = same & np.isfinite(ws)
    scale = normwise_bound(qf, w.numpy(), kf)
    assert_scores_close(got_s[fin], ws[fin], scale[fin], rtol=1e-5, atol=1e-7)


def test_normalized_hadamard_and_quantizer_match_reference_golden():
    """verifier_scoring.py:9-41 on float32: the same butterflies and the same quantizer
    arithmetic as the reference's float32 path."""
    from dsa_b200.verifier_scoring import fake_symmetric_quantize, normalized_hadamard

    g = load_golden("verifier")
    hk = normalized_hadamard(torch.from_numpy(g["k"]).cuda()).cpu().numpy()
    hq = normalized_hadamard(torch.from_numpy(g["q"]).cuda()).cpu().numpy()
    np.testing.assert_allclose(hk, g["had_k"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(hq, g["had_q"], rtol=1e-6, atol=1e-8)
    for bits in (2, 4, 8):
        qk, sc = fake_symmetric_quantize(torch.from_numpy(g["k"]).cuda(), bits)
        assert sc == pytest.approx(float(g[f"fq{bits}_scale"]), rel=1e-7)
        np.testing.assert_array_equal(qk.cpu().numpy(), g[f"fq{bits}_k"])
    with pytest.raises(ValueError):
        normalized_hadamard(torch.zeros(3, 64, device="cuda"))
    with pytest.raises(ValueError):
        fake_symmetric_quantize(torch.zeros(3, 128, device="cuda"), 3)


@pytest.mark.parametrize("rotation", ["none", "hadamard"])
@pytest.mark.parametrize("bits", [None, 4, 8])
def test_score_dim_sparse_matches_reference_golden(rotation, bits):
    from dsa_b200.verifier_scoring import score_dim_sparse

    g = load_golden("verifier")
    q, w, k = (torch.from_numpy(g[n]).cuda() for n in ("q", "w", "k"))
    got = score_dim_sparse(q, w, k, torch.from_numpy(g["dims"]), rotation=rotation,
                           bits=bits).cpu().numpy()
    want = g[f"ds_{rotation}_{bits or 0}"]
    dims = g["dims"]
    qs, ks = g["q"][..., dims], g["k"][..., dims]
    scale = np.stack([(np.abs(g["w"][i])[:, None] * np.abs(qs[i] @ ks.T)).sum(0)
                      for i in range(2)])
    assert_scores_close(got, want, scale + 1e-3, rtol=1e-4, atol=1e-6)


def test_score_dim_sparse_fixed_scales_bf16_and_full_width():
    from dsa_b200 import score_dense
    from dsa_b200.verifier_scoring import score_dim_sparse

    g = load_golden("verifier")
    q, w, k = (torch.from_numpy(g[n]).cuda() for n in ("q", "w", "k"))
    got = score_dim_sparse(q, w, k, g["dims"], bits=4, query_scale=0.05, key_scale=0.5)
    np.testing.assert_allclose(got.cpu().numpy(), g["ds_none_4_fixed"], rtol=1e-4, atol=1e-5)
    # bf16 inputs: the reference rounds every butterfly stage to bf16, the kernel once
    qb = torch.from_numpy(bf16_from_bits(g["q_bf16"])).cuda().to(torch.bfloat16)
    kb = torch.from_numpy(bf16_from_bits(g["k_bf16"])).cuda().to(torch.bfloat16)
    for rot in ("none", "hadamard"):
        got = score_dim_sparse(qb, w, kb, g["dims"], rotation=rot, bits=8).cpu().numpy()
        np.testing.assert_allclose(got, g[f"dsb_{rot}_8"], rtol=5e-2, atol=5e-2)
    # all 128 dimensions, no rotation: the dense score (reference test_verifier_scoring.py:23-30)
    full = score_dim_sparse(q, w, k, torch.arange(128)).cpu().numpy()
    dense = torch.stack([score_dense(q[i], w[i], k) for i in range(2)]).cpu().numpy()
    np.testing.assert_allclose(full, dense, rtol=1e-6, atol=1e-7)
