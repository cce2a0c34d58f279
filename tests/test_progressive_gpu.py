"""GPU parity of the block-structured kernels (H8 probe, masked, fused progressive).

Mirrors the reference's GPU tests (tests/test_progressive_kernel.py:139-197: same inputs
shape, same assertions and tolerances) with CPU-seeded inputs, and compares every output
with the oracle's restatement of the Triton kernels' semantics for all block sizes.
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


def cuda_inputs(length: int, seed: int = 1582):
    """tests/test_progressive_kernel.py:131-136 of the reference, seeded on the CPU."""
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(64, 128, generator=g) * 0.1).to(torch.bfloat16).cuda()
    w = torch.randn(64, generator=g).cuda()
    k = (torch.randn(length, 128, generator=g) * 0.1).to(torch.bfloat16).cuda()
    return q, w, k


def np32(t):
    return t.float().cpu().numpy()


def test_triton_full_matches_torch_reference():
    from dsa_b200.progressive_kernel import full_scores_triton

    q, w, k = cuda_inputs(257)
    actual = full_scores_triton(q, w, k)
    expected = torch.from_numpy(oracle.full_scores(np32(q), np32(w), np32(k))).cuda()
    torch.testing.assert_close(actual, expected, rtol=3e-3, atol=3e-3)


def test_triton_progressive_all_promoted_matches_full_kernel():
    from dsa_b200.progressive_kernel import (dynamic_head_ids, full_scores_triton,
                                             progressive_scores_triton)

    q, w, k = cuda_inputs(257)
    direct = torch.zeros(math.ceil(len(k) / 64), device="cuda", dtype=torch.int8)
    result = progressive_scores_triton(q, w, k, dynamic_head_ids(w.cpu()), direct, -math.inf)
    expected = full_scores_triton(q, w, k)
    torch.testing.assert_close(result.scores, expected, rtol=1e-5, atol=1e-5)
    assert result.accepted_blocks.bool().all()


def test_triton_progressive_direct_and_rejected_blocks():
    from dsa_b200.progressive_kernel import full_scores_triton, progressive_scores_triton

    q, w, k = cuda_inputs(128)
    direct = torch.tensor([1, 0], device="cuda", dtype=torch.int8)
    result = progressive_scores_triton(q, w, k, torch.arange(8), direct, math.inf)
    expected = full_scores_triton(q, w, k)
    torch.testing.assert_close(result.scores[:64], expected[:64], rtol=1e-5, atol=1e-5)
    assert torch.isneginf(result.scores[64:]).all()


def test_two_pass_matches_fused_decisions():
    from dsa_b200.progressive_kernel import (dynamic_head_ids, progressive_scores_triton,
                                             two_pass_scores_triton)

    q, w, k = cuda_inputs(256)
    direct = torch.tensor([1, 0, 0, 1], device="cuda", dtype=torch.int8)
    heads = dynamic_head_ids(w.cpu())
    probe = progressive_scores_triton(q, w, k, heads, direct, math.inf)
    threshold = torch.quantile(probe.block_max[1:3], 0.5)
    fused = progressive_scores_triton(q, w, k, heads, direct, threshold)
    two_pass = two_pass_scores_triton(q, w, k, heads, direct, threshold)
    assert torch.equal(fused.accepted_blocks, two_pass.accepted_blocks)
    torch.testing.assert_close(fused.scores, two_pass.scores, rtol=1e-5, atol=1e-5)


def test_compact_output_matches_dense_candidates():
    from dsa_b200.progressive_kernel import dynamic_head_ids, progressive_scores_triton

    q, w, k = cuda_inputs(192)
    direct = torch.tensor([1, 0, 1], device="cuda", dtype=torch.int8)
    heads = dynamic_head_ids(w.cpu())
    dense = progressive_scores_triton(q, w, k, heads, direct, math.inf)
    compact = progressive_scores_triton(q, w, k, heads, direct, math.inf, compact=True)
    assert compact.candidate_count == 128
    assert compact.candidate_indices is not None
    order = torch.argsort(compact.candidate_indices.long())
    indices = compact.candidate_indices[order].long()
    torch.testing.assert_close(compact.scores[order], dense.scores[indices])


def test_compact_ragged_last_block_counts_valid_keys_only():
    from dsa_b200.progressive_kernel import progressive_scores_triton

    q, w, k = cuda_inputs(65)
    direct = torch.tensor([1, 1], device="cuda", dtype=torch.int8)
    compact = progressive_scores_triton(q, w, k, torch.arange(8), direct, math.inf, compact=True)
    assert compact.candidate_count == 65
    assert compact.candidate_indices.tolist() == list(range(65))


BLOCKS = [16, 32, 64, 128]


@pytest.mark.parametrize("block_size", BLOCKS)
@pytest.mark.parametrize("length", [1, 100, 257, 1000])
def test_h8_block_max_matches_oracle(block_size, length):
    from dsa_b200.progressive_kernel import dynamic_head_ids, h8_block_max_triton

    q, w, k = cuda_inputs(length, seed=length + block_size)
    nb = math.ceil(length / block_size)
    rng = np.random.default_rng(length)
    cold = torch.from_numpy(rng.random(nb) < 0.6)
    heads = dynamic_head_ids(w.cpu())
    partial, maxima = h8_block_max_triton(q, w, k, heads, cold, block_size=block_size)
    wp, wm = oracle.h8_block_max(np32(q), np32(w), np32(k), heads.numpy(), cold.numpy(),
                                 block_size=block_size)
    got_p, got_m = partial.cpu().numpy(), maxima.cpu().numpy()
    np.testing.assert_array_equal(np.isneginf(got_p), np.isneginf(wp))
    np.testing.assert_array_equal(np.isneginf(got_m), np.isneginf(wm))
    fin = np.isfinite(wp)
    scale = normwise_bound(np32(q), np32(w), np32(k))
    assert_scores_close(got_p[fin], wp[fin], scale[fin], rtol=1e-5, atol=1e-7)
    fm = np.isfinite(wm)
    np.testing.assert_allclose(got_m[fm], wm[fm], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("block_size", BLOCKS)
@pytest.mark.parametrize("length", [1, 100, 257, 4099])
def test_masked_full_matches_oracle(block_size, length):
    from dsa_b200.progressive_kernel import masked_full_scores_triton

    q, w, k = cuda_inputs(length, seed=7 * length + block_size)
    nb = math.ceil(length / block_size)
    keep = torch.from_numpy(np.random.default_rng(length).random(nb) < 0.5)
    got = masked_full_scores_triton(q, w, k, keep.cuda(), block_size=block_size).cpu().numpy()
    want = oracle.masked_full_scores(np32(q), np32(w), np32(k), keep.numpy(),
                                     block_size=block_size)
    np.testing.assert_array_equal(np.isneginf(got), np.isneginf(want))
    fin = np.isfinite(want)
    scale = normwise_bound(np32(q), np32(w), np32(k))
    assert_scores_close(got[fin], want[fin], scale[fin], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("block_size", BLOCKS)
@pytest.mark.parametrize("length", [65, 257, 3000])
def test_progressive_matches_oracle(block_size, length):
    from dsa_b200.progressive_kernel import dynamic_head_ids, progressive_scores_triton

    q, w, k = cuda_inputs(length, seed=3 * length + block_size)
    nb = math.ceil(length / block_size)
    rng = np.random.default_rng(block_size)
    direct = torch.from_numpy(rng.random(nb) < 0.3)
    heads = dynamic_head_ids(w.cpu())
    probe = progressive_scores_triton(q, w, k, heads, direct.cuda(), math.inf,
                                      block_size=block_size)
    cold_max = probe.block_max[~direct.cuda()]
    thr = float(torch.quantile(cold_max, 0.6)) if cold_max.numel() else 0.0
    res = progressive_scores_triton(q, w, k, heads, direct.cuda(), thr, block_size=block_size)
    ws, wa, wm = oracle.progressive_scores_fused(np32(q), np32(w), np32(k), heads.numpy(),
                                                 direct.numpy(), thr, block_size=block_size)
    got_a = res.accepted_blocks.cpu().numpy()
    got_m = res.block_max.cpu().numpy()
    fm = np.isfinite(wm)
    np.testing.assert_array_equal(np.isneginf(got_m), np.isneginf(wm))
    np.testing.assert_allclose(got_m[fm], wm[fm], rtol=1e-5, atol=1e-5)
    near = np.abs(wm.astype(np.float64) - thr) <= 1e-5 * max(1.0, abs(thr))
    differ = got_a != wa
    assert not np.any(differ & ~near)
    same = np.repeat(~differ, block_size)[:length]
    got_s = res.scores.cpu().numpy()
    np.testing.assert_array_equal(np.isneginf(got_s[same]), np.isneginf(ws[same]))
    fin = same & np.isfinite(ws)
    scale = normwise_bound(np32(q), np32(w), np32(k))
    assert_scores_close(got_s[fin], ws[fin], scale[fin], rtol=1e-5, atol=1e-7)


def test_progressive_golden_shapes_bf16():
    """The reference's own golden bf16 inputs through every block kernel."""
    from dsa_b200.progressive_kernel import masked_full_scores_triton, progressive_scores_triton

    g = load_golden("progressive_kernel")
    q = torch.from_numpy(bf16_from_bits(g["bf16_q"])).to(torch.bfloat16).cuda()
    w = torch.from_numpy(g["bf16_w"]).cuda()
    for length in (63, 64, 65, 129, 257):
        k = torch.from_numpy(bf16_from_bits(g[f"bf16_L{length}_keys"])).to(torch.bfloat16).cuda()
        nb = math.ceil(length / 64)
        full = g[f"bf16_L{length}_scores"]
        keep = torch.ones(nb, dtype=torch.bool, device="cuda")
        got = masked_full_scores_triton(q, w, k, keep).cpu().numpy()
        np.testing.assert_allclose(got, full, rtol=1e-5, atol=1e-5)
        res = progressive_scores_triton(q, w, k, torch.arange(8), torch.zeros(nb), -math.inf)
        np.testing.assert_allclose(res.scores.cpu().numpy(), full, rtol=1e-5, atol=1e-5)


def test_block_api_errors():
    from dsa_b200.progressive_kernel import h8_block_max_triton, progressive_scores_triton

    q, w, k = cuda_inputs(100)
    with pytest.raises(ValueError):
        h8_block_max_triton(q, w, k, torch.arange(8), torch.ones(3, dtype=torch.bool))
    with pytest.raises(ValueError):
        h8_block_max_triton(q, w, k, torch.arange(8), torch.ones(2, dtype=torch.bool),
                            block_size=48)
    with pytest.raises(ValueError):
        progressive_scores_triton(q, w, k, torch.tensor([0, 1]), torch.zeros(2), 0.0)
    with pytest.raises(ValueError):
        progressive_scores_triton(q, w, k, torch.arange(8).cuda(), torch.zeros(2), 0.0,
                                  remaining_heads=torch.arange(8, 60).cuda())
