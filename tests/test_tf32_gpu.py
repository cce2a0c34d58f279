"""GPU parity of the float32 scoring path on the tensor cores (error-compensated TF32).

``tdsa_score_dense`` with float32 queries and keys runs ``score_dense_tf32_kernel``
(q_hi.k_hi + q_lo.k_hi + q_hi.k_lo per product) when the layout admits TMA and the FP32
CUDA-core kernel otherwise.  Both are held to the float64 oracle at the FP32 bar (1e-5,
norm-wise: relative to sum_h |w_h| |q_h . k|), and the TF32 kernel to a 4e-6 bound that the
uncompensated TF32 product (2^-11 ~ 4.9e-4 relative per operand) misses by two orders of
magnitude -- so a change in how the tensor cores read float32 operands (the residuals
assume the low 13 mantissa bits are dropped) fails here.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from tests._util import assert_scores_close, normwise_bound

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()
    yield
    from dsa_b200 import device_status

    assert device_status() == 0, "a kernel raised a device status bit"


def inputs(batch, length, seed, key_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, 64, 128, generator=g) / math.sqrt(128)
    w = torch.randn(batch, 64, generator=g) / 8
    k = torch.randn(batch, length, 128, generator=g) * key_scale
    return q, w, k


def oracle_scores(q, w, k):
    """float64 scores of the float32 inputs."""
    return np.stack([oracle.relu_index_score(q[b].numpy(), k[b].numpy(), w[b].numpy())
                     for b in range(q.shape[0])])


@pytest.mark.parametrize("batch,length", [(1, 1), (1, 100), (1, 128), (1, 129), (1, 4096),
                                          (3, 4099), (2, 32768)])
def test_tf32_scores_match_float64(batch, length):
    from dsa_b200 import score_dense

    q, w, k = inputs(batch, length, length + batch)
    got = score_dense(q.cuda(), w.cuda(), k.cuda()).cpu().numpy()
    want = oracle_scores(q, w, k)
    for b in range(batch):
        scale = normwise_bound(q[b].numpy(), w[b].numpy(), k[b].numpy())
        assert_scores_close(got[b], want[b], scale, rtol=4e-6, atol=1e-30, msg=f"row {b}")


def test_tf32_wide_dynamic_range_and_low_bits():
    """Keys spanning 2^-20 .. 2^20 per element, and values whose bits below TF32 precision
    carry the answer (1 + 2^-11 + 2^-12 patterns)."""
    from dsa_b200 import score_dense

    g = torch.Generator().manual_seed(5)
    length = 3000
    q = torch.randn(1, 64, 128, generator=g)
    w = torch.randn(1, 64, generator=g)
    exps = torch.randint(-20, 21, (1, length, 128), generator=g).float()
    k = torch.randn(1, length, 128, generator=g) * torch.pow(2.0, exps)
    k[0, :500] = 1.0 + 2.0 ** -11 + 2.0 ** -12 * torch.randint(0, 2, (500, 128), generator=g)
    q[0, :8] = 1.0 + 2.0 ** -11 + 2.0 ** -13
    got = score_dense(q.cuda(), w.cuda(), k.cuda()).cpu().numpy()
    want = oracle_scores(q, w, k)
    scale = normwise_bound(q[0].numpy(), w[0].numpy(), k[0].numpy())
    assert_scores_close(got[0], want[0], scale, rtol=4e-6, atol=1e-30, msg="range")


def test_tf32_strided_batch_and_simt_fallback_agree():
    """Keys inside a wider row (stride 132 floats: tensor cores) and an odd stride (129:
    the FP32 CUDA-core kernel) give the same scores within the FP32 bar."""
    from dsa_b200 import score_dense

    q, w, k = inputs(3, 2000, 11)
    want = oracle_scores(q, w, k)
    for stride in (132, 129):
        buf = torch.zeros(3, 2000, stride)
        buf[:, :, :128] = k
        kc = buf.cuda()[:, :, :128]
        got = score_dense(q.cuda(), w.cuda(), kc).cpu().numpy()
        for b in range(3):
            scale = normwise_bound(q[b].numpy(), w[b].numpy(), k[b].numpy())
            assert_scores_close(got[b], want[b], scale, rtol=1e-5, atol=1e-30,
                                msg=f"stride {stride} row {b}")


def test_tf32_topk_through_scores_topk():
    """scores_topk on float32 keys (config 1's dtype) returns stable_topk of its own scores."""
    from dsa_b200 import score_dense, scores_topk

    q, w, k = inputs(2, 9000, 3)
    idx, val = scores_topk(q.cuda(), w.cuda(), k.cuda(), 512, sorted=True)
    s = score_dense(q.cuda(), w.cuda(), k.cuda()).cpu().numpy()
    for b in range(2):
        np.testing.assert_array_equal(idx[b].cpu().numpy(), oracle.stable_topk(s[b], 512))
        np.testing.assert_array_equal(val[b].cpu().numpy(), s[b][idx[b].cpu().numpy()])
