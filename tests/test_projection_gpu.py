"""GPU parity of the fused query epilogue (RoPE + head-weight scale) of the projection."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sidecar as osc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_query_projector_matches_oracle(dtype):
    from dsa_b200.sidecar import QueryProjector, encode_queries

    g = torch.Generator().manual_seed(5)
    hidden = 512
    wq = (torch.randn(8192, hidden, generator=g) * hidden ** -0.5).to(dtype).cuda()
    ww = (torch.randn(64, hidden, generator=g) * hidden ** -0.5).cuda()
    x = torch.randn(3, hidden, generator=g).to(dtype).cuda()
    pos = torch.tensor([0, 17, 32767], device="cuda")
    proj = QueryProjector(wq, ww, 3)
    q, w = proj.project(x, pos)
    # RoPE on the GEMM's own output: float32 math, one final rounding to the 16-bit dtype.
    # The float32 angle pos * inv_freq is only good to ~pos * 2^-23 rad (one ulp of
    # inv_freq, which CUDA's powf and numpy may round differently), so the tolerance at
    # position 32767 is |x| * 32767 * 2^-23 ~ 1.5e-2; small positions are held to 2^-7.
    want_q = osc.rope_heads(proj.qraw.float().cpu().numpy(), pos.cpu().numpy())
    got_q = q.float().cpu().numpy()
    np.testing.assert_allclose(got_q[:2], want_q[:2], rtol=2 ** -7, atol=1e-4)
    np.testing.assert_allclose(got_q[2], want_q[2], rtol=2 ** -7, atol=2e-2)
    want_w = (x.float().cpu().numpy().astype(np.float64) @ ww.cpu().numpy().T.astype(np.float64)
              ) * (64 * 128) ** -0.5
    np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=1e-5, atol=1e-6)
    # against the torch restatement of the reference's encode_queries
    tq, tw = encode_queries(x, wq, ww, pos)
    np.testing.assert_allclose(q.float().cpu().numpy(), tq.float().cpu().numpy(), rtol=2e-2,
                               atol=2e-2)
    np.testing.assert_allclose(w.cpu().numpy(), tw.cpu().numpy(), rtol=1e-5, atol=1e-6)


def test_rope_only_on_first_64_dims():
    from dsa_b200.sidecar import QueryProjector

    wq = torch.zeros(8192, 64, dtype=torch.bfloat16, device="cuda")
    for h in range(64):
        wq[h * 128: (h + 1) * 128, :] = torch.eye(128, 64, dtype=torch.bfloat16, device="cuda")
    ww = torch.zeros(64, 64, device="cuda")
    x = torch.arange(1, 65, dtype=torch.bfloat16, device="cuda")[None] / 64
    proj = QueryProjector(wq, ww, 1)
    q, _ = proj.project(x, torch.tensor([0], device="cuda"))
    # position 0: RoPE is the identity
    torch.testing.assert_close(q[0], proj.qraw.view(64, 128))
    q, _ = proj.project(x, torch.tensor([9], device="cuda"))
    torch.testing.assert_close(q[0, :, 64:], proj.qraw.view(64, 128)[:, 64:])
