"""GPU parity of the decode-step query projection (reference sidecar.py:78-87).

tdsa_query_project (W_q GEMM on tcgen05 + RoPE + float32 head weights, one launch) against
float64 products and the oracle's RoPE; tdsa_query_prep (RoPE + head weights on a given
W_q output) against the same oracle.
"""

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
    yield
    from dsa_b200 import device_status

    assert device_status() == 0


def _inputs(dtype, batch, hidden, seed=5):
    g = torch.Generator().manual_seed(seed)
    wq = (torch.randn(8192, hidden, generator=g) * hidden ** -0.5).to(dtype).cuda()
    ww = (torch.randn(64, hidden, generator=g) * hidden ** -0.5).cuda()
    x = torch.randn(batch, hidden, generator=g).to(dtype).cuda()
    pos = torch.randint(0, 32768, (batch,), generator=g)
    pos[0] = 0
    pos[-1] = 32767
    return wq, ww, x, pos.cuda()


def _check_rope(q, qraw, pos, dtype):
    """RoPE on the projection's own 16-bit output: float32 math, one final rounding.  The
    float32 angle pos * inv_freq is only good to ~pos * 2^-23 rad (one ulp of inv_freq,
    which CUDA's powf and numpy may round differently), so large positions get
    |x| * 32767 * 2^-23 ~ 1.5e-2; the rest is held to the 16-bit rounding."""
    want = osc.rope_heads(qraw.float().cpu().numpy(), pos.cpu().numpy())
    got = q.float().cpu().numpy()
    rtol = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    small = pos.cpu().numpy() < 64
    np.testing.assert_allclose(got[small], want[small], rtol=rtol, atol=1e-4)
    np.testing.assert_allclose(got[~small], want[~small], rtol=rtol, atol=2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("batch,hidden", [(3, 512), (64, 2048), (5, 64), (40, 1000), (130, 1000),
                                          (300, 2048)])
@pytest.mark.parametrize("packed", [True, False])
def test_query_project_matches_oracle(dtype, batch, hidden, packed):
    from dsa_b200.sidecar import QueryProjector, encode_queries

    wq, ww, x, pos = _inputs(dtype, batch, hidden, seed=batch + hidden)
    proj = QueryProjector(wq, ww, batch, keep_qraw=True, packed=packed)
    q, w = proj.project(x, pos)
    x64 = x.double().cpu().numpy()
    # the GEMM output rounded once to the 16-bit dtype (accumulation order differs)
    raw64 = x64 @ wq.double().cpu().numpy().T
    rtol = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    np.testing.assert_allclose(proj.qraw.double().cpu().numpy(), raw64, rtol=rtol,
                               atol=rtol * np.abs(raw64).max() * 1e-2)
    _check_rope(q, proj.qraw, pos, dtype)
    want_w = (x64 @ ww.double().cpu().numpy().T) * (64 * 128) ** -0.5
    np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=1e-5, atol=1e-6)
    # the torch restatement of the reference's encode_queries
    tq, tw = encode_queries(x, wq, ww, pos)
    np.testing.assert_allclose(q.float().cpu().numpy(), tq.float().cpu().numpy(), rtol=2e-2,
                               atol=2e-2)
    np.testing.assert_allclose(w.cpu().numpy(), tw.cpu().numpy(), rtol=1e-5, atol=1e-6)
    # a second call on the same buffers gives the same result
    q2, w2 = proj.project(x, pos)
    assert torch.equal(q2, q) and torch.equal(w2, w)


def test_rope_only_on_first_64_dims():
    from dsa_b200.sidecar import QueryProjector

    wq = torch.zeros(8192, 64, dtype=torch.bfloat16, device="cuda")
    for h in range(64):
        wq[h * 128: (h + 1) * 128, :] = torch.eye(128, 64, dtype=torch.bfloat16, device="cuda")
    ww = torch.zeros(64, 64, device="cuda")
    x = torch.arange(1, 65, dtype=torch.bfloat16, device="cuda")[None] / 64
    proj = QueryProjector(wq, ww, 1, keep_qraw=True)
    q, _ = proj.project(x, torch.tensor([0], device="cuda"))
    # position 0: RoPE is the identity
    torch.testing.assert_close(q[0], proj.qraw.view(64, 128))
    q, _ = proj.project(x, torch.tensor([9], device="cuda"))
    torch.testing.assert_close(q[0, :, 64:], proj.qraw.view(64, 128)[:, 64:])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_query_prep_tail_matches_oracle(dtype):
    from dsa_b200 import _capi as capi

    wq, ww, x, pos = _inputs(dtype, 3, 512)
    qraw = x @ wq.t()
    q = torch.empty(3, 64, 128, dtype=dtype, device="cuda")
    w = torch.empty(3, 64, device="cuda")
    capi.call("tdsa_query_prep", qraw.data_ptr(), qraw.stride(0), x.data_ptr(), x.stride(0),
              512, ww.data_ptr(), pos.data_ptr(), q.data_ptr(), 8192, w.data_ptr(), 64,
              capi.TDSA_BF16 if dtype == torch.bfloat16 else capi.TDSA_F16, 3, 64, 10000.0,
              (64 * 128) ** -0.5, torch.cuda.current_stream().cuda_stream)
    _check_rope(q, qraw, pos, dtype)
    want_w = (x.double().cpu().numpy() @ ww.double().cpu().numpy().T) * (64 * 128) ** -0.5
    np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=1e-5, atol=1e-6)


def test_query_project_rejects_bad_arguments():
    from dsa_b200 import _capi as capi

    lib = capi.lib()
    # hidden size not a multiple of 8
    rc = lib.tdsa_query_project(16, 12, 12, 16, 12, 0, 16, 16, 16, 8192, 16, 64, capi.TDSA_BF16,
                                1, 64, 1e4, 1.0, None, 0, None)
    assert rc == capi.TDSA_ERR_UNSUPPORTED
    # odd rope_dim
    rc = lib.tdsa_query_project(16, 64, 64, 16, 64, 0, 16, 16, 16, 8192, 16, 64, capi.TDSA_BF16,
                                1, 63, 1e4, 1.0, None, 0, None)
    assert rc == capi.TDSA_ERR_INVALID
    # misaligned hidden pointer
    rc = lib.tdsa_query_project(18, 64, 64, 16, 64, 0, 16, 16, 16, 8192, 16, 64, capi.TDSA_BF16,
                                1, 64, 1e4, 1.0, None, 0, None)
    assert rc == capi.TDSA_ERR_ALIGN
