"""GPU parity of the fused decode-step key append (tdsa_key_append, sidecar.py:74-76).

RoPE(LayerNorm(hidden @ W_k^T)) for one new token per sequence, written into the key cache
row given by its slot.  Checked against the float64 oracle (``oracle.sidecar.encode_keys``
with the projection rounded to the 16-bit type as the reference's Linear does), against the
reference's own output (golden ``sidecar``), and for cache rows it must leave untouched.
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


def _tol(dtype):
    # one rounding of the stored key plus the float32 RoPE angle at large positions
    # (|y| * 32767 * 2^-23) and a possible one-ulp difference of the rounded projection
    # (dtype independent: ~1.3e-2 for |y| ~ 3 at position 32767)
    return (2 ** -7, 2e-2) if dtype == torch.bfloat16 else (2 ** -10, 2e-2)


def _case(dtype, batch, hidden, length, seed):
    g = torch.Generator().manual_seed(seed)
    wk = (torch.randn(128, hidden, generator=g) * hidden ** -0.5).to(dtype).cuda()
    x = torch.randn(batch, hidden, generator=g).to(dtype).cuda()
    ln_w = (1 + 0.1 * torch.randn(128, generator=g)).cuda()
    ln_b = (0.1 * torch.randn(128, generator=g)).cuda()
    pos = torch.randint(0, 32768, (batch,), generator=g)
    pos[0] = 0
    slots = torch.randint(0, length, (batch,), generator=g)
    cache = torch.randn(batch, length, 128, generator=g).to(dtype).cuda()
    return wk, x, ln_w, ln_b, pos.cuda(), slots.cuda(), cache


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("batch,hidden", [(1, 2048), (3, 16), (64, 2048), (5, 1000),
                                          (130, 2048), (7, 4104)])
def test_key_append_matches_oracle(dtype, batch, hidden):
    from dsa_b200.sidecar import KeyAppender, encode_keys

    length = 300
    wk, x, ln_w, ln_b, pos, slots, cache = _case(dtype, batch, hidden, length, batch + hidden)
    before = cache.clone()
    app = KeyAppender(wk, ln_w, ln_b)
    app.append(x, pos, cache, slots)
    got = cache.float().cpu().numpy()
    ref = before.float().cpu().numpy()
    b_idx = np.arange(batch)
    s_idx = slots.cpu().numpy()
    # every other row is untouched, bit for bit
    mask = np.ones((batch, length), bool)
    mask[b_idx, s_idx] = False
    np.testing.assert_array_equal(got[mask], ref[mask])
    want = osc.encode_keys(x.double().cpu().numpy(), wk.double().cpu().numpy(),
                           pos.cpu().numpy(), ln_w.cpu().numpy(), ln_b.cpu().numpy(),
                           raw_dtype="bf16" if dtype == torch.bfloat16 else "f16")
    rtol, atol = _tol(dtype)
    np.testing.assert_allclose(got[b_idx, s_idx], want, rtol=rtol, atol=atol)
    # the torch composition of the reference's encode_keys
    tk = encode_keys(x, wk, ln_w, ln_b, pos).float().cpu().numpy()
    np.testing.assert_allclose(got[b_idx, s_idx], tk, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("rope_dim", [0, 2, 128])
def test_key_append_rope_dims(rope_dim):
    from dsa_b200.sidecar import KeyAppender

    wk, x, ln_w, ln_b, pos, _, cache = _case(torch.bfloat16, 4, 512, 64, 11)
    pos = torch.tensor([0, 5, 63, 40], device="cuda")
    KeyAppender(wk, ln_w, ln_b, rope_dim=rope_dim, rope_theta=500.0).append(x, pos, cache)
    got = cache[torch.arange(4), pos].float().cpu().numpy()
    want = osc.encode_keys(x.double().cpu().numpy(), wk.double().cpu().numpy(),
                           pos.cpu().numpy(), ln_w.cpu().numpy(), ln_b.cpu().numpy(),
                           rope_dim=rope_dim, theta=500.0, raw_dtype="bf16")
    np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=2e-2)
    if rope_dim == 0:  # no rotation: position 0 and 63 rows are plain LayerNorm outputs
        plain = osc.encode_keys(x.double().cpu().numpy(), wk.double().cpu().numpy(),
                                np.zeros(4), ln_w.cpu().numpy(), ln_b.cpu().numpy(),
                                rope_dim=0, raw_dtype="bf16")
        np.testing.assert_allclose(got, plain, rtol=2 ** -7, atol=2e-2)


def test_key_append_reference_golden():
    """The reference's encode_keys (hidden 16, unit LayerNorm, positions 0..4), on float16
    copies of its float32 inputs."""
    from dsa_b200.sidecar import KeyAppender
    from tests.conftest import load_golden

    g = load_golden("sidecar")
    hk = torch.from_numpy(g["hk"][0]).to(torch.float16).cuda()  # [5, 16]
    wk = torch.from_numpy(g["wk"]).to(torch.float16).cuda()     # [128, 16]
    cache = torch.zeros(5, 8, 128, dtype=torch.float16, device="cuda")
    pos = torch.arange(5, device="cuda")
    KeyAppender(wk).append(hk, pos, cache)
    got = cache[torch.arange(5), pos].float().cpu().numpy()
    np.testing.assert_allclose(got, g["k"][0], rtol=1e-2, atol=2e-2)
    assert torch.count_nonzero(cache[torch.arange(5), pos + 1]) == 0


def test_key_append_slot_out_of_range():
    from dsa_b200 import _capi as capi
    from dsa_b200 import device_status
    from dsa_b200.sidecar import KeyAppender

    wk, x, ln_w, ln_b, pos, _, cache = _case(torch.bfloat16, 3, 256, 16, 3)
    before = cache.clone()
    slots = torch.tensor([2, 16, 5], device="cuda")
    KeyAppender(wk, ln_w, ln_b).append(x, pos, cache, slots)
    assert device_status(reset=True) & capi.TDSA_STATUS_RANGE
    assert torch.equal(cache[1], before[1])
    assert not torch.equal(cache[0, 2], before[0, 2]) and not torch.equal(cache[2, 5],
                                                                          before[2, 5])
    assert device_status() == 0


def test_key_append_rejects_bad_arguments():
    from dsa_b200 import _capi as capi

    lib = capi.lib()
    bf = capi.TDSA_BF16
    # hidden size not a multiple of 8
    assert lib.tdsa_key_append(16, 12, 12, 16, 12, None, None, 1e-6, 16, None, 16, 128 * 4,
                               128, 4, bf, 1, 64, 1e4, None) == capi.TDSA_ERR_UNSUPPORTED
    # odd rope_dim
    assert lib.tdsa_key_append(16, 16, 16, 16, 16, None, None, 1e-6, 16, None, 16, 128 * 4,
                               128, 4, bf, 1, 63, 1e4, None) == capi.TDSA_ERR_INVALID
    # misaligned w_k
    assert lib.tdsa_key_append(16, 16, 16, 24, 16, None, None, 1e-6, 16, None, 16, 128 * 4,
                               128, 4, bf, 1, 64, 1e4, None) == capi.TDSA_ERR_ALIGN
    # cache rows narrower than 128
    assert lib.tdsa_key_append(16, 16, 16, 16, 16, None, None, 1e-6, 16, None, 16, 64 * 4,
                               64, 4, bf, 1, 64, 1e4, None) == capi.TDSA_ERR_INVALID
    # f32 is not a key-cache type here
    assert lib.tdsa_key_append(16, 16, 16, 16, 16, None, None, 1e-6, 16, None, 16, 128 * 4,
                               128, 4, capi.TDSA_F32, 1, 64, 1e4, None) == capi.TDSA_ERR_INVALID
