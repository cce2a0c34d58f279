"""tdsa_score_topk_noalloc (static device scratch, no allocation) against tdsa_score_topk.

Collected last on purpose: it must pass alone and after every other test has run on the
same device.
"""

from __future__ import annotations

import math

import pytest
import torch

from dsa_b200 import _capi as capi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()


def _inputs(batch, length, seed):
    gen = torch.Generator().manual_seed(seed)
    q = (torch.randn(batch, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16).cuda()
    w = (torch.randn(batch, 64, generator=gen) / 8).cuda()
    keys = torch.randn(batch, length, 128, generator=gen).to(torch.bfloat16).cuda()
    return q, w, keys


def _args(q, w, keys, k, sorted_, idx, val):
    b, length = keys.shape[0], keys.shape[1]
    return [q.data_ptr(), q.stride(0), w.data_ptr(), w.stride(0), keys.data_ptr(),
            keys.stride(0), keys.stride(1), capi.TDSA_BF16, b, length, k, int(sorted_),
            idx.data_ptr(), idx.element_size(), idx.stride(0), val.data_ptr(), val.stride(0)]


def _with_workspace(q, w, keys, k, sorted_):
    b, length = keys.shape[0], keys.shape[1]
    idx = torch.empty(b, k, dtype=torch.int64, device="cuda")
    val = torch.empty(b, k, dtype=torch.float32, device="cuda")
    nbytes = capi.lib().tdsa_score_topk_workspace_bytes(b, length, k)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    capi.call("tdsa_score_topk", *_args(q, w, keys, k, sorted_, idx, val), ws.data_ptr(), nbytes,
              stream)
    return idx, val


def _no_alloc(q, w, keys, k, sorted_):
    b = keys.shape[0]
    idx = torch.empty(b, k, dtype=torch.int64, device="cuda")
    val = torch.empty(b, k, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    capi.call("tdsa_score_topk_noalloc", *_args(q, w, keys, k, sorted_, idx, val), stream)
    return idx, val


@pytest.mark.parametrize("batch,length,k,sorted_", [(2, 3000, 256, True),
                                                     (64, 32768, 2048, False),
                                                     (3, 100000, 2048, True)])
def test_no_alloc_matches_workspace_entry_point_twice_in_a_row(batch, length, k, sorted_):
    q, w, keys = _inputs(batch, length, seed=batch + length)
    want_i, want_v = _with_workspace(q, w, keys, k, sorted_)
    for call in range(2):  # the second call reuses the scratch the first one left behind
        got_i, got_v = _no_alloc(q, w, keys, k, sorted_)
        torch.cuda.synchronize()
        assert torch.equal(got_i, want_i), f"call {call}: indices differ"
        assert torch.equal(got_v, want_v), f"call {call}: values differ"
    from dsa_b200 import device_status

    assert device_status() == 0


def test_no_alloc_rejects_calls_beyond_the_static_scratch():
    q, w, keys = _inputs(1, 16, seed=0)
    idx = torch.empty(1, 16, dtype=torch.int64, device="cuda")
    val = torch.empty(1, 16, dtype=torch.float32, device="cuda")
    args = _args(q, w, keys, 16, True, idx, val)
    args[8], args[9] = 128, 32768  # batch 128 x length 32768 needs 18 MiB of scratch
    assert capi.lib().tdsa_score_topk_workspace_bytes(128, 32768, 16) > 16 << 20
    rc = capi.lib().tdsa_score_topk_noalloc(*args, torch.cuda.current_stream().cuda_stream)
    assert rc == capi.TDSA_ERR_UNSUPPORTED
    assert "static scratch" in capi.last_error()
