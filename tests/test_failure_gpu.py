"""Failure detection on the GPU without a fault: a wait that can never complete gives up
after its limit, the device status word reports TDSA_ERR_TIMEOUT, and the context keeps
working (the next scoring call is correct)."""

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


def test_bounded_wait_times_out_and_reports_status():
    from dsa_b200 import _capi as capi
    from dsa_b200 import device_status, score_dense

    assert device_status(reset=True) == 0
    capi.call("tdsa_selftest_bounded_wait", 200_000, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert device_status(reset=True) == capi.TDSA_ERR_TIMEOUT
    assert device_status(reset=False) == 0  # the read above cleared it
    # the context is intact: a normal call still gives the right scores
    gen = torch.Generator().manual_seed(1)
    q = (torch.randn(64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16)
    w = torch.randn(64, generator=gen) / 8
    k = torch.randn(1000, 128, generator=gen).to(torch.bfloat16)
    got = score_dense(q.cuda(), w.cuda(), k.cuda()).cpu().numpy()
    qf, kf = q.float().numpy(), k.float().numpy()
    assert_scores_close(got, oracle.full_scores(qf, w.numpy(), kf),
                        normwise_bound(qf, w.numpy(), kf), rtol=1e-5, atol=1e-7)
    assert device_status(reset=True) == 0


def test_selftest_rejects_bad_limit():
    from dsa_b200 import _capi as capi

    assert capi.lib().tdsa_selftest_bounded_wait(-1, None) == capi.TDSA_ERR_INVALID


def test_exchange_wait_for_a_silent_peer_times_out():
    """A two-rank peer exchange whose other rank (a helper process holding its region on the
    same GPU, launching nothing) never publishes: each row's bounded wait gives up after
    about a second, the device status word reports TDSA_ERR_TIMEOUT, and the context keeps
    working.  Only this process launches a kernel that waits."""
    import ctypes as C
    import os
    import subprocess
    import sys

    from dsa_b200 import _capi as capi
    from dsa_b200 import device_status, topk

    rows, k = 2, 64
    helper = os.path.join(os.path.dirname(__file__), "_exchange_silent_peer.py")
    proc = subprocess.Popen([sys.executable, helper, str(rows), str(k)],
                            stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True)
    lib = capi.lib()
    ex = C.c_void_p()
    try:
        peer_handle = bytes.fromhex(proc.stdout.readline().strip())
        assert len(peer_handle) == capi.TDSA_IPC_HANDLE_BYTES
        mine = (C.c_uint8 * capi.TDSA_IPC_HANDLE_BYTES)()
        capi.call("tdsa_exchange_create", 2, 0, rows, k, C.byref(ex), mine)
        capi.call("tdsa_exchange_connect", ex, bytes(mine) + peer_handle)
        assert device_status(reset=True) == 0
        vals = torch.randn(rows, k, device="cuda")
        idx = torch.arange(rows * k, dtype=torch.int32, device="cuda").view(rows, k) % k
        out_i = torch.empty(rows, k, dtype=torch.int64, device="cuda")
        out_v = torch.empty(rows, k, device="cuda")
        capi.call("tdsa_exchange_topk", ex, vals.data_ptr(), idx.data_ptr(), k, 0, 0,
                  out_i.data_ptr(), 8, k, out_v.data_ptr(), k,
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert device_status(reset=True) == capi.TDSA_ERR_TIMEOUT
        # the context is intact
        x = torch.randn(3, 5000, device="cuda")
        got_i, got_v = topk(x, 100, sorted=True)
        want_v, _ = torch.sort(x, dim=1, descending=True)
        assert torch.equal(got_v, want_v[:, :100])
        assert device_status(reset=True) == 0
    finally:
        if ex.value:
            torch.cuda.synchronize()
            lib.tdsa_exchange_destroy(ex)
        proc.stdin.write("done\n")
        proc.stdin.flush()
        proc.wait(timeout=60)
    assert proc.returncode == 0
