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
