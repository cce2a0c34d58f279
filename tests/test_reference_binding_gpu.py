"""The drop-in boundary exercised with the reference itself imported (its unmodified offline
install under ``baseline/_ref``; skipped when absent).

1. The sidecar mixin of the integration guide, ``B200Sidecar(SidecarScoring,
   LightningIndexerSidecar)``: its ``score_encoded`` (this library's kernel) against the
   reference module's own ``score_encoded`` (src/temporal_dsa/sidecar.py:89-107) on the same
   CUDA tensors, and the module's other methods left as the reference's.
2. Every function of ``temporal_dsa.progressive_kernel`` (its Triton kernels and torch
   references, :45-90 and :362-497) against ``dsa_b200.progressive_kernel`` on the same
   CUDA inputs.
3. The reference's own tests/test_progressive_kernel.py run unchanged by pytest with the
   name ``temporal_dsa.progressive_kernel`` bound to ``dsa_b200.progressive_kernel``
   (tests/_reference_binding.py).  Its four cases that pass float32 CPU tensors to the
   torch_* functions are deselected: those functions double as the reference's CPU
   implementation, and this library has no CPU path.

Tolerances: float32 inputs 1e-5 norm-wise (relative to sum_h |w_h| |q_h . k|); 16-bit
inputs 1e-2 relative (the reference's einsum rounds head dots to 16 bits, its Triton
kernels accumulate 16-bit products in float32 like these kernels, held to 1e-5 norm-wise).
"""

from __future__ import annotations

import math
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from tests._util import assert_scores_close, normwise_bound

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
REF_TESTS = REF / "reference_tests" / "test_progressive_kernel.py"
CPU_ONLY_CASES = ("test_torch_full_scores_matches_explicit_sum",
                  "test_torch_progressive_all_promoted_equals_full",
                  "test_torch_progressive_rejects_cold_blocks",
                  "test_torch_progressive_handles_ragged_last_block")


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not (REF / "temporal_dsa").is_dir():
        pytest.skip("the reference's offline install (baseline/_ref) is absent")
    from dsa_b200.build import build

    build()
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    yield
    from dsa_b200 import device_status

    assert device_status() == 0


def _inputs(length, dtype=torch.bfloat16, seed=0, batch=None):
    g = torch.Generator().manual_seed(seed)
    shape_q = (64, 128) if batch is None else (batch, 64, 128)
    shape_w = (64,) if batch is None else (batch, 64)
    shape_k = (length, 128) if batch is None else (batch, length, 128)
    q = (torch.randn(*shape_q, generator=g) / math.sqrt(128)).to(dtype).cuda()
    w = (torch.randn(*shape_w, generator=g) / 8).cuda()
    k = torch.randn(*shape_k, generator=g).to(dtype).cuda()
    return q, w, k


def _close(got, want, q, w, k, rtol=1e-5):
    got, want = got.float().cpu().numpy(), want.float().cpu().numpy()
    fin = np.isfinite(want)
    np.testing.assert_array_equal(np.isfinite(got), fin)
    np.testing.assert_array_equal(got[~fin], want[~fin])
    scale = normwise_bound(q.float().cpu().numpy(), w.float().cpu().numpy(),
                           k.float().cpu().numpy())
    assert_scores_close(got[fin], want[fin], scale[fin], rtol=rtol, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_b200_sidecar_mixin_against_reference_module(dtype):
    from temporal_dsa.sidecar import LightningIndexerSidecar

    from dsa_b200.sidecar import SidecarScoring

    class B200Sidecar(SidecarScoring, LightningIndexerSidecar):
        pass

    torch.manual_seed(0)
    ours = B200Sidecar().cuda()
    ref = LightningIndexerSidecar().cuda()
    ref.load_state_dict(ours.state_dict())
    b, nq, length = 3, 2, 1000
    g = torch.Generator().manual_seed(7)
    hidden = torch.randn(b, nq, 2048, generator=g).cuda()
    pos = torch.arange(nq).repeat(b, 1).cuda() + 500
    with torch.no_grad():
        q, w = ref.encode_queries(hidden, pos)
        # the methods other than score_encoded stay the reference's
        q2, w2 = ours.encode_queries(hidden, pos)
        assert torch.equal(q, q2) and torch.equal(w, w2)
        keys = torch.randn(b, length, 128, generator=g).cuda()
        q, keys = q.to(dtype), keys.to(dtype)
        got = ours.score_encoded(q, w, keys, key_chunk_size=256)
        want = ref.score_encoded(q, w, keys, key_chunk_size=256)
    assert got.shape == want.shape == (b, nq, length) and got.dtype == torch.float32
    if dtype == torch.float32:
        for i in range(b):
            for j in range(nq):
                _close(got[i, j], want[i, j], q[i, j], w[i, j], keys[i])
    else:
        np.testing.assert_allclose(got.cpu().numpy(), want.float().cpu().numpy(),
                                   rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("length", [1, 100, 257, 4096, 32768])
def test_progressive_kernel_functions_against_reference(length):
    from temporal_dsa import progressive_kernel as ref

    from dsa_b200 import progressive_kernel as ours

    q, w, k = _inputs(length, seed=length)
    bs = 64
    nb = math.ceil(length / bs)
    g = torch.Generator().manual_seed(length + 1)
    direct = (torch.rand(nb, generator=g) < 0.4).to(torch.int8).cuda()
    heads = ref.dynamic_head_ids(w.cpu())
    assert torch.equal(heads, ours.dynamic_head_ids(w.cpu()))
    sel_r, rem_r = ref.split_head_ids(heads)
    sel_o, rem_o = ours.split_head_ids(heads)
    assert torch.equal(sel_r, sel_o) and torch.equal(rem_r, rem_o)

    _close(ours.full_scores_triton(q, w, k), ref.full_scores_triton(q, w, k), q, w, k)
    _close(ours.torch_full_scores(q, w, k), ref.torch_full_scores(q, w, k), q, w, k)

    cold = direct == 0
    p_o, m_o = ours.h8_block_max_triton(q, w, k, heads, cold, block_size=bs)
    p_r, m_r = ref.h8_block_max_triton(q, w, k, heads, cold, block_size=bs)
    _close(p_o, p_r, q, w, k)
    fin = torch.isfinite(m_r)
    assert torch.equal(fin, torch.isfinite(m_o))
    np.testing.assert_allclose(m_o[fin].cpu().numpy(), m_r[fin].cpu().numpy(), rtol=1e-4,
                               atol=1e-5)

    keep = direct.bool() | (torch.rand(nb, generator=g) < 0.5).cuda()
    _close(ours.masked_full_scores_triton(q, w, k, keep, block_size=bs),
           ref.masked_full_scores_triton(q, w, k, keep, block_size=bs), q, w, k)

    # a threshold between probe maxima, away from any block's own maximum (a maximum equal
    # to the threshold could round either way in the two implementations)
    vals = m_r[cold & fin].sort().values if bool((cold & fin).any()) else None
    if vals is not None and vals.numel() >= 2:
        mid = vals.numel() // 2
        thr = float((vals[mid - 1] + vals[mid]) / 2)
    else:
        thr = 0.0
    r_o = ours.progressive_scores_triton(q, w, k, heads, direct, thr, block_size=bs)
    r_r = ref.progressive_scores_triton(q, w, k, heads, direct, thr, block_size=bs)
    assert torch.equal(r_o.accepted_blocks.to(torch.int8), r_r.accepted_blocks.to(torch.int8))
    _close(r_o.scores, r_r.scores, q, w, k)
    c_o = ours.progressive_scores_triton(q, w, k, heads, direct, thr, block_size=bs,
                                         compact=True)
    c_r = ref.progressive_scores_triton(q, w, k, heads, direct, thr, block_size=bs,
                                        compact=True)
    assert c_o.candidate_count == c_r.candidate_count
    o_r = torch.argsort(c_r.candidate_indices.long())
    assert torch.equal(c_o.candidate_indices.long(), c_r.candidate_indices.long()[o_r])
    _close(c_o.scores, c_r.scores[o_r], q, w, k[c_o.candidate_indices.long()])

    t_o = ours.two_pass_scores_triton(q, w, k, heads, direct, thr, block_size=bs)
    t_r = ref.two_pass_scores_triton(q, w, k, heads, direct, thr, block_size=bs)
    assert torch.equal(t_o.accepted_blocks.bool(), t_r.accepted_blocks.bool())
    _close(t_o.scores, t_r.scores, q, w, k)

    s_o, a_o, bm_o = ours.torch_progressive_scores(q, w, k, heads, direct.bool(), thr,
                                                   block_size=bs)
    s_r, a_r, bm_r = ref.torch_progressive_scores(q, w, k, heads, direct.bool(), thr,
                                                  block_size=bs)
    assert torch.equal(a_o.bool(), a_r.bool())
    np.testing.assert_allclose(bm_o.cpu().numpy(), bm_r.cpu().numpy(), rtol=1e-4, atol=1e-5)
    _close(s_o, s_r, q, w, k)

    assert ours.progressive_qk_reduction(length, nb // 3, nb // 4) == \
        ref.progressive_qk_reduction(length, nb // 3, nb // 4)


def test_reference_test_file_runs_against_the_b200_module():
    if not REF_TESTS.exists():
        pytest.skip("the reference's tests are not beside its install "
                    "(baseline/_ref/reference_tests)")
    cmd = [sys.executable, "-m", "pytest", str(REF_TESTS), "-q", "-p", "no:cacheprovider",
           "-p", "tests._reference_binding", "-k",
           " and ".join(f"not {name}" for name in CPU_ONLY_CASES)]
    run = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env=dict(os.environ, PYTHONPATH=str(ROOT)))
    assert run.returncode == 0, run.stdout[-4000:] + run.stderr[-2000:]
    assert " passed" in run.stdout and "skipped" not in run.stdout, run.stdout[-2000:]
