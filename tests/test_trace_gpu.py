"""GPU parity of score-trace emission (tdsa_score_dense_trace).

The score kernel writes each step's float16 trace row itself.  Rows must equal the
reference writer's rows built from the kernel's own float32 scores (``oracle.trace_matrix``,
training.py:166-178): bit-exact float16, -inf beyond each row's length, values past the
float16 range as +-inf.  The float32 scores are checked against the oracle's dense scores
(norm-wise rtol 1e-5), and a recorded trace round-trips through save_trace / load_trace.
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

    assert device_status() == 0


def _inputs(batch, length, dtype, seed, w_scale=1 / 8):
    gen = torch.Generator().manual_seed(seed)
    q = (torch.randn(batch, 64, 128, generator=gen) / math.sqrt(128)).to(dtype)
    w = torch.randn(batch, 64, generator=gen) * w_scale
    k = torch.randn(batch, length, 128, generator=gen).to(dtype)
    return q, w, k


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_score_trace_rows(dtype):
    from dsa_b200.trace import TraceRecorder, score_trace

    batch, max_len = 3, 520
    lengths = [100, 129, 517, 1, 256]
    q, w, k = _inputs(batch, max_len, dtype, seed=5)
    kd = k.cuda()
    rec = TraceRecorder(batch, len(lengths) + 1, max_len, "cuda")
    f32_rows = [[] for _ in range(batch)]
    for step, length in enumerate(lengths):
        got = score_trace(q.cuda(), w.cuda(), kd[:, :length], rec).cpu().numpy()
        for b in range(batch):
            qf, kf = q[b].float().numpy(), k[b, :length].float().numpy()
            assert_scores_close(got[b], oracle.full_scores(qf, w[b].numpy(), kf),
                                normwise_bound(qf, w[b].numpy(), kf), rtol=1e-5, atol=1e-7,
                                msg=f"{dtype} b={b} L={length}")
            f32_rows[b].append(got[b])
    assert rec.step == len(lengths) and rec.lengths[: rec.step].tolist() == lengths
    buf = rec.buffer.cpu().numpy()
    for b in range(batch):
        want, want_len = oracle.trace_matrix(f32_rows[b])
        np.testing.assert_array_equal(want_len, lengths)
        np.testing.assert_array_equal(buf[b, : len(lengths), : want.shape[1]].view(np.uint16),
                                      want.view(np.uint16))
        assert np.all(buf[b, : len(lengths), want.shape[1]:] == -np.inf)
        assert np.all(buf[b, len(lengths):] == -np.inf)  # the unrecorded step


def test_trace_overflow_and_rounding():
    """Scores past the float16 range become +-inf, others round to nearest even."""
    from dsa_b200.trace import TraceRecorder, score_trace

    q, w, k = _inputs(2, 700, torch.bfloat16, seed=9, w_scale=3e4)
    rec = TraceRecorder(2, 1, 700, "cuda")
    got = score_trace(q.cuda(), w.cuda(), k.cuda(), rec).cpu().numpy()
    assert np.abs(got).max() > 65520.0, "the case must reach past the float16 range"
    with np.errstate(over="ignore"):
        want = got.astype(np.float16)
    np.testing.assert_array_equal(rec.buffer[:, 0].cpu().numpy().view(np.uint16),
                                  want.view(np.uint16))


@pytest.mark.parametrize("length", [4096, 40000])
def test_plan_records_trace(tmp_path, length):
    """ScoreTopkPlan with a recorder: same top-k as without, trace rows from the kernel,
    one ScoreTrace per sequence that survives save_trace / load_trace."""
    from dsa_b200.indexer import ScoreTopkPlan
    from dsa_b200.trace import TraceRecorder, load_trace, save_trace

    batch, steps, kk = 2, 3, 512
    q, w, k = _inputs(batch, length, torch.bfloat16, seed=length)
    qd, wd, kd = q.cuda(), w.cuda(), k.cuda()
    rec = TraceRecorder(batch, steps, length, "cuda")
    plan = ScoreTopkPlan(qd, wd, kd, kk, sorted=True, trace=rec)
    plain = ScoreTopkPlan(qd.clone(), wd.clone(), kd, kk, sorted=True)
    gen = torch.Generator().manual_seed(1)
    rows = [[] for _ in range(batch)]
    for _ in range(steps):
        fresh = torch.randn(batch, 64, 128, generator=gen) / math.sqrt(128)
        fresh = fresh.to(torch.bfloat16)
        plan.q.copy_(fresh.cuda())
        plain.q.copy_(fresh.cuda())
        idx, val = plan.run()
        pidx, pval = plain.run()
        assert torch.equal(idx, pidx) and torch.equal(val, pval)
        for b in range(batch):
            rows[b].append(plan.scores[b].cpu().numpy())
    traces = rec.traces(layer=3, workload="synthetic", prompt_ids=["a", "b"],
                        metadata={"k": kk})
    for b, tr in enumerate(traces):
        want, want_len = oracle.trace_matrix(rows[b])
        np.testing.assert_array_equal(tr.scores.view(np.uint16), want.view(np.uint16))
        np.testing.assert_array_equal(tr.lengths, want_len)
        path = tmp_path / f"{tr.prompt_id}_layer_{tr.layer:02d}.npz"
        save_trace(path, tr)
        back = load_trace(path)
        np.testing.assert_array_equal(back.scores.view(np.uint16), want.view(np.uint16))
        assert back.metadata == {"k": kk} and back.prompt_id == ["a", "b"][b]
    with pytest.raises(ValueError, match="all are taken"):
        plan.run()


def test_trace_errors():
    from dsa_b200 import _capi as capi
    from dsa_b200.indexer import ScoreTopkPlan
    from dsa_b200.trace import TraceRecorder, score_trace

    q, w, k = _inputs(1, 256, torch.float32, seed=2)
    rec = TraceRecorder(1, 2, 256, "cuda")
    with pytest.raises(ValueError, match="16-bit|bfloat16"):
        score_trace(q.cuda(), w.cuda(), k.cuda(), rec)
    with pytest.raises(ValueError):
        ScoreTopkPlan(q.cuda(), w.cuda(), k.cuda(), 8, trace=rec)
    qb, kb = q.to(torch.bfloat16).cuda(), k.to(torch.bfloat16).cuda()
    with pytest.raises(ValueError, match="recorder holds 1 sequences"):
        score_trace(qb.expand(2, 64, 128).contiguous(), w.cuda().expand(2, 64).contiguous(),
                    kb.expand(2, 256, 128).contiguous(), rec)
    assert rec.step == 0
    out = torch.empty(1, 256, device="cuda")
    with pytest.raises(ValueError, match="trace is null"):
        capi.call("tdsa_score_dense_trace", qb.data_ptr(), 64 * 128, w.cuda().data_ptr(), 64,
                  kb.data_ptr(), 256 * 128, 128, capi.TDSA_BF16, 1, 256, out.data_ptr(), 256, None,
                  None, 0, torch.cuda.current_stream().cuda_stream)
    with pytest.raises(capi.TdsaError, match="traces need 16-bit"):
        capi.call("tdsa_score_dense_trace", q.cuda().data_ptr(), 64 * 128,
                  w.cuda().data_ptr(), 64, k.cuda().data_ptr(), 256 * 128, 128, capi.TDSA_F32, 1, 256, out.data_ptr(), 256,
                  None, rec.buffer.data_ptr(), 512, torch.cuda.current_stream().cuda_stream)
