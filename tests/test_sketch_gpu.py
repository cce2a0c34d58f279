"""GPU parity of the certified INT8 key sketch (dsa_b200.sketch).

- The sketch kernel's int8 values and scales equal the oracle's quantizer (oracle/sketch.py,
  the reference's symmetric quantizer of verifier_scoring.py:29-41 applied per key) bit for
  bit; its float16 norms are never below the exact float64 ones and within float16 rounding
  of them.
- The certified bounds hold: every key's lower bound and every 16-key block's upper bound
  enclose the float64 scores, tau <= the k-th largest float64 score, and every block holding
  a top-k key is read.
- The sketch top-k equals dense scoring's top-k (``scores_topk``) bit for bit -- indices and
  values, sorted and unsorted, ties included -- on i.i.d. and block-structured caches, at
  ragged lengths, k = length, and over decode steps of a growing cache.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from oracle import sketch as osk

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


def make_cache(kind, batch, length, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(batch, 64, 128, generator=g) / math.sqrt(128)).to(dtype)
    if kind == "iid":
        keys = torch.randn(batch, length, 128, generator=g)
        w = torch.randn(batch, 64, generator=g) / 8
    else:  # a quarter of the 64-key blocks at norm x3, the rest x0.05
        nb = (length + 63) // 64
        scale = torch.where(torch.rand(batch, nb, generator=g) < 0.25, 3.0, 0.05)
        keys = torch.randn(batch, length, 128, generator=g) * \
            scale.repeat_interleave(64, dim=1)[:, :length, None]
        w = torch.randn(batch, 64, generator=g).abs() / 8
    return q.cuda(), w.cuda(), keys.to(dtype).cuda()


def test_sketch_keys_match_oracle_quantizer():
    from dsa_b200.sketch import KeySketch

    q, w, keys = make_cache("iid", 2, 1000, 0)
    keys[0, 7] = 0  # an all-zero key: scale 0
    keys[1, 9] = keys[1, 9] * 1e-30  # tiny values
    sk = KeySketch(2, 1000, "cuda")
    sk.update(keys)
    vals = sk.values.cpu().numpy()
    scales = sk.scales.cpu().numpy()
    bounds = sk.bounds.float().cpu().numpy()
    for b in range(2):
        qv, s, r, n = osk.sketch_keys(keys[b].float().cpu().numpy())
        np.testing.assert_array_equal(vals[b], qv)
        np.testing.assert_array_equal(scales[b], s)
        assert np.all(bounds[b, :, 0] >= r) and np.all(bounds[b, :, 1] >= n)
        np.testing.assert_allclose(bounds[b, :, 0], r, rtol=2e-3, atol=1e-7)
        np.testing.assert_allclose(bounds[b, :, 1], n, rtol=2e-3, atol=1e-7)


@pytest.mark.parametrize("kind", ["iid", "structured"])
def test_sketch_bounds_are_certified(kind):
    from dsa_b200.sketch import KeySketch, SketchTopkPlan

    batch, length, k = 2, 5000, 256
    q, w, keys = make_cache(kind, batch, length, 1)
    sk = KeySketch(batch, length, "cuda")
    sk.update(keys)
    plan = SketchTopkPlan(q, w, keys, sk, k)
    plan.run()
    up, lo, tau = plan.bounds()
    up, lo, tau = up.cpu().numpy(), lo.cpu().numpy(), tau.cpu().numpy()
    nb = (length + 15) // 16
    for b in range(batch):
        exact = oracle.relu_index_score(q[b].float().cpu().numpy(),
                                        keys[b].float().cpu().numpy(), w[b].cpu().numpy())
        assert np.all(lo[b] <= exact), kind
        padded = np.full(nb * 16, -np.inf)
        padded[:length] = exact
        assert np.all(padded.reshape(nb, 16).max(axis=1) <= up[b]), kind
        assert tau[b] <= np.sort(exact)[-k]
        # every block holding a top-k key is read
        top_blocks = np.unique(np.argsort(-exact, kind="stable")[:k] // 16)
        assert np.all(up[b][top_blocks] >= tau[b])
    st = plan.stats()
    for b in range(batch):
        assert k <= st[b]["keys_read"] <= length
        assert st[b]["keys_read"] <= 16 * st[b]["blocks_read"] < st[b]["keys_read"] + 16
    if kind == "structured":  # most blocks hold small keys far below the k-th score
        assert all(s["keys_read"] < length // 2 for s in st)


@pytest.mark.parametrize("kind", ["iid", "structured"])
@pytest.mark.parametrize("batch,length,k", [(1, 16384, 2048), (3, 4099, 512), (2, 300, 300),
                                            (4, 40000, 1024)])
@pytest.mark.parametrize("sorted_", [True, False])
def test_sketch_topk_equals_dense(kind, batch, length, k, sorted_):
    from dsa_b200 import scores_topk
    from dsa_b200.sketch import KeySketch, sketch_topk

    q, w, keys = make_cache(kind, batch, length, length + k)
    if kind == "iid":
        keys[:, 100:140] = keys[:, 100:101]  # a run of tied scores
    sk = KeySketch(batch, length, "cuda")
    sk.update(keys)
    idx, val = sketch_topk(q, w, keys, sk, k, sorted=sorted_)
    want_i, want_v = scores_topk(q, w, keys, k, sorted=sorted_, index_dtype=torch.int64)
    assert torch.equal(idx, want_i) and torch.equal(val, want_v)


def test_sketch_plan_decode_steps_equal_dense():
    """A growing cache: one key appended and sketched per step, queries drifting."""
    from dsa_b200 import scores_topk
    from dsa_b200.sketch import KeySketch, SketchTopkPlan

    batch, l0, steps, k = 2, 8000, 6, 1024
    q, w, keys = make_cache("structured", batch, l0 + steps, 7)
    sk = KeySketch(batch, l0 + steps, "cuda")
    sk.update(keys, 0, l0)
    qbuf = q.clone()
    plan = SketchTopkPlan(qbuf, w, keys, sk, k, sorted=True, index_dtype=torch.int64)
    g = torch.Generator().manual_seed(8)
    for t in range(steps):
        length = l0 + t + 1
        sk.update(keys, length - 1, length)
        qbuf.copy_((qbuf.float() * 0.99 + 0.01 * torch.randn(batch, 64, 128, generator=g)
                    .cuda() / math.sqrt(128)).to(qbuf.dtype))
        got_i, got_v = plan.run(length)
        want_i, want_v = scores_topk(qbuf, w, keys[:, :length], k, sorted=True,
                                     index_dtype=torch.int64)
        assert torch.equal(got_i, want_i) and torch.equal(got_v, want_v), t
    st = plan.stats()
    assert all(s["keys_read"] < steps * (l0 + steps) for s in st)


def test_sketch_argument_errors():
    from dsa_b200.sketch import KeySketch, sketch_topk

    q, w, keys = make_cache("iid", 1, 500, 3)
    sk = KeySketch(1, 400, "cuda")
    with pytest.raises(ValueError):
        sk.update(keys)  # longer than the sketch
    sk = KeySketch(1, 500, "cuda")
    sk.update(keys)
    with pytest.raises(ValueError):
        sketch_topk(q, w, keys, sk, 501)
    with pytest.raises(ValueError):
        sketch_topk(q, w, keys.float(), sk, 10)
