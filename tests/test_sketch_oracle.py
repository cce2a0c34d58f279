"""CPU checks of the sketch oracle (oracle/sketch.py): its quantizer is the reference's
symmetric fake quantization (verifier_scoring.py:29-41, golden ``verifier`` written by the
reference), and the certified sketch bound holds on float64 scores."""

from __future__ import annotations

import numpy as np

import oracle
from oracle import sketch as osk
from tests.conftest import load_golden


def test_quantizer_matches_reference_fake_quantize():
    g = load_golden("verifier")
    k = g["k"]
    for bits in (2, 4, 8):
        scale = float(g[f"fq{bits}_scale"])
        q = osk.quantize_rows(k, np.full(k.shape[0], scale, np.float32), 2 ** (bits - 1) - 1)
        np.testing.assert_array_equal(q.astype(np.float32) * np.float32(scale), g[f"fq{bits}_k"])


def test_sketch_bound_holds_in_float64():
    rng = np.random.default_rng(0)
    keys = rng.normal(size=(3000, 128)).astype(np.float32)
    keys[::7] *= 0.01
    q = (rng.normal(size=(64, 128)) / np.sqrt(128)).astype(np.float32)
    w = (rng.normal(size=64) / 8).astype(np.float32)
    kq, s, r, n = osk.sketch_keys(keys)
    deq = s.astype(np.float64)[:, None] * kq.astype(np.float64)
    exact = oracle.relu_index_score(q, keys, w)
    sketch = oracle.relu_index_score(q, deq, w)
    G = float(np.sum(np.abs(w.astype(np.float64)) * np.linalg.norm(q.astype(np.float64), axis=1)))
    assert np.all(np.abs(exact - sketch) <= G * r * (1 + 1e-12))
    assert np.all(r <= s * np.sqrt(128) / 2 * (1 + 1e-12))  # rounding error <= s/2 per dim
