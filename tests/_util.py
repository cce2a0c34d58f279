"""Shared helpers for the parity tests (tolerances are stated where they are used)."""

from __future__ import annotations

import math

import numpy as np


def normwise_bound(q, w, keys) -> np.ndarray:
    """sum_h |w_h| * |q_h . k| per key: the scale a score's rounding error is relative to."""
    q = np.asarray(q, np.float64)
    w = np.asarray(w, np.float64)
    k = np.asarray(keys, np.float64)
    return (np.abs(w)[:, None] * np.abs(q @ k.T)).sum(axis=0)


def assert_scores_close(got, want, scale, rtol: float, atol: float = 0.0, msg: str = ""):
    """|got - want| <= rtol * scale + atol elementwise (norm-wise criterion)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    lim = rtol * np.asarray(scale, np.float64) + atol
    bad = np.flatnonzero(err > lim)
    assert bad.size == 0, (f"{msg}: {bad.size} scores off; worst err {err[bad].max():.3e} "
                           f"at {bad[np.argmax(err[bad])]} (limit {lim[bad].min():.3e})")


def assert_topk_equivalent(got_idx, want_idx, ref_scores, tol: float, msg: str = ""):
    """Index sets equal except for keys whose reference score ties the k-th within tol."""
    got = set(np.asarray(got_idx).tolist())
    want = set(np.asarray(want_idx).tolist())
    assert len(got) == len(want_idx), f"{msg}: duplicate or missing indices"
    if got == want:
        return
    ref = np.asarray(ref_scores, np.float64)
    kth = ref[np.asarray(want_idx)].min()
    for i in got ^ want:
        assert abs(ref[i] - kth) <= tol, (
            f"{msg}: index {i} differs with score {ref[i]:.8g} vs k-th {kth:.8g}")


def ar1_queries(rng, q0, steps: int, rho: float = 0.95):
    """q_t = rho q_{t-1} + sqrt(1-rho^2) N(0,1)/sqrt(128)."""
    out = [q0]
    for _ in range(steps):
        out.append(rho * out[-1] + math.sqrt(1 - rho * rho) * rng.normal(size=q0.shape) /
                   math.sqrt(128))
    return out
