"""Numpy restatement of the reference sidecar projection (test oracle).

Reference: ``src/temporal_dsa/sidecar.py:10-28`` (non-interleaved RoPE) and ``:74-87``
(encode_keys / encode_queries).  Computed in float64.
"""

from __future__ import annotations

import numpy as np


def apply_noninterleaved_rope(x, positions, theta: float = 10_000.0) -> np.ndarray:
    """sidecar.py:10-28 -- rotate (first half, second half) of the last axis by pos*inv_freq.

    ``positions`` broadcasts against x.shape[:-1] after the head axis is inserted, as in the
    reference (``cos`` is unsqueezed at -2 until it matches x's rank).
    """
    x = np.asarray(x, dtype=np.float64)
    if x.shape[-1] % 2:
        raise ValueError("RoPE dimension must be even")
    half = x.shape[-1] // 2
    inv_freq = np.float32(theta) ** (-np.arange(half, dtype=np.float32) / np.float32(half))
    angles = np.asarray(positions, dtype=np.float32)[..., None] * inv_freq.astype(np.float32)
    cos, sin = np.cos(angles.astype(np.float64)), np.sin(angles.astype(np.float64))
    while cos.ndim < x.ndim:
        cos = np.expand_dims(cos, -2)
        sin = np.expand_dims(sin, -2)
    first, second = x[..., :half], x[..., half:]
    return np.concatenate((first * cos - second * sin, second * cos + first * sin), axis=-1)


def rope_heads(qraw, positions, rope_dim: int = 64, theta: float = 10_000.0) -> np.ndarray:
    """sidecar.py:56-62 + :78-82 -- q [B, 64*128] -> [B,64,128] with RoPE on rope_dim dims."""
    q = np.asarray(qraw, dtype=np.float64).reshape(-1, 64, 128)
    out = q.copy()
    out[..., :rope_dim] = apply_noninterleaved_rope(q[..., :rope_dim], positions, theta)
    return out


def encode_queries(hidden, wq, ww, positions, rope_dim: int = 64, theta: float = 10_000.0):
    """sidecar.py:78-87 -- (q [B,64,128], w [B,64]) in float64."""
    h = np.asarray(hidden, dtype=np.float64)
    q = rope_heads(h @ np.asarray(wq, np.float64).T, positions, rope_dim, theta)
    w = (h @ np.asarray(ww, np.float64).T) * (64 * 128) ** -0.5
    return q, w
