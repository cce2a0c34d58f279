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


def round_to(x, dtype: str | None) -> np.ndarray:
    """Round float64 values to bfloat16 / float16 (nearest even, through float32 for bf16)
    and back to float64; dtype None leaves them unchanged."""
    x = np.asarray(x, dtype=np.float64)
    if dtype is None:
        return x
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float64)
    if dtype != "bf16":
        raise ValueError("dtype must be None, 'bf16' or 'f16'")
    bits = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    bits = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16 << 16
    return bits.astype(np.uint32).view(np.float32).astype(np.float64)


def encode_keys(hidden, wk, positions, ln_weight=None, ln_bias=None, *, rope_dim: int = 64,
                theta: float = 10_000.0, eps: float = 1e-6, raw_dtype: str | None = None):
    """sidecar.py:74-76 -- RoPE(LayerNorm(hidden @ wk^T)) [..., 128] in float64.

    LayerNorm(128, eps) as torch's: biased variance, then * weight + bias (None: 1 and 0).
    ``raw_dtype`` rounds the projection to the Linear's 16-bit output type first, as the
    reference's bf16 Linear does before its float32 LayerNorm."""
    h = np.asarray(hidden, dtype=np.float64)
    k = round_to(h @ np.asarray(wk, np.float64).T, raw_dtype)
    mean = k.mean(-1, keepdims=True)
    var = ((k - mean) ** 2).mean(-1, keepdims=True)
    y = (k - mean) / np.sqrt(var + eps)
    if ln_weight is not None:
        y = y * np.asarray(ln_weight, np.float64)
    if ln_bias is not None:
        y = y + np.asarray(ln_bias, np.float64)
    if rope_dim:
        y = y.copy()
        y[..., :rope_dim] = apply_noninterleaved_rope(y[..., :rope_dim], positions, theta)
    return y
