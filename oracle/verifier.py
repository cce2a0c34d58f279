"""Numpy restatement of the reference's dimension-sparse verifier scorer (test oracle).

Reference: ``src/temporal_dsa/verifier_scoring.py`` -- ``normalized_hadamard`` (:9-26),
``fake_symmetric_quantize`` (:29-41), ``score_dim_sparse`` (:95-139).  Arithmetic in
float32 like the reference's float32 path: the Hadamard butterflies run in the same
order (stride 1 first), the quantizer divides by the float32 scale and rounds half to
even (torch.round), scores sum the ReLU'd head dots times the weights over heads.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def normalized_hadamard(x) -> np.ndarray:
    """verifier_scoring.py:9-26 -- orthonormal Walsh-Hadamard transform on the last axis."""
    out = np.asarray(x, dtype=F32)
    size = out.shape[-1]
    if size <= 0 or size & (size - 1):
        raise ValueError("Hadamard dimension must be a positive power of two")
    stride = 1
    while stride < size:
        g = out.reshape(*out.shape[:-1], -1, 2 * stride)
        left, right = g[..., :stride], g[..., stride:]
        out = np.concatenate((left + right, left - right), axis=-1).reshape(out.shape)
        stride *= 2
    return (out * F32(size ** -0.5)).astype(F32)


def fake_symmetric_quantize(x, bits: int, scale: float | None = None):
    """verifier_scoring.py:29-41 -- symmetric fake quantization with one tensor scale.
    Returns (values, scale); the scale is max|x| / (2^(bits-1) - 1) unless given."""
    if bits not in {2, 4, 8}:
        raise ValueError("bits must be one of 2, 4, 8")
    t = np.asarray(x, dtype=F32)
    limit = 2 ** (bits - 1) - 1
    if scale is None:
        scale = float(np.abs(t).max()) / max(limit, 1)
    scale = max(float(scale), 1e-12)
    q = np.clip(np.round(t / F32(scale)), -limit, limit).astype(F32)
    return (q * F32(scale)).astype(F32), scale


def score_dim_sparse(queries, weights, keys, dimension_indices, *, rotation: str = "none",
                     bits: int | None = None, query_scale: float | None = None,
                     key_scale: float | None = None) -> np.ndarray:
    """verifier_scoring.py:95-139 -- all-head scores on a subset of (rotated, optionally
    quantized) dimensions: [Q,H,D] x [K,D] -> [Q,K] float32."""
    q, w, k = (np.asarray(a, dtype=F32) for a in (queries, weights, keys))
    if q.ndim != 3 or w.shape != q.shape[:2] or k.ndim != 2:
        raise ValueError("expected queries [Q,H,D], weights [Q,H], keys [K,D]")
    if rotation == "hadamard":
        q, k = normalized_hadamard(q), normalized_hadamard(k)
    elif rotation != "none":
        raise ValueError("rotation must be 'none' or 'hadamard'")
    dims = np.asarray(dimension_indices).astype(np.int64)
    qs, ks = q[..., dims], k[..., dims]
    if bits is not None:
        qs, _ = fake_symmetric_quantize(qs, bits, query_scale)
        ks, _ = fake_symmetric_quantize(ks, bits, key_scale)
    dots = np.einsum("qhd,kd->qhk", qs, ks).astype(F32)
    return (np.maximum(dots, F32(0)) * w[..., None]).sum(axis=1, dtype=F32)
