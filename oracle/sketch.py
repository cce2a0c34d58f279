"""Numpy restatement of the certified INT8 key sketch (test oracle).

The quantizer is the reference's symmetric fake quantization
(src/temporal_dsa/verifier_scoring.py:29-41: ``round(x / scale)`` clamped to
+-(2^(bits-1) - 1), ``scale = max|x| / limit``), applied with one scale per key instead of
one per tensor, in the float32 operations the device kernel uses; the residual and norm of
each key are exact (float64).  The certified statement the tests check against it:
|score - sketch score| <= G r + D n for score = sum_h w_h ReLU(q_h . k)
(progressive_kernel.py:45-55), G = sum_h |w_h| ||q_h||, D = sum_h |w_h| ||q_h - q~_h||.
"""

from __future__ import annotations

import numpy as np

LIMIT = 127  # 8-bit symmetric limit, verifier_scoring.py:36


def quantize_rows(x, scales, limit: int = LIMIT) -> np.ndarray:
    """verifier_scoring.py:38-40 per row: clamp(round(x / scale), -limit, limit) with each
    row's own float32 scale (a zero scale gives zeros)."""
    x = np.asarray(x, dtype=np.float32)
    s = np.asarray(scales, dtype=np.float32).reshape(-1, 1)
    safe = np.where(s > 0, s, np.float32(1))
    q = np.clip(np.rint(x / safe), -limit, limit)
    return np.where(s > 0, q, 0).astype(np.int8)


def sketch_keys(keys):
    """keys [L,128] (float values of 16-bit keys) -> (int8 [L,128], scale f32 [L],
    residual norm f64 [L], norm of the dequantized key f64 [L])."""
    k = np.asarray(keys, dtype=np.float32)
    s = (np.abs(k).max(axis=1) / np.float32(LIMIT)).astype(np.float32)
    q = quantize_rows(k, s)
    deq = s.astype(np.float64)[:, None] * q.astype(np.float64)
    resid = np.sqrt(((k.astype(np.float64) - deq) ** 2).sum(axis=1))
    norm = np.sqrt((deq ** 2).sum(axis=1))
    return q, s, resid, norm
