"""Numpy restatement of the reference certified temporal bound (test oracle).

Reference: ``src/temporal_dsa/certified.py:18-61``.  Both functions are float64.
"""

from __future__ import annotations

import numpy as np


def temporal_score_radius(q_now, q_prev, w_now, w_prev, block_key_norm) -> np.ndarray:
    """certified.py:18-48 -- per-block certified radius of |I_t - I_(t-1)|.

    coefficient_h = |w_t,h - w_p,h| * ||q_p,h|| + |w_t,h| * ||q_t,h - q_p,h||
    radius_b      = sum_h block_key_norm[b,h] * coefficient_h
    """
    q_now = np.asarray(q_now, dtype=np.float64)
    q_prev = np.asarray(q_prev, dtype=np.float64)
    w_now = np.asarray(w_now, dtype=np.float64)
    w_prev = np.asarray(w_prev, dtype=np.float64)
    norms = np.asarray(block_key_norm, dtype=np.float64)
    if q_now.shape != q_prev.shape or q_now.ndim != 2:
        raise ValueError("query tensors must have shape [heads,dim]")
    if w_now.shape != w_prev.shape or w_now.shape != (q_now.shape[0],):
        raise ValueError("weight tensors must have shape [heads]")
    if norms.ndim != 2 or norms.shape[1] != q_now.shape[0]:
        raise ValueError("block_key_norm must have shape [blocks,heads]")
    coefficient = (np.abs(w_now - w_prev) * np.linalg.norm(q_prev, axis=1)
                   + np.abs(w_now) * np.linalg.norm(q_now - q_prev, axis=1))
    return norms @ coefficient


def block_key_norms(keys, block_size: int) -> np.ndarray:
    """certified.py:51-61 -- max key L2 norm per block and head, keys [tokens,heads,dim]."""
    keys = np.asarray(keys, dtype=np.float64)
    if keys.ndim != 3:
        raise ValueError("keys must have shape [tokens,heads,dim]")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    rows = [np.linalg.norm(keys[s : s + block_size], axis=2).max(axis=0)
            for s in range(0, keys.shape[0], block_size)]
    return np.stack(rows)


def shared_block_key_norms(keys, block_size: int) -> np.ndarray:
    """block_key_norms for the indexer's shared key cache [tokens, dim] -> [blocks].

    With one key vector shared by all heads every column of block_key_norms is the same
    (the reference test builds exactly that, tests/test_certified.py:13-19), so the
    radius collapses to maxnorm_b * sum_h coefficient_h.
    """
    keys = np.asarray(keys, dtype=np.float64)
    norms = np.linalg.norm(keys, axis=1)
    return np.array([norms[s : s + block_size].max()
                     for s in range(0, keys.shape[0], block_size)])
