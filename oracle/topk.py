"""Numpy restatement of the reference top-K semantics (test oracle).

Reference: ``src/temporal_dsa/metrics.py:9-22`` (``stable_topk``): the k largest
values, returned in descending value order, equal values ordered by ascending
index, and the cutoff tie resolved by global index.
"""

from __future__ import annotations

import numpy as np


def stable_topk(values, k: int) -> np.ndarray:
    """metrics.py:9-22 -- descending top-k indices with the index as tie-breaker."""
    x = np.asarray(values)
    if x.ndim != 1:
        raise ValueError(f"expected a vector, got {x.shape}")
    if not 0 < k <= x.size:
        raise ValueError(f"k={k} is invalid for {x.size} values")
    cutoff = np.partition(x, x.size - k)[x.size - k]
    greater = np.flatnonzero(x > cutoff)
    equal = np.flatnonzero(x == cutoff)
    candidate = np.concatenate((greater, equal[: k - greater.size]))
    return candidate[np.lexsort((candidate, -x[candidate]))]


def topk_rows(scores, k: int, *, sorted: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """Row-wise ``stable_topk`` over a [B, L] score matrix.

    sorted=True returns stable_topk's order; sorted=False returns the same index set in
    ascending index order (the order the CUDA top-K emits without its final sort).
    Returns (indices int64 [B,k], values f32 [B,k]).
    """
    s = np.asarray(scores, dtype=np.float32)
    if s.ndim == 1:
        s = s[None]
    idx = np.stack([stable_topk(row, k) for row in s])
    if not sorted:
        idx = np.sort(idx, axis=1)
    vals = np.take_along_axis(s, idx, axis=1)
    return idx.astype(np.int64), vals


def merge_topk(cand_scores, cand_indices, k: int, *, sorted: bool = True):
    """Merge per-shard candidates into the global top-k (same tie rule as stable_topk).

    cand_scores / cand_indices are [B, M] (M = shards x k_local).  The global top-k of a
    row is the stable top-k of the union, because every member of the global top-k is in
    its own shard's local top-k.  Ties are resolved by the candidates' global index.
    """
    s = np.asarray(cand_scores, dtype=np.float32)
    i = np.asarray(cand_indices, dtype=np.int64)
    if s.ndim == 1:
        s, i = s[None], i[None]
    out_idx, out_val = [], []
    for row_s, row_i in zip(s, i):
        order = np.lexsort((row_i, -row_s.astype(np.float64)))[:k]
        sel_i, sel_s = row_i[order], row_s[order]
        if not sorted:
            o = np.argsort(sel_i, kind="stable")
            sel_i, sel_s = sel_i[o], sel_s[o]
        out_idx.append(sel_i)
        out_val.append(sel_s)
    return np.stack(out_idx), np.stack(out_val)
