"""Numpy restatement of the reference indexer scoring functions (test oracle).

Reference: ``src/temporal_dsa/progressive_kernel.py``, ``sidecar.py``,
``certified.py`` and ``verifier_scoring.py`` of psa1582/dsa.  All arithmetic is
float32 (float64 for ``relu_index_score``), inputs are upcast first, exactly as
the reference's torch paths upcast with ``.float()``.
"""

from __future__ import annotations

import math

import numpy as np

HEADS = 64  # progressive_kernel.py:18
HEAD_DIM = 128  # progressive_kernel.py:19
VERIFIER_HEADS = 8  # progressive_kernel.py:20

F32 = np.float32


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=F32)


def split_head_ids(selected) -> tuple[np.ndarray, np.ndarray]:
    """progressive_kernel.py:23-34 -- 8 unique ids in [0,64) and their sorted complement."""
    values = np.asarray(selected).astype(np.int64)
    if values.ndim != 1 or values.size != VERIFIER_HEADS:
        raise ValueError("selected head IDs must have shape [8]")
    if values.min() < 0 or values.max() >= HEADS:
        raise ValueError("head ID outside [0, 64)")
    if np.unique(values).size != VERIFIER_HEADS:
        raise ValueError("selected head IDs must be unique")
    mask = np.ones(HEADS, dtype=bool)
    mask[values] = False
    return values.astype(np.int32), np.arange(HEADS, dtype=np.int32)[mask]


def dynamic_head_ids(weights, width: int = VERIFIER_HEADS) -> np.ndarray:
    """progressive_kernel.py:37-42 -- |w| descending, ties to the lower head id."""
    w = np.asarray(weights)
    if w.shape != (HEADS,):
        raise ValueError("weights must have shape [64]")
    if not 0 < width <= HEADS:
        raise ValueError("invalid head width")
    return np.argsort(-np.abs(w.astype(np.float64)), kind="stable")[:width].astype(np.int32)


def full_scores(queries, weights, keys) -> np.ndarray:
    """progressive_kernel.py:45-55 (torch_full_scores): f32 matmul, ReLU, weighted head sum."""
    q, w, k = _f32(queries), _f32(weights), _f32(keys)
    if q.shape != (HEADS, HEAD_DIM) or w.shape != (HEADS,):
        raise ValueError("expected queries [64,128] and weights [64]")
    if k.ndim != 2 or k.shape[1] != HEAD_DIM:
        raise ValueError("expected keys [L,128]")
    dots = q @ k.T
    return (np.maximum(dots, F32(0)) * w[:, None]).sum(axis=0, dtype=F32)


def relu_index_score(q, keys, weights) -> np.ndarray:
    """certified.py:6-15 -- float64 I_s = sum_j w_j ReLU(q_j . k_s)."""
    q = np.asarray(q, dtype=np.float64)
    keys = np.asarray(keys, dtype=np.float64)
    weights = np.asarray(weights, dtype=np.float64)
    if q.ndim != 2 or keys.ndim != 2 or q.shape[1] != keys.shape[1]:
        raise ValueError("q must be [heads,dim] and keys [tokens,dim]")
    if weights.shape != (q.shape[0],):
        raise ValueError("weights must have one value per head")
    return (np.maximum(q @ keys.T, 0.0) * weights[:, None]).sum(axis=0)


def score_encoded(queries, weights, keys, *, key_chunk_size: int | None = None) -> np.ndarray:
    """sidecar.py:89-107 -- batched [B,Q,H,D] x [B,L,D] -> [B,Q,L], chunked over keys."""
    q, w, k = _f32(queries), _f32(weights), _f32(keys)
    if q.ndim != 4 or w.shape != q.shape[:-1]:
        raise ValueError("queries must be [batch,query,heads,dim]")
    if k.ndim != 3 or k.shape[0] != q.shape[0]:
        raise ValueError("keys must be [batch,key,dim]")
    chunk = key_chunk_size or k.shape[1]
    outs = []
    for start in range(0, k.shape[1], chunk):
        kc = k[:, start : start + chunk]
        dots = np.einsum("bqhd,bkd->bqhk", q, kc, dtype=F32)
        outs.append((np.maximum(dots, F32(0)) * w[..., None]).sum(axis=2, dtype=F32))
    return np.concatenate(outs, axis=-1) if outs else np.zeros(q.shape[:2] + (0,), F32)


def score_head_sparse(queries, weights, keys, head_indices) -> np.ndarray:
    """verifier_scoring.py:49-92 -- selected-head full-dim score, [Q,H,D] x [K,D] -> [Q,K]."""
    q, w, k = _f32(queries), _f32(weights), _f32(keys)
    if q.ndim != 3 or w.shape != q.shape[:2] or k.ndim != 2:
        raise ValueError("expected queries [Q,H,D], weights [Q,H], keys [K,D]")
    ids = np.asarray(head_indices).astype(np.int64)
    if ids.ndim not in (1, 2):
        raise ValueError("head_indices must be [h_v] or [Q,h_v]")
    if ids.ndim == 2 and ids.shape[0] != q.shape[0]:
        raise ValueError("dynamic head_indices must have one row per query")
    out = np.empty((q.shape[0], k.shape[0]), dtype=F32)
    for row in range(q.shape[0]):
        sel = ids if ids.ndim == 1 else ids[row]
        dots = q[row, sel] @ k.T
        out[row] = (np.maximum(dots, F32(0)) * w[row, sel][:, None]).sum(axis=0, dtype=F32)
    return out


def _head_sum(q, w, tile, heads) -> np.ndarray:
    dots = q[heads] @ tile.T
    return (np.maximum(dots, F32(0)) * w[heads][:, None]).sum(axis=0, dtype=F32)


def _block_count(length: int, block_size: int) -> int:
    return math.ceil(length / block_size)


def progressive_scores(queries, weights, keys, selected_heads, direct_full_blocks, threshold,
                       *, block_size: int = 64):
    """progressive_kernel.py:58-90 (torch_progressive_scores).

    block_max is the 8-head partial max of EVERY block (direct ones included);
    accepted blocks get partial(selected) + rest(remaining), the others -inf.
    """
    q, w, k = _f32(queries), _f32(weights), _f32(keys)
    selected, remaining = split_head_ids(selected_heads)
    length = k.shape[0]
    nblocks = _block_count(length, block_size)
    direct = np.asarray(direct_full_blocks).astype(bool).reshape(-1)
    if direct.size != nblocks:
        raise ValueError("direct_full_blocks length mismatch")
    out = np.full(length, -np.inf, dtype=F32)
    accepted = direct.copy()
    block_max = np.full(nblocks, -np.inf, dtype=F32)
    for b in range(nblocks):
        tile = k[b * block_size : min(length, (b + 1) * block_size)]
        partial = _head_sum(q, w, tile, selected)
        block_max[b] = partial.max()
        if accepted[b] or block_max[b] >= threshold:
            accepted[b] = True
            out[b * block_size : b * block_size + tile.shape[0]] = partial + _head_sum(
                q, w, tile, remaining
            )
    return out, accepted, block_max


def progressive_qk_reduction(length: int, direct_full_blocks: int, promoted_cold_blocks: int,
                             *, block_size: int = 64) -> float:
    """progressive_kernel.py:93-111 -- QK MAC reduction of the H8 progressive schedule."""
    nblocks = _block_count(length, block_size)
    if min(direct_full_blocks, promoted_cold_blocks) < 0:
        raise ValueError("block counts must be non-negative")
    if direct_full_blocks + promoted_cold_blocks > nblocks:
        raise ValueError("accepted block counts exceed total blocks")
    direct_tokens = min(length, direct_full_blocks * block_size)
    promoted_tokens = min(length - direct_tokens, promoted_cold_blocks * block_size)
    cold_tokens = length - direct_tokens
    work = (direct_tokens * HEADS + cold_tokens * VERIFIER_HEADS
            + promoted_tokens * (HEADS - VERIFIER_HEADS))
    return 1.0 - work / (length * HEADS)


def h8_block_max(queries, weights, keys, selected_heads, cold_blocks, *, block_size: int = 64):
    """Semantics of _h8_block_max_kernel, progressive_kernel.py:218-246 and :378-404.

    partial = 8-head score on cold blocks, -inf on the others; maxima = per-block max.
    """
    q, w, k = _f32(queries), _f32(weights), _f32(keys)
    sel = np.asarray(selected_heads).astype(np.int64).reshape(-1)
    length = k.shape[0]
    nblocks = _block_count(length, block_size)
    cold = np.asarray(cold_blocks).astype(bool).reshape(-1)
    if cold.size != nblocks:
        raise ValueError("cold block mask length mismatch")
    partial = _head_sum(q, w, k, sel) if length else np.zeros(0, F32)
    partial = np.where(np.repeat(cold, block_size)[:length], partial, F32(-np.inf)).astype(F32)
    maxima = np.array([partial[b * block_size : (b + 1) * block_size].max()
                       for b in range(nblocks)], dtype=F32)
    return partial, maxima


def masked_full_scores(queries, weights, keys, keep_blocks, *, block_size: int = 64):
    """Semantics of _masked_full_kernel, progressive_kernel.py:249-274 and :407-424."""
    k = _f32(keys)
    length = k.shape[0]
    nblocks = _block_count(length, block_size)
    keep = np.asarray(keep_blocks).astype(bool).reshape(-1)
    if keep.size != nblocks:
        raise ValueError("keep block mask length mismatch")
    full = full_scores(queries, weights, k)
    return np.where(np.repeat(keep, block_size)[:length], full, F32(-np.inf)).astype(F32)


def progressive_scores_fused(queries, weights, keys, selected_heads, direct_full_blocks,
                             threshold, *, block_size: int = 64, remaining_heads=None):
    """Semantics of _progressive_kernel, progressive_kernel.py:277-346 and :427-475.

    Direct blocks: all 64 heads, block_max -inf.  Cold blocks: 8-head partial, block_max =
    its max over valid keys, promoted when max >= threshold and then completed with the
    other 56 heads.  Rejected blocks score -inf.  Returns (scores, accepted int8, block_max).
    """
    q, w, k = _f32(queries), _f32(weights), _f32(keys)
    if remaining_heads is None:
        sel, rem = split_head_ids(selected_heads)
    else:
        sel = np.asarray(selected_heads).astype(np.int64).reshape(-1)
        rem = np.asarray(remaining_heads).astype(np.int64).reshape(-1)
    length = k.shape[0]
    nblocks = _block_count(length, block_size)
    direct = np.asarray(direct_full_blocks).astype(bool).reshape(-1)
    if direct.size != nblocks:
        raise ValueError("direct full block mask length mismatch")
    thr = F32(np.asarray(threshold, dtype=np.float64).reshape(-1)[0])
    scores = np.full(length, -np.inf, dtype=F32)
    accepted = np.zeros(nblocks, dtype=np.int8)
    block_max = np.full(nblocks, -np.inf, dtype=F32)
    for b in range(nblocks):
        lo, hi = b * block_size, min(length, (b + 1) * block_size)
        tile = k[lo:hi]
        if direct[b]:
            scores[lo:hi] = _head_sum(q, w, tile, np.arange(HEADS))
            accepted[b] = 1
            continue
        partial = _head_sum(q, w, tile, sel)
        block_max[b] = partial.max()
        if block_max[b] >= thr:
            accepted[b] = 1
            scores[lo:hi] = partial + _head_sum(q, w, tile, rem)
    return scores, accepted, block_max


def two_pass_scores(queries, weights, keys, selected_heads, direct_full_blocks, threshold,
                    *, block_size: int = 64):
    """progressive_kernel.py:478-497 -- H8 block max on cold blocks, then masked dense."""
    direct = np.asarray(direct_full_blocks).astype(bool).reshape(-1)
    _, maxima = h8_block_max(queries, weights, keys, selected_heads, ~direct,
                             block_size=block_size)
    thr = F32(np.asarray(threshold, dtype=np.float64).reshape(-1)[0])
    accepted = direct | (maxima >= thr)
    scores = masked_full_scores(queries, weights, keys, accepted, block_size=block_size)
    return scores, accepted.astype(np.int8), maxima
