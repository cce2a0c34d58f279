"""Numpy restatement of the exact (certified) progressive top-K step (test oracle).

The reference has no implementation of the exact path; it is the combination its own
code points at: the seed / hot-first / prune-below-running-K-th filter of
``replay.py:172-222`` and ``:263-266`` with the certified per-block bound of
``certified.py:18-48`` (``upper_b = previous_block_max_b + radius_b``).  This file states
the schedule the CUDA path runs, so tests can check its block decisions and its
invariant: the top-k equals dense scoring's top-k at every step.

Schedule of one step (per sequence):
  1. coefficient c = sum_h |w_t-w_p| ||q_p,h|| + |w_t| ||q_t,h - q_p,h||  (float64);
     slack = GAMMA * (sum_h |w_t,h| ||q_t,h|| + sum_h |w_p,h| ||q_p,h||) covers the float32
     rounding of the two computed scores the bound links.
  2. bound_b = U_b + maxnorm_b * (c + slack) for blocks fully seen last step; +inf for
     blocks holding keys that are new at this step (replay.py:263-266).
  3. wave 1 scores the hot blocks (those holding a previous top-k key) and new blocks --
     every block when those leave at most 1/16 of the blocks out;
     tau = the lower edge of the key bin (the top 24 bits of the order-preserving float
     key, found with two 4096-bin histograms) that holds the k-th largest wave-1 score --
     a lower bound of that score, read from histograms instead of a second top-k;
  4. wave 2 scores every other block with bound_b >= tau; the rest are pruned unread.
  5. top-k over the scored keys; U_b <- exact block max (scored) or bound_b (pruned).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .certified import shared_block_key_norms
from .indexer import full_scores
from .topk import stable_topk

GAMMA = 2.0 ** -12
ALL_HOT_FRACTION = 16  # wave 1 takes every block when at most 1/16 of them would be left


def _float_to_key(v: float) -> int:
    """Order-preserving uint32 key of a float32 (-0 as +0, every NaN above +inf)."""
    b = int(np.array([v], np.float32).view(np.uint32)[0])
    if b & 0x7FFFFFFF == 0:
        b = 0
    if (b & 0x7F800000) == 0x7F800000 and (b & 0x007FFFFF):
        return 0xFFFFFFFF
    return (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)


def _key_to_float(key: int) -> float:
    b = (key & 0x7FFFFFFF) if key & 0x80000000 else (~key & 0xFFFFFFFF)
    return float(np.array([b], np.uint32).view(np.float32)[0])


def _bin_floor(v: float) -> float:
    """Smallest float of v's key bin at 24-bit resolution: the 12-bit bin of the key, then
    the next 12 bits inside it (top-level bin 0: -inf; keys past +inf: +inf)."""
    key = _float_to_key(v)
    if key >> 20 == 0:
        return -math.inf
    lo = key & 0xFFFFFF00
    if lo > 0xFF800000:
        return math.inf
    return _key_to_float(lo)


@dataclass
class ExactState:
    block_size: int
    k: int
    length: int
    topk: np.ndarray
    upper: np.ndarray
    maxnorm: np.ndarray
    q: np.ndarray
    w: np.ndarray


def _block_max(scores: np.ndarray, block_size: int) -> np.ndarray:
    return np.array([scores[s : s + block_size].max()
                     for s in range(0, scores.size, block_size)], dtype=np.float64)


def exact_init(q, w, keys, k: int, block_size: int):
    """First step: dense scoring, stable top-k, exact block maxima and key norms."""
    keys = np.asarray(keys, dtype=np.float32)
    scores = full_scores(q, w, keys)
    topk = stable_topk(scores, k)
    state = ExactState(block_size, k, keys.shape[0], topk, _block_max(scores, block_size),
                       shared_block_key_norms(keys, block_size),
                       np.asarray(q, np.float32).copy(), np.asarray(w, np.float32).copy())
    return state, topk, scores


def bound_terms(state: ExactState, q, w) -> tuple[float, float]:
    qn = np.asarray(q, np.float64)
    wn = np.asarray(w, np.float64)
    qp = state.q.astype(np.float64)
    wp = state.w.astype(np.float64)
    coeff = float(np.sum(np.abs(wn - wp) * np.linalg.norm(qp, axis=1)
                         + np.abs(wn) * np.linalg.norm(qn - qp, axis=1)))
    slack = GAMMA * float(np.sum(np.abs(wn) * np.linalg.norm(qn, axis=1))
                          + np.sum(np.abs(wp) * np.linalg.norm(qp, axis=1)))
    return coeff, slack


def exact_step(state: ExactState, q, w, keys):
    """One exact progressive step.  Returns (topk, scores, stats, new_state).

    ``scores`` holds the float32 score of every scored key and -inf for pruned keys.
    """
    keys = np.asarray(keys, dtype=np.float32)
    bs, k = state.block_size, state.k
    length = keys.shape[0]
    if length < state.length:
        raise ValueError("the key cache may only grow between steps")
    nblocks = math.ceil(length / bs)
    first_new = state.length // bs
    maxnorm = np.concatenate([state.maxnorm[:first_new],
                              shared_block_key_norms(keys[first_new * bs:], bs)])
    coeff, slack = bound_terms(state, q, w)
    bound = np.full(nblocks, math.inf)
    bound[:first_new] = state.upper[:first_new] + maxnorm[:first_new] * (coeff + slack)
    hot = np.zeros(nblocks, dtype=bool)
    hot[state.topk // bs] = True
    hot[first_new:] = True
    cold = int((~hot).sum())
    if 0 < cold and cold * ALL_HOT_FRACTION <= nblocks:  # the last few cold blocks join wave 1
        hot[:] = True
    full = full_scores(q, w, keys)
    key_block = np.arange(length) // bs
    wave1 = hot[key_block]
    tau = _bin_floor(float(np.partition(full[wave1], -k)[-k])) if wave1.sum() >= k else -math.inf
    wave2_blocks = (~hot) & (bound >= tau)
    scored_blocks = hot | wave2_blocks
    scores = np.where(scored_blocks[key_block], full, np.float32(-np.inf)).astype(np.float32)
    topk = stable_topk(scores, k)
    block_max = _block_max(scores, bs)
    upper = np.where(scored_blocks, block_max, bound)
    keys_read = int(scored_blocks[key_block].sum())
    stats = {
        "blocks": nblocks,
        "hot_blocks": int(hot.sum()),
        "wave2_blocks": int(wave2_blocks.sum()),
        "pruned_blocks": int((~scored_blocks).sum()),
        "keys_read": keys_read,
        "tau": tau,
        "coeff": coeff,
    }
    new_state = ExactState(bs, k, length, topk, upper, maxnorm,
                           np.asarray(q, np.float32).copy(), np.asarray(w, np.float32).copy())
    return topk, scores, stats, new_state
