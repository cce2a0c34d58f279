"""Drop-in for the head-sparse scorer of ``temporal_dsa.verifier_scoring`` on B200.

``score_head_sparse`` (reference src/temporal_dsa/verifier_scoring.py:49-92) scores Q
queries against one shared key cache with only the selected heads.  Selecting heads is the
same as giving the other heads weight zero, so each query runs the dense tcgen05 kernel
with w'_h = w_h * (times head h is selected): sum_h w'_h ReLU(q_h . k) equals the
reference's sum over the selected list (its ReLU(.)*0 terms are exact zeros).  The
reference rounds 16-bit head dots to the input dtype before the ReLU; the kernel keeps
them in float32, so 16-bit results agree to the 16-bit tolerance, float32 ones to 1e-5.

``dynamic_head_indices`` (:142-159) is the reference's stable per-query head ranking.
"""

from __future__ import annotations

import torch

from .indexer import HEAD_DIM, HEADS, require_cuda, score_dense


def score_head_sparse(queries, weights, keys, head_indices, *, query_chunk_size: int = 1,
                      key_chunk_size: int = 8192) -> torch.Tensor:
    """:49-92 -- selected-head full-dimension scores, float32 [Q, K].

    head_indices: a fixed [h] vector or a per-query [Q, h] matrix of head ids (repeats
    count twice, as in the reference).  The chunk sizes are reference tiling knobs.
    """
    if queries.ndim != 3 or weights.shape != queries.shape[:2] or keys.ndim != 2:
        raise ValueError("expected queries [Q,H,D], weights [Q,H], keys [K,D]")
    require_cuda(queries, weights, keys)
    if queries.shape[1:] != (HEADS, HEAD_DIM) or keys.shape[1] != HEAD_DIM:
        raise ValueError("the B200 indexer kernels take 64 heads x 128 dims")
    ids = torch.as_tensor(head_indices, device=queries.device, dtype=torch.long)
    if ids.ndim not in {1, 2}:
        raise ValueError("head_indices must be [h_v] or [Q,h_v]")
    if ids.ndim == 2 and ids.shape[0] != queries.shape[0]:
        raise ValueError("dynamic head_indices must have one row per query")
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= HEADS):
        raise IndexError("head index outside [0, 64)")
    nq = queries.shape[0]
    rows = ids if ids.ndim == 2 else ids.unsqueeze(0).expand(nq, -1)
    counts = torch.zeros(nq, HEADS, device=queries.device, dtype=torch.float32)
    counts.scatter_add_(1, rows, torch.ones(rows.shape, device=queries.device))
    w_eff = weights.float() * counts
    q = queries if queries.dtype == keys.dtype else queries.to(keys.dtype)
    out = torch.empty(nq, keys.shape[0], device=keys.device, dtype=torch.float32)
    if keys.shape[0]:
        for i in range(nq):
            score_dense(q[i], w_eff[i], keys, out=out[i])
    return out


def dynamic_head_indices(weights, width: int, strategy: str) -> torch.Tensor:
    """:142-159 -- per-query head routing [Q, width]: heads by descending |w|
    ("high_weight") or max(w, 0) ("positive_weight"), ties to the lower head id."""
    if not 0 < width <= weights.shape[-1]:
        raise ValueError("invalid head width")
    if strategy == "high_weight":
        values = weights.abs()
    elif strategy == "positive_weight":
        values = torch.clamp_min(weights, 0)
    else:
        raise ValueError("strategy must be high_weight or positive_weight")
    order = torch.argsort(values, dim=-1, descending=True, stable=True)
    return order[:, :width]
