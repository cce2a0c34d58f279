"""Device top-k with the reference's tie rule.

Mirrors ``temporal_dsa.metrics.stable_topk`` (src/temporal_dsa/metrics.py:9-22): the k
largest values in descending order, equal values by ascending index, the cutoff tie
resolved by global index.  Runs the radix-select kernel of libtdsa on a CUDA tensor.
"""

from __future__ import annotations

import torch

from .indexer import require_cuda, topk


def stable_topk(values: torch.Tensor, k: int) -> torch.Tensor:
    """Descending top-k indices (int64) of a 1-D CUDA tensor, index as tie-breaker."""
    require_cuda(values)
    if values.dim() != 1:
        raise ValueError(f"expected a vector, got {tuple(values.shape)}")
    if not 0 < k <= values.numel():
        raise ValueError(f"k={k} is invalid for {values.numel()} values")
    idx, _ = topk(values.to(torch.float32), k, sorted=True, index_dtype=torch.int64)
    return idx
