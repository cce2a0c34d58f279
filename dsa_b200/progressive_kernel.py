"""Drop-in for ``temporal_dsa.progressive_kernel`` on B200 (sm_100a).

Same names, signatures, output types and error behaviour as the reference module
(src/temporal_dsa/progressive_kernel.py); the kernels behind them are the hand-written
tcgen05/TMA kernels of libtdsa, not Triton.  The ``*_triton`` names are kept so the
reference's call sites switch by import.  CUDA tensors are required (ValueError
otherwise, as in the reference's _check_cuda_inputs, :349-359).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .indexer import score_dense

HEADS = 64
HEAD_DIM = 128
VERIFIER_HEADS = 8


def split_head_ids(selected: torch.Tensor | np.ndarray) -> tuple[torch.Tensor, torch.Tensor]:
    """:23-34 -- validate 8 unique head ids in [0,64), return them and the sorted rest."""
    values = torch.as_tensor(selected, dtype=torch.int32)
    if values.ndim != 1 or values.numel() != VERIFIER_HEADS:
        raise ValueError("selected head IDs must have shape [8]")
    if values.min().item() < 0 or values.max().item() >= HEADS:
        raise ValueError("head ID outside [0, 64)")
    if torch.unique(values).numel() != VERIFIER_HEADS:
        raise ValueError("selected head IDs must be unique")
    mask = torch.ones(HEADS, dtype=torch.bool)
    mask[values.cpu().long()] = False
    remaining = torch.arange(HEADS, dtype=torch.int32)[mask]
    return values.contiguous(), remaining.contiguous()


def dynamic_head_ids(weights: torch.Tensor, width: int = VERIFIER_HEADS) -> torch.Tensor:
    """:37-42 -- the `width` heads of largest |w|, ties to the lower head id."""
    if weights.shape != (HEADS,):
        raise ValueError("weights must have shape [64]")
    if not 0 < width <= HEADS:
        raise ValueError("invalid head width")
    return torch.argsort(weights.abs(), descending=True, stable=True)[:width].to(torch.int32)


def progressive_qk_reduction(length: int, direct_full_blocks: int, promoted_cold_blocks: int,
                             *, block_size: int = 64) -> float:
    """:93-111 -- fraction of QK MACs the H8 progressive schedule skips."""
    block_count = math.ceil(length / block_size)
    if min(direct_full_blocks, promoted_cold_blocks) < 0:
        raise ValueError("block counts must be non-negative")
    if direct_full_blocks + promoted_cold_blocks > block_count:
        raise ValueError("accepted block counts exceed total blocks")
    direct_tokens = min(length, direct_full_blocks * block_size)
    promoted_tokens = min(length - direct_tokens, promoted_cold_blocks * block_size)
    cold_tokens = length - direct_tokens
    work = direct_tokens * HEADS + cold_tokens * VERIFIER_HEADS + promoted_tokens * (
        HEADS - VERIFIER_HEADS)
    return 1.0 - work / (length * HEADS)


@dataclass(frozen=True)
class ProgressiveResult:
    """:114-120."""

    scores: torch.Tensor
    accepted_blocks: torch.Tensor
    block_max: torch.Tensor
    candidate_indices: torch.Tensor | None = None
    candidate_count: int | None = None


def _check_cuda_inputs(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor) -> None:
    """:349-359."""
    if not queries.is_cuda or not weights.is_cuda or not keys.is_cuda:
        raise ValueError("the B200 indexer kernels require CUDA tensors")
    if queries.shape != (HEADS, HEAD_DIM) or weights.shape != (HEADS,):
        raise ValueError("expected queries [64,128] and weights [64]")
    if keys.ndim != 2 or keys.shape[1] != HEAD_DIM:
        raise ValueError("expected keys [L,128]")
    if queries.dtype not in {torch.float16, torch.bfloat16} or keys.dtype != queries.dtype:
        raise ValueError("queries and keys must share FP16/BF16 dtype")


def full_scores_triton(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor, *,
                       block_size: int = 64) -> torch.Tensor:
    """:362-375 -- dense scores [L] float32.  block_size is a reference tiling knob only."""
    _check_cuda_inputs(queries, weights, keys)
    return score_dense(queries, weights, keys)
