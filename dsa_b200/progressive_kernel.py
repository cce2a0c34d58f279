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

from . import _capi as capi
from .indexer import _DTYPES, score_dense, stream_ptr

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


# --------------------------------------------------------------------------- block kernels
class _Single:
    """One sequence's q [64,128], w [64] and keys [L,128] in the kernels' layout, with the
    accessors of a batch of one (the batch strides of a single sequence are unused)."""

    __slots__ = ("q", "w", "k", "length", "device", "dtype")

    def __init__(self, queries, weights, keys):
        k = keys
        if not (k.stride(1) == 1 and k.stride(0) % 8 == 0 and k.data_ptr() % 16 == 0):
            k = k.contiguous()
            if k.data_ptr() % 16:
                k = k.clone()
        q = queries
        if not (q.is_contiguous() and q.data_ptr() % 16 == 0):
            q = q.contiguous()
            if q.data_ptr() % 16:
                q = q.clone()
        w = weights
        if not (w.dtype == torch.float32 and w.is_contiguous()):
            w = w.to(torch.float32).contiguous()
        self.q, self.w, self.k = q, w, k
        self.length, self.device, self.dtype = k.shape[0], k.device, k.dtype

    def head(self) -> tuple:
        """(q, q stride, w, w stride, keys, batch stride, row stride, dtype, batch, length)"""
        return (self.q.data_ptr(), 0, self.w.data_ptr(), 0, self.k.data_ptr(), 0,
                self.k.stride(0), _DTYPES[self.dtype], 1, self.length)


def _block_inputs(queries, weights, keys, block_size):
    if block_size not in (16, 32, 64, 128):
        raise ValueError("block_size must be 16, 32, 64 or 128 on B200")
    one = _Single(queries, weights, keys)
    return one, math.ceil(one.length / block_size)


_BYTE_MASKS = (torch.bool, torch.int8, torch.uint8)


def _mask(mask: torch.Tensor, device) -> torch.Tensor:
    """A block mask the kernels read as one byte per block (nonzero = set): bool, int8 and
    uint8 masks already on the device are passed as they are, others are converted."""
    if mask.dtype in _BYTE_MASKS and mask.device == device and mask.is_contiguous():
        return mask
    return mask.to(device=device, dtype=torch.int8).contiguous()


def _head_ids(ids, device, count: int) -> torch.Tensor:
    if (isinstance(ids, torch.Tensor) and ids.dtype == torch.int32 and ids.device == device
            and ids.is_contiguous()):
        return ids
    return torch.as_tensor(ids).to(device=device, dtype=torch.int32).contiguous()


def _threshold(threshold, device) -> torch.Tensor:
    """The promotion threshold as a one-element float32 device tensor (a scalar is copied
    in; a device tensor is read by the kernel in place)."""
    if (isinstance(threshold, torch.Tensor) and threshold.dtype == torch.float32
            and threshold.device == device and threshold.numel() == 1):
        return threshold
    return torch.as_tensor(threshold, device=device, dtype=torch.float32).reshape(1)


def _selected_heads(selected_heads, device) -> torch.Tensor:
    if isinstance(selected_heads, torch.Tensor) and selected_heads.is_cuda:
        if selected_heads.numel() != VERIFIER_HEADS:
            raise ValueError("selected head IDs must have shape [8]")
        return _head_ids(selected_heads, device, VERIFIER_HEADS)
    selected, _ = split_head_ids(selected_heads)
    return selected.to(device)


def _call_blocks(name: str, *args) -> None:
    capi.call(name, *args)


def h8_block_max_triton(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                        selected_heads: torch.Tensor, cold_blocks: torch.Tensor, *,
                        block_size: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """:378-404 -- 8-head partial scores on cold blocks (-inf elsewhere) and block maxima."""
    _check_cuda_inputs(queries, weights, keys)
    one, nblocks = _block_inputs(queries, weights, keys, block_size)
    if cold_blocks.numel() != nblocks:
        raise ValueError("cold block mask length mismatch")
    dev = one.device
    selected = _selected_heads(selected_heads, dev)
    cold = _mask(cold_blocks, dev)
    partial = torch.empty(one.length, device=dev, dtype=torch.float32)
    maxima = torch.empty(nblocks, device=dev, dtype=torch.float32)
    _call_blocks("tdsa_h8_block_max", *one.head(), block_size, selected.data_ptr(),
                 cold.data_ptr(), partial.data_ptr(), one.length, maxima.data_ptr(), nblocks,
                 stream_ptr(dev))
    return partial, maxima


def masked_full_scores_triton(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                              keep_blocks: torch.Tensor, *, block_size: int = 64) -> torch.Tensor:
    """:407-424 -- dense scores on kept blocks, -inf elsewhere (dropped blocks are not read)."""
    _check_cuda_inputs(queries, weights, keys)
    one, nblocks = _block_inputs(queries, weights, keys, block_size)
    if keep_blocks.numel() != nblocks:
        raise ValueError("keep block mask length mismatch")
    dev = one.device
    keep = _mask(keep_blocks, dev)
    out = torch.empty(one.length, device=dev, dtype=torch.float32)
    _call_blocks("tdsa_masked_dense", *one.head(), block_size, keep.data_ptr(), nblocks,
                 out.data_ptr(), one.length, stream_ptr(dev))
    return out


def progressive_scores_triton(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                              selected_heads: torch.Tensor, direct_full_blocks: torch.Tensor,
                              threshold: float | torch.Tensor, *, block_size: int = 64,
                              compact: bool = False,
                              remaining_heads: torch.Tensor | None = None) -> ProgressiveResult:
    """:427-475 -- fused H8 probe -> promotion -> remaining 56 heads.

    Dense output: rejected blocks score -inf.  compact=True: the accepted blocks' valid
    keys packed in ascending key order, with candidate_count read back to the host (a sync,
    as in the reference).
    """
    _check_cuda_inputs(queries, weights, keys)
    one, nblocks = _block_inputs(queries, weights, keys, block_size)
    dev = one.device
    if remaining_heads is None:
        selected, remaining = split_head_ids(selected_heads.cpu())
        selected, remaining = selected.to(dev), remaining.to(dev)
    else:
        if (selected_heads.numel() != VERIFIER_HEADS
                or remaining_heads.numel() != HEADS - VERIFIER_HEADS):
            raise ValueError("expected 8 selected and 56 remaining head IDs")
        selected = _head_ids(selected_heads, dev, VERIFIER_HEADS)
        remaining = _head_ids(remaining_heads, dev, HEADS - VERIFIER_HEADS)
    if direct_full_blocks.numel() != nblocks:
        raise ValueError("direct full block mask length mismatch")
    direct = _mask(direct_full_blocks, dev)
    thr = _threshold(threshold, dev)
    length = one.length
    scores = torch.empty(length, device=dev, dtype=torch.float32)
    accepted = torch.empty(nblocks, device=dev, dtype=torch.int8)
    block_max = torch.empty(nblocks, device=dev, dtype=torch.float32)
    _call_blocks("tdsa_progressive_h8", *one.head(), block_size, selected.data_ptr(),
                 remaining.data_ptr(), direct.data_ptr(), thr.data_ptr(), scores.data_ptr(),
                 length, accepted.data_ptr(), block_max.data_ptr(), nblocks, stream_ptr(dev))
    if not compact:
        return ProgressiveResult(scores, accepted, block_max)
    packed = torch.empty(length, device=dev, dtype=torch.float32)
    indices = torch.empty(length, device=dev, dtype=torch.int32)
    count = torch.zeros(1, device=dev, dtype=torch.int32)
    _call_blocks("tdsa_compact_blocks", scores.data_ptr(), length, accepted.data_ptr(), nblocks,
                 1, length, block_size, packed.data_ptr(), indices.data_ptr(), length,
                 count.data_ptr(), stream_ptr(dev))
    candidate_count = int(count.item())
    return ProgressiveResult(packed[:candidate_count], accepted, block_max,
                             indices[:candidate_count], candidate_count)


def two_pass_scores_triton(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                           selected_heads: torch.Tensor, direct_full_blocks: torch.Tensor,
                           threshold: float | torch.Tensor, *,
                           block_size: int = 64) -> ProgressiveResult:
    """:478-497 -- H8 block max on cold blocks, then dense scoring of the accepted ones
    (direct, or probe max >= threshold): one C call (tdsa_two_pass), two launches."""
    _check_cuda_inputs(queries, weights, keys)
    one, nblocks = _block_inputs(queries, weights, keys, block_size)
    if direct_full_blocks.numel() != nblocks:
        raise ValueError("direct full block mask length mismatch")
    dev = one.device
    selected = _selected_heads(selected_heads, dev)
    direct = _mask(direct_full_blocks, dev)
    thr = _threshold(threshold, dev)
    length = one.length
    scores = torch.empty(length, device=dev, dtype=torch.float32)
    accepted = torch.empty(nblocks, device=dev, dtype=torch.int8)
    maxima = torch.empty(nblocks, device=dev, dtype=torch.float32)
    _call_blocks("tdsa_two_pass", *one.head(), block_size, selected.data_ptr(),
                 direct.data_ptr(), thr.data_ptr(), scores.data_ptr(), length,
                 accepted.data_ptr(), maxima.data_ptr(), nblocks, stream_ptr(dev))
    return ProgressiveResult(scores, accepted, maxima)


# --------------------------------------------------------------------------- torch-named
# The reference's torch_* functions (:45-90) are its readable specification of the same
# math.  Here they keep their names and outputs but run on the B200 kernels (CUDA tensors
# of any float dtype for the dense one; 16-bit for the progressive one).

def torch_full_scores(queries: torch.Tensor, weights: torch.Tensor,
                      keys: torch.Tensor) -> torch.Tensor:
    """:45-55 -- dense scores [L] float32 (float32 keys run the FP32 kernel)."""
    if queries.shape != (HEADS, HEAD_DIM) or weights.shape != (HEADS,):
        raise ValueError("expected queries [64,128] and weights [64]")
    if keys.ndim != 2 or keys.shape[1] != HEAD_DIM:
        raise ValueError("expected keys [L,128]")
    if not (queries.is_cuda and weights.is_cuda and keys.is_cuda):
        raise ValueError("the B200 indexer kernels require CUDA tensors")
    return score_dense(queries, weights, keys)


def torch_progressive_scores(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                             selected_heads: torch.Tensor, direct_full_blocks: torch.Tensor,
                             threshold: float, *, block_size: int = 64
                             ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """:58-90 -- (scores, accepted bool, block_max): the 8-head probe maximum of EVERY block
    (direct ones included), acceptance = direct or probe max >= threshold, full 64-head
    scores on accepted blocks and -inf elsewhere.  Two launches: the probe over all blocks,
    then dense scoring of the accepted blocks (rejected blocks are not read again)."""
    selected, _ = split_head_ids(selected_heads.cpu())
    length = keys.shape[0]
    nblocks = math.ceil(length / block_size)
    if direct_full_blocks.numel() != nblocks:
        raise ValueError("direct_full_blocks length mismatch")
    all_blocks = torch.ones(nblocks, dtype=torch.bool, device=keys.device)
    _, block_max = h8_block_max_triton(queries, weights, keys, selected.to(keys.device),
                                       all_blocks, block_size=block_size)
    accepted = direct_full_blocks.to(device=keys.device, dtype=torch.bool) | (
        block_max >= float(threshold))
    scores = masked_full_scores_triton(queries, weights, keys, accepted, block_size=block_size)
    return scores, accepted, block_max
