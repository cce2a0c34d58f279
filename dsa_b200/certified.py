"""Device (float64) versions of ``temporal_dsa.certified`` (src/temporal_dsa/certified.py).

Same names, argument meaning and ValueError checks as the reference; inputs are CUDA
tensors (any float dtype, computed in float64), outputs float64 CUDA tensors.
"""

from __future__ import annotations

import torch

from . import _capi as capi
from .indexer import require_cuda, stream_ptr


def _f64(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float64).contiguous()


def relu_index_score(q: torch.Tensor, keys: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """:6-15 -- I_s = sum_j w_j ReLU(q_j . k_s), q [heads,dim], keys [tokens,dim]."""
    require_cuda(q, keys, weights)
    if q.ndim != 2 or keys.ndim != 2 or q.shape[1] != keys.shape[1]:
        raise ValueError("q must be [heads,dim] and keys [tokens,dim]")
    if weights.shape != (q.shape[0],):
        raise ValueError("weights must have one value per head")
    q, keys, weights = _f64(q), _f64(keys), _f64(weights)
    out = torch.empty(keys.shape[0], device=keys.device, dtype=torch.float64)
    capi.call("tdsa_relu_index_score", q.data_ptr(), keys.data_ptr(), weights.data_ptr(),
              q.shape[0], q.shape[1], keys.shape[0], out.data_ptr(), stream_ptr(keys.device))
    return out


def temporal_score_radius(q_now: torch.Tensor, q_prev: torch.Tensor, w_now: torch.Tensor,
                          w_prev: torch.Tensor, block_key_norm: torch.Tensor) -> torch.Tensor:
    """:18-48 -- certified per-block radius of |I_t - I_(t-1)| (signed weights via |.|)."""
    require_cuda(q_now, q_prev, w_now, w_prev, block_key_norm)
    if q_now.shape != q_prev.shape or q_now.ndim != 2:
        raise ValueError("query tensors must have shape [heads,dim]")
    if w_now.shape != w_prev.shape or w_now.shape != (q_now.shape[0],):
        raise ValueError("weight tensors must have shape [heads]")
    if block_key_norm.ndim != 2 or block_key_norm.shape[1] != q_now.shape[0]:
        raise ValueError("block_key_norm must have shape [blocks,heads]")
    qn, qp, wn, wp, nrm = map(_f64, (q_now, q_prev, w_now, w_prev, block_key_norm))
    heads, dim = qn.shape
    out = torch.empty(nrm.shape[0], device=nrm.device, dtype=torch.float64)
    coeff = torch.empty(heads, device=nrm.device, dtype=torch.float64)
    capi.call("tdsa_temporal_radius", qn.data_ptr(), qp.data_ptr(), wn.data_ptr(), wp.data_ptr(),
              nrm.data_ptr(), heads, dim, nrm.shape[0], coeff.data_ptr(), out.data_ptr(),
              stream_ptr(nrm.device))
    return out


def block_key_norms(keys: torch.Tensor, block_size: int) -> torch.Tensor:
    """:51-61 -- max key L2 norm per block and head for keys [tokens,heads,dim]."""
    require_cuda(keys)
    if keys.ndim != 3:
        raise ValueError("keys must have shape [tokens,heads,dim]")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    k = _f64(keys)
    tokens, heads, dim = k.shape
    nb = (tokens + block_size - 1) // block_size
    out = torch.empty(nb, heads, device=k.device, dtype=torch.float64)
    if tokens:
        capi.call("tdsa_block_key_norms", k.data_ptr(), tokens, heads, dim, block_size,
                  out.data_ptr(), stream_ptr(k.device))
    return out
