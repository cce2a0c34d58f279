"""Drop-in for ``temporal_dsa.verifier_scoring`` on B200: the head-sparse and the
dimension-sparse verifier scorers.

``score_head_sparse`` (reference src/temporal_dsa/verifier_scoring.py:49-92) scores Q
queries against one shared key cache with only the selected heads.  Selecting heads is the
same as giving the other heads weight zero, so each query runs the dense tcgen05 kernel
with w'_h = w_h * (times head h is selected): sum_h w'_h ReLU(q_h . k) equals the
reference's sum over the selected list (its ReLU(.)*0 terms are exact zeros).  The
reference rounds 16-bit head dots to the input dtype before the ReLU; the kernel keeps
them in float32, so 16-bit results agree to the 16-bit tolerance, float32 ones to 1e-5.

``dynamic_head_indices`` (:142-159) is the reference's stable per-query head ranking.

``score_dim_sparse`` (:95-139) keeps a subset of the 128 dimensions, optionally after the
orthonormal Hadamard rotation (``normalized_hadamard``, :9-26) and with symmetric fake
quantization (``fake_symmetric_quantize``, :29-41).  On the device the rotation, the
selection and the quantization produce 128-wide rows with zeros in the dropped
dimensions (tdsa_hadamard128, tdsa_select_quantize), and the dense tcgen05 / FP32 scorer
runs on them: a dot product over the kept dimensions is the reference's dot product over
the selected ones.  The Hadamard transform takes 128-wide rows (the indexer's head_dim).
"""

from __future__ import annotations

import torch

from . import _capi as capi
from .indexer import _DTYPES, HEAD_DIM, HEADS, require_cuda, score_dense, stream_ptr


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


def normalized_hadamard(tensor: torch.Tensor) -> torch.Tensor:
    """:9-26 -- orthonormal Walsh-Hadamard transform on the last axis (128 wide)."""
    require_cuda(tensor)
    size = tensor.shape[-1]
    if size <= 0 or size & (size - 1):
        raise ValueError("Hadamard dimension must be a positive power of two")
    if size != HEAD_DIM:
        raise ValueError("the B200 kernel transforms 128-wide rows")
    if tensor.dtype not in _DTYPES:
        raise ValueError("dtype must be float32, bfloat16 or float16")
    x = tensor.reshape(-1, size)
    if x.stride(-1) != 1:
        x = x.contiguous()
    out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    capi.call("tdsa_hadamard128", x.data_ptr(), x.stride(0), x.shape[0], _DTYPES[x.dtype],
              out.data_ptr(), out.stride(0), stream_ptr(x.device))
    return out.view(tensor.shape)


def _select_quantize(x: torch.Tensor, keep: torch.Tensor | None, bits: int | None,
                     scale: float | None) -> tuple[torch.Tensor, float | None]:
    """Rows of x (last axis) with the dropped dimensions zeroed and the kept ones
    optionally fake-quantized; returns (values, scale used or None)."""
    if x.dtype not in _DTYPES:
        raise ValueError("dtype must be float32, bfloat16 or float16")
    width = x.shape[-1]
    flat = x.reshape(-1, width)
    if flat.stride(-1) != 1:
        flat = flat.contiguous()
    out = torch.empty(flat.shape, device=x.device, dtype=x.dtype)
    word = torch.zeros(1, device=x.device, dtype=torch.int32)
    nbits = 0 if bits is None else int(bits)
    capi.call("tdsa_select_quantize", flat.data_ptr(), flat.stride(0), flat.shape[0], width,
              _DTYPES[x.dtype], keep.data_ptr() if keep is not None else None, nbits,
              float(scale) if scale is not None else 0.0, word.data_ptr(), out.data_ptr(),
              out.stride(0), stream_ptr(x.device))
    used = None
    if nbits:
        if scale is None:
            absmax = float(word.view(torch.float32).item())  # host read, as the reference's
            scale = absmax / max(2 ** (nbits - 1) - 1, 1)
        used = max(float(scale), 1e-12)
    return out.view(x.shape), used


def fake_symmetric_quantize(tensor: torch.Tensor, bits: int, scale: float | None = None):
    """:29-41 -- (clamp(round(x / s), -L, L) * s in the tensor's dtype, s), L = 2^(bits-1)-1,
    s = max|x| / L unless given."""
    require_cuda(tensor)
    if bits not in {2, 4, 8}:
        raise ValueError("bits must be one of 2, 4, 8")
    return _select_quantize(tensor, None, bits, scale)


def score_dim_sparse(queries, weights, keys, dimension_indices, *, rotation: str = "none",
                     bits: int | None = None, query_scale: float | None = None,
                     key_scale: float | None = None, query_chunk_size: int = 1,
                     key_chunk_size: int = 8192) -> torch.Tensor:
    """:95-139 -- all-head scores on a subset of (rotated, optionally quantized)
    dimensions, float32 [Q, K].  The chunk sizes are reference tiling knobs."""
    if queries.ndim != 3 or weights.shape != queries.shape[:2] or keys.ndim != 2:
        raise ValueError("expected queries [Q,H,D], weights [Q,H], keys [K,D]")
    require_cuda(queries, weights, keys)
    if rotation not in ("none", "hadamard"):
        raise ValueError("rotation must be 'none' or 'hadamard'")
    if queries.shape[1:] != (HEADS, HEAD_DIM) or keys.shape[1] != HEAD_DIM:
        raise ValueError("the B200 indexer kernels take 64 heads x 128 dims")
    if bits is not None and bits not in {2, 4, 8}:
        raise ValueError("bits must be one of 2, 4, 8")
    q, k = queries, keys
    if rotation == "hadamard":
        q, k = normalized_hadamard(q), normalized_hadamard(k)
    dims = torch.as_tensor(dimension_indices, device=queries.device, dtype=torch.long)
    if dims.numel() and (int(dims.min()) < 0 or int(dims.max()) >= HEAD_DIM):
        raise IndexError("dimension index outside [0, 128)")
    keep = torch.zeros(HEAD_DIM, device=queries.device, dtype=torch.int8)
    keep[dims] = 1
    qs, _ = _select_quantize(q, keep, bits, query_scale)
    ks, _ = _select_quantize(k.to(q.dtype) if k.dtype != q.dtype else k, keep, bits, key_scale)
    out = torch.empty(queries.shape[0], keys.shape[0], device=keys.device, dtype=torch.float32)
    if keys.shape[0]:
        for i in range(queries.shape[0]):
            score_dense(qs[i], weights[i].float(), ks, out=out[i])
    return out
