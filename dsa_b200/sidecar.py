"""Batched indexer scoring with the signature of the reference sidecar.

Mirrors ``LightningIndexerSidecar.score_encoded`` (src/temporal_dsa/sidecar.py:89-107):
queries [B,Q,64,128], weights [B,Q,64], keys [B,L,128] -> scores [B,Q,L] float32.  The
reference materialises [B,Q,64,L] head dots per key chunk; the B200 kernel keeps them in
TMEM, so ``key_chunk_size`` is accepted for call-site compatibility and has no effect.
"""

from __future__ import annotations

import torch

from . import _capi as capi
from .indexer import HEAD_DIM, HEADS, require_cuda, score_dense, stream_ptr


def score_encoded(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor, *,
                  key_chunk_size: int | None = None) -> torch.Tensor:
    require_cuda(queries, weights, keys)
    if queries.ndim != 4 or weights.shape != queries.shape[:-1]:
        raise ValueError("queries must be [batch,query,heads,dim]")
    if keys.ndim != 3 or keys.shape[0] != queries.shape[0]:
        raise ValueError("keys must be [batch,key,dim]")
    if queries.shape[2:] != (HEADS, HEAD_DIM) or keys.shape[2] != HEAD_DIM:
        raise ValueError("the B200 indexer kernels take 64 heads x 128 dims")
    if queries.dtype != keys.dtype:
        raise ValueError("queries and keys must share a dtype")
    bsz, nq = queries.shape[:2]
    out = torch.empty(bsz, nq, keys.shape[1], device=keys.device, dtype=torch.float32)
    for qi in range(nq):
        score_dense(queries[:, qi], weights[:, qi], keys, out=out[:, qi])
    return out


class SidecarScoring:
    """Mixin giving a sidecar-like module the B200 ``score_encoded``."""

    def score_encoded(self, queries, weights, keys, *, key_chunk_size=None):
        return score_encoded(queries, weights, keys, key_chunk_size=key_chunk_size)


# --------------------------------------------------------------------------- projection
# The sidecar's query/key projections (sidecar.py:10-28, :66-87), run as plain library
# GEMMs (cuBLAS through torch.matmul) and elementwise ops on the device.

def apply_noninterleaved_rope(x: torch.Tensor, positions: torch.Tensor, *,
                              theta: float = 10_000.0) -> torch.Tensor:
    """sidecar.py:10-28 -- RoPE on the two halves of the last axis (V3.2 indexer layout)."""
    if x.shape[-1] % 2:
        raise ValueError("RoPE dimension must be even")
    half = x.shape[-1] // 2
    inv_freq = theta ** (-torch.arange(half, device=x.device, dtype=torch.float32) / half)
    angles = positions.to(torch.float32).unsqueeze(-1) * inv_freq
    cos = torch.cos(angles).to(x.dtype)
    sin = torch.sin(angles).to(x.dtype)
    while cos.ndim < x.ndim:
        cos = cos.unsqueeze(-2)
        sin = sin.unsqueeze(-2)
    first, second = x[..., :half], x[..., half:]
    return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)


def encode_queries(hidden: torch.Tensor, wq: torch.Tensor, ww: torch.Tensor,
                   positions: torch.Tensor, *, rope_dim: int = 64,
                   rope_theta: float = 10_000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """sidecar.py:78-87 -- hidden [...,2048] -> q [...,64,128] (hidden dtype), w [...,64] f32.

    wq [64*128, 2048] and ww [64, 2048] are the nn.Linear weights; the head weights are
    computed in float32 and scaled by (64*128)^-1/2 as in the reference.
    """
    require_cuda(hidden, wq, ww)
    q = torch.matmul(hidden, wq.t()).view(*hidden.shape[:-1], HEADS, HEAD_DIM)
    if rope_dim:
        q = torch.cat((apply_noninterleaved_rope(q[..., :rope_dim], positions, theta=rope_theta),
                       q[..., rope_dim:]), dim=-1)
    w = torch.matmul(hidden.float(), ww.float().t()) * (HEADS * HEAD_DIM) ** -0.5
    return q, w


class QueryProjector:
    """Decode-step query projection on fixed buffers, one launch (tdsa_query_project): the
    W_q GEMM on the tensor cores with RoPE in its epilogue, and the float32 head weights
    computed from the same staged hidden states.

    ``project(hidden, positions)`` -> (q [B,64,128], w [B,64] float32), written into
    ``self.q`` / ``self.w`` (stable addresses, so a ScoreTopkPlan can be built on them).
    keep_qraw=True also keeps the pre-RoPE projection in ``self.qraw`` [B, 8192].
    packed=True (default) re-lays W_q out once (tdsa_pack_query_weights) so that every tile
    the kernel streams is one contiguous block.
    """

    def __init__(self, wq: torch.Tensor, ww: torch.Tensor, batch: int, *, rope_dim: int = 64,
                 rope_theta: float = 10_000.0, keep_qraw: bool = False, packed: bool = True):
        require_cuda(wq, ww)
        if wq.shape[0] != HEADS * HEAD_DIM or ww.shape[0] != HEADS:
            raise ValueError("expected wq [8192, hidden] and ww [64, hidden]")
        if wq.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("wq must be bf16 or fp16")
        if ww.shape[1] != wq.shape[1]:
            raise ValueError("wq and ww must share the hidden size")
        if wq.shape[1] % 8:
            raise ValueError("the hidden size must be a multiple of 8")
        dev = wq.device
        self.hidden = wq.shape[1]
        wq = wq if (wq.stride(-1) == 1 and wq.stride(0) % 8 == 0
                    and wq.data_ptr() % 16 == 0) else wq.contiguous()
        lib = capi.lib()
        if packed:
            # one-time re-layout: every (head, 64-wide K chunk) tile one contiguous block
            nbytes = lib.tdsa_packed_query_weights_bytes(self.hidden)
            self.wq = torch.empty(nbytes // 2, device=dev, dtype=wq.dtype)
            capi.check(lib.tdsa_pack_query_weights(wq.data_ptr(), wq.stride(0), self.hidden,
                                                   self.wq.data_ptr(),
                                                   stream_ptr(dev)))
            self._wq_stride = 0
        else:
            self.wq, self._wq_stride = wq, wq.stride(0)
        self.packed = bool(packed)
        self.ww = ww.to(torch.float32).contiguous()
        self.dtype = wq.dtype
        self.batch, self.rope_dim, self.theta = batch, rope_dim, rope_theta
        self.qraw = (torch.empty(batch, HEADS * HEAD_DIM, device=dev, dtype=wq.dtype)
                     if keep_qraw else None)
        self.q = torch.empty(batch, HEADS, HEAD_DIM, device=dev, dtype=wq.dtype)
        self.w = torch.empty(batch, HEADS, device=dev, dtype=torch.float32)
        # the kernel reads W_q and W_w before it waits on the previous kernel of the stream:
        # the packed weights must be complete before the first projection
        torch.cuda.current_stream(dev).synchronize()
        self._fn = capi.lib().tdsa_query_project
        self._dt = capi.TDSA_BF16 if wq.dtype == torch.bfloat16 else capi.TDSA_F16

    def project(self, hidden: torch.Tensor, positions: torch.Tensor):
        if hidden.shape != (self.batch, self.hidden) or hidden.dtype != self.dtype:
            raise ValueError("hidden must be [batch, hidden] in the projection dtype")
        if hidden.stride(-1) != 1 or hidden.stride(0) % 8 or hidden.data_ptr() % 16:
            hidden = hidden.contiguous() if hidden.stride(-1) != 1 else hidden.clone()
        if positions.dtype != torch.int64 or not positions.is_contiguous():
            positions = positions.to(torch.int64).contiguous()
        capi.check(self._fn(hidden.data_ptr(), hidden.stride(0), self.hidden, self.wq.data_ptr(),
                            self._wq_stride, int(self.packed), self.ww.data_ptr(),
                            positions.data_ptr(),
                            self.q.data_ptr(), HEADS * HEAD_DIM, self.w.data_ptr(), HEADS,
                            self._dt, self.batch, self.rope_dim, self.theta,
                            (HEADS * HEAD_DIM) ** -0.5,
                            self.qraw.data_ptr() if self.qraw is not None else None,
                            HEADS * HEAD_DIM,
                            stream_ptr(self.q.device)))
        return self.q, self.w


def encode_keys(hidden: torch.Tensor, wk: torch.Tensor, norm_weight: torch.Tensor,
                norm_bias: torch.Tensor, positions: torch.Tensor, *, rope_dim: int = 64,
                rope_theta: float = 10_000.0, eps: float = 1e-6) -> torch.Tensor:
    """sidecar.py:74-76 -- k = RoPE(LayerNorm(hidden @ wk^T)) [..., 128]."""
    require_cuda(hidden, wk)
    k = torch.matmul(hidden, wk.t())
    k = torch.nn.functional.layer_norm(k, (HEAD_DIM,), norm_weight.to(k.dtype),
                                       norm_bias.to(k.dtype), eps)
    if rope_dim:
        k = torch.cat((apply_noninterleaved_rope(k[..., :rope_dim], positions, theta=rope_theta),
                       k[..., rope_dim:]), dim=-1)
    return k


class KeyAppender:
    """Decode-step key append, one launch (tdsa_key_append): for each sequence the new
    token's key RoPE(LayerNorm(hidden @ wk^T)) (sidecar.py:74-76) is computed and written
    straight into that sequence's cache row.

    ``append(hidden [B, hidden], positions [B], cache [B, L, 128], slots=None)``: the key of
    sequence b goes to ``cache[b, slots[b]]`` (``slots=None``: ``positions[b]``).  A slot
    outside ``[0, L)`` is skipped and raises TDSA_STATUS_RANGE in the device status word.
    """

    def __init__(self, wk: torch.Tensor, norm_weight: torch.Tensor | None = None,
                 norm_bias: torch.Tensor | None = None, *, rope_dim: int = 64,
                 rope_theta: float = 10_000.0, eps: float = 1e-6):
        require_cuda(wk)
        if wk.dim() != 2 or wk.shape[0] != HEAD_DIM:
            raise ValueError("expected wk [128, hidden]")
        if wk.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("wk must be bf16 or fp16")
        if wk.shape[1] % 8:
            raise ValueError("the hidden size must be a multiple of 8")
        dev = wk.device
        self.wk = wk if (wk.stride(-1) == 1 and wk.stride(0) % 8 == 0
                         and wk.data_ptr() % 16 == 0) else wk.contiguous()
        self.hidden, self.dtype = wk.shape[1], wk.dtype
        self.norm_weight = (None if norm_weight is None
                            else norm_weight.to(dev, torch.float32).contiguous())
        self.norm_bias = (None if norm_bias is None
                          else norm_bias.to(dev, torch.float32).contiguous())
        for t in (self.norm_weight, self.norm_bias):
            if t is not None and t.shape != (HEAD_DIM,):
                raise ValueError("LayerNorm weight and bias must be [128]")
        self.rope_dim, self.theta, self.eps = int(rope_dim), float(rope_theta), float(eps)
        # the kernel reads W_k before it waits on the previous kernel of the stream: the
        # weights must be complete before the first append
        torch.cuda.current_stream(dev).synchronize()
        self._fn = capi.lib().tdsa_key_append
        self._dt = capi.TDSA_BF16 if wk.dtype == torch.bfloat16 else capi.TDSA_F16

    def append(self, hidden: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor,
               slots: torch.Tensor | None = None) -> torch.Tensor:
        require_cuda(hidden, positions, cache)
        batch = hidden.shape[0]
        if hidden.shape != (batch, self.hidden) or hidden.dtype != self.dtype:
            raise ValueError("hidden must be [batch, hidden] in the weights' dtype")
        if cache.dim() != 3 or cache.shape[0] != batch or cache.shape[2] != HEAD_DIM:
            raise ValueError("cache must be [batch, L, 128]")
        if cache.dtype != self.dtype or cache.stride(-1) != 1:
            raise ValueError("cache must share the weights' dtype with unit last stride")
        if hidden.stride(-1) != 1 or hidden.stride(0) % 8 or hidden.data_ptr() % 16:
            hidden = hidden.contiguous() if hidden.stride(-1) != 1 else hidden.clone()
        positions = positions.to(torch.int64).contiguous()
        if positions.shape != (batch,):
            raise ValueError("positions must be [batch]")
        if slots is not None:
            slots = slots.to(torch.int64).contiguous()
            if slots.shape != (batch,):
                raise ValueError("slots must be [batch]")
        capi.check(self._fn(
            hidden.data_ptr(), hidden.stride(0), self.hidden, self.wk.data_ptr(),
            self.wk.stride(0),
            self.norm_weight.data_ptr() if self.norm_weight is not None else None,
            self.norm_bias.data_ptr() if self.norm_bias is not None else None, self.eps,
            positions.data_ptr(), slots.data_ptr() if slots is not None else None,
            cache.data_ptr(), cache.stride(0), cache.stride(1), cache.shape[1], self._dt, batch,
            self.rope_dim, self.theta, stream_ptr(cache.device)))
        return cache
