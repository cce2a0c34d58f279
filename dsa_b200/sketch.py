"""Certified INT8 key sketch and the exact top-k that reads full keys only where the sketch
cannot rule them out.

The reference quantizes keys with one symmetric scale per tensor and scores the quantized
keys as an approximate verifier (``fake_symmetric_quantize`` and ``score_dim_sparse``,
src/temporal_dsa/verifier_scoring.py:29-41, :95-139).  Here each key gets its own scale and
two rounded-up norms (136 bytes per key instead of 256), which bound how far its true score
can lie from its sketch score.  ``sketch_topk`` scores every key's sketch, takes tau = the
k-th largest certified lower bound (never above the k-th true score) and reads the full key
only for the 16-key blocks holding a key whose certified upper bound reaches tau.  The
returned top-k is dense scoring's, ties included.

    sk = KeySketch(batch, max_length, device="cuda")
    sk.update(keys)                          # or sk.update(keys, start, stop) after appends
    idx, val = sketch_topk(q, w, keys, sk, 2048)
    plan = SketchTopkPlan(q_buf, w_buf, keys, sk, 2048)   # the decode-loop form
    idx, val = plan.run(length)
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _capi as capi
from .indexer import _DTYPES, HEAD_DIM, as_batched, prepare_keys, prepare_queries, \
    prepare_weights, require_cuda, stream_ptr

BYTES_PER_KEY = HEAD_DIM + 4 + 4  # int8 values, float32 scale, two float16 bounds


class KeySketch:
    """The INT8 sketch of a [batch, max_length, 128] 16-bit key cache on the device:
    ``values`` int8 [B, L, 128], ``scales`` float32 [B, L], ``bounds`` float16 [B, L, 2]
    (residual norm, norm; both rounded up)."""

    def __init__(self, batch: int, max_length: int, device: torch.device | str = "cuda"):
        if batch < 1 or max_length < 1:
            raise ValueError("batch and max_length must be positive")
        dev = torch.device(device)
        self.batch, self.max_length, self.device = batch, max_length, dev
        self.values = torch.zeros(batch, max_length, HEAD_DIM, device=dev, dtype=torch.int8)
        self.scales = torch.zeros(batch, max_length, device=dev, dtype=torch.float32)
        self.bounds = torch.zeros(batch, max_length, 2, device=dev, dtype=torch.float16)
        self.length = 0

    def update(self, keys: torch.Tensor, start: int = 0, stop: int | None = None) -> None:
        """Sketch keys [start, stop) of ``keys`` [B, >= stop, 128] (bf16/fp16)."""
        require_cuda(keys)
        if keys.dim() == 2:
            keys = keys.unsqueeze(0)
        if keys.dim() != 3 or keys.shape[0] != self.batch or keys.shape[2] != HEAD_DIM:
            raise ValueError("keys must be [batch, L, 128]")
        if keys.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("the key sketch takes bf16/fp16 keys")
        stop = keys.shape[1] if stop is None else stop
        if not 0 <= start <= stop <= min(keys.shape[1], self.max_length):
            raise ValueError("need 0 <= start <= stop <= min(L, max_length)")
        keys = prepare_keys(keys)
        capi.call("tdsa_sketch_keys", keys.data_ptr(), keys.stride(0), keys.stride(1),
                  _DTYPES[keys.dtype], self.batch, start, stop, self.values.data_ptr(),
                  self.values.stride(0), self.scales.data_ptr(), self.bounds.data_ptr(),
                  self.scales.stride(0), stream_ptr(keys.device))
        self.length = max(self.length, stop)


class SketchTopkPlan:
    """``sketch_topk`` on fixed device buffers (the decode-loop form): the caller rewrites
    ``queries`` / ``weights`` in place and appends keys (then ``sketch.update``) between
    steps; ``run(length)`` is one C call.  Results land in ``indices`` / ``values``."""

    def __init__(self, queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                 sketch: KeySketch, k: int, *, sorted: bool = False,
                 index_dtype: torch.dtype = torch.int32):
        require_cuda(queries, weights, keys)
        q, w, kk, _ = as_batched(queries, weights, keys)
        if not (q.is_contiguous() and q.data_ptr() % 16 == 0 and q.dtype == kk.dtype):
            raise ValueError("plan queries must be contiguous, 16-byte aligned, keys' dtype")
        if not (w.dtype == torch.float32 and w.is_contiguous()):
            raise ValueError("plan weights must be contiguous float32")
        if prepare_keys(kk) is not kk or kk.dtype == torch.float32:
            raise ValueError("plan keys must be 16-bit and satisfy the TMA layout rules")
        if sketch.batch != kk.shape[0] or sketch.max_length < kk.shape[1]:
            raise ValueError("the sketch does not cover this key cache")
        self.q, self.w, self.keys, self.sketch = q, w, kk, sketch
        self.batch, self.max_length, self.k = kk.shape[0], kk.shape[1], k
        if not 0 < k <= self.max_length:
            raise ValueError(f"k={k} is invalid for {self.max_length} keys")
        dev = kk.device
        lib = capi.lib()
        nbytes = lib.tdsa_sketch_topk_workspace_bytes(self.batch, self.max_length, k)
        self.workspace = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        self._ws_bytes = nbytes
        self.indices = torch.empty(self.batch, k, device=dev, dtype=index_dtype)
        self.values = torch.empty(self.batch, k, device=dev, dtype=torch.float32)
        self.counters = torch.zeros(self.batch, 2, device=dev, dtype=torch.int64)
        self._head = (q.data_ptr(), q.stride(0), w.data_ptr(), w.stride(0), kk.data_ptr(),
                      kk.stride(0), kk.stride(1), _DTYPES[kk.dtype], sketch.values.data_ptr(),
                      sketch.values.stride(0), sketch.scales.data_ptr(),
                      sketch.bounds.data_ptr(), sketch.scales.stride(0), self.batch)
        self._tail = (self.max_length, k, int(bool(sorted)), self.indices.data_ptr(),
                      self.indices.element_size(), self.indices.stride(0),
                      self.values.data_ptr(), self.values.stride(0), self.counters.data_ptr(),
                      self.workspace.data_ptr(), nbytes)
        self.device = dev
        self.length = self.max_length

    def run(self, length: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        length = self.max_length if length is None else length
        if not self.k <= length <= self.max_length:
            raise ValueError("need k <= length <= the cache length")
        capi.check(capi.lib().tdsa_sketch_topk(*self._head, length, *self._tail,
                                               stream_ptr(self.device)))
        self.length = length
        return self.indices, self.values

    def stats(self) -> list[dict]:
        """Accumulated per-sequence counters: keys read in full, 16-key blocks read (reads
        device memory: synchronous)."""
        c = self.counters.cpu().tolist()
        return [{"keys_read": r[0], "blocks_read": r[1]} for r in c]

    def bounds(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Views of the last run's certified bounds: the largest upper bound of every 16-key
        block [B, ceil(length / 16)], the lower bound of every key [B, length], tau [B]."""
        off = (C.c_int64 * 6)()
        capi.check(capi.lib().tdsa_sketch_workspace_offsets(self.batch, self.max_length,
                                                            self.k, off))
        nb_stride, ld = off[4], off[5]

        def rows(o, width, used):
            n = self.batch * width * 4
            return self.workspace[o:o + n].view(torch.float32).view(self.batch, width)[:, :used]

        tau = self.workspace[off[3]:off[3] + 4 * self.batch].view(torch.float32)
        return (rows(off[0], nb_stride, (self.length + 15) // 16),
                rows(off[1], ld, self.length), tau)


def sketch_topk(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                sketch: KeySketch, k: int, *, sorted: bool = True,
                index_dtype: torch.dtype = torch.int64) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact top-k of the dense scores of ``keys`` [B, L, 128] (or one sequence [L, 128]),
    reading each key's sketch and the full keys only where the sketch's certified upper
    bound reaches the k-th score's lower bound -> (indices, values)."""
    require_cuda(queries, weights, keys)
    q, w, kk, single = as_batched(queries, weights, keys)
    kk = prepare_keys(kk)
    if kk.dtype == torch.float32:
        raise ValueError("the key sketch takes bf16/fp16 keys")
    q = prepare_queries(q, kk.dtype)
    w = prepare_weights(w)
    bsz, length = kk.shape[0], kk.shape[1]
    if sketch.batch != bsz or sketch.max_length < length:
        raise ValueError("the sketch does not cover these keys")
    if not 0 < k <= length:
        raise ValueError(f"k={k} is invalid for {length} keys")
    dev = kk.device
    nbytes = capi.lib().tdsa_sketch_topk_workspace_bytes(bsz, length, k)
    ws = torch.empty(nbytes, device=dev, dtype=torch.uint8)
    idx = torch.empty(bsz, k, device=dev, dtype=index_dtype)
    val = torch.empty(bsz, k, device=dev, dtype=torch.float32)
    capi.call("tdsa_sketch_topk", q.data_ptr(), q.stride(0), w.data_ptr(), w.stride(0),
              kk.data_ptr(), kk.stride(0), kk.stride(1), _DTYPES[kk.dtype],
              sketch.values.data_ptr(), sketch.values.stride(0), sketch.scales.data_ptr(),
              sketch.bounds.data_ptr(), sketch.scales.stride(0), bsz, length, length, k,
              int(bool(sorted)), idx.data_ptr(), idx.element_size(), idx.stride(0),
              val.data_ptr(), val.stride(0), None, ws.data_ptr(), nbytes, stream_ptr(dev))
    return (idx[0], val[0]) if single else (idx, val)
