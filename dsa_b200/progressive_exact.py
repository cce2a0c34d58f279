"""Exact (certified) progressive top-k over a growing key cache.

The reference project measures this schedule only in replay on precomputed scores
(src/temporal_dsa/replay.py:172-222, :263-266) and states the safe bound separately
(src/temporal_dsa/certified.py:18-48).  Here it runs on the device: each step seeds from
the previous step's top-k, scores the blocks holding those keys and the new keys first,
and skips every other block whose certified bound U_b + maxnorm_b * c falls below the
running k-th score -- those keys are never read from HBM.  The returned top-k is exactly
dense scoring's (same kernels, same arithmetic, strictly-below pruning).

    idx = ExactProgressiveTopK(batch, max_length, k, block_size=64)
    top, val = idx.init(q, w, keys)            # first step: dense
    top, val = idx.step(q, w, keys)            # later steps: keys may have grown
    idx.stats()                                # blocks/keys scored and pruned so far
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _capi as capi
from .indexer import (_DTYPES, as_batched, prepare_keys, prepare_queries, prepare_weights,
                      require_cuda, stream_ptr)

STAT_NAMES = ("steps", "blocks_visited", "blocks_scored", "blocks_pruned", "keys_scored",
              "keys_total", "first_wave_blocks", "second_wave_blocks")


class ExactProgressiveTopK:
    """Device state of the exact progressive path for `batch` sequences."""

    def __init__(self, batch: int, max_length: int, k: int, *, block_size: int = 64,
                 dtype: torch.dtype = torch.bfloat16, device: torch.device | str | None = None,
                 sorted: bool = True, index_dtype: torch.dtype = torch.int64):
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("the exact progressive path takes bf16/fp16 keys")
        if block_size not in (16, 32, 64, 128):
            raise ValueError("block_size must be 16, 32, 64 or 128")
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.batch, self.max_length, self.k = batch, max_length, k
        self.block_size, self.dtype, self.sorted = block_size, dtype, sorted
        self.index_dtype = index_dtype
        nbytes = capi.lib().tdsa_exact_state_bytes(batch, max_length, k, block_size)
        if nbytes == 0:
            raise ValueError("invalid geometry (need 1 <= k <= max_length)")
        self.state = torch.zeros(nbytes, device=self.device, dtype=torch.uint8)
        self.state_bytes = nbytes
        self.length = 0

    def _call(self, name: str, queries, weights, keys, extra):
        require_cuda(queries, weights, keys)
        q, w, kk, single = as_batched(queries, weights, keys)
        if single and self.batch != 1:
            raise ValueError("a batched state needs batched inputs")
        kk = prepare_keys(kk)
        if kk.dtype != self.dtype or kk.shape[0] != self.batch:
            raise ValueError("keys must be [batch, L, 128] in the state's dtype")
        q = prepare_queries(q, kk.dtype)
        w = prepare_weights(w)
        length = kk.shape[1]
        if length > self.max_length:
            raise ValueError("key cache longer than max_length")
        idx = torch.empty(self.batch, self.k, device=kk.device, dtype=self.index_dtype)
        val = torch.empty(self.batch, self.k, device=kk.device, dtype=torch.float32)
        args = [self.state.data_ptr(), self.state_bytes, q.data_ptr(), q.stride(0), w.data_ptr(),
                w.stride(0), kk.data_ptr(), kk.stride(0), kk.stride(1), _DTYPES[kk.dtype],
                self.batch]
        args += extra(length)
        args += [self.max_length, self.k, self.block_size, int(self.sorted), idx.data_ptr(),
                 idx.element_size(), idx.stride(0), val.data_ptr(), val.stride(0),
                 stream_ptr(kk.device)]
        capi.call(name, *args)
        self.length = length
        return (idx[0], val[0]) if single else (idx, val)

    def init(self, queries, weights, keys):
        """First step: dense scores, top-k, block maxima and key norms."""
        return self._call("tdsa_exact_init", queries, weights, keys, lambda n: [n])

    def step(self, queries, weights, keys):
        """Next decode step; keys may have grown since the last call (append-only)."""
        if self.length == 0:
            raise RuntimeError("call init() first")
        prev = self.length
        return self._call("tdsa_exact_step", queries, weights, keys, lambda n: [prev, n])

    def stats(self) -> list[dict]:
        """Accumulated per-sequence counters (reads device memory: synchronous)."""
        buf = (C.c_uint64 * (8 * self.batch))()
        capi.check(capi.lib().tdsa_exact_stats(self.state.data_ptr(), self.state_bytes,
                                               self.batch, self.max_length, self.k,
                                               self.block_size, buf))
        return [dict(zip(STAT_NAMES, buf[8 * b: 8 * b + 8])) for b in range(self.batch)]


class ExactProgressivePlan:
    """The exact progressive path on fixed buffers (the decode-loop form).

    ``queries`` [B,64,128] and ``weights`` [B,64] float32 are rewritten in place by the
    caller between steps, and new keys are appended to ``keys`` [B, max_length, 128] (the
    cache buffer, read up to the step's length).  ``init(length)`` / ``step(length)`` are one
    C call each with no per-call validation or allocation; the selection lands in
    ``indices`` / ``values`` [B, k]."""

    def __init__(self, queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor, k: int,
                 *, block_size: int = 64, sorted: bool = True,
                 index_dtype: torch.dtype = torch.int32):
        require_cuda(queries, weights, keys)
        q, w, kk, _ = as_batched(queries, weights, keys)
        if not (q.is_contiguous() and q.data_ptr() % 16 == 0 and q.dtype == kk.dtype):
            raise ValueError("plan queries must be contiguous, 16-byte aligned, keys' dtype")
        if not (w.dtype == torch.float32 and w.is_contiguous()):
            raise ValueError("plan weights must be contiguous float32")
        if prepare_keys(kk) is not kk:
            raise ValueError("plan keys must already satisfy the TMA layout rules")
        self.q, self.w, self.keys = q, w, kk
        self.batch, self.max_length = kk.shape[0], kk.shape[1]
        self.exact = ExactProgressiveTopK(self.batch, self.max_length, k, block_size=block_size,
                                          dtype=kk.dtype, device=kk.device, sorted=sorted,
                                          index_dtype=index_dtype)
        self.indices = torch.empty(self.batch, k, device=kk.device, dtype=index_dtype)
        self.values = torch.empty(self.batch, k, device=kk.device, dtype=torch.float32)
        ex = self.exact
        self._head = (ex.state.data_ptr(), ex.state_bytes, q.data_ptr(), q.stride(0),
                      w.data_ptr(), w.stride(0), kk.data_ptr(), kk.stride(0), kk.stride(1),
                      _DTYPES[kk.dtype], self.batch)
        self._tail = (self.max_length, k, block_size, int(bool(sorted)),
                      self.indices.data_ptr(), self.indices.element_size(),
                      self.indices.stride(0), self.values.data_ptr(), self.values.stride(0))
        self.length = 0

    def init(self, length: int):
        """First step over keys [:, :length]: dense scores, top-k, block maxima, key norms."""
        if not 0 < length <= self.max_length:
            raise ValueError("length outside the key buffer")
        capi.check(capi.lib().tdsa_exact_init(*self._head, length, *self._tail,
                                              stream_ptr(self.keys.device)))
        self.length = self.exact.length = length
        return self.indices, self.values

    def step(self, length: int):
        """Next decode step over keys [:, :length] (length >= the previous one)."""
        if self.length == 0:
            raise RuntimeError("call init() first")
        if not self.length <= length <= self.max_length:
            raise ValueError("the cache is append-only and bounded by the key buffer")
        capi.check(capi.lib().tdsa_exact_step(*self._head, self.length, length, *self._tail,
                                              stream_ptr(self.keys.device)))
        self.length = self.exact.length = length
        return self.indices, self.values

    def stats(self) -> list[dict]:
        return self.exact.stats()
