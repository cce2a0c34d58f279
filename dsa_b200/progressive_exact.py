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
