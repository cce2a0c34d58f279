"""Multi-GPU sharding of the indexer decode step: one process per GPU, torch.distributed.

Two layouts:

* batch sharding (independent sequences, configs 2 and 4): each rank scores and selects its
  own sequences.  There is nothing to exchange; ``batch_shard`` only says which rows a rank
  owns.
* L sharding (one long context split over GPUs, config 5): rank r holds the contiguous keys
  [start_r, stop_r) of every sequence, scores them and keeps its local top-k with global
  indices (local index + start_r).  The candidates of all ranks are all-gathered (NCCL over
  NVLink on GPUs) and merged by ``tdsa_merge_topk``.  This is exact, ties included: every
  member of the global top-k is in its own shard's local top-k, the gathered rows are in
  ascending index order (shards are contiguous and in rank order, each local list is in
  ascending index order), and the merge applies the same lowest-index-first tie rule.

The reference never shards (its scoring is single-GPU); the merge is new.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from .indexer import merge_topk, scores_topk

Candidates = tuple[torch.Tensor, torch.Tensor]  # values [B, k] f32, indices [B, k] int32


def shard_bounds(length: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous key range [start, stop) of `rank`: the first length % world ranks hold one
    key more than the others."""
    if not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    base, extra = divmod(length, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def batch_shard(batch: int, rank: int, world: int) -> slice:
    """Rows of the batch a rank owns under batch sharding."""
    start, stop = shard_bounds(batch, rank, world)
    return slice(start, stop)


def local_candidates(queries: torch.Tensor, weights: torch.Tensor, keys_shard: torch.Tensor,
                     k: int, offset: int) -> Candidates:
    """Dense scores of this rank's keys and their top-k (unsorted: ascending index order),
    with indices made global by `offset`."""
    idx, val = scores_topk(queries, weights, keys_shard, k, sorted=False,
                           index_dtype=torch.int32)
    if idx.dim() == 1:
        idx, val = idx.unsqueeze(0), val.unsqueeze(0)
    return val, idx + offset


def gather_candidates(values: torch.Tensor, indices: torch.Tensor,
                      group: dist.ProcessGroup | None = None) -> Candidates:
    """All-gather [B, k] candidate lists of every rank -> [B, world * k], rank-major.
    Without an initialized process group (one process) the lists are returned as they are."""
    if not (dist.is_available() and dist.is_initialized()):
        return values, indices
    world = dist.get_world_size(group)
    vs = [torch.empty_like(values) for _ in range(world)]
    js = [torch.empty_like(indices) for _ in range(world)]
    dist.all_gather(vs, values.contiguous(), group=group)
    dist.all_gather(js, indices.contiguous(), group=group)
    return torch.cat(vs, dim=1), torch.cat(js, dim=1)


@dataclass
class LShardedTopK:
    """Exact global top-k of a cache sharded along L over the ranks of `group`.

    `local_fn(queries, weights, keys_shard, k, offset)` and `merge_fn(values, indices, k,
    sorted)` default to the CUDA path (``local_candidates`` and ``merge_topk``); they are
    parameters so the exchange logic can run with other stand-ins (the CPU tests)."""

    k: int
    sorted: bool = True
    group: dist.ProcessGroup | None = None
    local_fn: Callable[..., Candidates] = local_candidates
    merge_fn: Callable[..., Candidates] | None = None

    def __call__(self, queries: torch.Tensor, weights: torch.Tensor, keys_shard: torch.Tensor,
                 offset: int) -> tuple[torch.Tensor, torch.Tensor]:
        if keys_shard.shape[-2] < self.k:
            raise ValueError(f"every shard needs at least k={self.k} keys "
                             f"(this one has {keys_shard.shape[-2]})")
        values, indices = self.local_fn(queries, weights, keys_shard, self.k, offset)
        all_v, all_i = gather_candidates(values, indices, self.group)
        if self.merge_fn is not None:
            return self.merge_fn(all_v, all_i, self.k, self.sorted)
        idx, val = merge_topk(all_v, all_i, self.k, sorted=self.sorted)
        return idx, val


class _CandidateMerge:
    """The exchange step of an L-sharded top-k on fixed buffers: the rank's local top-k
    (values f32, indices i32 already global) packed into one all-gather, reordered rank-major
    -> row-major, and merged by tdsa_merge_topk."""

    def __init__(self, batch: int, k: int, *, sorted: bool, group, device):
        self.batch, self.k, self.sorted, self.group = batch, k, bool(sorted), group
        self.world = (dist.get_world_size(group)
                      if dist.is_available() and dist.is_initialized() else 1)
        self.send = torch.empty(2, batch, k, device=device, dtype=torch.int32)
        self.recv = torch.empty(self.world, 2, batch, k, device=device, dtype=torch.int32)
        self.cand = torch.empty(2, batch, self.world, k, device=device, dtype=torch.int32)
        self.indices = torch.empty(batch, k, device=device, dtype=torch.int64)
        self.values = torch.empty(batch, k, device=device, dtype=torch.float32)

    def __call__(self, values: torch.Tensor, indices: torch.Tensor, offset: int):
        from . import _capi as capi
        from .indexer import stream_ptr

        self.send[0].copy_(values.view(torch.int32))
        torch.add(indices, offset, out=self.send[1])
        if self.world > 1:
            dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        else:
            self.recv[0].copy_(self.send)
        self.cand.copy_(self.recv.permute(1, 2, 0, 3))
        b, count = self.batch, self.world * self.k
        vals = self.cand[0].view(torch.float32).view(b, count)
        idx = self.cand[1].view(b, count)
        capi.call("tdsa_merge_topk", vals.data_ptr(), idx.data_ptr(), count, b, count, self.k,
                  int(self.sorted), self.indices.data_ptr(), 8, self.indices.stride(0),
                  self.values.data_ptr(), self.values.stride(0), stream_ptr(vals.device))
        return self.indices, self.values


class PeerExchange:
    """The exchange step of an L-sharded top-k over peer memory (NVLink) instead of an
    all-gather: one ``tdsa_exchange_topk`` launch per step writes this rank's candidates
    into its exchange region, raises its per-row flag in every rank's region, waits per row
    for every rank's flag, pulls the rows from peer memory and selects the global top-k --
    no collective library call on the data path.  The regions are shared once through CUDA
    IPC (handles all-gathered over `group`); all ranks must be on one node.  Call
    ``close()`` on every rank when done: it waits for all ranks before freeing the region
    the others read."""

    def __init__(self, batch: int, k: int, *, sorted: bool, group, device):
        import ctypes as C

        from . import _capi as capi

        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        self.batch, self.k, self.sorted, self.group = batch, k, bool(sorted), group
        self.device = torch.device(device)
        handle = (C.c_uint8 * capi.TDSA_IPC_HANDLE_BYTES)()
        ptr = C.c_void_p()
        capi.call("tdsa_exchange_create", self.world, self.rank, batch, k, C.byref(ptr),
                  handle)
        self._ex = ptr
        mine = torch.tensor(bytearray(handle), dtype=torch.uint8, device=self.device)
        if self.world > 1:
            every = torch.empty(self.world, capi.TDSA_IPC_HANDLE_BYTES, dtype=torch.uint8,
                                device=self.device)
            dist.all_gather_into_tensor(every, mine, group=group)
        else:
            every = mine.view(1, -1)
        blob = bytes(every.cpu().numpy().tobytes())
        try:
            capi.call("tdsa_exchange_connect", self._ex, blob)
        except Exception:
            capi.lib().tdsa_exchange_destroy(self._ex)
            self._ex = None
            raise
        self.indices = torch.empty(batch, k, device=self.device, dtype=torch.int64)
        self.values = torch.empty(batch, k, device=self.device, dtype=torch.float32)

    def __call__(self, values: torch.Tensor, indices: torch.Tensor, offset: int):
        from . import _capi as capi
        from .indexer import stream_ptr

        if self._ex is None:
            raise RuntimeError("exchange is closed")
        if values.dtype != torch.float32 or indices.dtype != torch.int32:
            raise ValueError("candidates must be float32 values and int32 indices")
        if values.stride() != indices.stride() or values.stride(-1) != 1:
            raise ValueError("values and indices need the same row-contiguous layout")
        capi.call("tdsa_exchange_topk", self._ex, values.data_ptr(), indices.data_ptr(),
                  values.stride(0), int(offset), int(self.sorted), self.indices.data_ptr(), 8,
                  self.indices.stride(0), self.values.data_ptr(), self.values.stride(0),
                  stream_ptr(self.device))
        return self.indices, self.values

    def close(self) -> None:
        """Free the exchange region once every rank is past its last merge."""
        from . import _capi as capi

        if self._ex is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        ex, self._ex = self._ex, None
        capi.call("tdsa_exchange_destroy", ex)


def _make_exchange(kind: str, batch: int, k: int, *, sorted: bool, group, device):
    if kind == "allgather":
        return _CandidateMerge(batch, k, sorted=sorted, group=group, device=device)
    if kind == "peer":
        return PeerExchange(batch, k, sorted=sorted, group=group, device=device)
    raise ValueError("exchange must be 'allgather' or 'peer'")


class LShardedPlan:
    """The L-sharded top-k on fixed buffers (the decode-loop form of ``LShardedTopK``).

    Per ``run()``: dense score + unsorted top-k of this rank's keys (``ScoreTopkPlan``),
    global indices, ONE all-gather of the packed (value bits, index) candidates, a
    rank-major -> row-major copy, and the merge.  The caller rewrites ``queries`` /
    ``weights`` in place between steps.  ``exchange="peer"`` replaces the all-gather, copy
    and merge by ``PeerExchange`` (peer memory, one node)."""

    def __init__(self, queries: torch.Tensor, weights: torch.Tensor, keys_shard: torch.Tensor,
                 k: int, offset: int, *, sorted: bool = True,
                 group: dist.ProcessGroup | None = None, exchange: str = "allgather"):
        from .indexer import ScoreTopkPlan

        if keys_shard.shape[-2] < k:
            raise ValueError(f"every shard needs at least k={k} keys")
        self.plan = ScoreTopkPlan(queries, weights, keys_shard, k, sorted=False,
                                  index_dtype=torch.int32)
        self.k, self.offset, self.sorted, self.group = k, int(offset), bool(sorted), group
        self.merge = _make_exchange(exchange, self.plan.batch, k, sorted=sorted, group=group,
                                    device=keys_shard.device)
        self.world = self.merge.world

    def run(self) -> tuple[torch.Tensor, torch.Tensor]:
        self.plan.run()
        return self.merge(self.plan.values, self.plan.indices, self.offset)

    def close(self) -> None:
        if hasattr(self.merge, "close"):
            self.merge.close()


class LShardedExact:
    """The exact certified progressive top-k of an L-sharded, append-only key cache.

    Each rank runs the exact progressive path (``ExactProgressiveTopK``) over its own
    contiguous key range, so its local top-k is exact: it prunes only blocks whose certified
    bound is below its local k-th score, which is at most the global k-th score.  The global
    top-k is in the union of the local ones; the candidates are all-gathered and merged as in
    ``LShardedPlan``.  New keys are appended to the last rank's range (the other ranges stay
    fixed), so every rank's cache is append-only."""

    def __init__(self, batch: int, max_shard_length: int, k: int, offset: int, *,
                 block_size: int = 64, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | None = None, sorted: bool = True,
                 group: dist.ProcessGroup | None = None, exchange: str = "allgather"):
        from .progressive_exact import ExactProgressiveTopK

        self.exact = ExactProgressiveTopK(batch, max_shard_length, k, block_size=block_size,
                                          dtype=dtype, device=device, sorted=False,
                                          index_dtype=torch.int32)
        self.k, self.offset = k, int(offset)
        self.merge = _make_exchange(exchange, batch, k, sorted=sorted, group=group,
                                    device=self.exact.device)
        self.world = self.merge.world

    def init(self, queries, weights, keys_shard):
        if keys_shard.shape[-2] < self.k:
            raise ValueError(f"every shard needs at least k={self.k} keys")
        idx, val = self.exact.init(queries, weights, keys_shard)
        return self.merge(val, idx, self.offset)

    def step(self, queries, weights, keys_shard):
        idx, val = self.exact.step(queries, weights, keys_shard)
        return self.merge(val, idx, self.offset)

    def stats(self) -> list[dict]:
        return self.exact.stats()

    def close(self) -> None:
        if hasattr(self.merge, "close"):
            self.merge.close()
