"""Device-tensor API of the indexer path (B200, sm_100a) on top of the C ABI.

Shapes follow the reference project temporal_dsa: H = 64 heads, D = 128 dims,
``score[s] = sum_h w[h] * ReLU(q[h] . k[s])``.  Inputs must be CUDA tensors; kernels run
on the current torch stream.  Nothing here computes on the CPU.
"""

from __future__ import annotations

import torch

from . import _capi as capi

HEADS = 64
HEAD_DIM = 128

_DTYPES = {torch.float32: capi.TDSA_F32, torch.float16: capi.TDSA_F16,
           torch.bfloat16: capi.TDSA_BF16}


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("the B200 indexer kernels require CUDA tensors")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """The cudaStream_t of torch's current stream on `device` (the raw-handle accessor
    torch's own generated code uses; it costs a tenth of building a Stream object)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None
                           else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _aligned(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def prepare_queries(q: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """[B,64,128] with contiguous rows, 16-byte aligned (small: copied if needed)."""
    if q.dtype != dtype:
        raise ValueError("queries and keys must share a dtype")
    q = q.contiguous()
    if not _aligned(q):
        q = q.clone()
    return q


def prepare_weights(w: torch.Tensor) -> torch.Tensor:
    w = w.to(torch.float32).contiguous()
    if not _aligned(w):
        w = w.clone()
    return w


def prepare_keys(keys: torch.Tensor) -> torch.Tensor:
    """[B,L,128]: unit stride on dims; TMA wants 16-byte aligned base and row/batch strides."""
    if keys.dtype not in _DTYPES:
        raise ValueError("keys must be float32, float16 or bfloat16")
    ok = keys.stride(-1) == 1
    if ok and keys.dtype != torch.float32:
        ok = _aligned(keys) and keys.stride(-2) % 8 == 0 and (
            keys.shape[0] == 1 or keys.stride(0) % 8 == 0)
    if not ok:
        keys = keys.contiguous()
        if keys.dtype != torch.float32 and not _aligned(keys):
            keys = keys.clone()
    return keys


def as_batched(q: torch.Tensor, w: torch.Tensor, keys: torch.Tensor):
    """Accepts the single-sequence ([64,128], [64], [L,128]) or batched layout."""
    single = keys.dim() == 2
    if single:
        if q.shape != (HEADS, HEAD_DIM) or w.shape != (HEADS,):
            raise ValueError("expected queries [64,128] and weights [64]")
        if keys.shape[1] != HEAD_DIM:
            raise ValueError("expected keys [L,128]")
        return q.unsqueeze(0), w.unsqueeze(0), keys.unsqueeze(0), True
    if keys.dim() != 3 or keys.shape[2] != HEAD_DIM:
        raise ValueError("expected keys [B,L,128]")
    b = keys.shape[0]
    if q.shape != (b, HEADS, HEAD_DIM) or w.shape != (b, HEADS):
        raise ValueError("expected queries [B,64,128] and weights [B,64]")
    return q, w, keys, False


def score_dense(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense indexer scores: [64,128],[64],[L,128] -> [L] or batched -> [B,L] (float32)."""
    require_cuda(queries, weights, keys)
    q, w, k, single = as_batched(queries, weights, keys)
    k = prepare_keys(k)
    q = prepare_queries(q, k.dtype)
    w = prepare_weights(w)
    bsz, length = k.shape[0], k.shape[1]
    if out is None:
        out = torch.empty(bsz, length, device=k.device, dtype=torch.float32)
    elif single:
        out = out.view(1, -1)
    if out.dtype != torch.float32 or out.shape != (bsz, length) or out.stride(-1) != 1:
        raise ValueError("out must be float32 [B,L] with unit last stride")
    if length:
        capi.call("tdsa_score_dense", q.data_ptr(), q.stride(0), w.data_ptr(), w.stride(0),
                  k.data_ptr(), k.stride(0), k.stride(1), _DTYPES[k.dtype], bsz, length,
                  out.data_ptr(), out.stride(0), stream_ptr(k.device))
    return out[0] if single else out


_WORKSPACE_BYTES: dict[tuple[int, int, int, int], int] = {}
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def topk_workspace(device: torch.device, batch: int, length: int,
                   k: int) -> tuple[torch.Tensor, int]:
    """Scratch of the size ``tdsa_topk`` asks for -> (buffer, bytes).  Outside CUDA-graph
    capture one buffer per (device, stream) is kept and reused: calls on one stream run in
    order, so they can share it, and the next call needs no allocation (it only grows).
    During a capture a fresh buffer is returned, which the graph keeps."""
    key = (device.index, batch, length, k)
    nbytes = _WORKSPACE_BYTES.get(key)
    if nbytes is None:
        with torch.cuda.device(device):  # the size depends on the device (cluster occupancy)
            nbytes = capi.lib().tdsa_topk_workspace_bytes(batch, length, k)
        _WORKSPACE_BYTES[key] = nbytes
    if torch.cuda.is_current_stream_capturing():
        return torch.empty(max(nbytes, 1), device=device, dtype=torch.uint8), nbytes
    skey = (device.index, stream_ptr(device))
    ws = _WORKSPACES.get(skey)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1), device=device, dtype=torch.uint8)
        _WORKSPACES[skey] = ws
    return ws, nbytes


def topk(scores: torch.Tensor, k: int, *, sorted: bool = True,
         index_dtype: torch.dtype = torch.int64) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact row-wise top-k with the reference's tie rule -> (indices, values).

    sorted=True: descending score, equal scores by ascending index (stable_topk order);
    sorted=False: the same set in ascending index order.
    """
    require_cuda(scores)
    if scores.dtype != torch.float32:
        raise ValueError("scores must be float32")
    nd = scores.dim()
    if nd not in (1, 2):
        raise ValueError("scores must be [L] or [B,L]")
    s = scores if scores.stride(-1) == 1 else scores.contiguous()
    if nd == 1:
        bsz, length, s_stride = 1, s.shape[0], s.shape[0]
    else:
        (bsz, length), s_stride = s.shape, s.stride(0)
    if not 0 < k <= length:
        raise ValueError(f"k={k} is invalid for {length} values")
    if index_dtype not in (torch.int32, torch.int64):
        raise ValueError("index_dtype must be int32 or int64")
    dev = s.device
    shape = (k,) if nd == 1 else (bsz, k)
    idx = torch.empty(shape, device=dev, dtype=index_dtype)
    val = torch.empty(shape, device=dev, dtype=torch.float32)
    ws, nbytes = topk_workspace(dev, bsz, length, k)
    capi.call("tdsa_topk", s.data_ptr(), s_stride, bsz, length, k, int(bool(sorted)),
              idx.data_ptr(), idx.element_size(), k, val.data_ptr(), k, ws.data_ptr(), nbytes,
              stream_ptr(dev))
    return idx, val


def merge_topk(cand_values: torch.Tensor, cand_indices: torch.Tensor, k: int, *,
               sorted: bool = True, index_dtype: torch.dtype = torch.int64):
    """Top-k of per-shard candidates (rows in ascending index order) -> (indices, values)."""
    require_cuda(cand_values, cand_indices)
    v = cand_values.to(torch.float32).contiguous()
    i = cand_indices.to(torch.int32).contiguous()
    single = v.dim() == 1
    if single:
        v, i = v.unsqueeze(0), i.unsqueeze(0)
    bsz, count = v.shape
    if not 0 < k <= count:
        raise ValueError(f"k={k} is invalid for {count} candidates")
    idx = torch.empty(bsz, k, device=v.device, dtype=index_dtype)
    val = torch.empty(bsz, k, device=v.device, dtype=torch.float32)
    capi.call("tdsa_merge_topk", v.data_ptr(), i.data_ptr(), v.stride(0), bsz, count, k,
              int(bool(sorted)), idx.data_ptr(), idx.element_size(), idx.stride(0),
              val.data_ptr(), val.stride(0), stream_ptr(v.device))
    return (idx[0], val[0]) if single else (idx, val)


def scores_topk(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor, k: int, *,
                sorted: bool = True, index_dtype: torch.dtype = torch.int32,
                workspace: torch.Tensor | None = None):
    """Fused dense score + top-k per sequence -> (indices [B,k], scores [B,k])."""
    require_cuda(queries, weights, keys)
    q, w, kk, single = as_batched(queries, weights, keys)
    kk = prepare_keys(kk)
    q = prepare_queries(q, kk.dtype)
    w = prepare_weights(w)
    bsz, length = kk.shape[0], kk.shape[1]
    if not 0 < k <= length:
        raise ValueError(f"k={k} is invalid for {length} keys")
    idx = torch.empty(bsz, k, device=kk.device, dtype=index_dtype)
    val = torch.empty(bsz, k, device=kk.device, dtype=torch.float32)
    nbytes = capi.lib().tdsa_score_topk_workspace_bytes(bsz, length, k)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, device=kk.device, dtype=torch.uint8)
    capi.call("tdsa_score_topk", q.data_ptr(), q.stride(0), w.data_ptr(), w.stride(0),
              kk.data_ptr(), kk.stride(0), kk.stride(1), _DTYPES[kk.dtype], bsz, length, k,
              int(bool(sorted)), idx.data_ptr(), idx.element_size(), idx.stride(0),
              val.data_ptr(), val.stride(0), workspace.data_ptr(), nbytes,
              stream_ptr(kk.device))
    return (idx[0], val[0]) if single else (idx, val)


class ScoreTopkPlan:
    """A prepared dense-score + top-k call on fixed device buffers (the decode loop form).

    The caller rewrites ``queries``/``weights`` in place between steps; ``score()`` and
    ``select()`` are one C-ABI call each with no per-call validation or allocation.
    Results land in ``scores`` [B,L], ``indices`` [B,k] and ``values`` [B,k].  With a
    ``trace`` (``dsa_b200.trace.TraceRecorder``) every ``score()`` also writes the next
    float16 trace row from the score kernel (16-bit keys).
    """

    def __init__(self, queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor, k: int,
                 *, sorted: bool = False, index_dtype: torch.dtype = torch.int32,
                 trace=None):
        require_cuda(queries, weights, keys)
        q, w, kk, _ = as_batched(queries, weights, keys)
        if not (q.is_contiguous() and _aligned(q) and q.dtype == kk.dtype):
            raise ValueError("plan queries must be contiguous, 16-byte aligned, keys' dtype")
        if not (w.dtype == torch.float32 and w.is_contiguous()):
            raise ValueError("plan weights must be contiguous float32")
        if prepare_keys(kk) is not kk:
            raise ValueError("plan keys must already satisfy the TMA layout rules")
        self.q, self.w, self.keys = q, w, kk
        self.batch, self.length, self.k = kk.shape[0], kk.shape[1], k
        if not 0 < k <= self.length:
            raise ValueError(f"k={k} is invalid for {self.length} keys")
        dev = kk.device
        # score rows padded to 16 bytes, so the top-k copies every row with bulk copies
        padded = (self.length + 3) // 4 * 4
        self.scores = torch.empty(self.batch, padded, device=dev,
                                  dtype=torch.float32)[:, :self.length]
        self.indices = torch.empty(self.batch, k, device=dev, dtype=index_dtype)
        self.values = torch.empty(self.batch, k, device=dev, dtype=torch.float32)
        lib = capi.lib()
        # 16-bit keys: the score kernel also histograms the keys (one histogram per 32768-key
        # segment) and the top-k starts from those histograms (which it leaves zeroed again)
        self.use_hist = kk.dtype != torch.float32
        nbytes = lib.tdsa_topk_workspace_bytes(self.batch, self.length, k)
        self.workspace = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
        if self.use_hist:
            hbytes = lib.tdsa_key_hist_bytes(self.batch, self.length)
            self.key_hist = torch.zeros(hbytes // 4, device=dev, dtype=torch.int32)
            self._score_fn, self._topk_fn = lib.tdsa_score_dense_hist, lib.tdsa_topk_hist_ws
            self._score_args = (q.data_ptr(), q.stride(0), w.data_ptr(), w.stride(0),
                                kk.data_ptr(), kk.stride(0), kk.stride(1), _DTYPES[kk.dtype],
                                self.batch, self.length, self.scores.data_ptr(),
                                self.scores.stride(0), self.key_hist.data_ptr())
            self._topk_args = (self.scores.data_ptr(), self.scores.stride(0), self.batch,
                               self.length, k, int(bool(sorted)), self.indices.data_ptr(),
                               self.indices.element_size(), self.indices.stride(0),
                               self.values.data_ptr(), self.values.stride(0),
                               self.key_hist.data_ptr(), self.workspace.data_ptr(), nbytes)
        else:
            self._score_fn, self._topk_fn = lib.tdsa_score_dense, lib.tdsa_topk
            self._score_args = (q.data_ptr(), q.stride(0), w.data_ptr(), w.stride(0),
                                kk.data_ptr(), kk.stride(0), kk.stride(1), _DTYPES[kk.dtype],
                                self.batch, self.length, self.scores.data_ptr(),
                                self.scores.stride(0))
            self._topk_args = (self.scores.data_ptr(), self.scores.stride(0), self.batch,
                               self.length, k, int(bool(sorted)), self.indices.data_ptr(),
                               self.indices.element_size(), self.indices.stride(0),
                               self.values.data_ptr(), self.values.stride(0),
                               self.workspace.data_ptr(), nbytes)
        self.device = dev
        # kernels per run(): score + top-k (one level, or more when the row splits)
        self.launches_per_run = 1 + capi.lib().tdsa_topk_levels(
            self.batch, self.length, k, int(self.use_hist) | (int(bool(sorted)) << 1))
        self.trace = trace
        if trace is not None:
            if kk.dtype == torch.float32:
                raise ValueError("score traces need bfloat16 or float16 keys")
            if trace.batch != self.batch or trace.max_length < self.length:
                raise ValueError("the trace recorder does not fit this plan's batch and length")
            if trace.buffer.device != dev:
                raise ValueError("the trace recorder's buffer is on another device")
            self._trace_args = self._score_args[:12] + (
                self.key_hist.data_ptr() if self.use_hist else None,)

    def score(self) -> None:
        if self.trace is not None:
            row, row_bs = self.trace.take_row(self.length)
            rc = capi.lib().tdsa_score_dense_trace(*self._trace_args, row, row_bs,
                                                   stream_ptr(self.device))
            if rc != capi.TDSA_OK:  # the row was not written: give it back
                self.trace.step -= 1
                self.trace.lengths[self.trace.step] = 0
            capi.check(rc)
            return
        capi.check(self._score_fn(*self._score_args, stream_ptr(self.device)))

    def select(self) -> None:
        capi.check(self._topk_fn(*self._topk_args, stream_ptr(self.device)))

    def run(self) -> tuple[torch.Tensor, torch.Tensor]:
        self.score()
        self.select()
        return self.indices, self.values


def device_status(reset: bool = True) -> int:
    """OR of error bits raised by kernels on the current device since the last reset."""
    return capi.device_status(reset)
