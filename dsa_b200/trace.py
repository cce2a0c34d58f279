"""Score traces: the reference's wire format, with rows written by the score kernel.

``ScoreTrace``, ``save_trace`` and ``load_trace`` keep the format of
``temporal_dsa.trace`` (src/temporal_dsa/trace.py:11-61), so ``temporal-dsa analyze`` and
the replay/verifier tools read these files unchanged:

* ``scores`` float16 ``[steps, width]``; row t holds keys ``[0, lengths[t])`` and ``-inf``
  beyond (the padding of training.py:176-178);
* ``lengths`` int32 ``[steps]``;
* ``metadata`` a 0-d string array holding the JSON (``sort_keys=True``) of the metadata
  dict merged with ``layer``, ``workload`` and ``prompt_id``; one ``np.savez_compressed``.

New here: ``TraceRecorder`` holds ``[batch, steps, max_length]`` float16 trace rows on the
device.  Each decode step's score kernel stores its scores rounded to float16 straight into
the step's row (``tdsa_score_dense_trace``), the rounding numpy's cast does in the
reference's writer (training.py:168).  Nothing crosses to the host until ``traces()``.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Sequence

import numpy as np
import torch

from . import _capi as capi
from .indexer import _DTYPES, as_batched, prepare_keys, prepare_queries, prepare_weights
from .indexer import require_cuda, stream_ptr


@dataclass(frozen=True)
class ScoreTrace:
    """One layer/prompt trace; row t holds the scores of keys [0, lengths[t])."""

    scores: np.ndarray
    lengths: np.ndarray
    layer: int
    workload: str
    prompt_id: str
    metadata: dict[str, Any]

    def __post_init__(self) -> None:
        if self.scores.ndim != 2:
            raise ValueError(f"scores must be [steps,max_length], got {self.scores.shape}")
        if self.lengths.shape != (self.scores.shape[0],):
            raise ValueError("lengths must have one entry per step")
        if np.any(self.lengths <= 0) or np.any(self.lengths > self.scores.shape[1]):
            raise ValueError("lengths are outside the score matrix")

    def row(self, step: int) -> np.ndarray:
        return np.asarray(self.scores[step, : self.lengths[step]], dtype=np.float32)


def save_trace(path: str | Path, trace: ScoreTrace) -> None:
    """trace.py:34-48: one compressed .npz of scores, lengths and the metadata JSON."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    meta = dict(trace.metadata)
    meta.update(layer=trace.layer, workload=trace.workload, prompt_id=trace.prompt_id)
    np.savez_compressed(path, scores=trace.scores, lengths=trace.lengths,
                        metadata=np.asarray(json.dumps(meta, sort_keys=True)))


def load_trace(path: str | Path) -> ScoreTrace:
    """trace.py:51-61: the inverse of save_trace (no pickles)."""
    with np.load(Path(path), allow_pickle=False) as data:
        meta = json.loads(str(data["metadata"].item()))
        layer, workload = int(meta.pop("layer")), str(meta.pop("workload"))
        prompt_id = str(meta.pop("prompt_id"))
        return ScoreTrace(scores=data["scores"], lengths=data["lengths"], layer=layer,
                          workload=workload, prompt_id=prompt_id, metadata=meta)


class TraceRecorder:
    """Device-resident trace rows of `batch` sequences over up to `steps` decode steps.

    ``buffer`` [batch, steps, max_length] float16 starts at -inf; ``take_row(length)``
    reserves the next step's row, and the score kernel writes keys [0, length) of it."""

    def __init__(self, batch: int, steps: int, max_length: int, device: torch.device | str):
        if batch < 1 or steps < 1 or max_length < 1:
            raise ValueError("batch, steps and max_length must be >= 1")
        self.batch, self.steps, self.max_length = int(batch), int(steps), int(max_length)
        self.buffer = torch.full((self.batch, self.steps, self.max_length), float("-inf"),
                                 device=device, dtype=torch.float16)
        self.lengths = np.zeros(self.steps, dtype=np.int32)
        self.step = 0

    def take_row(self, length: int) -> tuple[int, int]:
        """Reserve the next step's row for `length` keys -> (device address of row
        [0, step, 0], batch stride in elements)."""
        if self.step >= self.steps:
            raise ValueError(f"the recorder holds {self.steps} steps; all are taken")
        if not 0 < length <= self.max_length:
            raise ValueError(f"length {length} is outside [1, {self.max_length}]")
        row = self.buffer[:, self.step]
        self.lengths[self.step] = length
        self.step += 1
        return row.data_ptr(), self.buffer.stride(0)

    def reset(self) -> None:
        self.buffer.fill_(float("-inf"))
        self.lengths[:] = 0
        self.step = 0

    def traces(self, *, layer: int, workload: str, prompt_ids: Sequence[str],
               metadata: dict[str, Any] | Sequence[dict[str, Any]] | None = None
               ) -> list[ScoreTrace]:
        """One ScoreTrace per sequence over the recorded steps (one device->host copy),
        `width` = the longest recorded row, as the reference's writer pads."""
        if len(prompt_ids) != self.batch:
            raise ValueError("one prompt id per sequence")
        if self.step == 0:
            raise ValueError("no step has been recorded")
        lengths = self.lengths[: self.step].copy()
        width = int(lengths.max())
        host = self.buffer[:, : self.step, :width].cpu().numpy()
        metas = (list(metadata) if isinstance(metadata, (list, tuple))
                 else [dict(metadata or {}) for _ in range(self.batch)])
        if len(metas) != self.batch:
            raise ValueError("one metadata dict per sequence")
        return [ScoreTrace(scores=np.ascontiguousarray(host[b]), lengths=lengths.copy(),
                           layer=int(layer), workload=str(workload),
                           prompt_id=str(prompt_ids[b]), metadata=dict(metas[b]))
                for b in range(self.batch)]


def score_trace(queries: torch.Tensor, weights: torch.Tensor, keys: torch.Tensor,
                recorder: TraceRecorder, out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense scores (as ``indexer.score_dense``) that also fill the recorder's next row.

    Keys must be bfloat16 or float16 (the tensor-core score kernel emits the row)."""
    require_cuda(queries, weights, keys)
    q, w, k, single = as_batched(queries, weights, keys)
    k = prepare_keys(k)
    if k.dtype == torch.float32:
        raise ValueError("score traces need bfloat16 or float16 keys")
    q = prepare_queries(q, k.dtype)
    w = prepare_weights(w)
    bsz, length = k.shape[0], k.shape[1]
    if bsz != recorder.batch:
        raise ValueError(f"the recorder holds {recorder.batch} sequences, keys have {bsz}")
    if recorder.buffer.device != k.device:
        raise ValueError("the recorder's buffer is on another device")
    if out is None:
        out = torch.empty(bsz, length, device=k.device, dtype=torch.float32)
    elif single:
        out = out.view(1, -1)
    if out.dtype != torch.float32 or out.shape != (bsz, length) or out.stride(-1) != 1:
        raise ValueError("out must be float32 [B,L] with unit last stride")
    row, row_bs = recorder.take_row(length)
    try:
        capi.call("tdsa_score_dense_trace", q.data_ptr(), q.stride(0), w.data_ptr(),
                  w.stride(0), k.data_ptr(), k.stride(0), k.stride(1), _DTYPES[k.dtype], bsz,
                  length, out.data_ptr(), out.stride(0), None, row, row_bs,
                  stream_ptr(k.device))
    except Exception:
        recorder.step -= 1
        recorder.lengths[recorder.step] = 0
        raise
    return out[0] if single else out
