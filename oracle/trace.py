"""Numpy restatement of the reference's score-trace rows (test oracle).

Reference: ``src/temporal_dsa/training.py:146-178`` (``evaluate_and_trace``): each traced
query's float32 score row is cast to float16 (numpy's cast: round to nearest even, values
past the float16 range become +-inf) and the rows are stacked into a ``[steps, width]``
matrix, ``width`` = the longest row, padded with ``-inf``; the lengths are int32.
``src/temporal_dsa/trace.py:34-48`` (``save_trace``) then stores ``scores``, ``lengths``
and the metadata JSON in one ``.npz``.

Test infrastructure only: the device trace rows are checked against ``trace_matrix``.
"""

from __future__ import annotations

import numpy as np


def trace_matrix(rows) -> tuple[np.ndarray, np.ndarray]:
    """training.py:166-178 -- float16 rows padded with -inf, and their int32 lengths."""
    rows = [np.asarray(r, dtype=np.float32).reshape(-1) for r in rows]
    lengths = np.asarray([r.size for r in rows], dtype=np.int32)
    width = int(lengths.max()) if rows else 0
    out = np.full((len(rows), width), -np.inf, dtype=np.float16)
    with np.errstate(over="ignore"):
        for i, r in enumerate(rows):
            out[i, : r.size] = r.astype(np.float16)
    return out, lengths
