"""Score-trace wire format (CPU): dsa_b200.trace against files written by the reference.

``tests/golden/trace_ref.npz`` was written by the reference's ``save_trace``
(src/temporal_dsa/trace.py:34-48) from float16 rows padded the way its trace writer pads
them (training.py:166-178); ``trace_rows.npz`` holds the float32 rows it started from.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

import oracle
from dsa_b200.trace import ScoreTrace, load_trace, save_trace
from tests.conftest import GOLDEN, load_golden


def _rows():
    g = load_golden("trace_rows")
    rows, start = [], 0
    for n in g["lengths"]:
        rows.append(g["rows"][start:start + n])
        start += n
    return rows


def test_oracle_rows_match_reference_writer():
    want = load_golden("trace_ref")
    scores, lengths = oracle.trace_matrix(_rows())
    assert scores.dtype == np.float16 and lengths.dtype == np.int32
    np.testing.assert_array_equal(scores.view(np.uint16), want["scores"].view(np.uint16))
    np.testing.assert_array_equal(lengths, want["lengths"])


def test_load_reference_file():
    tr = load_trace(GOLDEN / "trace_ref.npz")
    assert (tr.layer, tr.workload, tr.prompt_id) == (7, "synthetic", "seed11")
    assert tr.metadata == {"query_ids": [4, 8, 11, 15], "research_sidecar": True,
                           "source": None}
    assert tr.scores.dtype == np.float16 and tr.scores.shape == (4, 16)
    assert tr.lengths.tolist() == [5, 9, 12, 16]
    row = tr.row(1)
    assert row.dtype == np.float32 and row.size == 9
    assert row[0] == np.inf and row[1] == -np.inf and row[2] == np.inf and row[3] == 65504.0
    assert row[4] == 0.0 and 0 < row[5] < 6.2e-5  # float16 subnormal
    assert np.all(tr.scores[0, 5:] == -np.inf)


def test_save_matches_reference_members(tmp_path):
    ref = load_trace(GOLDEN / "trace_ref.npz")
    out = tmp_path / "sub" / "trace.npz"
    save_trace(out, ref)
    with np.load(out, allow_pickle=False) as a, np.load(GOLDEN / "trace_ref.npz",
                                                        allow_pickle=False) as b:
        assert sorted(a.files) == sorted(b.files) == ["lengths", "metadata", "scores"]
        for name in a.files:
            assert a[name].dtype == b[name].dtype and a[name].shape == b[name].shape
            assert a[name].tobytes() == b[name].tobytes(), name
        meta = json.loads(str(a["metadata"].item()))
        assert list(meta) == sorted(meta)
    back = load_trace(out)
    np.testing.assert_array_equal(back.scores.view(np.uint16), ref.scores.view(np.uint16))
    assert back.metadata == ref.metadata and back.layer == ref.layer


@pytest.mark.parametrize("bad, msg", [
    (dict(scores=np.zeros(3, np.float16)), "scores must be"),
    (dict(lengths=np.array([1, 2], np.int32)), "one entry per step"),
    (dict(lengths=np.array([1, 2, 0], np.int32)), "outside the score matrix"),
    (dict(lengths=np.array([1, 2, 5], np.int32)), "outside the score matrix"),
])
def test_validation(bad, msg):
    args = dict(scores=np.zeros((3, 4), np.float16), lengths=np.array([1, 2, 4], np.int32),
                layer=0, workload="w", prompt_id="p", metadata={})
    args.update(bad)
    with pytest.raises(ValueError, match=msg):
        ScoreTrace(**args)
