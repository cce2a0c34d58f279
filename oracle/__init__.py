"""CPU oracle for the Lightning-Indexer decode path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithms of the reference project
``temporal_dsa`` (psa1582/dsa) for the indexer hot path: dense scoring,
stable top-K, the H8 progressive probe, the certified temporal bound, the
block-replay filter and the score-trace rows.  Every function cites the reference file:line it follows
(paths are relative to the reference project's root).

It exists to CHECK the CUDA path, never to stand in for it.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` leg
of ``bench.py`` may import it.  The product package ``dsa_b200`` never imports
anything from here and has no CPU fallback.

Pinning: the restatement is checked against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference and
writes ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` compares).
"""

from .indexer import (  # noqa: F401
    HEADS,
    HEAD_DIM,
    VERIFIER_HEADS,
    dynamic_head_ids,
    full_scores,
    h8_block_max,
    masked_full_scores,
    progressive_qk_reduction,
    progressive_scores,
    progressive_scores_fused,
    relu_index_score,
    score_encoded,
    score_head_sparse,
    split_head_ids,
    two_pass_scores,
)
from .topk import stable_topk, topk_rows, merge_topk  # noqa: F401
from .certified import block_key_norms, temporal_score_radius  # noqa: F401
from .trace import trace_matrix  # noqa: F401
