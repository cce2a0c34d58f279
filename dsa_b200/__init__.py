"""B200-native (sm_100a) Lightning-Indexer decode path with the temporal_dsa API.

Product code only: hand-written CUDA kernels in ``csrc/`` behind the C ABI of
``include/tdsa.h`` (built into ``_lib/libtdsa.so``), and the Python mirror of the
reference project's interface for this path (``progressive_kernel``, ``sidecar``,
``metrics``, ``certified``, ``verifier_scoring``) and the multi-GPU layouts
(``parallel``).  There is no CPU implementation.
"""

from .indexer import (  # noqa: F401
    HEAD_DIM,
    HEADS,
    device_status,
    merge_topk,
    score_dense,
    scores_topk,
    topk,
)

__version__ = "0.1.0"
