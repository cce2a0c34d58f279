"""pytest plugin that binds the reference's module names to this library's drop-ins.

Loaded with ``-p tests._reference_binding`` in a child pytest run over the reference's own
test file (``baseline/_ref/reference_tests/test_progressive_kernel.py``, the reference's
tests/test_progressive_kernel.py placed beside its offline install): before that file does
``from temporal_dsa.progressive_kernel import ...``, the name is bound to
``dsa_b200.progressive_kernel``, the import switch a maintainer makes at the reference's call
sites.  The reference package itself comes from its install under ``baseline/_ref``.
"""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
for path in (str(ROOT), str(REF)):
    if path not in sys.path:
        sys.path.insert(0, path)

import temporal_dsa  # noqa: E402  (the installed reference package)

from dsa_b200 import progressive_kernel as _pk  # noqa: E402

sys.modules["temporal_dsa.progressive_kernel"] = _pk
temporal_dsa.progressive_kernel = _pk
