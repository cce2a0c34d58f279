"""Helper process for test_failure_gpu: rank 1 of a two-rank exchange that never takes a
step.  It creates its exchange region, prints the region's IPC handle (hex) on one line,
keeps the region alive until a line arrives on stdin (or 120 s pass), then frees it.  It
launches no kernel."""

from __future__ import annotations

import ctypes as C
import os
import select
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from dsa_b200 import _capi as capi  # noqa: E402


def main() -> int:
    rows, k = int(sys.argv[1]), int(sys.argv[2])
    lib = capi.lib()
    handle = (C.c_uint8 * capi.TDSA_IPC_HANDLE_BYTES)()
    ex = C.c_void_p()
    capi.check(lib.tdsa_exchange_create(2, 1, rows, k, C.byref(ex), handle))
    print(bytes(handle).hex(), flush=True)
    select.select([sys.stdin], [], [], 120.0)
    capi.check(lib.tdsa_exchange_destroy(ex))
    return 0


if __name__ == "__main__":
    sys.exit(main())
