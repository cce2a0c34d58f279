"""ctypes binding of libtdsa.so (declared in include/tdsa.h).

The library is the product: there is no Python or CPU implementation behind these calls.
If the library is missing, every call raises RuntimeError.
"""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtdsa.so"
HEADER = Path(__file__).resolve().parent.parent / "include" / "tdsa.h"

TDSA_OK = 0
TDSA_ERR_INVALID = 1
TDSA_ERR_UNSUPPORTED = 2
TDSA_ERR_CUDA = 3
TDSA_ERR_TIMEOUT = 4
TDSA_ERR_ALIGN = 5
TDSA_ERR_WORKSPACE = 6
TDSA_STATUS_RANGE = 8  # device status bit: a device-side index was out of range
TDSA_STATUS_HIST = 16  # device status bit: a key histogram did not describe its row

TDSA_F32 = 0
TDSA_F16 = 1
TDSA_BF16 = 2

i32, i64, vp, sz = C.c_int, C.c_int64, C.c_void_p, C.c_size_t
TDSA_IPC_HANDLE_BYTES = 64


class TdsaPolicy(C.Structure):
    """struct tdsa_policy (include/tdsa.h)."""
    _fields_ = [("gamma", C.c_double), ("ema_alpha", C.c_double),
                ("volatility_lambda", C.c_double), ("age_slope", C.c_double),
                ("cold_streak", i32), ("dynamic_threshold", i32), ("order", i32),
                ("buckets", i32), ("age_cap", i32), ("recent_window", i32), ("risk_model", i32)]


class TdsaRescue(C.Structure):
    """struct tdsa_rescue (include/tdsa.h)."""
    _fields_ = [("rescue_fraction", C.c_double), ("promotion_threshold", C.c_double),
                ("use_threshold", i32)]


TDSA_ORDER_ADDRESS, TDSA_ORDER_PREVIOUS_MAX = 0, 1
TDSA_ORDER_BUCKET, TDSA_ORDER_ORACLE_CURRENT = 2, 3
TDSA_RISK_LAST_MAX, TDSA_RISK_EMA = 0, 1
POLICY_STATS = ["ERROR", "TAU_SEED", "TAU_FINAL", "SCORED", "UNION", "REFRESHED", "SKIPPED",
                "RESCUED", "COLD_BLOCKS", "SEED_BLOCKS", "PHYS16", "PHYS32", "PHYS64", "PHYS128",
                "TOP128", "TOP256", "TOP512", "TOP1024", "TOP2048", "MISSED", "WORST_MISSED",
                "NEWLY_HOT", "NEWLY_HOT_MISSED", "MASS_NUM", "MASS_DEN", "BLOCKS"]
TDSA_POLICY_NSTATS = len(POLICY_STATS)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "tdsa_version": (C.c_char_p, []),
    "tdsa_last_error": (C.c_char_p, []),
    "tdsa_device_status": (i32, [C.POINTER(C.c_int), i32]),
    "tdsa_score_dense": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, vp, i64, vp]),
    "tdsa_topk_workspace_bytes": (sz, [i32, i32, i32]),
    "tdsa_topk": (i32, [vp, i64, i32, i32, i32, i32, vp, i32, i64, vp, i64, vp, sz, vp]),
    "tdsa_merge_topk": (i32, [vp, vp, i64, i32, i32, i32, i32, vp, i32, i64, vp, i64, vp]),
    "tdsa_exchange_bytes": (sz, [i32, i32, i32]),
    "tdsa_exchange_create": (i32, [i32, i32, i32, i32, C.POINTER(vp), vp]),
    "tdsa_exchange_connect": (i32, [vp, vp]),
    "tdsa_exchange_topk": (i32, [vp, vp, vp, i64, i32, i32, vp, i32, i64, vp, i64, vp]),
    "tdsa_exchange_destroy": (i32, [vp]),
    "tdsa_score_topk_workspace_bytes": (sz, [i32, i32, i32]),
    "tdsa_score_topk": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, i32, vp, i32,
                              i64, vp, i64, vp, sz, vp]),
    "tdsa_score_topk_noalloc": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, i32,
                                      vp, i32, i64, vp, i64, vp]),
    "tdsa_query_project": (i32, [vp, i64, i32, vp, i64, i32, vp, vp, vp, i64, vp, i64, i32, i32,
                                 i32, C.c_float, C.c_float, vp, i64, vp]),
    "tdsa_packed_query_weights_bytes": (sz, [i32]),
    "tdsa_selftest_bounded_wait": (i32, [C.c_longlong, vp]),
    "tdsa_hadamard128": (i32, [vp, i64, i64, i32, vp, i64, vp]),
    "tdsa_select_quantize": (i32, [vp, i64, i64, i32, i32, vp, i32, C.c_double, vp, vp, i64,
                                   vp]),
    "tdsa_pack_query_weights": (i32, [vp, i64, i32, vp, vp]),
    "tdsa_score_dense_hist": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, vp, i64, vp,
                                    vp]),
    "tdsa_topk_hist": (i32, [vp, i64, i32, i32, i32, i32, vp, i32, i64, vp, i64, vp, vp]),
    "tdsa_key_hist_bytes": (sz, [i32, i32]),
    "tdsa_topk_levels": (i32, [i32, i32, i32, i32]),
    "tdsa_topk_hist_ws": (i32, [vp, i64, i32, i32, i32, i32, vp, i32, i64, vp, i64, vp, vp, sz,
                                vp]),
    "tdsa_key_append": (i32, [vp, i64, i32, vp, i64, vp, vp, C.c_float, vp, vp, vp, i64, i64,
                              i64, i32, i32, i32, C.c_float, vp]),
    "tdsa_policy_state_bytes": (sz, [i32, i32, i32]),
    "tdsa_policy_state_offsets": (i32, [i32, i32, i32, C.POINTER(C.c_int64)]),
    "tdsa_policy_workspace_bytes": (sz, [i32, i32, i32, i32]),
    "tdsa_policy_init": (i32, [vp, sz, vp, i64, i32, i32, i32, i32, i32, vp, sz, vp]),
    "tdsa_policy_step": (i32, [vp, sz, vp, i64, vp, i64, i32, i32, i32, i32, i32, i32,
                               C.POINTER(TdsaPolicy), i32, i32, C.POINTER(TdsaRescue), vp, sz,
                               vp, i64, vp, vp, vp, vp]),
    "tdsa_score_dense_trace": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, vp, i64, vp,
                                     vp, i64, vp]),
    "tdsa_h8_block_max": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, vp, vp, vp,
                                i64, vp, i64, vp]),
    "tdsa_masked_dense": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, vp, i64, vp,
                                i64, vp]),
    "tdsa_two_pass": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, vp, vp, vp, vp,
                            i64, vp, vp, i64, vp]),
    "tdsa_progressive_h8": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, vp, vp, vp,
                                  vp, vp, i64, vp, vp, i64, vp]),
    "tdsa_compact_blocks": (i32, [vp, i64, vp, i64, i32, i32, i32, vp, vp, i64, vp, vp]),
    "tdsa_sketch_keys": (i32, [vp, i64, i64, i32, i32, i32, i32, vp, i64, vp, vp, i64, vp]),
    "tdsa_sketch_topk_workspace_bytes": (sz, [i32, i32, i32]),
    "tdsa_sketch_workspace_offsets": (i32, [i32, i32, i32, C.POINTER(C.c_int64)]),
    "tdsa_sketch_topk": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, vp, i64, vp, vp, i64, i32,
                               i32, i32, i32, i32, vp, i32, i64, vp, i64, vp, vp, sz, vp]),
    "tdsa_exact_state_bytes": (sz, [i32, i32, i32, i32]),
    "tdsa_exact_init": (i32, [vp, sz, vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, i32, i32,
                              i32, vp, i32, i64, vp, i64, vp]),
    "tdsa_exact_step": (i32, [vp, sz, vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, i32, i32,
                              i32, i32, vp, i32, i64, vp, i64, vp]),
    "tdsa_exact_stats": (i32, [vp, sz, i32, i32, i32, i32, C.POINTER(C.c_uint64)]),
    "tdsa_block_key_norms": (i32, [vp, i32, i32, i32, i32, vp, vp]),
    "tdsa_temporal_radius": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp]),
    "tdsa_relu_index_score": (i32, [vp, vp, vp, i32, i32, i32, vp, vp]),
    "tdsa_query_prep": (i32, [vp, i64, vp, i64, i32, vp, vp, vp, i64, vp, i64, i32, i32, i32,
                              C.c_float, C.c_float, vp]),
}

_lib: C.CDLL | None = None


class TdsaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"tdsa error {code}: {message}")
        self.code = code


def header_functions() -> list[str]:
    """Names of the functions include/tdsa.h declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(tdsa_\w+)\s*\(", text, re.M)))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is not built: run `python -m dsa_b200.build` (nvcc, sm_100a)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().tdsa_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    if rc == TDSA_OK:
        return
    msg = last_error()
    if rc in (TDSA_ERR_INVALID, TDSA_ERR_ALIGN, TDSA_ERR_WORKSPACE):
        raise ValueError(msg)
    raise TdsaError(rc, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def device_status(reset: bool = True) -> int:
    out = C.c_int(0)
    check(lib().tdsa_device_status(C.byref(out), 1 if reset else 0))
    return out.value
