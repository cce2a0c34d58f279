"""The C-ABI library loads and exports its header; host-side argument checks (no GPU)."""

from __future__ import annotations

import ctypes as C

import pytest

from dsa_b200 import _capi as capi


@pytest.fixture(scope="module")
def lib():
    from dsa_b200.build import build

    build()
    return capi.lib()


def test_library_exports_every_declared_function(lib):
    names = capi.header_functions()
    assert "tdsa_score_dense" in names and "tdsa_topk" in names
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/tdsa.h but not exported"
        assert name in capi.SIGNATURES, f"{name} has no ctypes signature"


def test_library_carries_no_timeline_instrumentation(lib):
    # the device timeline (TDSA_TIMELINE) belongs to the measurement build
    # libtdsa_timeline.so only; the product library must not record or export it
    from dsa_b200.build import LIB, LIB_TIMELINE

    assert capi.LIB_PATH == LIB and LIB_TIMELINE != LIB
    for name in ("tdsa_timeline_proj", "tdsa_timeline_score", "tdsa_timeline_topk",
                 "tdsa_timeline_read_stream"):
        assert not hasattr(lib, name), f"{name} is exported by the product library"


def test_version_and_empty_error(lib):
    assert b"sm_100a" in lib.tdsa_version()


def test_score_dense_rejects_bad_arguments_before_launch(lib):
    rc = lib.tdsa_score_dense(None, 0, None, 0, None, 0, 128, 7, 1, 16, None, 16, None)
    assert rc == capi.TDSA_ERR_INVALID
    assert "dtype" in capi.last_error()
    rc = lib.tdsa_score_dense(None, 0, None, 0, None, 0, 128, capi.TDSA_BF16, 0, 16, None, 16,
                              None)
    assert rc == capi.TDSA_ERR_INVALID
    rc = lib.tdsa_score_dense(16, 0, 16, 0, 16, 0, 64, capi.TDSA_BF16, 1, 16, 16, 16, None)
    assert rc == capi.TDSA_ERR_INVALID and "row stride" in capi.last_error()
    # misaligned 16-bit key pointer
    rc = lib.tdsa_score_dense(16, 8192, 16, 64, 18, 0, 128, capi.TDSA_BF16, 1, 16, 16, 16, None)
    assert rc == capi.TDSA_ERR_ALIGN
    # zero length is a no-op
    rc = lib.tdsa_score_dense(None, 0, None, 0, None, 0, 128, capi.TDSA_BF16, 1, 0, None, 0, None)
    assert rc == capi.TDSA_OK


def test_topk_rejects_bad_arguments_before_launch(lib):
    out = C.c_void_p(16)
    rc = lib.tdsa_topk(16, 100, 1, 100, 101, 1, out, 8, 101, None, 0, None, 0, None)
    assert rc == capi.TDSA_ERR_INVALID
    rc = lib.tdsa_topk(16, 100, 1, 100, 0, 1, out, 8, 1, None, 0, None, 0, None)
    assert rc == capi.TDSA_ERR_INVALID
    rc = lib.tdsa_topk(16, 100, 1, 100, 10, 1, out, 3, 10, None, 0, None, 0, None)
    assert rc == capi.TDSA_ERR_INVALID
    rc = lib.tdsa_topk(16, 40000, 1, 40000, 9000, 0, out, 4, 9000, None, 0, None, 0, None)
    assert rc == capi.TDSA_ERR_UNSUPPORTED
    # multi-level rows need workspace
    rc = lib.tdsa_topk(16, 100000, 1, 100000, 2048, 1, out, 4, 2048, None, 0, None, 0, None)
    assert rc == capi.TDSA_ERR_WORKSPACE
    rc = lib.tdsa_merge_topk(16, 16, 40000, 1, 40000, 10, 1, out, 4, 10, None, 0, None)
    assert rc == capi.TDSA_ERR_UNSUPPORTED


def test_workspace_queries(lib):
    # one row per CTA when rows alone fill the GPU; short rows of a small batch split
    assert lib.tdsa_topk_workspace_bytes(256, 32768, 2048) == 0
    assert lib.tdsa_topk_workspace_bytes(4, 32768, 2048) > 0
    ws = lib.tdsa_topk_workspace_bytes(8, 131072, 2048)
    assert ws >= 2 * 8 * 4 * 2048 * 8
    assert lib.tdsa_score_topk_workspace_bytes(2, 1000, 10) >= 2 * 1000 * 4
    assert lib.tdsa_topk_workspace_bytes(1, 10, 11) == 0


def test_drop_in_module_rejects_cpu_tensors():
    import torch

    from dsa_b200.progressive_kernel import full_scores_triton

    q = torch.zeros(64, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        full_scores_triton(q, torch.zeros(64), torch.zeros(10, 128, dtype=torch.bfloat16))
