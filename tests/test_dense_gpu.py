"""GPU parity: dense scoring and top-k through the C ABI against the oracle and goldens.

Tolerances: BF16/FP16 scores within 1e-2 relative, FP32 within 1e-5
relative.  Both are applied norm-wise -- relative to sum_h |w_h| |q_h . k|, the magnitude a
score's rounding error scales with -- because the signed head weights can cancel a score
to ~0, where a plain relative error is undefined.  The tighter 1e-5 norm-wise bound is also
checked for BF16, since the kernel accumulates exact bf16 products in float32.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from tests._util import assert_scores_close, assert_topk_equivalent, normwise_bound
from tests.conftest import bf16_from_bits, cfg1_inputs, load_golden

pytestmark = pytest.mark.gpu

LENGTHS = [1, 17, 63, 64, 65, 127, 128, 129, 192, 256, 257]


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()
    yield
    from dsa_b200 import device_status

    assert device_status() == 0, "a kernel raised a device status bit"


def cuda(x, dtype=None):
    t = torch.as_tensor(np.asarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


@pytest.mark.parametrize("length", LENGTHS)
def test_full_scores_bf16_matches_reference_golden(length):
    from dsa_b200.progressive_kernel import full_scores_triton

    g = load_golden("progressive_kernel")
    q = bf16_from_bits(g["bf16_q"])
    k = bf16_from_bits(g[f"bf16_L{length}_keys"])
    w = g["bf16_w"]
    got = full_scores_triton(cuda(q, torch.bfloat16), cuda(w), cuda(k, torch.bfloat16))
    assert got.dtype == torch.float32 and got.shape == (length,)
    scale = normwise_bound(q, w, k)
    got = got.cpu().numpy()
    assert_scores_close(got, g[f"bf16_L{length}_scores"], scale, rtol=1e-5, atol=1e-7,
                        msg="bf16 vs reference golden")
    assert_scores_close(got, oracle.full_scores(q, w, k), scale, rtol=1e-5, atol=1e-7,
                        msg="bf16 vs oracle")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("length", [1, 100, 128, 1000, 4099])
def test_dense_16bit_matches_oracle(dtype, length):
    gen = torch.Generator().manual_seed(length)
    q = (torch.randn(64, 128, generator=gen) / math.sqrt(128)).to(dtype)
    w = torch.randn(64, generator=gen) / 8
    k = torch.randn(length, 128, generator=gen).to(dtype)
    from dsa_b200 import score_dense

    got = score_dense(q.cuda(), w.cuda(), k.cuda()).cpu().numpy()
    qf, kf = q.float().numpy(), k.float().numpy()
    want = oracle.full_scores(qf, w.numpy(), kf)
    scale = normwise_bound(qf, w.numpy(), kf)
    assert_scores_close(got, want, scale, rtol=1e-5, atol=1e-7, msg=str(dtype))
    # the stated BF16 bar, plain relative with an absolute floor
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("length", LENGTHS)
def test_full_scores_f32_matches_reference_golden(length):
    from dsa_b200 import score_dense

    g = load_golden("progressive_kernel")
    q, w, k = g["f32_q"], g["f32_w"], g[f"f32_L{length}_keys"]
    got = score_dense(cuda(q), cuda(w), cuda(k)).cpu().numpy()
    assert_scores_close(got, g[f"f32_L{length}_scores"], normwise_bound(q, w, k), rtol=1e-5,
                        msg="f32")


def test_config1_f32_scores_and_top512():
    """BASELINE config 1 (f32, L=4096, top-512, seed 0) against the reference golden."""
    from dsa_b200 import scores_topk

    g = load_golden("cfg1")
    q, w, k = cfg1_inputs()
    idx, val = scores_topk(q.cuda(), w.cuda(), k.cuda(), 512, sorted=True)
    scale = normwise_bound(q.numpy(), w.numpy(), k.numpy())
    from dsa_b200 import score_dense

    s = score_dense(q.cuda(), w.cuda(), k.cuda()).cpu().numpy()
    assert_scores_close(s, g["scores"], scale, rtol=1e-5, msg="cfg1 scores")
    np.testing.assert_allclose(s, g["scores"], rtol=1e-5, atol=1e-5)
    assert_topk_equivalent(idx.cpu().numpy(), g["top512"], g["scores"], tol=1e-5,
                           msg="cfg1 top-512")
    # our own top-k of our own scores is exactly stable_topk of them
    np.testing.assert_array_equal(idx.cpu().numpy(), oracle.stable_topk(s, 512))
    np.testing.assert_array_equal(val.cpu().numpy(), s[idx.cpu().numpy()])


def test_config2_batched_bf16_score_topk():
    """BASELINE config 2 shape: B=32, L=8192 bf16, top-2048, f32 accumulation."""
    from dsa_b200 import score_dense, scores_topk

    gen = torch.Generator().manual_seed(0)
    b, length, kk = 32, 8192, 2048
    q = (torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16)
    w = torch.randn(b, 64, generator=gen) / math.sqrt(64)
    k = torch.randn(b, length, 128, generator=gen).to(torch.bfloat16)
    qc, wc, kc = q.cuda(), w.cuda(), k.cuda()
    scores = score_dense(qc, wc, kc).cpu().numpy()
    idx, val = scores_topk(qc, wc, kc, kk, sorted=True)
    idx, val = idx.cpu().numpy(), val.cpu().numpy()
    for row in range(b):
        qf, kf = q[row].float().numpy(), k[row].float().numpy()
        want = oracle.full_scores(qf, w[row].numpy(), kf)
        scale = normwise_bound(qf, w[row].numpy(), kf)
        assert_scores_close(scores[row], want, scale, rtol=1e-5, atol=1e-7, msg=f"row {row}")
        assert_topk_equivalent(idx[row], oracle.stable_topk(want, kk), want,
                               tol=2e-5 * scale.max(), msg=f"row {row}")
        np.testing.assert_array_equal(idx[row], oracle.stable_topk(scores[row], kk))
        np.testing.assert_array_equal(val[row], scores[row][idx[row]])


def test_strided_and_sliced_key_cache():
    """Keys living in a larger cache: row stride 256 elements, batch stride != L*row."""
    from dsa_b200 import score_dense

    gen = torch.Generator().manual_seed(3)
    cache = torch.randn(3, 700, 256, generator=gen).to(torch.bfloat16).cuda()
    keys = cache[:, 5:605, 64:192]  # [3,600,128], row stride 256
    q = (torch.randn(3, 64, 128, generator=gen) / 11).to(torch.bfloat16).cuda()
    w = (torch.randn(3, 64, generator=gen) / 8).cuda()
    got = score_dense(q, w, keys).cpu().numpy()
    for r in range(3):
        qf, kf = q[r].float().cpu().numpy(), keys[r].float().cpu().numpy()
        want = oracle.full_scores(qf, w[r].cpu().numpy(), kf)
        assert_scores_close(got[r], want, normwise_bound(qf, w[r].cpu().numpy(), kf),
                            rtol=1e-5, atol=1e-7)


def test_score_encoded_matches_reference_golden():
    from dsa_b200.sidecar import score_encoded

    g = load_golden("batched")
    got = score_encoded(cuda(g["q"]), cuda(g["w"]), cuda(g["k"]), key_chunk_size=32)
    got = got.cpu().numpy()
    for b in range(2):
        for qi in range(2):
            scale = normwise_bound(g["q"][b, qi], g["w"][b, qi], g["k"][b])
            assert_scores_close(got[b, qi], g["encoded"][b, qi], scale, rtol=1e-5)
    # bf16 inputs (the sidecar's decode dtype)
    qb = cuda(g["q"], torch.bfloat16)
    kb = cuda(g["k"], torch.bfloat16)
    got = score_encoded(qb, cuda(g["w"]), kb).cpu().numpy()
    want = oracle.score_encoded(qb.float().cpu().numpy(), g["w"], kb.float().cpu().numpy())
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-3)


def test_stable_topk_edge_cases_bit_exact():
    """Same float values in, stable_topk's exact index list out (ties, -inf, +-0)."""
    from dsa_b200.metrics import stable_topk

    g = load_golden("topk")
    for name in g["names"]:
        x = g[f"{name}_x"]
        for key in g.files:
            if key.startswith(f"{name}_k"):
                k = int(key[len(name) + 2:])
                got = stable_topk(cuda(x), k).cpu().numpy()
                np.testing.assert_array_equal(got, g[key], err_msg=key)


@pytest.mark.parametrize("length,k", [(1, 1), (5, 5), (1000, 1), (32768, 2048),
                                      (32769, 2048), (40000, 512), (131072, 2048),
                                      (300000, 4096), (65536, 8192)])
@pytest.mark.parametrize("sorted_", [True, False])
def test_topk_rows_match_oracle(length, k, sorted_):
    from dsa_b200 import topk

    rng = np.random.default_rng(length + k)
    s = np.round(rng.normal(size=(2, length)) * 64).astype(np.float32) / 64  # many ties
    idx, val = topk(cuda(s), k, sorted=sorted_)
    want_i, want_v = oracle.topk_rows(s, k, sorted=sorted_)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)


def test_topk_unsorted_large_k_single_segment():
    from dsa_b200 import topk

    rng = np.random.default_rng(9)
    s = rng.normal(size=(3, 30000)).astype(np.float32)
    idx, _ = topk(cuda(s), 20000, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), oracle.topk_rows(s, 20000, sorted=False)[0])


@pytest.mark.parametrize("case", ["zeros", "two_values", "clustered", "misaligned"])
@pytest.mark.parametrize("k", [1, 2048, 8192, 20000])
@pytest.mark.parametrize("sorted_", [True, False])
def test_topk_tie_heavy_clustered_and_misaligned_rows(case, k, sorted_):
    """Rows whose k-th key has far more equal or near-equal neighbours than the candidate
    list holds, and rows that do not start on a 16-byte boundary."""
    from dsa_b200 import topk

    if sorted_ and k > 8192:
        pytest.skip("k > 8192 is unsorted only")
    rng = np.random.default_rng(k)
    n = 30000
    if case == "zeros":
        s = np.zeros((2, n), np.float32)
        s[1, -5:] = 1.0  # a few larger keys after all the ties
    elif case == "two_values":
        s = np.where(rng.random((2, n)) < 0.7, np.float32(0.5), np.float32(-0.25))
        s = s.astype(np.float32)
    elif case == "clustered":
        s = (1.0 + rng.integers(0, 1 << 14, size=(2, n)) * 2.0 ** -23).astype(np.float32)
    else:
        s = rng.normal(size=(2, n + 1)).astype(np.float32)
    dev = cuda(s)
    if case == "misaligned":
        dev, s = dev[:, 1:], s[:, 1:]
    idx, val = topk(dev, k, sorted=sorted_)
    want_i, want_v = oracle.topk_rows(np.ascontiguousarray(s), k, sorted=sorted_)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)


def test_merge_topk_matches_oracle():
    from dsa_b200 import merge_topk, topk

    rng = np.random.default_rng(11)
    s = np.round(rng.normal(size=(4, 65536)) * 16).astype(np.float32) / 16
    shards = np.split(np.arange(65536), 8)
    cv, ci = [], []
    for p in shards:
        li, lv = topk(cuda(s[:, p]), 1024, sorted=False, index_dtype=torch.int32)
        cv.append(lv)
        ci.append(li + int(p[0]))
    mi, mv = merge_topk(torch.cat(cv, 1), torch.cat(ci, 1), 1024, sorted=True)
    want_i, want_v = oracle.topk_rows(s, 1024)
    np.testing.assert_array_equal(mi.cpu().numpy(), want_i)
    np.testing.assert_array_equal(mv.cpu().numpy(), want_v)


def test_api_errors():
    from dsa_b200 import score_dense, topk
    from dsa_b200.progressive_kernel import full_scores_triton

    q = torch.zeros(64, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(64, device="cuda")
    k = torch.zeros(10, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        full_scores_triton(q.float(), w, k)
    with pytest.raises(ValueError):
        full_scores_triton(q, w, k.cpu())
    with pytest.raises(ValueError):
        score_dense(q[:32], w, k)
    with pytest.raises(ValueError):
        topk(torch.zeros(10, device="cuda"), 11)
    assert score_dense(q, w, k[:0]).shape == (0,)


@pytest.mark.parametrize("length", [100, 1000, 32768, 32769, 40000, 65536, 100000])
@pytest.mark.parametrize("sorted_", [True, False])
def test_score_topk_plan_with_key_histogram_matches_separate_calls(length, sorted_):
    """The fused path (score kernel histograms keys, top-k starts from it) gives the same
    result as scoring and a plain top-k, on repeated runs (the histogram is left zeroed)."""
    from dsa_b200 import score_dense, topk
    from dsa_b200.indexer import ScoreTopkPlan

    gen = torch.Generator().manual_seed(length)
    b, k = 3, min(256, length)
    q = (torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16).cuda()
    w = (torch.randn(b, 64, generator=gen) / 8).cuda()
    keys = torch.randn(b, length, 128, generator=gen).to(torch.bfloat16).cuda()
    plan = ScoreTopkPlan(q, w, keys, k, sorted=sorted_, index_dtype=torch.int64)
    assert plan.use_hist
    for rep in range(3):
        if rep:
            q.mul_(-1 if rep == 1 else 0.5)  # new queries in the same buffers
        idx, val = plan.run()
        s = score_dense(q, w, keys)
        want_i, want_v = topk(s, k, sorted=sorted_)
        assert torch.equal(idx, want_i), rep
        assert torch.equal(val, want_v), rep
        if length > 32768:  # rows of several segments: the oracle as well
            oi, ov = oracle.topk_rows(s.cpu().numpy(), k, sorted=sorted_)
            np.testing.assert_array_equal(idx.cpu().numpy(), oi)
            np.testing.assert_array_equal(val.cpu().numpy(), ov)
    assert int(plan.key_hist.abs().sum()) == 0


@pytest.mark.parametrize("k,sorted_,length", [(1, True, 32768), (2048, False, 32768),
                                              (8192, True, 32768), (20000, False, 32768),
                                              (2048, False, 70000), (8192, True, 70000),
                                              (1, True, 40000)])
def test_score_topk_plan_histogram_path_with_tied_scores(k, sorted_, length):
    """All-zero keys give one score value for the whole row: the histogram's k-th bin
    holds every key, and the tie rule (lowest index first) decides -- within one segment
    and across the segments and merge level of longer rows."""
    from dsa_b200 import score_dense
    from dsa_b200.indexer import ScoreTopkPlan

    gen = torch.Generator().manual_seed(k)
    b = 2
    q = (torch.randn(b, 64, 128, generator=gen) / math.sqrt(128)).to(torch.bfloat16).cuda()
    w = (torch.randn(b, 64, generator=gen) / 8).cuda()
    keys = torch.zeros(b, length, 128, dtype=torch.bfloat16, device="cuda")
    keys[1, 7000:7003] = 1.0  # a few distinct scores in the second row
    plan = ScoreTopkPlan(q, w, keys, k, sorted=sorted_, index_dtype=torch.int64)
    assert plan.use_hist
    idx, val = plan.run()
    s = score_dense(q, w, keys).cpu().numpy()
    want_i, want_v = oracle.topk_rows(s, k, sorted=sorted_)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(plan.key_hist.abs().sum()) == 0


def _key_hist(s: np.ndarray) -> np.ndarray:
    """Per-row counts of the order-preserving uint32 key's top 12 bits (-0 counts as +0)."""
    b = s.astype(np.float32).view(np.uint32).copy()
    b[b == 0x80000000] = 0
    key = np.where(b & 0x80000000, ~b, b | 0x80000000).astype(np.uint32)
    return np.stack([np.bincount(r >> 20, minlength=4096) for r in key]).astype(np.int32)


@pytest.mark.parametrize("length,k,sorted_", [(32768, 2048, False), (30000, 512, True),
                                              (20000, 20000, False), (32768, 1, True)])
def test_topk_hist_special_values_with_host_histogram(length, k, sorted_):
    """tdsa_topk_hist from a histogram made on the host: +-0, +-inf, denormals and ties."""
    from dsa_b200 import _capi as capi

    rng = np.random.default_rng(length + k)
    s = np.round(rng.normal(size=(3, length)) * 8).astype(np.float32) / 8
    s[0, rng.integers(0, length, 300)] = -0.0
    s[0, rng.integers(0, length, 300)] = 0.0
    s[1, rng.integers(0, length, 50)] = np.inf
    s[1, rng.integers(0, length, 50)] = -np.inf
    s[2, rng.integers(0, length, 400)] = np.float32(1e-45)  # denormal ties
    s[2, rng.integers(0, length, 400)] = np.float32(-1e-45)
    dev = cuda(s)
    hist = cuda(_key_hist(s))
    idx = torch.empty(3, k, dtype=torch.int64, device="cuda")
    val = torch.empty(3, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist", dev.data_ptr(), dev.stride(0), 3, length, k, int(sorted_),
              idx.data_ptr(), 8, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=sorted_)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(hist.abs().sum()) == 0  # consumed and zeroed


def _key_hist_segments(s: np.ndarray, seg: int = 32768) -> np.ndarray:
    """[rows][ceil(L / seg)][4096] per-segment key histograms (tdsa_key_hist_bytes layout)."""
    parts = [_key_hist(s[:, i:i + seg]) for i in range(0, s.shape[1], seg)]
    return np.stack(parts, axis=1).astype(np.int32)


@pytest.mark.parametrize("length,k,sorted_", [(40000, 2048, False), (70000, 512, True),
                                              (65536, 8192, False), (100000, 1, True)])
def test_topk_hist_ws_segments_with_host_histograms(length, k, sorted_):
    """tdsa_topk_hist_ws over rows of several segments, each started from its own histogram
    (made on the host), with special values and ties; the histograms end zeroed."""
    from dsa_b200 import _capi as capi

    rng = np.random.default_rng(length + k)
    s = np.round(rng.normal(size=(3, length)) * 8).astype(np.float32) / 8
    s[0, rng.integers(0, length, 300)] = -0.0
    s[1, rng.integers(0, length, 50)] = np.inf
    s[1, rng.integers(0, length, 50)] = -np.inf
    s[2, rng.integers(0, length, 400)] = np.float32(1e-45)
    dev = cuda(s)
    hist = cuda(_key_hist_segments(s))
    lib = capi.lib()
    assert hist.numel() * 4 == lib.tdsa_key_hist_bytes(3, length)
    nbytes = lib.tdsa_topk_workspace_bytes(3, length, k)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    idx = torch.empty(3, k, dtype=torch.int64, device="cuda")
    val = torch.empty(3, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist_ws", dev.data_ptr(), dev.stride(0), 3, length, k, int(sorted_),
              idx.data_ptr(), 8, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=sorted_)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(hist.abs().sum()) == 0


@pytest.mark.parametrize("sorted_", [True, False])
def test_topk_hist_ws_short_tail_segment_with_minus_inf_ties(sorted_):
    """The last 32768-key segment is shorter than k, so the merge level receives padding;
    most keys score -inf, so the k-th key is -inf and real -inf keys (lowest index first)
    must win over the padding."""
    from dsa_b200 import _capi as capi

    length, k = 32768 * 2 + 100, 2048
    rng = np.random.default_rng(7)
    s = np.full((2, length), -np.inf, dtype=np.float32)
    for r in range(2):
        live = rng.choice(length, 1000, replace=False)
        s[r, live] = rng.normal(size=1000).astype(np.float32)
    s[1, -50:] = 3.0  # ties inside the short tail segment
    dev = cuda(s)
    hist = cuda(_key_hist_segments(s))
    lib = capi.lib()
    nbytes = lib.tdsa_topk_workspace_bytes(2, length, k)
    ws = torch.full((max(nbytes, 1),), 0x7F, dtype=torch.uint8, device="cuda")  # not zero
    idx = torch.empty(2, k, dtype=torch.int64, device="cuda")
    val = torch.empty(2, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist_ws", dev.data_ptr(), dev.stride(0), 2, length, k, int(sorted_),
              idx.data_ptr(), 8, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=sorted_)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)


@pytest.mark.parametrize("batch,length,k", [
    (1, 32768, 2048),   # 8 CTAs per row, 4 keys per thread
    (1, 16384, 1),      # 8 CTAs, 2 keys per thread
    (1, 8192, 8192),    # 4 CTAs, k = length
    (1, 5000, 777),     # 2 CTAs, 4 keys per thread, the last threads partly outside the row
    (2, 4096, 2048),    # 2 CTAs, 2 keys per thread
    (9, 32768, 20000),  # 8 CTAs per row, k above the list capacity of one CTA
    (20, 32768, 2048),  # 4 CTAs per row, 8 keys per thread
    (64, 32768, 2048),  # 2 CTAs per row, 16 keys per thread (the config-4 shape)
    (40, 30001, 513),   # 2 CTAs per row, odd row stride (unaligned rows: scalar loads)
])
def test_cluster_topk_rows_match_oracle(batch, length, k):
    """The cluster top-k (a row over 2-8 CTAs, unsorted, from the score kernel's histogram)
    against stable_topk: rounded normals (heavy ties), +-0, +-inf, denormals, one row of a
    single value and one of -inf only; the histograms end zeroed."""
    from dsa_b200 import _capi as capi

    rng = np.random.default_rng(batch * 7 + length + k)
    s = np.round(rng.normal(size=(batch, length)) * 64).astype(np.float32) / 64
    s[0, rng.integers(0, length, length // 50)] = -0.0
    s[0, rng.integers(0, length, length // 50)] = 0.0
    if batch > 1:
        s[1] = 0.25  # one value: the tie rule alone decides
    if batch > 2:
        s[2, rng.integers(0, length, 50)] = np.inf
        s[2, rng.integers(0, length, length // 3)] = -np.inf
        s[-1, rng.integers(0, length, 400)] = np.float32(1e-45)
    if batch > 3:
        s[3] = -np.inf  # the k-th key is -inf: every key of the row ties
    dev = cuda(s)
    hist = cuda(_key_hist(s))
    idx = torch.empty(batch, k, dtype=torch.int32, device="cuda")
    val = torch.empty(batch, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist", dev.data_ptr(), dev.stride(0), batch, length, k, 0,
              idx.data_ptr(), 4, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(hist.abs().sum()) == 0  # consumed and zeroed


@pytest.mark.parametrize("batch,length,k", [
    (24, 32768, 1),      # one CTA per row (too many rows for clusters), 32 keys per thread
    (24, 32768, 8192),   # the list at its capacity
    (24, 32768, 9000),   # keys >= the k-th key's bin overflow the list: the general path
    (80, 20000, 2048),   # 32 keys per thread, the last threads partly outside the row
    (80, 12000, 1000),   # 16 keys per thread
    (80, 6000, 700),     # 8 keys per thread
    (80, 7001, 64),      # odd row stride (unaligned rows: loads instead of bulk copies)
])
def test_segment_topk_from_histogram_matches_oracle(batch, length, k):
    """The one-CTA top-k started from the score kernel's histogram (rows too many for the
    cluster top-k): every key at or above the k-th key's 12-bit bin goes to the list, two
    histogram levels over the bin find the exact k-th key, one ordered pass takes.  Rounded
    normals (heavy ties), +-0, +-inf, denormals, rows of one value and of -inf only, a row
    whose k-th bin holds most keys, against stable_topk in index order."""
    from dsa_b200 import _capi as capi

    rng = np.random.default_rng(batch * 5 + length + k)
    s = np.round(rng.normal(size=(batch, length)) * 64).astype(np.float32) / 64
    s[0, rng.integers(0, length, length // 50)] = -0.0
    s[0, rng.integers(0, length, length // 50)] = 0.0
    s[1] = 0.25  # one value: the tie rule alone decides
    s[2, rng.integers(0, length, 50)] = np.inf
    s[2, rng.integers(0, length, length // 3)] = -np.inf
    s[3] = -np.inf  # the k-th key is -inf: every key of the row ties
    s[4, rng.integers(0, length, 400)] = np.float32(1e-45)
    s[4, rng.integers(0, length, 400)] = np.float32(-1e-45)
    s[5] = np.float32(1.0) + rng.integers(0, 4096, length).astype(np.float32) * np.float32(2 ** -23)
    s[6, : length // 2] = np.float32(3.0)  # ties straddling the k-th key in one sub-bin
    s[7] = rng.normal(size=length).astype(np.float32)  # distinct values
    dev = cuda(s)
    hist = cuda(_key_hist(s))
    idx = torch.empty(batch, k, dtype=torch.int32, device="cuda")
    val = torch.empty(batch, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist", dev.data_ptr(), dev.stride(0), batch, length, k, 0,
              idx.data_ptr(), 4, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(hist.abs().sum()) == 0  # consumed and zeroed


@pytest.mark.parametrize("length,k", [(40000, 2048), (70000, 512), (36865, 2048)])
def test_segment_topk_merge_level_from_histogram(length, k):
    """Rows longer than one segment on a batch too large for clusters: each segment's top-k
    and then the merge level (explicit indices, started from the bins the first level
    passes on) against stable_topk."""
    from dsa_b200 import _capi as capi

    batch = 24
    rng = np.random.default_rng(length + k)
    s = np.round(rng.normal(size=(batch, length)) * 32).astype(np.float32) / 32
    s[0, rng.integers(0, length, 60)] = np.inf
    s[1] = -np.inf
    s[1, rng.integers(0, length, 100)] = 2.0
    s[2, -1000:] = 5.0  # ties at the top of the last segment
    dev = cuda(s)
    hist = cuda(_key_hist_segments(s))
    lib = capi.lib()
    assert lib.tdsa_topk_levels(batch, length, k, 1) == 2
    nbytes = lib.tdsa_topk_workspace_bytes(batch, length, k)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    idx = torch.empty(batch, k, dtype=torch.int64, device="cuda")
    val = torch.empty(batch, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist_ws", dev.data_ptr(), dev.stride(0), batch, length, k, 0,
              idx.data_ptr(), 8, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(hist.abs().sum()) == 0


@pytest.mark.parametrize("length,k", [(32769, 2048), (33001, 1), (34567, 8192),
                                      (36864, 2048), (36000, 36000 // 5)])
def test_wide_row_topk_one_level_from_two_histograms(length, k):
    """Rows just past one 32768-key segment on a batch too large for clusters: one CTA per
    row takes the row's 32768 + up to 4096 keys in one level, started from the sum of its
    two segment histograms, with no candidate list (any number of keys may tie in the k-th
    key's bin).  Heavy ties, +-0, +-inf, denormals, a row of one value, a row of -inf only,
    against stable_topk in index order; the histograms end zeroed."""
    from dsa_b200 import _capi as capi

    batch = 24
    rng = np.random.default_rng(length * 3 + k)
    s = np.round(rng.normal(size=(batch, length)) * 64).astype(np.float32) / 64
    s[0, rng.integers(0, length, length // 50)] = -0.0
    s[0, rng.integers(0, length, length // 50)] = 0.0
    s[1] = 0.25
    s[2, rng.integers(0, length, 50)] = np.inf
    s[2, rng.integers(0, length, length // 3)] = -np.inf
    s[3] = -np.inf
    s[4, rng.integers(0, length, 400)] = np.float32(1e-45)
    s[5, 32700:] = np.float32(7.0)  # ties straddling the segment edge and the tail
    s[6] = rng.normal(size=length).astype(np.float32)
    s[7, -3:] = np.float32(100.0)  # the largest keys in the tail
    dev = cuda(s)
    hist = cuda(_key_hist_segments(s))
    lib = capi.lib()
    assert lib.tdsa_topk_levels(batch, length, k, 1) == 1  # unsorted: one level
    assert lib.tdsa_topk_levels(batch, length, k, 3) == 2  # sorted: segments + merge
    nbytes = lib.tdsa_topk_workspace_bytes(batch, length, k)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    idx = torch.empty(batch, k, dtype=torch.int32, device="cuda")
    val = torch.empty(batch, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist_ws", dev.data_ptr(), dev.stride(0), batch, length, k, 0,
              idx.data_ptr(), 4, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(hist.abs().sum()) == 0


def test_cluster_topk_falls_back_when_histogram_is_short():
    """A histogram whose counts total less than k does not describe the row: the cluster
    kernel narrows from the full key range itself and still returns stable_topk."""
    from dsa_b200 import _capi as capi

    rng = np.random.default_rng(3)
    s = rng.normal(size=(2, 32768)).astype(np.float32)
    dev = cuda(s)
    hist = torch.zeros(2, 4096, dtype=torch.int32, device="cuda")
    idx = torch.empty(2, 2048, dtype=torch.int64, device="cuda")
    val = torch.empty(2, 2048, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist", dev.data_ptr(), dev.stride(0), 2, 32768, 2048, 0,
              idx.data_ptr(), 8, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, 2048, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)


def test_graph_capture_of_first_plan_run():
    """ScoreTopkPlan.run captured into a CUDA graph before it ever ran, in a fresh process
    (one-time setup such as kernel attributes and the cluster-size query happens inside
    the capture), for the cluster top-k (8 and 4 CTAs per row) and one CTA per row."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, PYTHONPATH=str(root))
    res = subprocess.run([sys.executable, str(root / "tests" / "_graph_capture_worker.py")],
                         cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]


@pytest.mark.parametrize("batch,length,k", [
    (8, 131072, 2048),   # config 5 on one GPU: 16 keys per thread over 8 CTAs
    (8, 65536, 2048),    # config 5 on two GPUs
    (15, 100001, 512),   # odd length, the last segment short
    (2, 131072, 8192),   # every key of row 0 tied: 131072 in the range, above 16 bits
])
def test_cluster_topk_long_rows_match_oracle(batch, length, k):
    """Rows of several histogram segments selected in one cluster launch (8 CTAs, the
    segments' histograms summed) against stable_topk: ties, +-0, -inf runs, a fully tied
    row (its in-range count exceeds 16 bits); the histograms end zeroed."""
    from dsa_b200 import _capi as capi

    rng = np.random.default_rng(length + k)
    s = np.round(rng.normal(size=(batch, length)) * 64).astype(np.float32) / 64
    if batch == 2:
        s[0] = 0.5
    if batch > 1:
        s[1, rng.integers(0, length, length // 4)] = -np.inf
        s[1, rng.integers(0, length, 100)] = -0.0
    dev = cuda(s)
    hist = cuda(_key_hist_segments(s))
    lib = capi.lib()
    nbytes = lib.tdsa_topk_workspace_bytes(batch, length, k)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    idx = torch.empty(batch, k, dtype=torch.int64, device="cuda")
    val = torch.empty(batch, k, dtype=torch.float32, device="cuda")
    capi.call("tdsa_topk_hist_ws", dev.data_ptr(), dev.stride(0), batch, length, k, 0,
              idx.data_ptr(), 8, idx.stride(0), val.data_ptr(), val.stride(0), hist.data_ptr(),
              ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
    want_i, want_v = oracle.topk_rows(s, k, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
    assert int(hist.abs().sum()) == 0


@pytest.mark.parametrize("batch,length,k", [(1, 32768, 2048), (3, 16384, 1024),
                                            (4, 20000, 512)])
def test_topk_device_histogram_special_rows(batch, length, k):
    """tdsa_topk on a few unsorted rows of one segment: the row histograms are built on the
    device (row_hist_part_kernel, up to 16 CTAs per row adding into one histogram) and the
    cluster top-k starts from them.  Rows with -inf runs, +inf, -0.0, ties, and one row of
    -inf only, against stable_topk (NaN is left out: the reference's stable_topk returns
    fewer than k indices for a row holding NaN, metrics.py:18-21)."""
    from dsa_b200 import _capi as capi
    from dsa_b200 import topk

    # the workspace covers the device histograms: the split path is the one taken
    assert capi.lib().tdsa_topk_workspace_bytes(batch, length, k) >= batch * 4096 * 4
    rng = np.random.default_rng(batch * 11 + length)
    s = np.round(rng.normal(size=(batch, length)) * 64).astype(np.float32) / 64
    s[0, rng.integers(0, length, length // 3)] = -np.inf
    s[0, rng.integers(0, length, 40)] = np.inf
    s[0, rng.integers(0, length, 200)] = -0.0
    if batch > 1:
        s[1, 1000:4000] = -np.inf
    if batch > 2:
        s[2] = -np.inf  # every key ties at -inf
    idx, val = topk(cuda(s), k, sorted=False, index_dtype=torch.int64)
    want_i, want_v = oracle.topk_rows(s, k, sorted=False)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(val.cpu().numpy(), want_v)
