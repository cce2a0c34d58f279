"""Pin the CPU oracle to golden vectors produced by the reference implementation."""

from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest

import oracle
from oracle import progressive_exact, replay
from oracle.certified import shared_block_key_norms
from tests.conftest import bf16_from_bits, cfg1_inputs, load_golden

LENGTHS = [1, 17, 63, 64, 65, 127, 128, 129, 192, 256, 257]


@pytest.mark.parametrize("length", LENGTHS)
def test_full_scores_f32_matches_reference(length):
    g = load_golden("progressive_kernel")
    got = oracle.full_scores(g["f32_q"], g["f32_w"], g[f"f32_L{length}_keys"])
    np.testing.assert_allclose(got, g[f"f32_L{length}_scores"], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("length", LENGTHS)
def test_full_scores_bf16_matches_reference(length):
    g = load_golden("progressive_kernel")
    q = bf16_from_bits(g["bf16_q"])
    k = bf16_from_bits(g[f"bf16_L{length}_keys"])
    got = oracle.full_scores(q, g["bf16_w"], k)
    np.testing.assert_allclose(got, g[f"bf16_L{length}_scores"], rtol=1e-5, atol=1e-6)


def test_head_routing_matches_reference():
    g = load_golden("progressive_kernel")
    assert oracle.dynamic_head_ids(g["dyn_ties_w"]).tolist() == g["dyn_ties_ids"].tolist()
    assert oracle.dynamic_head_ids(g["f32_w"]).tolist() == g["dyn_rand_ids"].tolist()
    sel, rem = oracle.split_head_ids(np.array([0, 2, 4, 6, 8, 10, 12, 63]))
    assert sel.tolist() == g["split_sel"].tolist()
    assert rem.tolist() == g["split_rem"].tolist()
    for bad in ([0, 1], [0, 1, 2, 3, 4, 5, 6, 64], [0, 1, 2, 3, 4, 5, 6, 6]):
        with pytest.raises(ValueError):
            oracle.split_head_ids(np.array(bad))


def test_torch_progressive_scores_matches_reference():
    g = load_golden("progressive_kernel")
    q, w = g["f32_q"], g["f32_w"]
    for tag in g["prog_cases"]:
        tag = str(tag)
        length, bs = int(tag.split("_")[1][1:]), int(tag.split("_")[2][1:])
        keys = g[f"f32_L{length}_keys"] if f"f32_L{length}_keys" in g else None
        if keys is None:
            from tests.golden.make_golden import cpu_inputs

            keys = cpu_inputs(length)[2].numpy()
        heads = oracle.dynamic_head_ids(w)
        thr = float(g[tag + "_thr"])
        out, acc, mx = oracle.progressive_scores(q, w, keys, heads, g[tag + "_direct"],
                                                 thr, block_size=bs)
        np.testing.assert_allclose(mx, g[tag + "_max"], rtol=1e-5, atol=1e-4)
        # a promotion decision may differ only where the block max ties the threshold
        # within float32 rounding (the q50 threshold is itself one of the block maxima)
        near = np.abs(g[tag + "_max"].astype(np.float64) - thr) <= 1e-5 * max(1.0, abs(thr))
        differ = acc != g[tag + "_accepted"]
        assert not np.any(differ & ~near), tag
        same = np.repeat(~differ, bs)[: keys.shape[0]]
        np.testing.assert_allclose(out[same], g[tag + "_scores"][same], rtol=1e-5, atol=1e-4)


def test_progressive_qk_reduction_matches_reference():
    g = load_golden("progressive_kernel")
    got = [oracle.progressive_qk_reduction(8192, 0, 0), oracle.progressive_qk_reduction(8192, 128, 0),
           oracle.progressive_qk_reduction(8192, 32, 16),
           oracle.progressive_qk_reduction(1000, 3, 5, block_size=128)]
    np.testing.assert_allclose(got, g["qkred"], rtol=0, atol=1e-15)
    with pytest.raises(ValueError):
        oracle.progressive_qk_reduction(8192, 129, 0)
    with pytest.raises(ValueError):
        oracle.progressive_qk_reduction(8192, -1, 0)


def test_cfg1_matches_reference():
    g = load_golden("cfg1")
    q, w, k = cfg1_inputs()
    assert hashlib.sha256(k.numpy().tobytes()).hexdigest() == str(g["keys_sha256"])
    np.testing.assert_array_equal(q.numpy(), g["q"])
    scores = oracle.full_scores(q.numpy(), w.numpy(), k.numpy())
    np.testing.assert_allclose(scores, g["scores"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(oracle.stable_topk(g["scores"], 512), g["top512"])
    f64 = oracle.relu_index_score(q.numpy(), k.numpy(), w.numpy())
    np.testing.assert_allclose(f64, g["relu_index_f64"], rtol=1e-12, atol=1e-12)


def test_stable_topk_matches_reference():
    g = load_golden("topk")
    for name in g["names"]:
        x = g[f"{name}_x"]
        for key in g.files:
            if key.startswith(f"{name}_k"):
                k = int(key[len(name) + 2 :])
                np.testing.assert_array_equal(oracle.stable_topk(x, k), g[key], err_msg=key)


def test_topk_rows_and_merge_agree_with_stable_topk():
    rng = np.random.default_rng(3)
    s = np.round(rng.normal(size=(3, 1000)) * 3).astype(np.float32)  # many ties
    idx, vals = oracle.topk_rows(s, 100)
    for r in range(3):
        np.testing.assert_array_equal(idx[r], oracle.stable_topk(s[r], 100))
    # shard into 4 contiguous ranges, take local top-k, merge
    parts = np.split(np.arange(1000), 4)
    cs, ci = [], []
    for p in parts:
        li, lv = oracle.topk_rows(s[:, p], 100, sorted=False)
        cs.append(lv)
        ci.append(li + p[0])
    mi, mv = oracle.merge_topk(np.concatenate(cs, 1), np.concatenate(ci, 1), 100)
    np.testing.assert_array_equal(mi, idx)
    np.testing.assert_array_equal(mv, vals)


def test_certified_matches_reference():
    g = load_golden("certified")
    from oracle.certified import block_key_norms, temporal_score_radius

    rep = np.repeat(g["keys"][:, 0][:, None, :], 8, axis=1)
    norms = block_key_norms(rep, 7)
    np.testing.assert_allclose(norms, g["norms"], rtol=1e-14)
    np.testing.assert_allclose(block_key_norms(g["keys"], 5), g["norms_full"], rtol=1e-14)
    rad = temporal_score_radius(g["qc"], g["qp"], g["wc"], g["wp"], norms)
    np.testing.assert_allclose(rad, g["radius"], rtol=1e-14)
    for b, s in enumerate(range(0, 37, 7)):
        assert np.all(np.abs(g["cur"][s : s + 7] - g["prev"][s : s + 7]) <= rad[b] + 1e-10)
    n64 = shared_block_key_norms(g["ikeys"], 64)
    np.testing.assert_allclose(n64, g["inorms"][:, 0], rtol=1e-14)
    rad = temporal_score_radius(g["iq1"], g["iq0"], g["iw1"], g["iw0"], g["inorms"])
    np.testing.assert_allclose(rad, g["iradius"], rtol=1e-13)


def test_replay_filter_matches_reference():
    g = load_golden("replay")
    for name in g["names"]:
        k, bs, gs = g[f"{name}_meta"]
        res = replay.replay_transition(g[f"{name}_prev"], g[f"{name}_cur"], k=int(k),
                                       block_size=int(bs), gamma_sigma=float(gs),
                                       method=str(g[f"{name}_method"]),
                                       scan_order_name=str(g[f"{name}_order"]))
        want = g[f"{name}_out"]
        got = [res["qk_scored"], res["blocks_pruned"], res["false_cold_blocks"], res["recall"],
               float(res["exact_match"]), res["tau_seed"], res["net_byte_reduction"]]
        np.testing.assert_allclose(got, want, rtol=1e-12, err_msg=str(name))


def test_certified_filter_matches_reference_compiled_filter():
    g = load_golden("replay")
    prev_s, cur_s = g["cert_prev"], g["cert_cur"]
    for bs in (16, 32, 64):
        upper = g[f"cert_B{bs}_upper"]
        nb = upper.size
        ptop = oracle.stable_topk(prev_s, 32)
        ttop = oracle.stable_topk(cur_s, 32)
        hot = np.zeros(nb, dtype=bool)
        hot[ptop // bs] = True
        pmax = np.array([prev_s[s : s + bs].max() for s in range(0, 300, bs)])
        order = replay.scan_order("previous_hot", upper, pmax, hot)
        got = replay.compiled_filter(cur_s, ptop, ttop, upper, order, bs,
                                     float(np.min(cur_s[ptop])), True)
        np.testing.assert_allclose(np.array(got, dtype=np.float64), g[f"cert_B{bs}_out"])
        assert got[3] == 32  # the certified bound never loses a true top-k key


def test_batched_paths_match_reference():
    g = load_golden("batched")
    enc = oracle.score_encoded(g["q"], g["w"], g["k"], key_chunk_size=32)
    np.testing.assert_allclose(enc, g["encoded"], rtol=1e-5, atol=1e-5)
    hs = oracle.score_head_sparse(g["q"][0], g["w"][0], g["k"][0], g["ids_fixed"])
    np.testing.assert_allclose(hs, g["hs_fixed"], rtol=1e-5, atol=1e-5)
    hs = oracle.score_head_sparse(g["q"][0], g["w"][0], g["k"][0], g["ids_dyn"])
    np.testing.assert_allclose(hs, g["hs_dyn"], rtol=1e-5, atol=1e-5)


def test_fused_semantics_consistent_with_torch_reference():
    """Triton-kernel semantics (direct blocks: 64 heads, block_max -inf) vs the torch ref."""
    g = load_golden("progressive_kernel")
    q, w, k = g["f32_q"], g["f32_w"], g["f32_L257_keys"]
    heads = oracle.dynamic_head_ids(w)
    direct = np.array([1, 0, 0, 1, 0], dtype=bool)
    for thr in (-math.inf, math.inf, 0.0):
        s1, a1, m1 = oracle.progressive_scores_fused(q, w, k, heads, direct, thr)
        s2, a2, m2 = oracle.progressive_scores(q, w, k, heads, direct, thr)
        np.testing.assert_array_equal(a1.astype(bool), a2)
        np.testing.assert_allclose(s1, s2, rtol=1e-5, atol=1e-4)
        np.testing.assert_array_equal(m1[~direct], m2[~direct])
        assert np.all(np.isneginf(m1[direct]))
        s3, a3, m3 = oracle.two_pass_scores(q, w, k, heads, direct, thr)
        np.testing.assert_array_equal(a3, a1)
        np.testing.assert_allclose(s3, s1, rtol=1e-5, atol=1e-4)


def test_exact_progressive_oracle_is_exact_over_ar1_trace():
    """Config-3-shaped trace (scaled down): the exact path's top-k equals dense every step."""
    rng = np.random.default_rng(0)
    length, k = 2048, 128
    q = rng.normal(size=(64, 128)) / math.sqrt(128)
    w = rng.normal(size=64) / 8
    keys = rng.normal(size=(length + 8, 128)).astype(np.float32)
    for bs in (16, 32, 64, 128):
        state, _, _ = progressive_exact.exact_init(q, w, keys[:length], k, bs)
        qt = q
        for step in range(1, 9):
            qt = 0.95 * qt + math.sqrt(1 - 0.95 ** 2) * rng.normal(size=(64, 128)) / math.sqrt(128)
            cur = keys[: length + step]
            top, scores, stats, state = progressive_exact.exact_step(state, qt, w, cur)
            dense = oracle.full_scores(qt, w, cur)
            np.testing.assert_array_equal(top, oracle.stable_topk(dense, k))
            assert stats["keys_read"] <= cur.shape[0]


def test_exact_progressive_prunes_structured_keys():
    """Keys with far-apart block norms: the bound prunes, and the result stays exact."""
    rng = np.random.default_rng(1)
    length, k, bs = 4096, 64, 64
    q = rng.normal(size=(64, 128)) / math.sqrt(128)
    w = np.abs(rng.normal(size=64)) / 8
    scale = np.repeat(np.where(rng.random(length // bs) < 0.1, 3.0, 0.05), bs)
    keys = (rng.normal(size=(length, 128)) * scale[:, None]).astype(np.float32)
    state, _, _ = progressive_exact.exact_init(q, w, keys, k, bs)
    q2 = 0.999 * q + 0.02 * rng.normal(size=(64, 128)) / math.sqrt(128)
    top, _, stats, _ = progressive_exact.exact_step(state, q2, w, keys)
    np.testing.assert_array_equal(top, oracle.stable_topk(oracle.full_scores(q2, w, keys), k))
    assert stats["pruned_blocks"] > 0


def test_sidecar_projection_matches_reference():
    from oracle import sidecar as osc

    g = load_golden("sidecar")
    q, w = osc.encode_queries(g["hq"][:, 0], g["wq"], g["ww"], g["qpos"][:, 0])
    # the float32 RoPE angle pos * inv_freq carries ~pos * 2^-24 rad of rounding, so at
    # position 1000 one ulp of inv_freq moves a rotated value by ~1e-4
    np.testing.assert_allclose(q, g["q"][:, 0], rtol=1e-5, atol=5e-4)
    np.testing.assert_allclose(w, g["w"][:, 0], rtol=1e-5, atol=1e-7)
    # encode_keys = RoPE(LayerNorm(h @ wk^T)); LayerNorm(eps=1e-6) with unit affine
    k = osc.encode_keys(g["hk"][0], g["wk"], np.arange(5))
    np.testing.assert_allclose(k, g["k"][0], rtol=1e-4, atol=1e-5)
    # the 16-bit rounding helper used for the Linear's output, against torch's casts
    import torch

    x = np.array([1.0, 1.00390625, 1.005859375, -3.0e38, 65520.0, 1e-9, 0.1, -2.5])
    want = torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16).double().numpy()
    np.testing.assert_array_equal(osc.round_to(x, "bf16"), want)
    with np.errstate(over="ignore"):
        want = torch.from_numpy(x).to(torch.float16).double().numpy()
    np.testing.assert_array_equal(osc.round_to(x, "f16"), want)


def test_verifier_dim_sparse_oracle_matches_reference_golden():
    """oracle.verifier (verifier_scoring.py:9-139) against the reference's own outputs."""
    from oracle import verifier as ov

    g = load_golden("verifier")
    np.testing.assert_allclose(ov.normalized_hadamard(g["k"]), g["had_k"], rtol=1e-6,
                               atol=1e-6)
    np.testing.assert_allclose(ov.normalized_hadamard(g["q"]), g["had_q"], rtol=1e-6,
                               atol=1e-7)
    for bits in (2, 4, 8):
        qk, sc = ov.fake_symmetric_quantize(g["k"], bits)
        assert sc == pytest.approx(float(g[f"fq{bits}_scale"]), rel=1e-12)
        np.testing.assert_array_equal(qk, g[f"fq{bits}_k"])
    for rot in ("none", "hadamard"):
        for bits in (None, 4, 8):
            got = ov.score_dim_sparse(g["q"], g["w"], g["k"], g["dims"], rotation=rot, bits=bits)
            np.testing.assert_allclose(got, g[f"ds_{rot}_{bits or 0}"], rtol=1e-4, atol=1e-5)
    got = ov.score_dim_sparse(g["q"], g["w"], g["k"], g["dims"], bits=4, query_scale=0.05,
                              key_scale=0.5)
    np.testing.assert_allclose(got, g["ds_none_4_fixed"], rtol=1e-4, atol=1e-5)
    # full width without rotation: the dimension path reconstructs the dense score
    # (tests/test_verifier_scoring.py:23-30 of the reference)
    full = ov.score_dim_sparse(g["q"], g["w"], g["k"], np.arange(128))
    dense = np.stack([oracle.full_scores(g["q"][i], g["w"][i], g["k"]) for i in range(2)])
    np.testing.assert_allclose(full, dense, rtol=1e-5, atol=1e-5)
