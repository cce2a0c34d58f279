"""Generate the golden vectors in this folder by running the REFERENCE implementation.

Run once, where the reference project is available (it is not on the GPU box):

    python tests/golden/make_golden.py --reference-src <path to temporal_dsa's src/>
    python tests/golden/make_golden.py --reference-src <...> --only verifier   # one fixture
    python tests/golden/make_golden.py --reference-src <...> --only trace
    python tests/golden/make_golden.py --reference-src <...> --only approx

Every output array below is computed by the reference's own functions
(``temporal_dsa.progressive_kernel``, ``.metrics``, ``.certified``, ``.replay``,
``.sidecar``, ``.verifier_scoring``, ``.trace``, ``.approx``, ``.verifier``).  Inputs are seeded; small inputs are stored
verbatim (bf16 tensors as their uint16 bit patterns), the config-1 key cache is
regenerated from its seed and pinned by a SHA-256 of its bytes.
"""

from __future__ import annotations

import argparse
import hashlib
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().astype(np.uint16)


def cfg1_inputs():
    """seed 0, q ~ N(0,1)/sqrt(128), w ~ N(0,1)/sqrt(64), K ~ N(0,1)."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(64, 128, generator=g) / math.sqrt(128)
    w = torch.randn(64, generator=g) / math.sqrt(64)
    k = torch.randn(4096, 128, generator=g)
    return q, w, k


def cpu_inputs(length: int):
    """tests/test_progressive_kernel.py:23-28 of the reference."""
    g = torch.Generator().manual_seed(1582)
    return (torch.randn(64, 128, generator=g), torch.randn(64, generator=g),
            torch.randn(length, 128, generator=g))


def bf16_inputs(length: int, seed: int = 1582):
    """CPU-seeded analogue of the reference's cuda_inputs (test_progressive_kernel.py:131-136)."""
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(64, 128, generator=g) * 0.1).to(torch.bfloat16)
    w = torch.randn(64, generator=g)
    k = (torch.randn(length, 128, generator=g) * 0.1).to(torch.bfloat16)
    return q, w, k


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--only", choices=["verifier", "trace", "approx"], default=None,
                    help="regenerate one fixture instead of all of them")
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    from temporal_dsa import certified, metrics, progressive_kernel as pk, replay, verifier_scoring
    from temporal_dsa.sidecar import LightningIndexerSidecar

    if args.only == "verifier":
        make_verifier(verifier_scoring)
        return
    if args.only == "trace":
        make_trace()
        return
    if args.only == "approx":
        make_approx()
        return

    # ---- dense scores (f32 and bf16) -------------------------------------------------
    out = {}
    lengths = [1, 17, 63, 64, 65, 127, 128, 129, 192, 256, 257]
    for length in lengths:
        q, w, k = cpu_inputs(length)
        out[f"f32_L{length}_keys"] = k.numpy()
        out[f"f32_L{length}_scores"] = pk.torch_full_scores(q, w, k).numpy()
    out["f32_q"], out["f32_w"] = q.numpy(), w.numpy()
    for length in lengths:
        q, w, k = bf16_inputs(length)
        out[f"bf16_L{length}_keys"] = bf16_bits(k)
        out[f"bf16_L{length}_scores"] = pk.torch_full_scores(q, w, k).numpy()
    out["bf16_q"], out["bf16_w"] = bf16_bits(q), w.numpy()

    # ---- head routing ------------------------------------------------------------------
    wt = torch.zeros(64)
    wt[20], wt[3] = -4, 4
    out["dyn_ties_w"] = wt.numpy()
    out["dyn_ties_ids"] = pk.dynamic_head_ids(wt).numpy()
    q, w, _ = cpu_inputs(1)
    out["dyn_rand_ids"] = pk.dynamic_head_ids(w).numpy()
    sel, rem = pk.split_head_ids(torch.tensor([0, 2, 4, 6, 8, 10, 12, 63]))
    out["split_sel"], out["split_rem"] = sel.numpy(), rem.numpy()

    # ---- torch_progressive_scores ------------------------------------------------------
    cases = []
    rng = np.random.default_rng(7)
    for length, bs in [(129, 64), (128, 64), (65, 64), (257, 32), (300, 128), (200, 16)]:
        q, w, k = cpu_inputs(length)
        heads = pk.dynamic_head_ids(w)
        nb = math.ceil(length / bs)
        direct = torch.from_numpy(rng.random(nb) < 0.3)
        probe = pk.torch_progressive_scores(q, w, k, heads, direct, math.inf, block_size=bs)[2]
        thr = float(torch.quantile(probe, 0.5))
        for tname, t in [("ninf", -math.inf), ("inf", math.inf), ("q50", thr)]:
            o, a, m = pk.torch_progressive_scores(q, w, k, heads, direct, t, block_size=bs)
            tag = f"prog_L{length}_B{bs}_{tname}"
            out[tag + "_direct"] = direct.numpy()
            out[tag + "_thr"] = np.float64(t)
            out[tag + "_scores"], out[tag + "_accepted"], out[tag + "_max"] = (
                o.numpy(), a.numpy(), m.numpy())
            cases.append(tag)
    out["prog_cases"] = np.array(cases)
    out["qkred"] = np.array([pk.progressive_qk_reduction(8192, 0, 0),
                             pk.progressive_qk_reduction(8192, 128, 0),
                             pk.progressive_qk_reduction(8192, 32, 16),
                             pk.progressive_qk_reduction(1000, 3, 5, block_size=128)])
    np.savez_compressed(HERE / "progressive_kernel.npz", **out)

    # ---- config 1 ----------------------------------------------------------------------
    q, w, k = cfg1_inputs()
    scores = pk.torch_full_scores(q, w, k)
    np.savez_compressed(
        HERE / "cfg1.npz", q=q.numpy(), w=w.numpy(),
        keys_sha256=np.array(hashlib.sha256(k.numpy().tobytes()).hexdigest()),
        scores=scores.numpy(), top512=metrics.stable_topk(scores.numpy(), 512),
        relu_index_f64=certified.relu_index_score(q.numpy(), k.numpy(), w.numpy()))

    # ---- stable_topk edge cases ----------------------------------------------------------
    tk = {}
    vectors = {
        "ties4": (np.array([1.0, 3.0, 3.0, 2.0], np.float32), [1, 2, 3, 4]),
        "ones64": (np.ones(64, np.float32), [1, 8, 63, 64]),
        "neg": (-np.arange(50, dtype=np.float32) % 7, [1, 5, 7, 49, 50]),
        "coarse": (np.round(rng.normal(size=3000) * 4).astype(np.float32), [1, 100, 512, 2999]),
        "ninf": (np.where(rng.random(400) < 0.5, -np.inf, rng.normal(size=400)).astype(np.float32),
                 [1, 150, 300, 400]),
        "signed_zero": (np.array([0.0, -0.0, 1.0, -0.0, 0.0, -1.0], np.float32), [1, 2, 3, 5]),
        "normal33k": (rng.normal(size=33000).astype(np.float32), [1, 2048, 4096]),
    }
    for name, (vec, ks) in vectors.items():
        tk[f"{name}_x"] = vec
        for kk in ks:
            tk[f"{name}_k{kk}"] = metrics.stable_topk(vec, kk)
    tk["names"] = np.array(list(vectors))
    np.savez_compressed(HERE / "topk.npz", **tk)

    # ---- certified bound -----------------------------------------------------------------
    r = np.random.default_rng(1582)
    keys = r.normal(size=(37, 8, 16))
    qp = r.normal(size=(8, 16))
    qc = qp + 0.05 * r.normal(size=(8, 16))
    wp = r.normal(size=8)
    wc = wp + 0.05 * r.normal(size=8)
    shared = keys[:, 0]
    rep = np.repeat(shared[:, None, :], 8, axis=1)
    norms = certified.block_key_norms(rep, 7)
    cert = dict(keys=keys, qp=qp, qc=qc, wp=wp, wc=wc, norms=norms,
                radius=certified.temporal_score_radius(qc, qp, wc, wp, norms),
                prev=certified.relu_index_score(qp, shared, wp),
                cur=certified.relu_index_score(qc, shared, wc),
                norms_full=certified.block_key_norms(keys, 5))
    # an indexer-shaped case: 64 heads x 128 dims, shared keys, AR(1) query
    g = torch.Generator().manual_seed(11)
    q0 = torch.randn(64, 128, generator=g) / math.sqrt(128)
    q1 = 0.95 * q0 + math.sqrt(1 - 0.95 ** 2) * torch.randn(64, 128, generator=g) / math.sqrt(128)
    w0 = torch.randn(64, generator=g) / 8
    w1 = w0 + 0.01 * torch.randn(64, generator=g)
    kk = torch.randn(300, 128, generator=g)
    n64 = certified.block_key_norms(np.repeat(kk.numpy()[:, None, :], 64, axis=1), 64)
    cert.update(iq0=q0.numpy(), iq1=q1.numpy(), iw0=w0.numpy(), iw1=w1.numpy(), ikeys=kk.numpy(),
                inorms=n64,
                iradius=certified.temporal_score_radius(q1.numpy(), q0.numpy(), w1.numpy(),
                                                        w0.numpy(), n64))
    np.savez_compressed(HERE / "certified.npz", **cert)

    # ---- replay filter -----------------------------------------------------------------
    rp = {}
    r4 = np.random.default_rng(4)
    prev = r4.normal(size=512)
    cur = np.concatenate([prev + 0.001 * r4.normal(size=512), [0.0]])
    r5 = np.random.default_rng(5)
    prev5 = r5.normal(size=257)
    cur5 = np.concatenate([r5.normal(size=257), [3.0]])
    prev6 = np.zeros(64)
    prev6[:4] = 2.0
    cur6 = prev6.copy()
    cur6[40:44] = 3.0
    rcases = [
        ("margin", prev, cur, 32, 16, 10.0, "dynamic", "previous_hot"),
        ("oracle", prev5, cur5, 16, 32, 0.0, "oracle", "oracle_current"),
        ("miss", prev6, cur6, 4, 8, 0.0, "dynamic", "previous_hot"),
        ("static", prev, cur, 32, 16, 1.0, "static", "address"),
        ("static_hot", prev, cur, 32, 16, 1.0, "static_hot_first", "previous_hot"),
        ("upper_hot", prev5, cur5, 16, 32, 2.0, "dynamic", "upper_hot"),
    ]
    for name, p, c, kk_, bs, gs, method, order in rcases:
        res = replay.replay_transition(p, c, k=kk_, block_size=bs, gamma_sigma=gs,
                                       method=method, scan_order=order)
        rp[f"{name}_prev"], rp[f"{name}_cur"] = p, c
        rp[f"{name}_meta"] = np.array([kk_, bs, gs])
        rp[f"{name}_method"], rp[f"{name}_order"] = np.array(method), np.array(order)
        rp[f"{name}_out"] = np.array([res.qk_scored, res.blocks_pruned, res.false_cold_blocks,
                                      res.recall, float(res.exact_match), res.tau_seed,
                                      res.net_byte_reduction])
    rp["names"] = np.array([c[0] for c in rcases])
    # certified-bound filter on indexer-shaped scores, through the reference's own filter
    prev_s = certified.relu_index_score(q0.numpy(), kk.numpy(), w0.numpy())
    cur_s = certified.relu_index_score(q1.numpy(), kk.numpy(), w1.numpy())
    for bs in (16, 32, 64):
        nb = math.ceil(300 / bs)
        nrm = certified.block_key_norms(np.repeat(kk.numpy()[:, None, :], 64, axis=1), bs)
        rad = certified.temporal_score_radius(q1.numpy(), q0.numpy(), w1.numpy(), w0.numpy(), nrm)
        pmax = np.array([prev_s[s : s + bs].max() for s in range(0, 300, bs)])
        upper = pmax + rad
        ptop = metrics.stable_topk(prev_s, 32)
        ttop = metrics.stable_topk(cur_s, 32)
        hot = np.zeros(nb, dtype=bool)
        hot[ptop // bs] = True
        order = replay._scan_order("previous_hot", upper, pmax, hot)
        res = replay._compiled_filter(cur_s, ptop.astype(np.int64), ttop.astype(np.int64), upper,
                                      order.astype(np.int64), bs, float(np.min(cur_s[ptop])), True)
        rp[f"cert_B{bs}_upper"] = upper
        rp[f"cert_B{bs}_out"] = np.array(res, dtype=np.float64)
    rp["cert_prev"], rp["cert_cur"] = prev_s, cur_s
    np.savez_compressed(HERE / "replay.npz", **rp)

    # ---- batched score_encoded + score_head_sparse ----------------------------------------
    g = torch.Generator().manual_seed(21)
    sq = torch.randn(2, 2, 64, 128, generator=g) / math.sqrt(128)
    sw = torch.randn(2, 2, 64, generator=g) / 8
    sk = torch.randn(2, 100, 128, generator=g)
    side = LightningIndexerSidecar.__new__(LightningIndexerSidecar)
    enc = LightningIndexerSidecar.score_encoded(side, sq, sw, sk, key_chunk_size=32)
    ids_fixed = torch.tensor([5, 1, 63, 7, 30, 2, 40, 9])
    ids_dyn = torch.stack([pk.dynamic_head_ids(sw[0, 0]), pk.dynamic_head_ids(sw[0, 1])]).long()
    hs_fixed = verifier_scoring.score_head_sparse(sq[0], sw[0], sk[0], ids_fixed,
                                                  key_chunk_size=37)
    hs_dyn = verifier_scoring.score_head_sparse(sq[0], sw[0], sk[0], ids_dyn, query_chunk_size=2)
    np.savez_compressed(HERE / "batched.npz", q=sq.numpy(), w=sw.numpy(), k=sk.numpy(),
                        encoded=enc.numpy(), ids_fixed=ids_fixed.numpy(),
                        ids_dyn=ids_dyn.numpy(), hs_fixed=hs_fixed.numpy(),
                        hs_dyn=hs_dyn.numpy())
    # ---- sidecar projection (encode_queries / encode_keys) -------------------------------
    torch.manual_seed(0)
    sc = LightningIndexerSidecar(hidden_size=16)
    with torch.no_grad():
        hq = torch.randn(2, 1, 16, generator=torch.Generator().manual_seed(31))
        qpos = torch.tensor([[3], [1000]])
        eq, ew = sc.encode_queries(hq, qpos)
        hk = torch.randn(1, 5, 16, generator=torch.Generator().manual_seed(32))
        ek = sc.encode_keys(hk, torch.arange(5).view(1, -1))
    np.savez_compressed(HERE / "sidecar.npz", wq=sc.wq.weight.detach().numpy(),
                        ww=sc.weights_proj.weight.detach().numpy(),
                        wk=sc.wk.weight.detach().numpy(), hq=hq.numpy(), qpos=qpos.numpy(),
                        q=eq.numpy(), w=ew.numpy(), hk=hk.numpy(), k=ek.numpy())
    make_verifier(verifier_scoring)
    make_trace()
    make_approx()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


def make_verifier(verifier_scoring) -> None:
    """verifier.npz: normalized_hadamard, fake_symmetric_quantize and score_dim_sparse
    (verifier_scoring.py:9-139) on seeded 64-head x 128-dim inputs."""
    g = torch.Generator().manual_seed(41)
    vq = torch.randn(2, 64, 128, generator=g) / math.sqrt(128)
    vw = torch.randn(2, 64, generator=g) / 8
    vk = torch.randn(160, 128, generator=g)
    dims = torch.tensor(sorted(torch.randperm(128, generator=g)[:32].tolist()))
    ver = {"q": vq.numpy(), "w": vw.numpy(), "k": vk.numpy(), "dims": dims.numpy()}
    ver["had_k"] = verifier_scoring.normalized_hadamard(vk).numpy()
    ver["had_q"] = verifier_scoring.normalized_hadamard(vq).numpy()
    for bits in (2, 4, 8):
        qk, sc = verifier_scoring.fake_symmetric_quantize(vk, bits)
        ver[f"fq{bits}_k"] = qk.numpy()
        ver[f"fq{bits}_scale"] = np.float64(sc)
    for rot in ("none", "hadamard"):
        for bits in (None, 4, 8):
            s = verifier_scoring.score_dim_sparse(vq, vw, vk, dims, rotation=rot, bits=bits)
            ver[f"ds_{rot}_{bits or 0}"] = s.numpy()
    s = verifier_scoring.score_dim_sparse(vq, vw, vk, dims, bits=4, query_scale=0.05,
                                          key_scale=0.5)
    ver["ds_none_4_fixed"] = s.numpy()
    qb, kb = vq.to(torch.bfloat16), vk.to(torch.bfloat16)
    ver["q_bf16"], ver["k_bf16"] = bf16_bits(qb), bf16_bits(kb)
    for rot in ("none", "hadamard"):
        s = verifier_scoring.score_dim_sparse(qb, vw, kb, dims, rotation=rot, bits=8)
        ver[f"dsb_{rot}_8"] = s.float().numpy()
    np.savez_compressed(HERE / "verifier.npz", **ver)


def trace_rows() -> tuple[list[np.ndarray], dict]:
    """Seeded float32 score rows of growing length for the trace fixture, with values that
    round to +-inf (65520 is the float16 halfway point above 65504), to float16 subnormals
    and to zero, plus the trace's identifying fields."""
    rng = np.random.default_rng(11)
    lengths = [5, 9, 12, 16]
    rows = [(rng.normal(size=n) * 3).astype(np.float32) for n in lengths]
    rows[1][:6] = [70000.0, -70000.0, 65520.0, 65519.0, 1e-8, 3e-6]
    rows[2][:3] = [1.0 / 3.0, -0.0, 2049.0]
    fields = {"layer": 7, "workload": "synthetic", "prompt_id": "seed11",
              "metadata": {"query_ids": [4, 8, 11, 15], "research_sidecar": True,
                           "source": None}}
    return rows, fields


def make_trace() -> None:
    """trace_rows.npz: the float32 rows; trace_ref.npz: those rows written by the reference's
    trace writer -- float16 rows padded with -inf to the widest (training.py:166-178),
    int32 lengths, saved by trace.save_trace (trace.py:34-48)."""
    from temporal_dsa.trace import ScoreTrace, save_trace

    rows, f = trace_rows()
    lengths = np.asarray([r.size for r in rows], dtype=np.int32)
    padded = np.full((len(rows), int(lengths.max())), -np.inf, dtype=np.float16)
    for i, r in enumerate(rows):
        padded[i, : r.size] = r.astype(np.float16)
    save_trace(HERE / "trace_ref.npz",
               ScoreTrace(scores=padded, lengths=lengths, layer=f["layer"],
                          workload=f["workload"], prompt_id=f["prompt_id"],
                          metadata=f["metadata"]))
    np.savez_compressed(HERE / "trace_rows.npz", rows=np.concatenate(rows), lengths=lengths)


def policy_trace(seed: int, steps: int = 7, length0: int = 1500, growth: int = 37):
    """A seeded decode-like score trace: every step appends `growth` keys; scores drift
    slowly (a persistent per-key level plus small noise) and a few regions jump, so blocks
    go hot and cold.  Returns float32 rows of increasing length."""
    rng = np.random.default_rng(seed)
    total = length0 + growth * (steps - 1)
    level = (rng.normal(size=total) * 1.5).astype(np.float32)
    rows = []
    for t in range(steps):
        length = length0 + growth * t
        row = level[:length] + (rng.normal(size=length) * 0.35).astype(np.float32)
        for _ in range(3):
            a = int(rng.integers(0, length - 80))
            row[a:a + 64] += np.float32(rng.uniform(1.5, 4.0))
        rows.append(row.astype(np.float32))
    return rows


APPROX_POLICIES = {
    # name: (ApproxPolicy keyword arguments, history_mode, block_size, fallback values)
    "static_addr": (dict(name="static", gamma=0.5), "own", 64, None),
    "dyn_addr": (dict(name="dynamic", gamma=0.25, dynamic_threshold=True), "own", 64, None),
    "dyn_prevmax": (dict(name="dynamic_pm", gamma=0.1, dynamic_threshold=True,
                         order="previous_max"), "own", 32, None),
    "dyn_bucket": (dict(name="bucket", gamma=0.2, dynamic_threshold=True, order="bucket8",
                        cold_streak=2), "own", 64, None),
    "ema_risk": (dict(name="ema", gamma=0.3, dynamic_threshold=True, order="predicted_risk",
                      risk_model="ema", ema_alpha=0.7, volatility_lambda=0.5, age_slope=0.05),
                 "own", 64, None),
    "refresh_age": (dict(name="refresh", gamma=0.0, refresh_interval=3, age_cap=2,
                         recent_window=100), "own", 128, None),
    "oracle_order": (dict(name="oracle", gamma=0.4, dynamic_threshold=True,
                          order="oracle_current"), "own", 16, None),
    "teacher": (dict(name="teacher", gamma=0.2, dynamic_threshold=True), "teacher", 64, None),
    "fallback": (dict(name="fallback", gamma=0.3, fallback_threshold=0.5), "own", 64,
                 [0.0, 0.1, 0.9, 0.2, 0.7, 0.0, 0.3]),
    "full": (dict(name="full"), "own", 64, None),
}


def make_approx() -> None:
    """approx.npz: approx.replay_step (approx.py:129-364) and verifier.verifier_step
    (verifier.py:173-375) run by the reference over seeded traces, per policy and step:
    the selection, the details, the next state and the counting metrics."""
    from temporal_dsa.approx import ApproxPolicy, initialize_state, replay_step
    from temporal_dsa.verifier import VerifierConfig, verifier_step

    k = 128
    out = {"k": np.int64(k)}
    metric_keys = ["qk_scored", "blocks_refreshed", "blocks_skipped", "exact_match", "recall",
                   "tau_seed", "tau_final", "full_refresh", "newly_hot_count",
                   "newly_hot_missed", "missed_count", "worst_missed_rank", "index_mass_ratio",
                   "top128_recall", "seed_blocks_touched", "physical_b16_blocks",
                   "physical_b128_blocks", "cache256_hbm_keys", "metadata_bytes",
                   "net_bf16_reduction"]
    out["metric_keys"] = np.array(metric_keys)
    for pi, (tag, (kw, mode, bs, fb)) in enumerate(APPROX_POLICIES.items()):
        rows = policy_trace(100 + pi)
        pol = ApproxPolicy(**kw)
        out[f"{tag}_bs"] = np.int64(bs)
        out[f"{tag}_mode"] = np.array(mode)
        for t, r in enumerate(rows):
            out[f"{tag}_s{t}_scores"] = r
        state = initialize_state(rows[0], k=k, block_size=bs)
        out[f"{tag}_s0_topk"] = state.topk
        out[f"{tag}_s0_cold"] = state.cold_streak
        for t in range(1, len(rows)):
            state, m, d = replay_step(state, rows[t], policy=pol, k=k, block_size=bs, step=t,
                                      history_mode=mode, previous_length=rows[t - 1].size,
                                      fallback_value=None if fb is None else fb[t])
            p = f"{tag}_s{t}_"
            for name in ("approximate", "baseline", "evaluated", "refreshed_blocks",
                         "skipped_blocks", "missed_ranks"):
                out[p + name] = d[name]
            for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
                out[p + name] = getattr(state, name)
            out[p + "metrics"] = np.array([float(m[key]) for key in metric_keys])
    # verifier_step: global-budget and fixed-threshold promotion over a dimension-sparse
    # stand-in for the verifier scores (the current scores plus noise)
    cfg = VerifierConfig(name="dimv", path="dim", width=32, score_ratio=0.25,
                         block_size=64, rescue_fraction=0.1)
    pol = ApproxPolicy(name="dynamic", gamma=0.2, dynamic_threshold=True)
    rows = policy_trace(300)
    rng = np.random.default_rng(301)
    for mode, thr in (("budget", None), ("thresh", 2.5)):
        state = initialize_state(rows[0], k=k, block_size=64)
        for t in range(1, len(rows)):
            vs = (rows[t] + rng.normal(size=rows[t].size) * 0.3).astype(np.float32)
            state, m, d = verifier_step(state, rows[t], vs, policy=pol, config=cfg, k=k, step=t,
                                        previous_length=rows[t - 1].size,
                                        promotion_threshold=thr)
            p = f"ver_{mode}_s{t}_"
            out[p + "vscores"] = vs
            for name in ("approximate", "rescued_blocks", "exact_candidates", "block_ranking"):
                out[p + name] = d[name]
            for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
                out[p + name] = getattr(state, name)
            out[p + "metrics"] = np.array([float(m[key]) for key in (
                "rescue_blocks", "rescue_exact_tokens", "candidate_union_tokens", "recall",
                "cold_blocks_scanned", "cold_tokens_scanned")])
    for t, r in enumerate(rows):
        out[f"ver_s{t}_scores"] = r
    np.savez_compressed(HERE / "approx.npz", **out)


if __name__ == "__main__":
    main()
