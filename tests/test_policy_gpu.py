"""GPU parity of the temporal policy state machine (tdsa_policy_init / tdsa_policy_step).

The device replay_step / verifier_step (dsa_b200.approx, dsa_b200.verifier) are run over
the seeded traces of ``tests/golden/approx.npz`` -- which the reference's own
approx.replay_step (approx.py:129-364) and verifier.verifier_step (verifier.py:173-375)
produced -- and must reproduce every step exactly: the selection, the details, the next
state (float32 arrays bit for bit) and the counting metrics.  The batched PolicyPlan and
config-scale rows are checked against the oracle restatement (oracle/approx.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import approx as oa
from tests.conftest import load_golden
from tests.test_approx_oracle import FALLBACK, POLICIES, policy_args, steps_of

pytestmark = pytest.mark.gpu
G = load_golden("approx")


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()
    yield
    from dsa_b200 import device_status

    assert device_status() == 0


def _policy(tag):
    from dsa_b200.approx import ApproxPolicy

    ns = policy_args(tag)
    return ApproxPolicy(**vars(ns))


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("tag", POLICIES)
def test_device_replay_matches_reference(tag):
    from dsa_b200.approx import initialize_state, replay_step

    k, bs, mode = int(G["k"]), int(G[f"{tag}_bs"]), str(G[f"{tag}_mode"])
    pol = _policy(tag)
    keys = [str(x) for x in G["metric_keys"]]
    rows = [torch.from_numpy(G[f"{tag}_s{t}_scores"]).cuda()
            for t in range(steps_of(f"{tag}_s"))]
    state = initialize_state(rows[0], k=k, block_size=bs)
    np.testing.assert_array_equal(_np(state.topk), G[f"{tag}_s0_topk"])
    np.testing.assert_array_equal(_np(state.cold_streak), G[f"{tag}_s0_cold"])
    fb = FALLBACK.get(tag)
    for t in range(1, len(rows)):
        state, m, d = replay_step(state, rows[t], policy=pol, k=k, block_size=bs, step=t,
                                  history_mode=mode, previous_length=rows[t - 1].numel(),
                                  fallback_value=None if fb is None else fb[t])
        p = f"{tag}_s{t}_"
        for name in ("approximate", "baseline", "evaluated", "refreshed_blocks",
                     "skipped_blocks", "missed_ranks"):
            np.testing.assert_array_equal(_np(d[name]), G[p + name], err_msg=p + name)
        for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
            got, want = _np(getattr(state, name)), G[p + name]
            assert got.dtype == want.dtype, name
            np.testing.assert_array_equal(got, want, err_msg=p + name)
        want = dict(zip(keys, G[p + "metrics"]))
        for key in keys:
            tol = 1e-9 if key == "index_mass_ratio" else 0.0
            assert abs(float(m[key]) - want[key]) <= tol * max(1.0, abs(want[key])), (p, key,
                                                                                    m[key])


@pytest.mark.parametrize("mode,thr", [("budget", None), ("thresh", 2.5)])
def test_device_verifier_matches_reference(mode, thr):
    from dsa_b200.approx import ApproxPolicy, initialize_state
    from dsa_b200.verifier import VerifierConfig, verifier_step

    k = int(G["k"])
    pol = ApproxPolicy(name="dynamic", gamma=0.2, dynamic_threshold=True)
    cfg = VerifierConfig(name="dimv", path="dim", width=32, score_ratio=0.25, block_size=64,
                         rescue_fraction=0.1)
    rows = [torch.from_numpy(G[f"ver_s{t}_scores"]).cuda() for t in range(steps_of("ver_s"))]
    state = initialize_state(rows[0], k=k, block_size=64)
    for t in range(1, len(rows)):
        p = f"ver_{mode}_s{t}_"
        vs = torch.from_numpy(G[p + "vscores"]).cuda()
        state, m, d = verifier_step(state, rows[t], vs, policy=pol, config=cfg, k=k, step=t,
                                    previous_length=rows[t - 1].numel(),
                                    promotion_threshold=thr)
        for name in ("approximate", "rescued_blocks", "exact_candidates", "block_ranking"):
            np.testing.assert_array_equal(_np(d[name]), G[p + name], err_msg=p + name)
        for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
            np.testing.assert_array_equal(_np(getattr(state, name)), G[p + name],
                                          err_msg=p + name)
        got = [m["rescue_blocks"], m["rescue_exact_tokens"], m["candidate_union_tokens"],
               m["recall"], m["cold_blocks_scanned"], m["cold_tokens_scanned"]]
        np.testing.assert_array_equal(np.asarray(got, np.float64), G[p + "metrics"])


def _drift_rows(seed, steps, length0, growth):
    rng = np.random.default_rng(seed)
    total = length0 + growth * steps
    level = (rng.normal(size=total) * 1.5).astype(np.float32)
    rows = []
    for t in range(steps):
        n = length0 + growth * t
        row = level[:n] + (rng.normal(size=n) * 0.35).astype(np.float32)
        a = int(rng.integers(0, n - 200))
        row[a:a + 128] += np.float32(2.5)
        rows.append(row.astype(np.float32))
    return rows


@pytest.mark.parametrize("tag", ["dyn_addr", "dyn_prevmax", "ema_risk", "static_addr"])
def test_policy_plan_batch_matches_oracle(tag):
    """Three sequences in one PolicyPlan (one CTA each), checked per sequence against the
    oracle over five steps at L ~ 4-5K, k = 256."""
    from dsa_b200.approx import PolicyPlan

    k, bs, batch, steps = 256, 32 if tag == "dyn_prevmax" else 64, 3, 5
    pol_ns = policy_args(tag)
    pol = _policy(tag)
    seqs = [_drift_rows(40 + b, steps, 4000, 50) for b in range(batch)]
    plan = PolicyPlan(batch, 4000 + 50 * steps, k, bs, "cuda")
    plan.init(torch.from_numpy(np.stack([s[0] for s in seqs])).cuda())
    states = [oa.initialize_state(s[0], k=k, block_size=bs) for s in seqs]
    for t in range(1, steps):
        x = torch.from_numpy(np.stack([s[t] for s in seqs])).cuda()
        sel = plan.step(x, pol, step=t, previous_length=seqs[0][t - 1].size)
        stats = plan.stats_host()
        for b in range(batch):
            states[b], m, d = oa.replay_step(states[b], seqs[b][t], policy=pol_ns, k=k,
                                             block_size=bs, step=t,
                                             previous_length=seqs[b][t - 1].size)
            np.testing.assert_array_equal(_np(sel[b]), d["approximate"])
            nb = d["refreshed_blocks"].size + d["skipped_blocks"].size
            for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
                np.testing.assert_array_equal(_np(plan.block_view(name)[b, :nb]),
                                              getattr(states[b], name), err_msg=name)
            assert stats[b]["SCORED"] == m["qk_scored"]
            assert stats[b]["REFRESHED"] == m["blocks_refreshed"]


def test_policy_config_scale_matches_oracle():
    """L = 32768 + growth, k = 2048, block 64, dynamic threshold in address order (the
    reference's default family at its headline K)."""
    from dsa_b200.approx import PolicyPlan

    k, bs = 2048, 64
    pol_ns = policy_args("dyn_addr")
    pol = _policy("dyn_addr")
    rows = _drift_rows(77, 3, 32768, 64)
    plan = PolicyPlan(1, 32768 + 64 * 3, k, bs, "cuda")
    plan.init(torch.from_numpy(rows[0]).cuda())
    state = oa.initialize_state(rows[0], k=k, block_size=bs)
    for t in range(1, 3):
        sel = plan.step(torch.from_numpy(rows[t]).cuda(), pol, step=t,
                        previous_length=rows[t - 1].size)
        state, m, d = oa.replay_step(state, rows[t], policy=pol_ns, k=k, block_size=bs,
                                     step=t, previous_length=rows[t - 1].size)
        np.testing.assert_array_equal(_np(sel[0]), d["approximate"])
        assert plan.stats_host()[0]["SCORED"] == m["qk_scored"]


def test_policy_rejects_bad_seed_and_arguments():
    from dsa_b200.approx import ApproxPolicy, PolicyPlan, initialize_state, replay_step

    rows = _drift_rows(5, 2, 3000, 0)
    state = initialize_state(torch.from_numpy(rows[0]).cuda(), k=64, block_size=64)
    pol = ApproxPolicy(name="x")
    # the seed holds keys beyond a shorter row: the reference raises RuntimeError
    short = torch.from_numpy(rows[1][:1000]).cuda()
    from dsa_b200 import device_status

    with pytest.raises(RuntimeError, match="seed"):
        replay_step(state, short, policy=pol, k=64, block_size=64, step=1)
    device_status(reset=True)
    with pytest.raises(ValueError, match="unknown block order"):
        replay_step(state, torch.from_numpy(rows[1]).cuda(),
                    policy=ApproxPolicy(name="x", order="sideways"), k=64, block_size=64, step=1)
    with pytest.raises(ValueError, match="history_mode"):
        replay_step(state, torch.from_numpy(rows[1]).cuda(), policy=pol, k=64, block_size=64,
                    step=1, history_mode="mixed")
    from dsa_b200 import _capi as capi

    with pytest.raises(capi.TdsaError, match="length <= 131072"):
        PolicyPlan(1, 200000, 64, 64, "cuda").init(torch.zeros(200000, device="cuda"))
