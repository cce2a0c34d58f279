"""The temporal policy oracle (oracle/approx.py) against the reference's own outputs.

``tests/golden/approx.npz`` holds, per policy and decode step, what the reference's
``approx.replay_step`` (approx.py:129-364) and ``verifier.verifier_step``
(verifier.py:173-375) returned on seeded traces: the selection, details, next state and
counting metrics.  Everything here must match exactly (float32 state bit for bit); the
index-mass ratio to 1e-12.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from oracle import approx as oa
from tests.conftest import load_golden

G = load_golden("approx")
POLICIES = ["static_addr", "dyn_addr", "dyn_prevmax", "dyn_bucket", "ema_risk", "refresh_age",
            "oracle_order", "teacher", "fallback", "full"]
FALLBACK = {"fallback": [0.0, 0.1, 0.9, 0.2, 0.7, 0.0, 0.3]}


def policy_args(tag: str) -> SimpleNamespace:
    """The ApproxPolicy fields of each golden case (defaults of approx.py:15-39)."""
    base = dict(name=tag, gamma=0.0, cold_streak=1, dynamic_threshold=False, order="address",
                refresh_interval=None, age_cap=None, recent_window=0, risk_model="last_max",
                ema_alpha=0.9, volatility_lambda=0.0, age_slope=0.0, fallback_threshold=None)
    kw = {
        "static_addr": dict(name="static", gamma=0.5),
        "dyn_addr": dict(name="dynamic", gamma=0.25, dynamic_threshold=True),
        "dyn_prevmax": dict(name="dynamic_pm", gamma=0.1, dynamic_threshold=True,
                            order="previous_max"),
        "dyn_bucket": dict(name="bucket", gamma=0.2, dynamic_threshold=True, order="bucket8",
                           cold_streak=2),
        "ema_risk": dict(name="ema", gamma=0.3, dynamic_threshold=True, order="predicted_risk",
                         risk_model="ema", ema_alpha=0.7, volatility_lambda=0.5,
                         age_slope=0.05),
        "refresh_age": dict(name="refresh", gamma=0.0, refresh_interval=3, age_cap=2,
                            recent_window=100),
        "oracle_order": dict(name="oracle", gamma=0.4, dynamic_threshold=True,
                             order="oracle_current"),
        "teacher": dict(name="teacher", gamma=0.2, dynamic_threshold=True),
        "fallback": dict(name="fallback", gamma=0.3, fallback_threshold=0.5),
        "full": dict(name="full"),
    }[tag]
    base.update(kw)
    return SimpleNamespace(**base)


def steps_of(prefix: str) -> int:
    return sum(1 for name in G.files if name.startswith(prefix) and name.endswith("_scores"))


@pytest.mark.parametrize("tag", POLICIES)
def test_replay_step_matches_reference(tag):
    k, bs, mode = int(G["k"]), int(G[f"{tag}_bs"]), str(G[f"{tag}_mode"])
    pol = policy_args(tag)
    keys = [str(x) for x in G["metric_keys"]]
    rows = [G[f"{tag}_s{t}_scores"] for t in range(steps_of(f"{tag}_s"))]
    state = oa.initialize_state(rows[0], k=k, block_size=bs)
    np.testing.assert_array_equal(state.topk, G[f"{tag}_s0_topk"])
    np.testing.assert_array_equal(state.cold_streak, G[f"{tag}_s0_cold"])
    fb = FALLBACK.get(tag)
    for t in range(1, len(rows)):
        state, m, d = oa.replay_step(state, rows[t], policy=pol, k=k, block_size=bs, step=t,
                                     history_mode=mode, previous_length=rows[t - 1].size,
                                     fallback_value=None if fb is None else fb[t])
        p = f"{tag}_s{t}_"
        for name in ("approximate", "baseline", "evaluated", "refreshed_blocks",
                     "skipped_blocks", "missed_ranks"):
            np.testing.assert_array_equal(d[name], G[p + name], err_msg=f"{p}{name}")
        for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
            got, want = getattr(state, name), G[p + name]
            assert got.dtype == want.dtype, name
            np.testing.assert_array_equal(got, want, err_msg=f"{p}{name}")
        want = dict(zip(keys, G[p + "metrics"]))
        for key in keys:
            tol = 1e-12 if key == "index_mass_ratio" else 0.0
            assert abs(float(m[key]) - want[key]) <= tol * max(1.0, abs(want[key])), (p, key)


@pytest.mark.parametrize("mode,thr", [("budget", None), ("thresh", 2.5)])
def test_verifier_step_matches_reference(mode, thr):
    k = int(G["k"])
    pol = policy_args("dyn_addr")
    pol.name, pol.gamma = "dynamic", 0.2
    cfg = SimpleNamespace(block_size=64, rescue_fraction=0.1)
    rows = [G[f"ver_s{t}_scores"] for t in range(steps_of("ver_s"))]
    state = oa.initialize_state(rows[0], k=k, block_size=64)
    for t in range(1, len(rows)):
        p = f"ver_{mode}_s{t}_"
        state, m, d = oa.verifier_step(state, rows[t], G[p + "vscores"], policy=pol, config=cfg,
                                       k=k, step=t, previous_length=rows[t - 1].size,
                                       promotion_threshold=thr)
        for name in ("approximate", "rescued_blocks", "exact_candidates", "block_ranking"):
            np.testing.assert_array_equal(d[name], G[p + name], err_msg=f"{p}{name}")
        for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
            np.testing.assert_array_equal(getattr(state, name), G[p + name], err_msg=p + name)
        want = G[p + "metrics"]
        got = [m["rescue_blocks"], m["rescue_exact_tokens"], m["candidate_union_tokens"],
               m["recall"], m["cold_blocks_scanned"], m["cold_tokens_scanned"]]
        np.testing.assert_array_equal(np.asarray(got, np.float64), want)
