"""Numpy restatement of the reference's temporal policy state machine (test oracle).

Reference (paths under ``src/temporal_dsa/``):

* ``approx.py`` -- ``ApproxPolicy`` (:15-39), ``ApproxState`` (:42-50), ``_block_max``
  (:53-55), ``_order_blocks`` (:92-109), ``initialize_state`` (:112-126), ``replay_step``
  (:129-364);
* ``verifier.py`` -- ``_block_max_masked`` (:52-65), ``_rank_blocks`` (:68-73),
  ``apply_rescue_to_state`` (:103-170), ``verifier_step`` (:173-375).

One decode step of the policy: the previous step's top-k (``seed``) is scored first and
its minimum is ``tau_seed``.  Blocks are visited in the policy's order; a block is read
("refreshed") when it is forced (full refresh, new or recent keys, age cap, short cold
streak) or when its risk (``last_max`` or ``ema`` plus margins) is not below the
threshold -- ``tau_seed``, or with ``dynamic_threshold`` the running k-th score of
everything read so far.  The result is the stable top-k of the keys read; only refreshed
blocks update their metadata (``last_max``/``ema``/``volatility``, ``age`` reset), the
others age.  The verifier step then rescues cold blocks by a cheaper score and reranks.

The running k-th score is kept here as a k-item set re-selected with ``np.lexsort`` per
block (the reference keeps a heap); both hold the top-k of (seed + refreshed keys) under
the order (score descending, index ascending), so the thresholds agree.

Test infrastructure only: the device implementation is checked against this file, and
this file against the reference's own outputs (``tests/golden/approx.npz``).
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np

from .topk import stable_topk

I16_MAX = 32767


def block_max(values, block_size: int) -> np.ndarray:
    """approx.py:53-55 -- per-block maximum (float32); the last block may be ragged."""
    v = np.asarray(values, dtype=np.float32)
    nb = (v.size + block_size - 1) // block_size
    pad = np.full(nb * block_size, -np.inf, dtype=np.float32)
    pad[: v.size] = v
    return pad.reshape(nb, block_size).max(axis=1)


def extend(values, size: int, fill) -> np.ndarray:
    """approx.py:58-61 -- truncate or pad with `fill` to `size` entries."""
    v = np.asarray(values)
    if v.size >= size:
        return v[:size].copy()
    out = np.full(size, fill, dtype=np.result_type(v.dtype, np.asarray(fill).dtype))
    out[: v.size] = v
    return out.astype(v.dtype)


def initialize_state(scores, *, k: int, block_size: int) -> SimpleNamespace:
    """approx.py:112-126."""
    s = np.asarray(scores, dtype=np.float32)
    top = stable_topk(s, k)
    maxima = block_max(s, block_size)
    cold = np.ones(maxima.size, dtype=np.int16)
    cold[top // block_size] = 0
    return SimpleNamespace(topk=top, baseline_topk=top.copy(), last_max=maxima,
                           ema=maxima.copy(), volatility=np.zeros(maxima.size, np.float32),
                           age=np.zeros(maxima.size, np.int16), cold_streak=cold)


def policy_risk(policy, last_max, ema, volatility, age) -> np.ndarray:
    """approx.py:186-198 -- float64 risk per block, summed left to right.  The reference's
    ``volatility_lambda * volatility`` multiplies a float32 array by a Python float, which
    NumPy 2 evaluates in float32; ``age_slope * age`` (int16 array) is float64."""
    slope = policy.age_slope * age.astype(np.float64)
    if policy.risk_model == "last_max":
        return last_max.astype(np.float64) + policy.gamma + slope
    if policy.risk_model == "ema":
        spread = (np.float32(policy.volatility_lambda) * volatility.astype(np.float32))
        return ema.astype(np.float64) + spread.astype(np.float64) + policy.gamma + slope
    raise ValueError(f"unknown risk model: {policy.risk_model}")


def _desc_then_address(values) -> np.ndarray:
    """Block ids by value descending (NaN as -inf), ties by ascending address."""
    v = np.nan_to_num(np.asarray(values, dtype=np.float64), nan=-np.inf)
    return np.lexsort((np.arange(v.size), -v))


def block_order(policy, risk, current_max) -> np.ndarray:
    """approx.py:92-109 and :200-204 -- the visiting order of the blocks."""
    nb = risk.size
    if policy.order == "address":
        return np.arange(nb)
    if policy.order in ("previous_max", "predicted_risk"):
        return _desc_then_address(risk)
    if policy.order.startswith("bucket"):
        buckets = int(policy.order[len("bucket"):])
        rank = np.empty(nb, dtype=np.int64)
        rank[_desc_then_address(risk)] = np.arange(nb)
        bucket = np.minimum(buckets - 1, rank * buckets // max(1, nb))
        return np.lexsort((np.arange(nb), bucket))
    if policy.order == "oracle_current":
        return np.lexsort((np.arange(nb), -np.asarray(current_max, np.float64)))
    raise ValueError(f"unknown block order: {policy.order}")


def _top_items(keys: np.ndarray, scores: np.ndarray, k: int) -> np.ndarray:
    """The k best keys under (score descending, index ascending), best first."""
    order = np.lexsort((keys, -scores[keys].astype(np.float64)))
    return keys[order[:k]]


def _vol_update(a: float, obs: float, mean: float, vol) -> np.float32:
    """approx.py:283-286 / verifier.py:155-158: ``a * |obs - mean| + (1 - a) * vol`` with
    ``vol`` a numpy float32 scalar and the rest Python floats.  NumPy 2 promotion makes the
    second product and the sum float32 operations: float32(1 - a) * vol, then
    float32(a * |obs - mean|) + that, each rounded to float32."""
    second = np.float32(1.0 - a) * np.float32(vol)
    return np.float32(np.float32(a * abs(obs - mean)) + second)


def _full_refresh(policy, step: int, fallback_value) -> tuple[bool, bool]:
    fallback = (policy.fallback_threshold is not None and fallback_value is not None
                and fallback_value > policy.fallback_threshold)
    full = bool(policy.name == "full"
                or (policy.refresh_interval and step % policy.refresh_interval == 0)
                or fallback)
    return full, bool(fallback)


def _metadata_bytes_per_block(policy) -> int:
    """approx.py:84-89."""
    raw = 6 + (1 if policy.order.startswith("bucket") else 0) + (8 if policy.risk_model == "ema"
                                                                 else 0)
    return int(math.ceil(raw / 4) * 4)


def _retention(approximate, ranked_baseline, count: int) -> float:
    count = min(count, ranked_baseline.size)
    if count == 0:
        return 1.0
    return float(np.isin(ranked_baseline[:count], approximate).sum() / count)


def _mass_ratio(scores, approximate, baseline) -> float:
    shift = float(np.max(scores[baseline]))
    num = np.exp(scores[approximate].astype(np.float64) - shift).sum()
    den = np.exp(scores[baseline].astype(np.float64) - shift).sum()
    return float(num / max(den, 1e-300))


def replay_step(state, current_scores, *, policy, k: int, block_size: int, step: int,
                history_mode: str = "own", previous_length=None, fallback_value=None):
    """approx.py:129-364 -> (next_state, metrics, details)."""
    if history_mode not in ("own", "teacher"):
        raise ValueError("history_mode must be 'own' or 'teacher'")
    s = np.asarray(current_scores, dtype=np.float32)
    length = s.size
    if k > length:
        raise ValueError("K cannot exceed the current trace length")
    prev_len = length if previous_length is None else int(previous_length)
    nb = (length + block_size - 1) // block_size
    last_max = extend(state.last_max, nb, -np.inf).astype(np.float32)
    ema = extend(state.ema, nb, -np.inf).astype(np.float32)
    vol = extend(state.volatility, nb, 0.0).astype(np.float32)
    age = extend(state.age, nb, 0).astype(np.int16)
    cold = extend(state.cold_streak, nb, 1).astype(np.int16)

    baseline = stable_topk(s, k)
    seed_src = state.baseline_topk if history_mode == "teacher" else state.topk
    seed = np.asarray(seed_src, dtype=np.int64)
    seed = seed[seed < length]
    if seed.size != k or np.unique(seed).size != k:
        raise RuntimeError(f"previous Top-K seed has {seed.size} unique keys, expected {k}")
    tau_seed = float(np.min(s[seed]))
    full, fallback = _full_refresh(policy, step, fallback_value)

    current_max = block_max(s, block_size)
    risk = policy_risk(policy, last_max, ema, vol, age)
    order = block_order(policy, risk, current_max)
    new_block = np.zeros(nb, bool)
    if prev_len < length:
        new_block[prev_len // block_size:] = True
    recent = np.zeros(nb, bool)
    if policy.recent_window:
        recent[max(0, length - policy.recent_window) // block_size:] = True
    forced = full | new_block | recent | (cold < policy.cold_streak)
    if policy.age_cap is not None:
        forced |= age >= policy.age_cap

    evaluated = np.zeros(length, bool)
    evaluated[seed] = True
    refreshed = np.zeros(nb, bool)
    threshold = tau_seed
    running = _top_items(seed, s, k) if policy.dynamic_threshold else None
    for b in order:
        if not forced[b] and risk[b] < threshold:
            continue
        lo, hi = b * block_size, min(length, (b + 1) * block_size)
        unseen = lo + np.flatnonzero(~evaluated[lo:hi])
        evaluated[lo:hi] = True
        refreshed[b] = True
        if running is not None and unseen.size:
            running = _top_items(np.concatenate((running, unseen)), s, k)
            threshold = float(s[running[-1]])
    skipped = ~refreshed
    scored = np.flatnonzero(evaluated)
    if scored.size < k:
        raise RuntimeError(f"policy scored {scored.size} keys, fewer than K={k}")
    approximate = running if running is not None else scored[stable_topk(s[scored], k)]

    # metadata of refreshed blocks only (own mode); teacher mode observes every block
    new_last, new_ema, new_vol = last_max.copy(), ema.copy(), vol.copy()
    new_age = np.minimum(age.astype(np.int32) + 1, I16_MAX).astype(np.int16)
    a = float(policy.ema_alpha)
    for b in np.flatnonzero(refreshed):
        obs = float(current_max[b])
        mean = float(ema[b]) if np.isfinite(ema[b]) else obs
        new_last[b] = obs
        new_ema[b] = a * obs + (1.0 - a) * mean
        new_vol[b] = _vol_update(a, obs, mean, vol[b])
        new_age[b] = 0
    if history_mode == "teacher":
        new_last, new_ema = current_max.copy(), current_max.copy()
        new_vol[:] = 0.0
        new_age[:] = 0
    hot = np.zeros(nb, bool)
    hot[(baseline if history_mode == "teacher" else approximate) // block_size] = True
    next_cold = np.where(hot, 0, np.minimum(cold.astype(np.int32) + 1, I16_MAX)).astype(np.int16)
    nxt = SimpleNamespace(topk=approximate, baseline_topk=baseline, last_max=new_last,
                          ema=new_ema, volatility=new_vol, age=new_age, cold_streak=next_cold)

    in_approx = np.zeros(length, bool)
    in_approx[approximate] = True
    newly_hot = np.setdiff1d(baseline, state.baseline_topk)
    missed_rank = np.flatnonzero(~in_approx[baseline]) + 1
    mbpb = _metadata_bytes_per_block(policy)
    mbytes = nb * mbpb
    m = {
        "step": step, "context_length": length, "history_mode": history_mode,
        "policy": policy.name, "gamma": policy.gamma, "k": k, "block_size": block_size,
        "qk_scored": int(scored.size), "qk_reduction": float(1.0 - scored.size / length),
        "exact_match": bool(np.array_equal(np.sort(approximate), np.sort(baseline))),
        "recall": float(in_approx[baseline].sum() / k),
        "index_mass_ratio": _mass_ratio(s, approximate, baseline),
        "newly_hot_count": int(newly_hot.size),
        "newly_hot_missed": int((~in_approx[newly_hot]).sum()) if newly_hot.size else 0,
        "missed_count": int(missed_rank.size),
        "worst_missed_rank": int(missed_rank.min()) if missed_rank.size else 0,
        "tau_seed": tau_seed, "tau_final": float(np.min(s[approximate])),
        "full_refresh": full, "fallback": fallback,
        "blocks_refreshed": int(refreshed.sum()), "blocks_skipped": int(skipped.sum()),
        "metadata_bytes_per_block": mbpb, "metadata_bytes": mbytes,
        "ideal_bf16_bytes": int(scored.size * 256 + mbytes),
        "ideal_fp8_bytes": int(scored.size * 128 + mbytes),
        "net_bf16_reduction": float(1.0 - (scored.size * 256 + mbytes) / (length * 256)),
        "net_fp8_reduction": float(1.0 - (scored.size * 128 + mbytes) / (length * 128)),
    }
    for n in (128, 256, 512, 1024, 2048):
        m[f"top{n}_recall"] = _retention(approximate, baseline, n)
    m["newly_hot_miss_rate"] = (float(m["newly_hot_missed"] / newly_hot.size)
                                if newly_hot.size else 0.0)
    seed_blocks = np.unique(seed // block_size).size
    m["seed_blocks_touched"] = int(seed_blocks)
    m["seed_block_fraction"] = float(seed_blocks / nb)
    for pb in (16, 32, 64, 128):
        touched = np.unique(scored // pb).size
        m[f"physical_b{pb}_blocks"] = int(touched)
        m[f"physical_b{pb}_reduction"] = float(1.0 - touched / ((length + pb - 1) // pb))
    for c in (0, 256, 512, 1024, 2048):
        uncached = evaluated.copy()
        uncached[seed[: min(c, seed.size)]] = False
        keys = int(uncached.sum())
        m[f"cache{c}_hbm_keys"] = keys
        m[f"cache{c}_net_bf16_reduction"] = float(1.0 - (keys * 256 + mbytes) / (length * 256))
    details = {"approximate": approximate, "baseline": baseline, "evaluated": scored,
               "seed": seed.copy(), "refreshed_blocks": np.flatnonzero(refreshed).astype(np.int32),
               "skipped_blocks": np.flatnonzero(skipped).astype(np.int32),
               "missed_ranks": missed_rank.astype(np.int32)}
    return nxt, m, details


# ------------------------------------------------------------------------------ verifier
def block_max_masked(values, available, block_size: int):
    """verifier.py:52-65 -- max of the available entries per block, and which blocks have
    any (-inf and False elsewhere)."""
    v = np.where(np.asarray(available, bool), np.asarray(values, np.float32), -np.inf)
    nb = (v.size + block_size - 1) // block_size
    avail = np.zeros(nb * block_size, bool)
    avail[: v.size] = available
    maxima = block_max(v, block_size)
    has = avail.reshape(nb, block_size).any(axis=1)
    return np.where(has, maxima, -np.inf).astype(np.float32), has


def rank_blocks(block_scores, eligible) -> np.ndarray:
    """verifier.py:68-73 -- eligible blocks by score descending, address ascending."""
    ids = np.flatnonzero(eligible)
    return ids[np.lexsort((ids, -np.asarray(block_scores, np.float64)[ids]))].astype(np.int64)


def apply_rescue(previous, temporal_next, scores, evaluated, rescued, *, policy, k: int,
                 block_size: int):
    """verifier.py:103-170 -> (state, approximate, exact_ids)."""
    s = np.asarray(scores, dtype=np.float32)
    exact = np.zeros(s.size, bool)
    exact[np.asarray(evaluated, np.int64)] = True
    for b in np.asarray(rescued, np.int64):
        exact[b * block_size: min(s.size, (b + 1) * block_size)] = True
    ids = np.flatnonzero(exact)
    if ids.size < k:
        raise RuntimeError(f"candidate union has {ids.size} keys, fewer than K={k}")
    approximate = ids[stable_topk(s[ids], k)]
    nb = (s.size + block_size - 1) // block_size
    last_max = extend(temporal_next.last_max, nb, -np.inf).astype(np.float32)
    ema = extend(temporal_next.ema, nb, -np.inf).astype(np.float32)
    vol = extend(temporal_next.volatility, nb, 0.0).astype(np.float32)
    age = extend(temporal_next.age, nb, 0).astype(np.int16)
    p_ema = extend(previous.ema, nb, -np.inf).astype(np.float32)
    p_vol = extend(previous.volatility, nb, 0.0).astype(np.float32)
    p_cold = extend(previous.cold_streak, nb, 1).astype(np.int16)
    a = float(policy.ema_alpha)
    for b in np.asarray(rescued, np.int64):
        obs = float(np.max(s[b * block_size: min(s.size, (b + 1) * block_size)]))
        mean = float(p_ema[b]) if np.isfinite(p_ema[b]) else obs
        last_max[b] = obs
        ema[b] = a * obs + (1.0 - a) * mean
        vol[b] = _vol_update(a, obs, mean, p_vol[b])
        age[b] = 0
    hot = np.zeros(nb, bool)
    hot[approximate // block_size] = True
    cold = np.where(hot, 0, np.minimum(p_cold.astype(np.int32) + 1, I16_MAX)).astype(np.int16)
    st = SimpleNamespace(topk=approximate, baseline_topk=temporal_next.baseline_topk,
                         last_max=last_max, ema=ema, volatility=vol, age=age, cold_streak=cold)
    return st, approximate, ids


def verifier_step(state, current_scores, verifier_scores, *, policy, config, k: int, step: int,
                  previous_length=None, promotion_threshold=None):
    """verifier.py:173-375 (the selection, state and the counting metrics) ->
    (state, metrics, details)."""
    s = np.asarray(current_scores, dtype=np.float32)
    vs = np.asarray(verifier_scores[: s.size], dtype=np.float32)
    if vs.shape != s.shape:
        raise ValueError("verifier score length must match current score length")
    t_next, _, t_det = replay_step(state, s, policy=policy, k=k, block_size=config.block_size,
                                   step=step, history_mode="own",
                                   previous_length=previous_length)
    cold_mask = np.ones(s.size, bool)
    cold_mask[t_det["evaluated"]] = False
    block_scores, cold_blocks = block_max_masked(vs, cold_mask, config.block_size)
    ranking = rank_blocks(block_scores, cold_blocks)
    if promotion_threshold is None:
        count = min(ranking.size, int(math.ceil(config.rescue_fraction * int(cold_blocks.sum()))))
        rescued = ranking[:count]
    else:
        rescued = ranking[block_scores[ranking] >= float(promotion_threshold)]
    nxt, approximate, exact_ids = apply_rescue(state, t_next, s, t_det["evaluated"], rescued,
                                               policy=policy, k=k,
                                               block_size=config.block_size)
    baseline = t_det["baseline"]
    in_approx = np.zeros(s.size, bool)
    in_approx[approximate] = True
    temporal_exact = int(t_det["evaluated"].size)
    m = {
        "temporal_exact_tokens": temporal_exact,
        "cold_tokens_scanned": int(cold_mask.sum()),
        "cold_blocks_scanned": int(cold_blocks.sum()),
        "rescue_blocks": int(rescued.size),
        "rescue_exact_tokens": int(exact_ids.size - temporal_exact),
        "candidate_union_tokens": int(exact_ids.size),
        "exact_match": bool(np.array_equal(np.sort(approximate), np.sort(baseline))),
        "recall": float(in_approx[baseline].sum() / k),
        "index_mass_ratio": _mass_ratio(s, approximate, baseline),
    }
    details = {"approximate": approximate, "baseline": baseline,
               "temporal_approximate": t_det["approximate"],
               "temporal_evaluated": t_det["evaluated"], "cold": np.flatnonzero(cold_mask),
               "block_ranking": ranking, "rescued_blocks": rescued,
               "exact_candidates": exact_ids}
    return nxt, m, details
