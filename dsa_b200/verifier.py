"""The two-path verifier step on the device, with the reference's API.

Mirrors ``temporal_dsa.verifier`` (src/temporal_dsa/verifier.py): ``VerifierConfig``
(:15-43) and ``verifier_step`` (:173-375).  The temporal filter, the cold-block ranking by
verifier score, the rescue (a global budget or a fixed promotion threshold), the exact
rerank of the candidate union and the state update run as one tdsa_policy_step with a
rescue; the metrics are assembled from the step's device statistics and device-side set
operations.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch

from .approx import ApproxState, _successor
from .indexer import require_cuda, topk as device_topk


@dataclass(frozen=True)
class VerifierConfig:
    """Runtime-legal current-query candidate generator (verifier.py:15-43)."""

    name: str
    path: str
    width: int
    score_ratio: float
    block_size: int = 64
    rescue_fraction: float = 0.05
    sketch_bytes_per_token: float = 0.0
    full_key_bytes_per_token: int = 256
    metadata_bytes_per_block: int = 4
    retain_candidate_keys: bool = False

    def __post_init__(self) -> None:
        if self.path not in {"head", "dim"}:
            raise ValueError("path must be 'head' or 'dim'")
        if self.width <= 0:
            raise ValueError("width must be positive")
        if not 0 <= self.rescue_fraction <= 1:
            raise ValueError("rescue_fraction must be in [0, 1]")
        if not 0 <= self.score_ratio <= 1:
            raise ValueError("score_ratio must be in [0, 1]")


def _retention(approximate: torch.Tensor, baseline: torch.Tensor, count: int) -> float:
    count = min(count, baseline.numel())
    if count == 0:
        return 1.0
    return float(torch.isin(baseline[:count], approximate).sum().item() / count)


def _average_precision(ranking: torch.Tensor, positives: torch.Tensor) -> float:
    """verifier.py:76-87 on device tensors."""
    if positives.numel() == 0:
        return 1.0
    hit = torch.isin(ranking, positives).to(torch.float64)
    if ranking.numel() == 0:
        return 0.0
    hits = torch.cumsum(hit, 0)
    ranks = torch.arange(1, ranking.numel() + 1, device=ranking.device, dtype=torch.float64)
    return float(((hits / ranks) * hit).sum().item() / positives.numel())


def _block_ids(mask: torch.Tensor, block: int) -> torch.Tensor:
    return torch.unique(torch.nonzero(mask).flatten() // block)


def verifier_step(state: ApproxState, current_scores: torch.Tensor,
                  verifier_scores: torch.Tensor, *, policy, config: VerifierConfig, k: int,
                  step: int, previous_length: int | None = None,
                  tail_critical_blocks: torch.Tensor | None = None,
                  promotion_threshold: float | None = None
                  ) -> tuple[ApproxState, dict[str, Any], dict[str, torch.Tensor]]:
    """verifier.py:173-375 on the device -> (state, metrics, details)."""
    require_cuda(current_scores, verifier_scores)
    scores = current_scores.to(torch.float32)
    length = scores.numel()
    vs = verifier_scores[:length].to(torch.float32)
    if vs.shape != scores.shape:
        raise ValueError("verifier score length must match current score length")
    if k != state.plan.k or config.block_size != state.plan.block_size:
        raise ValueError("k and block_size must match the state")
    seed = state.topk.to(torch.int64)
    plan = _successor(state, length)
    plan.step(scores, policy, step=step, history_mode="own", previous_length=previous_length,
              verifier_scores=vs, rescue_fraction=config.rescue_fraction,
              promotion_threshold=promotion_threshold)
    st = plan.stats_host()[0]
    bs = config.block_size
    nb = (length + bs - 1) // bs
    dev = scores.device

    flags = plan.block_flags[0, :nb]
    exact_mask = plan.evaluated_mask(0)
    rescued_block_mask = (flags & 4) != 0
    key_blocks = torch.arange(length, device=dev) // bs
    seed_mask = torch.zeros(length, dtype=torch.bool, device=dev)
    seed_mask[seed[seed < length]] = True
    temporal_mask = seed_mask | ((flags & 2) != 0)[key_blocks]
    cold_mask = ~temporal_mask
    ncold = int(st["COLD_BLOCKS"])
    ranking = plan.ranking[0, :ncold].to(torch.int64)
    rescued = ranking[rescued_block_mask[ranking]]
    approximate = plan.topk[0].to(torch.int64)
    baseline = plan.baseline_topk[0].to(torch.int64)
    exact_ids = torch.nonzero(exact_mask).flatten()
    temporal_ids = torch.nonzero(temporal_mask).flatten()

    temporal_exact = int(st["SCORED"])
    union = int(st["UNION"])
    rescue_new = union - temporal_exact
    verifier_tokens = int(cold_mask.sum().item())
    full_equivalent = temporal_exact + rescue_new + verifier_tokens * config.score_ratio
    metadata_bytes = nb * config.metadata_bytes_per_block
    temporal_key_bytes = temporal_exact * config.full_key_bytes_per_token
    if config.path == "head":
        verifier_key_bytes = verifier_tokens * config.full_key_bytes_per_token
        reread = 0 if config.retain_candidate_keys else rescue_new * config.full_key_bytes_per_token
        sketch_bytes = 0.0
    else:
        verifier_key_bytes = 0.0
        sketch_bytes = verifier_tokens * config.sketch_bytes_per_token
        reread = rescue_new * config.full_key_bytes_per_token
    total_key_bytes = temporal_key_bytes + verifier_key_bytes + sketch_bytes + reread + \
        metadata_bytes
    baseline_key_bytes = length * config.full_key_bytes_per_token

    newly_active = baseline[cold_mask[baseline]]
    newly_active_blocks = torch.unique(newly_active // bs)
    rescued_tokens = torch.isin(newly_active, exact_ids)
    rescued_positive = rescued[torch.isin(rescued, newly_active_blocks)]
    tail = (torch.zeros(0, dtype=torch.int64, device=dev) if tail_critical_blocks is None
            else torch.as_tensor(tail_critical_blocks, device=dev).to(torch.int64))
    rescued_tail = torch.unique(rescued[torch.isin(rescued, tail)])

    physical: dict[int, float] = {}
    for pb in (32, 64, 128):
        full_blocks = (length + pb - 1) // pb
        base_phys = full_blocks * pb * config.full_key_bytes_per_token
        if config.path == "head":
            reread_blocks = 0
            if not config.retain_candidate_keys and rescued.numel():
                reread_blocks = int(_block_ids(rescued_block_mask[key_blocks], pb).numel())
            phys = base_phys + reread_blocks * pb * config.full_key_bytes_per_token + \
                metadata_bytes
        else:
            phys = (int(_block_ids(exact_mask, pb).numel()) * pb * config.full_key_bytes_per_token
                    + int(_block_ids(cold_mask, pb).numel()) * pb * config.sketch_bytes_per_token
                    + metadata_bytes)
        physical[pb] = float(1.0 - phys / base_phys)

    missed = int(st["MISSED"])
    metrics: dict[str, Any] = {
        "step": step, "context_length": length, "policy": policy.name,
        "verifier": config.name, "path": config.path, "width": config.width,
        "block_size": bs, "rescue_fraction": config.rescue_fraction,
        "promotion_policy": "global_budget" if promotion_threshold is None else "fixed_threshold",
        "promotion_threshold": (math.nan if promotion_threshold is None
                                else float(promotion_threshold)),
        "promotion_fraction_of_cold": float(rescued.numel() / max(1, ncold)),
        "temporal_exact_tokens": temporal_exact,
        "cold_tokens_scanned": verifier_tokens,
        "cold_blocks_scanned": ncold,
        "rescue_blocks": int(rescued.numel()),
        "rescue_exact_tokens": rescue_new,
        "candidate_union_tokens": union,
        "duplicate_exact_tokens": 0,
        "qk_full_equivalent": float(full_equivalent),
        "net_qk_reduction": float(1.0 - full_equivalent / float(length)),
        "exact_match": missed == 0,
        "recall": float((k - missed) / k),
    }
    for n in (128, 256, 512, 1024, 2048):
        metrics[f"top{n}_recall"] = float(st[f"TOP{n}"] / min(n, k))
    metrics.update({
        "index_mass_ratio": float(st["MASS_NUM"] / max(st["MASS_DEN"], 1e-300)),
        "newly_active_tokens": int(newly_active.numel()),
        "newly_active_token_recall": (float(rescued_tokens.double().mean().item())
                                      if newly_active.numel() else 1.0),
        "newly_active_blocks": int(newly_active_blocks.numel()),
        "newly_active_block_recall": (float(rescued_positive.numel() / newly_active_blocks.numel())
                                      if newly_active_blocks.numel() else 1.0),
        "detector_ap": _average_precision(ranking, newly_active_blocks),
        "rescue_precision": (float(rescued_positive.numel() / rescued.numel())
                             if rescued.numel() else 1.0),
        "tail_critical_blocks": int(tail.numel()),
        "tail_critical_block_recall": (float(rescued_tail.numel() / tail.numel())
                                       if tail.numel() else 1.0),
        "temporal_key_bytes": float(temporal_key_bytes),
        "verifier_key_bytes": float(verifier_key_bytes),
        "sketch_bytes": float(sketch_bytes),
        "rescue_reread_key_bytes": float(reread),
        "metadata_bytes": int(metadata_bytes),
        "total_key_bytes": float(total_key_bytes),
        "ideal_key_byte_reduction": float(1.0 - total_key_bytes / baseline_key_bytes),
        "physical_key_byte_reduction": physical[64],
        "physical_b32_key_byte_reduction": physical[32],
        "physical_b64_key_byte_reduction": physical[64],
        "physical_b128_key_byte_reduction": physical[128],
    })
    masked = torch.where(temporal_mask, scores, torch.full_like(scores, float("-inf")))
    temporal_approx, _ = device_topk(masked, k, sorted=True, index_dtype=torch.int64)
    details = {
        "approximate": approximate, "baseline": baseline,
        "temporal_approximate": temporal_approx, "temporal_evaluated": temporal_ids,
        "cold": torch.nonzero(cold_mask).flatten(), "block_ranking": ranking,
        "rescued_blocks": rescued, "exact_candidates": exact_ids,
        "newly_active": newly_active, "newly_active_blocks": newly_active_blocks,
    }
    return ApproxState(plan), metrics, details
