"""The temporal policy state machine on the device, with the reference's API.

Mirrors ``temporal_dsa.approx`` (src/temporal_dsa/approx.py): ``ApproxPolicy`` (:15-39),
``ApproxState`` (:42-50), ``initialize_state`` (:112-126) and ``replay_step`` (:129-364),
with the same names, arguments, return values and errors.  The state arrays and the
selection live on the GPU (tdsa_policy_init / tdsa_policy_step); the reference runs the
same step in numpy on a host copy of every step's scores.

``PolicyPlan`` is the decode-loop form for a batch of sequences: fixed buffers, one
C call per step, nothing read back unless asked (``stats_host()``).

Differences: state arrays are device tensors (int32 key lists); scores must be finite (a
key scoring -inf ties with the keys the policy did not read).
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import asdict, dataclass, replace
from typing import Any

import torch

from . import _capi as capi
from .indexer import require_cuda, stream_ptr

_STAT = {name: i for i, name in enumerate(capi.POLICY_STATS)}


@dataclass(frozen=True)
class ApproxPolicy:
    """Runtime-legal temporal policy (approx.py:15-39): ``gamma`` is an absolute score
    margin; skipped blocks keep stale metadata and get older."""

    name: str
    gamma: float = 0.0
    cold_streak: int = 1
    dynamic_threshold: bool = False
    order: str = "address"
    refresh_interval: int | None = None
    age_cap: int | None = None
    recent_window: int = 0
    risk_model: str = "last_max"
    ema_alpha: float = 0.9
    volatility_lambda: float = 0.0
    age_slope: float = 0.0
    fallback_threshold: float | None = None

    def with_gamma(self, gamma: float) -> "ApproxPolicy":
        return replace(self, gamma=float(gamma))


def policy_dict(policy: ApproxPolicy) -> dict[str, Any]:
    return asdict(policy)


def _policy_struct(policy) -> capi.TdsaPolicy:
    order = policy.order
    buckets = 0
    if order == "address":
        code = capi.TDSA_ORDER_ADDRESS
    elif order in ("previous_max", "predicted_risk"):
        code = capi.TDSA_ORDER_PREVIOUS_MAX
    elif order.startswith("bucket"):
        code, buckets = capi.TDSA_ORDER_BUCKET, int(order.removeprefix("bucket"))
    elif order == "oracle_current":
        code = capi.TDSA_ORDER_ORACLE_CURRENT
    else:
        raise ValueError(f"unknown block order: {order}")
    if policy.risk_model == "last_max":
        risk = capi.TDSA_RISK_LAST_MAX
    elif policy.risk_model == "ema":
        risk = capi.TDSA_RISK_EMA
    else:
        raise ValueError(f"unknown risk model: {policy.risk_model}")
    return capi.TdsaPolicy(
        float(policy.gamma), float(policy.ema_alpha), float(policy.volatility_lambda),
        float(policy.age_slope), int(policy.cold_streak), int(bool(policy.dynamic_threshold)),
        code, buckets, -1 if policy.age_cap is None else int(policy.age_cap),
        int(policy.recent_window), risk)


def full_refresh_flags(policy, step: int, fallback_value) -> tuple[bool, bool]:
    """approx.py:172-181: (full refresh this step, fallback triggered)."""
    fallback = bool(policy.fallback_threshold is not None and fallback_value is not None
                    and fallback_value > policy.fallback_threshold)
    full = bool(policy.name == "full"
                or (policy.refresh_interval and step % policy.refresh_interval == 0)
                or fallback)
    return full, fallback


def metadata_bytes_per_block(policy) -> int:
    """approx.py:84-89: packed metadata per block."""
    raw = 6 + (1 if policy.order.startswith("bucket") else 0)
    raw += 8 if policy.risk_model == "ema" else 0
    return int(math.ceil(raw / 4) * 4)


class PolicyPlan:
    """Device state and buffers of the temporal policy for `batch` sequences of up to
    `max_length` keys (block capacity ceil(max_length / block_size))."""

    def __init__(self, batch: int, max_length: int, k: int, block_size: int,
                 device: torch.device | str):
        lib = capi.lib()
        self.batch, self.max_length, self.k, self.block_size = batch, max_length, k, block_size
        self.max_blocks = (max_length + block_size - 1) // block_size
        self.device = torch.device(device)
        nbytes = lib.tdsa_policy_state_bytes(batch, k, self.max_blocks)
        if nbytes == 0:
            raise ValueError("invalid policy plan shape")
        self.state = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        offs = (C.c_int64 * 8)()
        capi.check(lib.tdsa_policy_state_offsets(batch, k, self.max_blocks, offs))
        self._offsets = list(offs)
        wbytes = lib.tdsa_policy_workspace_bytes(batch, max_length, k, self.max_blocks)
        self.workspace = torch.empty(max(wbytes, 1), dtype=torch.uint8, device=self.device)
        self._wbytes = wbytes
        self.words = (max_length + 31) // 32
        self.evaluated_bits = torch.zeros(batch, self.words, dtype=torch.int32, device=self.device)
        self.block_flags = torch.zeros(batch, self.max_blocks, dtype=torch.uint8,
                                       device=self.device)
        self.ranking = torch.full((batch, self.max_blocks), -1, dtype=torch.int32,
                                  device=self.device)
        self.stats = torch.zeros(batch, capi.TDSA_POLICY_NSTATS, dtype=torch.float64,
                                 device=self.device)
        self.length = 0

    # ---- views of the state buffer
    def _view(self, i: int, dtype: torch.dtype, width: int) -> torch.Tensor:
        esize = torch.tensor([], dtype=dtype).element_size()
        n = self.batch * width
        return self.state[self._offsets[i]: self._offsets[i] + n * esize].view(dtype).view(
            self.batch, width)

    @property
    def topk(self) -> torch.Tensor:
        return self._view(0, torch.int32, self.k)

    @property
    def baseline_topk(self) -> torch.Tensor:
        return self._view(1, torch.int32, self.k)

    def block_view(self, name: str) -> torch.Tensor:
        idx, dt = {"last_max": (2, torch.float32), "ema": (3, torch.float32),
                   "volatility": (4, torch.float32), "age": (5, torch.int16),
                   "cold_streak": (6, torch.int16)}[name]
        return self._view(idx, dt, self.max_blocks)

    # ---- steps
    def _scores(self, scores: torch.Tensor) -> torch.Tensor:
        require_cuda(scores)
        if scores.dim() == 1:
            scores = scores.unsqueeze(0)
        if scores.shape[0] != self.batch or scores.shape[1] > self.max_length:
            raise ValueError(f"scores must be [{self.batch}, <= {self.max_length}]")
        return scores.to(torch.float32).contiguous()

    def init(self, scores: torch.Tensor) -> torch.Tensor:
        s = self._scores(scores)
        length = s.shape[1]
        capi.check(capi.lib().tdsa_policy_init(
            self.state.data_ptr(), self.state.numel(), s.data_ptr(), s.stride(0), self.batch,
            length, self.k, self.block_size, self.max_blocks, self.workspace.data_ptr(),
            self._wbytes, stream_ptr(self.device)))
        self.length = length
        return self.topk

    def step(self, scores: torch.Tensor, policy, *, step: int, history_mode: str = "own",
             previous_length: int | None = None, fallback_value: float | None = None,
             verifier_scores: torch.Tensor | None = None, rescue_fraction: float = 0.05,
             promotion_threshold: float | None = None) -> torch.Tensor:
        """One decode step for every sequence; returns the selection [batch, k] (int32,
        stable top-k order).  With verifier_scores it is verifier_step's rescue."""
        if history_mode not in ("own", "teacher"):
            raise ValueError("history_mode must be 'own' or 'teacher'")
        s = self._scores(scores)
        length = s.shape[1]
        if self.k > length:
            raise ValueError("K cannot exceed the current trace length")
        prev = length if previous_length is None else int(previous_length)
        full, _ = full_refresh_flags(policy, step, fallback_value)
        pol = _policy_struct(policy)
        rescue, v, vstride = None, None, 0
        if verifier_scores is not None:
            v = verifier_scores.to(torch.float32)
            if v.dim() == 1:
                v = v.unsqueeze(0)
            v = v[:, :length].contiguous()
            if v.shape != s.shape:
                raise ValueError("verifier score length must match current score length")
            vstride = v.stride(0)
            rescue = capi.TdsaRescue(float(rescue_fraction),
                                     0.0 if promotion_threshold is None
                                     else float(promotion_threshold),
                                     int(promotion_threshold is not None))
        capi.check(capi.lib().tdsa_policy_step(
            self.state.data_ptr(), self.state.numel(), s.data_ptr(), s.stride(0),
            v.data_ptr() if v is not None else None, vstride, self.batch, length, prev, self.k,
            self.block_size, self.max_blocks, C.byref(pol),
            1 if history_mode == "teacher" else 0, int(full),
            C.byref(rescue) if rescue is not None else None, self.workspace.data_ptr(),
            self._wbytes, self.evaluated_bits.data_ptr(), self.words,
            self.block_flags.data_ptr(), self.ranking.data_ptr(), self.stats.data_ptr(),
            stream_ptr(self.device)))
        self.length = length
        return self.topk

    def stats_host(self) -> list[dict[str, float]]:
        """The last step's statistics per sequence (one device->host copy)."""
        rows = self.stats.cpu().tolist()
        out = []
        for r in rows:
            d = {name: r[i] for name, i in _STAT.items()}
            if d["ERROR"]:
                raise RuntimeError(f"previous Top-K seed does not hold {self.k} unique keys "
                                   f"below the current length")
            out.append(d)
        return out

    def evaluated_mask(self, row: int = 0) -> torch.Tensor:
        """Bool [length] of the keys read at the last step (device)."""
        words = self.evaluated_bits[row, : (self.length + 31) // 32].to(torch.int64) & 0xFFFFFFFF
        shifts = torch.arange(32, device=self.device)
        bits = (words.unsqueeze(1) >> shifts) & 1
        return bits.reshape(-1)[: self.length].bool()


@dataclass
class ApproxState:
    """approx.py:42-50 on the device: views of a one-sequence PolicyPlan."""

    plan: PolicyPlan

    @property
    def _nb(self) -> int:
        return (self.plan.length + self.plan.block_size - 1) // self.plan.block_size

    @property
    def topk(self) -> torch.Tensor:
        return self.plan.topk[0]

    @property
    def baseline_topk(self) -> torch.Tensor:
        return self.plan.baseline_topk[0]

    @property
    def last_max(self) -> torch.Tensor:
        return self.plan.block_view("last_max")[0, : self._nb]

    @property
    def ema(self) -> torch.Tensor:
        return self.plan.block_view("ema")[0, : self._nb]

    @property
    def volatility(self) -> torch.Tensor:
        return self.plan.block_view("volatility")[0, : self._nb]

    @property
    def age(self) -> torch.Tensor:
        return self.plan.block_view("age")[0, : self._nb]

    @property
    def cold_streak(self) -> torch.Tensor:
        return self.plan.block_view("cold_streak")[0, : self._nb]


def _capacity(length: int) -> int:
    cap = 1024
    while cap < length:
        cap *= 2
    return cap


def _successor(state: ApproxState, length: int) -> PolicyPlan:
    """A fresh plan holding a copy of `state` (the reference returns a new state and leaves
    the old one as it was), with room for `length` keys."""
    old = state.plan
    cap = max(old.max_length, _capacity(length))
    plan = PolicyPlan(1, cap, old.k, old.block_size, old.device)
    plan.topk.copy_(old.topk)
    plan.baseline_topk.copy_(old.baseline_topk)
    n = old.max_blocks
    for name in ("last_max", "ema", "volatility", "age", "cold_streak"):
        plan.block_view(name)[:, :n].copy_(old.block_view(name))
    # the block count the old arrays hold (the kernel extends from there)
    plan.state[plan._offsets[7]: plan._offsets[7] + 4].copy_(
        old.state[old._offsets[7]: old._offsets[7] + 4])
    plan.length = old.length
    return plan


def initialize_state(scores: torch.Tensor, *, k: int, block_size: int) -> ApproxState:
    """approx.py:112-126 on the device."""
    require_cuda(scores)
    if scores.dim() != 1:
        raise ValueError(f"expected a vector, got {tuple(scores.shape)}")
    if not 0 < k <= scores.numel():
        raise ValueError(f"k={k} is invalid for {scores.numel()} values")
    plan = PolicyPlan(1, _capacity(scores.numel()), k, block_size, scores.device)
    plan.init(scores)
    return ApproxState(plan)


def replay_step(state: ApproxState, current_scores: torch.Tensor, *, policy, k: int,
                block_size: int, step: int, history_mode: str = "own",
                previous_length: int | None = None, fallback_value: float | None = None
                ) -> tuple[ApproxState, dict[str, Any], dict[str, torch.Tensor]]:
    """approx.py:129-364 on the device -> (next_state, metrics, details)."""
    if history_mode not in ("own", "teacher"):
        raise ValueError("history_mode must be 'own' or 'teacher'")
    require_cuda(current_scores)
    length = current_scores.numel()
    if k > length:
        raise ValueError("K cannot exceed the current trace length")
    if k != state.plan.k or block_size != state.plan.block_size:
        raise ValueError("k and block_size must match the state")
    old_topk = state.topk.clone()
    old_base = state.baseline_topk.clone()
    plan = _successor(state, length)
    plan.step(current_scores, policy, step=step, history_mode=history_mode,
              previous_length=previous_length, fallback_value=fallback_value)
    st = plan.stats_host()[0]
    nxt = ApproxState(plan)
    return nxt, _replay_metrics(policy, st, plan, k, block_size, step, history_mode,
                                fallback_value, current_scores), \
        _replay_details(plan, old_topk, old_base, history_mode, length)


def _replay_details(plan: PolicyPlan, old_topk, old_base, history_mode: str, length: int):
    approximate = plan.topk[0].to(torch.int64)
    baseline = plan.baseline_topk[0].to(torch.int64)
    seed = (old_base if history_mode == "teacher" else old_topk).to(torch.int64)
    seed = seed[seed < length]
    nb = (length + plan.block_size - 1) // plan.block_size
    flags = plan.block_flags[0, :nb]
    refreshed = (flags & 2) != 0
    missed = torch.nonzero(~torch.isin(baseline, approximate)).flatten() + 1
    return {
        "approximate": approximate,
        "baseline": baseline,
        "evaluated": torch.nonzero(plan.evaluated_mask(0)).flatten(),
        "seed": seed,
        "refreshed_blocks": torch.nonzero(refreshed).flatten().to(torch.int32),
        "skipped_blocks": torch.nonzero(~refreshed).flatten().to(torch.int32),
        "missed_ranks": missed.to(torch.int32),
    }


def _replay_metrics(policy, st: dict, plan: PolicyPlan, k: int, block_size: int, step: int,
                    history_mode: str, fallback_value, scores) -> dict[str, Any]:
    length = int(scores.numel())
    nb = int(st["BLOCKS"])
    scored = int(st["SCORED"])
    full, fallback = full_refresh_flags(policy, step, fallback_value)
    mbpb = metadata_bytes_per_block(policy)
    mbytes = nb * mbpb
    newly = int(st["NEWLY_HOT"])
    missed = int(st["MISSED"])
    m: dict[str, Any] = {
        "step": step, "context_length": length, "history_mode": history_mode,
        "policy": policy.name, "gamma": policy.gamma, "k": k, "block_size": block_size,
        "qk_scored": scored, "qk_reduction": float(1.0 - scored / length),
        "exact_match": missed == 0, "recall": float((k - missed) / k),
    }
    for n in (128, 256, 512, 1024, 2048):
        m[f"top{n}_recall"] = float(st[f"TOP{n}"] / min(n, k))
    m.update({
        "index_mass_ratio": float(st["MASS_NUM"] / max(st["MASS_DEN"], 1e-300)),
        "newly_hot_count": newly, "newly_hot_missed": int(st["NEWLY_HOT_MISSED"]),
        "newly_hot_miss_rate": float(st["NEWLY_HOT_MISSED"] / newly) if newly else 0.0,
        "missed_count": missed, "worst_missed_rank": int(st["WORST_MISSED"]),
        "tau_seed": float(st["TAU_SEED"]), "tau_final": float(st["TAU_FINAL"]),
        "full_refresh": full, "fallback": fallback,
        "blocks_refreshed": int(st["REFRESHED"]), "blocks_skipped": int(st["SKIPPED"]),
        "seed_blocks_touched": int(st["SEED_BLOCKS"]),
        "seed_block_fraction": float(st["SEED_BLOCKS"] / nb),
        "metadata_bytes_per_block": mbpb, "metadata_bytes": mbytes,
        "ideal_bf16_bytes": int(scored * 256 + mbytes),
        "ideal_fp8_bytes": int(scored * 128 + mbytes),
        "net_bf16_reduction": float(1.0 - (scored * 256 + mbytes) / (length * 256)),
        "net_fp8_reduction": float(1.0 - (scored * 128 + mbytes) / (length * 128)),
    })
    for pb in (16, 32, 64, 128):
        touched = int(st[f"PHYS{pb}"])
        m[f"physical_b{pb}_blocks"] = touched
        m[f"physical_b{pb}_reduction"] = float(1.0 - touched / ((length + pb - 1) // pb))
    for c in (0, 256, 512, 1024, 2048):
        hbm = scored - min(c, k)  # the first c seed keys are read and distinct
        m[f"cache{c}_hbm_keys"] = hbm
        m[f"cache{c}_net_bf16_reduction"] = float(1.0 - (hbm * 256 + mbytes) / (length * 256))
    return m
