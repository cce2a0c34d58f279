"""The reference's own policy, verifier and trace tests, on the device implementation.

Same vectors and assertions as the reference's tests/test_approx.py (state machine: full
refresh, seed counting, no leakage of skipped blocks, age cap, physical traffic),
tests/test_verifier.py (rescue, leakage, cost accounting, fixed-threshold promotion and its
address-stable tie break) and tests/test_trace_quality.py (trace round trip), with CUDA
tensors in and out.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dsa_b200.build import build

    build()
    yield
    from dsa_b200 import device_status

    assert device_status() == 0


def cuda(x):
    return torch.as_tensor(np.asarray(x, dtype=np.float32)).cuda()


def np_(t):
    return t.detach().cpu().numpy()


# ------------------------------------------------------------------- tests/test_approx.py
def test_full_refresh_matches_baseline_and_counts_every_key():
    from dsa_b200.approx import ApproxPolicy, initialize_state, replay_step

    previous = np.linspace(0, 1, 64, dtype=np.float32)
    current = previous[::-1].copy()
    state = initialize_state(cuda(previous), k=8, block_size=8)
    state, metrics, details = replay_step(state, cuda(current), policy=ApproxPolicy(name="full"),
                                          k=8, block_size=8, step=1, previous_length=64)
    assert metrics["exact_match"]
    assert metrics["qk_scored"] == 64
    assert np.array_equal(np.sort(np_(details["approximate"])), np.sort(np_(details["baseline"])))


def test_seed_rescore_is_not_double_counted():
    from dsa_b200.approx import ApproxPolicy, initialize_state, replay_step

    previous = np.arange(64, dtype=np.float32)
    state = initialize_state(cuda(previous), k=8, block_size=8)
    _, metrics, _ = replay_step(state, cuda(previous.copy()),
                                policy=ApproxPolicy(name="static", gamma=1e9), k=8,
                                block_size=8, step=1, previous_length=64)
    assert metrics["qk_scored"] == 64


def test_own_trajectory_never_updates_skipped_block_with_truth():
    from dsa_b200.approx import ApproxPolicy, initialize_state, replay_step

    previous = np.zeros(32, dtype=np.float32)
    previous[:4] = 3
    state = initialize_state(cuda(previous), k=4, block_size=8)
    current = previous.copy()
    current[16:20] = 10
    state, metrics, _ = replay_step(state, cuda(current),
                                    policy=ApproxPolicy(name="static", gamma=0), k=4,
                                    block_size=8, step=1, previous_length=32)
    assert metrics["recall"] == 0
    assert float(state.last_max[2]) == 0  # the current maximum (10) did not leak
    assert int(state.age[2]) == 1


def test_age_cap_forces_stale_block_refresh():
    from dsa_b200.approx import ApproxPolicy, initialize_state, replay_step

    previous = np.zeros(32, dtype=np.float32)
    previous[:4] = 3
    state = initialize_state(cuda(previous), k=4, block_size=8)
    current = previous.copy()
    current[16:20] = 10
    policy = ApproxPolicy(name="age", gamma=0, age_cap=1)
    state, first, _ = replay_step(state, cuda(current), policy=policy, k=4, block_size=8,
                                  step=1, previous_length=32)
    state, second, _ = replay_step(state, cuda(current), policy=policy, k=4, block_size=8,
                                   step=2, previous_length=32)
    assert first["recall"] == 0
    assert second["recall"] == 1


def test_scattered_seed_physical_traffic_is_reported():
    from dsa_b200.approx import ApproxPolicy, initialize_state, replay_step

    previous = np.zeros(64, dtype=np.float32)
    previous[::8] = 5
    state = initialize_state(cuda(previous), k=8, block_size=8)
    _, metrics, _ = replay_step(state, cuda(previous.copy()),
                                policy=ApproxPolicy(name="static", gamma=0), k=8,
                                block_size=8, step=1, previous_length=64)
    assert metrics["seed_blocks_touched"] == 8
    assert metrics["physical_b16_blocks"] == 4


# ----------------------------------------------------------------- tests/test_verifier.py
def _config(rescue_fraction: float = 0.5):
    from dsa_b200.verifier import VerifierConfig

    return VerifierConfig(name="head8", path="head", width=8, score_ratio=0.125, block_size=8,
                          rescue_fraction=rescue_fraction)


def test_verifier_rescues_newly_active_block_without_duplicate_scoring():
    from dsa_b200.approx import ApproxPolicy, initialize_state
    from dsa_b200.verifier import verifier_step

    previous = np.zeros(32, dtype=np.float32)
    previous[:4] = 3
    current = previous.copy()
    current[16:20] = 10
    partial = np.zeros_like(current)
    partial[16:20] = 5
    state = initialize_state(cuda(previous), k=4, block_size=8)
    state, metrics, details = verifier_step(state, cuda(current), cuda(partial),
                                            policy=ApproxPolicy(name="static", gamma=0),
                                            config=_config(), k=4, step=1, previous_length=32)
    assert metrics["recall"] == 1
    assert metrics["newly_active_token_recall"] == 1
    assert metrics["duplicate_exact_tokens"] == 0
    assert 2 in np_(details["rescued_blocks"])
    assert float(state.last_max[2]) == 10
    assert int(state.age[2]) == 0


def test_unrescued_block_does_not_leak_current_score():
    from dsa_b200.approx import ApproxPolicy, initialize_state
    from dsa_b200.verifier import verifier_step

    previous = np.zeros(32, dtype=np.float32)
    previous[:4] = 3
    current = previous.copy()
    current[16:20] = 10
    state = initialize_state(cuda(previous), k=4, block_size=8)
    state, metrics, _ = verifier_step(state, cuda(current), cuda(np.zeros_like(current)),
                                      policy=ApproxPolicy(name="static", gamma=0),
                                      config=_config(rescue_fraction=0), k=4, step=1,
                                      previous_length=32)
    assert metrics["recall"] == 0
    assert float(state.last_max[2]) == 0
    assert int(state.age[2]) == 1


def test_cost_includes_verifier_and_candidate_rerank():
    from dsa_b200.approx import ApproxPolicy, initialize_state
    from dsa_b200.verifier import verifier_step

    previous = np.arange(32, dtype=np.float32)
    state = initialize_state(cuda(previous), k=4, block_size=8)
    _, metrics, _ = verifier_step(state, cuda(previous.copy()), cuda(previous.copy()),
                                  policy=ApproxPolicy(name="static", gamma=1e9),
                                  config=_config(rescue_fraction=0.5), k=4, step=1,
                                  previous_length=32)
    expected = (metrics["temporal_exact_tokens"] + metrics["rescue_exact_tokens"]
                + metrics["cold_tokens_scanned"] * 0.125)
    assert metrics["qk_full_equivalent"] == expected
    assert metrics["candidate_union_tokens"] == (metrics["temporal_exact_tokens"]
                                                 + metrics["rescue_exact_tokens"])
    assert metrics["physical_b64_key_byte_reduction"] <= 0


def test_fixed_threshold_promotes_all_blocks_at_or_above_cutoff():
    from dsa_b200.approx import ApproxPolicy, initialize_state
    from dsa_b200.verifier import verifier_step

    previous = np.zeros(32, dtype=np.float32)
    previous[:4] = 3
    current = previous.copy()
    current[16:20] = 10
    verifier = np.zeros_like(current)
    verifier[8:16] = 4
    verifier[16:24] = 5
    state = initialize_state(cuda(previous), k=4, block_size=8)
    _, metrics, details = verifier_step(state, cuda(current), cuda(verifier),
                                        policy=ApproxPolicy(name="static", gamma=0),
                                        config=_config(rescue_fraction=0), k=4, step=1,
                                        previous_length=32, promotion_threshold=5)
    assert metrics["promotion_policy"] == "fixed_threshold"
    assert metrics["promotion_threshold"] == 5
    assert np.array_equal(np_(details["rescued_blocks"]), np.asarray([2]))


def test_fixed_threshold_tie_break_is_block_address_stable():
    from dsa_b200.approx import ApproxPolicy, initialize_state
    from dsa_b200.verifier import verifier_step

    values = np.zeros(32, dtype=np.float32)
    values[:4] = 3
    state = initialize_state(cuda(values), k=4, block_size=8)
    _, _, details = verifier_step(state, cuda(values), cuda(np.ones_like(values)),
                                  policy=ApproxPolicy(name="static", gamma=0),
                                  config=_config(rescue_fraction=0), k=4, step=1,
                                  previous_length=32, promotion_threshold=1)
    assert np.array_equal(np_(details["rescued_blocks"]), np.arange(1, 4))


# ------------------------------------------------------------ tests/test_trace_quality.py
def test_trace_round_trip(tmp_path):
    from dsa_b200.trace import ScoreTrace, load_trace, save_trace

    trace = ScoreTrace(scores=np.arange(18, dtype=np.float16).reshape(3, 6),
                       lengths=np.array([4, 5, 6]), layer=2, workload="code", prompt_id="p0",
                       metadata={"seed": 1})
    path = tmp_path / "trace.npz"
    save_trace(path, trace)
    loaded = load_trace(path)
    assert loaded.layer == 2
    assert np.array_equal(loaded.row(1), np.array([6, 7, 8, 9, 10], dtype=np.float32))
