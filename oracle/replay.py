"""Pure-Python restatement of the reference block-replay filter (test oracle, small cases).

Reference: ``src/temporal_dsa/replay.py``.  ``replay_transition`` (``:225-400``) seeds a
running top-k heap with the previous step's top-k (``tau_seed = min(current[prev_topk])``,
``:270``), orders blocks (``_scan_order`` ``:153-169``), prunes every block whose upper
bound is below the running threshold (``:87-90``), never prunes a block holding keys that
are new at this step (``:263-266``) and accounts bytes as ``qk_scored * key_bytes +
blocks * metadata_bytes`` (``:369-370``).  With numba present the reference runs
``_compiled_filter`` (``:46-109``, key-granular heap updates); that is what this file
restates.  ``certified_upper`` builds the exact bound of ``certified.py:18-48`` for it.
"""

from __future__ import annotations

import math

import numpy as np

from .topk import stable_topk


def _worse(sa: float, ia: int, sb: float, ib: int) -> bool:
    """replay.py:19-21 -- heap order: lower score, then higher index, is worse."""
    return sa < sb or (sa == sb and ia > ib)


def _sift_down(hs: list, hi: list, root: int) -> None:
    """replay.py:24-43."""
    size = len(hs)
    while True:
        left = 2 * root + 1
        if left >= size:
            return
        worst = left
        right = left + 1
        if right < size and _worse(hs[right], hi[right], hs[left], hi[left]):
            worst = right
        if not _worse(hs[worst], hi[worst], hs[root], hi[root]):
            return
        hs[root], hs[worst] = hs[worst], hs[root]
        hi[root], hi[worst] = hi[worst], hi[root]
        root = worst


def compiled_filter(current, previous_topk, true_topk, upper, order, block_size: int,
                    fixed_threshold: float, dynamic: bool):
    """replay.py:46-109 -- returns (scored, pruned, false_cold, true_evaluated, discovery)."""
    length = current.size
    k = true_topk.size
    seeded = np.zeros(length, dtype=bool)
    true_mask = np.zeros(length, dtype=bool)
    true_block = np.zeros(upper.size, dtype=np.int64)
    for key in true_topk:
        true_mask[key] = True
        true_block[key // block_size] = 1
    hs, hi = [], []
    scored = true_evaluated = last_true = 0
    for key in previous_topk:
        key = int(key)
        seeded[key] = True
        hs.append(float(current[key]))
        hi.append(key)
        scored += 1
        if true_mask[key]:
            true_evaluated += 1
            last_true = scored
    for root in range(k // 2 - 1, -1, -1):
        _sift_down(hs, hi, root)
    threshold = hs[0] if dynamic else fixed_threshold
    pruned = false_cold = 0
    for block_id in order:
        block_id = int(block_id)
        if upper[block_id] < threshold:
            pruned += 1
            false_cold += true_block[block_id]
            continue
        for key in range(block_id * block_size, min(length, (block_id + 1) * block_size)):
            if seeded[key]:
                continue
            scored += 1
            if true_mask[key]:
                true_evaluated += 1
                last_true = scored
            value = float(current[key])
            if dynamic and (value > hs[0] or (value == hs[0] and key < hi[0])):
                hs[0], hi[0] = value, key
                _sift_down(hs, hi, 0)
                threshold = hs[0]
    discovery = 1.0 if true_evaluated < k else last_true / length
    return scored, pruned, false_cold, true_evaluated, discovery


def scan_order(name: str, upper, current_max, previous_hot) -> np.ndarray:
    """replay.py:153-169."""
    address = np.arange(upper.size)
    if name == "address":
        return address
    if name == "previous_hot":
        return np.lexsort((address, -upper, -previous_hot.astype(np.int8)))
    if name == "upper_hot":
        return np.lexsort((address, -upper))
    if name == "oracle_current":
        return np.lexsort((address, -current_max))
    raise ValueError(f"unknown scan order: {name}")


def _block_max(values, length: int, block_size: int) -> np.ndarray:
    return np.array([values[s : min(length, s + block_size)].max()
                     for s in range(0, length, block_size)], dtype=np.float64)


def replay_transition(previous, current, *, k: int, block_size: int, gamma_sigma: float,
                      method: str, scan_order_name: str, key_bytes: int = 256,
                      metadata_bytes_per_block: int = 8, upper_override=None) -> dict:
    """replay.py:225-400 (numba branch) -- the fields the tests compare.

    ``upper_override`` replaces ``previous_max + gamma`` with a per-block bound (the
    certified radius); new-key blocks are still forced to +inf as in :263-266.
    """
    previous = np.asarray(previous, dtype=np.float64)
    current = np.asarray(current, dtype=np.float64)
    nblocks = math.ceil(current.size / block_size)
    current_max = _block_max(current, current.size, block_size)
    previous_max = np.full(nblocks, -math.inf)
    previous_max[: math.ceil(previous.size / block_size)] = _block_max(
        previous, previous.size, block_size)
    sigma = float(np.std(current[: previous.size] - previous))
    gamma = gamma_sigma * sigma
    upper = previous_max + gamma if upper_override is None else np.array(upper_override,
                                                                           dtype=np.float64)
    if previous.size < current.size:
        upper[previous.size // block_size:] = math.inf
    previous_topk = stable_topk(previous, k)
    true_topk = stable_topk(current, k)
    tau_seed = float(np.min(current[previous_topk]))
    previous_hot = np.zeros(nblocks, dtype=bool)
    previous_hot[previous_topk // block_size] = True
    if method == "full":
        qk_scored, pruned, false_cold, true_eval = current.size, 0, 0, k
    else:
        fixed, dynamic, filt, order_name = tau_seed, True, upper, scan_order_name
        if method == "static":
            order_name, dynamic = "address", False
        elif method == "static_hot_first":
            order_name, dynamic = "previous_hot", False
        elif method == "oracle":
            order_name, filt = "oracle_current", current_max
        elif method != "dynamic":
            raise ValueError(f"unknown method: {method}")
        order = scan_order(order_name, filt, current_max, previous_hot)
        qk_scored, pruned, false_cold, true_eval, _ = compiled_filter(
            current, previous_topk, true_topk, filt, order, block_size, fixed, dynamic)
    bytes_read = qk_scored * key_bytes + nblocks * metadata_bytes_per_block
    return {
        "qk_scored": int(qk_scored),
        "blocks_pruned": int(pruned),
        "false_cold_blocks": int(false_cold),
        "recall": true_eval / k,
        "exact_match": bool(true_eval == k),
        "tau_seed": tau_seed,
        "net_byte_reduction": 1.0 - bytes_read / (current.size * key_bytes),
    }
