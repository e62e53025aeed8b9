"""VRAM hot-block cache policy oracle (numpy / pure Python).  TEST INFRASTRUCTURE ONLY.

Restates, from ``llama3_neuroplastic/experiments/streaming_llama_runtime.py``:

* ``_plan_fixed_capacity_bank_update`` (``:2577-2617``): free slots first,
  then the lowest current score (first minimum on ties); novel block ``i``
  gets score ``base + (i+1)*1e-3`` with ``base = max(active scores) + 1``
  (``1.0`` when the bank is empty); the bank takes at most ``capacity``
  novel blocks.  Pinned by the reference's
  ``tests/test_throughput_contract.py:308-321``.
* the +1-per-decode-hit scoring of resident down blocks (``:5262-5271``);
* ``_record_hot_cache_calibration_blocks`` (``:2205-2243``): row ``r`` of
  ``R`` rows adds weight ``((r+1)/R) ** recency_power`` to each valid block
  (pinned by ``tests/test_throughput_contract.py:261-287``);
* ``_target_hot_blocks_for_layer`` (``:2275-2311``): budget-derived capacity
  (pinned by ``tests/test_throughput_contract.py:290-305``);
* the initial resident-bank scores ``linspace(n, 1, n)`` (``:2699-2706``).
"""
from __future__ import annotations

import numpy as np


def plan_fixed_capacity_bank_update(existing_block_ids, existing_scores, active_count, capacity, novel_blocks):
    """Returns ``(slots int64, block_ids int64, scores fp32, active_count)``."""
    cap = max(0, int(capacity))
    block_ids = np.asarray(existing_block_ids, np.int64).copy()
    scores = np.asarray(existing_scores, np.float32).copy()
    active = max(0, min(int(active_count), block_ids.size, cap))
    if cap <= 0:
        return np.zeros(0, np.int64), block_ids, scores, active
    novel = np.asarray(novel_blocks, np.int64).reshape(-1)
    if novel.size <= 0:
        return np.zeros(0, np.int64), block_ids, scores, active
    if novel.size > cap:
        novel = novel[:cap]
    cur = scores.copy()
    base = float(cur[:active].max()) + 1.0 if active > 0 else 1.0
    nxt = active
    slots = []
    for i in range(novel.size):
        if nxt < cap:
            slot = nxt
            nxt += 1
            active = max(active, slot + 1)
        else:
            slot = int(np.argmin(cur[:cap]))
        block_ids[slot] = int(novel[i])
        cur[slot] = np.float32(base + float(i + 1) * 1e-3)
        slots.append(slot)
    return np.asarray(slots, np.int64), block_ids, cur.astype(np.float32), active


def initial_bank_scores(n_hot: int, capacity: int) -> np.ndarray:
    s = np.zeros(int(capacity), np.float32)
    if n_hot > 0:
        s[:n_hot] = np.linspace(float(n_hot), 1.0, n_hot, dtype=np.float32)
    return s


def add_hit_scores(scores: np.ndarray, hit_slots: np.ndarray) -> np.ndarray:
    """``scores.index_add_(0, hit_slots, 1.0)`` (duplicates add twice)."""
    s = np.asarray(scores, np.float32).copy()
    np.add.at(s, np.asarray(hit_slots, np.int64).reshape(-1), np.float32(1.0))
    return s


def record_calibration_hits(counts: np.ndarray | None, active_blocks: np.ndarray, num_blocks: int,
                            recency_power: float) -> np.ndarray:
    c = np.zeros(int(num_blocks), np.float32) if counts is None or np.asarray(counts).size != int(num_blocks) \
        else np.asarray(counts, np.float32).copy()
    ab = np.asarray(active_blocks, np.int64)
    if ab.size == 0:
        return c
    rows = ab.reshape(-1, ab.shape[-1] if ab.ndim > 0 else 1)
    R = rows.shape[0]
    pos = np.arange(1, R + 1, dtype=np.float32)
    w = np.power(pos / np.float32(max(R, 1)), np.float32(recency_power)).astype(np.float32)
    for r in range(R):
        rb = rows[r]
        rb = rb[(rb >= 0) & (rb < int(num_blocks))]
        if rb.size:
            np.add.at(c, rb, w[r])
    return c


def target_hot_blocks(*, layer_idx: int, runtime_top_k: int, count_slots: int, previous_hot_count: int,
                      limit_bytes: int | None, used_bytes: int, sparse_layers: int, bytes_per_block: int,
                      env_target: int | None = None, env_cap: int | None = None) -> int:
    if env_target is not None and int(env_target) > 0:
        return max(1, min(int(env_target), int(count_slots)))
    fallback = int(previous_hot_count)
    if fallback <= 0:
        fallback = int(max(1, runtime_top_k))
    if limit_bytes is None or int(limit_bytes) <= 0:
        return max(1, min(fallback, int(count_slots)))
    layers = max(1, int(sparse_layers))
    bpb = max(1, int(bytes_per_block))
    remaining = max(int(limit_bytes) - int(used_bytes), 0)
    remaining_layers = max(1, layers - max(0, int(layer_idx)))
    per_layer = int((float(remaining) * 0.97) / float(remaining_layers))
    target = max(fallback, per_layer // bpb)
    if env_cap is not None:
        target = min(target, int(env_cap))
    return max(1, min(int(target), int(count_slots)))


def hot_cache_bytes_per_block(hidden: int, block_size: int = 32) -> int:
    """gate+up packed and fp32 absmax plus the down column slice and absmax
    (``_estimate_mlp_hot_cache_bytes_per_block``, ``:2245-2273``)."""
    per_proj = (hidden // 2) * block_size + (hidden // 64) * block_size * 4
    return 2 * per_proj + hidden * max(1, block_size // 2) + hidden * 4
