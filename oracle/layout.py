"""Active-block layout oracle (numpy).  TEST INFRASTRUCTURE ONLY.

Restates ``StreamingLlamaRuntime._build_sparse_active_layout``
(``llama3_neuroplastic/experiments/streaming_llama_runtime.py:4857-4908``)
together with ``_order_blocks_for_layer_hot_cache`` (``:1975-1980``).

Quirk reproduced on purpose: the runtime orders the union hot-first
(``:4871``) and then calls ``unique(sorted=False)`` (``:4873``).  On CPU
tensors (torch 2.11) that call returns ascending order, so the final
``ordered_blocks`` is the ascending set of valid blocks whatever the hot set
is.  The golden fixtures pin this behaviour against the reference itself.

Second quirk: ``slot_mask.scatter_(1, clamp(active_local, 0), valid)``
(``:4896-4897``) runs in column order on CPU, so an invalid entry (clamped to
slot 0, value 0) that comes after a valid entry for slot 0 clears that slot.
``flat_mask`` reproduces "last write wins".
"""
from __future__ import annotations

import numpy as np


def order_blocks_hot_first(blocks: np.ndarray, hot: np.ndarray | None) -> np.ndarray:
    """Hot blocks first, then the rest, each in input order (``:1975-1980``)."""
    b = np.asarray(blocks, dtype=np.int64).reshape(-1)
    if hot is None or np.asarray(hot).size == 0 or b.size <= 1:
        return b
    is_hot = np.isin(b, np.asarray(hot, dtype=np.int64))
    return np.concatenate([b[is_hot], b[~is_hot]])


def build_sparse_active_layout(active_blocks: np.ndarray, rows: int, block_size: int, max_valid_blocks: int,
                               hot_blocks: np.ndarray | None = None):
    """Returns ``(ordered_blocks int64 [U], active_local int32 [rows,k],
    flat_mask fp32 [rows, U*block_size], active_neurons int64 [U*block_size])``."""
    ab = np.asarray(active_blocks, dtype=np.int64).reshape(rows, -1)
    union = ab.reshape(-1)
    if rows > 1:
        union = np.unique(union)
    ordered = order_blocks_hot_first(union, hot_blocks)
    ordered = ordered[(ordered >= 0) & (ordered < int(max_valid_blocks))]
    ordered = np.unique(ordered)  # torch CPU unique(sorted=False) -> ascending
    U = int(ordered.size)
    if U <= 0:
        return (ordered, np.full((rows, ab.shape[1]), -1, dtype=np.int32),
                np.zeros((rows, 0), dtype=np.float32), np.zeros((0,), dtype=np.int64))
    lookup = np.full(int(max_valid_blocks), -1, dtype=np.int32)
    lookup[ordered] = np.arange(U, dtype=np.int32)
    valid = (ab >= 0) & (ab < int(max_valid_blocks))
    active_local = np.full(ab.shape, -1, dtype=np.int32)
    active_local[valid] = lookup[ab[valid]]
    slot_mask = np.zeros((rows, U), dtype=np.float32)
    vl = active_local >= 0
    if vl.any():
        safe = np.maximum(active_local, 0)
        for r in range(rows):
            for j in range(ab.shape[1]):
                slot_mask[r, safe[r, j]] = 1.0 if vl[r, j] else 0.0
    flat_mask = np.repeat(slot_mask, int(block_size), axis=1) if vl.any() else np.zeros((rows, U * block_size), np.float32)
    neurons = (ordered[:, None] * int(block_size) + np.arange(int(block_size))[None, :]).reshape(-1)
    return ordered, active_local, flat_mask.astype(np.float32), neurons.astype(np.int64)
