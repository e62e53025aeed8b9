"""Host side of the VRAM hot-block cache (no GPU): the bank replacement
policy, calibration weighting and capacity target of next_step_ai_b200.cache
against the reference's golden cases and the oracle, and the block record
layout."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import cache_policy as cp

torch = pytest.importorskip("torch")
from next_step_ai_b200 import cache  # noqa: E402


def test_bank_update_matches_reference_golden(cache_policy_golden):
    for c in cache_policy_golden["bank"]:
        bank = cache.FixedCapacityBank.from_state(c["ids"], c["scores"], c["active"], c["capacity"])
        slots = bank.plan_update(c["novel"])
        assert slots.tolist() == c["out_slots"]
        assert bank.block_ids.tolist() == c["out_ids"]
        assert np.array_equal(bank.scores, np.array(c["out_scores"], np.float32))
        assert bank.active == c["out_active"]


def test_bank_update_reference_unit_case():
    # the reference's own pinned case (tests/test_throughput_contract.py:308-321)
    bank = cache.FixedCapacityBank.from_state([10, 11, -1], [5.0, 1.0, 0.0], 2, 3)
    slots = bank.plan_update([20, 21])
    assert bank.active == 3 and slots.tolist() == [2, 1] and bank.block_ids.tolist() == [10, 21, 20]
    assert bank.scores[1] > 5.0 and bank.scores[2] > 5.0


def test_bank_sequence_matches_oracle():
    rng = np.random.default_rng(3)
    cap, nb = 24, 200
    bank = cache.FixedCapacityBank(cap)
    bank.prewarm(rng.choice(nb, 10, replace=False))
    ids, scores, active = bank.block_ids.copy(), bank.scores.copy(), bank.active
    assert np.array_equal(scores, cp.initial_bank_scores(10, cap))
    for step in range(40):
        resident = set(ids[:active].tolist())
        sel = rng.choice(nb, 12, replace=False)
        hits = [int(np.flatnonzero(ids[:active] == b)[0]) for b in sel if b in resident]
        misses = np.array([b for b in sel if b not in resident], np.int64)
        bank.add_hits(hits)
        scores = cp.add_hit_scores(scores, np.array(hits, np.int64))
        got = bank.plan_update(misses)
        slots, ids, scores, active = cp.plan_fixed_capacity_bank_update(ids, scores, active, cap, misses)
        assert got.tolist() == slots.tolist()
        assert np.array_equal(bank.block_ids, ids) and np.array_equal(bank.scores, scores)
        assert bank.active == active


def test_calibration_and_target_match_reference_golden(cache_policy_golden):
    for c in cache_policy_golden["calibration"]:
        ab = np.array(c["active_blocks"], np.int64)
        counts = cache.record_calibration_hits(None, ab, c["num_blocks"], c["power"])
        counts = cache.record_calibration_hits(counts, ab[::-1], c["num_blocks"], c["power"])
        assert np.allclose(counts, np.array(c["counts"], np.float32), rtol=0, atol=1e-6)
    for c in cache_policy_golden["target"]:
        got = cache.target_hot_blocks(layer_idx=c["layer_idx"], runtime_top_k=c["runtime_top_k"],
                                      count_slots=c["count_slots"], previous_hot_count=c["prev"],
                                      limit_bytes=c["limit"], used_bytes=c["used"], sparse_layers=c["layers"],
                                      bytes_per_block=c["bpb"])
        assert got == c["target"], c


@pytest.mark.parametrize("hidden", [256, 1024, 4096, 16384])
def test_record_layout(hidden):
    lay = cache.record_layout(hidden)
    end = 0
    for name in ("gate", "up", "down", "gate_absmax", "up_absmax", "down_absmax"):
        off, n = lay[name]
        assert off == end and off % 16 == 0 and n % 16 == 0
        end = off + n
    assert end == cache.record_bytes(hidden)
    # the per-block algorithmic bytes of the decode (gate+up packed+absmax, down packed+absmax)
    assert end == 2 * (16 * hidden + 2 * hidden) + 16 * hidden + 4 * hidden


# --------------------------------------------------------------------------- lookahead rows and calibration
def test_assign_staging_rows_keeps_prefetched_rows():
    rows, copy = cache.assign_staging_rows(np.array([7, 3, 9, 4]), {9: 0, 5: 1, 3: 2}, 6)
    assert rows.tolist() == [1, 2, 0, 3] and copy.tolist() == [True, False, False, True]
    rows, copy = cache.assign_staging_rows(np.array([1, 2]), {}, 4)
    assert rows.tolist() == [0, 1] and copy.all()
    rows, copy = cache.assign_staging_rows(np.zeros(0, np.int64), {2: 0}, 4)
    assert rows.size == 0
    with pytest.raises(RuntimeError, match="staging rows"):
        cache.assign_staging_rows(np.arange(5), {}, 4)


def test_top_count_blocks_order_and_ties():
    c = np.array([1.0, 3.0, 3.0, 0.0, 2.0, 3.0], np.float32)
    assert cache.top_count_blocks(c, 4).tolist() == [1, 2, 5, 4]
    assert cache.top_count_blocks(c, 10).tolist() == [1, 2, 5, 4, 0, 3]
    assert cache.top_count_blocks(c, 0).size == 0


def test_calibration_matches_reference_pieces():
    rng = np.random.default_rng(4)
    nb, k = 64, 6
    cal = cache.HotCacheCalibration(recency_power=1.0)
    ref = {}
    for tok in range(12):
        for li in (0, 2):
            sel = rng.choice(nb, size=(1 if tok % 3 else 2, k), replace=True if tok % 5 == 0 else False)
            cal.record(li, sel, nb)
            ref[li] = cp.record_calibration_hits(ref.get(li), sel, nb, 1.0)
    cal.record(5, np.zeros((1, 0), np.int64), nb)   # a layer without hits is skipped
    for li in (0, 2):
        assert np.array_equal(cal.hits[li], ref[li])
    kw = dict(limit_bytes=3 * 917504 * 20, used_bytes=917504, sparse_layers=4, bytes_per_block=917504)
    sets = cal.hot_sets(runtime_top_k={0: k, 2: k, 5: k}, previous_hot={2: 30}, **kw)
    assert sorted(sets) == [0, 2]
    for li, prev in ((0, 0), (2, 30)):
        cap = cp.target_hot_blocks(layer_idx=li, runtime_top_k=k, count_slots=nb, previous_hot_count=prev, **kw)
        assert sets[li].tolist() == np.argsort(-ref[li], kind="stable")[:cap].tolist()
    cal.active = False
    cal.record(0, np.arange(k)[None, :], nb)
    assert np.array_equal(cal.hits[0], ref[0])


def test_calibration_rebuild_matches_reference():
    """The rebuild loop of the reference's calibrate_vram_hot_cache, run on the
    same seeded hit counts when the fixture was made."""
    import json
    from pathlib import Path

    from tests.golden.make_golden import calibration_hits

    gold = json.loads((Path(__file__).parent / "golden" / "checkpoint.json").read_text())["calibration"]
    for c in gold:
        cal = cache.HotCacheCalibration()
        cal.hits = {li: v.copy() for li, v in calibration_hits(c["case"]).items()}
        rtk = {li: (4 + li if li % 2 == 0 else (c["sparse_runtime_top_k"] if c["sparse_runtime_top_k"] > 0
                                                else c["sparse_top_k"])) for li in range(8)}
        sets = cal.hot_sets(runtime_top_k=rtk, previous_hot={int(k): v for k, v in c["prev"].items()},
                            limit_bytes=c["limit"], used_bytes=0, sparse_layers=8,
                            bytes_per_block=cache.hot_cache_bytes_per_block(c["hidden"]))
        assert {str(k): v.tolist() for k, v in sets.items()} == c["hot"], c["case"]
        assert len(sets) == c["updated_layers"]
        assert sum(float(cal.hits[li].sum()) for li in sets) == pytest.approx(c["total_hits"], rel=1e-6)


def test_stage_rejects_ids_outside_the_store_before_any_copy():
    """nsm_cache_stage checks every block id against the host store and every
    destination row against the pool on the host, before queueing anything
    (no device is touched, so this runs without a GPU)."""
    import ctypes

    from next_step_ai_b200 import _lib

    lib = _lib.load()
    host = (ctypes.c_uint8 * 64)()
    pool = (ctypes.c_uint8 * 64)()

    def stage(blocks, rows, host_records=4, pool_rows=4):
        b = (ctypes.c_int32 * len(blocks))(*blocks)
        r = (ctypes.c_int32 * len(rows))(*rows)
        return lib.nsm_cache_stage(ctypes.addressof(host), host_records, b, len(blocks), 16,
                                   ctypes.addressof(pool), r, pool_rows, None)

    assert stage([4], [0]) == _lib.NSM_ERR_INVALID_ARG      # one past the store
    assert stage([-1], [0]) == _lib.NSM_ERR_INVALID_ARG
    assert stage([1, 2], [0, 4]) == _lib.NSM_ERR_INVALID_ARG  # one past the pool
    assert "outside the host store" in _lib.last_error() or "destination row" in _lib.last_error()
    assert stage([], []) == _lib.NSM_OK
