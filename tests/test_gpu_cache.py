"""The VRAM hot-block cache on the GPU: resident blocks computed from the bank,
misses staged from pinned host memory on a side stream, promotion after use.

Each token's output must match the oracle's fp32 dequant + matmul of the
selected blocks (evaluated on the bitsandbytes bytes the layer was generated
from) within the decode tolerances, whichever blocks were resident, staged or
prefetched; the device block table must mirror the host bank after every
promotion, and the bank must evolve exactly like the reference policy (the
oracle) on the same hit/miss sequence.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import cache_policy as cp  # noqa: E402
from oracle import synthetic as syn  # noqa: E402
from tests.gpu_oracle import host_router, oracle_mlp, oracle_route  # noqa: E402

MAX_ABS = 2e-2
REL_L2 = 5e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from next_step_ai_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def _close(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    assert rel <= REL_L2, f"relative L2 {rel:.3e}"
    assert float(np.abs(got - ref).max()) <= MAX_ABS


def _layer(shape_name, dev, seed=5):
    """(shape, resident weights, router, bitsandbytes bytes kept for the oracle)."""
    from next_step_ai_b200 import synthetic as dsyn

    shape = dsyn.SHAPES[shape_name]
    w, bnb = dsyn.make_layer_weights(shape, seed, 0, dev, keep_bnb=True)
    return shape, w, dsyn.make_router(shape, seed, 0, dev), bnb


def _oracle_y(shape, bnb, x, blocks):
    return oracle_mlp(bnb, shape.hidden, shape.intermediate, x, np.asarray(blocks, np.int64))


@pytest.mark.parametrize("shape_name,capacity,tokens", [("small", 40, 6), ("cfg0", 112, 6), ("cfg1", 416, 3)])
def test_cached_decode_matches_oracle_and_policy(dev, shape_name, capacity, tokens):
    """cfg1 with 416 of 1664 blocks resident is BASELINE config 3's bank."""
    from next_step_ai_b200 import synthetic as dsyn
    from next_step_ai_b200.cache import CachedSparseMlp, HostBlockStore

    shape, w, rw, bnb = _layer(shape_name, dev)
    store = HostBlockStore.from_weights(w)
    rng = np.random.default_rng(11)
    nb, k = shape.num_blocks, shape.top_k
    hot = rng.choice(nb, capacity, replace=False)
    cm = CachedSparseMlp(rw, store, capacity)
    cm.pre_warm(hot)
    # oracle bank state
    ids = np.full(capacity, -1, np.int64)
    ids[: hot.size] = hot
    scores, active = cp.initial_bank_scores(hot.size, capacity), hot.size
    for tok in range(tokens):
        x = dsyn.make_x(shape, 100 + tok, 1, dev)[0]
        res = set(ids[:active].tolist())
        n_hit = int(0.7 * k)
        sel = np.concatenate([rng.choice(sorted(res), n_hit, replace=False),
                              rng.choice(sorted(set(range(nb)) - res), k - n_hit, replace=False)])
        rng.shuffle(sel)
        idx = torch.from_numpy(sel.astype(np.int32)).to(dev)
        y, st = cm.decode(x, idx=idx)
        _close(y.cpu().numpy(), _oracle_y(shape, bnb, x, sel))
        assert (st.hits, st.misses) == (n_hit, k - n_hit)
        assert st.h2d_bytes == (k - n_hit) * 56 * shape.hidden
        # the reference policy on the same token
        hit_slots = np.array([int(np.flatnonzero(ids[:active] == b)[0]) for b in sel if b in res], np.int64)
        scores = cp.add_hit_scores(scores, hit_slots)
        misses = np.array([b for b in sel if b not in res], np.int64)
        _, ids, scores, active = cp.plan_fixed_capacity_bank_update(ids, scores, active, capacity, misses)
        assert np.array_equal(cm.bank.block_ids, ids) and np.array_equal(cm.bank.scores, scores)
        # device table == host mirror == bank
        torch.cuda.synchronize()
        table = cm.slot_dev.cpu().numpy()
        assert np.array_equal(table, cm.slot_host)
        for slot, b in enumerate(ids[:active]):
            assert table[b] == slot
        assert int((table >= 0).sum()) == active


def test_cached_decode_router_path_and_promoted_hits(dev):
    from next_step_ai_b200 import route_sparse_mlp
    from next_step_ai_b200 import synthetic as dsyn
    from next_step_ai_b200.cache import CachedSparseMlp, HostBlockStore

    shape, w, rw, bnb = _layer("small", dev, seed=9)
    store = HostBlockStore.from_weights(w)
    cm = CachedSparseMlp(rw, store, 24)
    cm.pre_warm(np.arange(24))
    x = dsyn.make_x(shape, 3, 1, dev)[0]
    y, st = cm.decode(x)  # router selection
    sel = route_sparse_mlp(x, rw)[0].to(torch.int32)
    ref_sel = oracle_route(host_router(rw), x.float().cpu().numpy(), shape.top_k, shape.rank)
    assert np.array_equal(sel.cpu().numpy(), ref_sel)
    ref = _oracle_y(shape, bnb, x, ref_sel)
    _close(y.cpu().numpy(), ref)
    assert st.hits + st.misses == shape.top_k and st.promoted == st.misses
    # the same token again: every block promoted last time is now a hit; a
    # block the promotion evicted (lowest score, possibly one of this token's
    # hits) is the only kind of miss left
    blocks = sel.cpu().numpy()
    resident = cm.slot_host[blocks] >= 0
    first_misses = set(blocks[~np.isin(blocks, np.arange(24))].tolist())
    assert all(cm.slot_host[b] >= 0 for b in first_misses)
    y2, st2 = cm.decode(x)
    assert st2.misses == int((~resident).sum()) and st2.hits == int(resident.sum())
    _close(y2.cpu().numpy(), ref)


def test_cache_rejects_bad_selections(dev):
    from next_step_ai_b200 import synthetic as dsyn
    from next_step_ai_b200.cache import CachedSparseMlp, HostBlockStore

    shape, w, rw, _ = _layer("tiny", dev, seed=2)
    cm = CachedSparseMlp(rw, HostBlockStore.from_weights(w), 8)
    cm.pre_warm(np.arange(8))
    x = dsyn.make_x(shape, 1, 1, dev)[0]
    with pytest.raises(RuntimeError):
        cm.decode(x, idx=torch.tensor([0, 0, 1, 2], dtype=torch.int32, device=dev))
    with pytest.raises(RuntimeError):
        cm.decode(x, idx=torch.tensor([0, 1, 2, shape.num_blocks], dtype=torch.int32, device=dev))


def _twin_caches(shape, w, rw, capacity, hot):
    from next_step_ai_b200.cache import CachedSparseMlp, HostBlockStore

    store = HostBlockStore.from_weights(w)
    a, b = CachedSparseMlp(rw, store, capacity), CachedSparseMlp(rw, store, capacity)
    a.pre_warm(hot)
    b.pre_warm(hot)
    return a, b


def test_prefetch_serves_misses_without_copies(dev):
    from next_step_ai_b200 import synthetic as dsyn

    shape, w, rw, bnb = _layer("small", dev, seed=13)
    nb, k, cap = shape.num_blocks, shape.top_k, 40
    rng = np.random.default_rng(3)
    a, b = _twin_caches(shape, w, rw, cap, rng.choice(nb, cap, replace=False))
    for tok, frac in enumerate((1.0, 0.5, 0.0)):
        res = set(a.bank.block_ids[: a.bank.active].tolist())
        cold = sorted(set(range(nb)) - res)
        sel = np.concatenate([rng.choice(sorted(res), 9, replace=False), rng.choice(cold, k - 9, replace=False)])
        misses = sel[9:]
        early = misses[: int(round(frac * misses.size))]
        others = rng.choice(sorted(set(cold) - set(misses.tolist())), 3, replace=False)
        assert a.prefetch(np.concatenate([early, others])) == early.size + 3
        x = dsyn.make_x(shape, 40 + tok, 1, dev)[0]
        idx = torch.from_numpy(sel.astype(np.int32)).to(dev)
        ya, sa = a.decode(x, idx=idx)
        yb, sb = b.decode(x, idx=idx)
        assert torch.equal(ya, yb)
        assert (sa.hits, sa.misses, sa.promoted) == (sb.hits, sb.misses, sb.promoted)
        assert sa.prefetched == early.size and sa.h2d_bytes == (misses.size - early.size) * 56 * shape.hidden
        assert np.array_equal(a.bank.block_ids, b.bank.block_ids) and np.array_equal(a.slot_host, b.slot_host)
        _close(ya.cpu().numpy(), _oracle_y(shape, bnb, x, sel))
    # promoted records came from the prefetched rows: the banks hold the same bytes
    torch.cuda.synchronize()
    assert torch.equal(a.pool[:cap], b.pool[:cap])


def test_layer_stack_lookahead_is_exact(dev):
    from next_step_ai_b200 import synthetic as dsyn
    from next_step_ai_b200.cache import CachedLayerStack, CachedSparseMlp, HostBlockStore

    layers = [_layer("small", dev, seed=20 + i) for i in range(3)]
    shape = layers[0][0]
    rng = np.random.default_rng(8)
    stacks = []
    hots = [rng.choice(shape.num_blocks, 40, replace=False) for _ in layers]
    for look in (True, False):
        cs = []
        for (_, w, rw, _), hot in zip(layers, hots):
            c = CachedSparseMlp(rw, HostBlockStore.from_weights(w), 40)
            c.pre_warm(hot)
            cs.append(c)
        stacks.append(CachedLayerStack(cs, lookahead=look))
    prefetched = 0
    for tok in range(3):
        h0 = dsyn.make_x(shape, 70 + tok, 1, dev)[0].float() * 3.0
        ra, rb, rr = h0.clone(), h0.clone(), h0.clone()
        sta = stacks[0].decode_token(ra)
        stb = stacks[1].decode_token(rb)
        assert torch.equal(ra, rb)
        assert [s.misses for s in sta] == [s.misses for s in stb]
        prefetched += sum(s.prefetched for s in sta)
        assert all(s.prefetched == 0 for s in stb)
        # the oracle chain: each layer's input from the stack's own RMSNorm of the
        # oracle residual, routed and multiplied by the oracle
        for li, (_, w, rw, bnb) in enumerate(layers):
            xi = stacks[1]._input(rr, li)
            sel = oracle_route(host_router(rw), xi.float().cpu().numpy(), shape.top_k, shape.rank)
            rr.add_(torch.from_numpy(_oracle_y(shape, bnb, xi, sel)).to(dev))
        _close(ra.cpu().numpy(), rr.cpu().numpy())
    assert prefetched > 0


def test_calibration_rebuild_prewarms_top_counts(dev):
    from next_step_ai_b200 import route_sparse_mlp
    from next_step_ai_b200 import synthetic as dsyn
    from next_step_ai_b200.cache import CachedSparseMlp, HostBlockStore, HotCacheCalibration, top_count_blocks

    shape, w, rw, bnb = _layer("small", dev, seed=31)
    cm = CachedSparseMlp(rw, HostBlockStore.from_weights(w), 24)
    cm.pre_warm(np.arange(24))
    cal = HotCacheCalibration()
    counts = np.zeros(shape.num_blocks, np.float32)
    for tok in range(5):
        x = dsyn.make_x(shape, 90 + tok, 1, dev)[0]
        cm.decode(x, calibration=cal, layer_idx=3)
        np.add.at(counts, route_sparse_mlp(x, rw)[0].cpu().numpy(), 1.0)
    assert np.array_equal(cal.hits[3], counts)
    out = cal.rebuild({3: cm})
    assert out["updated_layers"] == 1 and out["hits"] == 5 * shape.top_k
    assert cm.bank.block_ids[: cm.bank.active].tolist() == top_count_blocks(counts, 24).tolist()
    x = dsyn.make_x(shape, 99, 1, dev)[0]
    y, st = cm.decode(x)
    sel = route_sparse_mlp(x, rw)[0].cpu().numpy()
    _close(y.cpu().numpy(), _oracle_y(shape, bnb, x, sel))


@pytest.mark.parametrize("pinned", [True, False])
def test_stage_places_exact_records(dev, pinned):
    """The miss copy: pinned stores go through the gather kernel (device reads
    of mapped host memory), pageable ones through the copy engine; both put
    each record's bytes in its pool row, byte for byte, and leave the other
    rows alone."""
    import ctypes

    from next_step_ai_b200 import _lib

    lib = _lib.load()
    rec, nrec, prow = 56 * 256, 12, 6
    g = torch.Generator().manual_seed(3)
    host = torch.randint(0, 256, (nrec, rec), dtype=torch.uint8, generator=g)
    if pinned:
        host = host.pin_memory()
    pool = torch.full((prow, rec), 7, dtype=torch.uint8, device=dev)
    blocks = np.array([9, 0, 11, 4], np.int32)
    rows = np.array([5, 2, 0, 3], np.int32)
    s = torch.cuda.Stream(device=dev)
    _lib.check(lib.nsm_cache_stage(host.data_ptr(), nrec, blocks.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                   len(blocks), rec, pool.data_ptr(),
                                   rows.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), prow, s.cuda_stream),
               "nsm_cache_stage")
    s.synchronize()
    got = pool.cpu()
    for b, r in zip(blocks, rows):
        assert torch.equal(got[r], host[b])
    for r in (1, 4):
        assert bool((got[r] == 7).all())
