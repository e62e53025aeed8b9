"""GPU parity of the sm_100a decode path against the CPU oracle and the
reference's golden vectors.  Everything calls through libnsm.so's C ABI.

Tolerances (from the build's contract): selected block indices bit-exact
(same blocks, same order, ties to the lower index); MLP outputs within
max-abs-err <= 2e-2 and relative L2 <= 5e-3 of the fp32 oracle when the
kernel writes fp32.  For bf16 output the bf16 rounding of the result itself
is added to the absolute bound (half an ulp of the reference value).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import layout as lay  # noqa: E402
from oracle import linear4bit as l4  # noqa: E402
from oracle import mlp as om  # noqa: E402
from oracle import router as orr  # noqa: E402
from oracle import synthetic as syn  # noqa: E402
from oracle.nf4 import bf16_round  # noqa: E402

MAX_ABS = 2e-2
REL_L2 = 5e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from next_step_ai_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def T(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


def assert_close(got, ref, *, bf16_out=False):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    bound = MAX_ABS + (np.abs(ref) * 2.0 ** -8 if bf16_out else 0.0)
    err = np.abs(got - ref)
    assert rel <= REL_L2, f"relative L2 {rel:.3e} > {REL_L2}"
    assert np.all(err <= bound), f"max abs err {err.max():.3e} (bound {MAX_ABS})"
    return rel, float(err.max())


def router_for(shape, R, dev, dtype=torch.bfloat16, **kw):
    from next_step_ai_b200 import RouterWeights

    return RouterWeights(enc_w=T(R["enc_w"], dev, dtype), score_w=T(R["score_w"], dev, dtype),
                         enc_b=T(R["enc_b"], dev, dtype), score_b=T(R["score_b"], dev, dtype),
                         top_k=kw.pop("top_k", shape.top_k), basis_top_k=kw.pop("basis_top_k", shape.rank), **kw)


def weights_for(shape, full, dev):
    from next_step_ai_b200 import SparseMlpWeights

    return SparseMlpWeights.from_bnb_rowmajor(
        hidden=shape.hidden, intermediate=shape.intermediate, gate_packed=T(full["gate_packed"], dev),
        gate_absmax=T(full["gate_absmax"], dev), up_packed=T(full["up_packed"], dev),
        up_absmax=T(full["up_absmax"], dev), down_packed=T(full["down_packed"], dev),
        down_absmax=T(full["down_absmax"], dev), code=T(full["code"], dev))


_FULL_CACHE: dict = {}


def full_layer(name, seed):
    key = (name, seed)
    if key not in _FULL_CACHE:
        _FULL_CACHE[key] = syn.make_layer_full(syn.SHAPES[name], seed)
    return _FULL_CACHE[key]


# --------------------------------------------------------------------------- router
@pytest.mark.parametrize("name,rows", [("tiny", 3), ("small", 2), ("cfg0", 4), ("cfg1", 4)])
def test_router_bit_exact(dev, name, rows):
    from next_step_ai_b200 import route_sparse_mlp

    shape = syn.SHAPES[name]
    for seed in (0, 1):
        R = syn.make_router(shape, seed)
        x = syn.make_x(shape, seed, rows)
        ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)
        got, scores = route_sparse_mlp(T(x, dev, torch.bfloat16), router_for(shape, R, dev), return_scores=True)
        assert np.array_equal(got.cpu().numpy(), ref), (name, seed)
        lat = orr.basis_latent(x, R["enc_w"], R["enc_b"], shape.rank)
        s_ref = orr.block_scores(lat, R["score_w"], R["score_b"])
        s_ref_sel = np.take_along_axis(s_ref, ref, axis=1)
        assert np.allclose(scores.cpu().numpy(), s_ref_sel, rtol=1e-4, atol=1e-5)


def test_router_rows_match_single_row_calls(dev):
    """nsm_route_rows (all rows in three launches) gives, per row, the bits of
    nsm_route on that row alone, and the oracle's indices."""
    from next_step_ai_b200 import route_sparse_mlp

    shape = syn.SHAPES["cfg1"]
    R = syn.make_router(shape, 9)
    rows = 37
    x = syn.make_x(shape, 9, rows, shared=0.6)
    rw = router_for(shape, R, dev)
    xd = T(x, dev, torch.bfloat16)
    got, scores = route_sparse_mlp(xd, rw, return_scores=True)
    for r in range(rows):
        one, s_one = route_sparse_mlp(xd[r:r + 1], rw, return_scores=True)
        assert torch.equal(one, got[r:r + 1]), r
        assert torch.equal(s_one, scores[r:r + 1]), r
    ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)
    assert np.array_equal(got.cpu().numpy(), ref)
    # ties across several rows resolve to the lower block id in every row
    H, r_, NB = 128, 8, 40
    sb = np.zeros(NB, np.float32)
    sb[[3, 7, 11, 30]] = 1.0
    sb[[5, 9]] = 2.0
    from next_step_ai_b200 import RouterWeights

    tw = RouterWeights(enc_w=T(np.zeros((r_, H), np.float32), dev), score_w=T(np.zeros((NB, r_), np.float32), dev),
                       score_b=T(sb, dev), top_k=8, basis_top_k=r_)
    tie = route_sparse_mlp(torch.ones(5, H, device=dev), tw).cpu().numpy()
    assert all(row.tolist() == [5, 9, 3, 7, 11, 30, 0, 1] for row in tie)


def test_router_golden_cfg1(dev, golden):
    """Indices pinned by the reference's own _route_sparse_mlp (fp32)."""
    from next_step_ai_b200 import route_sparse_mlp

    cases = {c["name"]: c for c in json.loads(bytes(golden["router/cases.json"]).decode())}
    for name in ("cfg0_r1", "cfg0_r8", "cfg1_r1", "cfg1_r4"):
        c = cases[name]
        shape = syn.SHAPES[c["shape"]]
        R = syn.make_router(shape, c["seed"])
        x = syn.make_x(shape, c["seed"], c["rows"])
        got = route_sparse_mlp(T(x, dev, torch.bfloat16), router_for(shape, R, dev))
        assert np.array_equal(got.cpu().numpy(), golden[f"router/{name}/idx"]), name


def test_router_fp32_weights_and_variants(dev):
    from next_step_ai_b200 import route_sparse_mlp

    shape = syn.SHAPES["small"]
    R = syn.make_router(shape, 4)
    x = syn.make_x(shape, 4, 3)
    xd = T(x, dev, torch.float32)
    # fp32 router weights
    got = route_sparse_mlp(xd, router_for(shape, R, dev, torch.float32))
    ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)
    assert np.array_equal(got.cpu().numpy(), ref)
    # basis top-k < rank
    got = route_sparse_mlp(xd, router_for(shape, R, dev, torch.float32, basis_top_k=7))
    ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, 7)
    assert np.array_equal(got.cpu().numpy(), ref)
    # down_block_norm
    dbn = np.random.default_rng(3).uniform(0.5, 1.5, shape.num_blocks).astype(np.float32)
    got = route_sparse_mlp(xd, router_for(shape, R, dev, torch.float32, down_block_norm=T(dbn, dev)))
    ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank,
                               down_block_norm=dbn)
    assert np.array_equal(got.cpu().numpy(), ref)
    # prefill-style k override, and k clamped to NB
    got = route_sparse_mlp(xd, router_for(shape, R, dev, torch.float32), top_k=5)
    ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], 5, shape.rank)
    assert np.array_equal(got.cpu().numpy(), ref)
    got = route_sparse_mlp(xd, router_for(shape, R, dev, torch.float32), top_k=10 ** 6)
    assert got.shape[1] == shape.num_blocks
    ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.num_blocks, shape.rank)
    assert np.array_equal(got.cpu().numpy(), ref)


def test_router_legacy_abs_latent(dev):
    from next_step_ai_b200 import RouterWeights, route_sparse_mlp

    shape = syn.SHAPES["small"]
    R = syn.make_router(shape, 6)
    x = syn.make_x(shape, 6, 2)
    dnt = np.abs(np.random.default_rng(7).standard_normal((shape.rank, shape.num_blocks))).astype(np.float32)
    rw = RouterWeights(enc_w=T(R["enc_w"], dev), score_w=T(dnt.T, dev), enc_b=T(R["enc_b"], dev),
                       top_k=shape.top_k, basis_top_k=shape.rank, legacy_abs_latent=True)
    got = route_sparse_mlp(T(x, dev, torch.float32), rw)
    ref = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], None, None, shape.top_k, shape.rank, dec_norm_t=dnt)
    assert np.array_equal(got.cpu().numpy(), ref)


def test_router_tie_break_lower_index(dev):
    from next_step_ai_b200 import RouterWeights, route_sparse_mlp

    # all-zero score head: every score is clamp0(bias); equal biases tie
    H, r, NB = 128, 8, 40
    enc = np.zeros((r, H), np.float32)
    sw = np.zeros((NB, r), np.float32)
    sb = np.zeros(NB, np.float32)
    sb[[3, 7, 11, 30]] = 1.0
    sb[[5, 9]] = 2.0
    rw = RouterWeights(enc_w=T(enc, dev), score_w=T(sw, dev), score_b=T(sb, dev), top_k=8, basis_top_k=r)
    got = route_sparse_mlp(torch.ones(1, H, device=dev), rw).cpu().numpy()[0]
    assert got.tolist() == [5, 9, 3, 7, 11, 30, 0, 1]


@pytest.mark.parametrize("name,seed", [("small", 31), ("cfg0", 32)])
def test_decode_fused_selection_matches_topk_kernel(dev, name, seed):
    """Without idx_out the gate/up kernel selects the blocks itself (no top-k
    kernel); asking for idx_out runs the top-k kernel.  Same blocks, same
    block-id order of the pool rows: the outputs must be bit-identical."""
    from next_step_ai_b200 import sparse_mlp_decode

    shape = syn.SHAPES[name]
    w = weights_for(shape, full_layer(name, seed), dev)
    rw = router_for(shape, syn.make_router(shape, seed), dev)
    x = T(syn.make_x(shape, seed, 1)[0], dev, torch.bfloat16)
    y_fused = sparse_mlp_decode(x, rw, w, out_dtype=torch.float32)
    idx = torch.empty(shape.top_k, dtype=torch.int32, device=dev)
    y_topk = sparse_mlp_decode(x, rw, w, out_dtype=torch.float32, idx_out=idx)
    assert torch.equal(y_fused, y_topk)


def test_decode_fused_selection_matches_topk_kernel_cfg1(dev):
    """The same at the 405B shape the benchmark runs (1664 keys, k = 208):
    the selection inside the gate/up kernel and the top-k kernel give
    bit-identical outputs for several inputs, and the top-k kernel's indices
    equal the oracle router's."""
    from next_step_ai_b200 import sparse_mlp_decode
    from next_step_ai_b200 import synthetic as dsyn

    shape = dsyn.SHAPES["cfg1"]
    w = dsyn.make_layer_weights(shape, 3, 0, dev)
    rw = dsyn.make_router(shape, 3, 0, dev)
    R = {k: v.float().cpu().numpy() for k, v in
         (("enc_w", rw.enc_w), ("enc_b", rw.enc_b), ("score_w", rw.score_w), ("score_b", rw.score_b))}
    xs = dsyn.make_x(shape, 5, 4, dev)
    idx = torch.empty(shape.top_k, dtype=torch.int32, device=dev)
    for r in range(xs.shape[0]):
        y_fused = sparse_mlp_decode(xs[r], rw, w, out_dtype=torch.float32)
        y_topk = sparse_mlp_decode(xs[r], rw, w, out_dtype=torch.float32, idx_out=idx)
        assert torch.equal(y_fused, y_topk), r
        ref = orr.route_sparse_mlp(xs[r].float().cpu().numpy(), R["enc_w"], R["enc_b"], R["score_w"], R["score_b"],
                                   shape.top_k, shape.rank)[0]
        assert np.array_equal(idx.cpu().numpy(), ref), r


def test_decode_fused_selection_many_blocks(dev):
    """4096 blocks, more keys than the gate/up CTA holds in registers (8 per
    thread), so the fused selection takes its shared-memory radix select: the
    outputs equal the top-k kernel path's bit for bit and its indices equal
    the oracle router's."""
    from next_step_ai_b200 import sparse_mlp_decode
    from next_step_ai_b200 import synthetic as dsyn

    shape = dsyn.LayerShape(256, 4096 * 32, 300, 64)
    w = dsyn.make_layer_weights(shape, 7, 0, dev)
    rw = dsyn.make_router(shape, 7, 0, dev)
    R = {k: v.float().cpu().numpy() for k, v in
         (("enc_w", rw.enc_w), ("enc_b", rw.enc_b), ("score_w", rw.score_w), ("score_b", rw.score_b))}
    xs = dsyn.make_x(shape, 9, 3, dev)
    idx = torch.empty(shape.top_k, dtype=torch.int32, device=dev)
    for r in range(xs.shape[0]):
        y_fused = sparse_mlp_decode(xs[r], rw, w, out_dtype=torch.float32)
        y_topk = sparse_mlp_decode(xs[r], rw, w, out_dtype=torch.float32, idx_out=idx)
        assert torch.equal(y_fused, y_topk), r
        ref = orr.route_sparse_mlp(xs[r].float().cpu().numpy(), R["enc_w"], R["enc_b"], R["score_w"], R["score_b"],
                                   shape.top_k, shape.rank)[0]
        assert np.array_equal(idx.cpu().numpy(), ref), r


def test_decode_fused_selection_splits_ties_by_block_id(dev):
    """Tied scores at the threshold (all-zero score head, biases 2, 2, 1, 1, 1,
    1 and zeros): the fused selection keeps the lower block ids among the tied
    zeros, like the top-k kernel, and the MLP matches the oracle on that set."""
    from next_step_ai_b200 import RouterWeights, sparse_mlp_decode

    shape = syn.SHAPES["tiny"]
    full = full_layer("tiny", 33)
    w = weights_for(shape, full, dev)
    H, r, NB, k = shape.hidden, 8, shape.num_blocks, 8
    sb = np.zeros(NB, np.float32)
    sb[[3, 7, 11, 20]] = 1.0
    sb[[5, 9]] = 2.0
    rw = RouterWeights(enc_w=T(np.zeros((r, H), np.float32), dev), score_w=T(np.zeros((NB, r), np.float32), dev),
                       score_b=T(sb, dev), top_k=k, basis_top_k=r)
    xh = syn.make_x(shape, 34, 1)[0]
    x = T(xh, dev, torch.bfloat16)
    y_fused = sparse_mlp_decode(x, rw, w, out_dtype=torch.float32)
    idx = torch.empty(k, dtype=torch.int32, device=dev)
    y_topk = sparse_mlp_decode(x, rw, w, out_dtype=torch.float32, idx_out=idx)
    assert idx.cpu().numpy().tolist() == [5, 9, 3, 7, 11, 20, 0, 1]
    assert torch.equal(y_fused, y_topk)
    blocks = np.array([0, 1, 3, 5, 7, 9, 11, 20], np.int64)
    ref = om.sparse_mlp_full(bf16_round(xh), blocks, full["gate_packed"], full["gate_absmax"], full["up_packed"],
                             full["up_absmax"], full["down_packed"], full["down_absmax"], full["code"],
                             hidden=shape.hidden, intermediate=shape.intermediate)[0]
    assert_close(y_fused.cpu().numpy(), ref)


# --------------------------------------------------------------------------- decode, resident weights
@pytest.mark.parametrize("name,seed", [("tiny", 11), ("small", 12), ("cfg0", 0)])
def test_decode_resident_matches_oracle(dev, name, seed):
    from next_step_ai_b200 import sparse_mlp_decode

    shape = syn.SHAPES[name]
    full = full_layer(name, seed)
    R = syn.make_router(shape, seed)
    w = weights_for(shape, full, dev)
    rw = router_for(shape, R, dev)
    for rowseed in range(2):
        x = syn.make_x(shape, seed * 10 + rowseed, 1)[0]
        idx = torch.empty(shape.top_k, dtype=torch.int32, device=dev)
        y = sparse_mlp_decode(T(x, dev, torch.bfloat16), rw, w, out_dtype=torch.float32, idx_out=idx)
        ref_idx = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k,
                                       shape.rank)[0]
        assert np.array_equal(idx.cpu().numpy(), ref_idx)
        ref = om.sparse_mlp_full(x, ref_idx, full["gate_packed"], full["gate_absmax"], full["up_packed"],
                                 full["up_absmax"], full["down_packed"], full["down_absmax"], full["code"],
                                 hidden=shape.hidden, intermediate=shape.intermediate)[0]
        assert_close(y.cpu().numpy(), ref)
        yb = sparse_mlp_decode(T(x, dev, torch.bfloat16), rw, w, out_dtype=torch.bfloat16)
        assert_close(yb.float().cpu().numpy(), ref, bf16_out=True)


def test_decode_cfg1_device_generated(dev):
    """Full 405B-shaped layer generated on the GPU; the oracle checks the
    selected blocks copied back to the host."""
    from next_step_ai_b200 import sparse_mlp_decode
    from next_step_ai_b200 import synthetic as dsyn

    shape = dsyn.SHAPES["cfg1"]
    w, bnb = dsyn.make_layer_weights(shape, 0, 0, dev, keep_bnb=True)
    rw = dsyn.make_router(shape, 0, 0, dev)
    x = dsyn.make_x(shape, 0, 1, dev)[0]
    idx = torch.empty(shape.top_k, dtype=torch.int32, device=dev)
    y = sparse_mlp_decode(x, rw, w, out_dtype=torch.float32, idx_out=idx)
    torch.cuda.synchronize()
    sel = idx.cpu().numpy().astype(np.int64)
    xn = x.float().cpu().numpy()
    ref_idx = orr.route_sparse_mlp(xn, rw.enc_w.float().cpu().numpy(), rw.enc_b.float().cpu().numpy(),
                                   rw.score_w.float().cpu().numpy(), rw.score_b.float().cpu().numpy(), shape.top_k,
                                   shape.rank)[0]
    assert np.array_equal(sel, ref_idx)
    H, I = shape.hidden, shape.intermediate
    gm = om.Nf4ParamMeta(I, H)
    dmeta = om.Nf4ParamMeta(H, I)
    s = torch.from_numpy(sel).to(dev)
    gp = bnb["gate_packed"].view(-1, gm.bytes_per_block)[s].cpu().numpy()
    ga = bnb["gate_absmax"].view(-1, gm.absmax_per_block)[s].cpu().numpy()
    upk = bnb["up_packed"].view(-1, gm.bytes_per_block)[s].cpu().numpy()
    ua = bnb["up_absmax"].view(-1, gm.absmax_per_block)[s].cpu().numpy()
    # the reference's down column gather, done on the device for speed
    dcols = bnb["down_packed"].view(H, dmeta.bytes_per_row)[:, None, :].view(H, -1, 16)[:, s].contiguous().cpu().numpy()
    dabs = bnb["down_absmax"].view(H, dmeta.absmax_per_row)[:, s // 2].contiguous().cpu().numpy()
    code = bnb["code"].cpu().numpy()
    ref = om.sparse_mlp_gathered(xn, gp, ga, code, upk, ua, code, dcols, dabs, code)[0]
    assert_close(y.cpu().numpy(), ref)


def test_decode_explicit_idx_and_shards_sum(dev):
    from next_step_ai_b200 import sparse_mlp_decode

    shape = syn.SHAPES["small"]
    full = full_layer("small", 21)
    w = weights_for(shape, full, dev)
    x = syn.make_x(shape, 21, 1)[0]
    sel = np.array([0, 127, 5, 64, 63, 17, 90], np.int64)
    xd = T(x, dev, torch.bfloat16)
    y = sparse_mlp_decode(xd, None, w, idx=T(sel, dev), out_dtype=torch.float32).cpu().numpy()
    ref = om.sparse_mlp_full(x, sel, full["gate_packed"], full["gate_absmax"], full["up_packed"], full["up_absmax"],
                             full["down_packed"], full["down_absmax"], full["code"], hidden=shape.hidden,
                             intermediate=shape.intermediate)[0]
    assert_close(y, ref)
    # four shards over [0, NB): each pool holds its own blocks only
    nb = shape.num_blocks
    acc = np.zeros_like(ref)
    for lo in range(0, nb, nb // 4):
        hi = lo + nb // 4
        from next_step_ai_b200 import SparseMlpWeights

        ws = SparseMlpWeights(hidden=w.hidden, intermediate=w.intermediate, gate_packed=w.gate_packed[lo:hi].clone(),
                              gate_absmax=w.gate_absmax[lo:hi].clone(), up_packed=w.up_packed[lo:hi].clone(),
                              up_absmax=w.up_absmax[lo:hi].clone(), down_packed=w.down_packed[lo:hi].clone(),
                              down_absmax=w.down_absmax[lo:hi].clone(), gate_code=w.gate_code, up_code=w.up_code,
                              down_code=w.down_code, layout=w.layout)
        acc += sparse_mlp_decode(xd, None, ws, idx=T(sel, dev), block_range=(lo, hi),
                                 out_dtype=torch.float32).cpu().numpy()
    assert_close(acc, ref)


def untile_gateup(packed, absmax, H):
    """numpy inverse of the tiled gate/up layout (include/nsm.h) for one block."""
    p = packed.reshape(H // 64, 2, 8, 4, 2, 8)  # tile, rg, g, t, half(row g / g+8), byte
    rows = np.zeros((32, H // 2), np.uint8)
    for rg in range(2):
        for h in range(2):
            for g in range(8):
                r = rg * 16 + g + 8 * h
                rows[r] = p[:, rg, g, :, h, :].reshape(-1)
    a = absmax.reshape(H // 64, 8, 4)
    am = np.zeros((32, H // 64), np.float32)
    for g in range(8):
        for i in range(4):
            am[(i >> 1) * 16 + g + (i & 1) * 8] = a[:, g, i]
    return rows.reshape(-1), am.reshape(-1)


def untile_down(packed, absmax, H):
    p = packed.reshape(H // 32, 8, 4, 4, 4)  # rt, g, t, i(row), byte
    cols = np.zeros((H, 16), np.uint8)
    am = np.zeros(H, np.float32)
    a = absmax.reshape(H // 32, 8, 4)
    for i in range(4):
        for g in range(8):
            r = np.arange(H // 32) * 32 + (i >> 1) * 16 + g + (i & 1) * 8
            cols[r] = p[:, g, :, i, :].reshape(H // 32, 16)
            am[r] = a[:, g, i]
    return cols, am


def test_tiled_repack_round_trip(dev):
    shape = syn.SHAPES["small"]
    full = full_layer("small", 12)
    w = weights_for(shape, full, dev)
    assert w.layout == 3
    H, I = shape.hidden, shape.intermediate
    gm = om.Nf4ParamMeta(I, H)
    dm = om.Nf4ParamMeta(H, I)
    for b in (0, 7, shape.num_blocks - 1):
        gp, ga = untile_gateup(w.gate_packed[b].cpu().numpy(), w.gate_absmax[b].cpu().numpy(), H)
        ref_p, ref_a = om.gather_row_blocks(full["gate_packed"], full["gate_absmax"], gm, [b])
        assert np.array_equal(gp, ref_p[0]) and np.array_equal(ga, ref_a[0])
        up, ua = untile_gateup(w.up_packed[b].cpu().numpy(), w.up_absmax[b].cpu().numpy(), H)
        ref_p, ref_a = om.gather_row_blocks(full["up_packed"], full["up_absmax"], gm, [b])
        assert np.array_equal(up, ref_p[0]) and np.array_equal(ua, ref_a[0])
        dc, da = untile_down(w.down_packed[b].cpu().numpy(), w.down_absmax[b].cpu().numpy(), H)
        rc, ra = om.gather_down_cols(full["down_packed"], full["down_absmax"], dm, [b])
        assert np.array_equal(dc, rc[:, 0]) and np.array_equal(da, ra[:, 0])


def test_row_major_and_tiled_layouts_agree(dev):
    from next_step_ai_b200 import SparseMlpWeights, sparse_mlp_decode

    shape = syn.SHAPES["cfg0"]
    full = full_layer("cfg0", 0)
    rw = router_for(shape, syn.make_router(shape, 0), dev)
    xd = T(syn.make_x(shape, 5, 1)[0], dev, torch.bfloat16)
    kw = dict(hidden=shape.hidden, intermediate=shape.intermediate, gate_packed=T(full["gate_packed"], dev),
              gate_absmax=T(full["gate_absmax"], dev), up_packed=T(full["up_packed"], dev),
              up_absmax=T(full["up_absmax"], dev), down_packed=T(full["down_packed"], dev),
              down_absmax=T(full["down_absmax"], dev), code=T(full["code"], dev))
    a = sparse_mlp_decode(xd, rw, SparseMlpWeights.from_bnb_rowmajor(tiled=True, **kw), out_dtype=torch.float32)
    b = sparse_mlp_decode(xd, rw, SparseMlpWeights.from_bnb_rowmajor(tiled=False, **kw), out_dtype=torch.float32)
    # same products; the tiled layout's down kernel reduces 64-row groups, the
    # row-major one 32-row tiles, so the split of the block sum into segments
    # (and only the fp32 rounding of the sums) differs
    assert torch.allclose(a, b, rtol=1e-5, atol=1e-5), float((a - b).abs().max())


def test_decode_edge_cases(dev):
    from next_step_ai_b200 import sparse_mlp_decode

    shape = syn.SHAPES["tiny"]
    full = full_layer("tiny", 3)
    w = weights_for(shape, full, dev)
    x = syn.make_x(shape, 3, 1)[0]
    xd = T(x, dev, torch.bfloat16)
    args = (full["gate_packed"], full["gate_absmax"], full["up_packed"], full["up_absmax"], full["down_packed"],
            full["down_absmax"], full["code"])
    kw = dict(hidden=shape.hidden, intermediate=shape.intermediate)
    # k = 1 and k = all blocks
    for sel in (np.array([9]), np.arange(shape.num_blocks)):
        y = sparse_mlp_decode(xd, None, w, idx=T(sel, dev), out_dtype=torch.float32).cpu().numpy()
        assert_close(y, om.sparse_mlp_full(x, sel, *args, **kw)[0])
    # invalid ids are skipped (they are not present in the pool)
    sel = np.array([-1, 4, 10 ** 6, 7], np.int64)
    y = sparse_mlp_decode(xd, None, w, idx=T(sel, dev), out_dtype=torch.float32).cpu().numpy()
    assert_close(y, om.sparse_mlp_full(x, np.array([4, 7]), *args, **kw)[0])
    # a shard that holds none of the selected blocks returns zeros
    y = sparse_mlp_decode(xd, None, w, idx=T(np.array([1, 2]), dev), block_range=(10, 20),
                          out_dtype=torch.float32).cpu().numpy()
    assert np.all(y == 0)
    # bad shapes raise RuntimeError (no silent fallback)
    with pytest.raises(RuntimeError):
        sparse_mlp_decode(xd[:100], None, w, idx=T(np.array([1]), dev))


def test_misaligned_workspace_is_refused(dev):
    """The kernels stage x by bulk copies that need 16-byte aligned
    addresses; a workspace that is not 256-byte aligned is refused on the host
    (NSM_ERR_WORKSPACE) before anything is launched."""
    import ctypes

    from next_step_ai_b200 import _lib
    from next_step_ai_b200._torch import dtype_code, ptr, stream_handle

    lib = _lib.load()
    shape = syn.SHAPES["tiny"]
    full = full_layer("tiny", 3)
    w = weights_for(shape, full, dev)
    xd = T(syn.make_x(shape, 3, 1)[0], dev, torch.bfloat16)
    idx = T(np.array([1, 2]), dev).to(torch.int32)
    y = torch.empty(shape.hidden, dtype=torch.float32, device=dev)
    need = lib.nsm_decode_workspace_bytes(shape.hidden, shape.intermediate, 2, 1)
    buf = torch.zeros(need + 512, dtype=torch.uint8, device=dev)
    bm = _lib.BlockMapC()
    bm.block_begin, bm.block_end = 0, shape.intermediate // 32
    wc = w.to_c()

    def call(off):
        return lib.nsm_sparse_mlp_decode(ptr(xd), dtype_code(xd.dtype), shape.hidden, shape.intermediate, None, None,
                                         ptr(idx), 2, ctypes.byref(bm), ctypes.byref(wc), ptr(y),
                                         dtype_code(y.dtype), None, None, buf.data_ptr() + off, need,
                                         stream_handle(dev))

    for off in (8, 16, 128):
        assert call(off) == _lib.NSM_ERR_WORKSPACE, off
        assert b"256-byte aligned" in lib.nsm_last_error()
    assert call(256) == 0
    torch.cuda.synchronize()


def test_decode_deterministic(dev):
    from next_step_ai_b200 import sparse_mlp_decode

    shape = syn.SHAPES["cfg0"]
    full = full_layer("cfg0", 0)
    w = weights_for(shape, full, dev)
    rw = router_for(shape, syn.make_router(shape, 0), dev)
    xd = T(syn.make_x(shape, 0, 1)[0], dev, torch.bfloat16)
    a = sparse_mlp_decode(xd, rw, w, out_dtype=torch.float32)
    b = sparse_mlp_decode(xd, rw, w, out_dtype=torch.float32)
    assert torch.equal(a, b)


def test_decode_residual_rmsnorm(dev):
    from next_step_ai_b200 import sparse_mlp_decode

    shape = syn.SHAPES["small"]
    full = full_layer("small", 12)
    R = syn.make_router(shape, 12)
    w = weights_for(shape, full, dev)
    rw = router_for(shape, R, dev)
    rng = np.random.default_rng(1)
    resid = (rng.standard_normal(shape.hidden) * 3).astype(np.float32)
    yprev = bf16_round((rng.standard_normal(shape.hidden)).astype(np.float32))
    gamma = bf16_round(rng.uniform(0.5, 1.5, shape.hidden).astype(np.float32))
    r_d = T(resid, dev)
    idx = torch.empty(shape.top_k, dtype=torch.int32, device=dev)
    y = sparse_mlp_decode(None, rw, w, residual=r_d, y_prev=T(yprev, dev, torch.bfloat16),
                          norm_weight=T(gamma, dev, torch.bfloat16), eps=1e-5, out_dtype=torch.float32, idx_out=idx)
    r_ref = resid + yprev
    assert np.allclose(r_d.cpu().numpy(), r_ref, rtol=0, atol=0)
    xn = om.rms_norm(r_ref, gamma, 1e-5)
    ref_idx = orr.route_sparse_mlp(xn, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k,
                                   shape.rank)[0]
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    ref = om.sparse_mlp_full(xn, ref_idx, full["gate_packed"], full["gate_absmax"], full["up_packed"],
                             full["up_absmax"], full["down_packed"], full["down_absmax"], full["code"],
                             hidden=shape.hidden, intermediate=shape.intermediate)[0]
    assert_close(y.cpu().numpy(), ref)


# --------------------------------------------------------------------------- reference-layout drop-ins
@pytest.mark.parametrize("name", ["tiny_k4", "small_k16", "cfg0_k56"])
def test_single_kernel_dropin_matches_reference_golden(dev, golden, name):
    """The drop-in for triton_sparse_mlp_decode_4bit_single_kernel_sm75 against
    the reference kernel's own output (Triton interpreter)."""
    from next_step_ai_b200 import triton_sparse_mlp as tsm

    case = {c["name"]: c for c in json.loads(bytes(golden["single/cases.json"]).decode())}[name]
    shape = syn.SHAPES[case["shape"]]
    blocks = golden[f"single/{name}/blocks"]
    G = syn.selected_blocks_gathered(shape, case["seed"], 0, blocks)
    x = syn.make_x(shape, case["seed"], 1)
    H, k = shape.hidden, case["k"]
    out = torch.empty((1, H), dtype=torch.float16, device=dev)
    acc = torch.zeros(H, dtype=torch.float32, device=dev)
    code = T(G["code"], dev)
    res = tsm.triton_sparse_mlp_decode_4bit_single_kernel_sm75(
        T(x, dev, torch.bfloat16), T(blocks, dev), T(G["gate_packed"], dev), T(G["gate_absmax"], dev), code,
        T(G["up_packed"], dev), T(G["up_absmax"], dev), code, T(G["down_cols"], dev), T(G["down_absmax_cols"], dev),
        code, out, acc, H, 32, 64, k)
    ref = golden[f"single/{name}/y"]
    assert_close(acc.cpu().numpy(), ref)
    assert res.shape == (1, H) and res.dtype == torch.float16
    with pytest.raises(RuntimeError, match="block_size=32"):
        tsm.triton_sparse_mlp_decode_4bit_single_kernel_sm75(
            T(x, dev, torch.bfloat16), T(blocks, dev), T(G["gate_packed"], dev), T(G["gate_absmax"], dev), code,
            T(G["up_packed"], dev), T(G["up_absmax"], dev), code, T(G["down_cols"], dev),
            T(G["down_absmax_cols"], dev), code, out, acc, H, 16, 64, k)


def test_gathered_rows_with_flat_mask(dev):
    from next_step_ai_b200 import decode_gathered_rows

    shape = syn.SHAPES["small"]
    rows = 5
    X = syn.make_x(shape, 33, rows, shared=0.8)
    R = syn.make_router(shape, 33)
    ab = orr.route_sparse_mlp(X, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)
    ordered, active_local, flat_mask, _ = lay.build_sparse_active_layout(ab, rows, 32, shape.num_blocks)
    G = syn.selected_blocks_gathered(shape, 33, 0, ordered)
    y = decode_gathered_rows(T(X, dev, torch.bfloat16), T(flat_mask, dev), gate_packed=T(G["gate_packed"], dev),
                             gate_absmax=T(G["gate_absmax"], dev), gate_code=T(G["code"], dev),
                             up_packed=T(G["up_packed"], dev), up_absmax=T(G["up_absmax"], dev),
                             up_code=T(G["code"], dev), down_packed=T(G["down_cols"], dev),
                             down_absmax=T(G["down_absmax_cols"], dev), down_code=T(G["code"], dev),
                             out_dtype=torch.float32)
    ref = om.sparse_mlp_gathered(X, G["gate_packed"], G["gate_absmax"], G["code"], G["up_packed"], G["up_absmax"],
                                 G["code"], G["down_cols"], G["down_absmax_cols"], G["code"], flat_mask=flat_mask)
    for r in range(rows):
        assert_close(y[r].cpu().numpy(), ref[r])


@pytest.mark.parametrize("name", ["in_a", "in_b", "in_c"])
def test_input_linear_4bit_matches_reference_golden(dev, golden, name):
    from next_step_ai_b200 import triton_sparse_mlp as tsm

    c = {c["name"]: c for c in json.loads(bytes(golden["lin4/cases.json"]).decode())}[name]
    p = f"lin4/{name}/"
    bias = T(golden[p + "bias"], dev) if (p + "bias") in golden.files else None
    out = tsm.triton_sparse_input_linear_4bit(
        T(golden[p + "x"], dev), T(golden[p + "idx"], dev), packed_weight=T(golden[p + "packed"], dev),
        absmax=T(golden[p + "absmax"], dev), code=T(golden["lin4/code"], dev), out_features=c["out_features"],
        in_features=c["in_features"], quant_block_size=64, bias=bias, block_size=c["block_size"])
    assert np.allclose(out.cpu().numpy(), golden[p + "y_tiled"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["out_a", "out_b", "out_c"])
def test_output_linear_4bit_matches_reference_golden(dev, golden, name):
    from next_step_ai_b200 import triton_sparse_mlp as tsm

    c = {c["name"]: c for c in json.loads(bytes(golden["lin4/cases.json"]).decode())}[name]
    p = f"lin4/{name}/"
    bias = T(golden[p + "bias"], dev) if (p + "bias") in golden.files else None
    out = tsm.triton_sparse_output_linear_4bit(
        T(golden[p + "x"], dev), T(golden[p + "idx"], dev), T(golden[p + "mask"], dev),
        packed_weight=T(golden[p + "packed"], dev), absmax=T(golden[p + "absmax"], dev),
        code=T(golden["lin4/code"], dev), input_dim=c["input_dim"], quant_block_size=64, bias=bias,
        block_size=c["block_size"])
    assert np.allclose(out.cpu().numpy(), golden[p + "y"], rtol=1e-5, atol=1e-5)


def test_fused_v1_composition_matches_oracle(dev):
    from next_step_ai_b200 import triton_sparse_mlp as tsm

    rng = np.random.default_rng(77)
    code = syn.nf4_code()
    rows, H, bs, nslots, k = 2, 64, 8, 4, 3
    width = nslots * bs

    def proj(n_elem):
        return (rng.integers(0, 256, size=n_elem // 2, dtype=np.uint8),
                rng.uniform(0.01, 0.1, size=n_elem // 64).astype(np.float32))

    gp, ga = proj(((H * bs + width + 127) // 128) * 128)
    upk, ua = proj(((H * bs + width + 127) // 128) * 128)
    dp, da = proj(width * H)
    x = rng.standard_normal((rows, H)).astype(np.float32)
    idx = np.array([[0, 2, 3], [1, 2, 0]], np.int32)
    mask = np.zeros((rows, width), np.float32)
    for r in range(rows):
        for s in idx[r]:
            mask[r, s * bs:(s + 1) * bs] = 1
    out = tsm.triton_fused_sparse_mlp_decode_4bit(
        T(x, dev), T(idx, dev), T(mask, dev), gate_packed_weight=T(gp, dev), gate_absmax=T(ga, dev),
        gate_code=T(code, dev), gate_input_dim=H, gate_quant_block_size=64, gate_bias=None,
        up_packed_weight=T(upk, dev), up_absmax=T(ua, dev), up_code=T(code, dev), up_input_dim=H,
        up_quant_block_size=64, up_bias=None, down_packed_weight=T(dp, dev), down_absmax=T(da, dev),
        down_code=T(code, dev), down_out_features=H, down_in_features=width, down_quant_block_size=64,
        down_bias=None, block_size=bs)
    ref = l4.fused_sparse_mlp_decode_4bit(
        x, idx, mask, gate={"packed": gp, "absmax": ga, "code": code, "input_dim": H, "quant_block_size": 64},
        up={"packed": upk, "absmax": ua, "code": code, "input_dim": H, "quant_block_size": 64},
        down={"packed": dp, "absmax": da, "code": code, "out_features": H, "in_features": width,
              "quant_block_size": 64}, block_size=bs)
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)


def test_no_kernel_recorded_a_wait_timeout(dev):
    """Every bounded device wait of the calls above completed: the error word
    of each cached workspace is still zero."""
    from next_step_ai_b200._torch import WORKSPACES

    torch.cuda.synchronize()
    errs = WORKSPACES.errors()
    assert errs and all(v == 0 for v in errs.values()), errs


# --------------------------------------------------------------------------- codebooks
def _scaled_code_layer(name, seed, dev):
    """A layer whose up projection uses a different 16-value codebook (the
    stored nibbles are unchanged, so only the dequantised up values differ)."""
    from next_step_ai_b200 import SparseMlpWeights

    shape = syn.SHAPES[name]
    full = full_layer(name, seed)
    code = full["code"]
    up_code = (code * np.float32(0.75)).astype(np.float32)
    w = SparseMlpWeights.from_bnb_rowmajor(
        hidden=shape.hidden, intermediate=shape.intermediate, gate_packed=T(full["gate_packed"], dev),
        gate_absmax=T(full["gate_absmax"], dev), up_packed=T(full["up_packed"], dev),
        up_absmax=T(full["up_absmax"], dev), down_packed=T(full["down_packed"], dev),
        down_absmax=T(full["down_absmax"], dev), code=T(code, dev), up_code=T(up_code, dev))
    return shape, full, code, up_code, w


def test_distinct_up_codebook_uses_two_tables(dev):
    """Gate and up codebooks that differ: the tiled gate/up kernel keeps two
    lookup tables (the shared-codebook variant does not apply) and matches the
    oracle evaluated with each projection's own codebook."""
    from next_step_ai_b200 import sparse_mlp_decode

    shape, full, code, up_code, w = _scaled_code_layer("small", 14, dev)
    assert not w._shared_code
    H, I = shape.hidden, shape.intermediate
    gm, dm = om.Nf4ParamMeta(I, H), om.Nf4ParamMeta(H, I)
    rng = np.random.default_rng(5)
    for _ in range(2):
        x = syn.make_x(shape, int(rng.integers(1 << 30)), 1)[0]
        blocks = np.sort(rng.choice(shape.num_blocks, shape.top_k, replace=False)).astype(np.int64)
        y = sparse_mlp_decode(T(x, dev, torch.bfloat16), None, w, idx=T(blocks.astype(np.int32), dev),
                              out_dtype=torch.float32)
        gp, ga = om.gather_row_blocks(full["gate_packed"], full["gate_absmax"], gm, blocks)
        upk, ua = om.gather_row_blocks(full["up_packed"], full["up_absmax"], gm, blocks)
        dc, da = om.gather_down_cols(full["down_packed"], full["down_absmax"], dm, blocks)
        ref = om.sparse_mlp_gathered(np.asarray(x, np.float32).reshape(1, -1), gp, ga, code, upk, ua, up_code,
                                     dc, da, code)[0]
        assert_close(y.cpu().numpy(), ref)


def test_false_shared_codebook_claim_is_rejected(dev):
    """NSM_LAYOUT_SHARED_CODE on weights whose codebooks differ: the gate/up
    kernel checks the claim, records NSM_ERR_INVALID_ARG and computes nothing."""
    from next_step_ai_b200 import _lib, sparse_mlp_decode
    from next_step_ai_b200._torch import WORKSPACES

    shape, full, code, up_code, w = _scaled_code_layer("small", 15, dev)
    WORKSPACES.errors()  # start clean
    w._shared_code = True  # the false claim
    x = syn.make_x(shape, 3, 1)[0]
    blocks = np.arange(shape.top_k, dtype=np.int32)
    sparse_mlp_decode(T(x, dev, torch.bfloat16), None, w, idx=T(blocks, dev), out_dtype=torch.float32)
    errs = list(WORKSPACES.errors().values())
    assert _lib.NSM_ERR_INVALID_ARG in errs, errs
