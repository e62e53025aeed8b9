"""Pins the CPU oracle against golden vectors produced by the reference itself.

The fixtures (``tests/golden/golden.npz``, ``cache_policy.json``) were written by
``tests/golden/make_golden.py`` from the reference's own functions and Triton
kernels (Triton CPU interpreter).  Inputs are regenerated from seeds and
checked byte for byte against the recorded SHA-256 before use.
"""
from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from oracle import cache_policy as cp
from oracle import layout as lay
from oracle import linear4bit as l4
from oracle import mlp as om
from oracle import router as orr
from oracle import synthetic as syn
from oracle.nf4 import bf16_round, dequantize_nf4, nf4_code, quantize_nf4

# Published NF4 table (QLoRA paper, appendix); parity does not depend on it
# because the table is an input everywhere, but the construction must match.
PUBLISHED_NF4 = [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
                 -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
                 0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
                 0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0]


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def cases(golden, key):
    return json.loads(bytes(golden[key]).decode())


def test_nf4_code_matches_published_table(golden):
    code = nf4_code()
    assert np.allclose(code, np.array(PUBLISHED_NF4, np.float32), atol=2e-7)
    assert np.array_equal(code, golden["nf4_code"])


def test_nf4_quantize_roundtrip_error_bounded():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(64 * 200) * 0.02).astype(np.float32)
    code = nf4_code()
    packed, absmax = quantize_nf4(w, code)
    deq = dequantize_nf4(packed, absmax, code)
    # nearest-code: error at most half the widest code gap times absmax
    gap = np.max(np.diff(code)) / 2
    assert np.all(np.abs(deq - w) <= gap * np.repeat(absmax, 64) + 1e-7)
    # each absmax element is represented exactly (code[15] == 1)
    blocks = w.reshape(-1, 64)
    am_idx = np.argmax(np.abs(blocks), axis=1)
    got = deq.reshape(-1, 64)[np.arange(blocks.shape[0]), am_idx]
    assert np.allclose(np.abs(got), absmax)


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 3.0e-5], np.float32)
    r = bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0 + 2 ** -6)
    assert np.all(np.abs(r - x) <= np.abs(x) * 2 ** -8)


@pytest.mark.parametrize("name", ["tiny_r1", "tiny_r4_basisk", "small_r1", "small_r3_dbn", "small_r2_legacy",
                                  "small_r1_prefill", "cfg0_r1", "cfg0_r8", "cfg1_r1", "cfg1_r4"])
def test_router_matches_reference(golden, name):
    case = {c["name"]: c for c in cases(golden, "router/cases.json")}[name]
    shape = syn.SHAPES[case["shape"]]
    R = syn.make_router(shape, case["seed"])
    x = syn.make_x(shape, case["seed"], case["rows"])
    assert sha(R["enc_w"], R["score_w"], R["score_b"], x) == case["input_sha"]
    kw = {}
    score_w, score_b = R["score_w"], R["score_b"]
    if case["variant"] == "down_block_norm":
        kw["down_block_norm"] = golden[f"router/{name}/down_block_norm"]
    if case["variant"] == "legacy":
        kw["dec_norm_t"] = golden[f"router/{name}/dec_norm_t"]
        score_w, score_b = None, None
    k = shape.top_k if case["prefill_top_k"] < 0 else case["prefill_top_k"]
    got = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], score_w, score_b, k, case["basis_top_k"], **kw)
    ref = golden[f"router/{name}/idx"]
    assert got.shape == ref.shape
    # bit-exact: same blocks in the same (score-descending) order
    assert np.array_equal(got, ref), (got, ref)


def test_router_margins_are_far_from_fp32_noise(golden):
    for c in cases(golden, "router/cases.json"):
        if c["variant"]:
            continue
        shape = syn.SHAPES[c["shape"]]
        R = syn.make_router(shape, c["seed"])
        x = syn.make_x(shape, c["seed"], c["rows"])
        m = orr.selection_margin(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, c["basis_top_k"])
        assert np.all(m > 1e-6), (c["name"], m)


def test_top_k_desc_tie_rule():
    v = np.array([[1.0, 3.0, 3.0, 0.0, 3.0, 2.0]])
    assert orr.top_k_desc(v, 4).tolist() == [[1, 2, 4, 5]]


@pytest.mark.parametrize("name", ["r1", "r1_hot", "r3", "r4_hot", "r2_invalid", "r32_cfg4like"])
def test_active_layout_matches_reference(golden, name):
    case = {c["name"]: c for c in cases(golden, "layout/cases.json")}[name]
    ab = golden[f"layout/{name}/active_blocks"]
    ordered, active_local, flat_mask, neurons = lay.build_sparse_active_layout(
        ab, case["rows"], case["block_size"], case["max_valid_blocks"], np.array(case["hot"], np.int64))
    assert np.array_equal(ordered, golden[f"layout/{name}/ordered"])
    assert np.array_equal(active_local, golden[f"layout/{name}/active_local"])
    assert np.array_equal(flat_mask, golden[f"layout/{name}/flat_mask"])
    assert np.array_equal(neurons, golden[f"layout/{name}/neurons"])


def test_bank_update_matches_reference(cache_policy_golden):
    for c in cache_policy_golden["bank"]:
        slots, ids, scores, active = cp.plan_fixed_capacity_bank_update(
            np.array(c["ids"], np.int64), np.array(c["scores"], np.float32), c["active"], c["capacity"],
            np.array(c["novel"], np.int64))
        assert slots.tolist() == c["out_slots"]
        assert ids.tolist() == c["out_ids"]
        assert np.array_equal(scores, np.array(c["out_scores"], np.float32))
        assert active == c["out_active"]


def test_bank_update_reference_unit_case():
    # the reference's own pinned case (tests/test_throughput_contract.py:308-321)
    slots, ids, scores, active = cp.plan_fixed_capacity_bank_update(
        np.array([10, 11, -1]), np.array([5.0, 1.0, 0.0], np.float32), 2, 3, np.array([20, 21]))
    assert active == 3 and slots.tolist() == [2, 1] and ids.tolist() == [10, 21, 20]
    assert scores[1] > 5.0 and scores[2] > 5.0


def test_calibration_hits_match_reference(cache_policy_golden):
    for c in cache_policy_golden["calibration"]:
        ab = np.array(c["active_blocks"], np.int64)
        counts = cp.record_calibration_hits(None, ab, c["num_blocks"], c["power"])
        counts = cp.record_calibration_hits(counts, ab[::-1], c["num_blocks"], c["power"])
        assert np.allclose(counts, np.array(c["counts"], np.float32), rtol=0, atol=1e-6)


def test_target_hot_blocks_match_reference(cache_policy_golden):
    for c in cache_policy_golden["target"]:
        got = cp.target_hot_blocks(layer_idx=c["layer_idx"], runtime_top_k=c["runtime_top_k"],
                                   count_slots=c["count_slots"], previous_hot_count=c["prev"],
                                   limit_bytes=c["limit"], used_bytes=c["used"], sparse_layers=c["layers"],
                                   bytes_per_block=c["bpb"])
        assert got == c["target"], c


def test_down_column_gather_matches_reference(golden):
    shape = syn.SHAPES["tiny"]
    full = syn.make_layer_full(shape, 31)
    assert sha(full["down_packed"], full["down_absmax"]).encode() == bytes(golden["down_cols/input_sha"])
    meta = om.Nf4ParamMeta(shape.hidden, shape.intermediate)
    cols, absc = om.gather_down_cols(full["down_packed"], full["down_absmax"], meta, golden["down_cols/blocks"])
    assert np.array_equal(cols, golden["down_cols/packed"])
    assert np.array_equal(absc, golden["down_cols/absmax"])


@pytest.mark.parametrize("name", ["tiny_k4", "small_k16", "cfg0_k56"])
def test_mlp_oracle_matches_reference_single_kernel(golden, name):
    case = {c["name"]: c for c in cases(golden, "single/cases.json")}[name]
    shape = syn.SHAPES[case["shape"]]
    R = syn.make_router(shape, case["seed"])
    x = syn.make_x(shape, case["seed"], 1)
    blocks = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], case["k"], shape.rank)[0]
    assert np.array_equal(blocks, golden[f"single/{name}/blocks"])
    G = syn.selected_blocks_gathered(shape, case["seed"], 0, blocks)
    assert sha(x, G["gate_packed"], G["gate_absmax"], G["up_packed"], G["up_absmax"], G["down_cols"],
               G["down_absmax_cols"]) == case["input_sha"]
    y = om.sparse_mlp_gathered(x, G["gate_packed"], G["gate_absmax"], G["code"], G["up_packed"], G["up_absmax"],
                               G["code"], G["down_cols"], G["down_absmax_cols"], G["code"])[0]
    ref = golden[f"single/{name}/y"]
    err = np.abs(y - ref)
    assert np.max(err) <= 1e-4 * max(1.0, float(np.max(np.abs(ref)))), np.max(err)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5


@pytest.mark.parametrize("name", ["in_a", "in_b", "in_c"])
def test_input_linear_4bit_matches_reference_kernels(golden, name):
    c = {c["name"]: c for c in cases(golden, "lin4/cases.json")}[name]
    p = f"lin4/{name}/"
    bias = golden[p + "bias"] if (p + "bias") in golden.files else None
    got = l4.sparse_input_linear_4bit(golden[p + "x"], golden[p + "idx"], golden[p + "packed"], golden[p + "absmax"],
                                      golden["lin4/code"], c["out_features"], c["in_features"], 64, bias,
                                      c["block_size"])
    assert np.allclose(got, golden[p + "y_tiled"], rtol=1e-5, atol=1e-5)
    assert np.allclose(got, golden[p + "y_atomic"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["out_a", "out_b", "out_c"])
def test_output_linear_4bit_matches_reference_kernel(golden, name):
    c = {c["name"]: c for c in cases(golden, "lin4/cases.json")}[name]
    p = f"lin4/{name}/"
    bias = golden[p + "bias"] if (p + "bias") in golden.files else None
    got = l4.sparse_output_linear_4bit(golden[p + "x"], golden[p + "idx"], golden[p + "mask"], golden[p + "packed"],
                                       golden[p + "absmax"], golden["lin4/code"], c["input_dim"], 64, bias,
                                       c["block_size"])
    assert np.allclose(got, golden[p + "y"], rtol=1e-5, atol=1e-5)


def test_block_major_repack_is_the_column_slices():
    shape = syn.SHAPES["tiny"]
    full = syn.make_layer_full(shape, 3)
    meta = om.Nf4ParamMeta(shape.hidden, shape.intermediate)
    bm, bma = om.down_block_major(full["down_packed"], full["down_absmax"], meta)
    cols, absc = om.gather_down_cols(full["down_packed"], full["down_absmax"], meta, np.array([7, 2]))
    assert np.array_equal(bm[7], cols[:, 0]) and np.array_equal(bm[2], cols[:, 1])
    assert np.array_equal(bma[7], absc[:, 0]) and np.array_equal(bma[2], absc[:, 1])


def test_block_generators_agree_with_full_layer():
    shape = syn.SHAPES["tiny"]
    full = syn.make_layer_full(shape, 9)
    blocks = np.array([0, 5, 31, 12])
    G = syn.selected_blocks_gathered(shape, 9, 0, blocks)
    meta_g = om.Nf4ParamMeta(shape.intermediate, shape.hidden)
    meta_d = om.Nf4ParamMeta(shape.hidden, shape.intermediate)
    gp, ga = om.gather_row_blocks(full["gate_packed"], full["gate_absmax"], meta_g, blocks)
    dc, da = om.gather_down_cols(full["down_packed"], full["down_absmax"], meta_d, blocks)
    assert np.array_equal(gp, G["gate_packed"]) and np.array_equal(ga, G["gate_absmax"])
    assert np.array_equal(dc, G["down_cols"]) and np.array_equal(da, G["down_absmax_cols"])


@pytest.mark.parametrize("name", ["tiny_r4_basisk", "small_r3_dbn", "small_r2_legacy", "small_r1_prefill", "cfg0_r8"])
def test_routing_dict_conversion_routes_like_reference(golden, name):
    """The reference's in-memory routing dict -> RouterWeights.from_routing ->
    the oracle router on the converted fields gives the reference's indices."""
    torch = pytest.importorskip("torch")
    from next_step_ai_b200.weights import RouterWeights

    case = {c["name"]: c for c in cases(golden, "router/cases.json")}[name]
    shape = syn.SHAPES[case["shape"]]
    R = syn.make_router(shape, case["seed"])
    x = syn.make_x(shape, case["seed"], case["rows"])
    routing = {"enc_w": torch.from_numpy(R["enc_w"]), "enc_b": torch.from_numpy(R["enc_b"]),
               "route_score_weight": torch.from_numpy(R["score_w"]),
               "route_score_bias": torch.from_numpy(R["score_b"]),
               "top_k": shape.top_k, "basis_top_k": case["basis_top_k"], "num_blocks": shape.num_blocks}
    if case["variant"] == "down_block_norm":
        routing["down_block_norm"] = torch.from_numpy(golden[f"router/{name}/down_block_norm"])
    if case["variant"] == "legacy":
        del routing["route_score_weight"], routing["route_score_bias"]
        routing["dec_norm_t"] = torch.from_numpy(golden[f"router/{name}/dec_norm_t"])
    prefill = case["prefill_top_k"] if case["prefill_top_k"] > 0 else None
    rw = RouterWeights.from_routing(routing, prefill_top_k=prefill)
    assert rw.legacy_abs_latent == (case["variant"] == "legacy")
    kw = {"down_block_norm": rw.down_block_norm.numpy()} if rw.down_block_norm is not None else {}
    if rw.legacy_abs_latent:
        kw["dec_norm_t"] = rw.score_w.t().numpy()
        sw, sb = None, None
    else:
        sw, sb = rw.score_w.numpy(), rw.score_b.numpy() if rw.score_b is not None else None
    got = orr.route_sparse_mlp(x, rw.enc_w.numpy(), rw.enc_b.numpy(), sw, sb, rw.top_k, rw.basis_top_k, **kw)
    assert np.array_equal(got, golden[f"router/{name}/idx"])


def test_routing_dict_k_resolution():
    torch = pytest.importorskip("torch")
    from next_step_ai_b200.weights import RouterWeights

    base = {"enc_w": torch.zeros(16, 64), "enc_b": torch.zeros(16), "route_score_weight": torch.zeros(40, 16)}
    assert RouterWeights.from_routing(base, sparse_runtime_top_k=0, sparse_top_k=7).top_k == 7
    assert RouterWeights.from_routing(base, sparse_runtime_top_k=9, sparse_top_k=7).top_k == 9
    assert RouterWeights.from_routing(dict(base, top_k=500)).top_k == 40
    assert RouterWeights.from_routing(dict(base, top_k=5), prefill_top_k=0).top_k == 1
    assert RouterWeights.from_routing(base).basis_top_k == 8
    assert RouterWeights.from_routing(base, layer_idx=3, basis_top_k_by_layer={3: 99}).basis_top_k == 16
    rw = RouterWeights.from_routing(dict(base, down_block_norm=torch.ones(39)))
    assert rw.down_block_norm is None and rw.score_b is None


@pytest.mark.parametrize("name", ["small", "cfg0"])
def test_cpu_torch_arm_matches_numpy_oracle(name):
    """The torch restatement bench.py times as the CPU arm computes what the
    numpy oracle computes: the same selected blocks, the same MLP output
    (fp32, up to summation order)."""
    import torch

    from oracle import cpu_torch as ct
    from oracle import mlp as om
    from oracle import router as orr

    shape = syn.SHAPES[name]
    R = syn.make_router(shape, 3)
    x = syn.make_x(shape, 4, 2)
    ref_idx = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in R.items() if v is not None}
    got_idx = ct.route(torch.from_numpy(x), t["enc_w"], t.get("enc_b"), t["score_w"], t.get("score_b"), shape.top_k)
    assert np.array_equal(got_idx.numpy(), ref_idx)
    G = syn.selected_blocks_gathered(shape, 3, 0, ref_idx[0])
    y_ref = om.sparse_mlp_gathered(x[:1], G["gate_packed"], G["gate_absmax"], G["code"], G["up_packed"],
                                   G["up_absmax"], G["code"], G["down_cols"], G["down_absmax_cols"], G["code"])
    g = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in G.items()}
    y = ct.mlp_gathered(torch.from_numpy(x[:1]), g["gate_packed"], g["gate_absmax"], g["up_packed"],
                        g["up_absmax"], g["down_cols"], g["down_absmax_cols"], g["code"]).numpy()
    assert np.allclose(y, y_ref, rtol=1e-4, atol=1e-4), float(np.abs(y - y_ref).max())
