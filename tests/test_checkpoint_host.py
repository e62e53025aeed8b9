"""Host side of the checkpoint and router-artifact loaders (no GPU).

The bitsandbytes-format snapshot is written by ``oracle.bnb_checkpoint`` with
the seed the golden generator used, so the reference loader's recorded outputs
(``tests/golden/checkpoint.json``: weight map, quant-state grouping, packed
block reads) apply to the same bytes.  ``_derive_hot_blocks_for_layer`` cases
come from the reference too.  The nested absmax decode is checked against the
oracle's restatement bit for bit.
"""
from __future__ import annotations

import hashlib
import json
import warnings

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytest.importorskip("safetensors")

from oracle import bnb_checkpoint as bc  # noqa: E402
from oracle import synthetic as syn  # noqa: E402
from oracle.nf4 import nf4_code  # noqa: E402
from next_step_ai_b200 import checkpoint as ck  # noqa: E402
from next_step_ai_b200.cache import hot_cache_bytes_per_block  # noqa: E402

from tests.golden.make_golden import CHECKPOINT_SEED, CHECKPOINT_SHAPE, write_checkpoint_snapshot  # noqa: E402


@pytest.fixture(scope="module")
def golden_ck():
    from pathlib import Path

    return json.loads((Path(__file__).parent / "golden" / "checkpoint.json").read_text())


@pytest.fixture(scope="module")
def snapshot(tmp_path_factory):
    d = tmp_path_factory.mktemp("snap_index")
    expect = write_checkpoint_snapshot(d, index=True)
    return d, expect


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# --------------------------------------------------------------------------- nested statistics
def test_nested_absmax_roundtrip_and_decode():
    rng = np.random.default_rng(5)
    absmax = (np.abs(rng.standard_normal(3000)) * 0.05 + 0.01).astype(np.float32)
    table = bc.nested_table()
    q, scale, off = bc.nested_absmax_encode(absmax, table)
    dec = bc.nested_absmax_decode(q, scale, table, off)
    assert q.dtype == np.uint8 and scale.size == (absmax.size + 255) // 256
    assert np.max(np.abs(dec - absmax)) < 0.03 * np.max(np.abs(absmax - off)) + 1e-6  # table step <= 5.6 %
    aux = {"w.absmax": torch.from_numpy(q), "w.nested_absmax": torch.from_numpy(scale),
           "w.nested_quant_map": torch.from_numpy(table), "w.quant_map": torch.from_numpy(nf4_code()),
           "w.quant_state.bitsandbytes__nf4": torch.from_numpy(bc.quant_state_blob(
               {"quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [3000, 64],
                "nested_blocksize": 256, "nested_dtype": "float32", "nested_offset": float(off)}))}
    qs = ck.decode_quant_state(aux, "w")
    assert qs["absmax"].dtype == torch.float32
    assert np.array_equal(qs["absmax"].numpy().view(np.uint32), dec.view(np.uint32))


def test_decode_quant_state_errors():
    code = torch.from_numpy(nf4_code())
    with pytest.raises(RuntimeError, match="packed bitsandbytes"):
        ck.decode_quant_state({"w.absmax": torch.zeros(4), "w.quant_map": code}, "w")
    bad = torch.from_numpy(np.frombuffer(b"\xff\xfe{", np.uint8).copy())
    with pytest.raises(RuntimeError, match="malformed"):
        ck.decode_quant_state({"w.absmax": torch.zeros(4), "w.quant_state.bitsandbytes__nf4": bad}, "w")
    blob = torch.from_numpy(bc.quant_state_blob({"quant_type": "nf4", "blocksize": 64, "shape": [2, 64]}))
    with pytest.raises(RuntimeError, match="lacks 'quant_map'"):
        ck.decode_quant_state({"w.absmax": torch.zeros(2), "w.quant_state.bitsandbytes__nf4": blob}, "w")


# --------------------------------------------------------------------------- reader vs the reference loader
def test_reader_matches_reference_loader(golden_ck, snapshot):
    d, _ = snapshot
    assert golden_ck["shape"] == CHECKPOINT_SHAPE and golden_ck["seed"] == CHECKPOINT_SEED
    case = next(c for c in golden_ck["loader"] if c["index"])
    r = ck.Nf4Checkpoint(d)
    assert dict(sorted(r.weight_map.items())) == case["weight_map"]
    assert {k: sorted(v) for k, v in sorted(r.aux_names.items())} == case["aux"]
    for b in case["blocks"]:
        got = r.load_nf4_packed_blocks(b["name"], b["idx"], bytes_per_block=b["bytes_per_block"])
        assert list(got.shape) == b["shape"] and got.dtype == torch.uint8
        assert sha(got.numpy()) == b["sha"]
        w, aux = r.load_raw(b["name"])
        assert list(w.shape) == b["raw_shape"] and sorted(aux) == b["aux_keys"]


def test_reader_without_index_maps_first_shard(golden_ck, tmp_path):
    # the reference's own no-index path fails with the installed safetensors
    # (recorded in the fixture); the reader maps the first shard's names
    case = next(c for c in golden_ck["loader"] if not c["index"])
    assert "error" in case
    write_checkpoint_snapshot(tmp_path, index=False)
    from safetensors import safe_open

    first = sorted(tmp_path.glob("*.safetensors"))[0]
    with safe_open(str(first), framework="pt") as h:
        names = set(h.keys())
    r = ck.Nf4Checkpoint(tmp_path)
    assert set(r.weight_map) == names and set(r.weight_map.values()) == {first.name}
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(RuntimeError, match="No safetensors shards"):
        ck.Nf4Checkpoint(empty)


def test_load_param_recovers_bytes_and_absmax(snapshot):
    d, expect = snapshot
    shape = syn.SHAPES[CHECKPOINT_SHAPE]
    full = syn.make_layer_full(shape, CHECKPOINT_SEED, 1)
    r = ck.Nf4Checkpoint(d)
    ps = r.mlp_params(1)
    H, I = shape.hidden, shape.intermediate
    for proj, key, dims in (("gate", "gate", (I, H)), ("up", "up", (I, H)), ("down", "down", (H, I))):
        p = ps[proj]
        assert (p.out_features, p.in_features) == dims and p.blocksize == 64 and p.quant_type == "nf4"
        assert np.array_equal(p.packed.numpy(), full[f"{key}_packed"].reshape(-1))
        name = f"model.layers.1.mlp.{proj}_proj.weight"
        assert np.array_equal(p.absmax.numpy().view(np.uint32), expect[name].view(np.uint32))
        assert np.array_equal(p.code.numpy(), nf4_code())
        # nested statistics are lossy but close to the original absmax
        assert np.max(np.abs(p.absmax.numpy() - full[f"{key}_absmax"])) < 5e-3
        m = p.meta()
        assert m.bytes_per_block == 32 * dims[1] // 2 and m.absmax_per_block == 32 * dims[1] // 64


def test_packed_block_reads_match_whole_tensor(snapshot):
    d, _ = snapshot
    r = ck.Nf4Checkpoint(d)
    name = "model.layers.1.mlp.gate_proj.weight"
    w, _ = r.load_raw(name)
    shape = syn.SHAPES[CHECKPOINT_SHAPE]
    bpb = 16 * shape.hidden
    whole = w.reshape(-1).view(-1, bpb)
    for idx in ([5, 6, 7, 2, 3, 31, 0], [9], [], [4, 4, 1], list(range(32))[::-1]):
        got = r.load_nf4_packed_blocks(name, idx, bytes_per_block=bpb)
        assert got.shape == (len(idx), bpb) and torch.equal(got, whole[torch.tensor(idx, dtype=torch.long)])
    with pytest.raises(IndexError):
        r.load_nf4_packed_blocks(name, [32], bytes_per_block=bpb)
    with pytest.raises(RuntimeError, match="whole number"):
        r.load_nf4_packed_blocks(name, [0], bytes_per_block=bpb + 1)


def test_reader_context_releases_handles(snapshot):
    d, _ = snapshot
    with ck.Nf4Checkpoint(d) as r:
        r.load_raw("model.layers.0.mlp.up_proj.weight")
        assert r._handles
    assert not r._handles
    w, aux = r.load_raw("model.layers.0.mlp.up_proj.weight")   # reopens on demand
    assert w.dtype == torch.uint8 and aux


def test_load_param_plain_absmax_and_errors(tmp_path):
    shape = syn.SHAPES["tiny"]
    full = syn.make_layer_full(shape, 3, 0)
    params = bc.layer_params(full, shape.hidden, shape.intermediate, 0)
    bc.write_snapshot(tmp_path, params, shards=1, nested=False,
                      extra={"model.norm.weight": np.ones(shape.hidden, np.float32)})
    r = ck.Nf4Checkpoint(tmp_path)
    p = r.load_param("model.layers.0.mlp.gate_proj.weight")
    assert np.array_equal(p.absmax.numpy(), full["gate_absmax"])
    with pytest.raises(RuntimeError, match="expected quantized weights"):
        r.load_param("model.norm.weight")
    with pytest.raises(KeyError):
        r.load_param("model.layers.7.mlp.gate_proj.weight")


# --------------------------------------------------------------------------- hot blocks vs the reference
def _dec(v):
    if isinstance(v, dict) and set(v) == {"tensor"}:
        return torch.tensor(v["tensor"], dtype=torch.float32)
    if isinstance(v, dict) and set(v) == {"dict"}:
        return {k: _dec(x) for k, x in v["dict"].items()}
    return v


def test_hot_blocks_match_reference(golden_ck):
    ties = 0
    for c in golden_ck["hot_blocks"]:
        state = _dec(c["state"])
        got = ck.derive_hot_blocks(state, _dec(c["stats"]), _dec(c["importance"]), c["num_blocks"],
                                   runtime_top_k=c["runtime_top_k"], threshold=c["threshold"],
                                   limit_bytes=c["limit"], used_bytes=0, sparse_layers=c["routing_layers"],
                                   bytes_per_block=hot_cache_bytes_per_block(c["hidden"]))
        if c["hot"] is None:
            assert got is None
            continue
        assert got is not None and len(got) == len(c["hot"])
        if got.tolist() == c["hot"]:
            continue
        # only a tie at the capacity boundary may differ (torch.topk leaves
        # the order of equal scores unspecified): both picks hold every block
        # above the boundary score and otherwise only blocks at it
        s = ck.hot_block_scores(state, _dec(c["stats"]), _dec(c["importance"]), c["num_blocks"])
        edge = np.sort(s)[::-1][len(got) - 1]
        above, at = set(np.nonzero(s > edge)[0].tolist()), set(np.nonzero(s == edge)[0].tolist())
        for pick in (set(got.tolist()), set(c["hot"])):
            assert above <= pick and pick - above <= at, c
        ties += 1
    assert ties <= 2


# --------------------------------------------------------------------------- router artifact
def _artifact(shape, layers=(0, 1, 2), **cfg_over):
    g = np.random.default_rng(9)
    H, NB, r = shape.hidden, shape.num_blocks, shape.rank
    states = {}
    for li in layers:
        R = syn.make_router(shape, 5, li)
        states[str(li)] = {
            "encoder_weight": torch.from_numpy(R["enc_w"]), "encoder_bias": torch.from_numpy(R["enc_b"]),
            "score_weight": torch.from_numpy(R["score_w"]), "score_bias": torch.from_numpy(R["score_b"]),
            "block_importance": torch.from_numpy(g.random(NB).astype(np.float32)),
            "scale": torch.tensor(1.5), "samples": torch.tensor(4096.0),
            "rank_effective": torch.tensor(float(r - 3)), "explained_variance_ratio": torch.tensor(0.8),
        }
    cfg = {"artifact_target": "intermediate_block_scores", "block_size": 32, "num_blocks": NB, "basis_rank": r,
           "basis_top_k": r, "top_k_by_layer": {}, "basis_top_k_by_layer": {}}
    cfg.update(cfg_over)
    return {"config": cfg, "layer_selection": list(layers), "layer_states": states,
            "stats": {str(li): {"explained_variance_ratio": 0.8} for li in layers}}


def test_router_artifact_fields_and_overrides(tmp_path):
    shape = syn.SHAPES["tiny"]
    payload = _artifact(shape, top_k_by_layer={"1": 7, 2: 10_000}, basis_top_k_by_layer={"0": 3})
    path = tmp_path / "router.pt"
    torch.save(payload, path)
    a = ck.load_router_artifact(path, hidden=shape.hidden, intermediate=shape.intermediate, num_layers=4,
                                dtype=torch.bfloat16)
    NB, r = shape.num_blocks, shape.rank
    assert a.top_k == max(1, round(NB * 0.02)) and a.num_blocks == NB and a.layer_selection == {0, 1, 2}
    assert sorted(a.layers) == [0, 1, 2]
    assert a.layers[0].top_k == a.top_k and a.layers[1].top_k == 7 and a.layers[2].top_k == NB
    assert a.layers[0].basis_top_k == 3 and a.layers[1].basis_top_k == r - 3   # clamped to rank_effective
    R = syn.make_router(shape, 5, 1)
    rw = a.layers[1]
    assert rw.enc_w.dtype == torch.bfloat16 and rw.score_w.shape == (NB, r) and rw.down_block_norm is None
    assert np.array_equal(rw.enc_w.float().numpy(), R["enc_w"]) and np.array_equal(rw.score_b.float().numpy(),
                                                                                    R["score_b"])
    i1 = a.info[1]
    assert i1.scale == 1.5 and i1.samples == 4096.0 and i1.rank_effective == r - 3 and i1.block_domain == "intermediate"
    # the runtime's explicit top-k replaces the default, not the per-layer table
    b = ck.load_router_artifact(payload, hidden=shape.hidden, intermediate=shape.intermediate, num_layers=2,
                                sparse_top_k=5, sparse_basis_top_k=2)
    assert sorted(b.layers) == [0, 1] and b.layers[0].top_k == 5 and b.layers[1].top_k == 7
    assert b.layers[0].basis_top_k == 2 and b.layers[1].basis_top_k == 2


class _PickledNote:
    """An arbitrary class: the restricted unpickler refuses to build it."""

    def __init__(self, text: str):
        self.text = text


def test_router_artifact_restricted_unpickling(tmp_path):
    shape = syn.SHAPES["tiny"]
    payload = _artifact(shape, layers=(0,))
    payload["stats"]["note"] = _PickledNote("fitted elsewhere")
    torch.save(payload, tmp_path / "odd.pt")
    kw = dict(hidden=shape.hidden, intermediate=shape.intermediate, num_layers=2)
    with pytest.raises(RuntimeError, match="trusted=True"):
        ck.load_router_artifact(tmp_path / "odd.pt", **kw)
    assert sorted(ck.load_router_artifact(tmp_path / "odd.pt", trusted=True, **kw).layers) == [0]


def test_router_artifact_errors_and_domains():
    shape = syn.SHAPES["tiny"]
    H, I = shape.hidden, shape.intermediate
    kw = dict(hidden=H, intermediate=I, num_layers=4)
    p = _artifact(shape, layers=(0,))
    p["layer_states"]["0"]["encoder_weight"] = torch.zeros(shape.rank, H + 64)
    with pytest.raises(RuntimeError, match="encoder_weight has input dim"):
        ck.load_router_artifact(p, **kw)
    p = _artifact(shape, layers=(0,))
    del p["layer_states"]["0"]["score_weight"]
    with pytest.raises(RuntimeError, match="missing score_weight"):
        ck.load_router_artifact(p, **kw)
    p = _artifact(shape, layers=(0,))
    p["layer_states"]["0"]["score_weight"] = torch.zeros(shape.num_blocks, shape.rank + 1)
    with pytest.raises(RuntimeError, match="does not match basis_rank"):
        ck.load_router_artifact(p, **kw)
    p = _artifact(shape, layers=(0,))
    p["layer_states"]["0"]["score_weight"] = torch.zeros(shape.num_blocks // 2, shape.rank)
    with pytest.raises(RuntimeError, match="FFN blocks"):
        ck.load_router_artifact(p, **kw)
    p = _artifact(shape, layers=(0,))
    p["layer_states"]["0"]["score_bias"] = torch.zeros(3)
    with pytest.raises(RuntimeError, match="score_bias has 3 values"):
        ck.load_router_artifact(p, **kw)
    p = _artifact(shape, layers=(0,))
    p["layer_states"]["0"]["down_block_norm"] = torch.ones(5)
    with pytest.raises(RuntimeError, match="down_block_norm has 5 values"):
        ck.load_router_artifact(p, **kw)
    p = _artifact(shape, layers=(0, 1, 9))
    p["layer_states"]["1"] = {"artifact_target": "output_reconstruction", "block_domain": "output",
                              "decoder_blocks": torch.zeros(8, 32, 4)}
    p["layer_states"]["0"]["down_block_norm"] = torch.full((shape.num_blocks,), 2.0)
    p["layer_states"]["0"]["explained_variance_ratio"] = torch.tensor(0.1)
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        a = ck.load_router_artifact(p, **kw)
    assert sorted(a.layers) == [0] and a.output_domain_layers == [1] and a.low_evr_layers == [0]
    assert any("explained_variance_ratio" in str(x.message) for x in w)
    assert a.layers[0].down_block_norm.dtype == torch.float32


def test_router_artifact_matches_reference_constructor(golden_ck):
    """The reference constructor's artifact block, run on the same seeded
    artifacts when the fixture was made (``tests/golden/make_golden.py``)."""
    from tests.golden.make_golden import ARTIFACT_SHAPE, artifact_payload

    gold = golden_ck["artifact"]
    assert gold["shape"] == ARTIFACT_SHAPE
    shape = syn.SHAPES[ARTIFACT_SHAPE]
    for c in gold["cases"]:
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            a = ck.load_router_artifact(artifact_payload(c["case"]), hidden=shape.hidden,
                                        intermediate=shape.intermediate, num_layers=8,
                                        sparse_top_k=c["sparse_top_k"], sparse_basis_top_k=c["sparse_basis_top_k"],
                                        dtype=torch.float32, hot_blocks=c["hot"], hot_cache_limit_bytes=c["limit"])
        assert a.top_k == c["default_top_k"], c["case"]
        assert sorted(a.layer_selection) == c["layer_selection"]
        assert a.output_domain_layers == c["output_domain_layers"]
        assert sorted(str(k) for k in a.layers) == sorted(c["layers"])
        for k, ref in c["layers"].items():
            rw, info = a.layers[int(k)], a.info[int(k)]
            assert (rw.top_k, rw.basis_top_k, info.rank_effective) == (ref["top_k"], ref["basis_top_k"],
                                                                      ref["rank_effective"]), (c["case"], k)
            assert info.scale == ref["scale"] and info.explained_variance_ratio == pytest.approx(ref["evr"])
            assert info.num_blocks == ref["num_blocks"]
            assert (rw.score_b is not None) == ref["has_score_bias"]
            assert (rw.down_block_norm is not None) == ref["has_down_block_norm"]
            assert sha(rw.enc_w.numpy()) == ref["enc_w_sha"] and sha(rw.score_w.numpy()) == ref["score_w_sha"]
        ref_hot = {k: v for k, v in c["hot_blocks"].items() if k in c["layers"]}  # intermediate layers
        assert {str(k): v.tolist() for k, v in a.hot_blocks.items()} == ref_hot, c["case"]


def test_router_artifact_hot_blocks():
    shape = syn.SHAPES["tiny"]
    p = _artifact(shape)
    a = ck.load_router_artifact(p, hidden=shape.hidden, intermediate=shape.intermediate, num_layers=4,
                                hot_blocks=True, hot_cache_limit_bytes=200_000)
    bpb = hot_cache_bytes_per_block(shape.hidden)
    for n, li in enumerate(sorted(a.layers)):
        st = p["layer_states"][str(li)]
        exp = ck.derive_hot_blocks(st, p["stats"][str(li)], None, shape.num_blocks, runtime_top_k=a.top_k,
                                   limit_bytes=200_000, sparse_layers=n + 1, bytes_per_block=bpb)
        assert a.hot_blocks[li].tolist() == exp.tolist()
        assert np.all(np.diff(a.hot_blocks[li]) > 0)
