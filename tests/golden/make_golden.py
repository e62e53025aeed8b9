"""Generate the golden fixtures in ``tests/golden/`` from the reference itself.

Runs ONLY in the build container, where the reference tree is mounted
read-only (path from ``NSM_REFERENCE_ROOT``).  It imports the reference's own
code and records its outputs on seeded synthetic inputs:

* ``StreamingLlamaRuntime._route_sparse_mlp`` (router, fp32) and
  ``_build_sparse_active_layout`` on a ``__new__``-built runtime, with a stub
  ``bitsandbytes`` module (bitsandbytes is not installed here; these two
  functions never call it);
* ``_plan_fixed_capacity_bank_update``, ``_record_hot_cache_calibration_blocks``,
  ``_target_hot_blocks_for_layer`` and ``_load_down_proj_cold_cols``;
* the reference's Triton kernels ``_sparse_mlp_decode_4bit_single_kernel_sm75``,
  ``_sparse_output_linear_4bit_kernel``, ``_sparse_input_linear_4bit_tiled_kernel``
  and ``_sparse_input_linear_4bit_atomic_kernel`` executed by Triton's CPU
  interpreter (``TRITON_INTERPRET=1``);
* ``checkpoint.json`` (argument ``checkpoint`` regenerates only this file):
  ``ShardedSafetensorLoader`` (weight map, quant-state grouping,
  ``load_nf4_packed_blocks``, ``_load_raw_for_param``) on a seeded
  bitsandbytes-format snapshot written by ``oracle.bnb_checkpoint``,
  ``_derive_hot_blocks_for_layer`` on a ``__new__``-built runtime, and the
  constructor's router-artifact block and the rebuild loop of
  ``calibrate_vram_hot_cache`` (both taken from the reference source when the
  fixture is made) run on seeded artifacts and hit counts, and the LM head's
  quant block-size rule.

Inputs come from ``oracle.synthetic`` (seeded).  Small inputs are stored in the
fixtures; large ones are stored as seeds plus a SHA-256 of the regenerated
bytes, so the tests can rebuild them and prove they are the same bytes.

Usage: ``NSM_REFERENCE_ROOT=/path/to/next_step_ai python tests/golden/make_golden.py [checkpoint]``
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import types
from collections import OrderedDict
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402

from oracle import synthetic as syn  # noqa: E402
from oracle.nf4 import nf4_code  # noqa: E402


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _stub_bitsandbytes() -> None:
    def mk(name):
        m = types.ModuleType(name)
        m.__path__ = []
        sys.modules[name] = m
        return m

    bnb = mk("bitsandbytes")
    f = mk("bitsandbytes.functional")
    mk("bitsandbytes.backends")
    mk("bitsandbytes.backends.cuda")
    ops = mk("bitsandbytes.backends.cuda.ops")
    ops._dequantize_4bit_impl = None
    f.QuantState = object
    f.dequantize_blockwise = None
    f.dequantize_4bit = None
    bnb.functional = f


def load_reference():
    root = os.environ.get("NSM_REFERENCE_ROOT")
    if not root or not Path(root).is_dir():
        raise SystemExit("set NSM_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, root)
    _stub_bitsandbytes()
    import torch  # noqa: F401
    from llama3_neuroplastic import triton_sparse_mlp as tsm
    from llama3_neuroplastic.experiments import streaming_llama_runtime as rt
    return rt, tsm


def new_runtime(rt):
    import torch
    r = rt.StreamingLlamaRuntime.__new__(rt.StreamingLlamaRuntime)
    r._sparse_basis_top_k_by_layer = {}
    r._sparse_runtime_top_k = 0
    r._sparse_top_k = 1
    r._traffic_current_phase = "decode"
    r.device = torch.device("cpu")
    r._mlp_hot_blocks_by_layer = {}
    return r


# --------------------------------------------------------------------------- router
def gen_router(rt, out: dict) -> None:
    import torch
    cases = []
    specs = [
        # name, shape, seed, rows, basis_top_k, variant
        ("tiny_r1", "tiny", 1, 1, None, None),
        ("tiny_r4_basisk", "tiny", 2, 4, 5, None),
        ("small_r1", "small", 3, 1, None, None),
        ("small_r3_dbn", "small", 4, 3, None, "down_block_norm"),
        ("small_r2_legacy", "small", 5, 2, None, "legacy"),
        ("small_r1_prefill", "small", 6, 1, None, "prefill"),
        ("cfg0_r1", "cfg0", 0, 1, None, None),
        ("cfg0_r8", "cfg0", 7, 8, None, None),
        ("cfg1_r1", "cfg1", 0, 1, None, None),
        ("cfg1_r4", "cfg1", 8, 4, None, None),
    ]
    for name, shape_name, seed, rows, bk, variant in specs:
        shape = syn.SHAPES[shape_name]
        R = syn.make_router(shape, seed)
        x = syn.make_x(shape, seed, rows)
        basis_top_k = shape.rank if bk is None else bk
        routing = {
            "enc_w": torch.from_numpy(R["enc_w"]), "enc_b": torch.from_numpy(R["enc_b"]),
            "route_score_weight": torch.from_numpy(R["score_w"]),
            "route_score_bias": torch.from_numpy(R["score_b"]),
            "top_k": shape.top_k, "basis_top_k": basis_top_k, "num_blocks": shape.num_blocks,
        }
        extra = {}
        r = new_runtime(rt)
        if variant == "down_block_norm":
            dbn = np.random.default_rng(seed + 100).uniform(0.5, 1.5, shape.num_blocks).astype(np.float32)
            routing["down_block_norm"] = torch.from_numpy(dbn)
            extra["down_block_norm"] = dbn
        if variant == "legacy":
            dnt = np.abs(np.random.default_rng(seed + 200).standard_normal((shape.rank, shape.num_blocks))).astype(np.float32)
            routing.pop("route_score_weight")
            routing.pop("route_score_bias")
            routing["dec_norm_t"] = torch.from_numpy(dnt)
            extra["dec_norm_t"] = dnt
        prefill_k = None
        if variant == "prefill":
            r._traffic_current_phase = "prefill"
            r._sparse_mlp_prefill_mode = "sparse"
            prefill_k = shape.top_k // 2 + 1
            r._sparse_mlp_prefill_top_k = prefill_k
        r._sparse_routing = {0: routing}
        hidden = torch.from_numpy(x).view(rows, 1, shape.hidden)
        idx = r._route_sparse_mlp(hidden, 0).numpy().astype(np.int64)
        case = {"name": name, "shape": shape_name, "seed": seed, "rows": rows, "basis_top_k": basis_top_k,
                "variant": variant or "", "prefill_top_k": -1 if prefill_k is None else prefill_k,
                "input_sha": sha(R["enc_w"], R["score_w"], R["score_b"], x)}
        cases.append(case)
        out[f"router/{name}/idx"] = idx
        for k, v in extra.items():
            out[f"router/{name}/{k}"] = v
    out["router/cases.json"] = np.frombuffer(json.dumps(cases).encode(), dtype=np.uint8)


# --------------------------------------------------------------------------- layout
def gen_layout(rt, out: dict) -> None:
    import torch
    cases = []
    rng = np.random.default_rng(11)
    specs = [
        ("r1", 1, 6, 32, 4, None, False),
        ("r1_hot", 1, 6, 32, 4, [3, 9, 17], False),
        ("r3", 3, 5, 32, 8, None, False),
        ("r4_hot", 4, 6, 48, 2, [1, 2, 40], False),
        ("r2_invalid", 2, 4, 16, 4, None, True),
        ("r32_cfg4like", 32, 16, 128, 32, [0, 5, 64], False),
    ]
    for name, rows, k, maxb, bs, hot, invalid in specs:
        ab = np.stack([rng.choice(maxb, size=k, replace=False) for _ in range(rows)]).astype(np.int64)
        if invalid:
            ab[0, 1] = -1
            ab[1, 0] = maxb + 3
            ab[1, 2] = ab[0, 0]
        r = new_runtime(rt)
        if hot is not None:
            r._mlp_hot_blocks_by_layer = {0: torch.tensor(hot, dtype=torch.long)}
        ordered, active_local, flat_mask, neurons = r._build_sparse_active_layout(
            layer_idx=0, active_blocks=torch.from_numpy(ab), rows=rows, block_size=bs,
            max_valid_blocks=maxb, dtype=torch.float32)
        cases.append({"name": name, "rows": rows, "block_size": bs, "max_valid_blocks": maxb,
                      "hot": hot if hot is not None else []})
        out[f"layout/{name}/active_blocks"] = ab
        out[f"layout/{name}/ordered"] = ordered.numpy().astype(np.int64)
        out[f"layout/{name}/active_local"] = active_local.numpy().astype(np.int32)
        out[f"layout/{name}/flat_mask"] = flat_mask.numpy().astype(np.float32)
        out[f"layout/{name}/neurons"] = neurons.numpy().astype(np.int64)
    out["layout/cases.json"] = np.frombuffer(json.dumps(cases).encode(), dtype=np.uint8)


# --------------------------------------------------------------------------- cache policy
def gen_cache_policy(rt, out: dict) -> None:
    import torch
    R = rt.StreamingLlamaRuntime
    rng = np.random.default_rng(21)
    bank = []
    for t in range(24):
        cap = int(rng.integers(1, 12))
        active = int(rng.integers(0, cap + 1))
        ids = np.full(cap, -1, np.int64)
        ids[:active] = rng.choice(100, size=active, replace=False)
        scores = np.zeros(cap, np.float32)
        scores[:active] = rng.integers(0, 6, size=active).astype(np.float32)  # ties on purpose
        novel = rng.choice(np.arange(100, 200), size=int(rng.integers(0, 2 * cap + 2)), replace=False)
        slots, nids, nscores, nact = R._plan_fixed_capacity_bank_update(
            existing_block_ids_cpu=torch.from_numpy(ids), existing_scores_cpu=torch.from_numpy(scores),
            active_count=active, capacity=cap, novel_blocks_cpu=torch.from_numpy(novel))
        bank.append({"ids": ids.tolist(), "scores": scores.tolist(), "active": active, "capacity": cap,
                     "novel": novel.tolist(), "out_slots": slots.tolist(), "out_ids": nids.tolist(),
                     "out_scores": [float(v) for v in nscores.tolist()], "out_active": int(nact)})
    calib = []
    for t in range(6):
        nb = int(rng.integers(8, 40))
        rows = int(rng.integers(1, 6))
        k = int(rng.integers(1, 6))
        ab = rng.integers(-2, nb + 2, size=(rows, k))
        power = float(rng.choice([0.0, 1.0, 2.0, 0.5]))
        r = new_runtime(rt)
        r._hot_cache_calibration_active = True
        r._hot_cache_calibration_hits = {}
        r._hot_cache_calibration_recency_power = power
        r._sparse_num_blocks = nb
        r._sparse_routing = {0: {"num_blocks": nb}}
        r._record_hot_cache_calibration_blocks(0, torch.from_numpy(ab).long())
        r._record_hot_cache_calibration_blocks(0, torch.from_numpy(ab[::-1].copy()).long())
        calib.append({"num_blocks": nb, "active_blocks": ab.tolist(), "power": power,
                      "counts": [float(v) for v in r._hot_cache_calibration_hits[0].tolist()]})
    target = []
    for t in range(10):
        r = new_runtime(rt)
        limit = int(rng.integers(0, 8)) * (1024 ** 3)
        used = int(rng.integers(0, 2)) * (1024 ** 3) // 2
        layers = int(rng.choice([1, 32, 126]))
        r._vram_hot_cache_limit_bytes = limit
        r._vram_hot_cache_used_bytes = used
        r._sparse_routing = {i: {} for i in range(layers)}
        r.num_layers = layers
        bpb = int(rng.choice([256 * 1024, 917504, 229376]))
        r._estimate_mlp_hot_cache_bytes_per_block = (lambda v: (lambda layer_idx: v))(bpb)
        li = int(rng.integers(0, layers))
        rtk = int(rng.integers(1, 300))
        slots = int(rng.choice([256, 448, 1664]))
        prev = int(rng.integers(0, 3)) * 50
        os.environ.pop("STREAMING_HOT_CACHE_TARGET_BLOCKS", None)
        os.environ.pop("STREAMING_HOT_CACHE_MAX_BLOCKS", None)
        got = r._target_hot_blocks_for_layer(layer_idx=li, runtime_top_k=rtk, count_slots=slots,
                                             previous_hot_count=prev)
        target.append({"limit": limit, "used": used, "layers": layers, "bpb": bpb, "layer_idx": li,
                       "runtime_top_k": rtk, "count_slots": slots, "prev": prev, "target": int(got)})
    blob = {"bank": bank, "calibration": calib, "target": target}
    (HERE / "cache_policy.json").write_text(json.dumps(blob, indent=0))


# --------------------------------------------------------------------------- down column gather
def gen_down_cols(rt, out: dict) -> None:
    import torch
    shape = syn.SHAPES["tiny"]
    full = syn.make_layer_full(shape, 31)
    H, I = shape.hidden, shape.intermediate
    r = new_runtime(rt)
    r._down_proj_col_cache = {}
    r._down_proj_col_cache_max_blocks_per_layer = 64
    param = {"packed_weight": torch.from_numpy(full["down_packed"].copy()),
             "packed_blocks": torch.from_numpy(full["down_packed"].copy()).view(H, -1),
             "absmax_blocks": torch.from_numpy(full["down_absmax"].copy()).view(H, -1),
             "absmax": torch.from_numpy(full["down_absmax"].copy()), "full_name": "L0.down"}
    blocks = np.array([5, 0, 31, 6, 7], np.int64)
    packed, absmax = r._load_down_proj_cold_cols(
        param, torch.from_numpy(blocks), H_out=H, bytes_per_row=I // 2, bytes_per_cblk=16,
        absmax_per_row=I // 64, block_size=32, qbs=64, down_name="L0.down")
    out["down_cols/blocks"] = blocks
    out["down_cols/packed"] = packed.numpy()
    out["down_cols/absmax"] = absmax.numpy()
    out["down_cols/input_sha"] = np.frombuffer(sha(full["down_packed"], full["down_absmax"]).encode(), np.uint8)


# --------------------------------------------------------------------------- Triton kernels (interpreter)
def gen_single_kernel(tsm, out: dict) -> None:
    import torch
    specs = [("tiny", 41, 4, 64), ("small", 42, 16, 64), ("cfg0", 0, 56, 64)]
    cases = []
    for shape_name, seed, k, block_out in specs:
        shape = syn.SHAPES[shape_name]
        R = syn.make_router(shape, seed)
        x = syn.make_x(shape, seed, 1)
        from oracle.router import route_sparse_mlp
        blocks = route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], k, shape.rank)[0]
        G = syn.selected_blocks_gathered(shape, seed, 0, blocks)
        H = shape.hidden
        acc = torch.zeros(H, dtype=torch.float32)
        code = torch.from_numpy(G["code"])
        tsm._sparse_mlp_decode_4bit_single_kernel_sm75[(k,)](
            torch.from_numpy(x.reshape(-1).copy()),
            torch.from_numpy(G["gate_packed"].reshape(-1).copy()), torch.from_numpy(G["gate_absmax"].reshape(-1).copy()), code,
            torch.from_numpy(G["up_packed"].reshape(-1).copy()), torch.from_numpy(G["up_absmax"].reshape(-1).copy()), code,
            torch.from_numpy(G["down_cols"].reshape(-1).copy()), torch.from_numpy(G["down_absmax_cols"].reshape(-1).copy()), code,
            acc, H, 32, 64, k, H // 2, H // 64, 16, BLOCK_IN=64, BLOCK_OUT=block_out)
        name = f"{shape_name}_k{k}"
        cases.append({"name": name, "shape": shape_name, "seed": seed, "k": k,
                      "input_sha": sha(x, G["gate_packed"], G["gate_absmax"], G["up_packed"], G["up_absmax"],
                                       G["down_cols"], G["down_absmax_cols"])})
        out[f"single/{name}/blocks"] = blocks.astype(np.int64)
        out[f"single/{name}/y"] = acc.numpy().copy()
        print("single kernel", name, "done", flush=True)
    out["single/cases.json"] = np.frombuffer(json.dumps(cases).encode(), dtype=np.uint8)


def gen_linear4bit(tsm, out: dict) -> None:
    import torch
    rng = np.random.default_rng(51)
    code = nf4_code()
    cases = []
    # (name, rows, in_features, out_features, block_size, k, with_bias, x dtype)
    specs = [("in_a", 2, 64, 48, 8, 3, False), ("in_b", 3, 96, 40, 16, 4, True), ("in_c", 1, 128, 64, 32, 2, False)]
    for name, rows, fin, fout, bs, k, with_bias in specs:
        nb = fin // bs
        packed = rng.integers(0, 256, size=(fin * fout) // 2, dtype=np.uint8)
        absmax = rng.uniform(0.01, 0.1, size=(fin * fout) // 64).astype(np.float32)
        x = rng.standard_normal((rows, fin)).astype(np.float32)
        idx = np.stack([rng.choice(nb, size=k, replace=False) for _ in range(rows)]).astype(np.int32)
        idx[0, -1] = -1
        bias = rng.standard_normal(fout).astype(np.float32) if with_bias else None
        t_out = torch.zeros((rows, fout), dtype=torch.float32)
        tsm._sparse_input_linear_4bit_tiled_kernel.fn[(rows, (fout + 31) // 32)](
            torch.from_numpy(x), torch.from_numpy(idx), torch.from_numpy(packed), torch.from_numpy(absmax),
            torch.from_numpy(code), torch.from_numpy(bias) if bias is not None else t_out, t_out,
            rows, fout, fin, k, bs, 64, x.shape[1], idx.shape[1], 1, t_out.shape[1],
            TOPK_MAX=1 << (k - 1).bit_length(), BLOCK_IN=1 << (bs - 1).bit_length(), BLOCK_OUT=32,
            HAS_BIAS=bias is not None)
        a_out = torch.zeros((rows, fout), dtype=torch.float32)
        tsm._sparse_input_linear_4bit_atomic_kernel[(rows * k, (fout + 63) // 64)](
            torch.from_numpy(x), torch.from_numpy(idx), torch.from_numpy(packed), torch.from_numpy(absmax),
            torch.from_numpy(code), a_out, rows, fout, fin, k, bs, 64, x.shape[1], idx.shape[1], 1,
            a_out.shape[1], BLOCK_IN=1 << (bs - 1).bit_length(), BLOCK_OUT=64)
        if bias is not None:
            a_out += torch.from_numpy(bias)[None, :]
        cases.append({"name": name, "kind": "input", "rows": rows, "in_features": fin, "out_features": fout,
                      "block_size": bs, "k": k})
        for key, val in (("x", x), ("idx", idx), ("packed", packed), ("absmax", absmax), ("y_tiled", t_out.numpy()),
                         ("y_atomic", a_out.numpy())):
            out[f"lin4/{name}/{key}"] = val
        if bias is not None:
            out[f"lin4/{name}/bias"] = bias
    specs = [("out_a", 2, 64, 8, 3, 6, False), ("out_b", 1, 128, 16, 4, 5, True), ("out_c", 3, 64, 32, 2, 2, False)]
    for name, rows, din, bs, k, nslots, with_bias in specs:
        width = nslots * bs
        n_elem = din * bs + width  # covers e = k*bs + blk*bs + o for every blk < nslots
        n_elem = ((n_elem + 127) // 128) * 128
        packed = rng.integers(0, 256, size=n_elem // 2, dtype=np.uint8)
        absmax = rng.uniform(0.01, 0.1, size=n_elem // 64).astype(np.float32)
        x = rng.standard_normal((rows, din)).astype(np.float32)
        idx = np.stack([rng.choice(nslots, size=k, replace=False) for _ in range(rows)]).astype(np.int32)
        mask = np.zeros((rows, width), np.float32)
        for r_ in range(rows):
            for s in idx[r_]:
                mask[r_, s * bs:(s + 1) * bs] = 1.0
        if rows > 1:
            idx[1, 0] = -1
        bias = rng.standard_normal(width).astype(np.float32) if with_bias else None
        o = torch.zeros((rows, width), dtype=torch.float32)
        tsm._sparse_output_linear_4bit_kernel.fn[(rows * k, (bs + 31) // 32)](
            torch.from_numpy(x), torch.from_numpy(idx), torch.from_numpy(packed), torch.from_numpy(absmax),
            torch.from_numpy(code), torch.from_numpy(bias) if bias is not None else o, o,
            rows, din, k, bs, 64, x.shape[1], idx.shape[1], 1, o.shape[1],
            BLOCK_OUT=32, BLOCK_K=32, HAS_BIAS=bias is not None)
        y = (o * torch.from_numpy(mask)).numpy()
        cases.append({"name": name, "kind": "output", "rows": rows, "input_dim": din, "block_size": bs, "k": k,
                      "width": width})
        for key, val in (("x", x), ("idx", idx), ("packed", packed), ("absmax", absmax), ("mask", mask), ("y", y)):
            out[f"lin4/{name}/{key}"] = val
        if bias is not None:
            out[f"lin4/{name}/bias"] = bias
    out["lin4/code"] = code
    out["lin4/cases.json"] = np.frombuffer(json.dumps(cases).encode(), dtype=np.uint8)


# --------------------------------------------------------------------------- artifacts and checkpoints
CHECKPOINT_SHAPE = "tiny"
CHECKPOINT_SEED = 41


def write_checkpoint_snapshot(directory, index: bool) -> dict:
    """The seeded bitsandbytes-format snapshot the checkpoint fixtures use
    (layer 0 and 1 of the tiny shape, plus a dense bf16 norm weight)."""
    from oracle import bnb_checkpoint as bc
    shape = syn.SHAPES[CHECKPOINT_SHAPE]
    params = {}
    for layer in (0, 1):
        full = syn.make_layer_full(shape, CHECKPOINT_SEED, layer)
        params.update(bc.layer_params(full, shape.hidden, shape.intermediate, layer))
    extra = {"model.layers.0.post_attention_layernorm.weight":
             np.linspace(0.5, 1.5, shape.hidden, dtype=np.float32)}
    return bc.write_snapshot(directory, params, shards=2, index=index, extra=extra)


def gen_checkpoint(rt) -> None:
    import tempfile
    import types as _types

    import torch
    from llama3_neuroplastic.experiments.runtime import safetensor_loader as sl

    shape = syn.SHAPES[CHECKPOINT_SHAPE]
    H, NB = shape.hidden, shape.num_blocks
    loader_cases = []
    rng = np.random.default_rng(43)
    for index in (True, False):
        with tempfile.TemporaryDirectory() as tmp:
            write_checkpoint_snapshot(tmp, index)
            try:
                ld = sl.ShardedSafetensorLoader(Path(tmp), pin_ram_cache=False)
            except TypeError as e:
                # without an index the reference iterates a safe_open handle,
                # which safetensors 0.7 does not support
                loader_cases.append({"index": index, "error": f"TypeError: {e}"})
                continue
            case = {"index": index, "weight_map": dict(sorted(ld.weight_map.items())),
                    "aux": {k: sorted(v) for k, v in sorted(ld._quant_aux_by_base.items())}, "blocks": []}
            for name in sorted(ld._quant_aux_by_base):
                if name not in ld.weight_map:
                    continue
                is_down = "down_proj" in name
                bpb = (shape.intermediate // 2) * 32 if is_down else (H // 2) * 32
                nblk = (H if is_down else shape.intermediate) // 32
                idx = rng.choice(nblk, size=min(5, nblk), replace=False)
                got = ld.load_nf4_packed_blocks(name, torch.from_numpy(idx), bytes_per_block=bpb)
                w, aux = ld._load_raw_for_param(name, store_in_ram_cache=False)
                case["blocks"].append({"name": name, "bytes_per_block": bpb, "idx": idx.tolist(),
                                       "shape": list(got.shape), "sha": sha(got.numpy()),
                                       "raw_shape": list(w.shape), "aux_keys": sorted(aux)})
            loader_cases.append(case)

    R = rt.StreamingLlamaRuntime
    hot_cases = []
    g = np.random.default_rng(47)

    def runtime_for(limit, used, routing_layers, rtk):
        r = new_runtime(rt)
        r._hot_block_threshold = 0.8
        r._sparse_runtime_top_k = rtk
        r._sparse_top_k = max(1, rtk)
        r._vram_hot_cache_limit_bytes = limit
        r._vram_hot_cache_used_bytes = used
        r._sparse_routing = {i: {} for i in range(routing_layers)}
        r.num_layers = 126
        r._sparse_param_cache = {}
        r._sparse_block_size = 32
        r.config = _types.SimpleNamespace(hidden_size=H, intermediate_size=shape.intermediate)
        return r

    def vec(kind, n):
        if kind == "rand":
            return g.random(n).astype(np.float32)
        if kind == "peaky":   # a few blocks near the max, the rest well below the threshold
            v = (g.random(n) * 0.5).astype(np.float32)
            v[g.choice(n, size=4, replace=False)] = (0.85 + 0.15 * g.random(4)).astype(np.float32)
            return v
        return np.zeros(n, np.float32)

    specs = [
        ("state.block_importance", "rand", NB, None, 0.8),
        ("state.block_importance_probs", "rand", NB - 7, None, 0.8),
        ("state._block_importance_probs", "peaky", NB, None, 0.8),
        ("stats.scores", "rand", NB + 5, None, 0.8),
        ("stats.map", "rand", NB, None, 0.8),
        ("importance", "rand", NB, None, 0.8),
        ("state.block_importance", "zero", NB, None, 0.8),
        ("decoder_bias", "rand", NB, None, 0.8),
        ("none", "rand", NB, None, 0.8),
        ("state.block_importance", "peaky", NB, 150_000, 0.8),
        ("state.block_importance", "rand", NB, 260_000, 0.5),
        ("state.block_importance", "rand", NB, None, 0.0),
        ("state.block_importance", "rand", NB, None, 1.0),
        ("stats.map", "peaky", NB, 400_000, 0.9),
    ]
    for t, (where, kind, n, limit, thr) in enumerate(specs):
        v = vec(kind, n)
        state, stats, imp = {"layer_idx": int(t % 5)}, {"explained_variance_ratio": 0.9}, None
        if t % 3 == 0:
            state["top_k"] = int(3 + t)
        if where.startswith("state."):
            state[where.split(".", 1)[1]] = torch.from_numpy(v) if t % 2 == 0 else v.tolist()
        elif where == "stats.scores":
            stats = {"scores": torch.from_numpy(v)}
        elif where == "stats.map":
            nz = g.choice(n, size=n // 3, replace=False)
            stats = {str(int(i)): float(v[i]) for i in nz}
            stats["not_a_block"] = 3.0
            stats[str(n + 9)] = 99.0
        elif where == "importance":
            imp = torch.from_numpy(v)
        elif where == "decoder_bias":
            state["decoder_bias"] = torch.from_numpy(g.standard_normal((NB, 8)).astype(np.float32))
        rtk = int(g.integers(1, 12))
        routing_layers = int(g.integers(1, 4))
        r = runtime_for(limit, 0, routing_layers, rtk)
        r._hot_block_threshold = float(thr)
        got = R._derive_hot_blocks_for_layer(r, layer_state=state, layer_stats=stats,
                                             block_importance_by_layer=imp, layer_num_blocks=NB)
        def enc(x):
            if torch.is_tensor(x):
                return {"tensor": x.tolist()}
            if isinstance(x, dict):
                return {"dict": {k: enc(v) for k, v in x.items()}}
            return x
        hot_cases.append({"state": enc(state), "stats": enc(stats), "importance": enc(imp), "num_blocks": NB,
                          "hidden": H, "limit": limit, "routing_layers": routing_layers, "runtime_top_k": rtk,
                          "threshold": float(thr), "hot": None if got is None else got.tolist()})
    blob = {"shape": CHECKPOINT_SHAPE, "seed": CHECKPOINT_SEED, "loader": loader_cases, "hot_blocks": hot_cases}
    (HERE / "checkpoint.json").write_text(json.dumps(blob, indent=0))


ARTIFACT_SHAPE = "tiny"


def artifact_payload(case: int):
    """Seeded router artifacts in the fitting script's schema
    (``{config, layer_selection, layer_states, stats}``), one per case."""
    import torch
    shape = syn.SHAPES[ARTIFACT_SHAPE]
    NB, r = shape.num_blocks, shape.rank
    g = np.random.default_rng(900 + case)
    cfg = {"artifact_target": "intermediate_block_scores", "block_size": 32, "num_blocks": NB, "basis_rank": r}
    layers = [0, 1, 2, 5]
    if case == 1:
        cfg.update({"top_k_by_layer": {"1": 3, 2: 99}, "basis_top_k_by_layer": {"0": 2, 5: 40}, "basis_top_k": 6})
    if case == 2:
        cfg.pop("num_blocks")
        cfg["top_k_by_layer"] = {"0": 0}
    states, stats = {}, {}
    for li in layers:
        R = syn.make_router(shape, 31 + case, li)
        st = {"encoder_weight": torch.from_numpy(R["enc_w"]), "encoder_bias": torch.from_numpy(R["enc_b"]),
              "score_weight": torch.from_numpy(R["score_w"]), "scale": torch.tensor(1.0 + li)}
        if li != 1:
            st["score_bias"] = torch.from_numpy(R["score_b"])
        if li == 2:
            st["down_block_norm"] = torch.from_numpy(g.uniform(0.5, 1.5, NB).astype(np.float32))
        if li == 5:
            st["rank_effective"] = torch.tensor(float(r - 5))
            st["explained_variance_ratio"] = torch.tensor(0.2)
        imp = g.random(NB).astype(np.float32)
        if case == 1 and li == 0:
            st["block_importance"] = torch.from_numpy(imp)
        elif li == 1:
            stats[str(li)] = {"scores": torch.from_numpy(imp), "rank_effective": float(r - 2)}
        states[str(li)] = st
    if case == 2:
        states["9"] = states["0"]   # out of range for 8 layers: skipped
        states["3"] = {"artifact_target": "output_reconstruction", "block_domain": "output",
                       "decoder_blocks": torch.zeros(shape.hidden // 32, r, 32),
                       "encoder_weight": torch.zeros(r, shape.hidden), "encoder_bias": torch.zeros(r),
                       "scale": torch.tensor(1.0)}
    return {"config": cfg, "layer_selection": layers + [77], "layer_states": states, "stats": stats}


def gen_artifact(rt) -> None:
    """The reference constructor's artifact block (``StreamingLlamaRuntime.__init__``,
    from ``if sparse_basis_path ...`` up to its summary printout), taken from
    the reference source at generation time and run on a ``__new__``-built
    runtime for seeded artifacts; records what it loads."""
    import inspect
    import tempfile
    import textwrap
    import types as _types

    import torch
    shape = syn.SHAPES[ARTIFACT_SHAPE]
    lines = inspect.getsource(rt.StreamingLlamaRuntime.__init__).splitlines()
    a = next(i for i, ln in enumerate(lines) if ln.strip().startswith("if sparse_basis_path and str(sparse_basis_path)"))
    b = next(i for i, ln in enumerate(lines) if i > a and ln.strip().startswith("_pct = int(round(self._sparse_top_k"))
    code = compile(textwrap.dedent("\n".join(lines[a:b])), "<reference artifact block>", "exec")
    out = []
    for case, (top_k, basis_k, hot, limit) in enumerate([(None, None, False, None), (5, None, True, None),
                                                          (None, 3, True, 60_000)]):
        with tempfile.TemporaryDirectory() as tmp:
            path = Path(tmp) / "router.pt"
            torch.save(artifact_payload(case), path)
            r = new_runtime(rt)
            r.num_layers = 8
            r.config = _types.SimpleNamespace(hidden_size=shape.hidden, intermediate_size=shape.intermediate)
            r.dtype = torch.float32
            r._sparse_routing, r._sparse_top_k_by_layer, r._sparse_basis_top_k_by_layer = {}, {}, {}
            r._mlp_hot_blocks_by_layer = {}
            r._sparse_checkpoint_basis_rank = 64
            r._sparse_explicit_layer_selection = set()
            r._vram_hot_cache_enabled = hot
            r._sparse_mlp_prefill_mode = "dense"
            r._hot_block_threshold = 0.8
            r._vram_hot_cache_limit_bytes = limit
            r._vram_hot_cache_used_bytes = 0
            r._sparse_param_cache = {}
            env = dict(vars(rt))
            env.update(self=r, sparse_basis_path=str(path), sparse_top_k=top_k, sparse_basis_top_k=basis_k)
            exec(code, env)
            layers, output_layers = {}, []
            for li, d in sorted(r._sparse_routing.items()):
                if d.get("block_domain") != "intermediate":
                    output_layers.append(int(li))
                    continue
                layers[str(li)] = {"top_k": int(d["top_k"]), "basis_top_k": int(d["basis_top_k"]),
                                   "rank_effective": int(d["rank_effective"]), "scale": float(d["scale"]),
                                   "evr": float(d["explained_variance_ratio"]), "num_blocks": int(d["num_blocks"]),
                                   "has_score_bias": d["route_score_bias"] is not None,
                                   "has_down_block_norm": d["down_block_norm"] is not None,
                                   "enc_w_sha": sha(d["enc_w"].numpy()), "score_w_sha": sha(d["route_score_weight"].numpy())}
            out.append({"case": case, "sparse_top_k": top_k, "sparse_basis_top_k": basis_k, "hot": hot,
                        "limit": limit, "default_top_k": int(r._sparse_top_k),
                        "layer_selection": sorted(r._sparse_explicit_layer_selection), "layers": layers,
                        "output_domain_layers": output_layers,
                        "hot_blocks": {str(k): v.tolist() for k, v in sorted(r._mlp_hot_blocks_by_layer.items())}})
    blob = json.loads((HERE / "checkpoint.json").read_text())
    blob["artifact"] = {"shape": ARTIFACT_SHAPE, "cases": out}
    (HERE / "checkpoint.json").write_text(json.dumps(blob, indent=0))


def calibration_hits(case: int) -> dict:
    """Seeded per-layer hit counts (distinct floats: no ties for topk)."""
    g = np.random.default_rng(700 + case)
    nb = 48
    hits = {li: (g.permutation(nb).astype(np.float32) + g.random(nb).astype(np.float32) * 0.5)
            for li in (0, 2, 3, 6)}
    hits[3][:] = 0.0   # a layer without hits is skipped
    return hits


def gen_calibration(rt) -> None:
    """The rebuild loop of ``calibrate_vram_hot_cache`` (from ``updated_layers =
    0`` up to its summary printout), taken from the reference source when the
    fixture is made and run on seeded hit counts."""
    import inspect
    import textwrap
    import types as _types

    import torch
    lines = inspect.getsource(rt.StreamingLlamaRuntime.calibrate_vram_hot_cache).splitlines()
    a = next(i for i, ln in enumerate(lines) if ln.strip() == "updated_layers = 0")
    b = next(i for i, ln in enumerate(lines) if i > a and ln.strip().startswith("print("))
    code = compile(textwrap.dedent("\n".join(lines[a:b])), "<reference calibration rebuild>", "exec")
    out = []
    for case, (limit, prev, rtk) in enumerate([(None, {}, 0), (None, {2: 11}, 5), (900_000, {0: 3}, 0)]):
        r = new_runtime(rt)
        r.num_layers = 8
        r.config = _types.SimpleNamespace(hidden_size=1024, intermediate_size=48 * 32)
        r._sparse_routing = {li: ({"top_k": 4 + li} if li % 2 == 0 else {}) for li in range(8)}
        r._sparse_runtime_top_k, r._sparse_top_k = rtk, 6
        r._hot_cache_calibration_hits = {li: torch.from_numpy(v.copy()) for li, v in calibration_hits(case).items()}
        r._mlp_hot_blocks_by_layer = {li: torch.arange(n) for li, n in prev.items()}
        r._vram_hot_cache_limit_bytes = limit
        r._vram_hot_cache_used_bytes = 0
        r._sparse_param_cache = {}
        r._sparse_block_size = 32
        env = dict(vars(rt))
        env.update(self=r)
        exec(code, env)
        out.append({"case": case, "limit": limit, "prev": {str(k): v for k, v in prev.items()},
                    "sparse_runtime_top_k": rtk, "sparse_top_k": 6, "hidden": 1024,
                    "updated_layers": int(env["updated_layers"]), "total_hits": float(env["total_hits"]),
                    "hot": {str(k): v.tolist() for k, v in sorted(r._mlp_hot_blocks_by_layer.items())}})
    blob = json.loads((HERE / "checkpoint.json").read_text())
    blob["calibration"] = out
    (HERE / "checkpoint.json").write_text(json.dumps(blob, indent=0))


LM_HEAD_QBS_CASES = [(16384, None), (4096 + 128, None), (96, None), (100, None), (16384, "256"), (16384, "96"),
                     (16384, "x"), (8192, "128"), (64, "0")]


def gen_lm_head(rt) -> None:
    """``_resolve_lm_head_nf4_quant_block_size`` (a static method of the
    runtime's LM-head mixin) with and without its environment override."""
    R = rt.StreamingLlamaRuntime
    out = []
    for h, env in LM_HEAD_QBS_CASES:
        os.environ.pop("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", None)
        if env is not None:
            os.environ["STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE"] = env
        try:
            out.append({"in_features": h, "env": env, "qbs": int(R._resolve_lm_head_nf4_quant_block_size(h))})
        except RuntimeError as e:
            out.append({"in_features": h, "env": env, "error": str(e)})
    os.environ.pop("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", None)
    blob = json.loads((HERE / "checkpoint.json").read_text())
    blob["lm_head_qbs"] = out
    (HERE / "checkpoint.json").write_text(json.dumps(blob, indent=0))


def main() -> None:
    rt, tsm = load_reference()
    if sys.argv[1:] == ["checkpoint"]:
        gen_checkpoint(rt)
        gen_artifact(rt)
        gen_calibration(rt)
        gen_lm_head(rt)
        print("wrote", HERE / "checkpoint.json")
        return
    out: dict = {}
    gen_router(rt, out)
    print("router done", flush=True)
    gen_layout(rt, out)
    gen_cache_policy(rt, out)
    gen_down_cols(rt, out)
    print("host policy done", flush=True)
    gen_linear4bit(tsm, out)
    print("linear4bit done", flush=True)
    gen_single_kernel(tsm, out)
    out["nf4_code"] = nf4_code()
    np.savez_compressed(HERE / "golden.npz", **out)
    print("wrote", HERE / "golden.npz", (HERE / "golden.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
