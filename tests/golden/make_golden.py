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
  interpreter (``TRITON_INTERPRET=1``).

Inputs come from ``oracle.synthetic`` (seeded).  Small inputs are stored in the
fixtures; large ones are stored as seeds plus a SHA-256 of the regenerated
bytes, so the tests can rebuild them and prove they are the same bytes.

Usage: ``NSM_REFERENCE_ROOT=/path/to/next_step_ai python tests/golden/make_golden.py``
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


def main() -> None:
    rt, tsm = load_reference()
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
