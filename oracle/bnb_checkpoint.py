"""bitsandbytes-4bit checkpoints on disk (numpy + safetensors).  TEST INFRASTRUCTURE ONLY.

No real checkpoint exists here, so the loader tests write their own: a
snapshot directory with sharded ``*.safetensors`` files (and optionally
``model.safetensors.index.json``) holding NF4 weights from ``oracle.synthetic``
in the serialised form bitsandbytes 0.49.1 gives a ``Params4bit`` weight
(third party, not vendored, not installed here):

* ``P.weight``: uint8 ``[out*in/2, 1]``, row-major, high nibble = even element;
* ``P.weight.absmax``: fp32 per 64 values, or with nested statistics uint8
  codes plus ``P.weight.nested_absmax`` (fp32, one per 256 codes) and
  ``P.weight.nested_quant_map`` (256 fp32 values);
* ``P.weight.quant_map``: the 16 code values;
* ``P.weight.quant_state.bitsandbytes__nf4``: UTF-8 JSON (``quant_type``,
  ``blocksize``, ``dtype``, ``shape``, ``nested_blocksize``, ``nested_dtype``,
  ``nested_offset``) as a uint8 tensor.

The nested statistics follow bitsandbytes' double quantisation: subtract the
mean absmax (``nested_offset``), quantise the centred values blockwise (256 per
block, scaled by the block's max magnitude) to the nearest entry of a signed
256-entry table.  The table written here is this file's own monotone table, not
bitsandbytes' dynamic map: the reader takes the table from the file, so any
table exercises it.

``nested_absmax_decode`` is the checker's restatement of the decode the
reference applies (bitsandbytes blockwise dequantisation plus the offset,
``llama3_neuroplastic/experiments/streaming_llama_runtime.py:4621-4625`` and
``runtime/safetensor_loader.py:400-403``).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from .nf4 import nf4_code

NESTED_BLOCKSIZE = 256


def nested_table() -> np.ndarray:
    """A signed, ascending 256-entry table in [-1, 1] with an exact zero."""
    pos = np.geomspace(1e-3, 1.0, 128, dtype=np.float64)
    neg = -np.geomspace(1.0, 1e-3, 127, dtype=np.float64)
    return np.concatenate([neg, [0.0], pos]).astype(np.float32)


def nested_absmax_encode(absmax: np.ndarray, table: np.ndarray, blocksize: int = NESTED_BLOCKSIZE):
    """(uint8 codes, fp32 per-block scales, fp32 offset) of an fp32 absmax vector."""
    a = np.asarray(absmax, np.float32).reshape(-1)
    offset = np.float32(a.mean(dtype=np.float64))
    c = (a - offset).astype(np.float32)
    nblk = (c.size + blocksize - 1) // blocksize
    pad = np.zeros(nblk * blocksize, np.float32)
    pad[:c.size] = c
    scale = np.abs(pad.reshape(nblk, blocksize)).max(axis=1).astype(np.float32)
    scale[scale == 0] = 1.0
    v = (pad.reshape(nblk, blocksize) / scale[:, None]).reshape(-1)[:c.size]
    hi = np.clip(np.searchsorted(table, v), 1, table.size - 1)
    lo = hi - 1
    q = np.where(np.abs(table[hi] - v) < np.abs(v - table[lo]), hi, lo).astype(np.uint8)
    return q, scale, offset


def nested_absmax_decode(q: np.ndarray, scale: np.ndarray, table: np.ndarray, offset: float,
                         blocksize: int = NESTED_BLOCKSIZE) -> np.ndarray:
    """``table[q] * scale[i // blocksize]`` then ``+ offset``, each step in fp32."""
    q = np.asarray(q, np.int64).reshape(-1)
    prod = (table[q] * scale[np.arange(q.size) // blocksize]).astype(np.float32)
    return (prod + np.float32(offset)).astype(np.float32)


def quant_state_blob(fields: dict) -> np.ndarray:
    return np.frombuffer(json.dumps(fields).encode("utf-8"), dtype=np.uint8).copy()


def param_tensors(name: str, packed: np.ndarray, absmax: np.ndarray, shape, *, code=None, nested: bool = True,
                  dtype: str = "bfloat16", blocksize: int = 64) -> tuple[dict, np.ndarray]:
    """The safetensors entries of one 4-bit weight, and the fp32 absmax a
    reader must recover from them."""
    code = nf4_code() if code is None else np.asarray(code, np.float32)
    packed = np.ascontiguousarray(packed, np.uint8).reshape(-1, 1)
    fields = {"quant_type": "nf4", "blocksize": int(blocksize), "dtype": dtype, "shape": [int(s) for s in shape]}
    out = {name: packed, f"{name}.quant_map": code.astype(np.float32)}
    if nested:
        table = nested_table()
        q, scale, offset = nested_absmax_encode(absmax, table)
        fields.update({"nested_blocksize": NESTED_BLOCKSIZE, "nested_dtype": "float32",
                       "nested_offset": float(offset)})
        out[f"{name}.absmax"] = q
        out[f"{name}.nested_absmax"] = scale
        out[f"{name}.nested_quant_map"] = table
        expect = nested_absmax_decode(q, scale, table, float(offset))
    else:
        out[f"{name}.absmax"] = np.asarray(absmax, np.float32).reshape(-1)
        expect = out[f"{name}.absmax"]
    out[f"{name}.quant_state.bitsandbytes__nf4"] = quant_state_blob(fields)
    return out, expect


def write_snapshot(directory, params: dict[str, dict], *, shards: int = 2, index: bool = True,
                   nested: bool = True, extra: dict[str, np.ndarray] | None = None) -> dict[str, np.ndarray]:
    """Write ``params`` (name -> {packed, absmax, shape[, code]}) as a sharded
    snapshot; parameters go to shards round robin with their quant state.
    Returns name -> the fp32 absmax a reader must recover."""
    from safetensors.numpy import save_file
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    files = [f"model-{i + 1:05d}-of-{shards:05d}.safetensors" for i in range(shards)]
    per_shard: list[dict] = [{} for _ in range(shards)]
    expect = {}
    for i, (name, p) in enumerate(params.items()):
        ts, exp = param_tensors(name, p["packed"], p["absmax"], p["shape"], code=p.get("code"), nested=nested)
        per_shard[i % shards].update(ts)
        expect[name] = exp
    for j, (name, arr) in enumerate((extra or {}).items()):
        per_shard[j % shards][name] = np.ascontiguousarray(arr)
    weight_map = {}
    for f, tensors in zip(files, per_shard):
        save_file(tensors, str(d / f), metadata={"format": "pt"})
        weight_map.update({n: f for n in tensors})
    if index:
        total = sum(int(a.nbytes) for t in per_shard for a in t.values())
        (d / "model.safetensors.index.json").write_text(
            json.dumps({"metadata": {"total_size": total}, "weight_map": weight_map}, indent=1))
    return expect


def layer_params(full: dict, hidden: int, intermediate: int, layer: int) -> dict[str, dict]:
    """``oracle.synthetic.make_layer_full`` output as the three MLP weights of
    ``model.layers.{layer}.mlp``."""
    p = f"model.layers.{int(layer)}.mlp."
    H, I = int(hidden), int(intermediate)
    return {
        f"{p}gate_proj.weight": {"packed": full["gate_packed"], "absmax": full["gate_absmax"], "shape": (I, H)},
        f"{p}up_proj.weight": {"packed": full["up_packed"], "absmax": full["up_absmax"], "shape": (I, H)},
        f"{p}down_proj.weight": {"packed": full["down_packed"], "absmax": full["down_absmax"], "shape": (H, I)},
    }
