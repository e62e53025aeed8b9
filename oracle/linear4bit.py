"""Oracle for the reference's ``triton_sparse_mlp`` 4-bit API semantics (numpy).

TEST INFRASTRUCTURE ONLY.  These restate the index arithmetic of the
reference's generic Triton kernels, which the drop-in functions of the same
names must reproduce:

* ``triton_sparse_input_linear_4bit`` -> ``_sparse_input_linear_4bit_tiled_kernel`` /
  ``_sparse_input_linear_4bit_atomic_kernel``
  (``llama3_neuroplastic/triton_sparse_mlp.py:437-575``, wrapper ``:1101-1215``):
  ``out[r, n] = bias[n] + sum_{slot, blk=idx[r,slot] >= 0} sum_{i<bs}
  W(e=(blk*bs+i)*out_features + n) * x[r, blk*bs+i]``.
* ``triton_sparse_output_linear_4bit`` -> ``_sparse_output_linear_4bit_kernel``
  (``:578-651``, wrapper ``:1218-1300``):
  ``out[r, blk*bs+o] = bias[blk*bs+o] + sum_k W(e=k*bs + blk*bs + o) * x[r, k]``,
  then ``out * flat_mask``.
* ``triton_fused_sparse_mlp_decode_4bit`` (``:1519-1585``): output, output,
  ``silu(gate)*up``, input (call order pinned by the reference's
  ``tests/test_throughput_contract.py:364-407``).

``W(e) = code[nibble(e)] * absmax[e // quant_block_size]`` with the high nibble
holding the even element.  Accumulation is fp32; the oracle returns fp32
(the reference rounds the result to the activation dtype).
"""
from __future__ import annotations

import numpy as np


def _w(elem: np.ndarray, packed: np.ndarray, absmax: np.ndarray, code: np.ndarray, qbs: int) -> np.ndarray:
    byte = packed[elem >> 1]
    nib = np.where((elem & 1) == 0, byte >> 4, byte & 0x0F).astype(np.int64)
    return code[nib].astype(np.float32) * absmax[elem // qbs].astype(np.float32)


def sparse_input_linear_4bit(x, active_idx, packed, absmax, code, out_features, in_features, quant_block_size,
                             bias, block_size):
    x = np.asarray(x, np.float32).reshape(-1, int(in_features))
    idx = np.asarray(active_idx, np.int64).reshape(x.shape[0], -1)
    packed = np.asarray(packed, np.uint8).reshape(-1)
    absmax = np.asarray(absmax, np.float32).reshape(-1)
    code = np.asarray(code, np.float32)
    rows = x.shape[0]
    out = np.zeros((rows, int(out_features)), np.float64)
    if bias is not None:
        out += np.asarray(bias, np.float32)[None, :]
    n = np.arange(int(out_features), dtype=np.int64)
    bs = int(block_size)
    for r in range(rows):
        for blk in idx[r]:
            if blk < 0:
                continue
            for i in range(bs):
                col = int(blk) * bs + i
                e = col * int(out_features) + n
                out[r] += _w(e, packed, absmax, code, int(quant_block_size)).astype(np.float64) * float(x[r, col])
    return out.astype(np.float32)


def sparse_output_linear_4bit(x, active_idx, flat_mask, packed, absmax, code, input_dim, quant_block_size, bias,
                              block_size):
    x = np.asarray(x, np.float32).reshape(-1, int(input_dim))
    rows = x.shape[0]
    fm = np.asarray(flat_mask, np.float32).reshape(rows, -1)
    idx = np.asarray(active_idx, np.int64).reshape(rows, -1)
    packed = np.asarray(packed, np.uint8).reshape(-1)
    absmax = np.asarray(absmax, np.float32).reshape(-1)
    code = np.asarray(code, np.float32)
    bs = int(block_size)
    out = np.zeros(fm.shape, np.float64)
    k = np.arange(int(input_dim), dtype=np.int64)
    for r in range(rows):
        for blk in idx[r]:
            if blk < 0:
                continue
            for o in range(bs):
                col = int(blk) * bs + o
                e = k * bs + col
                acc = float(np.dot(_w(e, packed, absmax, code, int(quant_block_size)).astype(np.float64),
                                   x[r].astype(np.float64)))
                if bias is not None:
                    acc += float(np.asarray(bias, np.float32)[col])
                out[r, col] = acc
    return (out * fm).astype(np.float32)


def fused_sparse_mlp_decode_4bit(x, active_idx, flat_mask, *, gate, up, down, block_size):
    """``gate``/``up``: dicts with packed, absmax, code, input_dim, quant_block_size, bias;
    ``down``: packed, absmax, code, out_features, in_features, quant_block_size, bias."""
    g = sparse_output_linear_4bit(x, active_idx, flat_mask, gate["packed"], gate["absmax"], gate["code"],
                                  gate["input_dim"], gate["quant_block_size"], gate.get("bias"), block_size)
    u = sparse_output_linear_4bit(x, active_idx, flat_mask, up["packed"], up["absmax"], up["code"],
                                  up["input_dim"], up["quant_block_size"], up.get("bias"), block_size)
    act = (g / (1.0 + np.exp(-g))) * u
    return sparse_input_linear_4bit(act, active_idx, down["packed"], down["absmax"], down["code"],
                                    down["out_features"], down["in_features"], down["quant_block_size"],
                                    down.get("bias"), block_size)
