"""Sparse NF4 MLP oracle (numpy, fp32).  TEST INFRASTRUCTURE ONLY.

Restates the reference's exact blockwise-sparse MLP math on gathered NF4
blocks, i.e. the dequant fallback of ``StreamingLlamaRuntime._sparse_mlp_forward_fast``
(``llama3_neuroplastic/experiments/streaming_llama_runtime.py:5433-5492``), the
gathers that feed it (``:4004-4207`` gate/up, ``:4455-4528`` down columns) and
the NF4 parameter metadata (``:4627-4654``).  The reference's single-kernel
decode (``llama3_neuroplastic/triton_sparse_mlp.py:807-914``) computes the same
math and pins this restatement through the golden fixtures.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .nf4 import dequantize_nf4, unpack_nibbles


@dataclass(frozen=True)
class Nf4ParamMeta:
    """NF4 metadata of one projection (``streaming_llama_runtime.py:4627-4654``)."""

    out_features: int
    in_features: int
    block_size: int = 32
    quant_block_size: int = 64

    @property
    def bytes_per_row(self) -> int:
        return self.in_features // 2

    @property
    def bytes_per_block(self) -> int:
        return self.bytes_per_row * self.block_size

    @property
    def blocks_per_col(self) -> int:
        return self.out_features // max(self.block_size, 1)

    @property
    def absmax_per_row(self) -> int:
        return self.in_features // self.quant_block_size

    @property
    def absmax_per_block(self) -> int:
        return self.absmax_per_row * self.block_size


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gather_row_blocks(packed: np.ndarray, absmax: np.ndarray, meta: Nf4ParamMeta, blocks: np.ndarray):
    """gate/up gather: ``packed_blocks[blocks]``, ``absmax_blocks[blocks]``
    (``streaming_llama_runtime.py:4447-4452``, ``:4535-4540``)."""
    pb = np.asarray(packed, dtype=np.uint8).reshape(meta.blocks_per_col, meta.bytes_per_block)
    ab = np.asarray(absmax, dtype=np.float32).reshape(meta.blocks_per_col, meta.absmax_per_block)
    b = np.asarray(blocks, dtype=np.int64).reshape(-1)
    return pb[b].copy(), ab[b].copy()


def gather_down_cols(packed: np.ndarray, absmax: np.ndarray, meta: Nf4ParamMeta, blocks: np.ndarray):
    """down column gather: ``raw[H, I/2][:, b*bs/2 : +bs/2]`` stacked to
    ``[H, n, bs/2]`` and ``absmax[H, I/qbs][:, (b*bs)//qbs]`` to ``[H, n]``
    (``streaming_llama_runtime.py:4497-4527``)."""
    H = meta.out_features
    raw = np.asarray(packed, dtype=np.uint8).reshape(H, meta.bytes_per_row)
    am = np.asarray(absmax, dtype=np.float32).reshape(H, meta.absmax_per_row)
    cb = meta.block_size // 2
    b = np.asarray(blocks, dtype=np.int64).reshape(-1)
    cols = np.stack([raw[:, int(x) * cb:(int(x) + 1) * cb] for x in b], axis=1) if b.size else np.zeros((H, 0, cb), np.uint8)
    absc = np.stack([am[:, (int(x) * meta.block_size) // meta.quant_block_size] for x in b], axis=1) \
        if b.size else np.zeros((H, 0), np.float32)
    return np.ascontiguousarray(cols), np.ascontiguousarray(absc.astype(np.float32))


def down_block_major(packed: np.ndarray, absmax: np.ndarray, meta: Nf4ParamMeta):
    """Every down column block, block-major: ``[NB, H, bs/2]`` and ``[NB, H]``.

    This is the layout of the reference's down-proj column cache entries
    (one ``[H, bs/2]`` slice + one ``[H]`` absmax column per block,
    ``streaming_llama_runtime.py:4506-4513``) laid out for all blocks.
    """
    nb = meta.in_features // meta.block_size
    cols, absc = gather_down_cols(packed, absmax, meta, np.arange(nb))
    return np.ascontiguousarray(cols.transpose(1, 0, 2)), np.ascontiguousarray(absc.T)


def dequant_down_cols(cols: np.ndarray, absc: np.ndarray, code: np.ndarray) -> np.ndarray:
    """``[H, U, bs/2]`` bytes + ``[H, U]`` absmax -> ``[H, U*bs]`` fp32
    (``streaming_llama_runtime.py:5465-5483``: pair 0 = high nibble)."""
    H, U, cb = cols.shape
    nib = unpack_nibbles(cols.reshape(-1)).reshape(H, U, cb * 2)
    w = np.asarray(code, dtype=np.float32)[nib] * np.asarray(absc, dtype=np.float32)[:, :, None]
    return w.reshape(H, U * cb * 2).astype(np.float32)


def sparse_mlp_gathered(x: np.ndarray, gate_packed: np.ndarray, gate_absmax: np.ndarray, gate_code: np.ndarray,
                        up_packed: np.ndarray, up_absmax: np.ndarray, up_code: np.ndarray,
                        down_cols: np.ndarray, down_absmax_cols: np.ndarray, down_code: np.ndarray,
                        *, quant_block_size: int = 64, flat_mask: np.ndarray | None = None,
                        gate_bias: np.ndarray | None = None, up_bias: np.ndarray | None = None,
                        down_bias: np.ndarray | None = None, return_act: bool = False):
    """The fallback MLP on gathered blocks (``streaming_llama_runtime.py:5433-5492``).

    x: ``[N, H]``; gate/up: ``[U, bs*H/2]`` bytes and ``[U, bs*H/qbs]`` absmax;
    down: ``[H, U, bs/2]`` bytes and ``[H, U]`` absmax.  Returns ``y [N, H]``
    fp32 (and the ``[N, U*bs]`` activations if ``return_act``).
    """
    xf = np.asarray(x, dtype=np.float32)
    xf = xf.reshape(-1, xf.shape[-1])
    H = xf.shape[1]
    U = gate_packed.shape[0]
    wg = dequantize_nf4(gate_packed, gate_absmax, gate_code, quant_block_size).reshape(-1, H)
    wu = dequantize_nf4(up_packed, up_absmax, up_code, quant_block_size).reshape(-1, H)
    g = xf @ wg.T
    u = xf @ wu.T
    if gate_bias is not None:
        g = g + np.asarray(gate_bias, np.float32)[None, :]
    if up_bias is not None:
        u = u + np.asarray(up_bias, np.float32)[None, :]
    if flat_mask is not None:
        g = g * flat_mask
        u = u * flat_mask
    act = (silu(g) * u).astype(np.float32)
    wd = dequant_down_cols(down_cols, down_absmax_cols, down_code)
    assert wd.shape == (H, U * (down_cols.shape[2] * 2)), (wd.shape, H, U)
    y = act @ wd.T
    if down_bias is not None:
        y = y + np.asarray(down_bias, np.float32)[None, :]
    y = y.astype(np.float32)
    return (y, act) if return_act else y


def sparse_mlp_full(x: np.ndarray, blocks: np.ndarray, gate_packed: np.ndarray, gate_absmax: np.ndarray,
                    up_packed: np.ndarray, up_absmax: np.ndarray, down_packed: np.ndarray, down_absmax: np.ndarray,
                    code: np.ndarray, *, hidden: int, intermediate: int, block_size: int = 32,
                    quant_block_size: int = 64, return_act: bool = False):
    """Single-row decode MLP from full (resident) NF4 weights and a block set."""
    gm = Nf4ParamMeta(intermediate, hidden, block_size, quant_block_size)
    dm = Nf4ParamMeta(hidden, intermediate, block_size, quant_block_size)
    gp, ga = gather_row_blocks(gate_packed, gate_absmax, gm, blocks)
    upk, ua = gather_row_blocks(up_packed, up_absmax, gm, blocks)
    dc, da = gather_down_cols(down_packed, down_absmax, dm, blocks)
    return sparse_mlp_gathered(x, gp, ga, code, upk, ua, code, dc, da, code,
                               quant_block_size=quant_block_size, return_act=return_act)


def rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: float) -> np.ndarray:
    """Llama RMSNorm in fp32: ``x * rsqrt(mean(x^2) + eps) * weight``."""
    xf = np.asarray(x, dtype=np.float32)
    var = np.mean(xf.astype(np.float64) ** 2, axis=-1, keepdims=True)
    out = xf * (1.0 / np.sqrt(var + eps)).astype(np.float32)
    if weight is not None:
        out = out * np.asarray(weight, np.float32)
    return out.astype(np.float32)
