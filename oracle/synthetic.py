"""Seeded synthetic inputs for the oracle side (numpy).  TEST INFRASTRUCTURE ONLY.

The reference's benchmark needs a real 405B checkpoint and fitted router
artifacts, neither of which exists here.  These generators produce seeded
synthetic data with the shapes and value distributions of the build's
configurations: NF4 weights quantized from N(0, 0.02) (blocksize 64, fp32
absmax), bf16 RMS-normalized N(0,1) inputs, router weights N(0, 1/sqrt(H)) /
N(0, 1/8) / N(0, 0.1) rounded to bf16-representable values.

Every NF4 block is generated from its own seed, so any block of any layer can
be produced without materializing the whole layer: gate/up block ``b`` (32
rows x H) from ``(seed, layer, proj, b)``; the down projection in 64-column
groups (blocks ``2j`` and ``2j+1`` share one absmax group per row) from
``(seed, layer, 2, j)``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .nf4 import bf16_round, nf4_code, quantize_nf4

PROJ_GATE, PROJ_UP, PROJ_DOWN, PROJ_ROUTER, PROJ_X = 0, 1, 2, 3, 4
WEIGHT_STD = 0.02


@dataclass(frozen=True)
class Shape:
    hidden: int
    intermediate: int
    top_k: int
    rank: int = 64
    block_size: int = 32
    quant_block_size: int = 64

    @property
    def num_blocks(self) -> int:
        return self.intermediate // self.block_size


SHAPES = {
    "tiny": Shape(256, 1024, 4, 16),
    "small": Shape(1024, 4096, 16, 64),
    "cfg0": Shape(4096, 14336, 56, 64),
    "cfg1": Shape(16384, 53248, 208, 64),
}


def _rng(*key: int) -> np.random.Generator:
    return np.random.default_rng([int(k) & 0xFFFFFFFF for k in key])


def make_x(shape: Shape, seed: int, rows: int = 1, shared: float = 0.0) -> np.ndarray:
    """bf16-representable fp32 ``[rows, H]``: ``rms(a*z + sqrt(1-a^2)*e_t)``."""
    g = _rng(seed, PROJ_X, rows)
    z = g.standard_normal(shape.hidden)
    e = g.standard_normal((rows, shape.hidden))
    v = shared * z[None, :] + np.sqrt(max(0.0, 1.0 - shared * shared)) * e
    v = v / np.sqrt(np.mean(v * v, axis=1, keepdims=True))
    return bf16_round(v.astype(np.float32))


def make_router(shape: Shape, seed: int, layer: int = 0) -> dict:
    g = _rng(seed, layer, PROJ_ROUTER)
    H, r, NB = shape.hidden, shape.rank, shape.num_blocks
    enc_w = bf16_round((g.standard_normal((r, H)) / np.sqrt(H)).astype(np.float32))
    enc_b = np.zeros(r, np.float32)
    score_w = bf16_round((g.standard_normal((NB, r)) / 8.0).astype(np.float32))
    score_b = bf16_round((g.standard_normal(NB) * 0.1).astype(np.float32))
    return {"enc_w": enc_w, "enc_b": enc_b, "score_w": score_w, "score_b": score_b,
            "top_k": shape.top_k, "basis_top_k": r}


def gate_up_block(shape: Shape, seed: int, layer: int, proj: int, block: int, code=None):
    """Bytes ``[32*H/2]`` and absmax ``[32*H/64]`` of one gate/up block."""
    code = nf4_code() if code is None else code
    w = (_rng(seed, layer, proj, block).standard_normal((shape.block_size, shape.hidden)) * WEIGHT_STD)
    return quantize_nf4(w.astype(np.float32), code, shape.quant_block_size)


def down_pair_group(shape: Shape, seed: int, layer: int, group: int, code=None):
    """Down columns ``[64*group, 64*group+64)``: bytes ``[H, 32]`` and absmax ``[H]``."""
    code = nf4_code() if code is None else code
    qbs = shape.quant_block_size
    w = (_rng(seed, layer, PROJ_DOWN, group).standard_normal((shape.hidden, qbs)) * WEIGHT_STD)
    packed, absmax = quantize_nf4(w.astype(np.float32), code, qbs)
    return packed.reshape(shape.hidden, qbs // 2), absmax.reshape(shape.hidden)


def down_block_cols(shape: Shape, seed: int, layer: int, block: int, code=None):
    """Column slice of one down block: bytes ``[H, 16]`` and absmax ``[H]``."""
    per_group = shape.quant_block_size // shape.block_size
    grp, sub = divmod(int(block), per_group)
    packed, absmax = down_pair_group(shape, seed, layer, grp, code)
    cb = shape.block_size // 2
    return np.ascontiguousarray(packed[:, sub * cb:(sub + 1) * cb]), absmax


def make_layer_full(shape: Shape, seed: int, layer: int = 0, code=None) -> dict:
    """Whole-layer NF4 weights in bitsandbytes row-major layout (small shapes only)."""
    code = nf4_code() if code is None else code
    H, NB = shape.hidden, shape.num_blocks
    gp, ga, upk, ua = [], [], [], []
    for b in range(NB):
        p, a = gate_up_block(shape, seed, layer, PROJ_GATE, b, code)
        gp.append(p); ga.append(a)
        p, a = gate_up_block(shape, seed, layer, PROJ_UP, b, code)
        upk.append(p); ua.append(a)
    n_groups = shape.intermediate // shape.quant_block_size
    dp = np.zeros((H, shape.intermediate // 2), np.uint8)
    da = np.zeros((H, n_groups), np.float32)
    gb = shape.quant_block_size // 2
    for j in range(n_groups):
        p, a = down_pair_group(shape, seed, layer, j, code)
        dp[:, j * gb:(j + 1) * gb] = p
        da[:, j] = a
    return {
        "gate_packed": np.concatenate(gp), "gate_absmax": np.concatenate(ga),
        "up_packed": np.concatenate(upk), "up_absmax": np.concatenate(ua),
        "down_packed": dp.reshape(-1), "down_absmax": da.reshape(-1), "code": code,
    }


def selected_blocks_gathered(shape: Shape, seed: int, layer: int, blocks, code=None) -> dict:
    """Gathered gate/up ``[U, ...]`` and down ``[H, U, 16]`` for a block list,
    generated block by block (any shape, including cfg1)."""
    code = nf4_code() if code is None else code
    gp, ga, upk, ua, dc, da = [], [], [], [], [], []
    for b in np.asarray(blocks, np.int64).reshape(-1):
        p, a = gate_up_block(shape, seed, layer, PROJ_GATE, int(b), code)
        gp.append(p); ga.append(a)
        p, a = gate_up_block(shape, seed, layer, PROJ_UP, int(b), code)
        upk.append(p); ua.append(a)
        p, a = down_block_cols(shape, seed, layer, int(b), code)
        dc.append(p); da.append(a)
    return {
        "gate_packed": np.stack(gp), "gate_absmax": np.stack(ga),
        "up_packed": np.stack(upk), "up_absmax": np.stack(ua),
        "down_cols": np.ascontiguousarray(np.stack(dc, axis=1)),
        "down_absmax_cols": np.ascontiguousarray(np.stack(da, axis=1)), "code": code,
    }
