"""Seeded synthetic layers for benchmarks and GPU tests (generated on device).

There is no 405B checkpoint or fitted router artifact on the benchmark
machines, so layers are synthesized with the shapes and value distributions
of the benchmark configurations: gate/up/down weights N(0, 0.02) quantized to
NF4 (blocksize 64, fp32 absmax); router encoder N(0, 1/sqrt(H)), score head
N(0, 1/8), score bias N(0, 0.1), all rounded to bf16; inputs N(0,1)
RMS-normalised and rounded to bf16.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .nf4 import nf4_code, quantize_nf4
from .weights import RouterWeights, SparseMlpWeights

WEIGHT_STD = 0.02


@dataclass(frozen=True)
class LayerShape:
    hidden: int
    intermediate: int
    top_k: int
    rank: int = 64

    @property
    def num_blocks(self) -> int:
        return self.intermediate // 32


SHAPES = {
    "tiny": LayerShape(256, 1024, 4, 16),
    "small": LayerShape(1024, 4096, 16, 64),
    "cfg0": LayerShape(4096, 14336, 56, 64),   # Llama-3.1-8B MLP, k=56/448
    "cfg1": LayerShape(16384, 53248, 208, 64),  # Llama-3.1-405B MLP, k=208/1664
}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def _key(*parts: int) -> int:
    h = 1469598103934665603
    for p in parts:
        h = ((h ^ (int(p) & 0xFFFFFFFF)) * 1099511628211) & 0x7FFFFFFFFFFFFFFF
    return h


def make_x(shape: LayerShape, seed: int, rows: int = 1, device="cuda", shared: float = 0.0) -> torch.Tensor:
    """``rms(a*z + sqrt(1-a^2)*e_t)`` rows in bf16 (``shared`` = a)."""
    g = _gen(_key(seed, 4, rows), device)
    z = torch.randn(shape.hidden, generator=g, device=device)
    e = torch.randn((rows, shape.hidden), generator=g, device=device)
    v = shared * z[None, :] + (max(0.0, 1.0 - shared * shared) ** 0.5) * e
    v = v / v.pow(2).mean(dim=1, keepdim=True).sqrt()
    return v.to(torch.bfloat16)


def make_router(shape: LayerShape, seed: int, layer: int = 0, device="cuda",
                dtype: torch.dtype = torch.bfloat16) -> RouterWeights:
    g = _gen(_key(seed, layer, 3), device)
    H, r, NB = shape.hidden, shape.rank, shape.num_blocks
    enc_w = (torch.randn((r, H), generator=g, device=device) / H ** 0.5).to(torch.bfloat16).to(dtype)
    score_w = (torch.randn((NB, r), generator=g, device=device) / 8.0).to(torch.bfloat16).to(dtype)
    score_b = (torch.randn(NB, generator=g, device=device) * 0.1).to(torch.bfloat16).to(dtype)
    enc_b = torch.zeros(r, device=device, dtype=dtype)
    return RouterWeights(enc_w=enc_w, score_w=score_w, top_k=shape.top_k, basis_top_k=r, enc_b=enc_b,
                         score_b=score_b)


def make_nf4_matrix(rows: int, cols: int, seed: int, device="cuda", code: torch.Tensor | None = None,
                    chunk_elems: int = 1 << 25):
    """NF4 of an N(0, 0.02) ``[rows, cols]`` weight: packed ``[rows*cols/2]``, absmax ``[rows*cols/64]``."""
    code = nf4_code(device) if code is None else code
    g = _gen(seed, device)
    packed = torch.empty(rows * cols // 2, dtype=torch.uint8, device=device)
    absmax = torch.empty(rows * cols // 64, dtype=torch.float32, device=device)
    chunk_rows = max(1, chunk_elems // cols)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        w = torch.randn((r1 - r0, cols), generator=g, device=device) * WEIGHT_STD
        p, a = quantize_nf4(w, code, chunk_rows=chunk_rows)
        packed[r0 * cols // 2:r1 * cols // 2] = p
        absmax[r0 * cols // 64:r1 * cols // 64] = a
        del w
    return packed, absmax


def make_layer_bnb(shape: LayerShape, seed: int, layer: int = 0, device="cuda") -> dict:
    """Whole-layer NF4 weights in bitsandbytes row-major layout."""
    code = nf4_code(device)
    H, I = shape.hidden, shape.intermediate
    gp, ga = make_nf4_matrix(I, H, _key(seed, layer, 0), device, code)
    upk, ua = make_nf4_matrix(I, H, _key(seed, layer, 1), device, code)
    dp, da = make_nf4_matrix(H, I, _key(seed, layer, 2), device, code)
    return {"gate_packed": gp, "gate_absmax": ga, "up_packed": upk, "up_absmax": ua, "down_packed": dp,
            "down_absmax": da, "code": code}


def make_layer_weights(shape: LayerShape, seed: int, layer: int = 0, device="cuda",
                       keep_bnb: bool = False):
    """Device-resident ``SparseMlpWeights`` (down repacked block-major)."""
    bnb = make_layer_bnb(shape, seed, layer, device)
    w = SparseMlpWeights.from_bnb_rowmajor(hidden=shape.hidden, intermediate=shape.intermediate,
                                           gate_packed=bnb["gate_packed"], gate_absmax=bnb["gate_absmax"],
                                           up_packed=bnb["up_packed"], up_absmax=bnb["up_absmax"],
                                           down_packed=bnb["down_packed"], down_absmax=bnb["down_absmax"],
                                           code=bnb["code"])
    if keep_bnb:
        return w, bnb
    del bnb
    return w
