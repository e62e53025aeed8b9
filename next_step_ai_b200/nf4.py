"""NF4 helpers on torch tensors: codebook, quantizer and parameter metadata.

The hot path never quantizes; these build synthetic NF4 weights and describe
bitsandbytes NF4 parameters exactly as the reference does
(``llama3_neuroplastic/experiments/streaming_llama_runtime.py:4627-4654``).
Packing convention (as the reference's kernels read it): byte ``i`` holds
element ``2i`` in the high nibble and ``2i+1`` in the low nibble; value =
``code[nibble] * absmax[e // blocksize]``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

NF4_OFFSET = 0.9677083


def nf4_code(device: torch.device | str | None = None) -> torch.Tensor:
    """16-entry NF4 table (QLoRA construction: normal quantiles + exact zero)."""
    pos = torch.special.ndtri(torch.linspace(NF4_OFFSET, 0.5, 9, dtype=torch.float64)[:-1])
    neg = -torch.special.ndtri(torch.linspace(NF4_OFFSET, 0.5, 8, dtype=torch.float64)[:-1])
    vals = torch.sort(torch.cat([pos, torch.zeros(1, dtype=torch.float64), neg])).values
    vals = vals / vals.max()
    return vals.to(torch.float32).to(device if device is not None else "cpu")


def quantize_nf4(w: torch.Tensor, code: torch.Tensor, blocksize: int = 64, chunk_rows: int = 2048):
    """Blockwise NF4 quantization of a row-major weight (nearest code; a tie
    goes to the lower code).  Returns ``(packed uint8 [numel/2], absmax fp32
    [numel/blocksize])`` on ``w``'s device."""
    flat = w.reshape(-1)
    n = flat.numel()
    if n % blocksize or n % 2:
        raise RuntimeError("numel must be a multiple of blocksize and 2")
    code = code.to(device=w.device, dtype=torch.float32)
    mids = ((code[1:].double() + code[:-1].double()) * 0.5).float()
    packed = torch.empty(n // 2, dtype=torch.uint8, device=w.device)
    absmax = torch.empty(n // blocksize, dtype=torch.float32, device=w.device)
    row = w.shape[-1] if w.dim() > 1 else n
    step = max(blocksize, (chunk_rows * row) // blocksize * blocksize)
    for s in range(0, n, step):
        e = min(n, s + step)
        blk = flat[s:e].to(torch.float32).reshape(-1, blocksize)
        am = blk.abs().amax(dim=1)
        safe = torch.where(am > 0, am, torch.ones_like(am))
        nrm = (blk / safe[:, None]).reshape(-1)
        nib = torch.searchsorted(mids, nrm, right=False).to(torch.uint8)
        packed[s // 2:e // 2] = (nib[0::2] << 4) | nib[1::2]
        absmax[s // blocksize:e // blocksize] = am
    return packed, absmax


def dequantize_nf4(packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, blocksize: int = 64):
    p = packed.reshape(-1)
    nib = torch.stack([p >> 4, p & 0x0F], dim=1).reshape(-1).long()
    return code.to(p.device)[nib] * absmax.reshape(-1).repeat_interleave(blocksize)


@dataclass(frozen=True)
class Nf4ParamMeta:
    """Metadata the reference derives from a bitsandbytes QuantState
    (``streaming_llama_runtime.py:4627-4654``)."""

    out_features: int
    in_features: int
    block_size: int = 32
    quant_block_size: int = 64
    quant_type: str = "nf4"

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
