"""NF4 codebook, quantizer and dequantizer (numpy).  TEST INFRASTRUCTURE ONLY.

The reference never quantizes on the hot path: it reads bitsandbytes 0.49.1
(``requirements.txt:7``; third party, not vendored, not installed here) NF4
checkpoints and passes ``quant_state.code`` (16 fp32 values) into every kernel
(``llama3_neuroplastic/experiments/streaming_llama_runtime.py:4640-4643``,
``llama3_neuroplastic/triton_sparse_mlp.py:203``).  The dequant arithmetic the
reference relies on is visible in its own code:

* element ``e`` of a flattened row-major weight lives in byte ``e // 2``; the
  HIGH nibble holds the even element and the LOW nibble the odd element
  (``triton_sparse_mlp.py:856-858``; ``streaming_llama_runtime.py:5469-5476``);
* its value is ``code[nibble] * absmax[e // quant_block_size]``
  (``triton_sparse_mlp.py:859-866``; ``streaming_llama_runtime.py:5480``).

The codebook itself is the published NF4 construction (Dettmers et al.,
QLoRA, 2023): 8 positive and 7 negative normal quantiles at offset 0.9677083,
an exact zero, normalized by the maximum.  Parity never depends on the table
values because the table is an input to both the oracle and the kernels.
"""
from __future__ import annotations

import numpy as np

NF4_OFFSET = 0.9677083


def nf4_code() -> np.ndarray:
    """The 16-entry NF4 table (fp32, ascending), from the QLoRA construction."""
    from scipy.stats import norm

    pos = norm.ppf(np.linspace(NF4_OFFSET, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(NF4_OFFSET, 0.5, 8)[:-1])
    vals = np.sort(np.concatenate([pos, [0.0], neg]))
    vals = vals / vals.max()
    return vals.astype(np.float32)


def quantize_nf4(w: np.ndarray, code: np.ndarray, blocksize: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """Blockwise NF4 quantization of a row-major weight.

    Returns ``(packed uint8 [numel/2], absmax fp32 [numel/blocksize])``.
    ``absmax`` is ``max|w|`` over each run of ``blocksize`` consecutive
    elements of the flattened weight; each element maps to the nearest code
    value of ``w / absmax`` (a tie goes to the lower code).  Byte ``i`` packs
    element ``2i`` in its high nibble and ``2i+1`` in its low nibble.
    """
    flat = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    if flat.size % blocksize != 0 or flat.size % 2 != 0:
        raise ValueError("numel must be a multiple of blocksize and of 2")
    blocks = flat.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax > 0, absmax, np.float32(1.0)).astype(np.float32)
    norm_vals = (blocks / safe[:, None]).astype(np.float32).reshape(-1)
    code = np.asarray(code, dtype=np.float32)
    mids = ((code[1:].astype(np.float64) + code[:-1].astype(np.float64)) * 0.5).astype(np.float32)
    # searchsorted(side="left") => value == midpoint goes to the lower code.
    nib = np.searchsorted(mids, norm_vals, side="left").astype(np.uint8)
    packed = ((nib[0::2] << 4) | nib[1::2]).astype(np.uint8)
    return packed, absmax


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """uint8 bytes -> nibble per element (high nibble = even element)."""
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(p.size * 2, dtype=np.uint8)
    out[0::2] = p >> 4
    out[1::2] = p & 0x0F
    return out


def dequantize_nf4(packed: np.ndarray, absmax: np.ndarray, code: np.ndarray, blocksize: int = 64) -> np.ndarray:
    """``w[e] = code[nibble(e)] * absmax[e // blocksize]`` in fp32 (flat)."""
    nib = unpack_nibbles(packed)
    code = np.asarray(code, dtype=np.float32)
    absmax = np.asarray(absmax, dtype=np.float32).reshape(-1)
    scale = np.repeat(absmax, blocksize)
    if scale.size != nib.size:
        raise ValueError(f"absmax covers {scale.size} elements, packed holds {nib.size}")
    return (code[nib] * scale).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16-representable fp32 (ties to even)."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    # NaN payloads are not produced by the generators; keep inf/nan as is.
    return np.where(np.isfinite(a), out, a).astype(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)
