"""Drop-in for the reference module ``llama3_neuroplastic/triton_sparse_mlp.py``.

Same public names, argument meanings and ``RuntimeError`` behaviour, backed by
the sm_100a kernels of ``libnsm.so`` instead of Triton.  Differences, on
purpose:

* ``triton_sparse_mlp_decode_4bit_single_kernel_sm75`` runs on B200; the
  reference refuses anything but sm_75 (``:1401-1402``).
* The functions are forward-only (decode).  The reference's autograd
  backward needs bitsandbytes to re-materialise the weight (``:208-220``).
* ``triton_fused_sparse_mlp_decode_4bit`` keeps the reference's composition
  (output, output, SiLU*up, input; pinned by the reference's
  ``tests/test_throughput_contract.py:364-407``) and resolves the two
  building blocks through this module's globals, so monkeypatching them works
  the same way.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _lib
from ._torch import dtype_code, ptr, stream_handle
from .mlp import decode_gathered

_DEFAULT_MAX_FUSED_TOPK = 32


def triton_sparse_mlp_available() -> bool:
    """True when libnsm.so loads and the current CUDA device is sm_100."""
    try:
        _lib.load()
    except Exception:
        return False
    if not torch.cuda.is_available():
        return False
    return tuple(torch.cuda.get_device_capability()) == (10, 0)


def _prepare_activation_tensor(x: torch.Tensor) -> torch.Tensor:
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        x = x.to(torch.float16)
    return x.contiguous()


def _require_cuda(x: torch.Tensor, what: str) -> None:
    if x.device.type != "cuda":
        raise RuntimeError(f"{what} requires CUDA tensors")


def triton_sparse_input_linear_4bit(x_flat: torch.Tensor, active_idx: torch.Tensor, *, packed_weight: torch.Tensor,
                                    absmax: torch.Tensor, code: torch.Tensor, out_features: int, in_features: int,
                                    quant_block_size: int, bias: torch.Tensor | None, block_size: int,
                                    quant_weight_ref: torch.Tensor | None = None) -> torch.Tensor:
    """Reference: ``triton_sparse_mlp.py:1303-1337`` (kernels ``:437-575``)."""
    _require_cuda(x_flat, "4-bit sparse input kernel")
    x = _prepare_activation_tensor(x_flat)
    if int(block_size) <= 0:
        raise RuntimeError("block_size must be > 0 for triton_sparse_input_linear_4bit")
    if int(in_features) % int(block_size) != 0:
        raise RuntimeError(f"in_features ({int(in_features)}) must be divisible by block_size ({int(block_size)})")
    dev = x.device
    idx = active_idx.to(device=dev, dtype=torch.int32).contiguous()
    rows = int(x.shape[0])
    top_k = int(idx.shape[1]) if idx.dim() > 1 else int(idx.numel())
    packed = packed_weight.to(device=dev, dtype=torch.uint8).contiguous()
    am = absmax.to(device=dev, dtype=torch.float32).contiguous()
    cd = code.to(device=dev, dtype=torch.float32).contiguous()
    b = bias.to(device=dev, dtype=x.dtype).contiguous() if bias is not None else None
    out = torch.empty((rows, int(out_features)), device=dev, dtype=x.dtype)
    _lib.check(_lib.load().nsm_sparse_input_linear_4bit(
        ptr(x), dtype_code(x.dtype), rows, ptr(idx) if idx.numel() else None, top_k, ptr(packed), ptr(am), ptr(cd),
        int(out_features), int(in_features), int(quant_block_size), ptr(b), int(block_size), ptr(out),
        stream_handle(dev)), "triton_sparse_input_linear_4bit")
    return out


def triton_sparse_output_linear_4bit(x_flat: torch.Tensor, active_idx: torch.Tensor, flat_mask: torch.Tensor, *,
                                     packed_weight: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor,
                                     input_dim: int, quant_block_size: int, bias: torch.Tensor | None,
                                     block_size: int, quant_weight_ref: torch.Tensor | None = None) -> torch.Tensor:
    """Reference: ``triton_sparse_mlp.py:1340-1375`` (kernel ``:578-651``)."""
    _require_cuda(x_flat, "4-bit sparse output kernel")
    x = _prepare_activation_tensor(x_flat)
    if int(block_size) <= 0:
        raise RuntimeError("block_size must be > 0 for triton_sparse_output_linear_4bit")
    if int(input_dim) % int(block_size) != 0:
        raise RuntimeError(f"input_dim ({int(input_dim)}) must be divisible by block_size ({int(block_size)})")
    dev = x.device
    rows = int(x.shape[0])
    width = int(flat_mask.shape[1])
    idx = active_idx.to(device=dev, dtype=torch.int32).contiguous()
    top_k = int(idx.shape[1]) if idx.dim() > 1 else int(idx.numel())
    mask = flat_mask.to(device=dev, dtype=x.dtype).contiguous()
    packed = packed_weight.to(device=dev, dtype=torch.uint8).contiguous()
    am = absmax.to(device=dev, dtype=torch.float32).contiguous()
    cd = code.to(device=dev, dtype=torch.float32).contiguous()
    b = bias.to(device=dev, dtype=x.dtype).contiguous() if bias is not None else None
    out = torch.empty((rows, width), device=dev, dtype=x.dtype)
    _lib.check(_lib.load().nsm_sparse_output_linear_4bit(
        ptr(x), dtype_code(x.dtype), rows, ptr(idx) if idx.numel() else None, top_k, ptr(mask), width, ptr(packed),
        ptr(am), ptr(cd), int(input_dim), int(quant_block_size), ptr(b), int(block_size), ptr(out),
        stream_handle(dev)), "triton_sparse_output_linear_4bit")
    return out


def triton_sparse_mlp_decode_4bit_single_kernel_sm75(x_flat, active_blocks, gate_packed, gate_absmax, gate_code,
                                                     up_packed, up_absmax, up_code, down_packed, down_absmax,
                                                     down_code, out, out_accum, hidden_size, block_size,
                                                     quant_block_size, top_k):
    """Whole single-token decode MLP on gathered blocks.  Reference:
    ``triton_sparse_mlp.py:1378-1516`` (validation messages kept); runs on
    sm_100 instead of requiring sm_75."""
    if x_flat.device.type != "cuda":
        raise RuntimeError("Single-kernel sparse MLP decode requires CUDA")
    if int(block_size) != 32:
        raise RuntimeError("Single-kernel sparse MLP decode currently requires block_size=32")
    if int(top_k) <= 0:
        raise RuntimeError("Single-kernel sparse MLP decode requires top_k > 0")
    hidden_size = int(hidden_size)
    quant_block_size = int(quant_block_size)
    top_k = int(top_k)
    if hidden_size <= 0 or quant_block_size <= 0:
        raise RuntimeError("hidden_size and quant_block_size must be positive")
    if quant_block_size != 64:
        raise RuntimeError("this B200 path requires quant_block_size=64")
    x_vec = x_flat.reshape(-1)
    if int(x_vec.numel()) != hidden_size:
        raise RuntimeError(f"x_flat has {int(x_vec.numel())} elements but hidden_size={hidden_size}")
    ab = active_blocks.reshape(-1)
    if int(ab.numel()) != top_k:
        raise RuntimeError(f"active_blocks has {int(ab.numel())} entries but top_k={top_k}")
    bpr = hidden_size // 2
    apr = hidden_size // quant_block_size
    if int(gate_packed.numel()) != top_k * 32 * bpr:
        raise RuntimeError("gate_packed size does not match [top_k, block_size, hidden_size/2] layout")
    if int(up_packed.numel()) != top_k * 32 * bpr:
        raise RuntimeError("up_packed size does not match [top_k, block_size, hidden_size/2] layout")
    if int(gate_absmax.numel()) != top_k * 32 * apr:
        raise RuntimeError("gate_absmax size does not match [top_k, block_size, hidden_size/quant_block_size] layout")
    if int(up_absmax.numel()) != top_k * 32 * apr:
        raise RuntimeError("up_absmax size does not match [top_k, block_size, hidden_size/quant_block_size] layout")
    if int(down_absmax.numel()) != hidden_size * top_k:
        raise RuntimeError("down_absmax size does not match [hidden_size, top_k] layout")
    if int(down_packed.numel()) != hidden_size * top_k * 16:
        raise RuntimeError("down_packed size does not match [hidden_size, top_k, block_size/2] layout")
    if int(out_accum.numel()) < hidden_size:
        raise RuntimeError("out_accum scratch is smaller than hidden_size")
    dev = x_flat.device
    y32 = out_accum.reshape(-1)[:hidden_size]
    if y32.dtype != torch.float32 or not y32.is_contiguous():
        y32 = torch.empty(hidden_size, dtype=torch.float32, device=dev)
    decode_gathered(x_vec, hidden_size=hidden_size, gate_packed=gate_packed, gate_absmax=gate_absmax,
                    gate_code=gate_code, up_packed=up_packed, up_absmax=up_absmax, up_code=up_code,
                    down_packed=down_packed, down_absmax=down_absmax, down_code=down_code, out=y32)
    if y32.data_ptr() != out_accum.reshape(-1)[:hidden_size].data_ptr():
        out_accum.reshape(-1)[:hidden_size].copy_(y32)
    out.reshape(-1)[:hidden_size].copy_(y32.to(out.dtype))
    return out.view_as(x_flat)


def triton_fused_sparse_mlp_decode_4bit(x_flat, active_idx, flat_mask, *, gate_packed_weight, gate_absmax, gate_code,
                                        gate_input_dim, gate_quant_block_size, gate_bias, up_packed_weight, up_absmax,
                                        up_code, up_input_dim, up_quant_block_size, up_bias, down_packed_weight,
                                        down_absmax, down_code, down_out_features, down_in_features,
                                        down_quant_block_size, down_bias, block_size):
    """Reference: ``triton_sparse_mlp.py:1519-1585``."""
    g = globals()
    gate = g["triton_sparse_output_linear_4bit"](
        x_flat, active_idx, flat_mask, packed_weight=gate_packed_weight, absmax=gate_absmax, code=gate_code,
        input_dim=int(gate_input_dim), quant_block_size=int(gate_quant_block_size), bias=gate_bias,
        block_size=int(block_size), quant_weight_ref=None)
    up = g["triton_sparse_output_linear_4bit"](
        x_flat, active_idx, flat_mask, packed_weight=up_packed_weight, absmax=up_absmax, code=up_code,
        input_dim=int(up_input_dim), quant_block_size=int(up_quant_block_size), bias=up_bias,
        block_size=int(block_size), quant_weight_ref=None)
    activated = F.silu(gate)
    activated.mul_(up)
    return g["triton_sparse_input_linear_4bit"](
        activated, active_idx, packed_weight=down_packed_weight, absmax=down_absmax, code=down_code,
        out_features=int(down_out_features), in_features=int(down_in_features),
        quant_block_size=int(down_quant_block_size), bias=down_bias, block_size=int(block_size),
        quant_weight_ref=None)


__all__ = [
    "triton_sparse_mlp_available",
    "triton_sparse_input_linear_4bit",
    "triton_sparse_output_linear_4bit",
    "triton_sparse_mlp_decode_4bit_single_kernel_sm75",
    "triton_fused_sparse_mlp_decode_4bit",
]
del ctypes
