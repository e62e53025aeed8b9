"""GPU NF4 LM head (the reference's ``RuntimeLmHeadMixin``,
``llama3_neuroplastic/experiments/runtime/lm_head.py:148-468``).

``Nf4LmHead`` keeps one bitsandbytes-layout NF4 LM-head weight resident and
computes ``logits = hidden @ dequant(W).T (+ bias)`` with ``nsm_lm_head_nf4``
(``csrc/nsm_lmhead.cu``): a dense NF4 GEMV that streams the packed weight once
per call.  The weight comes from a checkpoint's quantised ``lm_head.weight``
(nested statistics decoded, as ``_materialize_lm_head_nf4_on_gpu`` does at
``:294-306``) or from a dense weight quantised blockwise on the device (the
reference quantises on the CPU with bitsandbytes, ``:177-265``; the block size
is chosen the same way, ``:160-175``).

Deviation on purpose: the reference's NF4 head calls
``triton_sparse_input_linear_4bit`` with every block active (``:450-468``); that
kernel reads its weight as ``weight.t()`` (``triton_sparse_mlp.py:495-496``)
while the LM head's bytes are row-major, so its GPU logits differ from its own
dense head (``F.linear``, ``:472-480``).  This head computes the dense head's
math.
"""
from __future__ import annotations

import os

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_handle
from .nf4 import nf4_code, quantize_nf4


def resolve_lm_head_nf4_quant_block_size(in_features: int) -> int:
    """``_resolve_lm_head_nf4_quant_block_size`` (``lm_head.py:160-175``): the
    ``STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE`` override when it divides
    ``in_features``, else the first of 64, 128, 256, 32 that does."""
    raw = os.getenv("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", "").strip()
    if raw:
        try:
            v = int(raw)
        except ValueError:
            v = 0
        if v > 0 and int(in_features) % v == 0:
            return v
    for c in (64, 128, 256, 32):
        if int(in_features) % c == 0:
            return c
    raise RuntimeError(f"Unable to select an NF4 quant block size for in_features={int(in_features)}; "
                       "set STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE to a positive divisor.")


class Nf4LmHead:
    """A resident NF4 LM head: ``packed`` uint8 ``[V*H/2]`` (row-major, high
    nibble = even element), ``absmax`` fp32 ``[V*H/qbs]``, ``code`` fp32 [16]."""

    def __init__(self, packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, *, out_features: int,
                 in_features: int, quant_block_size: int = 64, bias: torch.Tensor | None = None):
        for name, t in (("packed", packed), ("absmax", absmax), ("code", code)):
            require_cuda(t, name)
        V, H, qbs = int(out_features), int(in_features), int(quant_block_size)
        if packed.numel() * 2 != V * H:
            raise RuntimeError(f"packed has {packed.numel()} bytes for a [{V}, {H}] NF4 weight")
        if absmax.numel() * qbs != V * H:
            raise RuntimeError(f"absmax has {absmax.numel()} values for a [{V}, {H}] weight with blocksize {qbs}")
        if H % 256 or qbs % 64:
            raise RuntimeError(f"in_features ({H}) must be a multiple of 256 and quant_block_size ({qbs}) of 64")
        # the kernel copies 16-byte pieces of the weight and 16-byte absmax runs
        self.packed = packed.reshape(-1).contiguous()
        if self.packed.data_ptr() % 16:
            self.packed = self.packed.clone()
        self.absmax = absmax.reshape(-1).to(torch.float32).contiguous()
        if self.absmax.data_ptr() % 16:
            self.absmax = self.absmax.clone()
        self.code = code.reshape(-1).to(device=packed.device, dtype=torch.float32).contiguous()
        self.bias = bias.reshape(-1).contiguous() if bias is not None else None
        self.out_features, self.in_features, self.quant_block_size = V, H, qbs
        self.device = packed.device
        self._lib = _lib.load()
        self._ws: torch.Tensor | None = None

    # ---- construction
    @classmethod
    def from_param(cls, p, device: torch.device | str = "cuda", bias: torch.Tensor | None = None) -> "Nf4LmHead":
        """From a ``checkpoint.Nf4Param`` (host tensors)."""
        dev = torch.device(device)
        return cls(p.packed.to(dev), p.absmax.to(dev), p.code.to(dev), out_features=p.out_features,
                   in_features=p.in_features, quant_block_size=p.blocksize,
                   bias=bias.to(dev) if bias is not None else None)

    @classmethod
    def from_checkpoint(cls, ckpt, name: str = "lm_head.weight", device: torch.device | str = "cuda") -> "Nf4LmHead":
        """From a quantised weight of an ``Nf4Checkpoint``; a dense one is
        quantised on the device (``_materialize_lm_head_nf4_on_gpu``)."""
        w, aux = ckpt.load_raw(name)
        if aux:
            return cls.from_param(ckpt.load_param(name), device)
        return cls.from_dense(w, device)

    @classmethod
    def from_dense(cls, weight: torch.Tensor, device: torch.device | str = "cuda",
                   quant_block_size: int | None = None, bias: torch.Tensor | None = None) -> "Nf4LmHead":
        """Blockwise NF4 quantisation of a dense ``[V, H]`` weight on the device
        (nearest code value, absmax per block)."""
        if weight.dim() != 2:
            raise RuntimeError(f"Expected a rank-2 dense LM head weight, got shape {tuple(weight.shape)}")
        V, H = (int(s) for s in weight.shape)
        qbs = int(quant_block_size) if quant_block_size is not None else resolve_lm_head_nf4_quant_block_size(H)
        dev = torch.device(device)
        code = nf4_code(dev)
        packed, absmax = quantize_nf4(weight.to(dev), code, qbs)
        return cls(packed, absmax, code, out_features=V, in_features=H, quant_block_size=qbs,
                   bias=bias.to(dev) if bias is not None else None)

    # ---- forward
    @property
    def max_tokens_per_call(self) -> int:
        return int(self._lib.nsm_lm_head_max_tokens(self.in_features))

    def weight_bytes(self) -> int:
        return self.packed.numel() + 4 * self.absmax.numel() + 4 * self.code.numel()

    def __call__(self, hidden: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return self.forward(hidden, out_dtype)

    def forward(self, hidden: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """``hidden [..., H]`` -> ``logits [..., V]`` (``out_dtype``, default
        hidden's); tokens are processed in groups of ``max_tokens_per_call``,
        each group streaming the weight once."""
        require_cuda(hidden, "hidden")
        H, V = self.in_features, self.out_features
        if hidden.shape[-1] != H:
            raise RuntimeError(f"hidden has {hidden.shape[-1]} features but the LM head expects {H}")
        x = hidden.reshape(-1, H).contiguous()
        rows = x.shape[0]
        out = torch.empty((rows, V), dtype=out_dtype or hidden.dtype, device=self.device)
        per = self.max_tokens_per_call
        if per <= 0:
            raise RuntimeError(f"the NF4 LM head does not fit in_features={H}")
        for r0 in range(0, rows, per):
            n = min(per, rows - r0)
            need = int(self._lib.nsm_lm_head_workspace_bytes(n, V, H))
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=self.device)
            _lib.check(self._lib.nsm_lm_head_nf4(
                x[r0:r0 + n].data_ptr(), dtype_code(x.dtype), n, ptr(self.packed), ptr(self.absmax), ptr(self.code),
                V, H, self.quant_block_size, ptr(self.bias), dtype_code(self.bias.dtype) if self.bias is not None else 0,
                out[r0:r0 + n].data_ptr(), dtype_code(out.dtype), self._ws.data_ptr(), self._ws.numel(),
                stream_handle(self.device)), "nsm_lm_head_nf4")
        return out.reshape(*hidden.shape[:-1], V)
