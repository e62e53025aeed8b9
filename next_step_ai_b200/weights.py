"""Device-resident NF4 MLP weights and learned-basis router weights.

``SparseMlpWeights`` holds one decoder layer's gate/up/down NF4 weights in the
layout the decode kernels read:

* gate/up: bitsandbytes row-major, i.e. one 32-row block = ``32*H/2`` bytes +
  ``32*H/64`` fp32 absmax, blocks back to back (the reference's
  ``packed_blocks`` / ``absmax_blocks`` views, ``streaming_llama_runtime.py:4446-4452``);
* down: block-major ``[NB][H][16]`` + ``[NB][H]`` -- every 32-column block's
  column slice contiguous, the layout of the reference's down-proj column
  cache entries (``:4506-4513``) -- so one block's rows stream coalesced.

By default pools are repacked into the lane-interleaved "tiled" layout
(``include/nsm.h``, ``NSM_LAYOUT_*``): every warp load of the decode kernels
then covers 512 contiguous bytes and a lane's four absmax values arrive in one
16-byte load.  ``layout=0`` keeps the bitsandbytes / block-major layouts above.

A pool may hold only some blocks (a hot-block cache or a shard); ``pool_rows``
counts them and a block map sends block ids to pool rows.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib
from ._torch import dtype_code, ptr, row_ptr, stream_handle
from .nf4 import Nf4ParamMeta


@dataclass
class RouterWeights:
    """Per-layer learned-basis router (the reference's routing dict,
    ``streaming_llama_runtime.py:849-991``: enc_w, enc_b, route_score_weight,
    route_score_bias, down_block_norm, top_k, basis_top_k)."""

    enc_w: torch.Tensor               # [rank, H]
    score_w: torch.Tensor             # [NB, rank] (legacy: dec_norm_t.T)
    top_k: int
    basis_top_k: int
    enc_b: torch.Tensor | None = None
    score_b: torch.Tensor | None = None
    down_block_norm: torch.Tensor | None = None  # [NB] fp32
    legacy_abs_latent: bool = False
    _c: object = field(default=None, repr=False)

    def __post_init__(self) -> None:
        dt = self.enc_w.dtype
        for name in ("score_w", "enc_b", "score_b"):
            t = getattr(self, name)
            if t is not None and t.dtype != dt:
                setattr(self, name, t.to(dt))
        self.enc_w = self.enc_w.contiguous()
        self.score_w = self.score_w.contiguous()
        if self.down_block_norm is not None:
            self.down_block_norm = self.down_block_norm.to(torch.float32).contiguous()

    @classmethod
    def from_routing(cls, routing: dict, *, layer_idx: int = 0, sparse_runtime_top_k: int = 0, sparse_top_k: int = 1,
                     basis_top_k_by_layer: dict | None = None, prefill_top_k: int | None = None,
                     device: torch.device | str | None = None) -> "RouterWeights":
        """From one layer of the reference runtime's ``_sparse_routing`` dict,
        resolved as ``_route_sparse_mlp`` / ``_compute_sparse_basis_latent``
        read it (``streaming_llama_runtime.py:4209-4250``, ``:4311-4352``):
        the score head ``route_score_weight`` (+ ``route_score_bias``) when it
        is a tensor, else the legacy ``|latent| @ dec_norm_t``; the optional
        ``down_block_norm``; ``top_k`` else the runtime's k, a prefill
        override, clamped to ``[1, NB]``; ``basis_top_k`` else the by-layer
        table else 8, clamped to ``[1, rank]``.  Weights stay in ``enc_w``'s
        dtype (the runtime computes the router in it)."""
        def put(t):
            return t if t is None or device is None else t.to(device)

        enc_w = put(routing["enc_w"])
        enc_b = put(routing.get("enc_b"))
        sw = routing.get("route_score_weight")
        legacy = not torch.is_tensor(sw)
        if legacy:
            score_w = put(routing["dec_norm_t"]).t().contiguous()  # [NB, rank]
            score_b = None
        else:
            score_w = put(sw)
            sb = routing.get("route_score_bias")
            score_b = put(sb) if torch.is_tensor(sb) else None
        dbn = routing.get("down_block_norm")
        dbn = put(dbn.to(torch.float32).reshape(-1)) if torch.is_tensor(dbn) else None
        nb, rank = int(score_w.shape[0]), int(enc_w.shape[0])
        if dbn is not None and int(dbn.numel()) != nb:
            dbn = None  # the runtime ignores a norm of the wrong length
        k = int(routing.get("top_k", sparse_runtime_top_k if int(sparse_runtime_top_k) > 0 else sparse_top_k))
        if prefill_top_k is not None:
            k = int(prefill_top_k)
        btk = int(routing.get("basis_top_k", (basis_top_k_by_layer or {}).get(int(layer_idx), 8)))
        return cls(enc_w=enc_w, score_w=score_w, enc_b=enc_b, score_b=score_b, down_block_norm=dbn,
                   top_k=max(1, min(k, nb)), basis_top_k=max(1, min(btk, rank)), legacy_abs_latent=legacy)

    @property
    def rank(self) -> int:
        return int(self.enc_w.shape[0])

    @property
    def hidden(self) -> int:
        return int(self.enc_w.shape[1])

    @property
    def num_blocks(self) -> int:
        return int(self.score_w.shape[0])

    def to_c(self) -> _lib.RouterWeightsC:
        c = _lib.RouterWeightsC()
        c.enc_w = ptr(self.enc_w)
        c.enc_b = ptr(self.enc_b)
        c.score_w = ptr(self.score_w)
        c.score_b = ptr(self.score_b)
        c.down_block_norm = ptr(self.down_block_norm)
        c.weight_dtype = dtype_code(self.enc_w.dtype)
        c.rank = self.rank
        c.num_blocks = self.num_blocks
        c.top_k = int(self.top_k)
        c.basis_top_k = int(self.basis_top_k)
        c.legacy_abs_latent = int(self.legacy_abs_latent)
        self._c = c
        return c


@dataclass
class SparseMlpWeights:
    hidden: int
    intermediate: int
    gate_packed: torch.Tensor   # [P, 32*H/2] uint8
    gate_absmax: torch.Tensor   # [P, 32*H/64] fp32
    up_packed: torch.Tensor
    up_absmax: torch.Tensor
    down_packed: torch.Tensor   # [P, H, 16] uint8 (block-major)
    down_absmax: torch.Tensor   # [P, H] fp32
    gate_code: torch.Tensor
    up_code: torch.Tensor
    down_code: torch.Tensor
    gate_bias: torch.Tensor | None = None
    up_bias: torch.Tensor | None = None
    down_bias: torch.Tensor | None = None
    layout: int = 0
    _c: object = field(default=None, repr=False)

    def __post_init__(self) -> None:
        # equal gate and up codebooks (the standard NF4 one) let the tiled gate/up
        # kernel use one lookup table and more warps; checked once here, on the host
        self._shared_code = bool(self.gate_code.shape == self.up_code.shape
                                 and torch.equal(self.gate_code, self.up_code))

    @property
    def pool_rows(self) -> int:
        return int(self.gate_packed.shape[0])

    @property
    def num_blocks(self) -> int:
        return self.intermediate // 32

    def to_c(self) -> _lib.MlpWeightsC:
        c = _lib.MlpWeightsC()
        c.gate_packed = row_ptr(self.gate_packed)
        c.gate_absmax = row_ptr(self.gate_absmax)
        c.up_packed = row_ptr(self.up_packed)
        c.up_absmax = row_ptr(self.up_absmax)
        c.down_packed = row_ptr(self.down_packed)
        c.down_absmax = row_ptr(self.down_absmax)
        c.gate_code = ptr(self.gate_code)
        c.up_code = ptr(self.up_code)
        c.down_code = ptr(self.down_code)
        bias = next((b for b in (self.gate_bias, self.up_bias, self.down_bias) if b is not None), None)
        c.gate_bias = ptr(self.gate_bias)
        c.up_bias = ptr(self.up_bias)
        c.down_bias = ptr(self.down_bias)
        c.bias_dtype = dtype_code(bias.dtype) if bias is not None else 0
        c.pool_rows = self.pool_rows
        c.gateup_block_stride = int(self.gate_packed.stride(0))
        c.gateup_absmax_block_stride = int(self.gate_absmax.stride(0))
        c.down_block_stride = int(self.down_packed.stride(0))
        c.down_row_stride = 16
        c.down_absmax_block_stride = int(self.down_absmax.stride(0))
        c.down_absmax_row_stride = 1
        c.layout = int(self.layout) | (_lib.NSM_LAYOUT_SHARED_CODE if self._shared_code else 0)
        self._c = c
        return c

    @classmethod
    def from_bnb_rowmajor(cls, *, hidden: int, intermediate: int, gate_packed: torch.Tensor, gate_absmax: torch.Tensor,
                          up_packed: torch.Tensor, up_absmax: torch.Tensor, down_packed: torch.Tensor,
                          down_absmax: torch.Tensor, code: torch.Tensor, up_code: torch.Tensor | None = None,
                          down_code: torch.Tensor | None = None, tiled: bool = True,
                          **biases) -> "SparseMlpWeights":
        """From whole bitsandbytes NF4 weights (gate/up ``[I, H]``, down
        ``[H, I]``, packed row-major, fp32 absmax) already on the GPU."""
        H, I = int(hidden), int(intermediate)
        if H % 64 or I % 64:
            raise RuntimeError("hidden and intermediate must be multiples of 64")
        gm = Nf4ParamMeta(I, H)
        dev = gate_packed.device
        nb = I // 32
        code = code.to(device=dev, dtype=torch.float32).contiguous()
        uc = up_code.to(dev, torch.float32).contiguous() if up_code is not None else code
        dc = down_code.to(dev, torch.float32).contiguous() if down_code is not None else code
        lib = _lib.load()
        if tiled:
            w = cls(hidden=H, intermediate=I,
                    gate_packed=torch.empty((nb, gm.bytes_per_block), dtype=torch.uint8, device=dev),
                    gate_absmax=torch.empty((nb, gm.absmax_per_block), dtype=torch.float32, device=dev),
                    up_packed=torch.empty((nb, gm.bytes_per_block), dtype=torch.uint8, device=dev),
                    up_absmax=torch.empty((nb, gm.absmax_per_block), dtype=torch.float32, device=dev),
                    down_packed=torch.empty((nb, H, 16), dtype=torch.uint8, device=dev),
                    down_absmax=torch.empty((nb, H), dtype=torch.float32, device=dev),
                    gate_code=code, up_code=uc, down_code=dc,
                    layout=_lib.NSM_LAYOUT_GATEUP_TILED | _lib.NSM_LAYOUT_DOWN_TILED, **biases)
            src = [t.contiguous() for t in (gate_packed, gate_absmax.float(), up_packed, up_absmax.float(),
                                            down_packed, down_absmax.float())]
            _lib.check(lib.nsm_repack_tiled(*[ptr(t) for t in src], H, I, None, None, nb, ctypes.byref(w.to_c()),
                                            stream_handle(dev)), "nsm_repack_tiled")
            del src
            return w
        dp = torch.empty((nb, H, 16), dtype=torch.uint8, device=dev)
        da = torch.empty((nb, H), dtype=torch.float32, device=dev)
        _lib.check(lib.nsm_repack_down_block_major(
            ptr(down_packed.contiguous()), ptr(down_absmax.to(torch.float32).contiguous()), H, I, None, 0,
            ptr(dp), ptr(da), stream_handle(dev)), "nsm_repack_down_block_major")
        return cls(
            hidden=H, intermediate=I,
            gate_packed=gate_packed.reshape(nb, gm.bytes_per_block).contiguous(),
            gate_absmax=gate_absmax.to(torch.float32).reshape(nb, gm.absmax_per_block).contiguous(),
            up_packed=up_packed.reshape(nb, gm.bytes_per_block).contiguous(),
            up_absmax=up_absmax.to(torch.float32).reshape(nb, gm.absmax_per_block).contiguous(),
            down_packed=dp, down_absmax=da, gate_code=code, up_code=uc, down_code=dc, **biases)


def gathered_mlp_c(*, hidden: int, gate_packed: torch.Tensor, gate_absmax: torch.Tensor, up_packed: torch.Tensor,
                   up_absmax: torch.Tensor, down_packed: torch.Tensor, down_absmax: torch.Tensor,
                   gate_code: torch.Tensor, up_code: torch.Tensor, down_code: torch.Tensor,
                   gate_bias=None, up_bias=None, down_bias=None) -> tuple[_lib.MlpWeightsC, list]:
    """C descriptor for the reference runtime's gathered layout:
    gate/up ``[U, 32*H/2]`` + ``[U, 32*H/64]``, down ``[H, U, 16]`` + ``[H, U]``."""
    U = int(gate_packed.shape[0]) if gate_packed.dim() > 1 else int(gate_packed.numel() // (16 * hidden))
    keep = [t.contiguous() if t is not None else None for t in
            (gate_packed, gate_absmax, up_packed, up_absmax, down_packed, down_absmax, gate_code, up_code, down_code,
             gate_bias, up_bias, down_bias)]
    gp, ga, upk, ua, dp, da, gc, uc, dc, gb, ub, db = keep
    c = _lib.MlpWeightsC()
    c.gate_packed, c.gate_absmax, c.up_packed, c.up_absmax = ptr(gp), ptr(ga), ptr(upk), ptr(ua)
    c.down_packed, c.down_absmax = ptr(dp), ptr(da)
    c.gate_code, c.up_code, c.down_code = ptr(gc), ptr(uc), ptr(dc)
    c.gate_bias, c.up_bias, c.down_bias = ptr(gb), ptr(ub), ptr(db)
    bias = next((b for b in (gb, ub, db) if b is not None), None)
    c.bias_dtype = dtype_code(bias.dtype) if bias is not None else 0
    c.pool_rows = U
    c.gateup_block_stride = 16 * hidden
    c.gateup_absmax_block_stride = hidden // 2
    c.down_block_stride = 16
    c.down_row_stride = 16 * U
    c.down_absmax_block_stride = 1
    c.down_absmax_row_stride = U
    c.down_absmax_pair = 0
    return c, keep
