"""Torch-facing entry points of the blockwise-sparse NF4 decode MLP.

Each function checks shapes, takes raw pointers, and calls ``libnsm.so`` on
the current CUDA stream.  None of them has a CPU or eager fallback.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._torch import WORKSPACES, dtype_code, ptr, require_cuda, stream_handle
from .weights import RouterWeights, SparseMlpWeights, gathered_mlp_c


def _k_for(router: RouterWeights, top_k: int | None) -> int:
    k = int(router.top_k if top_k is None else top_k)
    return max(1, min(k, router.num_blocks))


def route_sparse_mlp(hidden: torch.Tensor, router: RouterWeights, *, top_k: int | None = None,
                     return_scores: bool = False):
    """Block indices ``[N, k]`` (int64, score-descending, ties to the lower
    block id) for ``hidden [..., H]`` -- ``StreamingLlamaRuntime._route_sparse_mlp``
    (``streaming_llama_runtime.py:4311-4352``).  ``top_k`` overrides the
    router's k (the reference's sparse-prefill override, ``:4344-4349``)."""
    require_cuda(hidden, "hidden")
    H = router.hidden
    flat = hidden.reshape(-1, H).contiguous()
    k = _k_for(router, top_k)
    lib = _lib.load()
    saved_k = router.top_k
    router.top_k = k
    rc = router.to_c()
    router.top_k = saved_k
    dev = hidden.device
    rows = int(flat.shape[0])
    idx = torch.empty((rows, k), dtype=torch.int32, device=dev)
    scores = torch.empty((rows, k), dtype=torch.float32, device=dev) if return_scores else None
    st = stream_handle(dev)
    if rows == 1:
        ws = WORKSPACES.get(lib.nsm_decode_workspace_bytes(H, router.num_blocks * 32, k, router.rank), dev)
        _lib.check(lib.nsm_route(flat.data_ptr(), dtype_code(flat.dtype), H, ctypes.byref(rc), idx.data_ptr(),
                                 scores.data_ptr() if scores is not None else None, None, ws.data_ptr(), ws.numel(),
                                 st), "nsm_route")
    elif rows > 1:
        # all rows in three launches (latent, scores, one top-k CTA per row)
        ws = WORKSPACES.get(lib.nsm_route_workspace_bytes(H, router.num_blocks, k, router.rank, rows), dev)
        _lib.check(lib.nsm_route_rows(flat.data_ptr(), dtype_code(flat.dtype), rows, H, ctypes.byref(rc),
                                      idx.data_ptr(), scores.data_ptr() if scores is not None else None, None,
                                      ws.data_ptr(), ws.numel(), st), "nsm_route_rows")
    out = idx.long()
    return (out, scores) if return_scores else out


def sparse_mlp_decode(x: torch.Tensor | None, router: RouterWeights | None, weights: SparseMlpWeights, *,
                      idx: torch.Tensor | None = None, slot_of_block: torch.Tensor | None = None,
                      block_range: tuple[int, int] | None = None, out_dtype: torch.dtype | None = None,
                      residual: torch.Tensor | None = None, y_prev: torch.Tensor | None = None,
                      norm_weight: torch.Tensor | None = None, eps: float = 1e-5, out: torch.Tensor | None = None,
                      idx_out: torch.Tensor | None = None, score_out: torch.Tensor | None = None) -> torch.Tensor:
    """One token through route -> gate/up gather-GEMV -> SiLU*up -> down.

    ``x``: ``[H]`` MLP input, or ``None`` with ``residual`` (fp32 ``[H]``,
    updated in place with ``y_prev`` and RMS-normalised with ``norm_weight``).
    ``idx``: precomputed block ids instead of the router.  ``slot_of_block`` /
    ``block_range``: which blocks this pool holds (hot cache / shard).
    Returns ``y [H]`` (``out_dtype``, default x's dtype or bf16).
    """
    H, I = weights.hidden, weights.intermediate
    lib = _lib.load()
    dev = weights.gate_packed.device
    if x is not None:
        require_cuda(x, "x")
        x = x.reshape(-1).contiguous()
        if x.numel() != H:
            raise RuntimeError(f"x has {x.numel()} elements but hidden_size={H}")
    elif residual is None:
        raise RuntimeError("either x or residual is required")
    io = None
    if residual is not None:
        if residual.dtype != torch.float32 or residual.numel() != H:
            raise RuntimeError("residual must be fp32 [H]")
        io = _lib.LayerIoC()
        io.residual = ptr(residual)
        io.y_prev = ptr(y_prev.contiguous()) if y_prev is not None else None
        io.y_prev_dtype = dtype_code(y_prev.dtype) if y_prev is not None else 0
        io.norm_weight = ptr(norm_weight) if norm_weight is not None else None
        io.norm_weight_dtype = dtype_code(norm_weight.dtype) if norm_weight is not None else 0
        io.eps = float(eps)
    if out_dtype is None:
        out_dtype = x.dtype if x is not None else torch.bfloat16
    y = out if out is not None else torch.empty(H, dtype=out_dtype, device=dev)
    rc = router.to_c() if router is not None else None
    if idx is not None:
        idx32 = idx.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
        k = int(idx32.numel())
    else:
        if router is None:
            raise RuntimeError("router weights are required when idx is not given")
        idx32 = None
        k = _k_for(router, None)
    rank = router.rank if router is not None else 1
    bm = _lib.BlockMapC()
    if slot_of_block is not None:
        bm.slot_of_block = ptr(slot_of_block)
    lo, hi = block_range if block_range is not None else (0, I // 32)
    bm.block_begin, bm.block_end = int(lo), int(hi)
    wc = weights.to_c()
    ws_bytes = lib.nsm_decode_workspace_bytes(H, I, k, rank)
    ws = WORKSPACES.get(ws_bytes, dev)
    _lib.check(lib.nsm_sparse_mlp_decode(
        ptr(x) if x is not None else None, dtype_code(x.dtype) if x is not None else 0, H, I,
        ctypes.byref(io) if io is not None else None, ctypes.byref(rc) if rc is not None else None,
        ptr(idx32) if idx32 is not None else None, k, ctypes.byref(bm), ctypes.byref(wc), ptr(y),
        dtype_code(y.dtype), ptr(idx_out) if idx_out is not None else None,
        ptr(score_out) if score_out is not None else None, ws.data_ptr(), ws.numel(), stream_handle(dev)),
        "nsm_sparse_mlp_decode")
    return y


def decode_gathered(x: torch.Tensor, *, hidden_size: int, gate_packed, gate_absmax, gate_code, up_packed, up_absmax,
                    up_code, down_packed, down_absmax, down_code, out_dtype: torch.dtype | None = None,
                    act_out: torch.Tensor | None = None, gate_bias=None, up_bias=None, down_bias=None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Single-token MLP on blocks gathered in the reference runtime's layout
    (gate/up ``[U, 32, H/2]``, down ``[H, U, 16]``; ``triton_sparse_mlp.py:1442-1462``)."""
    require_cuda(x, "x")
    H = int(hidden_size)
    xv = x.reshape(-1).contiguous()
    if xv.numel() != H:
        raise RuntimeError(f"x_flat has {xv.numel()} elements but hidden_size={H}")
    U = int(gate_packed.numel() // (16 * H))
    if U <= 0:
        raise RuntimeError("no gathered blocks")
    for name, t, n in (("gate_packed", gate_packed, U * 16 * H), ("up_packed", up_packed, U * 16 * H),
                       ("gate_absmax", gate_absmax, U * H // 2), ("up_absmax", up_absmax, U * H // 2),
                       ("down_packed", down_packed, H * U * 16), ("down_absmax", down_absmax, H * U)):
        if int(t.numel()) != n:
            raise RuntimeError(f"{name} size does not match the gathered layout for U={U}, H={H}")
    c, keep = gathered_mlp_c(hidden=H, gate_packed=gate_packed.reshape(U, -1), gate_absmax=gate_absmax.float(),
                             up_packed=up_packed.reshape(U, -1), up_absmax=up_absmax.float(), down_packed=down_packed,
                             down_absmax=down_absmax.float(), gate_code=gate_code.float(), up_code=up_code.float(),
                             down_code=down_code.float(), gate_bias=gate_bias, up_bias=up_bias, down_bias=down_bias)
    lib = _lib.load()
    y = out if out is not None else torch.empty(H, dtype=out_dtype or xv.dtype, device=xv.device)
    ws = WORKSPACES.get(lib.nsm_decode_rows_workspace_bytes(H, U, 1), xv.device)
    _lib.check(lib.nsm_decode_gathered(ptr(xv), dtype_code(xv.dtype), H, U, ctypes.byref(c), ptr(y),
                                       dtype_code(y.dtype), ptr(act_out) if act_out is not None else None,
                                       ws.data_ptr(), ws.numel(), stream_handle(xv.device)), "nsm_decode_gathered")
    del keep
    return y


def decode_gathered_rows(x: torch.Tensor, flat_mask: torch.Tensor | None, *, gate_packed, gate_absmax, gate_code,
                         up_packed, up_absmax, up_code, down_packed, down_absmax, down_code,
                         out_dtype: torch.dtype | None = None, gate_bias=None, up_bias=None,
                         down_bias=None) -> torch.Tensor:
    """Multi-row MLP on gathered blocks with the reference's per-row
    ``flat_mask`` (``streaming_llama_runtime.py:5451-5492``)."""
    require_cuda(x, "x")
    rows, H = int(x.shape[0]), int(x.shape[-1])
    xv = x.reshape(rows, H).contiguous()
    U = int(gate_packed.numel() // (16 * H))
    c, keep = gathered_mlp_c(hidden=H, gate_packed=gate_packed.reshape(U, -1), gate_absmax=gate_absmax.float(),
                             up_packed=up_packed.reshape(U, -1), up_absmax=up_absmax.float(), down_packed=down_packed,
                             down_absmax=down_absmax.float(), gate_code=gate_code.float(), up_code=up_code.float(),
                             down_code=down_code.float(), gate_bias=gate_bias, up_bias=up_bias, down_bias=down_bias)
    lib = _lib.load()
    y = torch.empty((rows, H), dtype=out_dtype or xv.dtype, device=xv.device)
    fm = flat_mask.reshape(rows, U * 32).to(xv.dtype).contiguous() if flat_mask is not None else None
    ws = WORKSPACES.get(lib.nsm_decode_rows_workspace_bytes(H, U, rows), xv.device)
    _lib.check(lib.nsm_decode_gathered_rows(ptr(xv), dtype_code(xv.dtype), rows, H, U,
                                            ptr(fm) if fm is not None else None,
                                            dtype_code(fm.dtype) if fm is not None else 0, ctypes.byref(c), ptr(y),
                                            dtype_code(y.dtype), ws.data_ptr(), ws.numel(), stream_handle(xv.device)),
               "nsm_decode_gathered_rows")
    del keep
    return y


def union_decode(x: torch.Tensor, idx: torch.Tensor, weights: SparseMlpWeights, *, slot_of_block=None,
                 block_range: tuple[int, int] | None = None, out_dtype: torch.dtype | None = None,
                 return_union: bool = False):
    """Multi-token decode (``rows <= 32``) over the union of the rows' selected
    blocks: each union block's NF4 tiles are dequantised once for all rows and
    row ``r`` only sees its own blocks -- ``_build_sparse_active_layout`` +
    ``_sparse_mlp_forward_fast`` for rows > 1 (``streaming_llama_runtime.py:4857-4908``,
    ``:5433-5492``) with resident weights.

    ``x [rows, H]``, ``idx [rows, k]`` block ids (device).  Returns ``y [rows, H]``
    (and the union's block ids when ``return_union``)."""
    require_cuda(x, "x")
    rows, H = int(x.shape[0]), int(x.shape[-1])
    if H != weights.hidden:
        raise RuntimeError(f"x has hidden {H}, weights {weights.hidden}")
    xv = x.reshape(rows, H).contiguous()
    iv = idx.reshape(rows, -1).to(device=xv.device, dtype=torch.int32).contiguous()
    k = int(iv.shape[1])
    lib = _lib.load()
    wc = weights.to_c()
    bm = _lib.BlockMapC()
    bm.slot_of_block = ptr(slot_of_block) if slot_of_block is not None else None
    lo, hi = block_range if block_range is not None else (0, weights.intermediate // 32)
    bm.block_begin, bm.block_end = int(lo), int(hi)
    y = torch.empty((rows, H), dtype=out_dtype or xv.dtype, device=xv.device)
    umax = min(weights.intermediate // 32, rows * k)
    uni = torch.empty(umax, dtype=torch.int32, device=xv.device)
    cnt = torch.zeros(1, dtype=torch.int32, device=xv.device)
    ws = WORKSPACES.get(lib.nsm_union_workspace_bytes(H, weights.intermediate, rows, k), xv.device)
    _lib.check(lib.nsm_union_decode(ptr(xv), dtype_code(xv.dtype), rows, H, weights.intermediate, ptr(iv), k,
                                    ctypes.byref(bm), ctypes.byref(wc), ptr(y), dtype_code(y.dtype), ptr(uni), ptr(cnt),
                                    ws.data_ptr(), ws.numel(), stream_handle(xv.device)), "nsm_union_decode")
    if return_union:
        return y, uni[: int(cnt.item())]
    return y
