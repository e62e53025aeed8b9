"""Decode-MLP methods of the reference runtime served by ``libnsm.so``.

The reference decodes through ``StreamingLlamaRuntime``
(``llama3_neuroplastic/experiments/streaming_llama_runtime.py``).  Its decode
MLP is five methods; this module gives each a counterpart with the same name,
arguments, return contract and log lines, backed by the sm_100a kernels:

=====================================  ==========================  =====================================
reference method                       here                        kernels
=====================================  ==========================  =====================================
``_route_sparse_mlp`` (:4311-4352)      same                        ``nsm_route`` / ``nsm_route_rows``
``_sparse_mlp_forward_fast`` (:5104)    same, resident pools        ``nsm_sparse_mlp_decode`` /
                                                                    ``nsm_union_decode``
  OOM policy (:5493-5524)               ``OomPolicy``
``_sparse_mlp_forward_fast_triton``     same keyword signature,     ``nsm_decode_gathered`` /
  (:5526-5685)                          ``None`` when unsupported   ``nsm_decode_gathered_rows``
``_mlp_forward_dispatch`` (:5833-5923)  same                        (host policy)
  static skip mask (:5839-5844)         ``DecodeMlpPolicy.skip``
  SMC output reuse (:5847-5860,         ``DecodeMlpPolicy.reuse`` /
  :5918-5921)                           ``DecodeMlpPolicy.remember``
=====================================  ==========================  =====================================

``B200SparseMlpMixin`` goes in front of the runtime class
(``class Runtime(B200SparseMlpMixin, StreamingLlamaRuntime)``); everything it
does not handle falls through to ``super()``.  ``DecodeMlpPolicy`` and
``OomPolicy`` are runtime-free: the skip mask, the reuse cache and the
k-halving retry for code that drives the kernels without the reference runtime.

Deliberate differences from the reference:

* a missing or unloadable ``libnsm.so`` raises instead of returning ``None``
  (the reference falls back to its dequant path when Triton is absent,
  :5553-5557); the B200 path has no silent fallback.
* the single-token gathered kernel runs on sm_100, where the reference runs its
  single kernel only on sm_75 (:5579-5589).
* a kernel error other than an out-of-memory raises; the reference prints it,
  disables its fused path and returns ``None`` (:5680-5685).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from . import _lib
from .mlp import decode_gathered, decode_gathered_rows, route_sparse_mlp, sparse_mlp_decode, union_decode
from .weights import RouterWeights, SparseMlpWeights

UNION_MAX_ROWS = 32  # rows per nsm_union_decode call


def is_cuda_oom_error(exc: BaseException) -> bool:
    """True for an allocation failure: torch's ``OutOfMemoryError``, a library
    status ``NSM_ERR_CUDA`` whose CUDA error is ``cudaErrorMemoryAllocation``,
    or any error whose text carries one of the markers the reference matches
    (``llama3_neuroplastic/experiments/runtime/_helpers.py:301-308``)."""
    if isinstance(exc, torch.cuda.OutOfMemoryError):
        return True
    if isinstance(exc, _lib.NsmError) and exc.status == _lib.NSM_ERR_CUDA and "cudaErrorMemoryAllocation" in exc.detail:
        return True
    text = str(exc).lower()
    return any(m in text for m in ("out of memory", "cudaerrormemoryallocation", "cublas_status_alloc_failed",
                                   "hip error out of memory"))


@dataclass
class OomPolicy:
    """The reference's answer to an allocation failure in the sparse MLP
    (``streaming_llama_runtime.py:5493-5524``): free the caching allocator's
    blocks, retry with the first half of each row's blocks while fewer than
    ``max_retries`` retries were made and more than one block is left, and
    give a zero MLP contribution after that.  ``on_clamp(k)`` is told each new
    k (the runtime lowers its ``_sparse_runtime_top_k`` there)."""

    max_retries: int = 2
    log: Callable[[str], None] = field(default=lambda msg: print(msg, flush=True))

    def run(self, fn: Callable[[torch.Tensor], torch.Tensor], hidden: torch.Tensor, active_blocks: torch.Tensor, *,
            on_clamp: Callable[[int], None] | None = None, depth: int = 0) -> torch.Tensor:
        try:
            return fn(active_blocks)
        except Exception as exc:  # noqa: BLE001 -- re-raised unless it is an allocation failure
            if not is_cuda_oom_error(exc):
                raise
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        k = int(active_blocks.shape[-1]) if active_blocks.ndim > 0 else 1
        if depth < self.max_retries and k > 1:
            new_k = max(1, k // 2)
            if on_clamp is not None:
                on_clamp(new_k)
            self.log(f"[sparse] CUDA OOM in sparse MLP fallback; retrying with top_k={new_k}.")
            return self.run(fn, hidden, active_blocks[..., :new_k].contiguous(), on_clamp=on_clamp, depth=depth + 1)
        self.log("[sparse] CUDA OOM in sparse MLP fallback at minimum retry budget; "
                 "using zero MLP contribution for this layer.")
        return torch.zeros_like(hidden)


class DecodeMlpPolicy:
    """Per-layer decode policy in front of the MLP kernels
    (``streaming_llama_runtime.py:5833-5860``, ``:5918-5921``).

    ``skip_mask``: bool ``[num_layers]``; a set layer's MLP output is zero.
    ``smc_threshold``: with ``enable_smc``, a layer whose input moved less
    than this relative L2 distance since the last computed call of that layer
    reuses that call's output.  The cache holds one ``[H]`` input and output
    per layer in ``dtype`` on ``device``.
    """

    def __init__(self, num_layers: int, hidden: int, *, device, dtype=torch.bfloat16,
                 skip_mask: torch.Tensor | None = None, enable_smc: bool = False, smc_threshold: float = 0.04):
        self.skip_mask = None if skip_mask is None else skip_mask.to(torch.bool).cpu()
        self.skip_set = set() if self.skip_mask is None else {int(i) for i in self.skip_mask.nonzero().reshape(-1)}
        self.enable_smc = bool(enable_smc)
        self.smc_threshold = float(smc_threshold)
        self.smc_x_in = torch.zeros(num_layers, hidden, device=device, dtype=dtype)
        self.smc_out = torch.zeros(num_layers, hidden, device=device, dtype=dtype)
        self.smc_valid = torch.zeros(num_layers, dtype=torch.bool, device=device)

    def skip(self, layer_idx: int) -> bool:
        m = self.skip_mask
        return m is not None and int(layer_idx) < int(m.shape[0]) and bool(m[int(layer_idx)])

    def reuse(self, layer_idx: int, x: torch.Tensor) -> torch.Tensor | None:
        """The cached output when the input is within the threshold (one host
        read of the relative distance, as the reference does), else ``None``."""
        li = int(layer_idx)
        if not self.enable_smc or li in self.skip_set or not bool(self.smc_valid[li].item()):
            return None
        ref = self.smc_x_in[li]
        delta = (x.reshape(-1) - ref).norm()
        if (delta / ref.norm().clamp(min=1e-6)).item() < self.smc_threshold:
            return self.smc_out[li].view_as(x)
        return None

    def remember(self, layer_idx: int, x: torch.Tensor, y: torch.Tensor) -> None:
        if not self.enable_smc:
            return
        li = int(layer_idx)
        self.smc_x_in[li].copy_(x.reshape(-1), non_blocking=True)
        self.smc_out[li].copy_(y.reshape(-1), non_blocking=True)
        self.smc_valid[li] = True

    def forward(self, layer_idx: int, x: torch.Tensor, compute: Callable[[torch.Tensor], torch.Tensor]) -> torch.Tensor:
        """Skip, reuse, or ``compute(x)`` and remember the result."""
        if self.skip(layer_idx):
            return torch.zeros_like(x)
        hit = self.reuse(layer_idx, x)
        if hit is not None:
            return hit
        y = compute(x)
        self.remember(layer_idx, x, y)
        return y


def runtime_top_k(runtime: Any, routing: dict) -> int:
    """k of ``_route_sparse_mlp`` before clamping to the block count
    (``streaming_llama_runtime.py:4338-4350``): the layer's ``top_k``, else the
    runtime's ``_sparse_runtime_top_k`` when positive, else ``_sparse_top_k``;
    the sparse-prefill override in the prefill phase."""
    rt_k = int(getattr(runtime, "_sparse_runtime_top_k", 0) or 0)
    k = int(routing.get("top_k", rt_k if rt_k > 0 else int(getattr(runtime, "_sparse_top_k", 1))))
    if (str(getattr(runtime, "_traffic_current_phase", None) or "idle") == "prefill"
            and str(getattr(runtime, "_sparse_mlp_prefill_mode", "dense")) == "sparse"
            and getattr(runtime, "_sparse_mlp_prefill_top_k", None) is not None):
        k = int(runtime._sparse_mlp_prefill_top_k)
    return k


class B200SparseMlpMixin:
    """Mixed in front of ``StreamingLlamaRuntime``.

    Resident layers: ``nsm_attach(mlp={layer: SparseMlpWeights})`` (tiled NF4
    pools, e.g. ``Nf4Checkpoint.layer_weights``) makes ``_sparse_mlp_forward_fast``
    run that layer from the pools; other layers take the runtime's own
    streaming path, whose gathered buffers reach ``_sparse_mlp_forward_fast_triton``
    below.  Routers are built from ``self._sparse_routing`` on first use.
    """

    # ---- state
    def nsm_attach(self, *, mlp: dict[int, SparseMlpWeights] | None = None,
                   routers: dict[int, RouterWeights] | None = None) -> None:
        _lib.load()  # fail here, not at the first token, when the library is missing
        self.__dict__.setdefault("_nsm_mlp", {}).update(mlp or {})
        cache = self.__dict__.setdefault("_nsm_routers", {})
        for li, rw in (routers or {}).items():
            cache[int(li)] = (None, rw)

    def _nsm_router(self, layer_idx: int, routing: dict) -> RouterWeights:
        cache = self.__dict__.setdefault("_nsm_routers", {})
        hit = cache.get(int(layer_idx))
        if hit is not None and (hit[0] is None or hit[0] is routing):
            return hit[1]
        rw = RouterWeights.from_routing(routing, layer_idx=int(layer_idx),
                                        basis_top_k_by_layer=getattr(self, "_sparse_basis_top_k_by_layer", None),
                                        device=self.device)
        cache[int(layer_idx)] = (routing, rw)
        return rw

    def _nsm_oom_policy(self) -> OomPolicy:
        pol = self.__dict__.get("_nsm_oom")
        if pol is None:
            pol = self.__dict__["_nsm_oom"] = OomPolicy()
        return pol

    def _nsm_clamp_top_k(self, new_k: int) -> None:
        """The runtime-wide clamp of ``:5501-5507``."""
        if int(self._sparse_runtime_top_k) <= 0 or new_k < int(self._sparse_runtime_top_k):
            self._sparse_runtime_top_k = int(new_k)
            print(f"[sparse] runtime top_k clamped to {int(self._sparse_runtime_top_k)} after CUDA OOM.", flush=True)

    # ---- router
    def _route_sparse_mlp(self, hidden: torch.Tensor, layer_idx: int) -> torch.Tensor | None:
        """Active block ids ``[rows, k]`` (int64, score-descending, ties to the
        lower id) or ``None`` when the layer has no routing."""
        routing = self._sparse_routing.get(layer_idx)
        if routing is None:
            return None
        rw = self._nsm_router(layer_idx, routing)
        k = max(1, min(runtime_top_k(self, routing), rw.num_blocks))
        return route_sparse_mlp(hidden.reshape(-1, hidden.shape[-1]), rw, top_k=k)

    # ---- resident decode
    def _nsm_resident_forward(self, w: SparseMlpWeights, hidden: torch.Tensor,
                              active_blocks: torch.Tensor) -> torch.Tensor:
        flat = hidden.reshape(-1, hidden.shape[-1])
        rows = int(flat.shape[0])
        idx = active_blocks.reshape(rows, -1)
        if rows == 1:
            y = sparse_mlp_decode(flat[0], None, w, idx=idx[0], out_dtype=hidden.dtype)
            return y.view_as(hidden)
        outs = [union_decode(flat[r:r + UNION_MAX_ROWS], idx[r:r + UNION_MAX_ROWS], w, out_dtype=hidden.dtype)
                for r in range(0, rows, UNION_MAX_ROWS)]
        return torch.cat(outs, 0).view_as(hidden)

    def _sparse_mlp_forward_fast(self, layer_idx: int, mlp, hidden: torch.Tensor, active_blocks: torch.Tensor,
                                 _oom_retry_depth: int = 0) -> torch.Tensor:
        w = self.__dict__.get("_nsm_mlp", {}).get(int(layer_idx))
        if w is None:
            return super()._sparse_mlp_forward_fast(layer_idx, mlp, hidden, active_blocks,
                                                    _oom_retry_depth=_oom_retry_depth)
        routing = self._sparse_routing.get(int(layer_idx))
        if isinstance(routing, dict) and str(routing.get("block_domain", "intermediate")) != "intermediate":
            raise RuntimeError(f"Layer {int(layer_idx)} does not provide intermediate FFN routing data required for "
                               "exact_blockwise_sparse execution.")
        self._decode_backend_name = "nsm_resident_sparse_decode_sm100"
        return self._nsm_oom_policy().run(lambda ab: self._nsm_resident_forward(w, hidden, ab), hidden,
                                          active_blocks, on_clamp=self._nsm_clamp_top_k, depth=int(_oom_retry_depth))

    # ---- gathered decode (the runtime's streaming path)
    def _nsm_log_once(self, msg: str) -> None:
        if not self._triton_sparse_mlp_path_logged:
            print(msg, flush=True)
            self._triton_sparse_mlp_path_logged = True

    def _sparse_mlp_forward_fast_triton(
        self,
        *,
        hidden: torch.Tensor,
        flat_hidden: torch.Tensor,
        ordered_blocks: torch.Tensor,
        active_local: torch.Tensor,
        flat_mask: torch.Tensor,
        active_neurons: torch.Tensor,
        gate_bias: torch.Tensor | None,
        up_bias: torch.Tensor | None,
        down_bias: torch.Tensor | None,
        gate_param: dict[str, Any],
        up_param: dict[str, Any],
        down_param: dict[str, Any],
        gate_packed_gpu: torch.Tensor,
        gate_absmax_gpu: torch.Tensor,
        up_packed_gpu: torch.Tensor,
        up_absmax_gpu: torch.Tensor,
        down_packed_gpu: torch.Tensor | None,
        down_absmax_gpu: torch.Tensor | None,
    ) -> torch.Tensor | None:
        """MLP output over the runtime's gathered blocks (gate/up
        ``[U, 32, H/2]`` + absmax ``[U, 32, H/64]``, down ``[H, U, 16]`` +
        absmax ``[H, U]``; ``U = ordered_blocks.numel()``), shaped like
        ``hidden``; ``None`` when the runtime disabled this path or the down
        buffers are missing, as in ``streaming_llama_runtime.py:5547-5563``."""
        self._decode_backend_name = "dequant_sparse_fallback"
        if not self._triton_fused_sparse_mlp:
            self._nsm_log_once("[sparse] Triton sparse MLP disabled by runtime flag; using fallback path.")
            return None
        _lib.load()
        if down_packed_gpu is None or down_absmax_gpu is None:
            self._nsm_log_once("[sparse] Triton sparse MLP missing down buffers; using fallback path.")
            return None
        if int(self._sparse_block_size) != 32:
            raise RuntimeError("the B200 sparse MLP requires block_size=32")
        for p in (gate_param, up_param):
            if int(p["quant_block_size"]) != 64:
                raise RuntimeError("the B200 sparse MLP requires quant_block_size=64")

        def code(p):
            c = p.get("code_gpu")
            return c if c is not None else p["code"].to(device=self.device, dtype=torch.float32)

        H = int(flat_hidden.shape[-1])
        rows = int(flat_hidden.shape[0])
        U = int(ordered_blocks.numel())
        if U <= 0:
            return torch.zeros_like(hidden)
        bufs = dict(gate_packed=gate_packed_gpu, gate_absmax=gate_absmax_gpu, gate_code=code(gate_param),
                    up_packed=up_packed_gpu, up_absmax=up_absmax_gpu, up_code=code(up_param),
                    down_packed=down_packed_gpu, down_absmax=down_absmax_gpu, down_code=code(down_param))
        # biases in the gathered neuron order (the reference indexes them the same way, :5646-5654)
        an = active_neurons.to(torch.long)
        gb = gate_bias[an].to(device=self.device, dtype=torch.float32) if gate_bias is not None else None
        ub = up_bias[an].to(device=self.device, dtype=torch.float32) if up_bias is not None else None
        db = down_bias.to(device=self.device, dtype=torch.float32) if down_bias is not None else None
        single = rows == 1 and int(active_local.numel()) > 0 and bool((active_local >= 0).all().item())
        if single and self._single_kernel_decode_enabled:
            y = decode_gathered(flat_hidden.reshape(-1), hidden_size=H, out_dtype=torch.float32, gate_bias=gb,
                                up_bias=ub, down_bias=db, **bufs)
            self._decode_backend_name = "nsm_single_kernel_sparse_decode_sm100"
            self._nsm_log_once("[sparse] B200 sparse MLP path active: single kernel sm100.")
        else:
            y = decode_gathered_rows(flat_hidden, flat_mask, out_dtype=torch.float32, gate_bias=gb, up_bias=ub,
                                     down_bias=db, **bufs)
            self._decode_backend_name = "nsm_gathered_rows_sparse_decode_sm100"
            self._nsm_log_once("[sparse] B200 sparse MLP path active: gathered rows sm100.")
        return y.view_as(hidden).to(dtype=hidden.dtype)

    # ---- dispatch
    def _mlp_forward_dispatch(self, layer_idx: int, layer, mlp_input: torch.Tensor) -> torch.Tensor:
        """Decode of a resident layer: skip mask, SMC reuse, route, resident MLP,
        SMC store (``:5839-5860``, ``:5907-5921``).  Everything else is the
        runtime's own dispatch."""
        li = int(layer_idx)
        phase = str(self._traffic_current_phase or "idle")
        resident = li in self.__dict__.get("_nsm_mlp", {})
        if phase != "decode" or not resident or li not in self._sparse_routing:
            return super()._mlp_forward_dispatch(layer_idx, layer, mlp_input)
        m = self._mlp_static_skip_mask
        if m is not None and li < int(m.shape[0]) and bool(m[li].item()):
            return torch.zeros_like(mlp_input)
        smc = bool(getattr(self, "_enable_smc", False))
        if smc and bool(self._smc_valid[li].item()) and li not in self._mlp_static_skip_set:
            ref = self._smc_x_in[li]
            delta = (mlp_input.view(-1) - ref).norm()
            if (delta / ref.norm().clamp(min=1e-6)).item() < self._smc_threshold:
                return self._smc_out[li].view_as(mlp_input)
        self._mlp_prefetch_active_blocks.pop(li, None)
        active_blocks = self._route_sparse_mlp(mlp_input, layer_idx)
        if active_blocks is None:
            raise RuntimeError(f"Sparse basis routing disappeared for layer {li}")
        self._decode_prefetch_route_cache[li] = active_blocks
        self._record_hot_cache_calibration_blocks(layer_idx, active_blocks)
        out = self._sparse_mlp_forward_fast(layer_idx, layer.mlp, mlp_input, active_blocks)
        if smc:
            self._smc_x_in[li].copy_(mlp_input.view(-1), non_blocking=True)
            self._smc_out[li].copy_(out.view(-1), non_blocking=True)
            self._smc_valid[li] = True
        return out


__all__ = ["B200SparseMlpMixin", "DecodeMlpPolicy", "OomPolicy", "is_cuda_oom_error", "runtime_top_k"]
