"""Multi-layer decode of the blockwise-sparse MLP stack (one token per step).

This is the B200 counterpart of the reference's per-token layer loop
(``streaming_llama_runtime.py:7612-7775``) restricted to the MLP path: for
every decoder layer the residual is updated with the previous layer's MLP
output, RMS-normalised, routed, and pushed through the sparse NF4 MLP.
Attention is out of scope (identity), as in the benchmark configuration.

Two execution paths compute the same thing:

* the token kernel (``nsm_decode_token``, the default when every layer
  qualifies): ONE persistent cooperative kernel runs the whole token, the
  phases of each layer linked by bounded waits inside the kernel;
* the per-layer path (``nsm_sparse_mlp_decode`` per layer, five kernels each
  with programmatic dependent launch), for layers the token kernel does not
  take (another router rank or dtype, row-major pools, biases, ...).

Multi-GPU: every rank holds a contiguous range of each layer's intermediate
blocks and a full copy of the router; all ranks select the same blocks, each
computes the partial output of the blocks it owns, and the partials are summed
over NVLink in rank order inside the next layer's first phase (CUDA-IPC
exchange buffers).  The whole token is captured once into a CUDA graph and
replayed.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._torch import WORKSPACES, dtype_code, ptr, stream_handle
from .weights import RouterWeights, SparseMlpWeights


@dataclass
class DecodeLayer:
    router: RouterWeights
    weights: SparseMlpWeights
    norm_weight: torch.Tensor | None = None


def shard_range(num_blocks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block range [lo, hi) of ``rank`` when ``num_blocks``
    intermediate blocks are split over ``world`` GPUs (sizes differ by at most
    one block).  Every rank routes all blocks (the router is replicated) and
    computes the MLP over the selected blocks inside its range; the partial
    outputs are summed across ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    return (num_blocks * rank) // world, (num_blocks * (rank + 1)) // world


class SparseMlpDecoder:
    """Runs ``num_layers`` decode steps over ``layers`` (cycled when fewer
    unique layers than ``num_layers`` are resident).

    A layer's output stays in the workspace as down-projection partials
    (``NSM_IO_DEFER_Y``); the next layer's router kernel sums them, adds them
    to the fp32 residual and applies the RMSNorm (``NSM_IO_PENDING_Y``), so
    there is no separate output kernel between layers.  With ``group`` (one
    process per GPU) the partials of all ranks are summed inside that same
    kernel over NVLink through an exchange buffer per rank (CUDA IPC), in rank
    order, instead of an NCCL all-reduce.

    ``block_range``: the intermediate blocks this rank's pools hold
    (``(0, NB)`` on one GPU).

    ``token_kernel=True`` runs the whole token as one persistent cooperative
    launch (``nsm_decode_token``) instead of five graph-captured kernels per
    layer; it measures slower than the per-layer kernels at the 405B shape
    (108 against 65 us per layer on a B200), so the per-layer path is the
    default.
    """

    def __init__(self, layers: list[DecodeLayer], num_layers: int, *, block_range: tuple[int, int] | None = None,
                 group=None, eps: float = 1e-5, token_kernel: bool = False):
        if not layers:
            raise RuntimeError("no layers")
        self.layers = layers
        self.num_layers = int(num_layers)
        w0 = layers[0].weights
        self.H, self.I = w0.hidden, w0.intermediate
        self.dev = w0.gate_packed.device
        self.block_range = block_range if block_range is not None else (0, self.I // 32)
        self.group = group
        self.eps = float(eps)
        self.residual = torch.zeros(self.H, dtype=torch.float32, device=self.dev)
        self.out = torch.zeros(self.H, dtype=torch.float32, device=self.dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self._lib = _lib.load()
        k = max(l.router.top_k for l in layers)
        rank = max(l.router.rank for l in layers)
        self._ws_bytes = self._lib.nsm_decode_workspace_bytes(self.H, self.I, k, rank)
        self._c = [(l.router.to_c(), l.weights.to_c()) for l in layers]
        self._bm = _lib.BlockMapC()
        self._bm.block_begin, self._bm.block_end = int(self.block_range[0]), int(self.block_range[1])
        self._ex = None
        if group is not None and torch.distributed.get_world_size(group) > 1:
            self._ex = self._connect_exchange(group)
        ok = self.token_kernel_applies()
        if token_kernel and not ok:
            raise RuntimeError("the token kernel does not apply to these layers (see token_kernel_applies)")
        self.use_token = bool(token_kernel)
        self._tk_ws = None
        if self.use_token:
            self._setup_token()

    # ---- the token kernel
    def token_kernel_applies(self) -> bool:
        """Whether nsm_decode_token takes every layer: router rank 64 in bf16 or
        fp16, k <= 256, at most 4096 blocks, hidden a multiple of 128 and at
        most 16384, tiled pools without biases, a down codebook equal to the
        gate or up codebook."""
        if self.H % 128 or self.H > 16384 or self.I // 32 > 4096:
            return False
        for l in self.layers:
            r, w = l.router, l.weights
            if r.rank != 64 or r.enc_w.dtype not in (torch.bfloat16, torch.float16) or min(r.top_k, r.num_blocks) > 256:
                return False
            if r.num_blocks != self.I // 32:
                return False
            if (w.layout & 3) != 3 or any(getattr(w, b, None) is not None for b in ("gate_bias", "up_bias", "down_bias")):
                return False
            if not (torch.equal(w.down_code, w.gate_code) or torch.equal(w.down_code, w.up_code)):
                return False
        return True

    def _setup_token(self) -> None:
        L = self.num_layers
        nbytes = self._lib.nsm_token_workspace_bytes(self.H, self.I, L)
        self._tk_ws = torch.empty(nbytes, dtype=torch.uint8, device=self.dev)
        st = stream_handle(self.dev)
        _lib.check(self._lib.nsm_workspace_init(self._tk_ws.data_ptr(), nbytes, st), "nsm_workspace_init")
        arr = (_lib.TokenLayerC * L)()
        for i in range(L):
            li = i % len(self.layers)
            rc, wc = self._c[li]
            arr[i].router = rc
            arr[i].mlp = wc
            arr[i].map = self._bm
            nw = self.layers[li].norm_weight
            arr[i].norm_weight = ptr(nw) if nw is not None else None
            arr[i].norm_weight_dtype = dtype_code(nw.dtype) if nw is not None else 0
        _lib.check(self._lib.nsm_token_set_layers(self._tk_ws.data_ptr(), nbytes, self.H, self.I, ctypes.byref(arr), L,
                                                  st), "nsm_token_set_layers")

    def _token(self, st: int, trace=None) -> None:
        tb, tk, tc, tr = (None, 0, None, None) if trace is None else trace
        _lib.check(self._lib.nsm_decode_token(self.residual.data_ptr(), self.H, self.I, self.num_layers, self.eps,
                                              self._ex, tb, tk, tc, tr, self._tk_ws.data_ptr(), self._tk_ws.numel(),
                                              st), "nsm_decode_token")

    def token_error(self) -> int:
        """Reads and clears the token workspace's device error word (0: every
        bounded wait of the token kernel completed).  Synchronises."""
        if self._tk_ws is None:
            return 0
        code = ctypes.c_int32(0)
        _lib.check(self._lib.nsm_workspace_error(self._tk_ws.data_ptr(), self._tk_ws.numel(), ctypes.byref(code),
                                                 stream_handle(self.dev)), "nsm_workspace_error")
        return int(code.value)

    def token_profile(self, stamps: torch.Tensor | None) -> None:
        """Switches the token kernel's phase timestamps on (``stamps``: int64
        ``[layers][SMs][8]`` on the device) or off (None)."""
        n = int(stamps.shape[0]) if stamps is not None else 0
        _lib.check(self._lib.nsm_token_profile(self._tk_ws.data_ptr(), self._tk_ws.numel(), self.H, self.I,
                                               self.num_layers, stamps.data_ptr() if stamps is not None else None, n,
                                               stream_handle(self.dev)), "nsm_token_profile")

    def _connect_exchange(self, group) -> ctypes.c_void_p:
        world = torch.distributed.get_world_size(group)
        rank = torch.distributed.get_rank(group)
        ex = ctypes.c_void_p()
        handle = (ctypes.c_char * _lib.NSM_IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.dev):
            _lib.check(self._lib.nsm_exchange_create(world, rank, self.H, ctypes.byref(ex), handle),
                       "nsm_exchange_create")
        handles = [None] * world
        torch.distributed.all_gather_object(handles, bytes(handle), group=group)
        blob = b"".join(handles)
        with torch.cuda.device(self.dev):
            _lib.check(self._lib.nsm_exchange_connect(ex, blob), "nsm_exchange_connect")
        torch.distributed.barrier(group=group)
        return ex

    def _io(self, flags: int, events=None, norm_weight=None) -> _lib.LayerIoC:
        io = _lib.LayerIoC()
        io.residual = self.residual.data_ptr()
        io.norm_weight = ptr(norm_weight) if norm_weight is not None else None
        io.norm_weight_dtype = dtype_code(norm_weight.dtype) if norm_weight is not None else 0
        io.eps = self.eps
        io.flags = flags
        io.exchange = self._ex
        io.stage_events = ctypes.cast(events, ctypes.c_void_p) if events is not None else None
        return io

    def _layer(self, i: int, ws: torch.Tensor, st: int, events=None) -> None:
        li = i % len(self.layers)
        layer = self.layers[li]
        rc, wc = self._c[li]
        flags = _lib.NSM_IO_DEFER_Y | (_lib.NSM_IO_PENDING_Y if i > 0 else 0)
        io = self._io(flags, events, layer.norm_weight)
        _lib.check(self._lib.nsm_sparse_mlp_decode(
            None, 0, self.H, self.I, ctypes.byref(io), ctypes.byref(rc), None, 0, ctypes.byref(self._bm),
            ctypes.byref(wc), None, 0, None, None, ws.data_ptr(), ws.numel(), st), "nsm_sparse_mlp_decode")

    def _flush(self, ws: torch.Tensor, st: int) -> None:
        io = self._io(_lib.NSM_IO_PENDING_Y)
        _lib.check(self._lib.nsm_residual_flush(self.H, ctypes.byref(io), ws.data_ptr(), ws.numel(), st),
                   "nsm_residual_flush")

    # kernels per layer: router latent (+ previous layer's output), block scores,
    # top-k, gate/up, gate/up reduction, down; plus one output kernel per token.
    # With the bulk-copy gate/up kernel (tiled pools, H <= 16384, H / 64 even,
    # k <= 1024) the gate/up kernel selects the blocks itself: no top-k kernel.
    KERNELS_PER_LAYER = 6

    def _kernels_for(self, li: int) -> int:
        layer = self.layers[li]
        k = min(layer.router.top_k, layer.router.num_blocks)
        fused = (bool(layer.weights.layout & _lib.NSM_LAYOUT_GATEUP_TILED) and self.H <= 16384
                 and (self.H // 64) % 2 == 0 and k <= 1024)
        return self.KERNELS_PER_LAYER - (1 if fused else 0)

    @property
    def kernels_per_step(self) -> int:
        """This library's kernel launches per token (the final copy to ``out``
        is not counted)."""
        if self.use_token:
            return 1
        return sum(self._kernels_for(i % len(self.layers)) for i in range(self.num_layers)) + 1

    def step_eager(self) -> None:
        """One token through all layers (no graph).  Input: ``residual``;
        output: ``out`` = final residual (residual + every layer's MLP output)."""
        st = stream_handle(self.dev)
        if self.use_token:
            self._token(st)
        else:
            ws = WORKSPACES.get(self._ws_bytes, self.dev)
            for i in range(self.num_layers):
                self._layer(i, ws, st)
            self._flush(ws, st)
        self.out.copy_(self.residual)

    def trace_layers(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """One eager token like :meth:`step_eager`, synchronising after every
        layer to record what that layer saw and chose: ``(residual, blocks)``
        per layer, where ``residual`` is the fp32 residual the layer's
        RMSNorm read (the previous layers' outputs already added) and
        ``blocks`` the selected blocks present in this rank's pool, ascending
        -- the selection the gate/up kernel makes itself on this path.  The
        launches are exactly those of :meth:`step_eager`; the records are
        copies taken between layers (the token kernel writes them itself while
        it runs).  ``out`` holds the final residual."""
        st = stream_handle(self.dev)
        if self.use_token:
            L = self.num_layers
            k_max = max(min(l.router.top_k, l.router.num_blocks) for l in self.layers)
            tb = torch.full((L, k_max), -1, dtype=torch.int32, device=self.dev)
            tc = torch.zeros(L, dtype=torch.int32, device=self.dev)
            tr = torch.empty((L, self.H), dtype=torch.float32, device=self.dev)
            self._token(st, (tb.data_ptr(), k_max, tc.data_ptr(), tr.data_ptr()))
            self.out.copy_(self.residual)
            torch.cuda.current_stream(self.dev).synchronize()
            counts = tc.cpu().tolist()
            return [(tr[i].clone(), tb[i, :counts[i]].clone()) for i in range(L)]
        ws = WORKSPACES.get(self._ws_bytes, self.dev)
        k_max = max(min(l.router.top_k, l.router.num_blocks) for l in self.layers)
        blocks = torch.empty(k_max, dtype=torch.int32, device=self.dev)
        count = torch.empty(1, dtype=torch.int32, device=self.dev)
        trace = []
        for i in range(self.num_layers):
            self._layer(i, ws, st)
            r = self.layers[i % len(self.layers)].router
            k = min(r.top_k, r.num_blocks)
            _lib.check(self._lib.nsm_workspace_selection(ws.data_ptr(), ws.numel(), self.H, self.I, k, r.rank,
                                                         blocks.data_ptr(), count.data_ptr(), st),
                       "nsm_workspace_selection")
            torch.cuda.current_stream(self.dev).synchronize()
            n = int(count.item())
            trace.append((self.residual.clone(), blocks[:n].clone()))
        self._flush(ws, st)
        self.out.copy_(self.residual)
        torch.cuda.current_stream(self.dev).synchronize()
        return trace

    STAGES = ("router", "gateup", "gateup_finalize", "down", "down_finalize")

    def time_stages(self, num_layers: int | None = None) -> dict[str, float]:
        """One eager pass over ``num_layers`` layers with the library's stage
        events recorded around each stage; returns the mean device time of
        each stage in microseconds.  The events separate the kernels (no
        programmatic dependent launch across stages), so the sum is larger
        than a graph replay's layer time.  "router" includes summing the
        previous layer's output (and the cross-GPU exchange); "down_finalize"
        is empty because each layer's output stays pending for the next.  The
        pass advances ``residual``."""
        if self.use_token:
            raise RuntimeError("time_stages times the per-layer path; the token kernel runs a token in one launch")
        n = int(num_layers or self.num_layers)
        ws = WORKSPACES.get(self._ws_bytes, self.dev)
        st = stream_handle(self.dev)
        evs, arrs = [], []
        for _ in range(n):
            row = [torch.cuda.Event(enable_timing=True) for _ in range(_lib.NSM_STAGE_EVENTS)]
            for e in row:
                e.record()  # creates the event
            evs.append(row)
            arrs.append((ctypes.c_void_p * _lib.NSM_STAGE_EVENTS)(*[e.cuda_event for e in row]))
        torch.cuda.synchronize(self.dev)
        for i in range(n):
            self._layer(i, ws, st, events=arrs[i])
        self._flush(ws, st)
        torch.cuda.synchronize(self.dev)
        out = {}
        for j, name in enumerate(self.STAGES):
            out[name] = 1e3 * sum(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(n)) / n
        return out

    def capture(self) -> torch.cuda.CUDAGraph:
        """Capture one token into a CUDA graph (after one eager warm-up)."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            saved = self.residual.clone()
            self.step_eager()  # warm-up: workspace for this stream, kernel attributes, NCCL comms
            self.residual.copy_(saved)
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.step_eager()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        self.graph = g
        return g

    def replay(self) -> None:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()

    def release(self) -> None:
        """Drops the captured graph (the exchange buffers stay until close())."""
        self.graph = None

    def close(self) -> None:
        self.graph = None
        if self._ex is not None:
            torch.cuda.synchronize(self.dev)
            self._lib.nsm_exchange_destroy(self._ex)
            self._ex = None
