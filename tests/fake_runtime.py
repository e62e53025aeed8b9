"""A stand-in for the reference runtime's state: the attributes and the
super-methods of ``StreamingLlamaRuntime`` that ``B200SparseMlpMixin``
touches (``streaming_llama_runtime.py:748-756``, ``:4311``, ``:5104``,
``:5833``).  Test infrastructure only."""
from __future__ import annotations

import torch

from next_step_ai_b200 import runtime_adapter as ra

H, NB, RANK = 64, 8, 4


def routing(**kw):
    g = torch.Generator().manual_seed(0)
    r = {"enc_w": torch.randn(RANK, H, generator=g), "enc_b": torch.zeros(RANK),
         "route_score_weight": torch.randn(NB, RANK, generator=g), "route_score_bias": torch.zeros(NB)}
    r.update(kw)
    return r


class FakeRuntime:
    """The attributes and super-methods of the reference runtime that the mixin touches."""

    def __init__(self, num_layers=4, hidden=H, device="cpu"):
        self.device = torch.device(device)
        self._sparse_routing = {0: routing(), 1: routing(top_k=3)}
        self._sparse_runtime_top_k = 0
        self._sparse_top_k = 6
        self._sparse_basis_top_k_by_layer = {}
        self._sparse_block_size = 32
        self._traffic_current_phase = "decode"
        self._sparse_mlp_prefill_mode = "dense"
        self._sparse_mlp_prefill_top_k = None
        self._triton_fused_sparse_mlp = True
        self._single_kernel_decode_enabled = True
        self._triton_sparse_mlp_path_logged = False
        self._decode_backend_name = ""
        self._mlp_static_skip_mask = None
        self._mlp_static_skip_set = set()
        self._enable_smc = False
        self._smc_threshold = 0.04
        self._smc_x_in = torch.zeros(num_layers, hidden, device=self.device)
        self._smc_out = torch.zeros(num_layers, hidden, device=self.device)
        self._smc_valid = torch.zeros(num_layers, dtype=torch.bool, device=self.device)
        self._mlp_prefetch_active_blocks = {}
        self._decode_prefetch_route_cache = {}
        self.calls = []

    def _record_hot_cache_calibration_blocks(self, layer_idx, active_blocks):
        self.calls.append(("calib", int(layer_idx)))

    def _sparse_mlp_forward_fast(self, layer_idx, mlp, hidden, active_blocks, _oom_retry_depth=0):
        self.calls.append(("super_fast", int(layer_idx)))
        return torch.full_like(hidden, -1.0)

    def _mlp_forward_dispatch(self, layer_idx, layer, mlp_input):
        self.calls.append(("super_dispatch", int(layer_idx)))
        return torch.full_like(mlp_input, -2.0)


class Runtime(ra.B200SparseMlpMixin, FakeRuntime):
    pass
