"""ctypes binding of ``libnsm.so`` (declarations in ``include/nsm.h``).

The library is loaded from the package directory (built in-tree by
``next_step_ai_b200.build``).  There is no fallback: if the library cannot
be loaded every kernel entry point raises.  Every call returns an int status;
:func:`check` turns a non-zero status into ``RuntimeError`` carrying the
library's own message, which is the error type the reference raises for bad
shapes, layouts and devices (``llama3_neuroplastic/triton_sparse_mlp.py:1122-1127``,
``:1397-1464``).
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnsm.so"

NSM_OK = 0
NSM_ERR_INVALID_ARG = -1
NSM_ERR_UNSUPPORTED = -2
NSM_ERR_CUDA = -3
NSM_ERR_TIMEOUT = -4
NSM_ERR_WORKSPACE = -5
NSM_ERR_DEVICE = -6

NSM_F32, NSM_F16, NSM_BF16 = 0, 1, 2
NSM_LAYOUT_GATEUP_TILED, NSM_LAYOUT_DOWN_TILED, NSM_LAYOUT_SHARED_CODE = 1, 2, 4
NSM_STAGE_EVENTS = 6
NSM_IO_PENDING_Y, NSM_IO_DEFER_Y = 1, 2
NSM_IPC_HANDLE_BYTES = 64
ABI_VERSION = 4

# every symbol include/nsm.h declares (checked by tests/test_abi.py)
EXPORTED = (
    "nsm_abi_version", "nsm_status_string", "nsm_last_error", "nsm_workspace_init",
    "nsm_decode_workspace_bytes", "nsm_route", "nsm_sparse_mlp_decode", "nsm_decode_gathered",
    "nsm_decode_rows_workspace_bytes", "nsm_decode_gathered_rows", "nsm_repack_down_block_major",
    "nsm_sparse_input_linear_4bit", "nsm_sparse_output_linear_4bit", "nsm_cache_split", "nsm_cache_promote",
    "nsm_repack_tiled", "nsm_decode_gathered_static", "nsm_workspace_error", "nsm_cache_stage",
    "nsm_union_workspace_bytes", "nsm_union_decode", "nsm_residual_flush", "nsm_exchange_bytes",
    "nsm_exchange_create", "nsm_exchange_connect", "nsm_exchange_destroy", "nsm_route_workspace_bytes",
    "nsm_lm_head_workspace_bytes", "nsm_lm_head_max_tokens", "nsm_lm_head_nf4",
    "nsm_route_rows", "nsm_workspace_selection", "nsm_exchange_connect_local", "nsm_exchange_set_spin_limit",
    "nsm_set_copy_wait_limit", "nsm_static_error", "nsm_token_workspace_bytes", "nsm_token_set_layers",
    "nsm_decode_token", "nsm_token_profile",
)


class RouterWeightsC(ctypes.Structure):
    _fields_ = [
        ("enc_w", c_void_p), ("enc_b", c_void_p), ("score_w", c_void_p), ("score_b", c_void_p),
        ("down_block_norm", c_void_p), ("weight_dtype", c_int32), ("rank", c_int32), ("num_blocks", c_int32),
        ("top_k", c_int32), ("basis_top_k", c_int32), ("legacy_abs_latent", c_int32),
    ]


class MlpWeightsC(ctypes.Structure):
    _fields_ = [
        ("gate_packed", c_void_p), ("gate_absmax", c_void_p), ("up_packed", c_void_p), ("up_absmax", c_void_p),
        ("down_packed", c_void_p), ("down_absmax", c_void_p), ("gate_code", c_void_p), ("up_code", c_void_p),
        ("down_code", c_void_p), ("gate_bias", c_void_p), ("up_bias", c_void_p), ("down_bias", c_void_p),
        ("bias_dtype", c_int32), ("pool_rows", c_int32),
        ("gateup_block_stride", c_int64), ("gateup_absmax_block_stride", c_int64),
        ("down_block_stride", c_int64), ("down_row_stride", c_int64),
        ("down_absmax_block_stride", c_int64), ("down_absmax_row_stride", c_int64),
        ("down_absmax_pair", c_int32), ("layout", c_int32),
    ]


class BlockMapC(ctypes.Structure):
    _fields_ = [("slot_of_block", c_void_p), ("block_begin", c_int32), ("block_end", c_int32)]


class TokenLayerC(ctypes.Structure):
    _fields_ = [("router", RouterWeightsC), ("mlp", MlpWeightsC), ("map", BlockMapC), ("norm_weight", c_void_p),
                ("norm_weight_dtype", c_int32), ("reserved", c_int32)]


class LayerIoC(ctypes.Structure):
    _fields_ = [
        ("residual", c_void_p), ("y_prev", c_void_p), ("y_prev_dtype", c_int32), ("norm_weight_dtype", c_int32),
        ("norm_weight", c_void_p), ("eps", c_float), ("flags", c_int32), ("reserved2", c_int32),
        ("exchange", c_void_p), ("stage_events", c_void_p),
    ]


_SIGS = {
    "nsm_abi_version": (c_int, []),
    "nsm_status_string": (c_char_p, [c_int]),
    "nsm_last_error": (c_char_p, []),
    "nsm_workspace_init": (c_int, [c_void_p, c_size_t, c_void_p]),
    "nsm_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "nsm_workspace_selection": (c_int, [c_void_p, c_size_t, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                                        c_void_p]),
    "nsm_route": (c_int, [c_void_p, c_int32, c_int32, POINTER(RouterWeightsC), c_void_p, c_void_p, c_void_p,
                          c_void_p, c_size_t, c_void_p]),
    "nsm_route_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "nsm_lm_head_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "nsm_lm_head_max_tokens": (c_int, [c_int32]),
    "nsm_lm_head_nf4": (c_int, [c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_size_t, c_void_p]),
    "nsm_route_rows": (c_int, [c_void_p, c_int32, c_int32, c_int32, POINTER(RouterWeightsC), c_void_p, c_void_p,
                               c_void_p, c_void_p, c_size_t, c_void_p]),
    "nsm_sparse_mlp_decode": (c_int, [c_void_p, c_int32, c_int32, c_int32, POINTER(LayerIoC),
                                      POINTER(RouterWeightsC), c_void_p, c_int32, POINTER(BlockMapC),
                                      POINTER(MlpWeightsC), c_void_p, c_int32, c_void_p, c_void_p, c_void_p,
                                      c_size_t, c_void_p]),
    "nsm_decode_gathered": (c_int, [c_void_p, c_int32, c_int32, c_int32, POINTER(MlpWeightsC), c_void_p, c_int32,
                                    c_void_p, c_void_p, c_size_t, c_void_p]),
    "nsm_workspace_error": (c_int, [c_void_p, c_size_t, POINTER(c_int32), c_void_p]),
    "nsm_decode_gathered_static": (c_int, [c_void_p, c_int32, c_int32, c_int32, POINTER(MlpWeightsC), c_void_p,
                                           c_int32, c_void_p, c_void_p]),
    "nsm_decode_rows_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "nsm_decode_gathered_rows": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int32,
                                         POINTER(MlpWeightsC), c_void_p, c_int32, c_void_p, c_size_t, c_void_p]),
    "nsm_repack_down_block_major": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p,
                                            c_void_p, c_void_p]),
    "nsm_sparse_input_linear_4bit": (c_int, [c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p,
                                             c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int32, c_void_p,
                                             c_void_p]),
    "nsm_sparse_output_linear_4bit": (c_int, [c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_int32,
                                              c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32,
                                              c_void_p, c_void_p]),
    "nsm_repack_tiled": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                 c_void_p, c_void_p, c_int32, POINTER(MlpWeightsC), c_void_p]),
    "nsm_cache_split": (c_int, [c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]),
    "nsm_residual_flush": (c_int, [c_int32, POINTER(LayerIoC), c_void_p, c_size_t, c_void_p]),
    "nsm_exchange_bytes": (c_size_t, [c_int, c_int]),
    "nsm_exchange_create": (c_int, [c_int32, c_int32, c_int32, POINTER(c_void_p), c_void_p]),
    "nsm_exchange_connect": (c_int, [c_void_p, c_void_p]),
    "nsm_exchange_destroy": (c_int, [c_void_p]),
    "nsm_exchange_connect_local": (c_int, [c_void_p, c_int32]),
    "nsm_exchange_set_spin_limit": (c_int, [c_void_p, c_int32]),
    "nsm_set_copy_wait_limit": (c_int, [c_int32]),
    "nsm_static_error": (c_int, [POINTER(c_int32), c_void_p]),
    "nsm_token_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "nsm_token_set_layers": (c_int, [c_void_p, c_size_t, c_int32, c_int32, c_void_p, c_int32, c_void_p]),
    "nsm_decode_token": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_float, c_void_p, c_void_p, c_int32, c_void_p,
                                 c_void_p, c_void_p, c_size_t, c_void_p]),
    "nsm_token_profile": (c_int, [c_void_p, c_size_t, c_int32, c_int32, c_int32, c_void_p, c_int32, c_void_p]),
    "nsm_union_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "nsm_union_decode": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int32,
                                 POINTER(BlockMapC), POINTER(MlpWeightsC), c_void_p, c_int32, c_void_p, c_void_p,
                                 c_void_p, c_size_t, c_void_p]),
    "nsm_cache_stage": (c_int, [c_void_p, c_int32, c_void_p, c_int32, c_size_t, c_void_p, c_void_p, c_int32,
                                c_void_p]),
    "nsm_cache_promote": (c_int, [POINTER(MlpWeightsC), c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_int32,
                                  c_void_p, c_void_p]),
}

_lock = threading.Lock()
_lib = None


def lib_path() -> Path:
    return LIB_PATH


def load(build_if_missing: bool = False):
    """Load (once) and return the ctypes handle of libnsm.so."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists() and build_if_missing:
            from .build import build
            build()
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m next_step_ai_b200.build` "
                               "(the CUDA path has no fallback)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().nsm_last_error()
    return msg.decode() if msg else ""


class NsmError(RuntimeError):
    """A non-zero status of a ``libnsm.so`` call: ``status`` (``NSM_ERR_*``)
    and ``detail`` (``nsm_last_error()`` of the failing call)."""

    def __init__(self, what: str, status: int, name: str, detail: str):
        super().__init__(f"{what} failed: {name} ({status}): {detail}")
        self.status = int(status)
        self.detail = detail


def check(status: int, what: str) -> None:
    if status != NSM_OK:
        lib = load()
        raise NsmError(what, status, lib.nsm_status_string(status).decode(), last_error())
