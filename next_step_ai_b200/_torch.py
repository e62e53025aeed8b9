"""Small torch <-> C-ABI helpers: dtype codes, raw pointers, streams, workspaces."""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

_DT = {torch.float32: _lib.NSM_F32, torch.float16: _lib.NSM_F16, torch.bfloat16: _lib.NSM_BF16}


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError as exc:
        raise RuntimeError(f"unsupported dtype {t}; expected float32, float16 or bfloat16") from exc


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError("expected a contiguous tensor")
    return t.data_ptr()


def row_ptr(t: torch.Tensor | None) -> int | None:
    """Base pointer of a pool tensor whose rows may be strided (a view into a
    larger record per row); each row itself must be contiguous."""
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("expected a CUDA tensor")
    if t.dim() == 0 or not t[0].is_contiguous():
        raise RuntimeError("expected contiguous pool rows")
    return t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} must be a CUDA tensor (the B200 path has no CPU fallback)")


class WorkspacePool:
    """Zero-initialised decode workspaces, cached per (device, stream, size class).

    Calls that share a workspace must not overlap on the GPU; keying by
    stream makes calls on different streams use different workspaces.
    """

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._ws: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        dev = device.index if device.index is not None else torch.cuda.current_device()
        key = (dev, stream_handle(device))
        with self._lock:
            buf = self._ws.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(int(nbytes), 1 << 20)
                buf = torch.empty(size, dtype=torch.uint8, device=torch.device("cuda", dev))
                _lib.check(_lib.load().nsm_workspace_init(buf.data_ptr(), buf.numel(), key[1]), "nsm_workspace_init")
                self._ws[key] = buf
            return buf

    def errors(self) -> dict[tuple[int, int], int]:
        """Read and clear the device error word of every cached workspace
        (non-zero: a kernel gave up on a bounded wait).  Synchronises."""
        out = {}
        with self._lock:
            for key, buf in self._ws.items():
                code = ctypes.c_int32(0)
                with torch.cuda.device(key[0]):
                    _lib.check(_lib.load().nsm_workspace_error(buf.data_ptr(), buf.numel(), ctypes.byref(code), key[1]),
                               "nsm_workspace_error")
                out[key] = int(code.value)
        return out

    def clear(self) -> None:
        with self._lock:
            self._ws.clear()


WORKSPACES = WorkspacePool()
