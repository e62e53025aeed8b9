"""nsm_decode_gathered_static: the gathered decode MLP with the library's
static scratch array instead of a caller workspace.

Each case runs two calls in a row with different inputs (the second call
finds the first one's scratch contents) and checks both against
nsm_decode_gathered with a fresh workspace and against the CPU oracle, with
the decode tests' tolerances (max-abs-err <= 2e-2, relative L2 <= 5e-3 for
fp32 output).  The file is named to be collected last, and it must also pass
on its own in a fresh process, where its first call does the static array's
set-up.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import mlp as om  # noqa: E402
from oracle import synthetic as syn  # noqa: E402

MAX_ABS = 2e-2
REL_L2 = 5e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from next_step_ai_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


def _close(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    err = float(np.abs(got - ref).max())
    assert rel <= REL_L2, f"relative L2 {rel:.3e} > {REL_L2}"
    assert err <= MAX_ABS, f"max abs err {err:.3e} > {MAX_ABS}"


def _descriptor(H, g):
    from next_step_ai_b200.weights import gathered_mlp_c

    U = int(g["gate_packed"].shape[0])
    return gathered_mlp_c(hidden=H, gate_packed=g["gate_packed"].reshape(U, -1), gate_absmax=g["gate_absmax"],
                          up_packed=g["up_packed"].reshape(U, -1), up_absmax=g["up_absmax"],
                          down_packed=g["down_cols"], down_absmax=g["down_absmax_cols"], gate_code=g["code"],
                          up_code=g["code"], down_code=g["code"])


def _static_call(x, H, U, c, y, act=None):
    from next_step_ai_b200 import _lib
    from next_step_ai_b200._torch import dtype_code, ptr, stream_handle

    lib = _lib.load()
    return lib.nsm_decode_gathered_static(ptr(x), dtype_code(x.dtype), H, U, ctypes.byref(c), ptr(y),
                                          dtype_code(y.dtype), ptr(act) if act is not None else None,
                                          stream_handle(x.device))


def _workspace_call(x, H, U, c, y, act=None):
    from next_step_ai_b200 import _lib
    from next_step_ai_b200._torch import dtype_code, ptr, stream_handle

    lib = _lib.load()
    ws = torch.zeros(lib.nsm_decode_rows_workspace_bytes(H, U, 1), dtype=torch.uint8, device=x.device)
    st = lib.nsm_decode_gathered(ptr(x), dtype_code(x.dtype), H, U, ctypes.byref(c), ptr(y), dtype_code(y.dtype),
                                 ptr(act) if act is not None else None, ws.data_ptr(), ws.numel(),
                                 stream_handle(x.device))
    torch.cuda.synchronize()
    return st


@pytest.mark.parametrize("name", ["small", "cfg0"])
def test_static_matches_workspace_entry_and_oracle(dev, name):
    from next_step_ai_b200 import _lib

    shape = syn.SHAPES[name]
    H = shape.hidden
    blocks = np.sort(np.random.default_rng(5).choice(shape.num_blocks, shape.top_k, replace=False))
    G = syn.selected_blocks_gathered(shape, 21, 0, blocks)
    g = {k: _t(v, dev) for k, v in G.items()}
    U = len(blocks)
    c, keep = _descriptor(H, g)
    xs = [syn.make_x(shape, seed, 1)[0] for seed in (3, 4)]
    outs = []
    for x_np in xs:  # two calls in a row on the shared array
        x = _t(x_np, dev, torch.bfloat16)
        y = torch.full((H,), float("nan"), dtype=torch.float32, device=dev)
        act = torch.full((U * 32,), float("nan"), dtype=torch.float32, device=dev)
        _lib.check(_static_call(x, H, U, c, y, act), "nsm_decode_gathered_static")
        outs.append((x, y, act))
    torch.cuda.synchronize()
    for x_np, (x, y, act) in zip(xs, outs):
        y_ws = torch.empty(H, dtype=torch.float32, device=dev)
        act_ws = torch.empty(U * 32, dtype=torch.float32, device=dev)
        _lib.check(_workspace_call(x, H, U, c, y_ws, act_ws), "nsm_decode_gathered")
        _close(y.cpu().numpy(), y_ws.cpu().numpy())
        _close(act.cpu().numpy(), act_ws.cpu().numpy())
        ref = om.sparse_mlp_gathered(x.float().cpu().numpy()[None], G["gate_packed"], G["gate_absmax"], G["code"],
                                     G["up_packed"], G["up_absmax"], G["code"], G["down_cols"],
                                     G["down_absmax_cols"], G["code"])[0]
        _close(y.cpu().numpy(), ref)
    _assert_no_static_timeout()
    del keep


def _assert_no_static_timeout():
    """Every bounded wait of the static calls so far completed: the array's
    error word (kept across calls, cleared by this read) is zero."""
    from next_step_ai_b200 import _lib
    from next_step_ai_b200._torch import stream_handle

    code = ctypes.c_int32(-99)
    _lib.check(_lib.load().nsm_static_error(ctypes.byref(code), stream_handle(torch.device("cuda", 0))),
               "nsm_static_error")
    assert code.value == 0


def test_static_at_its_size_limit(dev):
    """hidden = 16384 with 256 gathered blocks (the largest call the array
    holds), device-generated weights; compared with the workspace entry."""
    from next_step_ai_b200 import _lib

    H, U = 16384, 256
    gen = torch.Generator(device=dev).manual_seed(11)
    g = {
        "gate_packed": torch.randint(0, 256, (U, 16 * H), dtype=torch.uint8, device=dev, generator=gen),
        "up_packed": torch.randint(0, 256, (U, 16 * H), dtype=torch.uint8, device=dev, generator=gen),
        "down_cols": torch.randint(0, 256, (H, U, 16), dtype=torch.uint8, device=dev, generator=gen),
        "gate_absmax": torch.rand(U, 32 * H // 64, device=dev, generator=gen) * 0.05 + 0.01,
        "up_absmax": torch.rand(U, 32 * H // 64, device=dev, generator=gen) * 0.05 + 0.01,
        "down_absmax_cols": torch.rand(H, U, device=dev, generator=gen) * 0.05 + 0.01,
        "code": _t(syn.nf4_code(), dev).float(),
    }
    c, keep = _descriptor(H, g)
    for seed in (1, 2):
        x = (torch.randn(H, device=dev, generator=gen.manual_seed(seed))).to(torch.bfloat16)
        y = torch.empty(H, dtype=torch.float32, device=dev)
        _lib.check(_static_call(x, H, U, c, y), "nsm_decode_gathered_static")
        y_ws = torch.empty(H, dtype=torch.float32, device=dev)
        _lib.check(_workspace_call(x, H, U, c, y_ws), "nsm_decode_gathered")
        _close(y.cpu().numpy(), y_ws.cpu().numpy())
    _assert_no_static_timeout()
    del keep


def test_static_rejects_sizes_beyond_its_limit(dev):
    from next_step_ai_b200 import _lib

    lib = _lib.load()
    x = torch.zeros(16384 + 64, dtype=torch.bfloat16, device=dev)
    y = torch.zeros_like(x, dtype=torch.float32)
    c = _lib.MlpWeightsC()
    st = _static_call(x, 16384 + 64, 8, c, y)
    assert st == -2 and "16384" in lib.nsm_last_error().decode()
    st = _static_call(x[:1024], 1024, 257, c, y)
    assert st == -2 and "256" in lib.nsm_last_error().decode()
