"""Host logic of the runtime adapter (``next_step_ai_b200.runtime_adapter``),
no GPU: the kernels are replaced by recording fakes, so what is checked is
the control flow the reference runtime defines around them -- top-k
resolution (``streaming_llama_runtime.py:4338-4350``), the OOM k-halving
retry (``:5493-5524``), the ``None`` contract of
``_sparse_mlp_forward_fast_triton`` (``:5547-5563``), the static skip mask and
SMC reuse of ``_mlp_forward_dispatch`` (``:5839-5860``, ``:5918-5921``).

With ``NSM_REFERENCE_ROOT`` pointing at a reference checkout, the mixin is
also applied to the reference's own ``StreamingLlamaRuntime`` (built with
``__new__``) and the method signatures are compared with the reference's.
"""
from __future__ import annotations

import inspect
import os
import sys
import types

import pytest

torch = pytest.importorskip("torch")

from next_step_ai_b200 import _lib  # noqa: E402
from next_step_ai_b200 import runtime_adapter as ra  # noqa: E402

from tests.fake_runtime import H, NB, FakeRuntime, Runtime, routing as _routing  # noqa: E402


@pytest.fixture
def kernels(monkeypatch):
    """Recording fakes for the kernel entry points the adapter calls."""
    log = []

    def route(flat, rw, top_k=None):
        log.append(("route", int(flat.shape[0]), int(top_k)))
        return torch.arange(top_k, dtype=torch.int64).repeat(int(flat.shape[0]), 1)

    def decode(x, router, w, *, idx, out_dtype=None, **kw):
        log.append(("decode", int(idx.numel())))
        return torch.full((H,), float(idx.numel()), dtype=out_dtype)

    def union(x, idx, w, *, out_dtype=None, **kw):
        log.append(("union", int(x.shape[0]), int(idx.shape[1])))
        return torch.full((int(x.shape[0]), H), 7.0, dtype=out_dtype)

    def gathered(x, **kw):
        log.append(("gathered", kw))
        return torch.full((H,), 3.0)

    def gathered_rows(x, flat_mask, **kw):
        log.append(("gathered_rows", flat_mask, kw))
        return torch.full((int(x.shape[0]), H), 4.0)

    monkeypatch.setattr(ra, "route_sparse_mlp", route)
    monkeypatch.setattr(ra, "sparse_mlp_decode", decode)
    monkeypatch.setattr(ra, "union_decode", union)
    monkeypatch.setattr(ra, "decode_gathered", gathered)
    monkeypatch.setattr(ra, "decode_gathered_rows", gathered_rows)
    return log


def _oom():
    return torch.cuda.OutOfMemoryError("CUDA out of memory. Tried to allocate 2.00 GiB")


# --------------------------------------------------------------------------- OOM detection
def test_is_cuda_oom_error():
    assert ra.is_cuda_oom_error(_oom())
    assert ra.is_cuda_oom_error(_lib.NsmError("nsm_x", _lib.NSM_ERR_CUDA, "CUDA error",
                                              "cudaMalloc: cudaErrorMemoryAllocation (out of memory)"))
    assert ra.is_cuda_oom_error(RuntimeError("CUBLAS_STATUS_ALLOC_FAILED when calling cublasCreate"))
    assert not ra.is_cuda_oom_error(_lib.NsmError("nsm_x", _lib.NSM_ERR_TIMEOUT, "timeout", "wait gave up"))
    assert not ra.is_cuda_oom_error(ValueError("shape mismatch"))
    e = _lib.NsmError("nsm_route", _lib.NSM_ERR_INVALID_ARG, "invalid argument", "k > NB")
    assert isinstance(e, RuntimeError) and e.status == _lib.NSM_ERR_INVALID_ARG and "k > NB" in str(e)


# --------------------------------------------------------------------------- OomPolicy
def test_oom_policy_halves_k_twice_then_zero():
    seen, logs, clamps = [], [], []
    hidden = torch.ones(1, 1, H)

    def fn(ab):
        seen.append(int(ab.shape[-1]))
        raise _oom()

    pol = ra.OomPolicy(log=logs.append)
    out = pol.run(fn, hidden, torch.arange(8).view(1, 8), on_clamp=clamps.append)
    assert seen == [8, 4, 2] and clamps == [4, 2]
    assert torch.equal(out, torch.zeros_like(hidden))
    assert logs[0] == "[sparse] CUDA OOM in sparse MLP fallback; retrying with top_k=4."
    assert "using zero MLP contribution" in logs[-1]


def test_oom_policy_keeps_leading_blocks_and_succeeds():
    seen = []
    ab = torch.tensor([[5, 1, 7, 3, 2, 0]])

    def fn(a):
        seen.append(a.clone())
        if a.shape[-1] > 3:
            raise _oom()
        return torch.ones(1, H)

    out = ra.OomPolicy(log=lambda m: None).run(fn, torch.zeros(1, H), ab)
    assert torch.equal(seen[-1], torch.tensor([[5, 1, 7]])) and torch.equal(out, torch.ones(1, H))


def test_oom_policy_k1_and_non_oom():
    calls = []

    def oom(a):
        calls.append(int(a.shape[-1]))
        raise _oom()

    out = ra.OomPolicy(log=lambda m: None).run(oom, torch.ones(H), torch.tensor([[4]]))
    assert calls == [1] and torch.equal(out, torch.zeros(H))  # one block left: no retry

    def bad(a):
        raise ValueError("not an allocation failure")

    with pytest.raises(ValueError):
        ra.OomPolicy().run(bad, torch.ones(H), torch.tensor([[1, 2]]))


# --------------------------------------------------------------------------- DecodeMlpPolicy
def test_decode_policy_skip_and_reuse():
    pol = ra.DecodeMlpPolicy(3, H, device="cpu", dtype=torch.float32, skip_mask=torch.tensor([0, 1, 0]),
                             enable_smc=True, smc_threshold=0.04)
    n = []

    def compute(x):
        n.append(1)
        return x * 2

    x = torch.randn(H)
    assert torch.equal(pol.forward(1, x, compute), torch.zeros(H)) and not n      # skipped layer
    y0 = pol.forward(0, x, compute)
    assert len(n) == 1 and torch.equal(y0, x * 2)
    y1 = pol.forward(0, x + 0.01 * x.norm() / H ** 0.5 * torch.randn(H), compute)  # ~1% move: reuse
    assert len(n) == 1 and torch.equal(y1, y0)
    pol.forward(0, -x, compute)                                                   # far: recompute
    assert len(n) == 2
    assert pol.skip(1) and not pol.skip(0) and not pol.skip(9)
    off = ra.DecodeMlpPolicy(3, H, device="cpu", dtype=torch.float32)
    off.forward(0, x, compute)
    off.forward(0, x, compute)
    assert len(n) == 4                                                            # SMC off: always compute


# --------------------------------------------------------------------------- router k resolution
def test_route_top_k_resolution(kernels):
    rt = Runtime()
    assert rt._route_sparse_mlp(torch.zeros(1, 1, H), 5) is None                  # no routing: dense
    out = rt._route_sparse_mlp(torch.zeros(1, 2, H), 0)
    assert out.shape == (2, 6) and kernels[-1] == ("route", 2, 6)                 # _sparse_top_k
    rt._route_sparse_mlp(torch.zeros(1, 1, H), 1)
    assert kernels[-1] == ("route", 1, 3)                                         # the layer's own top_k
    rt._sparse_runtime_top_k = 2
    rt._route_sparse_mlp(torch.zeros(1, 1, H), 0)
    assert kernels[-1] == ("route", 1, 2)                                         # runtime k when > 0
    rt._sparse_runtime_top_k = 50
    rt._route_sparse_mlp(torch.zeros(1, 1, H), 0)
    assert kernels[-1] == ("route", 1, NB)                                        # clamped to NB
    rt._traffic_current_phase, rt._sparse_mlp_prefill_mode, rt._sparse_mlp_prefill_top_k = "prefill", "sparse", 5
    rt._route_sparse_mlp(torch.zeros(1, 1, H), 1)
    assert kernels[-1] == ("route", 1, 5)                                         # sparse-prefill override
    rw0 = rt._nsm_router(0, rt._sparse_routing[0])
    assert rt._nsm_router(0, rt._sparse_routing[0]) is rw0                        # built once per routing dict
    rt._sparse_routing[0] = _routing()
    assert rt._nsm_router(0, rt._sparse_routing[0]) is not rw0                    # rebuilt when replaced


# --------------------------------------------------------------------------- resident forward
def test_forward_fast_resident_and_fallthrough(kernels, capsys):
    rt = Runtime()
    rt.nsm_attach(mlp={0: object()})
    y = rt._sparse_mlp_forward_fast(1, None, torch.zeros(1, 1, H), torch.arange(4).view(1, 4))
    assert rt.calls == [("super_fast", 1)] and float(y[0, 0, 0]) == -1.0           # not resident: runtime's path
    y = rt._sparse_mlp_forward_fast(0, None, torch.zeros(1, 1, H), torch.arange(4).view(1, 4))
    assert kernels[-1] == ("decode", 4) and y.shape == (1, 1, H) and float(y[0, 0, 0]) == 4.0
    y = rt._sparse_mlp_forward_fast(0, None, torch.zeros(1, 40, H), torch.zeros(40, 4, dtype=torch.long))
    assert [c for c in kernels if c[0] == "union"] == [("union", 32, 4), ("union", 8, 4)]
    assert y.shape == (1, 40, H)
    rt._sparse_routing[0]["block_domain"] = "hidden"
    with pytest.raises(RuntimeError, match="intermediate FFN routing"):
        rt._sparse_mlp_forward_fast(0, None, torch.zeros(1, 1, H), torch.arange(4).view(1, 4))


def test_forward_fast_resident_oom_clamps_runtime_k(kernels, monkeypatch, capsys):
    rt = Runtime()
    rt.nsm_attach(mlp={0: object()})

    def decode(x, router, w, *, idx, out_dtype=None, **kw):
        if idx.numel() > 2:
            raise _oom()
        return torch.full((H,), float(idx.numel()), dtype=out_dtype)

    monkeypatch.setattr(ra, "sparse_mlp_decode", decode)
    y = rt._sparse_mlp_forward_fast(0, None, torch.zeros(1, 1, H), torch.arange(8).view(1, 8))
    assert float(y[0, 0, 0]) == 2.0 and rt._sparse_runtime_top_k == 2
    out = capsys.readouterr().out
    assert "runtime top_k clamped to 4 after CUDA OOM." in out and "retrying with top_k=2." in out


# --------------------------------------------------------------------------- gathered entry
def _gathered_kwargs(rows, U, *, down=True, bias=False, local=None):
    I = NB * 32
    an = (torch.arange(U).unsqueeze(-1) * 32 + torch.arange(32)).reshape(-1)
    p = {"quant_block_size": 64, "in_features": H, "out_features": I, "code": torch.linspace(-1, 1, 16)}
    return dict(
        hidden=torch.zeros(1, rows, H), flat_hidden=torch.zeros(rows, H), ordered_blocks=torch.arange(U),
        active_local=local if local is not None else torch.arange(U, dtype=torch.int32).repeat(rows, 1),
        flat_mask=torch.ones(rows, U * 32), active_neurons=an,
        gate_bias=torch.arange(I, dtype=torch.float32) if bias else None, up_bias=None,
        down_bias=torch.ones(H) if bias else None,
        gate_param=p, up_param=p, down_param=dict(p, out_features=H, in_features=I),
        gate_packed_gpu=torch.zeros(U, 32, H // 2, dtype=torch.uint8), gate_absmax_gpu=torch.ones(U, 32, H // 64),
        up_packed_gpu=torch.zeros(U, 32, H // 2, dtype=torch.uint8), up_absmax_gpu=torch.ones(U, 32, H // 64),
        down_packed_gpu=torch.zeros(H, U, 16, dtype=torch.uint8) if down else None,
        down_absmax_gpu=torch.ones(H, U) if down else None)


def test_forward_fast_triton_none_contract(kernels, capsys):
    rt = Runtime()
    rt._triton_fused_sparse_mlp = False
    assert rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 3)) is None
    assert rt._decode_backend_name == "dequant_sparse_fallback"
    assert "disabled by runtime flag" in capsys.readouterr().out
    assert rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 3)) is None
    assert capsys.readouterr().out == ""                                          # logged once
    rt = Runtime()
    assert rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 3, down=False)) is None
    assert "missing down buffers" in capsys.readouterr().out
    assert not kernels
    with pytest.raises(TypeError):
        rt._sparse_mlp_forward_fast_triton(torch.zeros(1, 1, H))                  # keyword-only


def test_forward_fast_triton_dispatch(kernels):
    rt = Runtime()
    y = rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 3, bias=True))
    name, kw = kernels[-1]
    assert name == "gathered" and y.shape == (1, 1, H) and float(y.flatten()[0]) == 3.0
    assert rt._decode_backend_name == "nsm_single_kernel_sparse_decode_sm100"
    assert torch.equal(kw["gate_bias"], torch.arange(96, dtype=torch.float32))   # gathered neuron order
    assert kw["up_bias"] is None and torch.equal(kw["down_bias"], torch.ones(H))
    assert torch.equal(kw["gate_code"], torch.linspace(-1, 1, 16))
    rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 3, local=torch.tensor([[0, -1, 2]], dtype=torch.int32)))
    assert kernels[-1][0] == "gathered_rows"                                      # a missing slot: masked rows
    y = rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(3, 4))
    assert kernels[-1][0] == "gathered_rows" and y.shape == (1, 3, H)
    assert rt._decode_backend_name == "nsm_gathered_rows_sparse_decode_sm100"
    rt._single_kernel_decode_enabled = False
    rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 3))
    assert kernels[-1][0] == "gathered_rows"
    kw0 = _gathered_kwargs(1, 0)
    assert torch.equal(rt._sparse_mlp_forward_fast_triton(**kw0), torch.zeros(1, 1, H))
    rt._sparse_block_size = 16
    with pytest.raises(RuntimeError, match="block_size=32"):
        rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 3))


# --------------------------------------------------------------------------- dispatch
def test_dispatch_skip_smc_and_fallthrough(kernels):
    rt = Runtime()
    rt.nsm_attach(mlp={0: object(), 1: object()})
    layer = types.SimpleNamespace(mlp=None)
    x = torch.randn(1, 1, H)
    rt._mlp_static_skip_mask = torch.tensor([False, True, False, False])
    rt._mlp_static_skip_set = {1}
    assert torch.equal(rt._mlp_forward_dispatch(1, layer, x), torch.zeros_like(x)) and not kernels
    y = rt._mlp_forward_dispatch(0, layer, x)
    assert [k[0] for k in kernels] == ["route", "decode"] and float(y.flatten()[0]) == 6.0
    assert ("calib", 0) in rt.calls and 0 in rt._decode_prefetch_route_cache
    rt._enable_smc = True
    rt._mlp_forward_dispatch(0, layer, x)
    assert bool(rt._smc_valid[0]) and len(kernels) == 4
    y2 = rt._mlp_forward_dispatch(0, layer, x * 1.001)                            # within 4%: reuse
    assert len(kernels) == 4 and torch.equal(y2, rt._smc_out[0].view_as(x))
    rt._mlp_forward_dispatch(0, layer, -x)                                        # far: recompute
    assert len(kernels) == 6
    rt._traffic_current_phase = "prefill"
    assert float(rt._mlp_forward_dispatch(0, layer, x).flatten()[0]) == -2.0      # runtime's own prefill
    rt._traffic_current_phase = "decode"
    rt._mlp_forward_dispatch(2, layer, x)                                         # not resident
    assert rt.calls[-1] == ("super_dispatch", 2)


# --------------------------------------------------------------------------- the reference's own class
def _reference_runtime_class():
    root = os.environ.get("NSM_REFERENCE_ROOT")
    if not root or not os.path.isdir(root):
        pytest.skip("NSM_REFERENCE_ROOT not set")
    if root not in sys.path:
        sys.path.insert(0, root)
    # bitsandbytes is not installed: stand-ins for the two names the module imports
    for name, pkg in (("bitsandbytes", True), ("bitsandbytes.functional", False), ("bitsandbytes.backends", True),
                      ("bitsandbytes.backends.cuda", True), ("bitsandbytes.backends.cuda.ops", False)):
        if name not in sys.modules:
            m = types.ModuleType(name)
            if pkg:
                m.__path__ = []
            sys.modules[name] = m
    sys.modules["bitsandbytes"].functional = sys.modules["bitsandbytes.functional"]
    sys.modules["bitsandbytes.backends.cuda.ops"]._dequantize_4bit_impl = lambda *a, **k: None
    try:
        from llama3_neuroplastic.experiments.streaming_llama_runtime import StreamingLlamaRuntime
    except Exception as exc:  # noqa: BLE001
        pytest.skip(f"reference runtime not importable: {exc}")
    return StreamingLlamaRuntime


@pytest.mark.parametrize("method", ["_route_sparse_mlp", "_sparse_mlp_forward_fast",
                                    "_sparse_mlp_forward_fast_triton", "_mlp_forward_dispatch"])
def test_signatures_match_reference(method):
    ref = inspect.signature(getattr(_reference_runtime_class(), method))
    ours = inspect.signature(getattr(ra.B200SparseMlpMixin, method))
    assert [(p.name, p.kind) for p in ours.parameters.values()] == \
        [(p.name, p.kind) for p in ref.parameters.values()]


def test_mixin_on_reference_runtime(kernels):
    Ref = _reference_runtime_class()
    Mixed = type("B200StreamingLlamaRuntime", (ra.B200SparseMlpMixin, Ref), {})
    rt = Mixed.__new__(Mixed)
    base = FakeRuntime()
    rt.__dict__.update({k: v for k, v in base.__dict__.items() if k != "calls"})
    rt._record_hot_cache_calibration_blocks = lambda li, ab: None
    rt.nsm_attach(mlp={0: object()})
    x = torch.randn(1, 1, H)
    y = rt._mlp_forward_dispatch(0, types.SimpleNamespace(mlp=None), x)
    assert [k[0] for k in kernels] == ["route", "decode"] and y.shape == x.shape
    rt._mlp_static_skip_mask = torch.tensor([True])
    assert torch.equal(rt._mlp_forward_dispatch(0, None, x), torch.zeros_like(x))
    rt._triton_fused_sparse_mlp = False
    assert rt._sparse_mlp_forward_fast_triton(**_gathered_kwargs(1, 2)) is None
