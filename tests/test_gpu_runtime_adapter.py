"""The runtime adapter's entries against the CPU oracle, on the GPU.

``B200SparseMlpMixin`` is applied to a stand-in of the reference runtime's
state (``tests/fake_runtime.py``) and called the way the reference runtime
calls its own methods: ``_route_sparse_mlp`` then ``_sparse_mlp_forward_fast``
on resident pools (one row, and several rows through the union kernels),
``_sparse_mlp_forward_fast_triton`` with the keyword arguments the runtime
builds from its gathered buffers (``streaming_llama_runtime.py:5385-5404``,
layout from ``_build_sparse_active_layout`` ``:4857-4908``), and
``_mlp_forward_dispatch`` with SMC reuse.  Block ids bit-exact; outputs within
max-abs 2e-2 and relative L2 5e-3 of the fp32 oracle (plus half a bf16 ulp of
the reference value for bf16 outputs).
"""
from __future__ import annotations

import types

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import layout as lay  # noqa: E402
from oracle import mlp as om  # noqa: E402
from oracle import router as orr  # noqa: E402
from oracle import synthetic as syn  # noqa: E402
from tests.fake_runtime import Runtime  # noqa: E402
from tests.test_gpu_decode import T, assert_close, full_layer, weights_for  # noqa: E402


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from next_step_ai_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def _runtime(name, seed, dev, *, resident=True):
    shape = syn.SHAPES[name]
    R = syn.make_router(shape, seed)
    routing = {"enc_w": T(R["enc_w"], dev, torch.bfloat16), "enc_b": T(R["enc_b"], dev, torch.bfloat16),
               "route_score_weight": T(R["score_w"], dev, torch.bfloat16),
               "route_score_bias": T(R["score_b"], dev, torch.bfloat16), "basis_top_k": shape.rank}
    rt = Runtime(num_layers=2, hidden=shape.hidden, device=dev)
    rt._sparse_routing = {0: routing}
    rt._sparse_top_k = shape.top_k
    rt._smc_x_in = rt._smc_x_in.to(torch.bfloat16)
    rt._smc_out = rt._smc_out.to(torch.bfloat16)
    full = full_layer(name, seed)
    if resident:
        rt.nsm_attach(mlp={0: weights_for(shape, full, dev)})
    return rt, shape, R, full


def _oracle_route(shape, R, X):
    return orr.route_sparse_mlp(np.asarray(X, np.float32), R["enc_w"], R["enc_b"], R["score_w"], R["score_b"],
                                shape.top_k, shape.rank)


def _oracle_mlp(shape, full, x, blocks):
    return om.sparse_mlp_full(np.asarray(x, np.float32).reshape(1, -1), np.asarray(blocks), full["gate_packed"],
                              full["gate_absmax"], full["up_packed"], full["up_absmax"], full["down_packed"],
                              full["down_absmax"], full["code"], hidden=shape.hidden,
                              intermediate=shape.intermediate)[0]


@pytest.mark.parametrize("name,seed,rows", [("small", 21, 1), ("small", 22, 5), ("cfg0", 23, 1), ("cfg0", 24, 3)])
def test_route_and_resident_forward_match_oracle(dev, name, seed, rows):
    rt, shape, R, full = _runtime(name, seed, dev)
    X = syn.make_x(shape, seed, rows, shared=0.5)
    hidden = T(X, dev, torch.bfloat16).view(1, rows, shape.hidden)
    ab = rt._route_sparse_mlp(hidden, 0)
    ref_idx = _oracle_route(shape, R, X)
    assert ab.dtype == torch.int64 and np.array_equal(ab.cpu().numpy(), ref_idx)
    y = rt._sparse_mlp_forward_fast(0, None, hidden, ab)
    assert y.shape == hidden.shape and y.dtype == torch.bfloat16
    assert rt._decode_backend_name == "nsm_resident_sparse_decode_sm100"
    for r in range(rows):
        assert_close(y[0, r].float().cpu().numpy(), _oracle_mlp(shape, full, X[r], ref_idx[r]), bf16_out=True)


@pytest.mark.parametrize("name,seed,rows", [("small", 31, 1), ("small", 32, 4), ("cfg0", 33, 1), ("cfg0", 34, 2)])
def test_gathered_keyword_entry_matches_oracle(dev, name, seed, rows):
    """``_sparse_mlp_forward_fast_triton`` over the runtime's gathered buffers:
    one row through the single gathered kernel, several rows through the
    masked rows kernel."""
    rt, shape, R, full = _runtime(name, seed, dev, resident=False)
    X = syn.make_x(shape, seed, rows, shared=0.5)
    ab = _oracle_route(shape, R, X)
    ordered, active_local, flat_mask, active_neurons = lay.build_sparse_active_layout(ab, rows, 32, shape.num_blocks)
    G = syn.selected_blocks_gathered(shape, seed, 0, ordered)
    code = T(G["code"], dev)
    p = {"quant_block_size": 64, "in_features": shape.hidden, "out_features": shape.intermediate, "code_gpu": code}
    hidden = T(X, dev, torch.bfloat16).view(1, rows, shape.hidden)
    y = rt._sparse_mlp_forward_fast_triton(
        hidden=hidden, flat_hidden=hidden.view(rows, -1), ordered_blocks=torch.from_numpy(ordered),
        active_local=T(active_local, dev), flat_mask=T(flat_mask, dev, torch.bfloat16),
        active_neurons=torch.from_numpy(active_neurons), gate_bias=None, up_bias=None, down_bias=None,
        gate_param=p, up_param=p, down_param=dict(p, in_features=shape.intermediate, out_features=shape.hidden),
        gate_packed_gpu=T(G["gate_packed"], dev), gate_absmax_gpu=T(G["gate_absmax"], dev),
        up_packed_gpu=T(G["up_packed"], dev), up_absmax_gpu=T(G["up_absmax"], dev),
        down_packed_gpu=T(G["down_cols"], dev), down_absmax_gpu=T(G["down_absmax_cols"], dev))
    assert y is not None and y.shape == hidden.shape and y.dtype == torch.bfloat16
    want = "nsm_single_kernel_sparse_decode_sm100" if rows == 1 else "nsm_gathered_rows_sparse_decode_sm100"
    assert rt._decode_backend_name == want
    ref = om.sparse_mlp_gathered(np.asarray(X, np.float32), G["gate_packed"], G["gate_absmax"], G["code"],
                                 G["up_packed"], G["up_absmax"], G["code"], G["down_cols"], G["down_absmax_cols"],
                                 G["code"], flat_mask=flat_mask)
    for r in range(rows):
        assert_close(y[0, r].float().cpu().numpy(), ref[r], bf16_out=True)
        # the gathered result is the resident result over the same blocks
        assert_close(y[0, r].float().cpu().numpy(), _oracle_mlp(shape, full, X[r], ab[r]), bf16_out=True)


def test_dispatch_with_smc_reuse(dev):
    rt, shape, R, full = _runtime("small", 41, dev)
    rt._enable_smc = True
    X = syn.make_x(shape, 41, 1)
    x = T(X, dev, torch.bfloat16).view(1, 1, shape.hidden)
    layer = types.SimpleNamespace(mlp=None)  # the decoder layer; the resident path does not read its module
    y0 = rt._mlp_forward_dispatch(0, layer, x)
    assert_close(y0.float().cpu().numpy().reshape(-1), _oracle_mlp(shape, full, X[0], _oracle_route(shape, R, X)[0]),
                 bf16_out=True)
    assert bool(rt._smc_valid[0].item())
    y1 = rt._mlp_forward_dispatch(0, layer, x)  # same input: the cached output
    assert torch.equal(y1, y0)
    X2 = syn.make_x(shape, 42, 1)
    y2 = rt._mlp_forward_dispatch(0, layer, T(X2, dev, torch.bfloat16).view(1, 1, -1))
    assert_close(y2.float().cpu().numpy().reshape(-1),
                 _oracle_mlp(shape, full, X2[0], _oracle_route(shape, R, X2)[0]), bf16_out=True)
