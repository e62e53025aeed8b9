"""The multi-layer decode engine (SparseMlpDecoder) on the GPU.

A token goes through L decoder layers: residual += previous layer's MLP output
(fp32), x = RMSNorm(residual) * gamma, learned-basis routing, NF4 MLP on the
selected blocks -- the per-layer tail of the reference's forward_token
(streaming_llama_runtime.py:7762-7775) with attention left out.  The oracle
chains the same steps in numpy; the eager pass and the CUDA-graph replay must
give identical bits, and both must match the oracle within the decode
tolerances (max-abs-err <= 2e-2, relative L2 <= 5e-3).
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import mlp as om  # noqa: E402
from oracle import router as orr  # noqa: E402
from oracle import synthetic as syn  # noqa: E402
from oracle.nf4 import bf16_round  # noqa: E402

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
    assert err <= MAX_ABS * max(1.0, float(np.abs(ref).max()) / 8), f"max abs err {err:.3e}"


def _build(shape_name, n_unique, dev, seed=40):
    from next_step_ai_b200 import RouterWeights, SparseMlpWeights
    from next_step_ai_b200.engine import DecodeLayer

    shape = syn.SHAPES[shape_name]
    host, layers = [], []
    for l in range(n_unique):
        full = syn.make_layer_full(shape, seed + l)
        R = syn.make_router(shape, seed + l)
        gamma = bf16_round(np.random.default_rng(seed + l).uniform(0.6, 1.4, shape.hidden).astype(np.float32))
        w = SparseMlpWeights.from_bnb_rowmajor(
            hidden=shape.hidden, intermediate=shape.intermediate, gate_packed=_t(full["gate_packed"], dev),
            gate_absmax=_t(full["gate_absmax"], dev), up_packed=_t(full["up_packed"], dev),
            up_absmax=_t(full["up_absmax"], dev), down_packed=_t(full["down_packed"], dev),
            down_absmax=_t(full["down_absmax"], dev), code=_t(full["code"], dev))
        rw = RouterWeights(enc_w=_t(R["enc_w"], dev, torch.bfloat16), score_w=_t(R["score_w"], dev, torch.bfloat16),
                           enc_b=_t(R["enc_b"], dev, torch.bfloat16), score_b=_t(R["score_b"], dev, torch.bfloat16),
                           top_k=shape.top_k, basis_top_k=shape.rank)
        layers.append(DecodeLayer(router=rw, weights=w, norm_weight=_t(gamma, dev, torch.bfloat16)))
        host.append((full, R, gamma))
    return shape, layers, host


def _oracle(shape, host, num_layers, x0, eps=1e-5):
    r = x0.astype(np.float32).copy()
    y_prev = None
    for i in range(num_layers):
        full, R, gamma = host[i % len(host)]
        if y_prev is not None:
            r = (r + y_prev).astype(np.float32)
        xn = om.rms_norm(r, gamma, eps)
        idx = orr.route_sparse_mlp(xn, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k,
                                   shape.rank)[0]
        y = om.sparse_mlp_full(xn, idx, full["gate_packed"], full["gate_absmax"], full["up_packed"],
                               full["up_absmax"], full["down_packed"], full["down_absmax"], full["code"],
                               hidden=shape.hidden, intermediate=shape.intermediate)[0]
        y_prev = y.astype(np.float32)  # the engine keeps each layer's output in fp32 for the next
    return (r + y_prev).astype(np.float32)


@pytest.mark.parametrize("shape_name,n_unique,num_layers", [("tiny", 2, 5), ("small", 3, 4)])
def test_engine_eager_and_graph_match_oracle(dev, shape_name, n_unique, num_layers):
    from next_step_ai_b200.engine import SparseMlpDecoder

    shape, layers, host = _build(shape_name, n_unique, dev)
    x0 = (np.random.default_rng(7).standard_normal(shape.hidden) * 2).astype(np.float32)
    dec = SparseMlpDecoder(layers, num_layers)
    dec.residual.copy_(_t(x0, dev))
    dec.step_eager()
    eager = dec.out.clone()
    dec.residual.copy_(_t(x0, dev))
    g = dec.capture()  # the capture's warm-up step also starts from x0
    dec.residual.copy_(_t(x0, dev))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(dec.out, eager)
    _close(eager.cpu().numpy(), _oracle(shape, host, num_layers, x0))
    dec.release()


def test_engine_stage_timing(dev):
    from next_step_ai_b200.engine import SparseMlpDecoder

    shape, layers, _ = _build("small", 1, dev)
    dec = SparseMlpDecoder(layers, 3)
    dec.residual.copy_(_t(np.ones(shape.hidden, np.float32), dev))
    t = dec.time_stages()
    assert list(t) == list(SparseMlpDecoder.STAGES)
    assert all(t[s] > 0 for s in ("router", "gateup", "down")), t
    assert t["gateup_finalize"] >= 0 and t["down_finalize"] >= 0  # folded into gate/up / the next layer
