"""The NF4 LM head (``nsm_lm_head_nf4``) against the fp64 oracle: logits =
x @ dequant(W).T (+ bias) for a bitsandbytes row-major NF4 weight, with the
decode path's tolerances (max-abs <= 2e-2, relative L2 <= 5e-3; for bf16
output the value's own half-ulp is added to the absolute bound)."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle.nf4 import bf16_round, dequantize_nf4, nf4_code, quantize_nf4  # noqa: E402

from tests.test_gpu_decode import assert_close  # noqa: E402


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from next_step_ai_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def _weights(V, H, qbs, seed):
    g = np.random.default_rng(seed)
    w = (g.standard_normal((V, H)) * 0.02).astype(np.float32)
    packed, absmax = quantize_nf4(w, nf4_code(), qbs)
    return packed, absmax


@pytest.mark.parametrize("V,H,qbs,T", [(1000, 1024, 64, 1), (1000, 1024, 128, 3), (517, 2048, 64, 8),
                                       (4096, 4096, 64, 2)])
def test_lm_head_matches_oracle(dev, V, H, qbs, T):
    from next_step_ai_b200.lm_head import Nf4LmHead

    packed, absmax = _weights(V, H, qbs, V + H + T)
    code = nf4_code()
    g = np.random.default_rng(T)
    x = bf16_round((g.standard_normal((T, H)) * 3.0).astype(np.float32))
    x[0, :5] = [300.0, -250.0, 1e-3, 0.0, 7.5]           # a wide dynamic range
    bias = bf16_round((g.standard_normal(V) * 0.5).astype(np.float32))
    W = dequantize_nf4(packed, absmax, code, qbs).reshape(V, H).astype(np.float64)
    ref = x.astype(np.float64) @ W.T + bias.astype(np.float64)
    head = Nf4LmHead(torch.from_numpy(packed).to(dev), torch.from_numpy(absmax).to(dev),
                     torch.from_numpy(code).to(dev), out_features=V, in_features=H, quant_block_size=qbs,
                     bias=torch.from_numpy(bias).to(dev, torch.bfloat16))
    xd = torch.from_numpy(x).to(dev, torch.bfloat16).view(1, T, H)
    y = head(xd, out_dtype=torch.float32)
    assert y.shape == (1, T, V)
    assert_close(y.view(T, V).cpu().numpy(), ref)
    yb = head(xd)                                         # bf16 logits, the runtime's dtype
    assert yb.dtype == torch.bfloat16
    assert_close(yb.view(T, V).float().cpu().numpy(), ref, bf16_out=True)
    # one token at a time gives the same logits (the token slots are independent)
    y1 = torch.cat([head(xd[:, t:t + 1], out_dtype=torch.float32) for t in range(T)], dim=1)
    assert torch.equal(y1, y)


def test_lm_head_from_dense_and_405b_vocab(dev):
    """405B shape (vocab 128256 x 16384), quantised on the device from a dense
    weight; 257 sampled rows checked against the oracle on the same bytes."""
    from next_step_ai_b200.lm_head import Nf4LmHead

    V, H = 128256, 16384
    gen = torch.Generator(device=dev).manual_seed(5)
    w = torch.randn((V, H), generator=gen, device=dev, dtype=torch.bfloat16) * 0.02
    head = Nf4LmHead.from_dense(w, dev)
    del w
    assert head.quant_block_size == 64 and head.max_tokens_per_call >= 1
    x = (torch.randn((2, H), generator=gen, device=dev) * 2.0).to(torch.bfloat16)
    y = head(x, out_dtype=torch.float32)
    rows = np.concatenate([[0, V - 1], np.random.default_rng(1).choice(V, 255, replace=False)])
    pk = head.packed.view(V, H // 2)[torch.from_numpy(rows).to(dev)].cpu().numpy()
    am = head.absmax.view(V, H // 64)[torch.from_numpy(rows).to(dev)].cpu().numpy()
    W = dequantize_nf4(pk.reshape(-1), am.reshape(-1), head.code.cpu().numpy(), 64).reshape(rows.size, H)
    ref = x.float().cpu().numpy().astype(np.float64) @ W.astype(np.float64).T
    assert_close(y[:, torch.from_numpy(rows).to(dev)].cpu().numpy(), ref)


def test_lm_head_rejects_bad_shapes(dev):
    from next_step_ai_b200.lm_head import Nf4LmHead

    packed, absmax = _weights(64, 1024, 64, 0)
    P, A, C = (torch.from_numpy(a).to(dev) for a in (packed, absmax, nf4_code()))
    with pytest.raises(RuntimeError, match="bytes"):
        Nf4LmHead(P[:-1], A, C, out_features=64, in_features=1024)
    head = Nf4LmHead(P, A, C, out_features=64, in_features=1024)
    with pytest.raises(RuntimeError, match="expects 1024"):
        head(torch.zeros(1, 512, device=dev, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="CUDA"):
        head(torch.zeros(1, 1024, dtype=torch.bfloat16))
