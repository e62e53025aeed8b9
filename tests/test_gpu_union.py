"""Multi-token decode over the union of the tokens' blocks (nsm_union_decode).

Row r of the output must equal the single-token MLP over row r's own blocks
(the reference's flat_mask semantics) from the fp32 oracle, within the decode
tolerances (max-abs-err <= 2e-2, relative L2 <= 5e-3), and the union must be
the reference's active layout: the rows' blocks, ascending.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import layout as lay  # noqa: E402
from oracle import mlp as om  # noqa: E402
from oracle import router as orr  # noqa: E402
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
    assert rel <= REL_L2, f"relative L2 {rel:.3e}"
    assert float(np.abs(got - ref).max()) <= MAX_ABS


_CACHE: dict = {}


def _layer(name, seed, dev):
    from next_step_ai_b200 import SparseMlpWeights

    key = (name, seed)
    if key not in _CACHE:
        shape = syn.SHAPES[name]
        full = syn.make_layer_full(shape, seed)
        w = SparseMlpWeights.from_bnb_rowmajor(
            hidden=shape.hidden, intermediate=shape.intermediate, gate_packed=_t(full["gate_packed"], dev),
            gate_absmax=_t(full["gate_absmax"], dev), up_packed=_t(full["up_packed"], dev),
            up_absmax=_t(full["up_absmax"], dev), down_packed=_t(full["down_packed"], dev),
            down_absmax=_t(full["down_absmax"], dev), code=_t(full["code"], dev))
        _CACHE[key] = (shape, full, w)
    return _CACHE[key]


def _ref_rows(shape, full, x, idx):
    out = []
    for r in range(x.shape[0]):
        blocks = np.array([b for b in idx[r] if 0 <= b < shape.num_blocks], np.int64)
        out.append(om.sparse_mlp_full(x[r], blocks, full["gate_packed"], full["gate_absmax"], full["up_packed"],
                                      full["up_absmax"], full["down_packed"], full["down_absmax"], full["code"],
                                      hidden=shape.hidden, intermediate=shape.intermediate)[0])
    return np.stack(out)


@pytest.mark.parametrize("name,rows,shared", [("small", 5, 0.5), ("small", 32, 0.8), ("cfg0", 32, 0.85),
                                              ("tiny", 1, 0.0)])
def test_union_decode_matches_per_row_oracle(dev, name, rows, shared):
    from next_step_ai_b200 import union_decode

    shape, full, w = _layer(name, 21, dev)
    R = syn.make_router(shape, 21)
    x = syn.make_x(shape, 60 + rows, rows, shared=shared)
    idx = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)
    y, uni = union_decode(_t(x, dev, torch.bfloat16), _t(idx.astype(np.int32), dev), w, out_dtype=torch.float32,
                          return_union=True)
    ordered, _, _, _ = lay.build_sparse_active_layout(idx, rows, 32, shape.num_blocks)
    assert np.array_equal(uni.cpu().numpy(), np.asarray(ordered))
    ref = _ref_rows(shape, full, x, idx)
    for r in range(rows):
        _close(y[r].cpu().numpy(), ref[r])


def test_union_decode_cfg1_config4(dev):
    """BASELINE config 4 as the benchmark runs it: a 405B-shaped layer (H =
    16384, 1664 blocks, k = 208), 32 tokens rms(0.85 z + sqrt(1 - 0.85^2) e_t)
    routed together on the GPU (bit-exact against the oracle router), the union
    in ascending order, and every row against the oracle's fp32 dequant +
    matmul over the union with the reference's per-row flat_mask."""
    from next_step_ai_b200 import route_sparse_mlp, union_decode
    from next_step_ai_b200 import synthetic as dsyn
    from tests.gpu_oracle import host_router, oracle_mlp_rows

    shape = dsyn.SHAPES["cfg1"]
    w, bnb = dsyn.make_layer_weights(shape, 1234, 0, dev, keep_bnb=True)
    rw = dsyn.make_router(shape, 1234, 0, dev)
    x = dsyn.make_x(shape, 99, 32, dev, shared=0.85)
    idx = route_sparse_mlp(x, rw).to(torch.int32)
    xh = x.float().cpu().numpy()
    R = host_router(rw)
    ref_idx = orr.route_sparse_mlp(xh, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    y, uni = union_decode(x, idx, w, out_dtype=torch.float32, return_union=True)
    ordered, _, flat_mask, _ = lay.build_sparse_active_layout(ref_idx, 32, 32, shape.num_blocks)
    assert np.array_equal(uni.cpu().numpy(), np.asarray(ordered))
    assert 600 <= len(ordered) <= 1000, len(ordered)
    ref = oracle_mlp_rows(bnb, shape.hidden, shape.intermediate, xh, np.asarray(ordered), flat_mask)
    got = y.cpu().numpy()
    for r in range(32):
        _close(got[r], ref[r])


def test_union_decode_ignores_invalid_ids_and_respects_shards(dev):
    from next_step_ai_b200 import union_decode

    shape, full, w = _layer("small", 22, dev)
    rng = np.random.default_rng(5)
    rows, k = 6, shape.top_k
    x = syn.make_x(shape, 77, rows, shared=0.3)
    idx = np.stack([rng.choice(shape.num_blocks, k, replace=False) for _ in range(rows)]).astype(np.int32)
    idx[0, :3] = -1
    idx[2, -2:] = shape.num_blocks + 7
    y = union_decode(_t(x, dev, torch.bfloat16), _t(idx, dev), w, out_dtype=torch.float32)
    ref = _ref_rows(shape, full, x, idx)
    for r in range(rows):
        _close(y[r].cpu().numpy(), ref[r])
    # two shards of a multi-GPU split: each pool holds its own block range and
    # the partial outputs sum to the whole
    from next_step_ai_b200 import SparseMlpWeights

    nb = shape.num_blocks
    parts = []
    for lo, hi in ((0, nb // 2), (nb // 2, nb)):
        ws = SparseMlpWeights(hidden=w.hidden, intermediate=w.intermediate, gate_packed=w.gate_packed[lo:hi],
                              gate_absmax=w.gate_absmax[lo:hi], up_packed=w.up_packed[lo:hi],
                              up_absmax=w.up_absmax[lo:hi], down_packed=w.down_packed[lo:hi],
                              down_absmax=w.down_absmax[lo:hi], gate_code=w.gate_code, up_code=w.up_code,
                              down_code=w.down_code, layout=w.layout)
        parts.append(union_decode(_t(x, dev, torch.bfloat16), _t(idx, dev), ws, block_range=(lo, hi),
                                  out_dtype=torch.float32))
    for r in range(rows):
        _close((parts[0][r] + parts[1][r]).cpu().numpy(), ref[r])


def test_union_decode_rejects_bad_arguments(dev):
    from next_step_ai_b200 import union_decode

    shape, full, w = _layer("tiny", 23, dev)
    x = syn.make_x(shape, 1, 33)
    idx = np.zeros((33, shape.top_k), np.int32)
    with pytest.raises(RuntimeError):
        union_decode(_t(x, dev, torch.bfloat16), _t(idx, dev), w)
