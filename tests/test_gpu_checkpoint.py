"""A bitsandbytes-4bit checkpoint and a router artifact on disk, loaded by
``next_step_ai_b200.checkpoint`` and decoded on the GPU: the selected blocks
are bit-exact against the oracle router, and the output is within the MLP
tolerance of the fp32 oracle evaluated on the bytes and the nested-statistics
absmax the loader decoded (what the reference computes from the same files)."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytest.importorskip("safetensors")

pytestmark = pytest.mark.gpu

from oracle import bnb_checkpoint as bc  # noqa: E402
from oracle import mlp as om  # noqa: E402
from oracle import router as orr  # noqa: E402
from oracle import synthetic as syn  # noqa: E402

from tests.test_gpu_decode import T, assert_close  # noqa: E402


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from next_step_ai_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


@pytest.mark.parametrize("tiled", [True, False])
def test_checkpoint_layer_decodes_like_oracle(dev, tmp_path, tiled):
    from next_step_ai_b200 import sparse_mlp_decode
    from next_step_ai_b200.checkpoint import Nf4Checkpoint, load_router_artifact

    shape, seed, layer = syn.SHAPES["small"], 23, 2
    full = syn.make_layer_full(shape, seed, layer)
    bc.write_snapshot(tmp_path, bc.layer_params(full, shape.hidden, shape.intermediate, layer), shards=2)
    R = syn.make_router(shape, seed, layer)
    payload = {"config": {"artifact_target": "intermediate_block_scores", "block_size": 32,
                          "num_blocks": shape.num_blocks, "basis_rank": shape.rank, "basis_top_k": shape.rank,
                          "top_k_by_layer": {str(layer): shape.top_k}},
               "layer_selection": [layer],
               "layer_states": {str(layer): {"encoder_weight": torch.from_numpy(R["enc_w"]),
                                             "encoder_bias": torch.from_numpy(R["enc_b"]),
                                             "score_weight": torch.from_numpy(R["score_w"]),
                                             "score_bias": torch.from_numpy(R["score_b"])}}}
    torch.save(payload, tmp_path / "router.pt")
    art = load_router_artifact(tmp_path / "router.pt", hidden=shape.hidden, intermediate=shape.intermediate,
                               num_layers=4, dtype=torch.bfloat16, device=dev)
    rw = art.layers[layer]
    ckpt = Nf4Checkpoint(tmp_path)
    w = ckpt.layer_weights(layer, device=dev, tiled=tiled)
    ps = ckpt.mlp_params(layer)
    args = [ps["gate"].packed.numpy(), ps["gate"].absmax.numpy(), ps["up"].packed.numpy(), ps["up"].absmax.numpy(),
            ps["down"].packed.numpy(), ps["down"].absmax.numpy(), full["code"]]
    for rowseed in range(2):
        x = syn.make_x(shape, seed * 10 + rowseed, 1)[0]
        idx = torch.empty(shape.top_k, dtype=torch.int32, device=dev)
        y = sparse_mlp_decode(T(x, dev, torch.bfloat16), rw, w, out_dtype=torch.float32, idx_out=idx)
        ref_idx = orr.route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k,
                                       shape.rank)[0]
        assert np.array_equal(idx.cpu().numpy(), ref_idx)
        ref = om.sparse_mlp_full(x, ref_idx, *args, hidden=shape.hidden, intermediate=shape.intermediate)[0]
        assert_close(y.cpu().numpy(), ref)
