"""Oracle evaluation for GPU tests whose layers are generated on the device.

The weights of the large shapes are generated on the GPU
(``next_step_ai_b200.synthetic``) and kept there in the bitsandbytes row-major
layout next to the repacked pools.  These helpers copy only the selected
blocks' bytes back to the host -- the reference's gathers: gate/up rows
(``streaming_llama_runtime.py:4447-4452``) and down columns
(``:4497-4527``) -- and evaluate the numpy oracle (``oracle.mlp``, the fp32
dequant + matmul of ``:5433-5492``) and the oracle router on them.  Test
infrastructure only.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import mlp as om
from oracle import router as orr


def host_router(rw) -> dict:
    """A RouterWeights' tensors as fp32 numpy arrays (the oracle's inputs)."""
    return {k: (None if v is None else v.float().cpu().numpy()) for k, v in
            (("enc_w", rw.enc_w), ("enc_b", rw.enc_b), ("score_w", rw.score_w), ("score_b", rw.score_b))}


def oracle_route(R: dict, x: np.ndarray, top_k: int, rank: int) -> np.ndarray:
    """The oracle router's top-k of one row (score desc, ties to the lower id)."""
    return orr.route_sparse_mlp(np.asarray(x, np.float32), R["enc_w"], R["enc_b"], R["score_w"], R["score_b"],
                                top_k, rank)[0]


def gather_blocks(bnb: dict, hidden: int, intermediate: int, blocks) -> dict:
    """The selected blocks' NF4 bytes from device-resident bitsandbytes weights."""
    H, I = hidden, intermediate
    gm, dm = om.Nf4ParamMeta(I, H), om.Nf4ParamMeta(H, I)
    dev = bnb["gate_packed"].device
    s = torch.as_tensor(np.asarray(blocks, np.int64), device=dev)
    return {
        "gp": bnb["gate_packed"].view(-1, gm.bytes_per_block)[s].cpu().numpy(),
        "ga": bnb["gate_absmax"].view(-1, gm.absmax_per_block)[s].cpu().numpy(),
        "up": bnb["up_packed"].view(-1, gm.bytes_per_block)[s].cpu().numpy(),
        "ua": bnb["up_absmax"].view(-1, gm.absmax_per_block)[s].cpu().numpy(),
        "dc": bnb["down_packed"].view(H, dm.bytes_per_row).view(H, -1, 16)[:, s].contiguous().cpu().numpy(),
        "da": bnb["down_absmax"].view(H, dm.absmax_per_row)[:, s // 2].contiguous().cpu().numpy(),
        "code": bnb["code"].cpu().numpy(),
    }


def oracle_mlp(bnb: dict, hidden: int, intermediate: int, x, blocks) -> np.ndarray:
    """fp32 oracle MLP output ``[H]`` of one row ``x`` over ``blocks``."""
    if isinstance(x, torch.Tensor):
        x = x.float().cpu().numpy()
    g = gather_blocks(bnb, hidden, intermediate, blocks)
    c = g["code"]
    return om.sparse_mlp_gathered(np.asarray(x, np.float32).reshape(1, -1), g["gp"], g["ga"], c, g["up"], g["ua"],
                                  c, g["dc"], g["da"], c)[0]


def assert_close(got, ref, what: str = "", max_abs: float = 2e-2, rel_l2: float = 5e-3) -> None:
    """The decode tolerances on fp32 outputs: max-abs-err and relative L2."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    err = float(np.abs(got - ref).max())
    assert rel <= rel_l2, f"{what}: relative L2 {rel:.3e} > {rel_l2}"
    assert err <= max_abs, f"{what}: max abs err {err:.3e} > {max_abs}"


def oracle_mlp_rows(bnb: dict, hidden: int, intermediate: int, x: np.ndarray, ordered: np.ndarray,
                    flat_mask: np.ndarray, chunk: int = 64) -> np.ndarray:
    """fp32 oracle of the multi-row MLP over the union ``ordered`` with the
    reference's per-row ``flat_mask`` (``streaming_llama_runtime.py:5451-5492``),
    evaluated over chunks of union blocks so that only ``chunk`` blocks are
    dequantised at a time; the chunks' outputs are summed."""
    x = np.asarray(x, np.float32)
    y = np.zeros((x.shape[0], hidden), np.float64)
    for c0 in range(0, len(ordered), chunk):
        blk = np.asarray(ordered[c0:c0 + chunk], np.int64)
        g = gather_blocks(bnb, hidden, intermediate, blk)
        c = g["code"]
        m = flat_mask[:, c0 * 32:(c0 + blk.size) * 32]
        y += om.sparse_mlp_gathered(x, g["gp"], g["ga"], c, g["up"], g["ua"], c, g["dc"], g["da"], c,
                                    flat_mask=m).astype(np.float64)
    return y.astype(np.float32)
