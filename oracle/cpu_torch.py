"""The reference's CPU torch path for one decode layer, restated in torch.
TEST INFRASTRUCTURE / CPU BASELINE ONLY -- never the product path.

Used by ``bench.py`` as the timed CPU arm (the reference runs this path in
torch on the host when no GPU kernel applies) and checked against the numpy
oracle by ``tests/test_oracle_golden.py``:

* router: ``latent = x @ enc_w.T + enc_b`` (``streaming_llama_runtime.py:4209-4238``),
  ``scores = clamp_min(latent @ score_w.T + score_b, 0)``, ``topk(k)``
  (``:4311-4352``), in fp32;
* MLP: the dequant fallback of ``_sparse_mlp_forward_fast`` (``:5433-5492``):
  gathered NF4 gate/up blocks dequantised as ``code[nibble] * absmax[e // 64]``
  (high nibble = even element), ``F.linear``, ``silu(g) * u``, the gathered
  down columns dequantised as at ``:5465-5483``, ``F.linear``.

Torch runs the elementwise dequant and the matmuls on all host threads, as
the reference's own torch code would.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def route(x: torch.Tensor, enc_w: torch.Tensor, enc_b: torch.Tensor | None, score_w: torch.Tensor,
          score_b: torch.Tensor | None, top_k: int) -> torch.Tensor:
    """Block ids ``[N, k]`` (score descending) for rows ``x [N, H]``."""
    lat = F.linear(x.float(), enc_w.float(), None if enc_b is None else enc_b.float())
    scores = F.linear(lat, score_w.float(), None if score_b is None else score_b.float()).clamp_min(0.0)
    k = max(1, min(int(top_k), scores.shape[-1]))
    return torch.topk(scores, k, dim=-1).indices


def dequant_rows(packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, qbs: int = 64) -> torch.Tensor:
    """Flat NF4 bytes -> fp32 elements (``code[nibble] * absmax[e // qbs]``)."""
    p = packed.reshape(-1)
    nib = torch.stack([p >> 4, p & 15], dim=-1).reshape(-1).long()
    return code.float()[nib].reshape(-1, qbs).mul_(absmax.float().reshape(-1, 1)).reshape(-1)


def mlp_gathered(x: torch.Tensor, gate_packed: torch.Tensor, gate_absmax: torch.Tensor, up_packed: torch.Tensor,
                 up_absmax: torch.Tensor, down_cols: torch.Tensor, down_absmax_cols: torch.Tensor,
                 code: torch.Tensor) -> torch.Tensor:
    """``y [N, H]`` of the MLP over the U gathered blocks.
    gate/up ``[U, 32*H/2]`` bytes + ``[U, 32*H/64]`` absmax; down ``[H, U, 16]``
    bytes + ``[H, U]`` absmax."""
    xf = x.float().reshape(-1, x.shape[-1])
    H = xf.shape[1]
    wg = dequant_rows(gate_packed, gate_absmax, code).reshape(-1, H)
    wu = dequant_rows(up_packed, up_absmax, code).reshape(-1, H)
    act = F.silu(F.linear(xf, wg)) * F.linear(xf, wu)
    U = down_cols.shape[1]
    p = down_cols.reshape(H, U, 16)
    nib = torch.stack([p >> 4, p & 15], dim=-1).reshape(H, U, 32).long()
    wd = (code.float()[nib] * down_absmax_cols.float().reshape(H, U, 1)).reshape(H, U * 32)
    return F.linear(act, wd)
