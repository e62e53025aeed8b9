"""Learned-basis router oracle (numpy).  TEST INFRASTRUCTURE ONLY.

Restates ``StreamingLlamaRuntime._compute_sparse_basis_latent``
(``llama3_neuroplastic/experiments/streaming_llama_runtime.py:4209-4238``) and
``StreamingLlamaRuntime._route_sparse_mlp`` (``:4311-4352``).

Tie rule.  ``torch.topk`` leaves the order of equal scores unspecified; the
oracle (and the CUDA router) order by score descending, then by block index
ascending.  ``top_k_desc`` implements exactly that order.
"""
from __future__ import annotations

import numpy as np


def top_k_desc(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries per row: value desc, index asc."""
    v = np.asarray(values)
    if v.ndim == 1:
        return top_k_desc(v[None, :], k)[0]
    n = v.shape[-1]
    idx = np.broadcast_to(np.arange(n), v.shape)
    # lexsort sorts by the last key first: primary -value, secondary index.
    order = np.stack([np.lexsort((idx[r], -v[r].astype(np.float64))) for r in range(v.shape[0])])
    return order[:, :k].astype(np.int64)


def basis_latent(x: np.ndarray, enc_w: np.ndarray, enc_b: np.ndarray | None, basis_top_k: int,
                 dtype=np.float32) -> np.ndarray:
    """``latent = x @ enc_w.T + enc_b``; keep the ``basis_top_k`` largest
    ``|latent|`` entries per row when ``basis_top_k < rank``
    (``streaming_llama_runtime.py:4220-4238``)."""
    x2 = np.asarray(x, dtype=dtype).reshape(-1, enc_w.shape[1])
    lat = x2 @ np.asarray(enc_w, dtype=dtype).T
    if enc_b is not None:
        lat = lat + np.asarray(enc_b, dtype=dtype)[None, :]
    lat = lat.astype(dtype)
    rank = lat.shape[-1]
    if rank <= 0:
        return lat
    bk = max(1, min(int(basis_top_k), rank))
    if bk >= rank:
        return lat
    keep = top_k_desc(np.abs(lat), bk)
    mask = np.zeros_like(lat)
    np.put_along_axis(mask, keep, 1.0, axis=1)
    return (lat * mask).astype(dtype)


def block_scores(latent: np.ndarray, score_w: np.ndarray | None, score_b: np.ndarray | None,
                 dec_norm_t: np.ndarray | None = None, down_block_norm: np.ndarray | None = None,
                 dtype=np.float32) -> np.ndarray:
    """Block scores (``streaming_llama_runtime.py:4324-4337``).

    ``clamp_min(latent @ score_w.T + score_b, 0)`` when a learned score head
    exists, else the legacy ``|latent| @ dec_norm_t``; then multiplied by
    ``down_block_norm`` when one of length NB is present.
    """
    lat = np.asarray(latent, dtype=dtype)
    if score_w is not None:
        s = lat @ np.asarray(score_w, dtype=dtype).T
        if score_b is not None:
            s = s + np.asarray(score_b, dtype=dtype)[None, :]
        s = np.maximum(s.astype(dtype), dtype(0.0))
    else:
        s = np.abs(lat) @ np.asarray(dec_norm_t, dtype=dtype)
    s = s.astype(dtype)
    if down_block_norm is not None and np.asarray(down_block_norm).size == s.shape[-1]:
        s = (s * np.asarray(down_block_norm, dtype=dtype)[None, :]).astype(dtype)
    return s


def runtime_top_k(routing_top_k: int | None, sparse_runtime_top_k: int, sparse_top_k: int, num_blocks: int,
                  prefill_top_k: int | None = None) -> int:
    """k used by the router (``streaming_llama_runtime.py:4338-4350``)."""
    k = routing_top_k if routing_top_k is not None else (
        sparse_runtime_top_k if int(sparse_runtime_top_k) > 0 else sparse_top_k)
    if prefill_top_k is not None:
        k = int(prefill_top_k)
    return max(1, min(int(k), int(num_blocks)))


def route_sparse_mlp(hidden: np.ndarray, enc_w: np.ndarray, enc_b: np.ndarray | None,
                     score_w: np.ndarray | None, score_b: np.ndarray | None, top_k: int,
                     basis_top_k: int, *, dec_norm_t: np.ndarray | None = None,
                     down_block_norm: np.ndarray | None = None, dtype=np.float32) -> np.ndarray:
    """Selected block indices ``[N, k]`` (score desc, index asc) for ``hidden [..., H]``."""
    lat = basis_latent(hidden, enc_w, enc_b, basis_top_k, dtype=dtype)
    s = block_scores(lat, score_w, score_b, dec_norm_t=dec_norm_t, down_block_norm=down_block_norm, dtype=dtype)
    k = max(1, min(int(top_k), s.shape[-1]))
    return top_k_desc(s, k)


def selection_margin(hidden, enc_w, enc_b, score_w, score_b, top_k, basis_top_k, **kw) -> np.ndarray:
    """Relative gap between the k-th and (k+1)-th fp64 scores, per row.

    Used to classify a routing mismatch: a gap near fp32 rounding (~1e-6)
    means a near-tie, not a kernel bug.
    """
    lat = basis_latent(hidden, enc_w, enc_b, basis_top_k, dtype=np.float64)
    s = block_scores(lat, score_w, score_b, dtype=np.float64, **kw)
    srt = -np.sort(-s, axis=1)
    k = max(1, min(int(top_k), s.shape[-1]))
    if k >= s.shape[-1]:
        return np.full(s.shape[0], np.inf)
    top = np.maximum(np.abs(srt[:, k - 1]), 1e-30)
    return (srt[:, k - 1] - srt[:, k]) / top
