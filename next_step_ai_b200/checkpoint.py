"""Loading the reference's on-disk artifacts into the decode path.

* ``load_router_artifact`` reads the learned-basis router artifact (the
  ``torch.save`` payload ``{config, layer_selection, layer_states, stats}``
  written by ``init_learned_basis_from_dense_mlp.py:350-397``) the way the
  reference runtime does for intermediate-domain layers
  (``streaming_llama_runtime.py:779-991``): per-layer ``RouterWeights`` with the
  same top-k / basis-top-k resolution, the same shape checks and the same
  ``RuntimeError`` messages.
* ``derive_hot_blocks`` restates ``_derive_hot_blocks_for_layer`` /
  ``_coerce_block_score_vector`` (``:1863-1972``): a layer's initial VRAM hot
  set from the artifact's block-importance scores.
* ``Nf4Checkpoint`` reads bitsandbytes-4bit safetensors checkpoints (the
  reference's ``ShardedSafetensorLoader``, ``runtime/safetensor_loader.py:73-475``,
  and ``_get_sparse_4bit_param``, ``streaming_llama_runtime.py:4580-4682``):
  packed bytes, the packed quant state, nested absmax statistics decoded to
  fp32, and per-layer ``SparseMlpWeights`` repacked on the GPU into the decode
  kernels' tiled layout.

Format facts this module depends on (bitsandbytes 0.49.1 serialisation,
``QuantState.as_dict(packed=True)`` / ``from_dict``; bitsandbytes is a third
party library, not vendored and not needed here):

* a 4-bit weight ``P.weight`` is a flat uint8 tensor (``[out*in/2, 1]``),
  element ``e = row*in + col`` in byte ``e // 2``, high nibble first;
* its quant state is stored beside it as ``P.weight.absmax``,
  ``P.weight.quant_map`` (16 fp32 code values) and
  ``P.weight.quant_state.bitsandbytes__nf4`` (or ``__fp4``): a uint8 tensor
  holding UTF-8 JSON with ``quant_type``, ``blocksize``, ``dtype``, ``shape`` and,
  for nested ("double-quantised") statistics, ``nested_blocksize``,
  ``nested_dtype``, ``nested_offset``;
* nested statistics add ``P.weight.nested_absmax`` (fp32, one per
  ``nested_blocksize`` absmax values) and ``P.weight.nested_quant_map``
  (256 fp32 values); the absmax tensor is then uint8 codes and the fp32 absmax
  is ``nested_quant_map[q] * nested_absmax[i // nested_blocksize] + nested_offset``
  (bitsandbytes' blockwise dequantisation plus the offset, as the reference
  applies it at ``streaming_llama_runtime.py:4621-4625``), computed in fp32.
"""
from __future__ import annotations

import json
import math
import warnings
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np
import torch

from .cache import hot_cache_bytes_per_block, target_hot_blocks
from .nf4 import Nf4ParamMeta
from .weights import RouterWeights, SparseMlpWeights

DEFAULT_SPARSE_BASIS_TOP_K = 8          # runtime/_helpers.py:52
DEFAULT_HOT_BLOCK_THRESHOLD = 0.80      # streaming_llama_runtime.py:167
MIN_EXPLAINED_VARIANCE = 0.30           # streaming_llama_runtime.py:836
QUANT_STATE_KEYS = ("bitsandbytes__nf4", "bitsandbytes__fp4")
_SCORE_VECTOR_KEYS = ("block_importance", "block_importance_probs", "_block_importance_probs", "block_scores",
                      "importance", "scores")


# --------------------------------------------------------------------------- router artifact
@dataclass
class LayerRouteInfo:
    """Per-layer facts the reference keeps in its routing dict next to the
    weights (``streaming_llama_runtime.py:954-976``)."""

    top_k: int
    basis_top_k: int
    basis_rank: int
    rank_effective: int
    explained_variance_ratio: float
    scale: float
    samples: float
    artifact_target: str
    block_domain: str
    num_blocks: int
    block_size: int


@dataclass
class RouterArtifact:
    block_size: int
    num_blocks: int
    top_k: int                                   # the runtime default (``_sparse_top_k``)
    layer_selection: set[int]
    layers: dict[int, RouterWeights] = field(default_factory=dict)
    info: dict[int, LayerRouteInfo] = field(default_factory=dict)
    hot_blocks: dict[int, np.ndarray] = field(default_factory=dict)
    output_domain_layers: list[int] = field(default_factory=list)
    low_evr_layers: list[int] = field(default_factory=list)


def _stat(state: dict, stats: Any, key: str, default: Any) -> Any:
    """``_coerce_sparse_layer_stat`` (``:1594-1609``): the layer state first,
    then the stats dict; a one-element tensor becomes its Python value."""
    for src in (state, stats if isinstance(stats, dict) else None):
        if src is not None and key in src:
            v = src.get(key)
            if torch.is_tensor(v) and int(v.numel()) == 1:
                return v.detach().cpu().reshape(-1)[0].item()
            return v
    return default


def _by_layer(table: dict, lidx: int, default: Any) -> Any:
    return table.get(str(lidx), table.get(lidx, default))


def load_router_artifact(source, *, hidden: int, intermediate: int, num_layers: int,
                         sparse_top_k: int | None = None, sparse_basis_top_k: int | None = None,
                         dtype: torch.dtype = torch.float16, device: torch.device | str = "cpu",
                         hot_blocks: bool = False, hot_block_threshold: float = DEFAULT_HOT_BLOCK_THRESHOLD,
                         hot_cache_limit_bytes: int | None = None, hot_cache_used_bytes: int = 0,
                         trusted: bool = False) -> RouterArtifact:
    """Read a router artifact (a path or an already-loaded payload dict).

    Mirrors the reference's constructor (``streaming_llama_runtime.py:779-991``):
    the default top-k is ``max(1, round(0.02 * num_blocks))`` unless
    ``sparse_top_k`` is given; per-layer overrides come from
    ``config.top_k_by_layer`` / ``basis_top_k_by_layer`` (string or int keys);
    top-k is clamped to ``[1, NB]`` and basis top-k to ``[1, rank_effective]``.
    Weights are cast to ``dtype`` (the runtime's, fp16 by default);
    ``down_block_norm`` stays fp32.  Output-domain layers (the older
    ``decoder_blocks`` artifacts) belong to a different execution mode and are
    listed in ``output_domain_layers`` without weights.  With ``hot_blocks``,
    each layer's initial hot set is derived as the reference does when its VRAM
    hot cache is enabled (``:979-990``), counting the layers loaded so far
    (output-domain ones included) as the sparse layers of the capacity
    formula, as the reference does while it fills its routing table; output-
    domain layers get no hot set here (their execution mode is not this path).

    A file is read with torch's restricted unpickler (tensors, containers and
    numbers: everything the artifact schema holds); ``trusted=True`` allows
    arbitrary pickled objects, as the reference's ``weights_only=False`` load
    does, and should only be used for files from a trusted source.
    """
    if isinstance(source, dict):
        payload = source
    else:
        try:
            payload = torch.load(str(source), map_location="cpu", weights_only=not trusted)
        except Exception as e:
            if trusted:
                raise
            raise RuntimeError(f"{source}: not loadable with the restricted unpickler ({type(e).__name__}: {e}); "
                               "pass trusted=True for an artifact from a trusted source") from e
    cfg = payload.get("config", {}) or {}
    raw_sel = payload.get("layer_selection", [])
    selection = {int(i) for i in raw_sel if 0 <= int(i) < num_layers} if isinstance(raw_sel, (list, tuple)) else set()
    block_size = int(cfg.get("block_size", 32))
    target_default = str(cfg.get("artifact_target", "output_reconstruction")).strip().lower()
    domain_default = str(cfg.get("block_domain", "intermediate" if target_default == "intermediate_block_scores"
                                 else "output")).strip().lower()
    nb_default = (hidden if domain_default == "output" else intermediate) // max(block_size, 1)
    num_blocks = int(cfg.get("num_blocks", nb_default))
    default_top_k = int(sparse_top_k) if sparse_top_k is not None else max(1, int(round(max(1, num_blocks) * 0.02)))
    states = payload.get("layer_states", {}) or {}
    stats = payload.get("stats", {}) or {}
    top_k_by_layer = cfg.get("top_k_by_layer", {}) or {}
    basis_top_k_by_layer = cfg.get("basis_top_k_by_layer", {}) or {}
    default_basis_top_k = int(sparse_basis_top_k) if sparse_basis_top_k is not None \
        else int(cfg.get("basis_top_k", DEFAULT_SPARSE_BASIS_TOP_K))
    importance_by_layer = {}
    if isinstance(stats, dict) and isinstance(stats.get("block_importance_by_layer"), dict):
        importance_by_layer = stats["block_importance_by_layer"]
    out = RouterArtifact(block_size=block_size, num_blocks=num_blocks, top_k=default_top_k,
                         layer_selection=selection)
    for key, state in states.items():
        lidx = int(key)
        if not 0 <= lidx < num_layers:
            continue
        lstats = stats.get(str(lidx), {}) if isinstance(stats, dict) else {}
        target = str(state.get("artifact_target", cfg.get("artifact_target", target_default))).strip().lower()
        domain = str(state.get("block_domain", cfg.get(
            "block_domain", "intermediate" if target == "intermediate_block_scores" else domain_default))).strip().lower()
        if domain != "intermediate":
            out.output_domain_layers.append(lidx)
            continue
        enc_w = state["encoder_weight"].to(device=device, dtype=dtype).contiguous()
        enc_b = state["encoder_bias"].to(device=device, dtype=dtype).contiguous()
        rank = int(enc_w.shape[0])
        if int(enc_w.shape[1]) != int(hidden):
            raise RuntimeError(f"Sparse intermediate-router layer {lidx}: encoder_weight has input dim "
                               f"{int(enc_w.shape[1])}, expected hidden_size={int(hidden)}.")
        rank_eff = int(max(1, min(int(_stat(state, lstats, "rank_effective", rank)), rank)))
        evr = float(_stat(state, lstats, "explained_variance_ratio", 1.0))
        if evr < MIN_EXPLAINED_VARIANCE:
            out.low_evr_layers.append(lidx)
            warnings.warn(f"[sparse_basis] Layer {lidx} explained_variance_ratio={evr:.3f} < "
                          f"{MIN_EXPLAINED_VARIANCE:.2f}. The intermediate router may have poor recall.",
                          RuntimeWarning, stacklevel=2)
        sw_raw = state.get("score_weight")
        if not torch.is_tensor(sw_raw):
            raise RuntimeError(f"Sparse intermediate-router layer {lidx} is missing score_weight.")
        score_w = sw_raw.to(device=device, dtype=dtype).contiguous()
        if score_w.ndim != 2 or int(score_w.shape[1]) != rank:
            raise RuntimeError(f"Sparse intermediate-router layer {lidx}: score_weight shape "
                               f"{tuple(score_w.shape)} does not match basis_rank={rank}.")
        nb = int(score_w.shape[0])
        expected_nb = int(intermediate) // block_size
        if nb != expected_nb:
            raise RuntimeError(f"Sparse intermediate-router layer {lidx} stores {nb} FFN blocks, "
                               f"expected {expected_nb}.")
        score_b = None
        if torch.is_tensor(state.get("score_bias")):
            score_b = state["score_bias"].to(device=device, dtype=dtype).contiguous().view(-1)
            if int(score_b.numel()) != nb:
                raise RuntimeError(f"Sparse intermediate-router layer {lidx}: score_bias has "
                                   f"{int(score_b.numel())} values, expected {nb}.")
        dbn = None
        if torch.is_tensor(state.get("down_block_norm")):
            dbn = state["down_block_norm"].to(device="cpu", dtype=torch.float32).contiguous().view(-1)
            if int(dbn.numel()) != nb:
                raise RuntimeError(f"Sparse intermediate-router layer {lidx}: down_block_norm has "
                                   f"{int(dbn.numel())} values, expected {nb}.")
            dbn = dbn.to(device)
        top_k = int(max(1, min(int(_by_layer(top_k_by_layer, lidx, default_top_k)), nb)))
        btk = int(sparse_basis_top_k) if sparse_basis_top_k is not None \
            else int(_by_layer(basis_top_k_by_layer, lidx, default_basis_top_k))
        btk = int(max(1, min(btk, rank_eff)))
        scale = state.get("scale")
        out.layers[lidx] = RouterWeights(enc_w=enc_w, enc_b=enc_b, score_w=score_w, score_b=score_b,
                                         down_block_norm=dbn, top_k=top_k, basis_top_k=btk)
        out.info[lidx] = LayerRouteInfo(
            top_k=top_k, basis_top_k=btk, basis_rank=rank, rank_effective=rank_eff, explained_variance_ratio=evr,
            scale=float(scale.item()) if torch.is_tensor(scale) and int(scale.numel()) == 1 else 1.0,
            samples=float(_stat(state, lstats, "samples", -1.0)), artifact_target=target, block_domain=domain,
            num_blocks=nb, block_size=block_size)
        if hot_blocks:
            hb = derive_hot_blocks(
                state, lstats, importance_by_layer.get(str(lidx)), nb, runtime_top_k=default_top_k,
                threshold=hot_block_threshold, limit_bytes=hot_cache_limit_bytes, used_bytes=hot_cache_used_bytes,
                sparse_layers=len(out.layers) + len(out.output_domain_layers),
                bytes_per_block=hot_cache_bytes_per_block(hidden, block_size))
            if hb is not None and hb.size > 0:
                out.hot_blocks[lidx] = hb
    return out


def coerce_block_score_vector(value: Any, num_blocks: int) -> np.ndarray | None:
    """A length-``num_blocks`` fp32 score vector from a tensor, a list, or a
    dict (nested score keys first, else ``{block_id: score}``); truncated or
    zero-padded (``_coerce_block_score_vector``, ``:1863-1908``)."""
    if value is None:
        return None
    vec = None
    if torch.is_tensor(value):
        vec = value.detach().flatten().to(device="cpu", dtype=torch.float32).numpy()
    elif isinstance(value, (list, tuple)):
        if len(value) == 0:
            return None
        vec = np.asarray(value, dtype=np.float32).reshape(-1)
    elif isinstance(value, dict):
        for key in _SCORE_VECTOR_KEYS:
            if key in value:
                nested = coerce_block_score_vector(value[key], num_blocks)
                if nested is not None:
                    return nested
        tmp = np.zeros(num_blocks, np.float32)
        found = False
        for key, raw in value.items():
            try:
                i = int(key)
            except Exception:
                continue
            if not 0 <= i < num_blocks:
                continue
            try:
                tmp[i] = float(raw)
                found = True
            except Exception:
                continue
        if found:
            vec = tmp
    if vec is None:
        return None
    if vec.size >= num_blocks:
        return np.ascontiguousarray(vec[:num_blocks], np.float32)
    pad = np.zeros(num_blocks, np.float32)
    pad[:vec.size] = vec
    return pad


def hot_block_scores(state: dict, layer_stats: Any, importance: Any, num_blocks: int) -> np.ndarray | None:
    """The score vector ``derive_hot_blocks`` ranks: the first usable one among
    the state's ``block_importance`` / ``block_importance_probs`` /
    ``_block_importance_probs``, the layer's stats and
    ``stats.block_importance_by_layer``; else the mean absolute decoder bias /
    blocks (``:1918-1944``)."""
    scores = None
    for cand in (state.get("block_importance"), state.get("block_importance_probs"),
                 state.get("_block_importance_probs"), layer_stats, importance):
        v = coerce_block_score_vector(cand, num_blocks)
        if v is not None and v.size == num_blocks:
            scores = v
            break
    if scores is None:
        db = state.get("decoder_bias")
        blocks = state.get("decoder_blocks")
        if torch.is_tensor(db) and db.ndim == 2:
            scores = db.detach().abs().mean(dim=-1).to(torch.float32).cpu().numpy()
        elif torch.is_tensor(blocks) and blocks.ndim >= 2:
            scores = blocks.detach().abs().mean(dim=tuple(range(1, blocks.ndim))).to(torch.float32).cpu().numpy()
    if scores is None or scores.size == 0:
        return None
    return np.ascontiguousarray(scores[:num_blocks], np.float32)


def derive_hot_blocks(state: dict, layer_stats: Any, importance: Any, num_blocks: int, *, runtime_top_k: int,
                      threshold: float = DEFAULT_HOT_BLOCK_THRESHOLD, limit_bytes: int | None = None,
                      used_bytes: int = 0, sparse_layers: int = 1,
                      bytes_per_block: int = 1_048_576) -> np.ndarray | None:
    """A layer's initial hot blocks, ascending (``_derive_hot_blocks_for_layer``,
    ``:1910-1972``) from ``hot_block_scores``.  Blocks scoring at least
    ``threshold`` of the maximum are kept if there are exactly as many as the
    layer's hot capacity, otherwise the capacity's top scores: ties at the
    capacity boundary go to the lower block ids here, while the reference's
    ``torch.topk`` leaves them unspecified.  All scores <= 0 keep blocks
    ``[0, capacity)``."""
    thr = float(max(0.0, min(1.0, threshold)))
    scores = hot_block_scores(state, layer_stats, importance, num_blocks)
    if scores is None:
        return None
    s_max = float(scores.max())
    layer_idx = int(state.get("layer_idx", -1))
    rtk = int(state.get("top_k", runtime_top_k))
    cap = target_hot_blocks(layer_idx=layer_idx, runtime_top_k=rtk, count_slots=num_blocks, previous_hot_count=0,
                            limit_bytes=limit_bytes, used_bytes=used_bytes, sparse_layers=sparse_layers,
                            bytes_per_block=bytes_per_block)
    if s_max <= 0.0:
        return np.arange(cap, dtype=np.int64)
    norm = scores / np.float32(max(s_max, 1e-8))
    hot = np.nonzero(norm >= np.float32(thr))[0]
    if hot.size != cap:
        hot = np.argsort(-norm, kind="stable")[:cap]
    return np.sort(hot).astype(np.int64)


# --------------------------------------------------------------------------- bitsandbytes checkpoints
@dataclass
class Nf4Param:
    """One 4-bit weight as the reference's ``_get_sparse_4bit_param`` sees it."""

    name: str
    packed: torch.Tensor        # flat uint8, out*in/2 bytes, row-major, high nibble first
    absmax: torch.Tensor        # fp32, out*in/blocksize
    code: torch.Tensor          # fp32 [16]
    out_features: int
    in_features: int
    blocksize: int
    quant_type: str
    dtype: str

    def meta(self, block_size: int = 32) -> Nf4ParamMeta:
        return Nf4ParamMeta(self.out_features, self.in_features, block_size=block_size,
                            quant_block_size=self.blocksize, quant_type=self.quant_type)


def decode_quant_state(aux: dict[str, torch.Tensor], name: str = "") -> dict[str, Any]:
    """The packed quant state of one weight: its JSON fields plus the tensors
    under their last name component; nested statistics decoded into an fp32
    ``absmax``."""
    qs_keys = [k for k, v in aux.items() if "quant_state" in k and torch.is_tensor(v)]
    if len(qs_keys) != 1 or qs_keys[0].split(".")[-1] not in QUANT_STATE_KEYS:
        raise RuntimeError(f"{name}: expected one packed bitsandbytes 4-bit quant state, found {sorted(aux)}")
    blob = aux[qs_keys[0]].detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()
    try:
        fields = json.loads(blob.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise RuntimeError(f"{name}: malformed quant state ({e})") from None
    qs = dict(fields)
    for k, v in aux.items():
        if k != qs_keys[0]:
            qs[k.split(".")[-1]] = v
    for req in ("absmax", "quant_map", "blocksize", "shape", "quant_type"):
        if req not in qs:
            raise RuntimeError(f"{name}: quant state lacks '{req}'")
    absmax = qs["absmax"].detach().cpu()
    if "nested_absmax" in qs:
        q = absmax.contiguous().view(torch.uint8).numpy().reshape(-1).astype(np.int64)
        code2 = qs["nested_quant_map"].detach().cpu().to(torch.float32).numpy().reshape(-1)
        am2 = qs["nested_absmax"].detach().cpu().to(torch.float32).numpy().reshape(-1)
        nbs = int(qs.get("nested_blocksize", 256))
        if q.size and (q.max() >= code2.size or (q.size - 1) // nbs >= am2.size):
            raise RuntimeError(f"{name}: nested absmax statistics do not cover {q.size} values")
        deq = (code2[q] * am2[np.arange(q.size) // nbs]).astype(np.float32)
        deq = (deq + np.float32(float(qs.get("nested_offset", 0.0)))).astype(np.float32)
        qs["absmax"] = torch.from_numpy(deq)
    else:
        qs["absmax"] = absmax.to(torch.float32).reshape(-1).contiguous()
    return qs


class Nf4Checkpoint:
    """Read access to a bitsandbytes-4bit safetensors snapshot directory.

    The tensor -> shard map comes from ``model.safetensors.index.json``; without
    an index the first ``*.safetensors`` file (sorted by name) is the whole map,
    as in the reference loader (``runtime/safetensor_loader.py:74-98``).  Quant
    state tensors ``P.weight.<aux>`` are grouped under ``P.weight``."""

    def __init__(self, snapshot_dir) -> None:
        from safetensors import safe_open  # noqa: F401  (fail here, not mid-load)
        self.snapshot_dir = Path(snapshot_dir)
        index = self.snapshot_dir / "model.safetensors.index.json"
        self.weight_map: dict[str, str] = {}
        if index.exists():
            raw = json.loads(index.read_text(encoding="utf-8")).get("weight_map", {})
            self.weight_map = {str(k): str(v) for k, v in raw.items()}
        else:
            files = sorted(self.snapshot_dir.glob("*.safetensors"))
            if not files:
                raise RuntimeError(f"No safetensors shards found in {self.snapshot_dir}")
            with safe_open(str(files[0]), framework="pt", device="cpu") as h:
                self.weight_map = {str(n): files[0].name for n in h.keys()}
        self.aux_names: dict[str, list[str]] = {}
        for n in self.weight_map:
            if ".weight." in n:
                self.aux_names.setdefault(n.split(".weight.", 1)[0] + ".weight", []).append(n)
        self._handles: dict[str, Any] = {}
        self._headers: dict[str, tuple[int, dict]] = {}

    def close(self) -> None:
        """Release the open shard handles (reopened on the next read)."""
        self._handles.clear()

    def __enter__(self) -> "Nf4Checkpoint":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def _tensors(self, names) -> dict[str, torch.Tensor]:
        from safetensors import safe_open
        out = {}
        for n in names:
            shard = self.weight_map.get(n)
            if shard is None:
                continue
            h = self._handles.get(shard)
            if h is None:
                h = self._handles[shard] = safe_open(str(self.snapshot_dir / shard), framework="pt", device="cpu")
            out[n] = h.get_tensor(n)
        return out

    def load_raw(self, name: str) -> tuple[torch.Tensor, dict[str, torch.Tensor]]:
        """(weight bytes, quant-state tensors) of one parameter."""
        t = self._tensors([name, *self.aux_names.get(name, [])])
        if name not in t:
            raise KeyError(f"Tensor '{name}' not found in safetensors index")
        w = t.pop(name)
        return w, t

    def load_param(self, name: str) -> Nf4Param:
        w, aux = self.load_raw(name)
        if not aux:
            raise RuntimeError(f"Sparse 4-bit path expected quantized weights for {name}")
        qs = decode_quant_state(aux, name)
        shape = [int(s) for s in qs["shape"]]
        if len(shape) != 2:
            raise RuntimeError(f"{name}: 4-bit weight shape {shape} is not 2-D")
        out_f, in_f = shape
        bs = int(qs["blocksize"])
        packed = w.detach().contiguous().view(torch.uint8).reshape(-1)
        if packed.numel() * 2 < out_f * in_f:
            raise RuntimeError(f"{name}: {packed.numel()} packed bytes for a [{out_f}, {in_f}] weight")
        code = qs["quant_map"].detach().cpu().to(torch.float32).reshape(-1).contiguous()
        if code.numel() != 16:
            raise RuntimeError(f"{name}: quant_map has {code.numel()} entries, expected 16")
        absmax = qs["absmax"]
        if absmax.numel() != math.ceil(out_f * in_f / bs):
            raise RuntimeError(f"{name}: {absmax.numel()} absmax values for a [{out_f}, {in_f}] weight "
                               f"with blocksize {bs}")
        return Nf4Param(name=name, packed=packed[: out_f * in_f // 2], absmax=absmax, code=code,
                        out_features=out_f, in_features=in_f, blocksize=bs, quant_type=str(qs["quant_type"]),
                        dtype=str(qs.get("dtype", "")))

    def _tensor_extent(self, name: str) -> tuple[Path, int, int]:
        """(shard path, absolute byte offset, byte length) of a tensor's data,
        from the shard's safetensors header (8-byte little-endian header size,
        JSON header, then the data block)."""
        shard = self.weight_map.get(name)
        if shard is None:
            raise KeyError(f"Tensor '{name}' not found in safetensors index")
        hdr = self._headers.get(shard)
        if hdr is None:
            path = self.snapshot_dir / shard
            with open(path, "rb") as f:
                n = int.from_bytes(f.read(8), "little")
                hdr = self._headers[shard] = (8 + n, json.loads(f.read(n).decode("utf-8")))
        base, meta = hdr
        ent = meta.get(name)
        if not isinstance(ent, dict):
            raise KeyError(f"Tensor '{name}' metadata missing from safetensors header")
        start, end = (int(v) for v in ent["data_offsets"])
        return self.snapshot_dir / shard, base + start, end - start

    def load_nf4_packed_blocks(self, name: str, block_indices, *, bytes_per_block: int) -> torch.Tensor:
        """``[n, bytes_per_block]`` uint8 rows of the flat weight, in the order
        given (``ShardedSafetensorLoader.load_nf4_packed_blocks``,
        ``runtime/safetensor_loader.py:291-350``).  Only the listed blocks are
        read: sorted block ids are read as runs of consecutive blocks with one
        seek each (the reference's direct path), then put back in the given
        order."""
        bpb = int(bytes_per_block)
        idx = torch.as_tensor(block_indices, dtype=torch.long).reshape(-1)
        path, off, nbytes = self._tensor_extent(name)
        if bpb <= 0 or nbytes % bpb:
            raise RuntimeError(f"{name}: {nbytes} bytes are not a whole number of {bpb}-byte blocks")
        nblk = nbytes // bpb
        if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= nblk):
            raise IndexError(f"block index out of range for '{name}' with {nblk} blocks")
        out = torch.empty((idx.numel(), bpb), dtype=torch.uint8)
        if idx.numel() == 0:
            return out
        order = torch.argsort(idx, stable=True)
        srt = idx[order].tolist()
        buf = out.numpy()
        with open(path, "rb") as f:
            i = 0
            while i < len(srt):
                j = i + 1
                while j < len(srt) and srt[j] == srt[j - 1] + 1:
                    j += 1
                f.seek(off + srt[i] * bpb)
                run = f.read((j - i) * bpb)
                if len(run) != (j - i) * bpb:
                    raise RuntimeError(f"{name}: short read at block {srt[i]}")
                chunk = np.frombuffer(run, dtype=np.uint8).reshape(j - i, bpb)
                for k in range(i, j):
                    buf[int(order[k])] = chunk[k - i]
                i = j
        return out

    def mlp_params(self, layer_idx: int, prefix: str | None = None) -> dict[str, Nf4Param]:
        p = prefix if prefix is not None else f"model.layers.{int(layer_idx)}.mlp."
        return {proj: self.load_param(f"{p}{proj}_proj.weight") for proj in ("gate", "up", "down")}

    def layer_weights(self, layer_idx: int, *, device: torch.device | str = "cuda", prefix: str | None = None,
                      tiled: bool = True, block_size: int = 32) -> SparseMlpWeights:
        """One decoder layer's MLP as device ``SparseMlpWeights``: the whole NF4
        weights are copied to ``device`` and repacked there by the library's
        repack kernels (``tiled``: the decode kernels' lane-interleaved layout)."""
        ps = self.mlp_params(layer_idx, prefix)
        g, u, d = ps["gate"], ps["up"], ps["down"]
        H, I = g.in_features, g.out_features
        if (u.out_features, u.in_features) != (I, H) or (d.out_features, d.in_features) != (H, I):
            raise RuntimeError(f"layer {layer_idx}: gate {g.out_features}x{g.in_features}, up "
                               f"{u.out_features}x{u.in_features}, down {d.out_features}x{d.in_features} "
                               "do not form an MLP")
        if block_size != 32 or I % block_size:
            raise RuntimeError(f"layer {layer_idx}: intermediate {I} must be a multiple of the block size 32")
        for p in (g, u, d):
            if p.blocksize != 64:
                raise RuntimeError(f"{p.name}: quant blocksize {p.blocksize} unsupported (the kernels read 64)")
        dev = torch.device(device)

        def put(t):
            return t.to(dev, non_blocking=False).contiguous()

        return SparseMlpWeights.from_bnb_rowmajor(
            hidden=H, intermediate=I, gate_packed=put(g.packed), gate_absmax=put(g.absmax),
            up_packed=put(u.packed), up_absmax=put(u.absmax), down_packed=put(d.packed),
            down_absmax=put(d.absmax), code=g.code, up_code=u.code, down_code=d.code, tiled=tiled)
