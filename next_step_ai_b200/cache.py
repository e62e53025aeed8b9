"""VRAM hot-block cache for the decode MLP, with misses streamed from pinned host memory.

Reference behaviour (``llama3_neuroplastic/experiments/streaming_llama_runtime.py``):
a per-layer VRAM bank of hot blocks addressed by a block -> slot table
(``:2619-2786``); blocks the router selects that are not resident are copied
from pinned host memory on a side stream (``_copy_cpu_to_gpu``, ``:3443-3493``;
cold loads ``:3885-4002``) and merged with the resident ones; after use, the
misses are promoted into the bank by the fixed-capacity policy
``_plan_fixed_capacity_bank_update`` (``:2577-2617``) -- free slots first, then
the lowest score; a novel block gets ``max(active scores) + 1 + (i+1)*1e-3`` --
and every decode hit adds 1 to the hit block's score (``:5262-5271``).  The
initial bank of ``n`` pre-warmed blocks is scored ``linspace(n, 1)``
(``:2699-2706``).

Design here:

* one device pool of ``capacity + staging`` block *records*; a record holds
  all of one block's bytes in the tiled layout (gate, up and down packed, then
  their fp32 absmax: 56*H bytes, the per-block algorithmic bytes), so a miss is
  ONE contiguous ``cudaMemcpyAsync`` and the decode kernels read bank and
  staging rows through the same strided descriptor;
* a pinned host store with every block of the layer in the same record layout;
* per token: route on the main stream, read the selection back, stage the
  misses on a side stream (``nsm_cache_stage``) while the main stream computes
  the resident blocks (the block map drops the misses), then compute the staged
  blocks and add the two partial outputs;
* promotion after the token: the bank policy picks the slots on the host, the
  staged records are copied device-to-device into them and the block table is
  rewritten.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._torch import WORKSPACES, dtype_code, stream_handle
from .weights import RouterWeights, SparseMlpWeights


# --------------------------------------------------------------------------- record layout
def record_layout(hidden: int) -> dict[str, tuple[int, int]]:
    """Byte (offset, size) of each part of one block record (tiled layout)."""
    H = int(hidden)
    g = 16 * H  # 32 rows x H/2 bytes
    return {"gate": (0, g), "up": (g, g), "down": (2 * g, g),
            "gate_absmax": (3 * g, 2 * H), "up_absmax": (3 * g + 2 * H, 2 * H), "down_absmax": (3 * g + 4 * H, 4 * H)}


def record_bytes(hidden: int) -> int:
    return 56 * int(hidden)


def pool_weights(pool: torch.Tensor, hidden: int, intermediate: int, gate_code: torch.Tensor,
                 up_code: torch.Tensor, down_code: torch.Tensor) -> SparseMlpWeights:
    """Decode-kernel view of a record pool ``[P, 56*H]`` uint8 (rows strided by the record)."""
    H = int(hidden)
    lay = record_layout(H)

    def part(name, dtype=torch.uint8):
        o, n = lay[name]
        v = pool[:, o:o + n]
        return v.view(dtype) if dtype != torch.uint8 else v

    return SparseMlpWeights(hidden=H, intermediate=int(intermediate), gate_packed=part("gate"),
                            gate_absmax=part("gate_absmax", torch.float32), up_packed=part("up"),
                            up_absmax=part("up_absmax", torch.float32),
                            down_packed=part("down").view(pool.shape[0], H, 16),
                            down_absmax=part("down_absmax", torch.float32), gate_code=gate_code, up_code=up_code,
                            down_code=down_code,
                            layout=_lib.NSM_LAYOUT_GATEUP_TILED | _lib.NSM_LAYOUT_DOWN_TILED)


def records_from_weights(w: SparseMlpWeights, blocks: torch.Tensor | None = None) -> torch.Tensor:
    """Device records ``[n, 56*H]`` of the listed blocks (all when None) of a
    full tiled layer."""
    if w.layout != (_lib.NSM_LAYOUT_GATEUP_TILED | _lib.NSM_LAYOUT_DOWN_TILED):
        raise RuntimeError("records are built from tiled gate/up and down pools")
    H = w.hidden
    idx = torch.arange(w.pool_rows, device=w.gate_packed.device) if blocks is None else blocks.to(torch.int64)
    out = torch.empty((idx.numel(), record_bytes(H)), dtype=torch.uint8, device=w.gate_packed.device)
    lay = record_layout(H)
    for name, src in (("gate", w.gate_packed), ("up", w.up_packed), ("down", w.down_packed),
                      ("gate_absmax", w.gate_absmax), ("up_absmax", w.up_absmax), ("down_absmax", w.down_absmax)):
        o, n = lay[name]
        out[:, o:o + n].copy_(src.reshape(src.shape[0], -1).index_select(0, idx).view(torch.uint8))
    return out


class HostBlockStore:
    """Every block of one layer in pinned host memory, one record per block."""

    def __init__(self, records: torch.Tensor, hidden: int, intermediate: int, gate_code: torch.Tensor,
                 up_code: torch.Tensor, down_code: torch.Tensor):
        if records.device.type != "cpu" or not records.is_pinned():
            raise RuntimeError("the host block store must be pinned host memory")
        if records.dtype != torch.uint8 or records.shape[1] != record_bytes(hidden) or not records.is_contiguous():
            raise RuntimeError("records must be contiguous uint8 [NB, 56*H]")
        self.records = records
        self.hidden, self.intermediate = int(hidden), int(intermediate)
        self.codes = (gate_code, up_code, down_code)

    @property
    def num_blocks(self) -> int:
        return int(self.records.shape[0])

    @classmethod
    def from_weights(cls, w: SparseMlpWeights, chunk: int = 128) -> "HostBlockStore":
        nb = w.pool_rows
        host = torch.empty((nb, record_bytes(w.hidden)), dtype=torch.uint8, pin_memory=True)
        for b0 in range(0, nb, chunk):
            ids = torch.arange(b0, min(nb, b0 + chunk), device=w.gate_packed.device)
            host[b0:b0 + ids.numel()].copy_(records_from_weights(w, ids))
        return cls(host, w.hidden, w.intermediate, w.gate_code, w.up_code, w.down_code)


# --------------------------------------------------------------------------- bank policy
class FixedCapacityBank:
    """Host-side state and replacement policy of a fixed-capacity block bank.

    ``block_ids[slot]`` / ``scores[slot]`` for the first ``active`` slots; the
    policy is the reference's ``_plan_fixed_capacity_bank_update``
    (``streaming_llama_runtime.py:2577-2617``) and hit scoring (``:5262-5271``).
    """

    def __init__(self, capacity: int):
        self.capacity = int(capacity)
        self.block_ids = np.full(self.capacity, -1, np.int64)
        self.scores = np.zeros(self.capacity, np.float32)
        self.active = 0

    @classmethod
    def from_state(cls, block_ids, scores, active: int, capacity: int | None = None) -> "FixedCapacityBank":
        ids = np.asarray(block_ids, np.int64).reshape(-1)
        cap = int(capacity) if capacity is not None else ids.size
        bank = cls(cap)
        n = min(ids.size, cap)
        bank.block_ids[:n] = ids[:n]
        bank.scores[:n] = np.asarray(scores, np.float32).reshape(-1)[:n]
        bank.active = max(0, min(int(active), n, cap))
        return bank

    def prewarm(self, blocks) -> None:
        b = np.asarray(blocks, np.int64).reshape(-1)[: self.capacity]
        n = b.size
        self.block_ids[:] = -1
        self.block_ids[:n] = b
        self.scores[:] = 0
        if n:
            self.scores[:n] = np.linspace(float(n), 1.0, n, dtype=np.float32)
        self.active = n

    def add_hits(self, slots) -> None:
        np.add.at(self.scores, np.asarray(slots, np.int64).reshape(-1), np.float32(1.0))

    def plan_update(self, novel) -> np.ndarray:
        """Slots that receive the novel blocks (in order), updating ids/scores.
        Free slots are used first, then the lowest current score (the first
        one on ties); at most ``capacity`` novel blocks are taken."""
        cap = self.capacity
        novel = np.asarray(novel, np.int64).reshape(-1)
        if cap <= 0 or novel.size == 0:
            return np.zeros(0, np.int64)
        novel = novel[:cap]
        cur = self.scores
        base = float(cur[: self.active].max()) + 1.0 if self.active > 0 else 1.0
        slots = np.empty(novel.size, np.int64)
        for i, blk in enumerate(novel):
            if self.active < cap:
                slot = self.active
                self.active += 1
            else:
                slot = int(np.argmin(cur[:cap]))
            self.block_ids[slot] = int(blk)
            cur[slot] = np.float32(base + float(i + 1) * 1e-3)
            slots[i] = slot
        return slots


def record_calibration_hits(counts: np.ndarray | None, active_blocks: np.ndarray, num_blocks: int,
                            recency_power: float) -> np.ndarray:
    """Recency-weighted hit counts for choosing a layer's hot set: row ``r`` of
    ``R`` selection rows adds ``((r+1)/R) ** recency_power`` to each of its
    valid blocks (``_record_hot_cache_calibration_blocks``,
    ``streaming_llama_runtime.py:2205-2243``)."""
    nb = int(num_blocks)
    c = np.zeros(nb, np.float32) if counts is None or np.asarray(counts).size != nb \
        else np.asarray(counts, np.float32).copy()
    ab = np.asarray(active_blocks, np.int64)
    if ab.size == 0:
        return c
    rows = ab.reshape(-1, ab.shape[-1])
    n = rows.shape[0]
    w = np.power(np.arange(1, n + 1, dtype=np.float32) / np.float32(n), np.float32(recency_power)).astype(np.float32)
    for r in range(n):
        valid = rows[r][(rows[r] >= 0) & (rows[r] < nb)]
        np.add.at(c, valid, w[r])
    return c


def target_hot_blocks(*, layer_idx: int, runtime_top_k: int, count_slots: int, previous_hot_count: int,
                      limit_bytes: int | None, used_bytes: int, sparse_layers: int, bytes_per_block: int) -> int:
    """Hot-bank capacity of a layer from the VRAM budget left for the
    remaining layers, at least the previous size or k
    (``_target_hot_blocks_for_layer``, ``streaming_llama_runtime.py:2275-2311``)."""
    fallback = int(previous_hot_count) if int(previous_hot_count) > 0 else max(1, int(runtime_top_k))
    if limit_bytes is None or int(limit_bytes) <= 0:
        return max(1, min(fallback, int(count_slots)))
    remaining = max(int(limit_bytes) - int(used_bytes), 0)
    remaining_layers = max(1, max(1, int(sparse_layers)) - max(0, int(layer_idx)))
    per_layer = int((float(remaining) * 0.97) / float(remaining_layers))
    return max(1, min(max(fallback, per_layer // max(1, int(bytes_per_block))), int(count_slots)))


def hot_cache_bytes_per_block(hidden: int, block_size: int = 32) -> int:
    """VRAM bytes of one hot block: gate and up packed rows with fp32 absmax,
    plus the down column slice and its absmax
    (``_estimate_mlp_hot_cache_bytes_per_block``, ``streaming_llama_runtime.py:2245-2273``)."""
    per_proj = (int(hidden) // 2) * int(block_size) + (int(hidden) // 64) * int(block_size) * 4
    return 2 * per_proj + int(hidden) * max(1, int(block_size) // 2) + int(hidden) * 4


def top_count_blocks(counts: np.ndarray, k: int) -> np.ndarray:
    """The ``k`` blocks with the highest counts, count-descending, ties to the
    lower block id (``torch.topk`` in the reference leaves tie order open)."""
    c = np.asarray(counts, np.float32).reshape(-1)
    k = max(0, min(int(k), c.size))
    return np.argsort(-c, kind="stable")[:k].astype(np.int64)


def assign_staging_rows(misses: np.ndarray, prefetched: dict[int, int], staging: int) -> tuple[np.ndarray, np.ndarray]:
    """Staging row of every miss -- a prefetched block keeps its row, the
    others take the remaining rows in ascending order -- and the mask of the
    misses whose records still have to be copied."""
    misses = np.asarray(misses, np.int64).reshape(-1)
    if misses.size > int(staging):
        raise RuntimeError(f"{misses.size} misses exceed the {int(staging)} staging rows")
    rows = np.full(misses.size, -1, np.int32)
    copy = np.ones(misses.size, bool)
    taken = np.zeros(int(staging), bool)
    for i, blk in enumerate(misses.tolist()):
        r = prefetched.get(int(blk))
        if r is not None:
            rows[i], copy[i], taken[r] = r, False, True
    free = np.nonzero(~taken)[0]
    rows[copy] = free[: int(copy.sum())]
    return rows, copy


class HotCacheCalibration:
    """Live calibration of the layers' hot sets from decode routes
    (``calibrate_vram_hot_cache``, ``streaming_llama_runtime.py:2374-2500``):
    while active, every decode selection adds recency-weighted hits
    (``record_calibration_hits``); ``hot_sets`` then gives each layer with hits
    its capacity (``target_hot_blocks``, at least the previous hot count) of
    top-count blocks, and ``rebuild`` pre-warms the caches with them."""

    def __init__(self, recency_power: float = 0.0):
        self.recency_power = float(recency_power)
        self.hits: dict[int, np.ndarray] = {}
        self.active = True

    def record(self, layer_idx: int, active_blocks, num_blocks: int) -> None:
        if self.active:
            self.hits[int(layer_idx)] = record_calibration_hits(self.hits.get(int(layer_idx)), active_blocks,
                                                                num_blocks, self.recency_power)

    def hot_sets(self, *, runtime_top_k, previous_hot: dict[int, int] | None = None, limit_bytes: int | None = None,
                 used_bytes: int = 0, sparse_layers: int | None = None,
                 bytes_per_block: int = 1_048_576) -> dict[int, np.ndarray]:
        """``runtime_top_k``: one k, or a dict layer -> k (the routing's top-k)."""
        out = {}
        n_layers = int(sparse_layers) if sparse_layers is not None else max(1, len(self.hits))
        for li, counts in sorted(self.hits.items()):
            if float(counts.sum()) <= 0.0:
                continue
            rtk = runtime_top_k[li] if isinstance(runtime_top_k, dict) else runtime_top_k
            cap = target_hot_blocks(layer_idx=li, runtime_top_k=int(rtk), count_slots=counts.size,
                                    previous_hot_count=int((previous_hot or {}).get(li, 0)), limit_bytes=limit_bytes,
                                    used_bytes=used_bytes, sparse_layers=n_layers, bytes_per_block=bytes_per_block)
            out[li] = top_count_blocks(counts, cap)
        return out

    def rebuild(self, caches: dict[int, "CachedSparseMlp"], **kw) -> dict:
        """Pre-warm each calibrated layer's cache with its new hot set (the
        first ``capacity`` blocks of it: the banks here do not grow)."""
        kw.setdefault("runtime_top_k", {li: c.router.top_k for li, c in caches.items()})
        kw.setdefault("previous_hot", {li: c.bank.active for li, c in caches.items()})
        kw.setdefault("bytes_per_block", hot_cache_bytes_per_block(next(iter(caches.values())).H) if caches else 1)
        sets = self.hot_sets(**kw)
        cached = 0
        for li, blocks in sets.items():
            if li in caches:
                caches[li].pre_warm(blocks)
                cached += min(blocks.size, caches[li].capacity)
        return {"updated_layers": len(sets), "hits": float(sum(float(self.hits[li].sum()) for li in sets)),
                "cached_blocks": cached}


# --------------------------------------------------------------------------- cached decode
@dataclass
class CacheStats:
    hits: int
    misses: int
    h2d_bytes: int        # bytes copied host -> device for this token (prefetched misses excluded)
    promoted: int
    prefetched: int = 0   # misses whose records a lookahead prefetch had already staged


class CachedSparseMlp:
    """One layer's decode MLP over a VRAM bank of ``capacity`` hot blocks plus
    ``staging`` rows for the misses of one token (default: the router's k)."""

    def __init__(self, router: RouterWeights, store: HostBlockStore, capacity: int, *, staging: int | None = None,
                 device: torch.device | None = None, promote: bool = True):
        self.router = router
        self.store = store
        self.H, self.I = store.hidden, store.intermediate
        self.NB = self.I // 32
        self.dev = device or router.enc_w.device
        self.capacity = int(capacity)
        self.staging = int(staging or router.top_k)
        self.promote = bool(promote)
        self.rec = record_bytes(self.H)
        self.pool = torch.empty((self.capacity + self.staging, self.rec), dtype=torch.uint8, device=self.dev)
        codes = [c.to(self.dev) for c in store.codes]
        self.bank_w = pool_weights(self.pool[: self.capacity], self.H, self.I, *codes)
        self.stage_w = pool_weights(self.pool[self.capacity:], self.H, self.I, *codes)
        self.bank = FixedCapacityBank(self.capacity)
        self.slot_host = np.full(self.NB, -1, np.int32)  # block -> bank slot
        self.slot_dev = torch.full((self.NB,), -1, dtype=torch.int32, device=self.dev)
        self.stage_map_host = torch.full((self.NB,), -1, dtype=torch.int32, pin_memory=True)
        self.stage_map_dev = torch.full((self.NB,), -1, dtype=torch.int32, device=self.dev)
        self.table_host = torch.full((self.NB,), -1, dtype=torch.int32, pin_memory=True)
        self.idx_dev = torch.empty(self.router.top_k, dtype=torch.int32, device=self.dev)
        self.idx_host = torch.empty(self.router.top_k, dtype=torch.int32, pin_memory=True)
        self.side = torch.cuda.Stream(device=self.dev)
        self.prefetched: dict[int, int] = {}  # block -> staging row, staged ahead by prefetch()
        self._lib = _lib.load()

    # ---- bank contents
    def _upload_table(self, stream: torch.cuda.Stream) -> None:
        self.table_host.numpy()[:] = self.slot_host
        with torch.cuda.stream(stream):
            self.slot_dev.copy_(self.table_host, non_blocking=True)

    def pre_warm(self, blocks) -> None:
        """Load ``blocks`` (at most ``capacity``) into the bank, scored
        ``linspace(n, 1)`` in the given order (the reference's pre-warm)."""
        b = np.asarray(blocks, np.int64).reshape(-1)[: self.capacity]
        self.bank.prewarm(b)
        self.slot_host[:] = -1
        self.slot_host[b] = np.arange(b.size, dtype=np.int32)
        main = torch.cuda.current_stream(self.dev)
        self._stage(b, np.arange(b.size, dtype=np.int32), self.pool, self.capacity, main)
        self._upload_table(main)
        torch.cuda.synchronize(self.dev)

    # ---- lookahead
    def prefetch(self, blocks) -> int:
        """Start copying the records of ``blocks`` that are not resident into
        the staging rows on the side stream, ahead of this layer's next
        ``decode`` (the reference's decode lookahead,
        ``streaming_llama_runtime.py:7780-7795``, ``:4910-5102``).  A block the
        next selection also lists is then served from its staged row without a
        copy; rows of blocks it does not list are reused.  Returns the number
        of records copied."""
        b = np.asarray(blocks, np.int64).reshape(-1)
        b = b[(b >= 0) & (b < self.NB)]
        b = b[self.slot_host[b] < 0]
        b = np.unique(b)[: self.staging] if b.size else b
        self.prefetched = {int(blk): i for i, blk in enumerate(b.tolist())}
        if b.size:
            # staging rows are free once the work queued so far (this layer's
            # previous token included) has run
            self.side.wait_stream(torch.cuda.current_stream(self.dev))
            self._stage(b, np.arange(b.size, dtype=np.int32), self.pool[self.capacity:], self.staging, self.side)
        return int(b.size)

    # ---- one token
    def decode(self, x: torch.Tensor, idx: torch.Tensor | None = None, out_dtype=torch.float32, *,
               calibration: "HotCacheCalibration | None" = None, layer_idx: int = 0):
        """MLP output for one token ``x [H]``.  The router always runs; ``idx``
        (int32 block ids on the device) replaces its selection when given.
        With ``calibration`` the selection is recorded as layer ``layer_idx``'s
        live route."""
        from .mlp import sparse_mlp_decode

        main = torch.cuda.current_stream(self.dev)
        k = self.router.top_k
        # route on the main stream; the selection comes back to the host
        sel = self.idx_dev
        sparse_route_only(x, self.router, sel)
        if idx is not None:
            sel = idx.to(device=self.dev, dtype=torch.int32).reshape(-1)
            k = int(sel.numel())
        self.idx_host[:k].copy_(sel[:k], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(main)
        ev.synchronize()
        blocks = self.idx_host[:k].numpy().astype(np.int64)
        if blocks.size and (blocks.min() < 0 or blocks.max() >= self.NB):
            raise RuntimeError("selected block id out of range")
        if np.unique(blocks).size != blocks.size:
            raise RuntimeError("the selection lists a block twice")
        if calibration is not None:
            calibration.record(layer_idx, blocks[None, :], self.NB)
        slots = self.slot_host[blocks]
        hit_mask = slots >= 0
        misses = blocks[~hit_mask]
        if misses.size > self.staging:
            raise RuntimeError(f"{misses.size} misses exceed the {self.staging} staging rows")
        # misses: pinned host -> staging rows on the side stream (prefetched
        # records are already there or on their way, queued on the same stream)
        rows, copy = assign_staging_rows(misses, self.prefetched, self.staging)
        smap = self.stage_map_host.numpy()
        smap[:] = -1
        smap[misses] = rows
        self.side.wait_stream(main)  # staging rows are free once the previous token is done
        if copy.any():
            self._stage(misses[copy], rows[copy], self.pool[self.capacity:], self.staging, self.side)
        self.prefetched = {}
        with torch.cuda.stream(self.side):
            self.stage_map_dev.copy_(self.stage_map_host, non_blocking=True)
        staged = torch.cuda.Event()
        staged.record(self.side)
        # resident blocks while the copies land (the block map drops the misses)
        y = sparse_mlp_decode(x, None, self.bank_w, idx=sel, slot_of_block=self.slot_dev, out_dtype=torch.float32)
        main.wait_event(staged)
        if misses.size:
            y2 = sparse_mlp_decode(x, None, self.stage_w, idx=sel, slot_of_block=self.stage_map_dev,
                                   out_dtype=torch.float32)
            y.add_(y2)
        promoted = 0
        if hit_mask.any():
            self.bank.add_hits(slots[hit_mask])
        if self.promote and misses.size:
            promoted = self._promote(misses, rows, main)
        n_copy = int(copy.sum())
        stats = CacheStats(hits=int(hit_mask.sum()), misses=int(misses.size), h2d_bytes=n_copy * self.rec,
                           promoted=promoted, prefetched=int(misses.size) - n_copy)
        return (y if out_dtype == torch.float32 else y.to(out_dtype)), stats

    def _stage(self, blocks: np.ndarray, rows: np.ndarray, pool: torch.Tensor, pool_rows: int,
               stream: torch.cuda.Stream) -> None:
        blk = np.ascontiguousarray(blocks, dtype=np.int32)
        dst = np.ascontiguousarray(rows, dtype=np.int32)
        _lib.check(self._lib.nsm_cache_stage(self.store.records.data_ptr(), int(self.store.num_blocks),
                                             blk.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), int(blk.size),
                                             self.rec, pool.data_ptr(),
                                             dst.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), int(pool_rows),
                                             stream.cuda_stream), "nsm_cache_stage")

    def _promote(self, misses: np.ndarray, rows: np.ndarray, main: torch.cuda.Stream) -> int:
        old = self.bank.block_ids.copy()
        active_before = self.bank.active
        slots = self.bank.plan_update(misses)
        n = slots.size
        if n == 0:
            return 0
        for i, slot in enumerate(slots):
            ob = old[slot] if slot < active_before else -1
            if ob >= 0 and self.slot_host[ob] == slot:
                self.slot_host[ob] = -1
            self.slot_host[misses[i]] = slot
        # staged record of miss i -> bank slot (device to device), after the staged compute
        src = torch.from_numpy(rows[:n].astype(np.int64) + self.capacity).to(self.dev, non_blocking=True)
        dst = torch.from_numpy(slots.astype(np.int64)).to(self.dev, non_blocking=True)
        self.pool.index_copy_(0, dst, self.pool.index_select(0, src))
        self._upload_table(main)
        return int(n)


class CachedLayerStack:
    """A token through several cached layers with the residual carried
    (``residual += MLP(rmsnorm(residual) * norm_weight)``; attention is
    identity, as in the benchmark's layer stack).  With ``lookahead``, each
    layer first routes the NEXT layer from its own pre-MLP residual and starts
    that layer's predicted misses on the next layer's side stream, so the
    copies overlap this layer's MLP (the reference predicts the next layer from
    the residual before the next attention, ``:7780-7795``).  A prediction
    only decides what is copied early: the selection is always the real
    router's, so outputs do not depend on ``lookahead``."""

    def __init__(self, caches: list[CachedSparseMlp], norm_weights: list[torch.Tensor | None] | None = None, *,
                 eps: float = 1e-5, lookahead: bool = True):
        self.caches = list(caches)
        self.norm = list(norm_weights) if norm_weights is not None else [None] * len(self.caches)
        self.eps = float(eps)
        self.lookahead = bool(lookahead)
        dev = self.caches[0].dev
        self._pred = torch.empty(max(c.router.top_k for c in self.caches), dtype=torch.int32, device=dev)
        self._pred_host = torch.empty(self._pred.numel(), dtype=torch.int32, pin_memory=True)

    def _input(self, residual: torch.Tensor, li: int) -> torch.Tensor:
        r = residual.float()
        x = r * torch.rsqrt(r.square().mean() + self.eps)
        if self.norm[li] is not None:
            x = x * self.norm[li].float()
        return x.to(torch.bfloat16)

    def _predict(self, x: torch.Tensor, li: int) -> np.ndarray:
        c = self.caches[li]
        k = c.router.top_k
        sparse_route_only(x, c.router, self._pred[:k])
        self._pred_host[:k].copy_(self._pred[:k], non_blocking=True)
        torch.cuda.current_stream(c.dev).synchronize()
        return self._pred_host[:k].numpy().astype(np.int64)

    def decode_token(self, residual: torch.Tensor, *, calibration: HotCacheCalibration | None = None):
        """Run every layer on ``residual`` (fp32 ``[H]``, updated in place);
        returns the per-layer ``CacheStats``."""
        stats = []
        for li, c in enumerate(self.caches):
            x = self._input(residual, li)
            if self.lookahead and li + 1 < len(self.caches):
                self.caches[li + 1].prefetch(self._predict(self._input(residual, li + 1), li + 1))
            y, st = c.decode(x, calibration=calibration, layer_idx=li)
            residual.add_(y)
            stats.append(st)
        return stats


def sparse_route_only(x: torch.Tensor, router: RouterWeights, idx_out: torch.Tensor) -> None:
    """Router for one token into ``idx_out`` (int32, score-descending)."""
    lib = _lib.load()
    H = router.hidden
    xv = x.reshape(-1).contiguous()
    ws = WORKSPACES.get(lib.nsm_decode_workspace_bytes(H, router.num_blocks * 32, router.top_k, router.rank),
                        xv.device)
    rc = router.to_c()
    _lib.check(lib.nsm_route(xv.data_ptr(), dtype_code(xv.dtype), H, ctypes.byref(rc), idx_out.data_ptr(), None, None,
                             ws.data_ptr(), ws.numel(), stream_handle(xv.device)), "nsm_route")
