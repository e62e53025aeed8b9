"""Benchmark: 126-layer 405B-shaped sparse-MLP decode step (tokens/s).

Workload: per token, 126 decoder layers of hidden 16384,
intermediate 53248 (1664 blocks of 32), learned-basis router rank 64, top-k
208, NF4 gate/up/down weights (synthetic N(0, 0.02), seeded per layer); the
residual is carried across layers with attention replaced by identity.
Intermediate blocks are sharded across ranks (one process per GPU); every rank
routes the token, and each layer's fp32 [16384] partial outputs are summed
across ranks inside the next layer's router kernel: every rank stores its
partial into every rank's CUDA-IPC exchange buffer over NVLink and sums the
ranks' words in rank order (no NCCL collective on the data path).  On one GPU
the 126 layers do not all fit in HBM (126 x 1.47 GB), so as many unique
layers as fit are cycled; every layer is far larger than L2, so HBM traffic is
unchanged.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
(N > 1 is launched with torch.distributed.run, one rank per GPU).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

HIDDEN, INTERMEDIATE, TOP_K, RANK, LAYERS = 16384, 53248, 208, 64, 126
NB = INTERMEDIATE // 32
METRIC = "sparse-MLP decode tok/s (126-layer 405B shape)"
LAYER_BYTES_GPU = 3 * (INTERMEDIATE * HIDDEN // 2 + INTERMEDIATE * HIDDEN // 64 * 4)


def algorithmic_bytes_per_layer(k: int = TOP_K, H: int = HIDDEN, nb: int = NB, rank: int = RANK) -> int:
    """Bytes a layer-step must read or write: per selected block gate and up
    (32*H/2 packed + 32*H/64 fp32 absmax each) and down (16*H packed + 4*H
    absmax); router bf16 (rank*H encoder + NB*rank score head + NB bias);
    x and y bf16."""
    per_block = 2 * (16 * H + 2 * H) + 16 * H + 4 * H
    router = 2 * rank * H + 2 * rank * nb + 2 * nb
    return k * per_block + router + 4 * H


def gateup_bytes_per_launch(k: int = TOP_K, H: int = HIDDEN) -> int:
    """Bytes one gate/up launch must read: per selected block, gate and up each
    32*H/2 packed bytes + 32*H/64 fp32 absmax."""
    return k * 2 * (16 * H + 2 * H)


# DRAM bytes (read + write) per layer of the token kernel (SparseMlpDecoder(token_kernel=True)) from
# an ncu capture of a 2-layer token, scaled to the 126-layer token; the opt-in
# token kernel has no capture of its current build, so its line reports none.
TOKEN_DRAM_BYTES_PER_LAYER = None
TOKEN_TRAFFIC_SOURCE = None


# DRAM bytes (read + write) of one gateup_tma_kernel launch from the ncu capture in
# profiles/gateup_tma_kernel_cfg1.txt (dram__bytes_read.sum + dram__bytes_write.sum),
# the same workload on one GPU.
GATEUP_DRAM_BYTES_PER_LAUNCH = 122_852_608 + 3_301_120
GATEUP_TRAFFIC_SOURCE = "profiles/gateup_tma_kernel_cfg1.txt (ncu --set full, one launch, 1 GPU)"


def token_traffic(world: int):
    if TOKEN_DRAM_BYTES_PER_LAYER is None or world != 1:
        return None
    return int(TOKEN_DRAM_BYTES_PER_LAYER * LAYERS)


def headline_config(world: int) -> dict:
    """The ``config`` both arms print for the headline workload at ``world`` GPUs."""
    return {"workload": "BASELINE config 2: 126-layer 405B-shaped sparse-MLP decode step",
            "hidden": HIDDEN, "intermediate": INTERMEDIATE, "blocks": NB, "top_k": TOP_K, "rank": RANK,
            "layers": LAYERS, "tokens_per_step": 1,
            "parallelism": (f"block-shard x{world}, router on every rank, fp32 partial sums exchanged over "
                            "CUDA-IPC NVLink buffers inside the next router kernel" if world > 1
                            else "single GPU, all blocks resident"),
            "l2": "inputs larger than L2 (each layer >= 184 MB per rank)"}


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        try:
            rows = [r.split(", ") for r in Path(self.path).read_text().strip().splitlines() if r.strip()]
        except Exception:
            return out
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except Exception:
                continue
        if sm:
            out.update(sm_mhz=statistics.median(sm), sm_max_mhz=max(mx), reasons=sorted(reasons), samples=len(sm))
        return out


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------------------------------- our arm
def run_ours(args) -> None:
    import torch

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
        group = torch.distributed.group.WORLD
    from next_step_ai_b200 import synthetic as dsyn
    from next_step_ai_b200.engine import DecodeLayer, SparseMlpDecoder
    from next_step_ai_b200.weights import SparseMlpWeights

    from next_step_ai_b200.engine import shard_range

    lo, hi = shard_range(NB, world, rank)
    shape = dsyn.SHAPES["cfg1"]
    shard_bytes = LAYER_BYTES_GPU // world
    free, _ = torch.cuda.mem_get_info(dev)
    budget = free - (12 << 30)
    unique = max(1, min(LAYERS, budget // (shard_bytes + (3 << 20))))
    if args.unique_layers:
        unique = max(1, min(unique, args.unique_layers))
    t0 = time.time()
    layers = []
    for l in range(unique):
        w = dsyn.make_layer_weights(shape, 1234, l, dev)
        if world > 1:
            w = SparseMlpWeights(hidden=w.hidden, intermediate=w.intermediate,
                                 gate_packed=w.gate_packed[lo:hi].clone(), gate_absmax=w.gate_absmax[lo:hi].clone(),
                                 up_packed=w.up_packed[lo:hi].clone(), up_absmax=w.up_absmax[lo:hi].clone(),
                                 down_packed=w.down_packed[lo:hi].clone(), down_absmax=w.down_absmax[lo:hi].clone(),
                                 gate_code=w.gate_code, up_code=w.up_code, down_code=w.down_code, layout=w.layout)
            torch.cuda.empty_cache()
        torch.cuda.empty_cache()
        rw = dsyn.make_router(shape, 1234, l, dev)
        layers.append(DecodeLayer(router=rw, weights=w,
                                  norm_weight=torch.ones(HIDDEN, dtype=torch.bfloat16, device=dev)))
    torch.cuda.synchronize(dev)
    gen_s = time.time() - t0
    dec = SparseMlpDecoder(layers, LAYERS, block_range=(lo, hi), group=group)
    x0 = dsyn.make_x(shape, 99, 1, dev)[0].float()
    dec.residual.copy_(x0)
    g = dec.capture()

    def barrier():
        if group is not None:
            torch.distributed.barrier(device_ids=[local])

    for _ in range(args.warmup):
        dec.residual.copy_(x0)
        g.replay()
    torch.cuda.synchronize(dev)

    # device-timed region: inputs resident, K token steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        ev0.record()
        for _ in range(args.steps):
            g.replay()
        ev1.record()
        torch.cuda.synchronize(dev)
    barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev)
    if group is not None:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    ms_step = ms / args.steps

    # end-to-end through the public API: pinned H2D input, graph step, D2H result read
    h_in = torch.empty(HIDDEN, dtype=torch.float32, pin_memory=True)
    h_in.copy_(x0.cpu())
    h_out = torch.empty(HIDDEN, dtype=torch.float32, pin_memory=True)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        dec.residual.copy_(h_in, non_blocking=True)
        g.replay()
        h_out.copy_(dec.out, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    e1.record()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    t = torch.tensor([e2e_ms], device=dev)
    if group is not None:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = float(t.item())

    alg_layer = algorithmic_bytes_per_layer()
    pk = peaks()
    layer_us = ms_step * 1e3 / LAYERS
    # whole layer (router + gate/up + down) inside the timed region; at N > 1 each rank
    # reads 1/N of the block bytes plus the whole router
    router_b = 2 * RANK * HIDDEN + 2 * RANK * NB + 2 * NB
    rank_layer_bytes = (alg_layer - router_b) / world + router_b
    group_gbs = rank_layer_bytes / (layer_us * 1e-6) / 1e9
    if dec.use_token:
        # the token kernel is the only kernel of a step: its device time per launch is
        # the CUDA-event time of the timed region per step (one graph node per step)
        kern_name = ("token_kernel (one persistent cooperative launch per token: all 126 layers' router, "
                     "block selection, NF4 gate/up and down gather-GEMVs)")
        kern_bytes = rank_layer_bytes * LAYERS
        kern_us = ms_step * 1e3
        stage_us = None
    else:
        # dominant kernel (gate/up gather-GEMV): device time per launch from CUDA events the
        # library records around each stage, in an eager pass after the timed region
        kern_name = ("gateup_tma_kernel (block selection from the router's scores + NF4 gate+up gather-GEMV, one "
                     "launch per layer)")
        stage_us = dec.time_stages(min(LAYERS, 2 * unique))
        kern_bytes = gateup_bytes_per_launch() / world  # expected share of the selected blocks per rank
        kern_us = stage_us["gateup"]
    # selected blocks each rank held per layer (one eager token with records
    # between layers, every rank together): the ranks' shares of the 208
    # blocks differ, and each layer's exchange waits for the rank with the most
    counts = [int(b.numel()) for _, b in dec.trace_layers()]
    mine = {"mean": round(statistics.mean(counts), 1), "min": min(counts), "max": max(counts)}
    blocks_per_rank = [mine]
    if group is not None:
        blocks_per_rank = [None] * world
        torch.distributed.all_gather_object(blocks_per_rank, mine)
    kern_gbs = kern_bytes / (kern_us * 1e-6) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": args.steps / (ms / 1e3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": ("nf4 weights; x and SiLU*up as fp16 hi+lo pairs, prescaled fp16 codebook, fp16 x fp16 -> "
                      "fp32 MMA; fp32 residual"),
            "data": "synthetic: seeded N(0,0.02) NF4 weights, bf16 RMS-normalised N(0,1) input, random-init router",
            "config": headline_config(world),
            "run": {"unique_layers_resident": unique, "layer_cycling": unique < LAYERS, "cuda_graph": True,
                    "synthetic_gen_s": round(gen_s, 1), "blocks_per_rank_per_layer": blocks_per_rank},
            "e2e": {"value": args.steps / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": HIDDEN * 4,
                    "d2h_bytes_per_step": HIDDEN * 4},
            "gpu_launches": args.steps * dec.kernels_per_step,
            "roofline": {"bound": "hbm", "achieved": round(kern_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(kern_gbs / pk["hbm_gbs"], 4),
                         "traffic": (token_traffic(world) if dec.use_token
                                     else GATEUP_DRAM_BYTES_PER_LAUNCH if world == 1 else None),
                         "traffic_source": (TOKEN_TRAFFIC_SOURCE if dec.use_token
                                            else GATEUP_TRAFFIC_SOURCE if world == 1 else None),
                         "kernel": kern_name,
                         "algorithmic_bytes": int(kern_bytes), "us_per_launch": round(kern_us, 3),
                         "peak_source": pk["source"], "peak_note": "of measured (MEASURED_PEAKS.json hbm_gbs)",
                         "stage_us": {k: round(v, 3) for k, v in stage_us.items()} if stage_us else None,
                         "layer_group": {"algorithmic_bytes": alg_layer, "us_per_layer": round(layer_us, 3),
                                         "achieved": round(group_gbs, 1),
                                         "frac": round(group_gbs / pk["hbm_gbs"], 4)}},
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    dec.release()
    del g
    if group is not None:
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------------------------------------------- CPU arms
def cpu_layer_sample(seed: int, layer: int):
    """One layer of the workload, generated block by block on the host (only the
    router and the selected blocks are materialised), as torch CPU tensors."""
    import numpy as np
    import torch

    from oracle import synthetic as syn
    from oracle.router import route_sparse_mlp

    shape = syn.SHAPES["cfg1"]
    R = syn.make_router(shape, seed, layer)
    x = syn.make_x(shape, seed + layer, 1)
    blocks = route_sparse_mlp(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], shape.top_k, shape.rank)[0]
    G = syn.selected_blocks_gathered(shape, seed, layer, blocks)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    return {"R": {k: (None if v is None else t(v)) for k, v in R.items()}, "x": t(x),
            "G": {k: t(v) for k, v in G.items()}}


def cpu_step(state) -> None:
    """The reference's CPU torch path for one layer (router, then the fp32
    dequant + matmul of the selected NF4 blocks), on all host threads."""
    from oracle import cpu_torch as ct

    R, x, G = state["R"], state["x"], state["G"]
    ct.route(x, R["enc_w"], R["enc_b"], R["score_w"], R["score_b"], TOP_K)
    ct.mlp_gathered(x, G["gate_packed"], G["gate_absmax"], G["up_packed"], G["up_absmax"], G["down_cols"],
                    G["down_absmax_cols"], G["code"])


def cpu_threads() -> int:
    import torch

    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


CPU_SAMPLE_SECONDS = 12.0


def cpu_baseline() -> dict:
    """Layer-steps timed until ~12 s of CPU work (at least 3), tok/s scaled x126."""
    cores = cpu_threads()
    state = cpu_layer_sample(7, 0)
    cpu_step(state)  # warm
    n, t0 = 0, time.perf_counter()
    while n < 3 or time.perf_counter() - t0 < CPU_SAMPLE_SECONDS:
        cpu_step(state)
        n += 1
    per_layer = (time.perf_counter() - t0) / n
    return {"value": 1.0 / (per_layer * LAYERS), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} timed layer-steps of the 126-layer workload (router + 208-block NF4 MLP, torch fp32 "
                      f"on {cores} host threads: the reference's CPU torch path restated); "
                      f"tok/s = 1 / (126 x mean layer time)"}


def run_reference(args) -> None:
    """The reference arm: the reference's CPU torch path for this workload
    (restated -- the reference's own module needs bitsandbytes and is not
    present on the GPU box), one layer-step per step, on all host threads."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cores = cpu_threads()
    state = cpu_layer_sample(7, 0)
    for _ in range(args.warmup):
        cpu_step(state)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(state)
    dt = time.perf_counter() - t0
    per_layer = dt / args.steps
    value = 1.0 / (per_layer * LAYERS)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_layer * 1e3 * LAYERS,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (same generator family)", "config": headline_config(world),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": "each step = one layer-step (router + 208-block NF4 MLP) in torch fp32 on the "
                                   "host; ms_per_step and tok/s scaled to the 126-layer token"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------- config 3
CACHE_CAPACITY = 416  # 25 % of the 1664 blocks resident
CACHE_HITS = 146      # per-token draw: 146 resident + 62 non-resident blocks (~70 % constructed hit rate)


def zipf_selections(n_tokens: int, seed: int = 0):
    """Seeded config-3 workload: Zipf(s=1.1) popularity over a permutation of
    the block ids; the 416 most popular blocks start resident; each token draws
    146 resident and 62 non-resident blocks without replacement, each in
    proportion to its popularity."""
    import numpy as np

    rng = np.random.default_rng(seed)
    perm = rng.permutation(NB)
    weight = np.empty(NB)
    weight[perm] = 1.0 / np.arange(1, NB + 1) ** 1.1
    hot = perm[:CACHE_CAPACITY]
    cold = perm[CACHE_CAPACITY:]
    ph, pc = weight[hot] / weight[hot].sum(), weight[cold] / weight[cold].sum()
    sels = []
    for _ in range(n_tokens):
        s = np.concatenate([rng.choice(hot, CACHE_HITS, replace=False, p=ph),
                            rng.choice(cold, TOP_K - CACHE_HITS, replace=False, p=pc)])
        rng.shuffle(s)
        sels.append(s.astype(np.int32))
    return hot, sels


def pinned_h2d_peak_gbs(dev, nbytes: int = 1 << 30) -> float:
    """Measured pinned host -> device copy bandwidth (one large cudaMemcpyAsync)."""
    import torch

    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    d.copy_(h, non_blocking=True)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 0.0
    for _ in range(3):
        e0.record()
        d.copy_(h, non_blocking=True)
        e1.record()
        torch.cuda.synchronize(dev)
        best = max(best, nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9)
    del h, d
    return best


def run_cache(args) -> None:
    """one 405B-shaped layer decoding from a 25 % VRAM
    hot-block bank, misses staged from pinned host memory, promotion on."""
    import numpy as np
    import torch

    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from next_step_ai_b200 import synthetic as dsyn
    from next_step_ai_b200.cache import CachedSparseMlp, HostBlockStore

    shape = dsyn.SHAPES["cfg1"]
    t0 = time.time()
    w = dsyn.make_layer_weights(shape, 1234, 0, dev)
    store = HostBlockStore.from_weights(w)
    del w
    torch.cuda.empty_cache()
    rw = dsyn.make_router(shape, 1234, 0, dev)
    n_tok = args.warmup + args.steps
    hot, sels = zipf_selections(n_tok, seed=0)
    xs = dsyn.make_x(shape, 99, n_tok, dev)
    idx = [torch.from_numpy(s).to(dev) for s in sels]
    cm = CachedSparseMlp(rw, store, CACHE_CAPACITY)
    cm.pre_warm(hot)
    gen_s = time.time() - t0
    peak = pinned_h2d_peak_gbs(dev)
    for t in range(args.warmup):
        cm.decode(xs[t], idx=idx[t])
    torch.cuda.synchronize(dev)
    hits = misses = h2d = launches = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for t in range(args.warmup, n_tok):
            y, st = cm.decode(xs[t], idx=idx[t])
            hits += st.hits
            misses += st.misses
            h2d += st.h2d_bytes
            # this library's kernels per token: router (3), resident decode (4: selection map,
            # gate/up with SiLU*up, down, down reduction) and, when there are misses, the
            # gather kernel that stages them and the staged decode (4); the promotion
            # copies are torch's
            launches += 7 + (5 if st.misses else 0)
        e1.record()
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    h2d_gbs = h2d / (ms * 1e-3) / 1e9
    line = {
        "metric": "sparse-MLP decode tok/s, one 405B-shaped layer from a 25% VRAM hot-block cache",
        "value": args.steps / (ms / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
        "dtype": "nf4 weights, fp16 x fp16 -> fp32 MMA, bf16 io",
        "data": "synthetic: seeded NF4 layer; Zipf(1.1) block popularity; per-token draws of 146 resident + 62 "
                "non-resident blocks (the router runs, its selection is replaced by the draw)",
        "config": {"workload": "BASELINE config 3: single 405B-shaped layer, 416/1664 blocks resident, misses "
                               "from pinned host, decode-time promotion", "hidden": HIDDEN, "blocks": NB,
                   "top_k": TOP_K, "capacity": CACHE_CAPACITY, "staging_rows": cm.staging,
                   "record_bytes": cm.rec, "synthetic_gen_s": round(gen_s, 1)},
        "hit_rate": {"constructed": CACHE_HITS / TOP_K, "measured": hits / max(1, hits + misses)},
        "h2d": {"bound": "host link", "achieved_gbs": round(h2d_gbs, 2), "peak_gbs": round(peak, 2),
                "frac": round(h2d_gbs / peak, 4) if peak > 0 else None,
                "peak_note": "measured here: one 1 GiB pinned host-to-device cudaMemcpyAsync",
                "bytes_per_token": h2d / args.steps},
        "e2e": {"value": args.steps / (ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": h2d / args.steps,
                "d2h_bytes_per_step": TOP_K * 4},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------- config 4
UNION_ROWS = 32
UNION_SHARED = 0.85  # shared component of the token inputs (x_t = rms(a z + sqrt(1-a^2) e_t))


def run_union(args) -> None:
    """32 tokens of one 405B-shaped layer, each routed to its
    own top-208 blocks; the union is gathered once and contracted on the tensor
    cores (route + union decode in one CUDA graph), against 32 per-token GEMV
    decodes of the same tokens (route + MLP each, also one graph)."""
    import numpy as np
    import torch

    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from next_step_ai_b200 import route_sparse_mlp, sparse_mlp_decode, union_decode
    from next_step_ai_b200 import synthetic as dsyn

    shape = dsyn.SHAPES["cfg1"]
    t0 = time.time()
    w = dsyn.make_layer_weights(shape, 1234, 0, dev)
    rw = dsyn.make_router(shape, 1234, 0, dev)
    x = dsyn.make_x(shape, 99, UNION_ROWS, dev, shared=UNION_SHARED)
    idx = torch.empty((UNION_ROWS, TOP_K), dtype=torch.int32, device=dev)
    y = torch.empty((UNION_ROWS, HIDDEN), dtype=torch.bfloat16, device=dev)
    y_tok = torch.empty((UNION_ROWS, HIDDEN), dtype=torch.bfloat16, device=dev)
    gen_s = time.time() - t0

    def union_step():
        idx.copy_(route_sparse_mlp(x, rw).to(torch.int32))
        y.copy_(union_decode(x, idx, w))

    def per_token_step():
        for r in range(UNION_ROWS):
            sparse_mlp_decode(x[r], rw, w, out=y_tok[r])

    def graph_of(fn):
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            fn()
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        return g

    def timed(g, n):
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    gu, gt = graph_of(union_step), graph_of(per_token_step)
    with ClockSampler(local) as clk:
        ms_union = timed(gu, args.steps)
        ms_tok = timed(gt, max(3, args.steps // 4))
    _, uni = union_decode(x, idx, w, return_union=True)
    U = int(uni.numel())
    err = float((y.float() - y_tok.float()).abs().max())
    rel = float((y.float() - y_tok.float()).norm() / y_tok.float().norm())
    bytes_union = U * (2 * (16 * HIDDEN + 2 * HIDDEN) + 16 * HIDDEN + 4 * HIDDEN) + 2 * RANK * HIDDEN + 2 * RANK * NB
    flops = U * 3 * 2 * 32 * HIDDEN * UNION_ROWS
    pk = peaks()
    gbs = bytes_union / (ms_union * 1e-3) / 1e9
    line = {
        "metric": "multi-token sparse-MLP decode tok/s, one 405B-shaped layer, 32 tokens per step",
        "value": UNION_ROWS / (ms_union * 1e-3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_union, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "nf4 weights, fp16 x fp16 -> fp32 MMA, bf16 io",
        "data": f"synthetic: seeded NF4 layer; 32 token inputs rms(a z + sqrt(1-a^2) e_t), a={UNION_SHARED}",
        "config": {"workload": "BASELINE config 4: 32-token decode over the union of the tokens' top-208 sets",
                   "hidden": HIDDEN, "blocks": NB, "top_k": TOP_K, "rows": UNION_ROWS, "union_blocks": U,
                   "synthetic_gen_s": round(gen_s, 1)},
        "per_token_gemv": {"ms_per_step": ms_tok, "tok_s": UNION_ROWS / (ms_tok * 1e-3),
                           "speedup_of_union": ms_tok / ms_union},
        "parity_vs_per_token": {"max_abs": err, "rel_l2": rel},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / pk["hbm_gbs"], 4), "algorithmic_bytes": bytes_union,
                     "tensor_tflops": round(flops / (ms_union * 1e-3) / 1e12, 2),
                     "unit_of_launch": "32-row router (3 launches) + union decode launch group"},
        # this library's kernels per 32-token step: multi-row router (3) + union build, x, gate/up,
        # SiLU*up, down, output (6)
        "gpu_launches": args.steps * 9,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


LM_HEAD_VOCAB = 128256   # Llama-3.1 vocabulary (405B LM head: 128256 x 16384)


def run_lm_head(args) -> None:
    """NF4 LM head of the 405B shape (vocab 128256 x hidden 16384, NF4 blocksize
    64): one decode token's logits per step through ``Nf4LmHead`` (prep, GEMV
    and split-K finalize launches), the whole 1.18 GB weight streamed per step
    (larger than L2, so no flush is needed).  Not a BASELINE config: the row of
    the build's scope table that follows the MLP path."""
    import numpy as np
    import torch

    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from next_step_ai_b200.lm_head import Nf4LmHead

    V, H = LM_HEAD_VOCAB, HIDDEN
    t0 = time.time()
    gen = torch.Generator(device=dev).manual_seed(77)
    w = torch.randn((V, H), generator=gen, device=dev, dtype=torch.bfloat16) * 0.02
    head = Nf4LmHead.from_dense(w, dev)
    del w
    torch.cuda.empty_cache()
    x = (torch.randn((1, H), generator=gen, device=dev)).to(torch.bfloat16)
    out = torch.empty((1, V), dtype=torch.bfloat16, device=dev)
    gen_s = time.time() - t0

    def step():
        out.copy_(head(x))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / args.steps
        # end to end: pinned host x -> device, logits -> pinned host, every step
        xh = x.cpu().pin_memory()
        oh = torch.empty((1, V), dtype=torch.bfloat16).pin_memory()
        for _ in range(args.warmup):
            oh.copy_(head(xh.to(dev, non_blocking=True)), non_blocking=True)
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(args.steps):
            oh.copy_(head(xh.to(dev, non_blocking=True)), non_blocking=True)
        e1.record()
        torch.cuda.synchronize(dev)
        ms_e2e = e0.elapsed_time(e1) / args.steps
    # parity spot check on 64 rows (fp64 dequant of the same bytes)
    rows = torch.from_numpy(np.random.default_rng(3).choice(V, 64, replace=False)).to(dev)
    pk = head.packed.view(V, H // 2)[rows]
    nib = torch.stack([pk >> 4, pk & 15], dim=-1).reshape(64, H).long()
    wd = head.code.double()[nib] * head.absmax.view(V, H // 64)[rows].double().repeat_interleave(64, dim=1)
    ref = wd @ x.double().reshape(H)
    got = head(x, out_dtype=torch.float32).reshape(V)[rows].double()
    max_abs = float((got - ref).abs().max())
    algo = V * H // 2 + V * (H // 64) * 4 + 2 * H + 2 * V
    pk_ = peaks()
    gbs = algo / (ms * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        # the reference's CPU head is F.linear on the dense weight: time it on
        # a 2048-row slice with all host threads and scale to the vocabulary
        torch.set_num_threads(os.cpu_count() or 1)
        wc = torch.randn((2048, H), dtype=torch.float32) * 0.02
        xc = torch.randn((1, H), dtype=torch.float32)
        torch.nn.functional.linear(xc, wc)
        c0 = time.time()
        reps = 20
        for _ in range(reps):
            torch.nn.functional.linear(xc, wc)
        per = (time.time() - c0) / reps * (V / 2048)
        cpu = {"value": 1.0 / per, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": "F.linear fp32 [1,16384] x [2048,16384].T, 20 reps, scaled to 128256 rows"}
    line = {
        "metric": "NF4 LM head tok/s (405B shape: vocab 128256 x 16384, one decode token)",
        "value": 1e3 / ms, "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
        "dtype": "nf4 weights, fp16 x fp16 -> fp32 MMA, bf16 io",
        "data": "synthetic: N(0, 0.02) weight quantised to NF4 on the device, N(0,1) bf16 hidden",
        "config": {"workload": "NF4 LM head, 405B shape", "vocab": V, "hidden": H, "quant_block_size": 64,
                   "l2": "weight (1.18 GB) larger than L2", "synthetic_gen_s": round(gen_s, 1)},
        "e2e": {"value": 1e3 / ms_e2e, "unit": "tok/s", "h2d_bytes_per_step": 2 * H, "d2h_bytes_per_step": 2 * V},
        "gpu_launches": 3 * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk_["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / pk_["hbm_gbs"], 4), "algorithmic_bytes": algo,
                     "kernel": "nsm_lm_head_nf4 (prep + GEMV + finalize launches, timed together)",
                     "peak_source": pk_["source"]},
        "parity_spot_check": {"rows": 64, "max_abs_vs_fp64": max_abs},
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--unique-layers", type=int, default=0,
                    help="cap the resident layers (cycled over the 126); for small profiling captures")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5],
                    help="2: the 126-layer headline step (default); 3: hot-block cache layer; "
                         "4: 32-token union decode; 5: NF4 LM head (405B vocab)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.config == 3 and args.impl != "reference":
        run_cache(args)
        return
    if args.config == 4 and args.impl != "reference":
        run_union(args)
        return
    if args.config == 5 and args.impl != "reference":
        run_lm_head(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    main()
