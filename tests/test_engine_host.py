"""Host logic of the multi-GPU engine, without a GPU: the block sharding over
ranks, checked in two gloo processes (world size 2) and for larger worlds."""
from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, nb: int, out) -> None:
    from next_step_ai_b200.engine import shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = shard_range(nb, world, rank)
    got = [None] * world
    dist.all_gather_object(got, (lo, hi))
    # each rank sums "partial outputs" = ids of its blocks among a selection;
    # the all-reduced sum must equal the full selection's sum
    sel = torch.arange(0, nb, 7)
    part = sel[(sel >= lo) & (sel < hi)].sum().to(torch.float64).reshape(1)
    dist.all_reduce(part)
    if rank == 0:
        out.put((got, float(part.item()), float(sel.sum().item())))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("nb", [1664, 448, 37])
def test_shard_ranges_tile_blocks_over_two_gloo_ranks(nb):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, nb, q)) for r in range(2)]
    for p in procs:
        p.start()
    ranges, total, want = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert ranges[0][0] == 0 and ranges[-1][1] == nb
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(len(ranges) - 1))
    assert total == want


@pytest.mark.parametrize("world", [1, 3, 4, 8])
def test_shard_ranges_balanced(world):
    from next_step_ai_b200.engine import shard_range

    nb = 1664
    rs = [shard_range(nb, world, r) for r in range(world)]
    sizes = [hi - lo for lo, hi in rs]
    assert sum(sizes) == nb and max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(nb, world, world)
