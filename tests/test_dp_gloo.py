"""Host logic of the data-parallel SpecDec runner on CPU: shard bounds and the one
all-gather of per-rank token blocks, with world_size-2 gloo process groups."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from specdec_b200.engine.dp import check_shardable, gather_rows, max_over_ranks, shard_bounds, synthetic_prompts


@pytest.mark.parametrize("total,world", [(256, 1), (256, 2), (256, 8), (10, 3), (3, 4), (0, 2)])
def test_shard_bounds_cover_every_sequence_once(total, world):
    seen = []
    sizes = []
    for r in range(world):
        s, e = shard_bounds(total, world, r)
        assert 0 <= s <= e <= total
        seen.extend(range(s, e))
        sizes.append(e - s)
    assert seen == list(range(total))
    assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)


def test_fewer_sequences_than_ranks_is_rejected_on_every_rank():
    """An empty shard is refused up front by a check every rank computes alike."""
    check_shardable(8, 8)
    with pytest.raises(ValueError):
        check_shardable(3, 4)


def test_synthetic_prompts_are_identical_across_calls():
    a = synthetic_prompts(6, 16, 1000, 3)
    b = synthetic_prompts(6, 16, 1000, 3)
    assert a.dtype == torch.int32 and a.shape == (6, 16)
    assert torch.equal(a, b)
    assert int(a.min()) >= 0 and int(a.max()) < 1000


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s, e = shard_bounds(total, world, rank)
        # stand-in for a rank's decode output: row b holds b * 100 + column
        local = (torch.arange(s, e).unsqueeze(1) * 100 + torch.arange(5).unsqueeze(0)).to(torch.int32)
        full = gather_rows(local, total, world)
        t = max_over_ranks(float(rank + 1), world, "cpu")
        if rank == 0:
            torch.save({"full": full, "t": t}, out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [7, 8])
def test_gather_rows_assembles_all_blocks_in_order(tmp_path, total):
    world = 2
    out = tmp_path / "gathered.pt"
    mp.start_processes(_worker, args=(world, _free_port(), total, str(out)), nprocs=world, join=True,
                       start_method="spawn")
    res = torch.load(out)
    want = (torch.arange(total).unsqueeze(1) * 100 + torch.arange(5).unsqueeze(0)).to(torch.int32)
    assert torch.equal(res["full"], want)
    assert res["t"] == 2.0
