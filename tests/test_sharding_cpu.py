"""Host logic of the column-sharded layers: the lane plan, the per-rank weight
blocks, and the all-gather ordering the reassembly kernel relies on, run as two
gloo ranks on CPU."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cim22_b200.sharding import ColumnShardPlan, gather_blocks


@pytest.mark.parametrize("lanes,world", [(4096, 8), (4096, 2), (100, 8), (10, 3), (1, 4), (84, 2)])
def test_plan_covers_every_lane_once(lanes, world):
    plan = ColumnShardPlan(lanes, world)
    covered = []
    for r in range(world):
        lo, hi = plan.lane_range(r)
        assert 0 <= lo <= hi <= lanes and hi - lo <= plan.block
        covered += list(range(lo, hi))
    assert covered == list(range(lanes))
    # The smallest equal block that covers every lane.
    assert plan.block * world >= lanes > (plan.block - 1) * world


def test_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        ColumnShardPlan(0, 2)
    with pytest.raises(ValueError):
        ColumnShardPlan(8, 2).lane_range(2)


def test_local_blocks_pad_with_zero_lanes():
    w = torch.arange(10 * 3, dtype=torch.float32).reshape(10, 3) + 1
    b = torch.arange(10, dtype=torch.float32) + 1
    plan = ColumnShardPlan(10, 4)  # block 3: lanes 0-2, 3-5, 6-8, 9 + 2 padding
    assert plan.block == 3
    last = plan.local_weight(w, 3)
    assert last.shape == (3, 3)
    assert torch.equal(last[0], w[9]) and not last[1:].any()
    assert torch.equal(plan.local_bias(b, 3), torch.tensor([10.0, 0.0, 0.0]))
    assert torch.equal(torch.cat([plan.local_weight(w, r) for r in range(4)])[:10], w)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, rows, lanes, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ColumnShardPlan(lanes, world)
        full = torch.arange(rows * lanes, dtype=torch.float32).reshape(rows, lanes)
        lo, hi = plan.lane_range(rank)
        local = torch.zeros(rows, plan.block)
        local[:, : hi - lo] = full[:, lo:hi]
        gathered = torch.empty(world, rows, plan.block)
        gather_blocks(local, gathered)
        # The reassembly contract: block r of the gather holds lanes
        # r*block .. r*block+block-1 of every row.
        rebuilt = torch.cat(list(gathered), dim=1)[:, :lanes]
        result[rank] = bool(torch.equal(rebuilt, full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("lanes", [64, 37])
def test_gather_blocks_order_two_gloo_ranks(lanes):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        mp.start_processes(_gather_worker, args=(2, _free_port(), 5, lanes, result), nprocs=2,
                           start_method="spawn")
        assert dict(result) == {0: True, 1: True}
