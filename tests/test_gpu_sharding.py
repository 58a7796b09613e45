"""Column-sharded CIM layers on the GPU: the reassembly kernel, and (with two
or more GPUs) a two-rank NCCL run of a sharded Linear+GELU stack that must
match the single-device layers bit for bit."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("ranks,rows,cols,total", [(2, 5, 4, 8), (8, 33, 64, 500), (3, 1, 7, 15)])
def test_unshard_columns_kernel(ranks, rows, cols, total):
    from cim22_b200 import cim_ops

    src = torch.randn(ranks, rows, cols)
    got = cim_ops.unshard_columns(src.to(DEV), total).cpu()
    expected = torch.cat(list(src), dim=1)[:, :total]
    torch.testing.assert_close(got, expected, rtol=0, atol=0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stack(seed=0):
    g = torch.Generator().manual_seed(seed)
    widths = [320, 256, 130, 256]
    ws = [torch.randn(widths[i + 1], widths[i], generator=g) * 0.05 for i in range(3)]
    bs = [torch.randn(widths[i + 1], generator=g) for i in range(3)]
    acts = ["gelu", "relu", None]
    x = torch.randn(48, widths[0], generator=g)
    x[torch.rand(x.shape, generator=g) < 0.01] *= 20
    return ws, bs, acts, x


def _sharded_worker(rank, world, port, result):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from cim22_b200.sharding import ColumnShardedStack

        ws, bs, acts, x = _stack()
        stack = ColumnShardedStack(ws, bs, acts, rows=x.shape[0], device=rank)
        y = stack(x.to(f"cuda:{rank}"))
        torch.cuda.synchronize()
        stack.check_status()
        result[rank] = y.cpu().numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_column_shard_matches_single_device():
    from cim22_b200.cim_ops import CimLayer

    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        mp.start_processes(_sharded_worker, args=(2, _free_port(), result), nprocs=2,
                           start_method="spawn")
        got = dict(result)
    ws, bs, acts, x = _stack()
    y = x.to(DEV)
    branches = 4
    for w, b, act in zip(ws, bs, acts):
        y = CimLayer(w).linear_bf16(y, bias=b.to(DEV), activation=act, branches=branches)
        branches = 2 if act == "relu" else 4
    expected = y.cpu().numpy()
    for rank in (0, 1):
        np.testing.assert_array_equal(bits(got[rank]), bits(expected))
