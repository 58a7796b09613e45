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


def _wide_stack(seed=1):
    """Layers wide enough that every rank's lane block (two ranks) takes BF16
    operands, as the fused column shard requires."""
    g = torch.Generator().manual_seed(seed)
    widths = [300, 512, 600, 512]
    ws = [torch.randn(widths[i + 1], widths[i], generator=g) * 0.05 for i in range(3)]
    bs = [torch.randn(widths[i + 1], generator=g) for i in range(3)]
    acts = ["gelu", "relu", None]
    x = torch.randn(200, widths[0], generator=g)
    x[torch.rand(x.shape, generator=g) < 0.01] *= 20
    return ws, bs, acts, x


def _expected(ws, bs, acts, x):
    from cim22_b200.cim_ops import CimLayer

    y = x.to(DEV)
    branches = 4
    for w, b, act in zip(ws, bs, acts):
        y = CimLayer(w).linear_bf16(y, bias=b.to(DEV), activation=act, branches=branches)
        branches = 2 if act == "relu" else 4
    return y.cpu().numpy()


def test_fused_column_shard_single_rank_matches_layers():
    """The fused form on one rank: the contraction stores through the peer
    output table (one entry, this device) and the device barrier passes on
    its own epoch; the outputs equal the plain layers' bit for bit, on
    repeated forwards."""
    from cim22_b200.sharding import ColumnShardedStack

    ws, bs, acts, x = _wide_stack()
    stack = ColumnShardedStack(ws, bs, acts, rows=x.shape[0], device=DEV, fused=True)
    try:
        expected = _expected(ws, bs, acts, x)
        for _ in range(3):
            y = stack(x.to(DEV))
            torch.cuda.synchronize()
            stack.check_status()
            np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(expected))
    finally:
        stack.close()


def test_peer_barrier_wait_runs_out_and_reports():
    """A barrier of two ranks in which the second never arrives (its flag is
    a word nothing writes): the wait gives up after its limit, reports
    CIM22_STATUS_TIMEOUT and leaves the context usable. No copy or MMA is in
    flight in this kernel."""
    import ctypes
    import time

    from cim22_b200 import abi
    from cim22_b200.native import lib

    own = torch.zeros(3, dtype=torch.int32, device=DEV)
    absent = torch.zeros(3, dtype=torch.int32, device=DEV)
    flags = abi.PeerFlags()
    flags.flags[0], flags.flags[1] = own.data_ptr(), absent.data_ptr()
    flags.ranks, flags.rank = 2, 0
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    t0 = time.perf_counter()
    assert lib().cim22_cuda_peer_barrier(ctypes.byref(flags), 20_000_000, status.data_ptr(),
                                         stream) == 0
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10
    assert int(status.item()) == 0x40  # CIM22_STATUS_TIMEOUT
    # The epoch was published to both ranks' words 0, and this rank's epoch is 1.
    assert own.tolist() == [1, 0, 1] and absent.tolist() == [1, 0, 0]
    assert float((torch.ones(4, device=DEV) * 2).sum().item()) == 8.0


def _fused_worker(rank, world, port, result):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from cim22_b200.sharding import ColumnShardedStack

        ws, bs, acts, x = _wide_stack()
        stack = ColumnShardedStack(ws, bs, acts, rows=x.shape[0], device=rank, fused=True)
        try:
            outs = []
            for _ in range(3):
                outs.append(stack(x.to(f"cuda:{rank}")).cpu().numpy())
            torch.cuda.synchronize()
            stack.check_status()
            dist.barrier()
        finally:
            stack.close()
        result[rank] = outs
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_fused_column_shard_matches_single_device():
    """Two ranks, each storing its lane block into both ranks' outputs over
    NVLink and meeting at the device barrier after every layer: three
    forwards in a row equal the single-device layers bit for bit."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        mp.start_processes(_fused_worker, args=(2, _free_port(), result), nprocs=2,
                           start_method="spawn")
        got = dict(result)
    expected = _expected(*_wide_stack())
    for rank in (0, 1):
        for y in got[rank]:
            np.testing.assert_array_equal(bits(y), bits(expected))
