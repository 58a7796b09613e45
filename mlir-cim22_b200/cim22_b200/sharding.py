"""Column-sharded CIM layers over several GPUs, one process per GPU.

The output lanes of a CIM layer (the crossbar columns) are independent: each
lane's K-tile dots, per-tile restore, f32 sum in tile order, BF16 rounding and
sign-split merge use only that lane's weights and the shared input column
(lib/Execution/CIMSoftwareRunner.cpp:406-430, lib/Conversion/LinalgToCIM/
Passes.cpp:828-857,2405-2416). Splitting a layer's lanes over the ranks of a
process group therefore reproduces the single-device result bit for bit. Each
rank holds 1/world of every layer's weights, computes its block of lanes for
every input row, and an all-gather (NCCL over NVLink) plus one reassembly
kernel give every rank the full layer output before the next layer.

Ranks hold equal lane blocks (NCCL gathers equal sizes): the last blocks are
padded with all-zero weight lanes, whose outputs (+0, and the activation of
+0, which is +0) are dropped by the reassembly.

The fused form (`fused=True`, layers with BF16 operands) has no collective
call between layers: every rank's full layer outputs and a small flag array
live in device memory exported by CUDA IPC and mapped by the other ranks of
the node, the contraction's epilogue stores each rank's lane block straight
into every rank's output over NVLink, and a one-thread device barrier per
layer (cim22_cuda_peer_barrier, bounded waits) orders the layers.
"""

from __future__ import annotations

from dataclasses import dataclass

import ctypes

import torch
import torch.distributed as dist

from . import abi, cim_ops
from .cim_ops import CimLayer, StatusWord, Workspace
from .native import check, lib


@dataclass(frozen=True)
class ColumnShardPlan:
    """Equal contiguous lane blocks of a layer with `lanes` outputs over `world` ranks."""

    lanes: int
    world: int

    def __post_init__(self) -> None:
        if self.lanes <= 0 or self.world <= 0:
            raise ValueError("a column shard plan needs lanes > 0 and world > 0")

    @property
    def block(self) -> int:
        """Lanes per rank, padding included."""
        return -(-self.lanes // self.world)

    def lane_range(self, rank: int) -> tuple[int, int]:
        """Real lanes [lo, hi) of a rank (empty for trailing all-padding ranks)."""
        if not 0 <= rank < self.world:
            raise ValueError(f"rank {rank} outside a world of {self.world}")
        lo = min(self.lanes, rank * self.block)
        return lo, min(self.lanes, lo + self.block)

    def local_weight(self, weight: torch.Tensor, rank: int) -> torch.Tensor:
        """The rank's [block, K] weight rows, zero rows for the padding lanes."""
        lo, hi = self.lane_range(rank)
        out = torch.zeros(self.block, weight.shape[1], dtype=torch.float32)
        out[: hi - lo] = torch.as_tensor(weight, dtype=torch.float32)[lo:hi]
        return out

    def local_bias(self, bias: torch.Tensor | None, rank: int) -> torch.Tensor | None:
        if bias is None:
            return None
        lo, hi = self.lane_range(rank)
        out = torch.zeros(self.block, dtype=torch.float32)
        out[: hi - lo] = torch.as_tensor(bias, dtype=torch.float32)[lo:hi]
        return out


def gather_blocks(local: torch.Tensor, gathered: torch.Tensor, group=None) -> None:
    """All-gather each rank's [rows, block] output into gathered [world, rows, block]
    (a copy when there is one rank and no process group)."""
    world, rows, block = gathered.shape
    if tuple(local.shape) != (rows, block):
        raise ValueError(f"local block {tuple(local.shape)} does not match {(rows, block)}")
    if world == 1 and not dist.is_initialized():
        gathered[0].copy_(local)
        return
    dist.all_gather_into_tensor(gathered.view(world * rows, block), local, group=group)


class _DeviceArray:
    """A device pointer presented through __cuda_array_interface__, so that
    torch.as_tensor wraps it without a copy (the owner keeps it alive)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str) -> None:
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerBuffer:
    """One device buffer per rank of the group, each mapped on every rank.

    ptrs[p] is rank p's buffer as this process addresses it (its own
    allocation for p == rank, a CUDA IPC mapping otherwise); `local` wraps the
    own buffer as a torch tensor of `shape` and `dtype`. Every rank of the
    group constructs its PeerBuffers in the same order (the handle exchange is
    a collective). unmap_peers() then free(), with every rank unmapped before
    any rank frees, releases them.
    """

    def __init__(self, shape: tuple, dtype: torch.dtype, device: torch.device, group=None):
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > abi.MAX_PEERS:
            raise ValueError(f"peer memory spans at most {abi.MAX_PEERS} ranks")
        nbytes = int(torch.Size(shape).numel()) * torch.empty((), dtype=dtype).element_size()
        own = ctypes.c_void_p()
        check(lib().cim22_cuda_device_alloc(nbytes, ctypes.byref(own)), "peer buffer")
        self._own = own.value
        self.ptrs = [0] * self.world
        self.ptrs[self.rank] = self._own
        self._opened = []
        if self.world > 1:
            handle = (ctypes.c_ubyte * abi.IPC_HANDLE_BYTES)()
            check(lib().cim22_cuda_ipc_get_handle(self._own, handle), "IPC handle")
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
            every = torch.empty(self.world * abi.IPC_HANDLE_BYTES, dtype=torch.uint8,
                                device=device)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = every.view(self.world, abi.IPC_HANDLE_BYTES).cpu()
            for p in range(self.world):
                if p == self.rank:
                    continue
                raw = (ctypes.c_ubyte * abi.IPC_HANDLE_BYTES)(*every[p].tolist())
                peer = ctypes.c_void_p()
                check(lib().cim22_cuda_ipc_open_handle(raw, ctypes.byref(peer)), "IPC mapping")
                self.ptrs[p] = peer.value
                self._opened.append(peer.value)
        typestr = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
        self.local = torch.as_tensor(_DeviceArray(self._own, tuple(shape), typestr),
                                     device=device)

    def unmap_peers(self) -> None:
        """Unmap the other ranks' buffers (before any rank frees its own)."""
        for ptr in self._opened:
            lib().cim22_cuda_ipc_close_handle(ptr)
        self._opened = []

    def free(self) -> None:
        """Free this rank's buffer (after every rank has unmapped it)."""
        self.unmap_peers()
        if self._own:
            self.local = None
            lib().cim22_cuda_device_free(self._own)
            self._own = 0


class ColumnShardedStack:
    """A chain of Linear layers, each followed by an optional activation
    ("relu", "gelu" or None), with every layer's lanes split over the ranks.

    forward(x) takes the full [rows, K0] input on this rank's device (every
    rank passes the same rows) and returns the full [rows, N_last] output.
    """

    # A barrier wait that runs out after this long marks the step failed
    # (CIM22_STATUS_TIMEOUT) instead of hanging the GPU.
    BARRIER_LIMIT_NS = 5_000_000_000

    def __init__(self, weights, biases, activations, rows: int, *, group=None,
                 device: torch.device | int = 0, input_nonnegative: bool = False,
                 fused: bool = False) -> None:
        if not (len(weights) == len(biases) == len(activations)) or not weights:
            raise ValueError("one bias and one activation per weight")
        self.group = group
        if dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        self.device = torch.device("cuda", device) if isinstance(device, int) else device
        self.rows = rows
        self.workspace = Workspace(self.device)
        self.status = StatusWord(self.device)
        self.plans, self.layers, self.biases, self.acts, self.branches = [], [], [], [], []
        self.local, self.gathered, self.full = [], [], []
        nonneg = input_nonnegative
        k = None
        for w, b, act in zip(weights, biases, activations):
            w = torch.as_tensor(w, dtype=torch.float32)
            if k is not None and w.shape[1] != k:
                raise ValueError("layer input width does not match the previous layer's lanes")
            plan = ColumnShardPlan(w.shape[0], self.world)
            self.plans.append(plan)
            self.layers.append(CimLayer(plan.local_weight(w, self.rank), device=self.device))
            lb = plan.local_bias(b, self.rank)
            self.biases.append(None if lb is None else lb.to(self.device))
            self.acts.append(act)
            self.branches.append(2 if nonneg else 4)
            self.local.append(torch.empty(rows, plan.block, device=self.device))
            self.gathered.append(torch.empty(self.world, rows, plan.block, device=self.device))
            self.full.append(torch.empty(rows, plan.lanes, device=self.device))
            nonneg = act == "relu"
            k = w.shape[0]
        self.fused = fused
        self.peer_out, self.peer_args = [], []
        self.flags = None
        if fused:
            if not all(layer.bf16_operands for layer in self.layers):
                raise ValueError("the fused column shard needs every rank's lane block to take "
                                 "BF16 operands (at least 64 lanes with admitted weights)")
            for plan in self.plans:
                buf = PeerBuffer((rows, plan.lanes), torch.float32, self.device, group)
                self.peer_out.append(buf)
                lo, hi = plan.lane_range(self.rank)
                args = abi.PeerOutputs()
                for p, ptr in enumerate(buf.ptrs):
                    args.out[p] = ptr
                args.ranks, args.row_stride = self.world, plan.lanes
                args.lane_offset, args.lanes = lo, hi - lo
                self.peer_args.append(args)
            self.flags = PeerBuffer((self.world + 1,), torch.int32, self.device, group)
            self.flag_args = abi.PeerFlags()
            for p, ptr in enumerate(self.flags.ptrs):
                self.flag_args.flags[p] = ptr
            self.flag_args.ranks, self.flag_args.rank = self.world, self.rank
            # Every rank has mapped every buffer before any rank writes.
            torch.cuda.synchronize(self.device)
            if dist.is_initialized() and self.world > 1:
                dist.barrier(group=group)

    def _forward_fused(self, x: torch.Tensor) -> torch.Tensor:
        stream = torch.cuda.current_stream(self.device).cuda_stream
        for i, layer in enumerate(self.layers):
            if self.peer_args[i].lanes > 0:
                layer.prepare_bf16(x, self.rows, branches=self.branches[i],
                                   workspace=self.workspace, status=self.status)
                ws = self.workspace.get(layer.workspace_bytes(self.rows, self.branches[i]))
                b = self.biases[i]
                check(lib().cim22_cuda_layer_contract_bf16_peers(
                    layer._handle, self.rows, None if b is None else b.data_ptr(),
                    cim_ops.ACT[self.acts[i]], self.branches[i],
                    ctypes.byref(self.peer_args[i]), ws.data_ptr(), ws.numel(),
                    self.status.tensor.data_ptr(), stream), "column-sharded contraction")
            check(lib().cim22_cuda_peer_barrier(ctypes.byref(self.flag_args),
                                                self.BARRIER_LIMIT_NS,
                                                self.status.tensor.data_ptr(), stream),
                  "peer barrier")
            x = self.peer_out[i].local
        return x

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if tuple(x.shape) != (self.rows, self.layers[0].k):
            raise ValueError(f"input must be [{self.rows}, {self.layers[0].k}]")
        if self.fused:
            return self._forward_fused(x)
        for i, layer in enumerate(self.layers):
            layer.forward_bf16(x, self.local[i], self.rows, bias=self.biases[i],
                               activation=self.acts[i], branches=self.branches[i],
                               workspace=self.workspace, status=self.status)
            gather_blocks(self.local[i], self.gathered[i], self.group)
            cim_ops.unshard_columns(self.gathered[i], self.plans[i].lanes, out=self.full[i])
            x = self.full[i]
        return x

    __call__ = forward

    def check_status(self) -> None:
        self.status.raise_if_set(f"rank {self.rank}: ")

    def close(self) -> None:
        """Release the peer memory of the fused form. Every rank calls it
        after its last forward: each rank unmaps the others' buffers, the
        group meets, then each rank frees its own."""
        bufs = self.peer_out + ([self.flags] if self.flags is not None else [])
        if not bufs:
            return
        torch.cuda.synchronize(self.device)
        for buf in bufs:
            buf.unmap_peers()
        if dist.is_initialized() and self.world > 1:
            dist.barrier(group=self.group)
        for buf in bufs:
            buf.free()
        self.peer_out, self.flags = [], None
