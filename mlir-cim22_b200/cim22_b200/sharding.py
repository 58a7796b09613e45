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
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import cim_ops
from .cim_ops import CimLayer, StatusWord, Workspace


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


class ColumnShardedStack:
    """A chain of Linear layers, each followed by an optional activation
    ("relu", "gelu" or None), with every layer's lanes split over the ranks.

    forward(x) takes the full [rows, K0] input on this rank's device (every
    rank passes the same rows) and returns the full [rows, N_last] output.
    """

    def __init__(self, weights, biases, activations, rows: int, *, group=None,
                 device: torch.device | int = 0, input_nonnegative: bool = False) -> None:
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

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if tuple(x.shape) != (self.rows, self.layers[0].k):
            raise ValueError(f"input must be [{self.rows}, {self.layers[0].k}]")
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
