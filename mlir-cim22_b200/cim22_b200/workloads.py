"""The five CIM simulation workloads, as PyTorch modules with synthetic inputs.

Weights are random-initialised with the stated distributions (no checkpoints)
and inputs are seeded synthetic tensors of the stated shapes; the event frames
stand in for DVSGesture, which is not available offline.

  mlp        784 -> 256 -> 128 -> 10, ReLU, W ~ N(0, 0.05), x ~ U[0,1] 1x28x28, batch 64
  lenet      conv5x5 1->6, pool, conv5x5 6->16, pool, fc 400->120->84->10, ReLU,
             He-normal weights, x ~ U[0,1] 1x32x32, batch 256
  resnet18   CIFAR ResNet-18 (BasicBlock [2,2,2,2], 64/128/256/512, 3x3 stem,
             10-way head), He-normal, x ~ N(0,1) 3x32x32, batch 1024
  bf16_4x4096  4 x Linear(4096, 4096, bias=False) with GELU between,
             W ~ N(0, 0.02), x ~ N(0,1) with 1% outliers x20, 512 rows
  event_cnn  conv3x3 2->32 (s1), 32->64, 64->128, 128->128 (s2), pad 1, ReLU,
             global average pool, fc 128->11; Bernoulli(0.05) binary
             2x128x128 frames; batch 4096 over 8 GPUs (512 per GPU)
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn as nn
import torch.nn.functional as F


def _he(module: nn.Module) -> None:
    for m in module.modules():
        if isinstance(m, (nn.Conv2d, nn.Linear)):
            nn.init.kaiming_normal_(m.weight, mode="fan_in", nonlinearity="relu")


class MLP(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(784, 256)
        self.fc2 = nn.Linear(256, 128)
        self.fc3 = nn.Linear(128, 10)
        for p in self.parameters():
            nn.init.normal_(p, 0.0, 0.05)

    def forward(self, x):
        x = torch.flatten(x, 1)
        x = F.relu(self.fc1(x))
        x = F.relu(self.fc2(x))
        return self.fc3(x)


class LeNet(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.conv1 = nn.Conv2d(1, 6, 5)
        self.conv2 = nn.Conv2d(6, 16, 5)
        self.fc1 = nn.Linear(400, 120)
        self.fc2 = nn.Linear(120, 84)
        self.fc3 = nn.Linear(84, 10)
        _he(self)

    def forward(self, x):
        x = F.max_pool2d(F.relu(self.conv1(x)), 2)
        x = F.max_pool2d(F.relu(self.conv2(x)), 2)
        x = torch.flatten(x, 1)
        x = F.relu(self.fc1(x))
        x = F.relu(self.fc2(x))
        return self.fc3(x)


class BasicBlock(nn.Module):
    def __init__(self, cin: int, cout: int, stride: int) -> None:
        super().__init__()
        self.conv1 = nn.Conv2d(cin, cout, 3, stride, 1, bias=False)
        self.bn1 = nn.BatchNorm2d(cout)
        self.conv2 = nn.Conv2d(cout, cout, 3, 1, 1, bias=False)
        self.bn2 = nn.BatchNorm2d(cout)
        self.shortcut = nn.Identity()
        if stride != 1 or cin != cout:
            self.shortcut = nn.Sequential(nn.Conv2d(cin, cout, 1, stride, 0, bias=False),
                                          nn.BatchNorm2d(cout))

    def forward(self, x):
        out = F.relu(self.bn1(self.conv1(x)))
        out = self.bn2(self.conv2(out))
        return F.relu(out + self.shortcut(x))


class ResNet18(nn.Module):
    def __init__(self, classes: int = 10) -> None:
        super().__init__()
        self.conv1 = nn.Conv2d(3, 64, 3, 1, 1, bias=False)
        self.bn1 = nn.BatchNorm2d(64)
        blocks = []
        cin = 64
        for cout, stride in ((64, 1), (128, 2), (256, 2), (512, 2)):
            blocks += [BasicBlock(cin, cout, stride), BasicBlock(cout, cout, 1)]
            cin = cout
        self.layers = nn.Sequential(*blocks)
        self.fc = nn.Linear(512, classes)
        _he(self)

    def forward(self, x):
        x = F.relu(self.bn1(self.conv1(x)))
        x = self.layers(x)
        x = F.adaptive_avg_pool2d(x, 1)
        return self.fc(torch.flatten(x, 1))


class BF16Stack(nn.Module):
    def __init__(self, width: int = 4096, depth: int = 4) -> None:
        super().__init__()
        self.layers = nn.ModuleList(nn.Linear(width, width, bias=False) for _ in range(depth))
        for layer in self.layers:
            nn.init.normal_(layer.weight, 0.0, 0.02)

    def forward(self, x):
        for i, layer in enumerate(self.layers):
            x = layer(x)
            if i + 1 < len(self.layers):
                x = F.gelu(x)
        return x


class EventCNN(nn.Module):
    def __init__(self, classes: int = 11) -> None:
        super().__init__()
        self.conv1 = nn.Conv2d(2, 32, 3, 1, 1)
        self.conv2 = nn.Conv2d(32, 64, 3, 2, 1)
        self.conv3 = nn.Conv2d(64, 128, 3, 2, 1)
        self.conv4 = nn.Conv2d(128, 128, 3, 2, 1)
        self.fc = nn.Linear(128, classes)
        _he(self)

    def forward(self, x):
        x = F.relu(self.conv1(x))
        x = F.relu(self.conv2(x))
        x = F.relu(self.conv3(x))
        x = F.relu(self.conv4(x))
        x = F.adaptive_avg_pool2d(x, 1)
        return self.fc(torch.flatten(x, 1))


@dataclass
class Workload:
    name: str
    batch: int
    make_model: Callable[[], nn.Module]
    make_input: Callable[[int, torch.Generator], torch.Tensor]
    description: str


def _uniform(shape):
    return lambda b, g: torch.rand((b, *shape), generator=g)


def _normal(shape):
    return lambda b, g: torch.randn((b, *shape), generator=g)


def _outliers(b, g):
    x = torch.randn((b, 4096), generator=g)
    mask = torch.rand((b, 4096), generator=g) < 0.01
    return torch.where(mask, x * 20, x)


def _events(b, g):
    return (torch.rand((b, 2, 128, 128), generator=g) < 0.05).float()


WORKLOADS = {
    "mlp": Workload("mlp", 64, MLP, _uniform((1, 28, 28)),
                    "3-layer MLP 784-256-128-10, batch 64"),
    "lenet": Workload("lenet", 256, LeNet, _uniform((1, 32, 32)),
                      "LeNet-5 conv5x5 1-6/6-16, fc 400-120-84-10, batch 256"),
    "resnet18": Workload("resnet18", 1024, ResNet18, _normal((3, 32, 32)),
                         "CIFAR ResNet-18, batch 1024"),
    "bf16_4x4096": Workload("bf16_4x4096", 512, BF16Stack, _outliers,
                            "4 x BF16 sign-split Linear 4096x4096 + GELU, 512 rows"),
    "event_cnn": Workload("event_cnn", 512, EventCNN, _events,
                          "event-frame CNN 2x128x128, 512 per GPU (4096 over 8)"),
}


def build(name: str, batch: int | None = None, seed: int = 0):
    """Return (eval model, input batch) for a workload, deterministically seeded."""
    w = WORKLOADS[name]
    torch.manual_seed(seed)
    model = w.make_model().eval()
    g = torch.Generator().manual_seed(seed + 1)
    x = w.make_input(batch or w.batch, g)
    return model, x
