"""The fused layer chain (one persistent kernel for a Conv/Linear chain with
ReLU/GELU and 2x2 max pools): bit-identical to the per-layer kernels and to
the oracle."""

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def run(prog, x):
    prog.inputs[0].tensor.copy_(x.to(DEV))
    prog.status.reset()
    prog.launch()
    torch.cuda.synchronize()
    prog.check_status()
    return prog.output_tensors[0].cpu().numpy()


@pytest.mark.parametrize("name,batch", [("lenet", 1), ("lenet", 37), ("lenet", 256),
                                        ("lenet", 1000), ("mlp", 3), ("mlp", 64)])
def test_workload_chains_match_layers_and_oracle(name, batch):
    from cim22_b200 import program, workloads

    model, x = workloads.build(name, batch, seed=batch)
    chained = program.from_module(model, x, chain=True)
    assert chained.chained and [s.name for s in chained.steps] == ["chain"]
    plain = program.from_module(model, x, chain=False)
    assert not plain.chained
    got = run(chained, x)
    np.testing.assert_array_equal(bits(got), bits(run(plain, x)))
    if batch <= 256:  # the benchmarked LeNet batch included
        expected = oracle.cim_forward(model, x.numpy(), branches=4, threads=8)
        np.testing.assert_array_equal(bits(got), bits(expected))


class Mixed(nn.Module):
    """Strided padded convs without pools, GELU, signed activations (4-branch
    layers after GELU), multi-tile Linear layers."""

    def __init__(self):
        super().__init__()
        self.c1 = nn.Conv2d(3, 12, 3, 2, 1)
        self.c2 = nn.Conv2d(12, 20, 3, 1, 1)
        self.c3 = nn.Conv2d(20, 8, 2, 1, 0)
        self.f1 = nn.Linear(8 * 3 * 3, 150)
        self.f2 = nn.Linear(150, 7, bias=False)

    def forward(self, x):
        x = F.gelu(self.c1(x))
        x = F.max_pool2d(F.relu(self.c2(x)), 2)
        x = self.c3(x)
        x = torch.flatten(x, 1)
        return self.f2(F.relu(self.f1(x)))


def test_mixed_chain_matches_layers_and_oracle():
    from cim22_b200 import program

    torch.manual_seed(0)
    model = Mixed().eval()
    x = torch.randn(9, 3, 16, 16) * 3
    chained = program.from_module(model, x, chain=True)
    assert chained.chained
    plain = program.from_module(model, x, chain=False)
    got = run(chained, x)
    np.testing.assert_array_equal(bits(got), bits(run(plain, x)))
    # Linear-and-conv layers against the oracle layer by layer on the same
    # glue (GELU within the reference's float tolerance).
    expected = oracle.cim_forward(model, x.numpy(), branches=4, threads=8)
    assert np.max(np.abs(got - expected)) <= 1e-3 * np.max(np.abs(expected))


@pytest.mark.parametrize("widths", [(300, 300, 10), (120, 84, 10)])
def test_chain_wide_linear_stack(widths):
    """Linear stacks with an all-zero group, a subnormal input and a group
    exponent above the fast window; layers of fewer lanes than threads (all
    of the (120, 84, 10) stack) restore per (lane, sign, tile) and sum in tile
    order."""
    from cim22_b200 import program

    torch.manual_seed(1)
    a, b, c = widths
    model = nn.Sequential(nn.Flatten(), nn.Linear(1000, a), nn.ReLU(), nn.Linear(a, b),
                          nn.ReLU(), nn.Linear(b, c)).eval()
    x = torch.randn(33, 1000)
    x[0, :64] = 0.0  # an all-zero group
    x[1, 5] = 1e-40  # subnormal input
    x[2, 7] = 3e34  # group exponent above the fast window (exact path)
    chained = program.from_module(model, x, chain=True)
    assert chained.chained
    got = run(chained, x)
    np.testing.assert_array_equal(bits(got), bits(run(program.from_module(model, x, chain=False),
                                                      x)))
    expected = oracle.cim_forward(model, x.numpy(), branches=4, threads=8)
    np.testing.assert_array_equal(bits(got), bits(expected))


def test_chain_reports_non_finite_input():
    from cim22_b200 import program, workloads

    model, x = workloads.build("lenet", 4)
    prog = program.from_module(model, x)
    bad = x.clone()
    bad[2, 0, 5, 5] = float("inf")
    prog.inputs[0].tensor.copy_(bad.to(DEV))
    prog.status.reset()
    prog.launch()
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="NaN or infinity"):
        prog.check_status()


def test_non_chain_graphs_keep_layer_kernels():
    from cim22_b200 import program, workloads

    model, x = workloads.build("resnet18", 1)
    assert not program.from_module(model, x).chained


def test_pipelined_host_batches_match():
    """Host batches (pinned or pageable) through a chained program give the
    device-resident run's bits."""
    from cim22_b200 import program, workloads

    model, x = workloads.build("lenet", 256, seed=3)
    prog = program.from_module(model, x, chain=True)
    prog.capture()
    expected = run(prog, x)
    got = prog(x.pin_memory())
    assert got.device.type == "cpu"
    np.testing.assert_array_equal(bits(got.numpy()), bits(expected))
    got2 = prog(x.pin_memory())
    np.testing.assert_array_equal(bits(got2.numpy()), bits(expected))
    np.testing.assert_array_equal(bits(prog(x).numpy()), bits(expected))
