"""LayerOffload with runtime="cuda": selected Conv2d/Linear leaves of a CPU
model run as CIM layers on the GPU, the rest of the model on CPU, and the
outputs equal the oracle's forward that computes exactly those layers as CIM
layers (the rest as PyTorch CPU eager) - bit for bit."""

import copy

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,selected", [("lenet", ["conv1", "fc1"]),
                                           ("mlp", ["fc2"]),
                                           ("resnet18", ["conv1", "layers.1.conv2", "fc"])])
def test_layer_offload_matches_oracle_on_selected_layers(name, selected):
    from cim22_b200 import layers, workloads

    model, x = workloads.build(name, 3, seed=5)
    # The oracle runs on its own copy: the offloaded model's selected leaves
    # are compiled in place (the reference asks for a separate instance too).
    reference = copy.deepcopy(model)
    offload = layers.LayerOffload(model, selected, (x,))
    assert offload.cim_layers == tuple(selected)
    assert set(offload.layer_compile_seconds) == set(selected)
    got = offload(x)
    assert got.device.type == "cpu"
    assert offload.dispatch_count >= len(selected)
    expected = oracle.cim_forward(reference, x.numpy(), branches=4, threads=4,
                                  layers=selected)
    np.testing.assert_array_equal(got.numpy().view(np.uint32), expected.view(np.uint32))
    # Another batch of the same shape reuses the compiled layers.
    _, x2 = workloads.build(name, 3, seed=6)
    got2 = offload(x2)
    expected2 = oracle.cim_forward(reference, x2.numpy(), branches=4, threads=4,
                                   layers=selected)
    np.testing.assert_array_equal(got2.numpy().view(np.uint32), expected2.view(np.uint32))


def test_layer_offload_rejects_recompilation():
    from cim22_b200 import layers, workloads

    model, x = workloads.build("lenet", 2, seed=1)
    offload = layers.LayerOffload(model, ["fc1"], (x,))
    _, bigger = workloads.build("lenet", 5, seed=2)
    with pytest.raises(RuntimeError, match="Input triggered additional compilation"):
        offload(bigger)
