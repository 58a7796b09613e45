"""Leaf discovery and LayerOffload argument checks (python/cim22/layers.py
of mlir-cim22: the same checks and error texts), on CPU."""

import pytest
import torch
import torch.nn as nn

from cim22_b200 import layers, workloads


def test_discover_lists_conv_and_linear_leaves_with_shapes():
    model, x = workloads.build("lenet", 2)
    found = layers.discover_cim_layers(model, (x,))
    assert [f["name"] for f in found] == ["conv1", "conv2", "fc1", "fc2", "fc3"]
    conv1 = found[0]
    assert conv1["type"] == "Conv2d" and conv1["weight_shape"] == [6, 1, 5, 5]
    assert conv1["input_shape"] == [2, 1, 32, 32] and conv1["output_shape"] == [2, 6, 28, 28]
    assert found[2]["input_shape"] == [2, 400] and found[2]["output_shape"] == [2, 120]
    # Without inputs the shapes stay empty and no hook is left behind.
    bare = layers.discover_cim_layers(model)
    assert bare[0]["input_shape"] == [] and not model.conv1._forward_hooks


class Aliased(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(4, 4)
        self.b = self.a
        self.block = nn.Sequential(nn.Linear(4, 4))
        self.act = nn.ReLU()


@pytest.mark.parametrize("selected,message", [
    ("a", "CIM layer names must be a sequence of non-empty strings"),
    (["a", ""], "CIM layer names must be a sequence of non-empty strings"),
    ([], "Select at least one CIM layer"),
    (["block.0", "block.0"], "CIM layer names must be unique"),
    (["nope"], "Unknown CIM layer: nope"),
    (["block"], "CIM layer must be a leaf module: block"),
    (["act"], "Unsupported CIM layer type: act"),
    (["a"], "CIM layer has multiple names for the same module: a"),
])
def test_validate_cim_layers_rejections(selected, message):
    with pytest.raises(ValueError, match=message):
        layers.validate_cim_layers(Aliased(), selected)


def test_validate_cim_layers_accepts_leaves():
    assert layers.validate_cim_layers(Aliased(), ["block.0"]) == ("block.0",)
    assert layers.validate_cim_layers(Aliased(), None) == ()


def test_layer_offload_argument_checks():
    model, x = workloads.build("lenet", 2)
    with pytest.raises(ValueError, match="Layer offload requires runtime='cuda'"):
        layers.LayerOffload(model, ["fc1"], (x,), runtime="simulator")
    model.train()
    with pytest.raises(ValueError, match="Layer offload requires a model in eval mode"):
        layers.LayerOffload(model, ["fc1"], (x,))
    model.eval()
    with pytest.raises(ValueError, match="Unknown CIM layer: fc9"):
        layers.LayerOffload(model, ["fc9"], (x,))
