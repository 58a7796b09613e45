"""Whole workloads on the GPU against the oracle.

* MLP and LeNet use only exact glue (ReLU, max-pool, flatten), so the whole
  network is bit-exact against the oracle's forward.
* For ResNet-18, the BF16 4x4096 stack and the event CNN (batch norm, GELU,
  average pooling in f32 glue), every CIM layer is checked bit-exact on the
  very inputs the GPU produced for it, and the network output within the
  reference's float tolerance (1e-3 relative to the output scale).
* The torch.compile backend with runtime="cuda" returns the oracle's result
  for CPU inputs and raises the reference's error text for NaN inputs.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def run_program(program, x):
    program.inputs[0].tensor.copy_(x.to(DEV))
    program.status.reset()
    program.launch()
    torch.cuda.synchronize()
    program.check_status()
    return [t.cpu().numpy() for t in program.output_tensors]


@pytest.mark.parametrize("layout", ["nchw", "nhwc"])
@pytest.mark.parametrize("name,batch", [("mlp", 8), ("lenet", 6)])
def test_exact_glue_networks_bit_exact(name, batch, layout):
    from cim22_b200 import program, workloads

    model, x = workloads.build(name, batch)
    prog = program.from_module(model, x, layout=layout)
    (got,) = run_program(prog, x)
    expected = oracle.cim_forward(model, x.numpy(), branches=4, threads=8)
    np.testing.assert_array_equal(bits(got), bits(expected))
    # Graph replay gives the same bits.
    prog.capture()
    prog.inputs[0].tensor.copy_(x.to(DEV))
    prog.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(prog.output_tensors[0].cpu().numpy()), bits(expected))


def _check_layers(prog):
    checked = 0
    for step in prog.steps:
        step.fn()
        if not step.cim:
            continue
        torch.cuda.synchronize()
        meta = step.meta
        x = meta["x"].cpu().numpy()
        w = meta["weight"].numpy()
        b = None if meta["bias"] is None else meta["bias"].numpy()
        got = meta["out"].cpu().numpy()
        if meta["kind"] == "conv":
            if meta["layout"] == "nhwc":
                x = x.transpose(0, 3, 1, 2)
            exp = oracle.conv2d_bf16(x, w, b, meta["stride"], meta["pad"], branches=4,
                                     threads=8)
            if meta["out_layout"] == "nhwc":
                exp = exp.transpose(0, 2, 3, 1)
        else:
            exp = oracle.linear_bf16(x.reshape(x.shape[0], -1), w, b, branches=4, threads=8)
        assert meta["act"] is None
        np.testing.assert_array_equal(bits(got.reshape(exp.shape)), bits(exp),
                                      err_msg=step.name)
        checked += 1
    return checked


@pytest.mark.parametrize("layout", ["nchw", "nhwc"])
def test_residual_adds_fold_into_conv_epilogues(layout):
    """Conv -> BatchNorm -> add -> ReLU of every residual block folds the add
    into the contraction epilogue of the operand computed last (conv2 of an
    identity block, the shortcut conv of a projection block); the outputs are
    bit-identical to the unfused glue."""
    from cim22_b200 import program, workloads

    model, x = workloads.build("resnet18", 2)
    fused = program.from_module(model, x, layout=layout)
    assert not [s.name for s in fused.steps if s.name.startswith("add")]
    assert sum(1 for s in fused.steps if s.cim and s.meta.get("residual") is not None) == 8
    plain = program.from_module(model, x, fuse=False, layout=layout)
    (a,) = run_program(fused, x)
    (b,) = run_program(plain, x)
    np.testing.assert_array_equal(bits(a), bits(b))


@pytest.mark.parametrize("layout", ["nchw", "nhwc"])
@pytest.mark.parametrize("name,batch,layers", [("resnet18", 1, 21), ("bf16_4x4096", 2, 4),
                                               ("event_cnn", 1, 5)])
def test_every_cim_layer_bit_exact_on_recorded_inputs(name, batch, layers, layout):
    from cim22_b200 import program, workloads

    model, x = workloads.build(name, batch)
    prog = program.from_module(model, x, fuse=False, layout=layout)
    prog.inputs[0].tensor.copy_(x.to(DEV))
    prog.status.reset()
    assert _check_layers(prog) == layers
    prog.check_status()


@pytest.mark.parametrize("layout", ["nchw", "nhwc"])
@pytest.mark.parametrize("name,batch", [("resnet18", 2), ("bf16_4x4096", 3), ("event_cnn", 2)])
def test_float_glue_networks_within_tolerance(name, batch, layout):
    from cim22_b200 import program, workloads

    model, x = workloads.build(name, batch)
    prog = program.from_module(model, x, layout=layout)
    (got,) = run_program(prog, x)
    expected = oracle.cim_forward(model, x.numpy(), branches=4, threads=8)
    scale = np.max(np.abs(expected))
    err = np.max(np.abs(got - expected))
    assert err <= 1e-3 * scale, (err, scale)


@pytest.mark.parametrize("layout", ["nchw", "nhwc"])
def test_fused_epilogues_match_separate_glue(layout):
    """Batch norm + ReLU folded into the conv epilogues (and pools into the
    gathers) give the same bits as the separate glue kernels."""
    from cim22_b200 import program, workloads

    model, x = workloads.build("resnet18", 2)
    fused = program.from_module(model, x, layout=layout)
    plain = program.from_module(model, x, fuse=False, layout=layout)
    names = [s.name for s in fused.steps]
    assert "batch_norm" not in names, names
    assert sum(s.name == "batch_norm" for s in plain.steps) == 20
    (a,) = run_program(fused, x)
    (b,) = run_program(plain, x)
    np.testing.assert_array_equal(bits(a), bits(b))


def test_torch_compile_cuda_runtime():
    from cim22_b200 import backend, workloads

    name = backend.register()
    model, x = workloads.build("lenet", 4)
    compiled = torch.compile(model, backend=name, fullgraph=True, dynamic=False,
                             options={"runtime": "cuda"})
    expected = oracle.cim_forward(model, x.numpy(), branches=4, threads=8)
    with torch.inference_mode():
        got = compiled(x)
        assert got.device.type == "cpu"
        np.testing.assert_array_equal(bits(got.numpy()), bits(expected))
        bad = x.clone()
        bad[0, 0, 3, 3] = float("nan")
        with pytest.raises(RuntimeError, match="NaN or infinity"):
            compiled(bad)
        # A failed call does not poison the next one.
        np.testing.assert_array_equal(bits(compiled(x).numpy()), bits(expected))
    # Device-resident inputs go straight to the lowered program (no copies).
    gm = torch.fx.symbolic_trace(model)
    from cim22_b200.program import Program

    prog = Program(gm, [x], device=0)
    got2 = prog(x.to(DEV))
    assert got2.device == DEV
    np.testing.assert_array_equal(bits(got2.cpu().numpy()), bits(expected))


@pytest.mark.parametrize(("transpose_weight", "overflow", "wide_sum"),
                         [(False, False, False), (True, False, False), (False, True, False),
                          (False, False, True)])
def test_torch_compile_int_mm(transpose_weight, overflow, wide_sum):
    """python/tests/test_backend.py:225-330 of the reference: tiled INT8, or
    range-unsafe weights (all -128) computed exactly as the Host does, and
    sums beyond the i21 range of one tile."""
    from cim22_b200 import backend

    name = backend.register()
    reduction, output = (64, 16) if overflow else (128, 17) if wide_sum else (65, 17)

    class Int8Matmul(torch.nn.Module):
        def __init__(self):
            super().__init__()
            shape = (output, reduction) if transpose_weight else (reduction, output)
            w = (torch.arange(reduction * output).reshape(shape) % 15 - 7).to(torch.int8)
            if overflow:
                w.fill_(-128)
            elif wide_sum:
                w.fill_(127)
            self.weight = torch.nn.Parameter(w, requires_grad=False)

        def forward(self, v):
            return torch._int_mm(v, self.weight.t() if transpose_weight else self.weight)

    model = Int8Matmul().eval()
    compiled = torch.compile(model, backend=name, fullgraph=True, dynamic=False,
                             options={"runtime": "cuda"})
    values = [torch.full((2, reduction), 127 if wide_sum else -128, dtype=torch.int8),
              (torch.arange(2 * reduction).reshape(2, reduction) % 256 - 128).to(torch.int8)]
    if wide_sum:
        values[1].fill_(-128)
    weight = model.weight.t() if transpose_weight else model.weight
    for value in (*values, values[0]):
        with torch.inference_mode():
            got = compiled(value)
        assert got.dtype == torch.int32
        exp = (value.to(torch.int64) @ weight.to(torch.int64)).to(torch.int32)
        assert torch.equal(got.cpu(), exp)
        if wide_sum:
            assert torch.all(exp.abs() > 2**20)


def test_torch_compile_int_mm_bias():
    """MatMulInteger + Add (generate_integer_bias_onnx.py): the int32 bias,
    including one that wraps past 2^31, folds into the INT8 epilogue."""
    from cim22_b200 import backend

    name = backend.register()
    g = np.load(Path(__file__).resolve().parent / "golden" / "int8_conv_ref.npz")
    for case in ("linear_bias", "linear_bias_fold", "linear_bias_exact"):
        w, b, x = g[f"{case}.w"], g[f"{case}.bias"], g[f"{case}.x"]

        class Biased(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.weight = torch.nn.Parameter(torch.from_numpy(w), requires_grad=False)
                self.register_buffer("bias", torch.from_numpy(b))

            def forward(self, v):
                return torch._int_mm(v, self.weight) + self.bias

        compiled = torch.compile(Biased().eval(), backend=name, fullgraph=True, dynamic=False,
                                 options={"runtime": "cuda"})
        with torch.inference_mode():
            got = compiled(torch.from_numpy(x))
        np.testing.assert_array_equal(got.cpu().numpy(), g[f"{case}.y"])


@pytest.mark.parametrize("mode", ["legacy", "none"])
def test_torch_compile_diagnostic_compensation_modes(mode):
    """bf16_compensation="legacy" / "none" through torch.compile runtime="cuda"
    against the oracle's layers in the same mode (exact glue: MLP)."""
    from cim22_b200 import backend, workloads

    name = backend.register()
    model, x = workloads.build("mlp", 4)
    compiled = torch.compile(model, backend=name, fullgraph=True, dynamic=False,
                             options={"runtime": "cuda", "bf16_compensation": mode})
    try:
        expected = oracle.cim_forward(model, x.numpy(), compensation=mode)
    except oracle.OracleError as e:
        # None mode hands raw chip bits (non-finite here) to the next layer.
        with torch.inference_mode(), pytest.raises(RuntimeError, match=str(e)):
            compiled(x)
        return
    with torch.inference_mode():
        got = compiled(x).numpy()
    both_nan = np.isnan(got) & np.isnan(expected)
    np.testing.assert_array_equal(np.where(both_nan, 0, bits(got)),
                                  np.where(both_nan, 0, bits(expected)))
