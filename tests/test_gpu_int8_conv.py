"""INT8 Conv / MatMulInteger with bias on the GPU: bit-exact against the
reference corpus outputs (tests/golden/int8_conv_ref.npz) and the oracle."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from cim22_b200 import abi
from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLDEN = Path(__file__).resolve().parent / "golden"
CONV_CASES = ("canonical", "odd", "pointwise", "rectangular", "conv_bias", "conv_bias_fold",
              "conv_bias_exact", "compile_tool0", "compile_tool1")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("name", CONV_CASES)
def test_conv_int8_golden(name):
    g = np.load(GOLDEN / "int8_conv_ref.npz")
    x, w = g[f"{name}.x"], g[f"{name}.w"]
    sh, sw, *pads = (int(v) for v in g[f"{name}.geom"])
    bias = dev(g[f"{name}.bias"]) if f"{name}.bias" in g.files else None
    layer = CimLayer(w.reshape(w.shape[0], -1), kind="int8", device=DEV)
    y = layer.conv2d_int8(dev(x), w.shape[2:], (sh, sw), tuple(pads), bias)
    np.testing.assert_array_equal(y.cpu().numpy(), g[f"{name}.y"])
    # Same result from an NHWC image.
    y2 = layer.conv2d_int8(dev(x.transpose(0, 2, 3, 1)), w.shape[2:], (sh, sw), tuple(pads),
                           bias, layout="nhwc")
    np.testing.assert_array_equal(y2.cpu().numpy(), g[f"{name}.y"])


@pytest.mark.parametrize("name", ("linear_bias", "linear_bias_fold", "linear_bias_exact"))
def test_linear_int8_bias_golden(name):
    g = np.load(GOLDEN / "int8_conv_ref.npz")
    x, w, b = g[f"{name}.x"], g[f"{name}.w"], g[f"{name}.bias"]
    layer = CimLayer(np.ascontiguousarray(w.T), kind="int8", device=DEV)
    m = x.shape[0]
    out = torch.empty(m, w.shape[1], dtype=torch.int32, device=DEV)
    status = StatusWord(DEV)
    layer.forward_int8(dev(x), out, m, bias=dev(b), workspace=Workspace(DEV), status=status)
    status.raise_if_set()
    np.testing.assert_array_equal(out.cpu().numpy(), g[f"{name}.y"])


@pytest.mark.parametrize("n,c,h,w,f,k,stride,pads", [
    (4, 16, 20, 18, 70, (3, 3), (1, 1), (1, 1, 1, 1)),
    (3, 5, 17, 13, 33, (5, 3), (2, 1), (2, 0, 1, 2)),
    (2, 64, 9, 9, 128, (3, 3), (2, 2), (0, 1, 1, 0)),
    (8, 3, 32, 32, 16, (1, 1), (1, 1), (0, 0, 0, 0)),
])
def test_conv_int8_batches_match_oracle(n, c, h, w, f, k, stride, pads):
    rng = np.random.default_rng(n * 1000 + c)
    x = rng.integers(-128, 128, (n, c, h, w)).astype(np.int8)
    wt = rng.integers(-20, 21, (f, c, *k)).astype(np.int8)
    bias = rng.integers(-(1 << 30), 1 << 30, f).astype(np.int32)
    expected = oracle.conv2d_int8(x, wt, bias, stride, pads)
    layer = CimLayer(wt.reshape(f, -1), kind="int8", device=DEV)
    assert layer.range_safe == oracle.int8_range_safe(wt.reshape(f, -1))
    y = layer.conv2d_int8(dev(x), k, stride, pads, dev(bias))
    np.testing.assert_array_equal(y.cpu().numpy(), expected)


def test_unproven_conv_weights_exact_or_checked():
    """All -128 weights fail the proof: exact as the Host computes them, or
    the checked per-tile kernel that rejects an i21 overflow."""
    rng = np.random.default_rng(3)
    wt = np.full((20, 4, 4, 4), -128, np.int8)
    x = rng.integers(-128, 128, (2, 4, 9, 9)).astype(np.int8)
    bias = np.arange(20, dtype=np.int32) * 1000 - 7
    layer = CimLayer(wt.reshape(20, -1), kind="int8", device=DEV)
    assert not layer.range_safe
    expected = oracle.conv2d_int8(x, wt, bias, (1, 1), (0, 0, 0, 0))
    y = layer.conv2d_int8(dev(x), (4, 4), 1, (0, 0, 0, 0), dev(bias))
    np.testing.assert_array_equal(y.cpu().numpy(), expected)
    # Checked tiles (CUDA-core kernel, bias and NCHW epilogue): small inputs pass.
    small = rng.integers(-3, 4, (2, 4, 9, 9)).astype(np.int8)
    y = layer.conv2d_int8(dev(small), (4, 4), 1, (0, 0, 0, 0), dev(bias), exact_unproven=False)
    np.testing.assert_array_equal(y.cpu().numpy(),
                                  oracle.conv2d_int8(small, wt, bias, (1, 1), (0, 0, 0, 0)))
    with pytest.raises(RuntimeError, match="signed i21"):
        layer.conv2d_int8(dev(np.full((2, 4, 9, 9), -128, np.int8)), (4, 4), 1, (0, 0, 0, 0),
                          exact_unproven=False)


def test_int8_rows_out_pixels_and_argument_checks():
    rng = np.random.default_rng(9)
    x = rng.integers(-128, 128, (24, 200)).astype(np.int8)
    w = rng.integers(-127, 128, (40, 200)).astype(np.int8)
    layer = CimLayer(w, kind="int8", device=DEV)
    out = torch.empty(2, 40, 12, dtype=torch.int32, device=DEV)
    status = StatusWord(DEV)
    layer.forward_int8(dev(x), out, 24, out_pixels=12, workspace=Workspace(DEV), status=status)
    status.raise_if_set()
    rows = oracle.linear_int8(x, w)
    np.testing.assert_array_equal(out.cpu().numpy(), rows.reshape(2, 12, 40).transpose(0, 2, 1))
    # out_pixels must divide m; a pooled conv gather is not an INT8 gather.
    with pytest.raises(RuntimeError, match="invalid arguments"):
        layer.forward_int8(dev(x), out, 24, out_pixels=7, workspace=Workspace(DEV), status=status)
    g = abi.Gather()
    g.kind = abi.GATHER_CONV_NCHW
    g.batch, g.channels, g.height, g.width = 1, 8, 5, 5
    g.kernel_h = g.kernel_w = 5
    g.stride_h = g.stride_w = 1
    g.out_h = g.out_w = 1
    g.pool_kernel, g.pool_stride, g.pool_src_h, g.pool_src_w = 2, 2, 10, 10
    with pytest.raises(RuntimeError, match="invalid arguments"):
        layer.forward_int8(dev(np.zeros((1, 8, 10, 10), np.int8)), out, 1, gather=g,
                           workspace=Workspace(DEV), status=status)


def test_int8_persistent_kernel_large_linear():
    """Shapes with enough 128 x 256 tiles for every SM take the persistent
    kernel (two TMEM accumulators, ragged M, N and K): exact int32 sums."""
    from cim22_b200.native import lib

    rng = np.random.default_rng(21)
    m, k, n = 4133, 1000, 2053
    x = rng.integers(-128, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    bias = rng.integers(-1000, 1000, n).astype(np.int32)
    layer = CimLayer(w, kind="int8", device=DEV)
    assert layer.range_safe
    out = torch.empty(m, n, dtype=torch.int32, device=DEV)
    before = lib().cim22_cuda_tensor_core_launches()
    status = StatusWord(DEV)
    layer.forward_int8(dev(x), out, m, bias=dev(bias), workspace=Workspace(DEV), status=status)
    status.raise_if_set()
    assert lib().cim22_cuda_tensor_core_launches() == before + 1
    exact = (x.astype(np.float64) @ w.T.astype(np.float64)).astype(np.int64) + bias
    np.testing.assert_array_equal(out.cpu().numpy(), exact.astype(np.int32))


def test_int8_persistent_kernel_conv_nchw():
    rng = np.random.default_rng(22)
    x = rng.integers(-128, 128, (64, 16, 32, 32)).astype(np.int8)
    wt = rng.integers(-20, 21, (64, 16, 3, 3)).astype(np.int8)
    bias = rng.integers(-(1 << 20), 1 << 20, 64).astype(np.int32)
    layer = CimLayer(wt.reshape(64, -1), kind="int8", device=DEV)
    y = layer.conv2d_int8(dev(x), (3, 3), 1, (1, 1, 1, 1), dev(bias))
    np.testing.assert_array_equal(y.cpu().numpy(),
                                  oracle.conv2d_int8(x, wt, bias, (1, 1), (1, 1, 1, 1)))
