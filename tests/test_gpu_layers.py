"""Layer-level CUDA kernels against the oracle (bit-exact) and glue against
PyTorch CPU eager f32 (the reference's own float oracle, 1e-3 relative)."""

import itertools

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_doc_example_on_gpu():
    from cim22_b200.cim_ops import CimLayer

    layer = CimLayer(np.full((16, 64), 0.5, np.float32))
    y = layer.linear_bf16(torch.ones(1, 64, device=DEV))
    assert torch.all(y == 32.0)


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (3, 64, 16), (37, 150, 20), (130, 400, 120),
                                   (64, 784, 256), (5, 4096, 33), (200, 25, 6)])
@pytest.mark.parametrize("branches", [2, 4])
def test_linear_bf16_bit_exact(m, k, n, branches):
    from cim22_b200.cim_ops import CimLayer

    rng = np.random.default_rng(m * 1000 + k + n + branches)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[rng.random((m, k)) < 0.01] *= 20
    if branches == 2:
        x = np.maximum(x, 0)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    expected = oracle.linear_bf16(x, w, b, branches=4, threads=8)
    layer = CimLayer(w)
    got = layer.linear_bf16(torch.from_numpy(x).to(DEV), bias=torch.from_numpy(b).to(DEV),
                            branches=branches).cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(expected))


def test_linear_bf16_extreme_exponents_slow_path():
    """Scales far from 2^0 force the exact subnormal/overflow restore path."""
    from cim22_b200.cim_ops import CimLayer

    rng = np.random.default_rng(3)
    for (scale_x, scale_w), k in itertools.product(
            ((1e-30, 1e-8), (1e-38, 1.0), (1e20, 1e-20), (1e-20, 1e-20)), (130, 50)):
        x = (rng.standard_normal((17, k)) * scale_x).astype(np.float32)
        w = (rng.standard_normal((19, k)) * scale_w).astype(np.float32)
        expected = oracle.linear_bf16(x, w, None, branches=4)
        got = CimLayer(w).linear_bf16(torch.from_numpy(x).to(DEV)).cpu().numpy()
        np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("scale_w", [1e-37, 1e36])
def test_wide_layer_with_extreme_weights_keeps_int8_operands(scale_w):
    """A 300-lane layer whose weight exponents fall outside the BF16 operand
    range (below 8: |w| < 2^-119; above 241: |w| >= 2^114) keeps int8
    mantissas and the int8 tensor-core kernel, bit-exact with the oracle."""
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace
    from cim22_b200.native import lib

    rng = np.random.default_rng(5)
    m, k, n = 600, 200, 300
    x = rng.standard_normal((m, k)).astype(np.float32)
    x *= (1e-10 if scale_w > 1 else 1e10)  # keep the tile values finite and normal
    w = (rng.standard_normal((n, k)) * scale_w).astype(np.float32)
    expected = oracle.linear_bf16(x, w, None, branches=4, threads=8)
    layer = CimLayer(w)
    assert not layer.bf16_operands
    xt = torch.from_numpy(x).to(DEV)
    ws, status = Workspace(torch.device(DEV)), StatusWord(torch.device(DEV))
    out = torch.empty(m, n, device=DEV)
    before = lib().cim22_cuda_tensor_core_launches()
    layer.prepare_bf16(xt, m, branches=4, workspace=ws, status=status)
    layer.contract_bf16(out, m, branches=4, workspace=ws, status=status)
    status.raise_if_set()
    assert lib().cim22_cuda_tensor_core_launches() == before + 1
    np.testing.assert_array_equal(bits(out.cpu().numpy()), bits(expected))


def test_linear_bf16_overflow_and_nan_status():
    from cim22_b200.cim_ops import CimLayer

    w = np.full((16, 64), 3e38, np.float32)
    x = np.full((1, 64), 3e38, np.float32)
    with pytest.raises(oracle.OracleError, match="exceeds BF16"):
        oracle.linear_bf16(x, w)
    with pytest.raises(RuntimeError, match="exceeds BF16"):
        CimLayer(w).linear_bf16(torch.from_numpy(x).to(DEV))
    x = np.ones((2, 64), np.float32)
    x[1, 5] = np.nan
    with pytest.raises(RuntimeError, match="NaN or infinity"):
        CimLayer(np.ones((4, 64), np.float32)).linear_bf16(torch.from_numpy(x).to(DEV))


@pytest.mark.parametrize("layout", ["nchw", "nhwc"])
@pytest.mark.parametrize("c,h,f,kk,stride,pad", [(1, 32, 6, 5, 1, 0), (6, 14, 16, 5, 1, 0),
                                                 (3, 9, 8, 3, 2, 1), (2, 16, 32, 3, 1, 1)])
def test_conv_bf16_bit_exact(layout, c, h, f, kk, stride, pad):
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(c * 100 + h + f)
    n = 3
    x = rng.standard_normal((n, c, h, h)).astype(np.float32)
    w = (rng.standard_normal((f, c, kk, kk)) * 0.2).astype(np.float32)
    b = rng.standard_normal(f).astype(np.float32)
    expected = oracle.conv2d_bf16(x, w, b, stride, pad, branches=4)  # NCHW
    layer = CimLayer(w.reshape(f, -1))
    kind = abi.GATHER_CONV_NCHW if layout == "nchw" else abi.GATHER_CONV_NHWC
    g = conv_gather(kind, n, c, h, h, kk, kk, stride, pad)
    xt = torch.from_numpy(x if layout == "nchw" else x.transpose(0, 2, 3, 1).copy()).to(DEV)
    m = n * g.out_h * g.out_w
    out = torch.empty(m, f, device=DEV)
    status = StatusWord(torch.device(DEV))
    layer.forward_bf16(xt, out, m, gather=g, bias=torch.from_numpy(b).to(DEV),
                       workspace=Workspace(torch.device(DEV)), status=status)
    status.raise_if_set()
    got = out.cpu().numpy().reshape(n, g.out_h, g.out_w, f).transpose(0, 3, 1, 2)
    np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("layout,n,c,h,f,kk,stride,pad,branches,pool", [
    ("nhwc", 64, 16, 32, 64, 3, 1, 1, 4, 0),   # several columns per prepare thread
    ("nhwc", 64, 16, 32, 64, 3, 1, 1, 2, 0),
    ("nchw", 64, 16, 32, 64, 3, 1, 1, 2, 0),
    ("nchw", 48, 3, 40, 32, 5, 2, 2, 4, 0),    # K = 75: ragged K tail
    ("nhwc", 32, 8, 34, 48, 3, 2, 0, 2, 0),
    ("nchw", 40, 6, 14, 16, 5, 1, 0, 2, 2),    # LeNet conv2 shape over a fused pool
    ("nchw", 64, 32, 16, 32, 3, 1, 1, 4, 2),
    ("nhwc", 64, 32, 16, 32, 3, 1, 1, 4, 2),   # fused 2x2 max pool over 32x32
    # 256 lanes: BF16 operand values from every prepare kernel (TMA-staged
    # whole rows and whole images, thread per group over a fused pool, eight
    # threads per group) into the contraction with BF16 operands, several
    # lane blocks per output row
    ("nchw", 16, 64, 16, 256, 3, 1, 1, 2, 0),
    ("nchw", 8, 32, 16, 256, 3, 2, 1, 4, 0),
    ("nchw", 16, 32, 8, 256, 3, 1, 1, 2, 2),
    ("nhwc", 16, 32, 16, 256, 3, 1, 1, 4, 0)])
@pytest.mark.parametrize("out_layout", ["rows", "nchw"])
def test_conv_bf16_large_batch_bit_exact(layout, n, c, h, f, kk, stride, pad, branches, pool,
                                         out_layout):
    """Batches large enough that each prepare thread serves several columns
    and the tensor-core contraction runs, for both input layouts, both
    branch counts, ragged K and a fused max pool, with the output as [m, n]
    rows or as NCHW planes."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(n * 7 + c + h + f + pool)
    src = h * 2 if pool else h
    x = rng.standard_normal((n, c, src, src)).astype(np.float32)
    if branches == 2:
        x = np.maximum(x, 0)
    x[rng.random(x.shape) < 0.2] = 0
    pooled = x.reshape(n, c, h, 2, h, 2).max(axis=(3, 5)) if pool else x
    w = (rng.standard_normal((f, c, kk, kk)) * 0.2).astype(np.float32)
    b = rng.standard_normal(f).astype(np.float32)
    expected = oracle.conv2d_bf16(pooled, w, b, stride, pad, branches=4, threads=8)
    layer = CimLayer(w.reshape(f, -1))
    assert layer.bf16_operands == (f >= 64)
    kind = abi.GATHER_CONV_NCHW if layout == "nchw" else abi.GATHER_CONV_NHWC
    g = conv_gather(kind, n, c, h, h, kk, kk, stride, pad)
    if pool:
        g.pool_kernel, g.pool_stride, g.pool_src_h, g.pool_src_w = 2, 2, src, src
    xt = torch.from_numpy(x if layout == "nchw" else x.transpose(0, 2, 3, 1).copy()).to(DEV)
    m = n * g.out_h * g.out_w
    out = torch.empty(m, f, device=DEV)
    status = StatusWord(torch.device(DEV))
    pixels = g.out_h * g.out_w if out_layout == "nchw" else 0
    layer.forward_bf16(xt, out, m, gather=g, bias=torch.from_numpy(b).to(DEV),
                       branches=branches, out_pixels=pixels,
                       workspace=Workspace(torch.device(DEV)), status=status)
    status.raise_if_set()
    if out_layout == "nchw":
        got = out.cpu().numpy().reshape(n, f, g.out_h, g.out_w)
    else:
        got = out.cpu().numpy().reshape(n, g.out_h, g.out_w, f).transpose(0, 3, 1, 2)
    np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("m,k,n", [(2, 65, 17), (2, 128, 17), (33, 1000, 70), (300, 64, 16)])
def test_linear_int8_exact(m, k, n):
    from cim22_b200.cim_ops import CimLayer

    rng = np.random.default_rng(k)
    x = rng.integers(-128, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    layer = CimLayer(w, kind="int8")
    assert layer.range_safe == oracle.int8_range_safe(w)
    got = layer.linear_int8(torch.from_numpy(x).to(DEV)).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.linear_int8(x, w))
    np.testing.assert_array_equal(got, (x.astype(np.int64) @ w.T.astype(np.int64)).astype(np.int32))


def test_linear_int8_unproven_weights_report_i21():
    from cim22_b200.cim_ops import CimLayer

    w = np.full((16, 64), -128, np.int8)
    layer = CimLayer(w, kind="int8")
    assert not layer.range_safe
    ok = np.zeros((1, 64), np.int8)
    ok[0, 0] = 3
    np.testing.assert_array_equal(layer.linear_int8(torch.from_numpy(ok).to(DEV)).cpu().numpy(),
                                  oracle.linear_int8(ok, w))
    with pytest.raises(RuntimeError, match="signed i21"):
        layer.linear_int8(torch.from_numpy(np.full((1, 64), -128, np.int8)).to(DEV))


def test_glue_against_torch_cpu():
    from cim22_b200 import cim_ops

    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal((4, 10, 12, 7)).astype(np.float32))
    y = torch.from_numpy(rng.standard_normal((4, 10, 12, 7)).astype(np.float32))
    xd, yd = x.to(DEV), y.to(DEV)
    tol = dict(rtol=1e-3, atol=1e-6)
    torch.testing.assert_close(cim_ops.relu(xd).cpu(), torch.relu(x), **tol)
    torch.testing.assert_close(cim_ops.gelu(xd).cpu(), torch.nn.functional.gelu(x), **tol)
    torch.testing.assert_close(cim_ops.add(xd, yd, "relu").cpu(), torch.relu(x + y), **tol)
    nchw = x.permute(0, 3, 1, 2)
    torch.testing.assert_close(cim_ops.maxpool2d_nhwc(xd, 2, 2).cpu(),
                               torch.nn.functional.max_pool2d(nchw, 2, 2).permute(0, 2, 3, 1), **tol)
    torch.testing.assert_close(cim_ops.maxpool2d_nhwc(xd, 3, 2, 1).cpu(),
                               torch.nn.functional.max_pool2d(nchw, 3, 2, 1).permute(0, 2, 3, 1),
                               **tol)
    torch.testing.assert_close(cim_ops.avgpool2d_nhwc(xd, 2, 2).cpu(),
                               torch.nn.functional.avg_pool2d(nchw, 2, 2).permute(0, 2, 3, 1), **tol)
    torch.testing.assert_close(cim_ops.global_avgpool_nhwc(xd).cpu(), nchw.mean((2, 3)), **tol)
    scale = torch.rand(7) + 0.5
    shift = torch.randn(7)
    torch.testing.assert_close(
        cim_ops.channel_affine_nhwc(xd, scale.to(DEV), shift.to(DEV), "relu").cpu(),
        torch.relu(x * scale + shift), **tol)
    flat = x.reshape(-1, 7)
    torch.testing.assert_close(cim_ops.softmax(flat.to(DEV)).cpu(), torch.softmax(flat, -1), **tol)
    torch.testing.assert_close(cim_ops.nhwc_to_nchw(xd).cpu(), nchw.contiguous(), rtol=0, atol=0)
    torch.testing.assert_close(cim_ops.nchw_to_nhwc(nchw.contiguous().to(DEV)).cpu(), x,
                               rtol=0, atol=0)
    # NCHW variants, exact where torch's CPU result is exact.
    nd = nchw.contiguous().to(DEV)
    torch.testing.assert_close(cim_ops.maxpool2d_nchw(nd, 2, 2).cpu(),
                               torch.nn.functional.max_pool2d(nchw, 2, 2), rtol=0, atol=0)
    torch.testing.assert_close(cim_ops.maxpool2d_nchw(nd, 3, 2, 1).cpu(),
                               torch.nn.functional.max_pool2d(nchw, 3, 2, 1), rtol=0, atol=0)
    torch.testing.assert_close(cim_ops.avgpool2d_nchw(nd, 2, 2).cpu(),
                               torch.nn.functional.avg_pool2d(nchw, 2, 2), **tol)
    torch.testing.assert_close(cim_ops.global_avgpool_nchw(nd).cpu(), nchw.mean((2, 3)), **tol)
    # Planes of at most 64 elements (one thread per plane), ResNet-18's 4x4 among them.
    for shape in [(64, 512, 4, 4), (3, 5, 2, 6), (2, 3, 8, 8)]:
        small = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
        torch.testing.assert_close(cim_ops.global_avgpool_nchw(small.to(DEV)).cpu(),
                                   small.mean((2, 3)), **tol)
    torch.testing.assert_close(
        cim_ops.channel_affine_nchw(nd, scale.to(DEV), shift.to(DEV), "relu").cpu(),
        torch.relu(nchw * scale[:, None, None] + shift[:, None, None]), **tol)
    # More planes than one grid dimension holds.
    big = torch.randn(1100, 64, 2, 2)
    bs, bb = torch.rand(64) + 0.5, torch.randn(64)
    torch.testing.assert_close(
        cim_ops.channel_affine_nchw(big.to(DEV), bs.to(DEV), bb.to(DEV)).cpu(),
        big * bs[:, None, None] + bb[:, None, None], **tol)


@pytest.mark.parametrize("pool", [0, 2])
def test_conv_with_fused_pool_and_flatten_gathers(pool):
    """Max pool folded into the conv gather, and flatten->Linear as a conv whose
    kernel covers the whole (pooled) NHWC image."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(17 + pool)
    n, c, src = 3, 6, 28
    pre = rng.standard_normal((n, src, src, c)).astype(np.float32)  # NHWC, pre-pool
    if pool:
        pooled = pre.reshape(n, src // 2, 2, src // 2, 2, c).max(axis=(2, 4))
    else:
        pooled = pre
    h = pooled.shape[1]
    dev = torch.device(DEV)
    status = StatusWord(dev)
    # conv 5x5 on the pooled image
    w = (rng.standard_normal((16, c, 5, 5)) * 0.2).astype(np.float32)
    g = conv_gather(abi.GATHER_CONV_NHWC, n, c, h, h, 5, 5, 1, 0)
    if pool:
        g.pool_kernel, g.pool_stride, g.pool_src_h, g.pool_src_w = 2, 2, src, src
    m = n * g.out_h * g.out_w
    out = torch.empty(m, 16, device=dev)
    CimLayer(w.reshape(16, -1)).forward_bf16(torch.from_numpy(pre).to(dev), out, m, gather=g,
                                             workspace=Workspace(dev), status=status)
    status.raise_if_set()
    exp = oracle.conv2d_bf16(pooled.transpose(0, 3, 1, 2).copy(), w, None, 1, 0)
    got = out.cpu().numpy().reshape(n, g.out_h, g.out_w, 16).transpose(0, 3, 1, 2)
    np.testing.assert_array_equal(bits(got), bits(exp))
    # flatten (NCHW order) -> Linear via the whole-image conv gather
    wl = (rng.standard_normal((30, c * h * h)) * 0.05).astype(np.float32)
    gf = conv_gather(abi.GATHER_CONV_NHWC, n, c, h, h, h, h, 1, 0)
    if pool:
        gf.pool_kernel, gf.pool_stride, gf.pool_src_h, gf.pool_src_w = 2, 2, src, src
    outl = torch.empty(n, 30, device=dev)
    CimLayer(wl).forward_bf16(torch.from_numpy(pre).to(dev), outl, n, gather=gf,
                              workspace=Workspace(dev), status=status)
    status.raise_if_set()
    flat = pooled.transpose(0, 3, 1, 2).reshape(n, -1)
    np.testing.assert_array_equal(bits(outl.cpu().numpy()), bits(oracle.linear_bf16(flat, wl)))


@pytest.mark.parametrize("m,k,n", [(1000, 4096, 1000), (4096, 256, 256), (129, 8192, 130)])
def test_linear_int8_tensor_core_shapes(m, k, n):
    """Range-proven INT8 layers run whole-K int32 accumulation on tcgen05."""
    from cim22_b200.cim_ops import CimLayer

    rng = np.random.default_rng(m + k + n)
    x = rng.integers(-128, 128, (m, k)).astype(np.int8)
    w = rng.integers(-8, 8, (n, k)).astype(np.int8)  # provably in range
    from cim22_b200.native import lib

    layer = CimLayer(w, kind="int8")
    assert layer.range_safe
    before = lib().cim22_cuda_tensor_core_launches()
    got = layer.linear_int8(torch.from_numpy(x).to(DEV)).cpu().numpy()
    assert lib().cim22_cuda_tensor_core_launches() == before + 1
    exp = (x.astype(np.int64) @ w.T.astype(np.int64)).astype(np.int32)
    np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("m,k,n,branches,scale", [
    (1024, 4096, 512, 4, 1.0), (2000, 150, 40, 2, 1.0), (777, 640, 96, 4, 1.0),
    (600, 200, 64, 4, 1e-30), (512, 64, 32, 4, 1e18),
    # one crossbar tile, hundreds of output tiles per persistent CTA
    (40000, 18, 64, 4, 1.0), (30000, 27, 32, 2, 1.0),
    # odd tile count, several output tiles per CTA
    (5000, 300, 160, 4, 1.0),
    # per-row scales from 1e-38 to 1e30: fast and exact-path rows share a
    # CTA, and whole rows of zero groups
    (3000, 256, 96, 4, "rows"), (2048, 130, 64, 2, "rows"), (3000, 256, 48, 4, "rows"),
    (2048, 130, 40, 2, "rows"),
    # BF16 operands over many output tiles, with unscaled groups (rows
    # outside the layer's exponent window) restored exactly
    (3000, 256, 300, 4, "rows"), (2048, 130, 256, 2, "rows"), (700, 640, 260, 4, 1.0),
    (512, 4096, 512, 2, 1.0), (600, 200, 320, 4, 1e-30), (512, 64, 256, 4, 1e18)])
def test_linear_bf16_tensor_core_bit_exact(m, k, n, branches, scale):
    """Wide layers run a tcgen05 sign-split kernel (launch counter checked):
    int8 mantissas below 64 lanes, BF16 operands from 64 lanes on. The
    prepare + contract form always takes it; one-tile layers of at most 64
    lanes, which forward_bf16 runs as one thread-per-column kernel, are
    checked through both."""
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace
    from cim22_b200.native import lib

    rng = np.random.default_rng(m + k + n)
    if scale == "rows":
        x = rng.standard_normal((m, k)).astype(np.float64)
        x *= 10.0 ** rng.uniform(-38, 30, (m, 1))
        x[rng.random(m) < 0.1] = 0
        x = x.astype(np.float32)
    else:
        x = (rng.standard_normal((m, k)) * scale).astype(np.float32)
    x[rng.random((m, k)) < 0.01] *= 20
    if branches == 2:
        x = np.maximum(x, 0)
    x[rng.random((m, k)) < 0.3] = 0  # zero groups and sparse inputs
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    expected = oracle.linear_bf16(x, w, b, branches=4, threads=8)
    layer = CimLayer(w)
    assert layer.bf16_operands == (n >= 64)
    xt, bt = torch.from_numpy(x).to(DEV), torch.from_numpy(b).to(DEV)
    ws, status = Workspace(torch.device(DEV)), StatusWord(torch.device(DEV))
    out = torch.empty(m, n, device=DEV)
    before = lib().cim22_cuda_tensor_core_launches()
    layer.prepare_bf16(xt, m, branches=branches, workspace=ws, status=status)
    layer.contract_bf16(out, m, bias=bt, branches=branches, workspace=ws, status=status)
    status.raise_if_set()
    assert lib().cim22_cuda_tensor_core_launches() == before + 1
    np.testing.assert_array_equal(bits(out.cpu().numpy()), bits(expected))
    if layer.fused_forward:
        got = layer.linear_bf16(xt, bias=bt, branches=branches).cpu().numpy()
        np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("layout,n,c,h,f,kk,stride,pad,branches,pool", [
    ("nchw", 64, 1, 32, 6, 5, 1, 0, 4, 0),    # LeNet conv1: K = 25, 6 lanes
    ("nchw", 16, 3, 20, 8, 3, 2, 1, 2, 0),
    ("nhwc", 16, 2, 18, 5, 3, 1, 1, 4, 0),
    ("nchw", 16, 4, 10, 7, 3, 1, 0, 2, 2),    # fused 2x2 pool, K = 36
    ("nhwc", 8, 1, 12, 1, 7, 1, 3, 4, 2),     # K = 49, one lane
    ("nchw", 32, 2, 16, 12, 5, 1, 2, 4, 0),   # 12 lanes, K = 50: fused CUDA-core kernel
    ("nchw", 32, 4, 12, 16, 5, 1, 2, 2, 0),   # 16 lanes, K = 100: two tiles, fused
    ("nchw", 8, 2, 24, 32, 3, 1, 1, 2, 0),    # event-frame conv0: K = 18, 32 lanes, direct
    ("nchw", 4, 1, 20, 64, 8, 1, 3, 4, 0),    # K = 64, 64 lanes
    ("nhwc", 4, 3, 8, 40, 3, 2, 1, 4, 2),     # fused pool, K = 27, 40 lanes
    ("nchw", 6, 5, 12, 48, 3, 1, 1, 2, 0)])   # K = 45, 48 lanes
@pytest.mark.parametrize("out_layout", ["rows", "nchw"])
def test_narrow_fused_layers_bit_exact(layout, n, c, h, f, kk, stride, pad, branches, pool,
                                       out_layout):
    """Layers of one K tile and at most 64 lanes (one thread per column), or of
    at most 16 lanes and two K tiles (the CUDA-core contraction building its
    own activation tiles), run as one kernel: bit-exact against the oracle."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(n + c * 7 + h + f * 3 + pool)
    src = h * 2 if pool else h
    x = rng.standard_normal((n, c, src, src)).astype(np.float32)
    x *= (10.0 ** rng.uniform(-30, 30, (n, 1, 1, 1))).astype(np.float32)  # exact-path images
    if branches == 2:
        x = np.maximum(x, 0)
    x[rng.random(x.shape) < 0.2] = 0
    pooled = x.reshape(n, c, h, 2, h, 2).max(axis=(3, 5)) if pool else x
    w = (rng.standard_normal((f, c, kk, kk)) * 0.2).astype(np.float32)
    b = rng.standard_normal(f).astype(np.float32)
    expected = oracle.conv2d_bf16(pooled, w, b, stride, pad, branches=4, threads=8)
    layer = CimLayer(w.reshape(f, -1))
    assert layer.fused_forward
    kind = abi.GATHER_CONV_NCHW if layout == "nchw" else abi.GATHER_CONV_NHWC
    g = conv_gather(kind, n, c, h, h, kk, kk, stride, pad)
    if pool:
        g.pool_kernel, g.pool_stride, g.pool_src_h, g.pool_src_w = 2, 2, src, src
    xt = torch.from_numpy(x if layout == "nchw" else x.transpose(0, 2, 3, 1).copy()).to(DEV)
    m = n * g.out_h * g.out_w
    out = torch.empty(m, f, device=DEV)
    status = StatusWord(torch.device(DEV))
    pixels = g.out_h * g.out_w if out_layout == "nchw" else 0
    # NCHW outputs take a fused ReLU (the branch-free epilogue of the direct kernel).
    act = "relu" if out_layout == "nchw" else None
    layer.forward_bf16(xt, out, m, gather=g, bias=torch.from_numpy(b).to(DEV),
                       activation=act, branches=branches, out_pixels=pixels,
                       workspace=Workspace(torch.device(DEV)), status=status)
    status.raise_if_set()
    if out_layout == "nchw":
        got = out.cpu().numpy().reshape(n, f, g.out_h, g.out_w)
        expected = np.where(expected > 0, expected, np.float32(0))
    else:
        got = out.cpu().numpy().reshape(n, g.out_h, g.out_w, f).transpose(0, 3, 1, 2)
    np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("f,branches", [(6, 4), (40, 2), (96, 4)])
def test_contract_residual_epilogue_bit_exact(f, branches):
    """contract_bf16 with a residual: y = relu(conv + residual), bit-exact
    against the oracle conv followed by the f32 glue (CUDA-core contraction
    for 6 lanes, tcgen05 above). The batch norm before the add is covered by
    the fused-versus-glue ResNet-18 program test."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(f + branches)
    n, c, h = 3, 8, 12
    x = rng.standard_normal((n, c, h, h)).astype(np.float32)
    if branches == 2:
        x = np.maximum(x, 0)
    w = (rng.standard_normal((f, c, 3, 3)) * 0.2).astype(np.float32)
    res = rng.standard_normal((n, f, h, h)).astype(np.float32)
    bn = oracle.conv2d_bf16(x, w, None, 1, 1, branches=4, threads=8)
    expected = (bn + res).astype(np.float32)
    expected = np.where(expected > 0, expected, np.float32(0))
    layer = CimLayer(w.reshape(f, -1))
    g = conv_gather(abi.GATHER_CONV_NCHW, n, c, h, h, 3, 3, 1, 1)
    m = n * h * h
    ws, status = Workspace(torch.device(DEV)), StatusWord(torch.device(DEV))
    out = torch.empty(m, f, device=DEV)
    layer.prepare_bf16(torch.from_numpy(x).to(DEV), m, gather=g, branches=branches,
                       workspace=ws, status=status)
    layer.contract_bf16(out, m, activation="relu", branches=branches, out_pixels=h * h,
                        residual=torch.from_numpy(res).to(DEV), workspace=ws, status=status)
    status.raise_if_set()
    got = out.cpu().numpy().reshape(n, f, h, h)
    np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("f,n", [(64, 3), (128, 2)])
def test_residual_bf16_operand_conv_many_tiles(f, n):
    """A 64-channel 3x3 residual conv (9 crossbar tiles per output tile, BF16
    operands, 2 branches) through the residual instance, whose stage ring has
    an odd number of stages. Bit-exact against the oracle, and the launch
    ends in well under the pipelines' 2 s wait limit: an exit drain that
    waits on a stage parity it will never see shows up as a launch of about
    2 s, not as a wrong result."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(f * 7 + n)
    c, h = 64, 8
    x = np.maximum(rng.standard_normal((n, c, h, h)), 0).astype(np.float32)
    w = (rng.standard_normal((f, c, 3, 3)) * 0.1).astype(np.float32)
    res = rng.standard_normal((n, f, h, h)).astype(np.float32)
    conv = oracle.conv2d_bf16(x, w, None, 1, 1, branches=4, threads=8)
    expected = (conv + res).astype(np.float32)
    expected = np.where(expected > 0, expected, np.float32(0))
    layer = CimLayer(w.reshape(f, -1))
    g = conv_gather(abi.GATHER_CONV_NCHW, n, c, h, h, 3, 3, 1, 1)
    m = n * h * h
    dev = torch.device(DEV)
    ws, status = Workspace(dev), StatusWord(dev)
    out = torch.empty(m, f, device=DEV)
    xt, rt = torch.from_numpy(x).to(DEV), torch.from_numpy(res).to(DEV)
    layer.prepare_bf16(xt, m, gather=g, branches=2, workspace=ws, status=status)
    assert layer.bf16_operands
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    layer.contract_bf16(out, m, activation="relu", branches=2, out_pixels=h * h, residual=rt,
                        workspace=ws, status=status)
    end.record()
    torch.cuda.synchronize()
    status.raise_if_set()
    assert start.elapsed_time(end) < 500.0
    got = out.cpu().numpy().reshape(n, f, h, h)
    np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("act", [None, "relu"])
def test_direct_conv_dead_negative_branch(act):
    """A 4-branch one-tile conv over binary event frames, with negative pixels
    in some images: warps whose xn groups are all zero take the 2-branch merge,
    the others all four branches; bit-exact either way."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(11)
    n, c, h, f = 6, 2, 40, 32
    x = (rng.random((n, c, h, h)) < 0.05).astype(np.float32)
    x[3] *= -1.0                 # an image of non-positive pixels
    x[4, :, 10:20, :] -= 0.5     # negative rows inside an image
    w = (rng.standard_normal((f, c, 3, 3)) * 0.3).astype(np.float32)
    b = rng.standard_normal(f).astype(np.float32)
    expected = oracle.conv2d_bf16(x, w, b, 1, 1, branches=4, threads=8)
    if act == "relu":
        expected = np.where(expected > 0, expected, np.float32(0))
    layer = CimLayer(w.reshape(f, -1))
    assert layer.fused_forward
    g = conv_gather(abi.GATHER_CONV_NCHW, n, c, h, h, 3, 3, 1, 1)
    m = n * h * h
    out = torch.empty(m, f, device=DEV)
    status = StatusWord(torch.device(DEV))
    layer.forward_bf16(torch.from_numpy(x).to(DEV), out, m, gather=g,
                       bias=torch.from_numpy(b).to(DEV), activation=act, branches=4,
                       out_pixels=h * h, workspace=Workspace(torch.device(DEV)), status=status)
    status.raise_if_set()
    got = out.cpu().numpy().reshape(n, f, h, h)
    np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("m,k,n,branches", [(300, 25, 6, 4), (129, 64, 8, 2), (77, 100, 10, 4),
                                            (1000, 3, 1, 2), (300, 64, 64, 2), (50, 40, 33, 4)])
def test_narrow_fused_linear_bit_exact(m, k, n, branches):
    from cim22_b200.cim_ops import CimLayer

    rng = np.random.default_rng(m + k + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if branches == 2:
        x = np.maximum(x, 0)
    w = (rng.standard_normal((n, k)) * 0.1).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    layer = CimLayer(w)
    assert layer.fused_forward
    got = layer.linear_bf16(torch.from_numpy(x).to(DEV), bias=torch.from_numpy(b).to(DEV),
                            branches=branches).cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(oracle.linear_bf16(x, w, b)))


def nan_equal_bits(a, b):
    """Bit equality with every NaN treated alike (the None mode returns raw
    chip bits, and NaN payloads after f32 adds are not specified)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    return np.array_equal(np.where(both_nan, 0, a.view(np.uint32)),
                          np.where(both_nan, 0, b.view(np.uint32)))


@pytest.mark.parametrize("mode", ["legacy", "none"])
@pytest.mark.parametrize("m,k,n,scale", [(70, 150, 40, 1.0), (300, 64, 16, 1e-3),
                                         (33, 400, 130, 1e20), (5, 7, 3, 1e-25)])
def test_linear_bf16_legacy_none_modes(mode, m, k, n, scale):
    """The reference's diagnostic BF16 modes at layer level, vs the oracle."""
    from cim22_b200.cim_ops import CimLayer

    rng = np.random.default_rng(m + k + n)
    x = (rng.standard_normal((m, k)) * scale).astype(np.float32)
    x[rng.random((m, k)) < 0.2] = 0
    w = (rng.standard_normal((n, k)) * 0.1).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    layer = CimLayer(w, compensation=mode)
    try:
        expected = oracle.linear_bf16_mode(x, w, b, mode)
    except oracle.OracleError as e:
        with pytest.raises(RuntimeError, match=str(e)):
            layer.linear_bf16(torch.from_numpy(x).to(DEV), bias=torch.from_numpy(b).to(DEV))
        return
    got = layer.linear_bf16(torch.from_numpy(x).to(DEV), bias=torch.from_numpy(b).to(DEV))
    assert nan_equal_bits(got.cpu().numpy(), expected)


def test_legacy_mode_errors_match_reference_texts():
    from cim22_b200.cim_ops import CimLayer

    # All -128 prealigned input and weight lane (-1.9921875 = BF16 0xbfff,
    # mantissa 0xff at the group exponent): validateBF16Group rejects it.
    x = np.full((2, 64), -1.9921875, np.float32)
    w = np.full((3, 64), -1.9921875, np.float32)
    with pytest.raises(RuntimeError, match="exceeds signed i21 range"):
        oracle.linear_bf16_mode(x, w, None, "legacy")
    with pytest.raises(RuntimeError, match="CIM BF16 result exceeds signed i21 range"):
        CimLayer(w, compensation="legacy").linear_bf16(torch.from_numpy(x).to(DEV))
    # NaN input.
    x = np.ones((2, 64), np.float32)
    x[1, 3] = np.nan
    with pytest.raises(RuntimeError, match="NaN or infinity"):
        CimLayer(np.ones((4, 64), np.float32), compensation="none").linear_bf16(
            torch.from_numpy(x).to(DEV))


def test_relu_propagates_nan_like_torch():
    from cim22_b200 import cim_ops

    x = torch.tensor([float("nan"), -1.0, 2.0, float("-inf"), float("inf"), -0.0])
    got = cim_ops.relu(x.to(DEV)).cpu()
    torch.testing.assert_close(got, torch.relu(x), equal_nan=True, rtol=0, atol=0)


@pytest.mark.parametrize("layout,n,c,h,f,kk,stride,pad", [
    ("nchw", 64, 16, 32, 64, 3, 1, 1),   # TMA-staged window gather
    ("nchw", 64, 16, 30, 32, 3, 1, 1),   # thread-per-group NCHW gather
    ("nhwc", 64, 16, 32, 64, 3, 1, 1),   # NHWC gather
    ("nchw", 4, 1, 28, 6, 5, 1, 0),      # one-tile direct kernel
    ("rows", 512, 256, 0, 128, 0, 0, 0)])  # Linear rows
def test_two_branch_signed_zero_and_negative_input(layout, n, c, h, f, kk, stride, pad):
    """A 2-branch layer (nonnegative input) clears -0 to +0, as the
    reference's preparation does, and rejects a negative nonzero input with
    the reference's error text, on every prepare path."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    rng = np.random.default_rng(n + c + h + f)
    shape = (n, c) if layout == "rows" else (n, c, h, h)
    x = np.maximum(rng.standard_normal(shape), 0).astype(np.float32)
    x[rng.random(x.shape) < 0.3] = 0
    w = (rng.standard_normal((f, c * max(kk, 1) ** 2)) * 0.1).astype(np.float32)
    b = rng.standard_normal(f).astype(np.float32)
    if layout == "rows":
        m, g, expected = n, None, oracle.linear_bf16(x, w, b, branches=2, threads=8)
    else:
        kind = abi.GATHER_CONV_NCHW if layout == "nchw" else abi.GATHER_CONV_NHWC
        g = conv_gather(kind, n, c, h, h, kk, kk, stride, pad)
        m = n * g.out_h * g.out_w
        conv = oracle.conv2d_bf16(x, w.reshape(f, c, kk, kk), b, stride, pad, branches=2,
                                  threads=8)
        expected = conv.transpose(0, 2, 3, 1).reshape(m, f)
    layer = CimLayer(w)
    ws = Workspace(DEV)
    bias = torch.from_numpy(b).to(DEV)

    def run(values):
        host = values if layout != "nhwc" else values.transpose(0, 2, 3, 1).copy()
        out = torch.empty(m, f, device=DEV)
        status = StatusWord(DEV)
        layer.forward_bf16(torch.from_numpy(host).to(DEV), out, m, gather=g, bias=bias,
                           branches=2, workspace=ws, status=status)
        torch.cuda.synchronize()
        return out.cpu().numpy(), status

    signed = x.copy()
    signed[(x == 0) & (rng.random(x.shape) < 0.5)] = -0.0
    assert np.signbit(signed).any()
    got, status = run(signed)
    status.raise_if_set()
    np.testing.assert_array_equal(bits(got), bits(expected))
    negative = x.copy()
    negative.flat[rng.integers(negative.size)] = -0.5
    _, status = run(negative)
    with pytest.raises(RuntimeError, match="rejects negative inputs"):
        status.raise_if_set()
