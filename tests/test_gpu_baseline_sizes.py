"""Parity at the benchmarked sizes.

Every workload runs at the batch the benchmark times (MLP 64, LeNet 256,
ResNet-18 1024, the BF16 4x4096 stack 512 rows, the event CNN 512 per GPU),
on the kernels those sizes select:

* MLP and LeNet (exact glue only): the whole output bit-exact vs the oracle.
* ResNet-18, the 4x4096 stack and the event CNN: every CIM layer of the
  unfused program bit-exact vs the oracle on a seeded sample of its output
  columns (computed from the inputs the GPU recorded for that layer); the
  benchmarked (fused) program bit-identical to the unfused one over the whole
  batch; the network output of sampled inputs within 1e-3 relative error of
  the oracle's forward (CIM layers by the oracle, float glue by PyTorch CPU,
  as the reference's own reference mode), with the max-abs and max-relative
  errors printed.
* The NCHW prepare kernel's several-chunks-per-block schedules (two or four
  256-column chunks per block), which only layers of 2,368 x chunks / T or
  more reach: bit-identical over the whole output to the NHWC input path
  (a different prepare kernel) and bit-exact vs the oracle on a sample.
"""

import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
THREADS = os.cpu_count() or 1


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def sample_conv_columns(x, kh, kw, stride, pad, n_idx, oh_idx, ow_idx):
    """im2col rows (K order c, i, j) of the sampled output pixels of an NCHW batch."""
    n, c, h, w = x.shape
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    rows = (oh_idx * stride)[:, None] + np.arange(kh)[None, :]
    cols = (ow_idx * stride)[:, None] + np.arange(kw)[None, :]
    patch = xp[n_idx[:, None, None, None], np.arange(c)[None, :, None, None],
               rows[:, None, :, None], cols[:, None, None, :]]
    return patch.reshape(len(n_idx), c * kh * kw)


def sample_size(k, n, branches, columns):
    return int(min(columns, max(256, min(4096, 5e8 // (k * n * branches)))))


def check_layers_sampled(prog, seed=0):
    """Run an unfused program step by step; check every CIM layer's output on
    sampled columns against the oracle on the GPU's own inputs for it."""
    rng = np.random.default_rng(seed)
    checked = 0
    for step in prog.steps:
        step.fn()
        if not step.cim:
            continue
        torch.cuda.synchronize()
        prog.check_status()
        meta = step.meta
        assert meta["act"] is None and meta.get("post") is None
        w = meta["weight"].numpy()
        b = None if meta["bias"] is None else meta["bias"].numpy()
        branches = meta["branches"]
        x = meta["x"].cpu().numpy()
        out = meta["out"]
        if meta["kind"] == "conv":
            f, c, kh, kw = w.shape
            n, _, h, wd = x.shape
            s, p = meta["stride"], meta["pad"]
            oh, ow = (h + 2 * p - kh) // s + 1, (wd + 2 * p - kw) // s + 1
            cols = n * oh * ow
            S = sample_size(c * kh * kw, f, branches, cols)
            idx = rng.choice(cols, S, replace=False)
            n_i, rem = idx // (oh * ow), idx % (oh * ow)
            oh_i, ow_i = rem // ow, rem % ow
            a = sample_conv_columns(x, kh, kw, s, p, n_i, oh_i, ow_i)
            exp = oracle.linear_bf16(a, w.reshape(f, -1), b, branches=branches,
                                     threads=THREADS)
            got = out.cpu().numpy().reshape(n, f, oh, ow)[n_i, :, oh_i, ow_i]
        else:
            rows = x.reshape(x.shape[0], -1)
            S = sample_size(rows.shape[1], w.shape[0], branches, rows.shape[0])
            idx = np.sort(rng.choice(rows.shape[0], S, replace=False))
            exp = oracle.linear_bf16(rows[idx], w, b, branches=branches, threads=THREADS)
            got = out.cpu().numpy().reshape(rows.shape[0], -1)[idx]
        np.testing.assert_array_equal(bits(got), bits(exp), err_msg=step.name)
        checked += 1
    return checked


def run_program(prog, x):
    prog.inputs[0].tensor.copy_(x.to(DEV))
    prog.status.reset()
    prog.launch()
    torch.cuda.synchronize()
    prog.check_status()
    return prog.output_tensors[0].cpu().numpy()


def float_errors(got, expected):
    """Max-abs error, and the max relative error over outputs whose magnitude
    is at least 1% of the output scale (relative error is undefined at 0)."""
    scale = float(np.max(np.abs(expected)))
    diff = np.abs(got.astype(np.float64) - expected.astype(np.float64))
    big = np.abs(expected) >= 0.01 * scale
    rel = float(np.max(diff[big] / np.abs(expected[big]))) if big.any() else 0.0
    return float(diff.max()), rel, scale


@pytest.mark.parametrize("name", ["mlp", "lenet"])
def test_exact_glue_workloads_at_benchmark_batch(name):
    """The benchmarked program (fused chain or per-layer kernels, whichever
    the program picks) bit-exact vs the oracle over the whole batch."""
    from cim22_b200 import program, workloads

    batch = workloads.WORKLOADS[name].batch
    model, x = workloads.build(name, batch, seed=1000)
    prog = program.from_module(model, x, name=name)
    prog.capture()
    prog.inputs[0].tensor.copy_(x.to(DEV))
    prog.replay()
    torch.cuda.synchronize()
    prog.check_status()
    got = prog.output_tensors[0].cpu().numpy()
    expected = oracle.cim_forward(model, x.numpy(), branches="reference", threads=THREADS)
    np.testing.assert_array_equal(bits(got), bits(expected))


@pytest.mark.parametrize("name,layers,sample", [("resnet18", 21, 8), ("event_cnn", 5, 16),
                                                ("bf16_4x4096", 4, 16)])
def test_float_glue_workloads_at_benchmark_batch(name, layers, sample):
    from cim22_b200 import program, workloads

    batch = workloads.WORKLOADS[name].batch
    model, x = workloads.build(name, batch, seed=1000)
    # Every CIM layer on sampled columns, unfused (the layer output alone).
    plain = program.from_module(model, x, fuse=False, name=name)
    plain.inputs[0].tensor.copy_(x.to(DEV))
    plain.status.reset()
    assert check_layers_sampled(plain) == layers
    torch.cuda.synchronize()
    plain.check_status()
    reference_bits = plain.output_tensors[0].cpu().numpy()
    del plain
    # The benchmarked program (epilogue-fused BN/ReLU/residual/GELU, CUDA
    # graph) gives the unfused program's bits over the whole batch.
    fused = program.from_module(model, x, name=name)
    fused.capture()
    fused.inputs[0].tensor.copy_(x.to(DEV))
    fused.replay()
    torch.cuda.synchronize()
    fused.check_status()
    got = fused.output_tensors[0].cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(reference_bits))
    # Whole-network outputs of sampled inputs against the oracle's forward.
    idx = np.sort(np.random.default_rng(7).choice(batch, sample, replace=False))
    expected = oracle.cim_forward(model, x[idx].numpy(), branches="reference",
                                  threads=THREADS)
    max_abs, max_rel, scale = float_errors(got[idx], expected)
    print(f"{name} b{batch}: max-abs {max_abs:.3e}, max-rel {max_rel:.3e} "
          f"(outputs >= 1% of scale {scale:.3e})")
    assert max_abs <= 1e-3 * scale, (max_abs, scale)
    assert max_rel <= 1e-3, max_rel


def prepare_schedule(m, T):
    """Chunks of 256 columns per block the NCHW prepare kernel uses for a
    layer of m columns and T crossbar K tiles (the dispatch rule of
    cim22_cuda_layer_prepare_bf16: as many as still give four waves)."""
    chunks = -(-(-(-m // 128) * 128) // 256)
    per_block = 4
    while per_block > 1 and (-(-chunks // per_block)) * T < 148 * 4 * 4:
        per_block //= 2
    return per_block


@pytest.mark.parametrize("batch,h,branches,pool,per_block", [
    (140, 32, 2, 0, 2), (264, 32, 2, 0, 4), (264, 32, 4, 0, 4),   # TMA-staged window
    (264, 32, 2, 2, 4), (140, 32, 4, 2, 2),                       # fused 2x2 pool
    (150, 30, 2, 0, 2), (300, 30, 4, 0, 4)])                      # rows not in 256 columns
def test_prepare_nchw_large_layers(batch, h, branches, pool, per_block):
    """A 64 -> 64 channel 3x3 conv (ResNet-18's first stage, T = 9) at
    batches of 135 k - 270 k columns, 2 and 4 branches. 32x32 outputs without
    a pool take the TMA-staged window gather (a block's 256 columns are eight
    whole output rows); with a fused 2x2 max pool, or with 30x30 outputs
    (rows that do not tile 256 columns), the thread-per-group kernel with two
    or four 256-column chunks per block, a schedule only layers of
    2,368 x chunks / T or more reach. The whole output equals the NHWC input
    path's (a different prepare kernel) bit for bit, and sampled columns
    equal the oracle's."""
    from cim22_b200 import abi
    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace, conv_gather

    c = f = 64
    m = batch * h * h
    assert prepare_schedule(m, 9) == per_block
    rng = np.random.default_rng(batch + branches + pool)
    src = 2 * h if pool else h
    x = rng.standard_normal((batch, c, src, src)).astype(np.float32)
    if branches == 2:
        x = np.maximum(x, 0)
    x[rng.random(x.shape) < 0.1] = 0
    w = (rng.standard_normal((f, c, 3, 3)) * 0.06).astype(np.float32)
    b = rng.standard_normal(f).astype(np.float32)
    layer = CimLayer(w.reshape(f, -1))
    dev = torch.device(DEV)
    ws, status = Workspace(dev), StatusWord(dev)
    bias = torch.from_numpy(b).to(DEV)
    outs = {}
    for layout in ("nchw", "nhwc"):
        kind = abi.GATHER_CONV_NCHW if layout == "nchw" else abi.GATHER_CONV_NHWC
        g = conv_gather(kind, batch, c, h, h, 3, 3, 1, 1)
        if pool:
            g.pool_kernel, g.pool_stride, g.pool_src_h, g.pool_src_w = 2, 2, src, src
        xt = torch.from_numpy(x if layout == "nchw" else x.transpose(0, 2, 3, 1).copy()).to(DEV)
        out = torch.empty(m, f, device=DEV)
        layer.forward_bf16(xt, out, m, gather=g, bias=bias, branches=branches, workspace=ws,
                           status=status)
        torch.cuda.synchronize()
        status.raise_if_set()
        outs[layout] = out.cpu().numpy()
        del xt
    np.testing.assert_array_equal(bits(outs["nchw"]), bits(outs["nhwc"]))
    pooled = x.reshape(batch, c, h, 2, h, 2).max(axis=(3, 5)) if pool else x
    idx = rng.choice(m, 4096, replace=False)
    n_i, rem = idx // (h * h), idx % (h * h)
    a = sample_conv_columns(pooled, 3, 3, 1, 1, n_i, rem // h, rem % h)
    exp = oracle.linear_bf16(a, w.reshape(f, -1), b, branches=branches, threads=THREADS)
    np.testing.assert_array_equal(bits(outs["nchw"][idx]), bits(exp))
