"""The allocation-free BF16 layer entry point, through the C ABI.

cim22_cuda_layer_forward_bf16_noalloc serves callers that cannot allocate
device memory (generated model code that owns only stack buffers, embedders
whose device memory another component budgets); its scratch is a
library-owned static device array. Its output must equal the
workspace-taking entry point's, bit for bit, on consecutive calls (the array
keeps the previous call's contents, which must not leak into the next result),
and sizes beyond the array are rejected before any launch. This file sorts
last so that a failure here does not hide the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

from cim22_b200 import abi
from cim22_b200.cim_ops import ACT, CimLayer, StatusWord, Workspace, conv_gather
from cim22_b200.native import lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def _with_workspace(layer, x, gather, m, bias, act, branches):
    out = torch.empty(m, layer.n, device=DEV)
    status = StatusWord(DEV)
    layer.forward_bf16(x, out, m, gather=gather, bias=bias, activation=act, branches=branches,
                       workspace=Workspace(DEV), status=status)
    torch.cuda.synchronize()
    status.raise_if_set()
    return out.cpu().numpy()


def _noalloc(layer, x, gather, m, bias, act, branches):
    out = torch.full((m, layer.n), float("nan"), device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib().cim22_cuda_layer_forward_bf16_noalloc(
        layer._handle, _ptr(x), None if gather is None else ctypes.byref(gather), m,
        _ptr(bias), ACT[act], branches, _ptr(out), _ptr(status), _stream())
    assert rc == 0, lib().cim22_cuda_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    torch.cuda.set_device(DEV)
    rng = np.random.default_rng(11)
    # Call 1: a 4-branch linear layer with bias and GELU.
    w1 = (rng.standard_normal((70, 300)) * 0.05).astype(np.float32)
    x1 = torch.from_numpy(rng.standard_normal((96, 300)).astype(np.float32)).to(DEV)
    b1 = torch.from_numpy(rng.standard_normal(70).astype(np.float32)).to(DEV)
    l1 = CimLayer(w1, device=DEV)
    # Call 2: a 2-branch conv on nonnegative NHWC input, smaller footprint, so
    # stale bytes of call 1 remain in the array beyond call 2's region.
    w2 = (rng.standard_normal((16, 6, 5, 5)) * 0.2).astype(np.float32)
    x2 = torch.from_numpy(np.maximum(rng.standard_normal((2, 14, 14, 6)), 0)
                          .astype(np.float32)).to(DEV)
    g2 = conv_gather(abi.GATHER_CONV_NHWC, 2, 6, 14, 14, 5, 5, 1, 0)
    l2 = CimLayer(w2.reshape(16, -1), device=DEV)
    m2 = 2 * 10 * 10
    for _ in range(2):
        got1 = _noalloc(l1, x1, None, 96, b1, "gelu", 4)
        exp1 = _with_workspace(l1, x1, None, 96, b1, "gelu", 4)
        np.testing.assert_array_equal(got1.view(np.uint32), exp1.view(np.uint32))
        got2 = _noalloc(l2, x2, g2, m2, None, "relu", 2)
        exp2 = _with_workspace(l2, x2, g2, m2, None, "relu", 2)
        np.testing.assert_array_equal(got2.view(np.uint32), exp2.view(np.uint32))


def test_noalloc_rejects_sizes_beyond_the_static_scratch():
    torch.cuda.set_device(DEV)
    limit = lib().cim22_cuda_layer_noalloc_scratch_bytes()
    assert limit == 16 << 20
    layer = CimLayer(np.ones((16, 4096), np.float32), device=DEV)
    m = 4096  # 2 branches x 4096 columns x (4096 + 4 * 64) bytes > 16 MiB
    assert layer.workspace_bytes(m, 4) > limit
    x = torch.ones(m, 4096, device=DEV)
    y = torch.empty(m, 16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib().cim22_cuda_layer_forward_bf16_noalloc(layer._handle, _ptr(x), None, m, None, 0,
                                                     4, _ptr(y), _ptr(status), _stream())
    assert rc == 0x10  # CIM22_STATUS_BAD_ARGUMENT
    assert "static scratch" in lib().cim22_cuda_last_error().decode()
