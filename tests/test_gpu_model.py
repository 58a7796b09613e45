"""Compiled model libraries on the CUDA session, end to end.

Each model is a gcc-built shared library exporting cim22_model_v1 with a
Protobuf artifact (serialized by the official protobuf runtime) and an entry
point that calls the _mlir_ciface_cim22_dispatch* tile ABI, the shape of what
the reference compiler emits. Results are checked against the supplier INT8
known answers and against the oracle's transaction runner.
"""

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import model_fixtures as mf
import oracle
import txn_fixtures as fx
from cim22_b200 import native
from cim22_b200.abi import BF16_SIGN_SPLIT, BF16_NONE, DATA_BF16, TxnWeight
from cim22_b200.runtime import Session

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def int8_model(tmp_path, name, weights, backend=0):
    kernels = [(f"__cim_kernel_{i}", fx.make_supplier_case(w)) for i, w in enumerate(weights)]
    outputs = [((8, 16), mf.INT32)] * len(weights)
    data = mf.artifact(kernels, [((8, 64), mf.INT8)], outputs, backend).SerializeToString()
    body = mf.INT8_BODY if len(weights) == 1 else mf.TWO_KERNEL_BODY
    return mf.build_model_library(tmp_path, name, data, body, ROWS=8)


def test_supplier_int8_model(tmp_path):
    data = json.loads((GOLDEN / "supplier_int8.json").read_text())
    for index, case in enumerate(data["cases"]):
        weight = np.array(case["weight"], np.int8)
        path = int8_model(tmp_path, f"supplier{index}", [weight])
        with Session(path) as session:
            assert session.input_shapes == ((8, 64),)
            assert session.output_shapes == ((8, 16),)
            assert session.input_dtypes == (np.dtype(np.int8),)
            assert session.output_dtypes == (np.dtype(np.int32),)
            assert session.num_transactions == 1
            (out,) = session(np.array(case["inputs"], np.int8))
            np.testing.assert_array_equal(out, np.array(case["expected"]))
            assert session.dispatch_count == 1


def test_two_kernel_model_matches_oracle(tmp_path):
    rng = np.random.default_rng(11)
    weights = [rng.integers(-128, 128, (16, 64)).astype(np.int8) for _ in range(2)]
    path = int8_model(tmp_path, "two", weights)
    session = Session(path)
    assert session.num_transactions == 2
    ref = oracle.Runner()
    for _ in range(3):
        x = rng.integers(-128, 128, (8, 64)).astype(np.int8)
        a, b = session(x)
        assert session.dispatch_count == 2
        for got, w in ((a, weights[0]), (b, weights[1])):
            outs = [np.zeros(16, np.int32) for _ in range(8)]
            assert ref.run(fx.make_supplier_case(w), BF16_NONE, list(x), outs) is None
            np.testing.assert_array_equal(got, np.stack(outs))
    session.close()
    with pytest.raises(RuntimeError, match="session is closed"):
        session(np.zeros((8, 64), np.int8))


def bf16_rows(rng, rows):
    exp = np.clip(120 + rng.integers(0, 10, (rows, 64)), 1, 254).astype(np.uint32)
    bits = (exp << 23) | (rng.integers(0, 1 << 23, (rows, 64)).astype(np.uint32))
    return bits.view(np.float32)


@pytest.mark.parametrize("dispatch,mode", [("_mlir_ciface_cim22_dispatch_sign_split",
                                            BF16_SIGN_SPLIT),
                                           ("_mlir_ciface_cim22_dispatch", BF16_NONE)])
def test_bf16_model_with_host_glue_matches_oracle(tmp_path, dispatch, mode):
    rng = np.random.default_rng(5)
    lane_bits = ((np.clip(124 + rng.integers(0, 6, (16, 64)), 1, 254) << 7)
                 | rng.integers(0, 128, (16, 64))).astype(np.uint16)
    values, exps = oracle.prealign_tile(lane_bits)
    spec = fx.make_bf16_executable(True, 0, TxnWeight(0, 0, 0, 0, values, exps, DATA_BF16))
    data = mf.artifact([("__cim_kernel_0", spec)], [((1, 64), mf.FP32)],
                       [((1, 16), mf.FP32)]).SerializeToString()
    path = mf.build_model_library(tmp_path, f"bf16_{mode}", data, mf.BF16_BODY, ROWS=1,
                                  DISPATCH=dispatch)
    session = Session(path)
    ref = oracle.Runner()
    for _ in range(4):
        x = bf16_rows(rng, 1)
        (y,) = session(x)
        u = x.view(np.uint32)
        row = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)[0]
        out = np.zeros(16, np.uint16)
        assert ref.run(spec, mode, [row], [out]) is None
        np.testing.assert_array_equal(y.view(np.uint32)[0], out.astype(np.uint32) << 16)
    # A runner error names the kernel; the outputs of the failed call are discarded.
    bad = x.copy()
    bad[0, 3] = np.inf
    with pytest.raises(RuntimeError) as info:
        session(bad)
    assert str(info.value) == "__cim_kernel_0: CIM BF16 input does not support NaN or infinity"
    (y,) = session(x)  # the session stays usable after an error
    session.close()


def test_invoke_argument_errors(tmp_path):
    weight = np.ones((16, 64), np.int8)
    path = int8_model(tmp_path, "args", [weight])
    session = Session(path)
    lib = native.lib()
    x = np.ones((8, 64), np.int8)
    y = np.zeros((8, 16), np.int32)
    ptrs = (ctypes.c_void_p * 2)(x.ctypes.data, y.ctypes.data)
    counts = (ctypes.c_int64 * 2)(x.size, y.size)
    assert lib.cim22_cuda_model_invoke(session._handle, ptrs, counts, 1) == 1
    assert lib.cim22_cuda_model_error(session._handle) == b"runtime buffer count mismatch"
    assert session.dispatch_count == 0
    counts[1] = 127
    assert lib.cim22_cuda_model_invoke(session._handle, ptrs, counts, 2) == 1
    assert lib.cim22_cuda_model_error(session._handle) == \
        b"runtime buffer element count mismatch"
    counts[1] = y.size
    assert lib.cim22_cuda_model_invoke(session._handle, ptrs, counts, 2) == 0
    assert lib.cim22_cuda_model_error(session._handle) == b""
    np.testing.assert_array_equal(y, np.full((8, 16), 64, np.int32))
    with pytest.raises(TypeError, match="Input 0 must be a NumPy int8 array"):
        session(np.zeros((8, 64), np.int32))
    with pytest.raises(ValueError, match="requires aligned, contiguous shape"):
        session(np.zeros((8, 65), np.int8)[:, :64])
    with pytest.raises(ValueError, match="Input count differs"):
        session()
    session.close()


def test_usb_backend_model_fails_each_dispatch(tmp_path):
    weight = np.ones((16, 64), np.int8)
    path = int8_model(tmp_path, "usb", [weight], backend=1)
    session = Session(path)
    x = np.ones((8, 64), np.int8)
    y = np.full((8, 16), 7, np.int32)
    ptrs = (ctypes.c_void_p * 2)(x.ctypes.data, y.ctypes.data)
    counts = (ctypes.c_int64 * 2)(x.size, y.size)
    lib = native.lib()
    assert lib.cim22_cuda_model_invoke(session._handle, ptrs, counts, 2) == 1
    assert lib.cim22_cuda_model_error(session._handle) == \
        b"USB runtime is not configured; call configure_usb first"
    assert np.all(y == 0)  # zero-filled before the backend check
    assert session.dispatch_count == 0
    session.close()
