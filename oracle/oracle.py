"""ORACLE - test infrastructure only.

Python access to the CPU restatement in ``oracle/cim_oracle.cpp`` plus the
pieces of the reference's Host glue that the compiler emits as plain loops
(im2col gathers, pooling, activations), computed with NumPy/PyTorch CPU eager
exactly as the reference's ``runtime="reference"`` mode evaluates them
(python/cim22/backend.py:141-150 of mlir-cim22).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this
module. The CUDA backend never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
sys.path.insert(0, str(REPO / "mlir-cim22_b200"))

from cim22_b200 import abi  # noqa: E402  (data layout only)

_LIB = None
_REF = None


class OracleError(RuntimeError):
    pass


def build(reference: bool = True) -> None:
    """Compile liboracle.so and, when the mlir-cim22 source tree is present
    (the Makefile's REFERENCE, or CIM22_REFERENCE), the reference pieces in
    oracle/_ref. The Makefile alone knows where that tree lives."""
    targets = ["oracle"]
    if reference:
        targets.append("ref-if-present")
    env = dict(os.environ)
    if "CIM22_REFERENCE" in os.environ:
        env["REFERENCE"] = os.environ["CIM22_REFERENCE"]
    subprocess.run(["make", "-s", "-C", str(HERE), *targets], check=True, env=env)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = HERE / "liboracle.so"
        source = HERE / "cim_oracle.cpp"
        if not path.exists() or path.stat().st_mtime < source.stat().st_mtime:
            build(reference=False)
        L = ctypes.CDLL(str(path))
        c = ctypes
        L.oracle_int21_to_bf16.restype = c.c_uint16
        L.oracle_int21_to_bf16.argtypes = [c.c_int32, c.c_uint8, c.c_uint8]
        L.oracle_prealign.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p]
        L.oracle_prealign_tile.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p]
        L.oracle_scale_bf16.restype = c.c_uint16
        L.oracle_scale_bf16.argtypes = [c.c_uint16, c.c_int]
        L.oracle_float_to_bf16.restype = c.c_uint16
        L.oracle_float_to_bf16.argtypes = [c.c_float]
        L.oracle_prepare_input.argtypes = [c.c_void_p, c.c_int, c.c_void_p, c.c_void_p,
                                           c.c_void_p, c.c_void_p, c.c_void_p,
                                           c.c_char_p, c.c_size_t]
        L.oracle_restore.argtypes = [c.c_uint16, c.c_uint8, c.c_int, c.c_int32, c.c_int32,
                                     c.c_int, c.c_void_p, c.c_char_p, c.c_size_t]
        L.oracle_runner_create.restype = c.c_void_p
        L.oracle_runner_destroy.argtypes = [c.c_void_p]
        L.oracle_runner_stats.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p]
        L.oracle_runner_clear.argtypes = [c.c_void_p]
        L.oracle_runner_run.argtypes = [c.c_void_p, c.c_void_p, c.c_int, c.c_int,
                                        c.c_void_p, c.c_int64, c.c_void_p, c.c_int64,
                                        c.c_int, abi.TraceCallback, c.c_void_p,
                                        c.c_char_p, c.c_size_t]
        L.oracle_int8_range_safe.argtypes = [c.c_void_p, c.c_int64, c.c_int64]
        L.oracle_linear_int8.argtypes = [c.c_void_p, c.c_int64, c.c_int64, c.c_void_p,
                                         c.c_int64, c.c_void_p, c.c_char_p, c.c_size_t]
        L.oracle_linear_bf16_mode.argtypes = [c.c_void_p, c.c_int64, c.c_int64, c.c_void_p,
                                              c.c_int64, c.c_void_p, c.c_int, c.c_void_p,
                                              c.c_char_p, c.c_size_t]
        for name in ("oracle_linear_bf16", "oracle_linear_bf16_runner"):
            getattr(L, name).argtypes = [c.c_void_p, c.c_int64, c.c_int64, c.c_void_p,
                                         c.c_int64, c.c_void_p, c.c_int, c.c_void_p,
                                         c.c_int, c.c_char_p, c.c_size_t]
        _LIB = L
    return _LIB


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own BF16Support.cpp, when oracle/_ref was built here."""
    global _REF
    if _REF is None:
        path = HERE / "_ref" / "libref_bf16support.so"
        if not path.exists():
            return None
        L = ctypes.CDLL(str(path))
        L.ref_int21_to_bf16.restype = ctypes.c_uint16
        L.ref_int21_to_bf16.argtypes = [ctypes.c_int32, ctypes.c_uint8, ctypes.c_uint8]
        L.ref_prealign.argtypes = [ctypes.c_void_p] * 3
        L.ref_prealign_tile.argtypes = [ctypes.c_void_p] * 3
        _REF = L
    return _REF


_REF_RUNNER = None


def ref_runner_lib() -> ctypes.CDLL | None:
    """The reference's own CIMSoftwareRunner + BF16Compensation (with
    BF16Support), compiled unmodified into oracle/_ref against the clean-room
    LLVM support headers of oracle/llvm_shim, when that was built here."""
    global _REF_RUNNER
    if _REF_RUNNER is None:
        path = HERE / "_ref" / "libref_runner.so"
        if not path.exists():
            return None
        L = ctypes.CDLL(str(path))
        c = ctypes
        L.ref_linear_bf16_runner.argtypes = [c.c_void_p, c.c_int64, c.c_int64, c.c_void_p,
                                             c.c_int64, c.c_void_p, c.c_int, c.c_void_p,
                                             c.c_int, c.c_char_p, c.c_size_t]
        L.ref_runner_create.restype = c.c_void_p
        L.ref_runner_create.argtypes = [c.c_int]
        L.ref_runner_destroy.argtypes = [c.c_void_p]
        L.ref_runner_stats.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p]
        L.ref_runner_run.argtypes = [c.c_void_p, c.c_void_p, c.c_int, c.c_void_p, c.c_int64,
                                     c.c_void_p, c.c_int64, c.c_int, c.c_char_p, c.c_size_t]
        _REF_RUNNER = L
    return _REF_RUNNER


def reference_runner_available() -> bool:
    return ref_runner_lib() is not None


class RefRunner:
    """The reference's own CIMSoftwareRunner (oracle/_ref) in one compensation
    mode, with a session-owned weight catalog and residency; the same run()
    contract as Runner."""

    def __init__(self, mode: int) -> None:
        L = ref_runner_lib()
        if L is None:
            raise OracleError("the reference runner was not built (oracle/_ref)")
        self._handle = L.ref_runner_create(mode)

    def close(self) -> None:
        if self._handle:
            ref_runner_lib().ref_runner_destroy(self._handle)
            self._handle = None

    def __del__(self) -> None:  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    @property
    def stats(self) -> tuple[int, int]:
        w, h = ctypes.c_uint64(), ctypes.c_uint64()
        ref_runner_lib().ref_runner_stats(self._handle, ctypes.byref(w), ctypes.byref(h))
        return w.value, h.value

    def run(self, spec, inputs, outputs, *, batch: bool = False, residency: bool = False):
        txn = spec.to_c()
        in_ptrs = (ctypes.c_void_p * max(1, len(inputs)))(
            *[None if a is None else a.ctypes.data for a in inputs])
        out_ptrs = (ctypes.c_void_p * max(1, len(outputs)))(
            *[None if a is None else a.ctypes.data for a in outputs])
        err = _err()
        rc = ref_runner_lib().ref_runner_run(self._handle, txn.pointer, int(batch), in_ptrs,
                                             len(inputs), out_ptrs, len(outputs),
                                             int(residency), err, len(err))
        return err.value.decode() if rc else None


def _err() -> ctypes.Array:
    return ctypes.create_string_buffer(512)


# ---------------------------------------------------------------------------
# Scalar peripherals.


def int21_to_bf16(value: int, we: int, ie: int) -> int:
    return int(lib().oracle_int21_to_bf16(value, we, ie))


def prealign(values) -> tuple[int, np.ndarray]:
    row = np.ascontiguousarray(values, dtype=np.uint16)
    assert row.shape == (64,)
    exp = ctypes.c_uint8()
    out = np.zeros(64, np.int8)
    lib().oracle_prealign(row.ctypes.data, ctypes.byref(exp), out.ctypes.data)
    return exp.value, out


def prealign_tile(bits) -> tuple[np.ndarray, np.ndarray]:
    tile = np.ascontiguousarray(bits, dtype=np.uint16).reshape(16, 64)
    values = np.zeros((16, 64), np.int8)
    exps = np.zeros(16, np.uint8)
    lib().oracle_prealign_tile(tile.ctypes.data, values.ctypes.data, exps.ctypes.data)
    return values, exps


def scale_bf16(bits: int, exponent: int) -> int:
    return int(lib().oracle_scale_bf16(bits, exponent))


def float_to_bf16(x) -> np.ndarray:
    """RNE FP32 -> BF16 bits, elementwise (arith.truncf)."""
    flat = np.asarray(x, dtype=np.float32).reshape(-1)
    f = lib().oracle_float_to_bf16
    return np.array([f(float(v)) for v in flat], np.uint16).reshape(np.shape(x))


def prepare_input(row, mode: int):
    """prepareBF16Input: returns (mantissas, exponent, effective, scale_delta, support)."""
    data = np.ascontiguousarray(row, dtype=np.uint16)
    mant = np.zeros(64, np.int8)
    exp = ctypes.c_uint8()
    eff = ctypes.c_int32()
    delta = ctypes.c_int32()
    sup = ctypes.c_uint64()
    err = _err()
    if lib().oracle_prepare_input(data.ctypes.data, mode, mant.ctypes.data, ctypes.byref(exp),
                                  ctypes.byref(eff), ctypes.byref(delta), ctypes.byref(sup),
                                  err, len(err)):
        raise OracleError(err.value.decode())
    return mant, exp.value, eff.value, delta.value, sup.value


def restore(bits: int, we: int, support: bool, effective: int, scale_delta: int, mode: int) -> int:
    out = ctypes.c_uint16()
    err = _err()
    if lib().oracle_restore(bits, we, int(support), effective, scale_delta, mode,
                            ctypes.byref(out), err, len(err)):
        raise OracleError(err.value.decode())
    return out.value


# ---------------------------------------------------------------------------
# Runner.


class Runner:
    """The restated CIMSoftwareRunner with a session-owned catalog and residency."""

    def __init__(self) -> None:
        self._handle = lib().oracle_runner_create()

    def close(self) -> None:
        if self._handle:
            lib().oracle_runner_destroy(self._handle)
            self._handle = None

    def __del__(self) -> None:  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    @property
    def stats(self) -> tuple[int, int]:
        w, h = ctypes.c_uint64(), ctypes.c_uint64()
        lib().oracle_runner_stats(self._handle, ctypes.byref(w), ctypes.byref(h))
        return w.value, h.value

    def clear(self) -> None:
        lib().oracle_runner_clear(self._handle)

    def run(self, spec, mode: int, inputs, outputs, *, batch: bool = False,
            residency: bool = False, trace: list | None = None):
        """Run one transaction; inputs/outputs are lists of NumPy rows (views allowed).

        Returns None on success or the error string.
        """
        txn = spec.to_c()
        in_ptrs = (ctypes.c_void_p * max(1, len(inputs)))(
            *[None if a is None else a.ctypes.data for a in inputs])
        out_ptrs = (ctypes.c_void_p * max(1, len(outputs)))(
            *[None if a is None else a.ctypes.data for a in outputs])
        events = trace

        def record(_ctx, event):
            e = event.contents
            events.append((e.sequence, e.kind, e.group_id, e.work_id, e.macro_slot,
                           e.packet_index, e.cache_row_or_address))

        callback = abi.TraceCallback(record) if trace is not None else abi.TraceCallback()
        err = _err()
        rc = lib().oracle_runner_run(self._handle, txn.pointer, int(batch), mode, in_ptrs,
                                     len(inputs), out_ptrs, len(outputs), int(residency),
                                     callback, None, err, len(err))
        return err.value.decode() if rc else None


# ---------------------------------------------------------------------------
# Layer level.


def int8_range_safe(w: np.ndarray) -> bool:
    w = np.ascontiguousarray(w, dtype=np.int8)
    return bool(lib().oracle_int8_range_safe(w.ctypes.data, w.shape[0], w.shape[1]))


def linear_int8(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    m, k = x.shape
    n = w.shape[0]
    assert w.shape[1] == k
    y = np.zeros((m, n), np.int32)
    err = _err()
    if lib().oracle_linear_int8(x.ctypes.data, m, k, w.ctypes.data, n, y.ctypes.data, err, len(err)):
        raise OracleError(err.value.decode())
    return y


def linear_bf16(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None,
                branches: int = 4, threads: int = 1, via_runner: bool | str = False) -> np.ndarray:
    """Sign-split BF16 CIM layer, y[m, n] for columns x[m, k] and weights w[n, k].

    via_runner: False computes the layer directly from the restated numerics;
    True drives the restated CIMSoftwareRunner with 40-Work transactions;
    "reference" drives the reference's own runner (oracle/_ref); "auto" the
    reference's runner when it was built, else the restated one."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, k = x.shape
    n = w.shape[0]
    assert w.shape[1] == k and branches in (2, 4)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.zeros((m, n), np.float32)
    err = _err()
    if via_runner == "reference":
        ref = ref_runner_lib()
        if ref is None:
            raise OracleError("the reference runner was not built (oracle/_ref)")
        fn = ref.ref_linear_bf16_runner
    elif via_runner == "auto" and ref_runner_lib() is not None:
        fn = ref_runner_lib().ref_linear_bf16_runner
    elif via_runner:
        fn = lib().oracle_linear_bf16_runner
    else:
        fn = lib().oracle_linear_bf16
    if fn(x.ctypes.data, m, k, w.ctypes.data, n, None if b is None else b.ctypes.data,
          branches, y.ctypes.data, threads, err, len(err)):
        raise OracleError(err.value.decode())
    return y


MODES = {"none": 0, "legacy": 1}


def linear_bf16_mode(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None,
                     mode: str = "legacy") -> np.ndarray:
    """BF16 CIM layer in the Legacy or None compensation mode (no sign split)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, k = x.shape
    n = w.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.zeros((m, n), np.float32)
    err = _err()
    if lib().oracle_linear_bf16_mode(x.ctypes.data, m, k, w.ctypes.data, n,
                                     None if b is None else b.ctypes.data, MODES[mode],
                                     y.ctypes.data, err, len(err)):
        raise OracleError(err.value.decode())
    return y


def im2col(x: np.ndarray, kh: int, kw: int, stride: int, pad: int) -> tuple[np.ndarray, int, int]:
    """Columns (n, oh, ow) x K (c, i, j) of an NCHW batch (Passes.cpp:1185-1191)."""
    n, c, h, w = x.shape
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    oh = (h + 2 * pad - kh) // stride + 1
    ow = (w + 2 * pad - kw) // stride + 1
    cols = np.empty((n, oh, ow, c, kh, kw), np.float32)
    for i in range(kh):
        for j in range(kw):
            patch = xp[:, :, i:i + stride * oh:stride, j:j + stride * ow:stride]
            cols[:, :, :, :, i, j] = patch.transpose(0, 2, 3, 1)
    return cols.reshape(n * oh * ow, c * kh * kw), oh, ow


def conv2d_bf16(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None, stride: int = 1,
                pad: int = 0, branches: int = 4, threads: int = 1,
                via_runner: bool = False) -> np.ndarray:
    """Sign-split BF16 CIM convolution of an NCHW batch, returned NCHW."""
    f, c, kh, kw = weight.shape
    cols, oh, ow = im2col(np.asarray(x, np.float32), kh, kw, stride, pad)
    y = linear_bf16(cols, weight.reshape(f, -1), bias, branches, threads, via_runner)
    n = x.shape[0]
    return y.reshape(n, oh, ow, f).transpose(0, 3, 1, 2).copy()


# ---------------------------------------------------------------------------
# INT8 Conv / MatMulInteger with bias, as the compiler lowers them.


def prove_int8_ranges(w: np.ndarray, input_ranges) -> bool:
    """proveMatMulIntegerRanges (Passes.cpp:593-627): every 64-wide K tile of
    every output lane keeps its lowest and highest possible partial sum, given
    per-K input ranges [lo, hi], inside signed i21."""
    w = np.asarray(w, np.int64)
    lo = np.array([r[0] for r in input_ranges], np.int64)
    hi = np.array([r[1] for r in input_ranges], np.int64)
    upper = np.where(w >= 0, w * hi, w * lo)
    lower = np.where(w >= 0, w * lo, w * hi)
    for t in range(0, w.shape[1], 64):
        for part in (upper[:, t:t + 64].sum(1), lower[:, t:t + 64].sum(1)):
            if np.any(part < -(1 << 20)) or np.any(part >= (1 << 20)):
                return False
    return True


def wrap_i32(values: np.ndarray) -> np.ndarray:
    """Two's-complement int32 of an int64 array."""
    return ((np.asarray(values, np.int64) + (1 << 31)) % (1 << 32) - (1 << 31)).astype(np.int32)


def im2col_int8(x: np.ndarray, kh: int, kw: int, strides=(1, 1),
                pads=(0, 0, 0, 0)) -> tuple[np.ndarray, int, int]:
    """Columns (n, oh, ow) x K (c, i, j) of an int8 NCHW batch with ONNX pads
    (top, left, bottom, right); the im2col of normalizeCIMInt8Conv
    (Passes.cpp:1511-1552) after the importer's zero padding."""
    n, c, h, w = x.shape
    top, left, bottom, right = pads
    xp = np.pad(np.asarray(x, np.int8), ((0, 0), (0, 0), (top, bottom), (left, right)))
    sh, sw = strides
    oh = (h + top + bottom - kh) // sh + 1
    ow = (w + left + right - kw) // sw + 1
    cols = np.empty((n, oh, ow, c, kh, kw), np.int8)
    for i in range(kh):
        for j in range(kw):
            patch = xp[:, :, i:i + sh * (oh - 1) + 1:sh, j:j + sw * (ow - 1) + 1:sw]
            cols[:, :, :, :, i, j] = patch.transpose(0, 2, 3, 1)
    return cols.reshape(n * oh * ow, c * kh * kw), oh, ow


def linear_int8_bias(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None, *,
                     allow_extra_k_tile: bool = True) -> np.ndarray:
    """An INT8 contraction plus optional int32 bias, as the compiler lowers it.

    Weights that fail the range proof stay on the Host: exact wrapping int32
    (Passes.cpp:1402-1450, 2075-2155). Otherwise the layer runs as CIM tiles
    (linear_int8). A bias whose values all fit int8 is folded into the tiles
    as one more K column (weight = bias, input = 1), inserted before the last
    column when K is a multiple of 64, if the folded weights pass the proof
    with that column's input range [1, 1] (FoldCIMInt8BiasPattern,
    Passes.cpp:1863-2012); any other bias is a wrapping Host add."""
    x = np.ascontiguousarray(x, np.int8)
    w = np.ascontiguousarray(w, np.int8)
    k = w.shape[1]
    if not int8_range_safe(w):
        y = wrap_i32(x.astype(np.int64) @ w.T.astype(np.int64))
        return y if bias is None else wrap_i32(y.astype(np.int64) + np.asarray(bias, np.int64))
    if bias is not None:
        b = np.asarray(bias, np.int64)
        exact_k = k % 64 == 0
        if np.all((b >= -128) & (b <= 127)) and (not exact_k or allow_extra_k_tile):
            lane = k - 1 if exact_k else k
            wf = np.insert(w, lane, b.astype(np.int8), axis=1)
            xf = np.insert(x, lane, np.int8(1), axis=1)
            ranges = [(-128, 127)] * (k + 1)
            ranges[lane] = (1, 1)
            if prove_int8_ranges(wf, ranges):
                return linear_int8(xf, wf)
        return wrap_i32(linear_int8(x, w).astype(np.int64) + b)
    return linear_int8(x, w)


def conv2d_int8(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None = None,
                strides=(1, 1), pads=(0, 0, 0, 0), **kw) -> np.ndarray:
    """INT8 convolution (ConvInteger with zero zero-points, or a marked
    linalg conv) of an int8 NCHW batch with int8 [F, C, KH, KW] weights,
    returned as int32 NCHW."""
    f, c, kh, kwid = weight.shape
    cols, oh, ow = im2col_int8(x, kh, kwid, strides, pads)
    y = linear_int8_bias(cols, np.asarray(weight, np.int8).reshape(f, -1), bias, **kw)
    return y.reshape(x.shape[0], oh, ow, f).transpose(0, 3, 1, 2).copy()


def reference_branches(model) -> dict:
    """Sign-split branch count of every Linear/Conv2d module of a model, as
    the reference's lowering decides it: 2 when the layer's input is directly
    the result of a ReLU (isNonnegativeFloat, Passes.cpp:2239-2303), else 4
    (graph inputs, pools, flattens of pools, GELU, additions)."""
    import torch
    import torch.fx as fx
    import torch.nn.functional as F

    relu_calls = {F.relu, torch.relu}
    gm = fx.symbolic_trace(model)
    modules = dict(gm.named_modules())
    out = {}
    for node in gm.graph.nodes:
        if node.op != "call_module":
            continue
        module = modules[str(node.target)]
        if not isinstance(module, (torch.nn.Linear, torch.nn.Conv2d)):
            continue
        src = node.args[0]
        relu = isinstance(src, fx.Node) and (
            (src.op == "call_function" and src.target in relu_calls) or
            (src.op == "call_method" and src.target == "relu") or
            (src.op == "call_module" and isinstance(modules[str(src.target)], torch.nn.ReLU)))
        out[module] = 2 if relu else 4
    return out


def cim_forward(model, x, *, branches: int | str = 4, threads: int = 1,
                via_runner: bool | str = False, compensation: str = "sign-split",
                layers=None):
    """Run a torch model on CPU with every Linear/Conv2d computed by the oracle.

    Everything else runs as PyTorch CPU eager in f32, which is the reference's
    own oracle for the float glue. compensation "legacy" / "none" computes the
    layers in those diagnostic modes. branches: 4, 2, or "reference" for the
    per-layer counts of the reference's lowering (reference_branches); the
    results are the same bits, only the work differs. layers: names of the
    Linear/Conv2d modules to compute as CIM layers (default: all of them); the
    others run as PyTorch CPU eager, as LayerOffload leaves them. Returns a
    NumPy array.
    """
    import torch

    saved = {}
    per_layer = reference_branches(model) if branches == "reference" else {}

    def contract(cols, weight, bias, module):
        if compensation == "sign-split":
            return linear_bf16(cols, weight, bias, per_layer.get(module, branches), threads,
                               via_runner)
        return linear_bf16_mode(cols, weight, bias, compensation)

    def linear_forward(module):
        def fn(inp):
            flat = inp.detach().float().reshape(-1, inp.shape[-1]).numpy()
            bias = None if module.bias is None else module.bias.detach().float().numpy()
            y = contract(flat, module.weight.detach().float().numpy(), bias, module)
            return torch.from_numpy(y).reshape(*inp.shape[:-1], y.shape[-1])
        return fn

    def conv_forward(module):
        def fn(inp):
            assert module.groups == 1 and module.dilation == (1, 1)
            assert module.stride[0] == module.stride[1]
            assert module.padding[0] == module.padding[1]
            bias = None if module.bias is None else module.bias.detach().float().numpy()
            weight = module.weight.detach().float().numpy()
            f, c, kh, kw = weight.shape
            cols, oh, ow = im2col(inp.detach().float().numpy(), kh, kw, module.stride[0],
                                  module.padding[0])
            y = contract(cols, weight.reshape(f, -1), bias, module)
            n = inp.shape[0]
            return torch.from_numpy(y.reshape(n, oh, ow, f).transpose(0, 3, 1, 2).copy())
        return fn

    selected = None if layers is None else {
        module for name, module in model.named_modules() if name in set(layers)}
    for module in model.modules():
        if selected is not None and module not in selected:
            continue
        if isinstance(module, torch.nn.Linear):
            saved[module] = module.forward
            module.forward = linear_forward(module)
        elif isinstance(module, torch.nn.Conv2d):
            saved[module] = module.forward
            module.forward = conv_forward(module)
    try:
        with torch.no_grad():
            out = model(torch.as_tensor(x).float())
    finally:
        for module, fwd in saved.items():
            module.forward = fwd
    return out.detach().numpy()
