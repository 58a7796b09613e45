"""ctypes binding of libcim22_cuda.so (include/cim22_cuda.h).

The library is built in-tree by ``mlir-cim22_b200/build.py``. Loading fails
with an ImportError when it is missing: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

from . import abi

LIBRARY = Path(__file__).resolve().parent / "libcim22_cuda.so"
_lock = threading.Lock()
_lib = None

c = ctypes
P = c.c_void_p
I32, I64, SZ = c.c_int32, c.c_int64, c.c_size_t
CHARP = c.c_char_p

_SIGNATURES = {
    "cim22_cuda_status_message": (CHARP, [I32]),
    "cim22_cuda_last_error": (CHARP, []),
    "cim22_cuda_abi_sizes": (c.c_int, [P, c.c_int]),
    "cim22_cuda_tensor_core_launches": (I64, []),
    "cim22_cuda_check_wait_timeout": (c.c_int, [c.c_uint64, P, P]),
    "cim22_cuda_runner_create": (P, [c.c_int, CHARP, SZ]),
    "cim22_cuda_runner_destroy": (None, [P]),
    "cim22_cuda_plan_create": (P, [P, P, c.c_int, CHARP, SZ]),
    "cim22_cuda_plan_destroy": (None, [P]),
    "cim22_cuda_runner_run": (c.c_int, [P, P, I32, P, I64, P, I64, c.c_int,
                                        abi.TraceCallback, P, CHARP, SZ]),
    "cim22_cuda_runner_weight_stats": (None, [P, P, P]),
    "cim22_cuda_runner_clear_residency": (None, [P]),
    "cim22_cuda_session_create": (P, [c.c_int, CHARP, SZ]),
    "cim22_cuda_session_destroy": (None, [P]),
    "cim22_cuda_session_add_transaction": (I64, [P, P, CHARP, CHARP, SZ]),
    "cim22_cuda_session_num_transactions": (I64, [P]),
    "cim22_cuda_session_begin_invoke": (None, [P]),
    "cim22_cuda_session_end_invoke": (c.c_int, [P]),
    "cim22_cuda_session_dispatch_count": (c.c_uint64, [P]),
    "cim22_cuda_session_error": (CHARP, [P]),
    "cim22_cuda_model_validate": (c.c_int, [P, c.c_uint64, CHARP, SZ]),
    "cim22_cuda_model_load_shared": (P, [CHARP, c.c_int, CHARP, SZ]),
    "cim22_cuda_model_destroy": (None, [P]),
    "cim22_cuda_model_num_inputs": (I64, [P]),
    "cim22_cuda_model_num_outputs": (I64, [P]),
    "cim22_cuda_model_rank": (I64, [P, I64]),
    "cim22_cuda_model_dim": (I64, [P, I64, I64]),
    "cim22_cuda_model_dtype": (I64, [P, I64]),
    "cim22_cuda_model_num_transactions": (I64, [P]),
    "cim22_cuda_model_dispatch_count": (c.c_uint64, [P]),
    "cim22_cuda_model_error": (CHARP, [P]),
    "cim22_cuda_model_invoke": (c.c_int, [P, c.POINTER(P), c.POINTER(I64), I64]),
    "_mlir_ciface_cim22_dispatch": (None, [I64, P, P]),
    "_mlir_ciface_cim22_dispatch_sign_split": (None, [I64, P, P]),
    "_mlir_ciface_cim22_dispatch_legacy": (None, [I64, P, P]),
    "_mlir_ciface_cim22_dispatch_int8": (None, [I64, P, P]),
    "cim22_cuda_layer_create_bf16": (P, [c.c_int, P, I64, I64, CHARP, SZ]),
    "cim22_cuda_layer_create_int8": (P, [c.c_int, P, I64, I64, CHARP, SZ]),
    "cim22_cuda_layer_destroy": (None, [P]),
    "cim22_cuda_layer_range_safe": (c.c_int, [P]),
    "cim22_cuda_layer_bf16_operands": (c.c_int, [P]),
    "cim22_cuda_device_alloc": (c.c_int, [SZ, c.POINTER(c.c_void_p)]),
    "cim22_cuda_device_free": (c.c_int, [P]),
    "cim22_cuda_ipc_get_handle": (c.c_int, [P, P]),
    "cim22_cuda_ipc_open_handle": (c.c_int, [P, c.POINTER(c.c_void_p)]),
    "cim22_cuda_ipc_close_handle": (c.c_int, [P]),
    "cim22_cuda_layer_contract_bf16_peers": (c.c_int, [P, I64, P, I32, I32, P, P, SZ, P, P]),
    "cim22_cuda_peer_barrier": (c.c_int, [P, c.c_uint64, P, P]),
    "cim22_cuda_layer_n": (I64, [P]),
    "cim22_cuda_layer_k": (I64, [P]),
    "cim22_cuda_layer_workspace_bf16": (SZ, [P, I64, I32]),
    "cim22_cuda_layer_workspace_int8": (SZ, [P, I64]),
    "cim22_cuda_layer_forward_bf16": (c.c_int, [P, P, P, I64, P, I32, I32, P, P, SZ, P, P]),
    "cim22_cuda_layer_forward_int8": (c.c_int, [P, P, I64, P, P, SZ, P, P]),
    "cim22_cuda_layer_forward_int8_ex": (c.c_int, [P, P, P, I64, I32, I32, P, I64, I32, P, P,
                                                   SZ, P, P]),
    "cim22_cuda_layer_prepare_bf16": (c.c_int, [P, P, P, I64, I32, P, SZ, P, P]),
    "cim22_cuda_layer_contract_bf16": (c.c_int, [P, I64, P, I32, I32, P, P, SZ, P, P]),
    "cim22_cuda_layer_forward_bf16_ex": (c.c_int, [P, P, P, I64, I64, P, P, P, I32, I32, P, P,
                                                   SZ, P, P]),
    "cim22_cuda_layer_fused_forward": (c.c_int, [P]),
    "cim22_cuda_layer_create_bf16_mode": (c.c_void_p, [c.c_int, P, I64, I64, I32, c.c_char_p, SZ]),
    "cim22_cuda_layer_compensation": (I32, [P]),
    "cim22_cuda_layer_contract_bf16_ex": (c.c_int, [P, I64, I64, P, P, P, I32, I32, P, P, SZ, P,
                                                    P]),
    "cim22_cuda_layer_contract_bf16_res": (c.c_int, [P, I64, I64, P, P, P, P, I32, I32, P, P,
                                                     SZ, P, P]),
    "cim22_cuda_layer_forward_bf16_noalloc": (c.c_int, [P, P, P, I64, P, I32, I32, P, P, P]),
    "cim22_cuda_layer_noalloc_scratch_bytes": (SZ, []),
    "cim22_cuda_relu": (c.c_int, [P, P, I64, P]),
    "cim22_cuda_add": (c.c_int, [P, P, P, I64, I32, P]),
    "cim22_cuda_gelu": (c.c_int, [P, P, I64, P]),
    "cim22_cuda_maxpool2d_nhwc": (c.c_int, [P, P, I32, I32, I32, I32, I32, I32, I32, P]),
    "cim22_cuda_avgpool2d_nhwc": (c.c_int, [P, P, I32, I32, I32, I32, I32, I32, P]),
    "cim22_cuda_global_avgpool_nhwc": (c.c_int, [P, P, I32, I32, I32, I32, P]),
    "cim22_cuda_channel_affine_nhwc": (c.c_int, [P, P, P, P, I64, I32, I32, P]),
    "cim22_cuda_softmax": (c.c_int, [P, P, I64, I32, P]),
    "cim22_cuda_nhwc_to_nchw": (c.c_int, [P, P, I32, I32, I32, I32, P]),
    "cim22_cuda_nchw_to_nhwc": (c.c_int, [P, P, I32, I32, I32, I32, P]),
    "cim22_cuda_unshard_columns": (c.c_int, [P, P, I32, I64, I64, I64, P]),
    "cim22_cuda_binary": (c.c_int, [P, P, P, I64, I32, c.c_float, c.c_float, P]),
    "cim22_cuda_fill": (c.c_int, [P, I64, c.c_float, P]),
    "cim22_cuda_copy": (c.c_int, [P, P, I64, P]),
    "cim22_cuda_slice_copy": (c.c_int, [P, P, I64, I64, I64, I64, P]),
    "cim22_cuda_chain_forward": (c.c_int, [P, I32, P, I64, P, P, P]),
    "cim22_cuda_maxpool2d_nchw": (c.c_int, [P, P, I32, I32, I32, I32, I32, I32, I32, P]),
    "cim22_cuda_avgpool2d_nchw": (c.c_int, [P, P, I32, I32, I32, I32, I32, I32, P]),
    "cim22_cuda_global_avgpool_nchw": (c.c_int, [P, P, I32, I32, I32, I32, P]),
    "cim22_cuda_channel_affine_nchw": (c.c_int, [P, P, P, P, I32, I32, I64, I32, P]),
}

EXPORTED = tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Load the CUDA backend. Raises ImportError when it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise ImportError(
                    f"{LIBRARY} is missing: build the CUDA backend with "
                    "`python mlir-cim22_b200/build.py` (no CPU fallback exists)")
            L = ctypes.CDLL(str(LIBRARY))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = L
    return _lib


def abi_sizes() -> list[int]:
    sizes = (ctypes.c_int64 * 16)()
    n = lib().cim22_cuda_abi_sizes(sizes, 16)
    return list(sizes[:n])


def last_error() -> str:
    return lib().cim22_cuda_last_error().decode(errors="replace")


def status_message(status: int) -> str:
    return lib().cim22_cuda_status_message(status).decode()


class CudaError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc:
        raise CudaError(f"{what}: {last_error() or status_message(rc)}")


def _err() -> ctypes.Array:
    return ctypes.create_string_buffer(512)


# ---------------------------------------------------------------------------
# Transaction executor (CIMRunner drop-in).


class CudaRunner:
    """CIM transaction executor on one CUDA device.

    Mirrors the reference's CIMSoftwareRunner: ``run`` takes a transaction,
    a BF16 compensation mode and host row views in binding order, and returns
    None or the runner's error message. Plans are cached per transaction spec
    object identity only for the duration of a call.
    """

    def __init__(self, device: int = 0) -> None:
        err = _err()
        self._handle = lib().cim22_cuda_runner_create(device, err, len(err))
        if not self._handle:
            raise CudaError(err.value.decode())

    def close(self) -> None:
        if getattr(self, "_handle", None):
            lib().cim22_cuda_runner_destroy(self._handle)
            self._handle = None

    def __del__(self) -> None:  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    @property
    def stats(self) -> tuple[int, int]:
        w, h = ctypes.c_uint64(), ctypes.c_uint64()
        lib().cim22_cuda_runner_weight_stats(self._handle, ctypes.byref(w), ctypes.byref(h))
        return w.value, h.value

    def clear(self) -> None:
        lib().cim22_cuda_runner_clear_residency(self._handle)

    def plan(self, spec: abi.TransactionSpec, batch: bool = False) -> "CudaPlan":
        return CudaPlan(self, spec, batch)

    def run(self, spec, mode: int, inputs, outputs, *, batch: bool = False,
            residency: bool = False, trace: list | None = None):
        plan = spec if isinstance(spec, CudaPlan) else self.plan(spec, batch)
        try:
            return plan.run(mode, inputs, outputs, residency=residency, trace=trace)
        finally:
            if plan is not spec:
                plan.close()


class CudaPlan:
    def __init__(self, runner: CudaRunner, spec: abi.TransactionSpec, batch: bool) -> None:
        self.runner = runner
        txn = spec.to_c()
        err = _err()
        self._handle = lib().cim22_cuda_plan_create(runner._handle, txn.pointer, int(batch),
                                                    err, len(err))
        if not self._handle:
            raise CudaError(err.value.decode())

    def close(self) -> None:
        if getattr(self, "_handle", None):
            lib().cim22_cuda_plan_destroy(self._handle)
            self._handle = None

    def run(self, mode: int, inputs, outputs, *, residency: bool = False,
            trace: list | None = None):
        in_ptrs = (ctypes.c_void_p * max(1, len(inputs)))(
            *[None if a is None else a.ctypes.data for a in inputs])
        out_ptrs = (ctypes.c_void_p * max(1, len(outputs)))(
            *[None if a is None else a.ctypes.data for a in outputs])

        def record(_ctx, event):
            e = event.contents
            trace.append((e.sequence, e.kind, e.group_id, e.work_id, e.macro_slot,
                          e.packet_index, e.cache_row_or_address))

        callback = abi.TraceCallback(record) if trace is not None else abi.TraceCallback()
        err = _err()
        rc = lib().cim22_cuda_runner_run(self.runner._handle, self._handle, mode, in_ptrs,
                                         len(inputs), out_ptrs, len(outputs), int(residency),
                                         callback, None, err, len(err))
        return err.value.decode() if rc else None


# ---------------------------------------------------------------------------
# Session and tile dispatch ABI.


class CudaSession:
    """Transactions in id order executed through the _mlir_ciface dispatch ABI."""

    def __init__(self, device: int = 0) -> None:
        err = _err()
        self._handle = lib().cim22_cuda_session_create(device, err, len(err))
        if not self._handle:
            raise CudaError(err.value.decode())

    def close(self) -> None:
        if getattr(self, "_handle", None):
            lib().cim22_cuda_session_destroy(self._handle)
            self._handle = None

    def add(self, spec: abi.TransactionSpec, kernel: str = "__cim_kernel_0") -> int:
        txn = spec.to_c()
        err = _err()
        index = lib().cim22_cuda_session_add_transaction(self._handle, txn.pointer,
                                                         kernel.encode(), err, len(err))
        if index < 0:
            raise CudaError(err.value.decode())
        return index

    @property
    def num_transactions(self) -> int:
        return lib().cim22_cuda_session_num_transactions(self._handle)

    def begin(self) -> None:
        lib().cim22_cuda_session_begin_invoke(self._handle)

    def end(self) -> int:
        return lib().cim22_cuda_session_end_invoke(self._handle)

    @property
    def dispatch_count(self) -> int:
        return lib().cim22_cuda_session_dispatch_count(self._handle)

    @property
    def error(self) -> str:
        return lib().cim22_cuda_session_error(self._handle).decode()


def memref(array: np.ndarray) -> abi.Memref2D:
    d = abi.Memref2D()
    d.allocated = d.aligned = array.ctypes.data
    d.offset = 0
    d.sizes[0], d.sizes[1] = array.shape
    d.strides[0], d.strides[1] = (s // array.itemsize for s in array.strides)
    return d


def dispatch(kind: str, transaction_id: int, inputs: np.ndarray, outputs: np.ndarray) -> None:
    """Call one _mlir_ciface_cim22_dispatch* symbol as generated model code does."""
    name = {"none": "_mlir_ciface_cim22_dispatch",
            "sign-split": "_mlir_ciface_cim22_dispatch_sign_split",
            "legacy": "_mlir_ciface_cim22_dispatch_legacy",
            "int8": "_mlir_ciface_cim22_dispatch_int8"}[kind]
    a, b = memref(inputs), memref(outputs)
    getattr(lib(), name)(transaction_id, ctypes.byref(a), ctypes.byref(b))
