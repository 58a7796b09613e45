"""Compiled CIM22 models on the CUDA runtime.

``Session`` mirrors ``cim22.runtime.Session`` (python/cim22/runtime.py of
mlir-cim22): it opens a compiled model library, exposes its static boundary
signature and runs synchronous inferences on NumPy arrays, with the same
argument checks and exception types. The model's tile calls
(_mlir_ciface_cim22_dispatch*) execute on a CUDA device instead of the
software runner. The USB board path (configure_usb, share_usb, clocks) is not
part of this runtime: a USB-backend model fails on its first tile call, as an
unconfigured reference Session does.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import numpy as np

from . import native

MODEL_SUFFIX = ".so"

# Artifact DataType -> NumPy dtype of a boundary tensor.
_BOUNDARY_DTYPES = {1: np.dtype(np.int8), 3: np.dtype(np.float32), 4: np.dtype(np.int32)}


def validate_artifact(data: bytes) -> None:
    """Decode and check a Protobuf model artifact; raise RuntimeError with the
    runtime's message when it is invalid."""
    error = ctypes.create_string_buffer(16384)
    buf = (ctypes.c_uint8 * max(1, len(data))).from_buffer_copy(data or b"\0")
    if native.lib().cim22_cuda_model_validate(buf, len(data), error, len(error)):
        raise RuntimeError(error.value.decode(errors="replace"))


class Session:
    """One loaded model on one CUDA device."""

    def __init__(self, artifact: str | os.PathLike, device: int = 0) -> None:
        artifact = Path(artifact)
        if artifact.suffix != MODEL_SUFFIX:
            raise ValueError(f"Session requires a compiled {MODEL_SUFFIX} model, got {artifact}")
        lib = native.lib()
        self._lock = threading.RLock()
        self._handle = None
        error = ctypes.create_string_buffer(16384)
        path = os.fsencode(artifact.resolve(strict=True))
        handle = lib.cim22_cuda_model_load_shared(path, device, error, len(error))
        if not handle:
            raise RuntimeError(error.value.decode(errors="replace"))
        self._handle = handle
        num_inputs = lib.cim22_cuda_model_num_inputs(handle)
        num_outputs = lib.cim22_cuda_model_num_outputs(handle)
        shapes = tuple(
            tuple(lib.cim22_cuda_model_dim(handle, i, d)
                  for d in range(lib.cim22_cuda_model_rank(handle, i)))
            for i in range(num_inputs + num_outputs))
        self.input_shapes = shapes[:num_inputs]
        self.output_shapes = shapes[num_inputs:]
        dtypes = tuple(_BOUNDARY_DTYPES[lib.cim22_cuda_model_dtype(handle, i)]
                       for i in range(num_inputs + num_outputs))
        self.input_dtypes = dtypes[:num_inputs]
        self.output_dtypes = dtypes[num_inputs:]
        self.num_transactions = lib.cim22_cuda_model_num_transactions(handle)

    def _require_open(self) -> None:
        if self._handle is None:
            raise RuntimeError("CIM22 session is closed")

    @property
    def dispatch_count(self) -> int:
        """Tile calls made by the last inference."""
        with self._lock:
            self._require_open()
            return native.lib().cim22_cuda_model_dispatch_count(self._handle)

    def __call__(self, *inputs: np.ndarray) -> tuple[np.ndarray, ...]:
        """Execute one synchronous inference; returns new output arrays."""
        with self._lock:
            self._require_open()
            if len(inputs) != len(self.input_shapes):
                raise ValueError("Input count differs from compiled signature")
            for index, (array, shape, dtype) in enumerate(
                    zip(inputs, self.input_shapes, self.input_dtypes, strict=True)):
                if not isinstance(array, np.ndarray) or array.dtype != dtype:
                    raise TypeError(f"Input {index} must be a NumPy {dtype.name} array")
                if array.shape != shape or not array.flags.c_contiguous \
                        or not array.flags.aligned:
                    raise ValueError(f"Input {index} requires aligned, contiguous shape {shape}")
            outputs = tuple(np.empty(shape, dtype=dtype)
                            for shape, dtype in zip(self.output_shapes, self.output_dtypes,
                                                    strict=True))
            arrays = (*inputs, *outputs)
            pointers = (ctypes.c_void_p * len(arrays))(*(a.ctypes.data for a in arrays))
            counts = (ctypes.c_int64 * len(arrays))(*(a.size for a in arrays))
            lib = native.lib()
            if lib.cim22_cuda_model_invoke(self._handle, pointers, counts, len(arrays)):
                raise RuntimeError(
                    lib.cim22_cuda_model_error(self._handle).decode(errors="replace"))
            return outputs

    def close(self) -> None:
        """Release the model library and its device state; outputs stay valid."""
        with self._lock:
            if self._handle is not None:
                native.lib().cim22_cuda_model_destroy(self._handle)
                self._handle = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self) -> "Session":
        self._require_open()
        return self

    def __exit__(self, *exc) -> None:
        self.close()
