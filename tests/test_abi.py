"""The C ABI library loads and exports every entry point include/*.h declares.

CPU only: nothing here launches a kernel.
"""

import re
from pathlib import Path

import pytest

from cim22_b200 import abi, native

REPO = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    names = set()
    for header in (REPO / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"\b((?:cim22_cuda|_mlir_ciface_cim22)\w*)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = native.lib()
    declared = declared_functions()
    assert len(declared) >= 40
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    assert declared == set(native.EXPORTED)


def test_ctypes_layout_matches_c_layout():
    import ctypes

    assert native.abi_sizes() == [ctypes.sizeof(s) for s in abi.ABI_STRUCTS]


def test_status_messages_follow_reference_text():
    assert native.status_message(0) == ""
    assert native.status_message(1) == "CIM BF16 input does not support NaN or infinity"
    assert native.status_message(2) == "CIM BF16 compensated tile exceeds BF16"
    assert native.status_message(4) == "CIM software result exceeds signed i21 range"


def test_host_argument_checks_fail_without_launching():
    lib = native.lib()
    # Null arguments are rejected before any device work.
    assert lib.cim22_cuda_relu(None, None, 4, None) != 0
    assert "cim22_cuda_relu" in native.last_error()
    assert lib.cim22_cuda_layer_forward_bf16(None, None, None, 1, None, 0, 4, None, None, 0,
                                             None, None) != 0


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(native, "LIBRARY", tmp_path / "absent.so")
    monkeypatch.setattr(native, "_lib", None)
    with pytest.raises(ImportError, match="no CPU fallback"):
        native.lib()
