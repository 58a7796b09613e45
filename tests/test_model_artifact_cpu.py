"""Model artifact decoding and checking, and the model loader's error paths.

Artifacts are serialized by the official protobuf runtime from the schema of
schema/cim22_model.proto; every rejection below is one check of
runtime/src/ModelArtifact.cpp:101-266 and must give its exact text. Nothing
here creates a CUDA context: each load below fails before the session is made.
"""

import copy

import numpy as np
import pytest

import model_fixtures as mf
import txn_fixtures as fx
from cim22_b200 import native
from cim22_b200.runtime import Session, validate_artifact


def supplier_model(backend: int = 0):
    weight = np.arange(1024, dtype=np.int64).reshape(16, 64) % 7 - 3
    spec = fx.make_supplier_case(weight.astype(np.int8))
    return mf.artifact([("__cim_kernel_0", spec)], [((8, 64), mf.INT8)],
                       [((8, 16), mf.INT32)], backend)


def bf16_model():
    spec = fx.make_bf16_executable(True, 0, fx.bf16_weight(64, 126))
    return mf.artifact([("__cim_kernel_0", spec)], [((1, 64), mf.FP32)],
                       [((1, 16), mf.FP32)])


def reason(text: str) -> str:
    return f"invalid CIM22 Protobuf model: {text}; recompile the model"


def check(model, text):
    with pytest.raises(RuntimeError) as info:
        validate_artifact(model.SerializeToString())
    assert str(info.value) == reason(text)


def test_valid_artifacts_decode():
    validate_artifact(supplier_model().SerializeToString())
    validate_artifact(supplier_model(backend=1).SerializeToString())
    validate_artifact(bf16_model().SerializeToString())
    validate_artifact(mf.artifact([], [((2, 3), mf.FP32)], []).SerializeToString())


def test_unknown_fields_are_ignored():
    data = supplier_model().SerializeToString()
    # Field 99 as a varint and field 100 as length-delimited bytes.
    validate_artifact(data + bytes([0x98, 0x06, 0x01, 0xA2, 0x06, 0x02, 0x41, 0x42]))


def test_malformed_data():
    data = supplier_model().SerializeToString()
    for bad in (b"", data[:-3], b"\x0a\xff\xff\xff\xff\x0f", b"\x00\x01"):
        with pytest.raises(RuntimeError) as info:
            validate_artifact(bad)
        assert str(info.value) == reason("malformed data (old custom binary is unsupported)")


def test_model_level_checks():
    m = supplier_model()
    m.backend = 2
    check(m, "unsupported runtime backend")
    m = supplier_model()
    m.inputs[0].data_type = mf.BF16
    check(m, "boundary requires contiguous CPU INT8, FP32 or INT32 tensors")
    m = supplier_model()
    m.outputs[0].dimensions[1] = 0
    check(m, "static tensor shape/element count")
    m = supplier_model()
    m.outputs[0].dimensions[:] = [1 << 40, 1 << 40]
    check(m, "static tensor shape/element count")
    m = supplier_model()
    m.kernels.add().CopyFrom(m.kernels[0])
    check(m, "missing/duplicate kernel name or transaction")
    m = supplier_model()
    m.kernels[0].kernel_name = ""
    check(m, "missing/duplicate kernel name or transaction")
    m = supplier_model()
    m.kernels[0].ClearField("transaction")
    check(m, "missing/duplicate kernel name or transaction")


def txn(m):
    return m.kernels[0].transaction


def test_group_work_and_weight_checks():
    m = supplier_model()
    txn(m).target_profile = "cim22-4x4-v1"
    check(m, "unsupported transaction profile")
    m = supplier_model()
    txn(m).groups[1].group_id = 0
    check(m, "missing/duplicate group or empty works")
    m = supplier_model()
    txn(m).groups[0].ClearField("group_id")
    check(m, "missing/duplicate group or empty works")
    m = supplier_model()
    del txn(m).groups[0].works[:]
    check(m, "missing/duplicate group or empty works")
    for field, value in (("core_slot", 20), ("macro_slot", 2), ("work_id", -1)):
        m = supplier_model()
        setattr(txn(m).groups[0].works[0], field, value)
        check(m, "missing/duplicate work, placement or route length")
    m = supplier_model()
    del txn(m).groups[0].works[0].route[5]
    check(m, "missing/duplicate work, placement or route length")
    m = supplier_model()
    txn(m).groups[0].works[0].ClearField("macro_slot")
    check(m, "missing/duplicate work, placement or route length")
    m = supplier_model()
    txn(m).groups[0].works.add().CopyFrom(txn(m).groups[0].works[0])
    txn(m).groups[0].works[1].work_id = 99
    check(m, "missing/duplicate work, placement or route length")
    m = supplier_model()
    del txn(m).flits[:]
    check(m, "empty transaction works/flits")
    for mutate in (lambda w: w.words.pop(), lambda w: setattr(w, "values", w.values[:-1]),
                   lambda w: setattr(w, "exponents", w.exponents + b"\0"),
                   lambda w: setattr(w, "resource", ""),
                   lambda w: w.route.__setitem__(0, 1),
                   lambda w: setattr(w, "core_slot", 3),
                   lambda w: setattr(w, "macro_slot", 1),
                   lambda w: setattr(w, "data_type", mf.FP32)):
        m = supplier_model()
        mutate(txn(m).weights[0])
        check(m, "weight binding, array length or datatype")
    m = supplier_model()
    txn(m).weights.add().CopyFrom(txn(m).weights[0])
    check(m, "weight binding, array length or datatype")


def test_input_readback_and_datatype_checks():
    for field, value in (("input_cache_address", 8), ("input_slot", -1), ("work_id", 77)):
        m = supplier_model()
        setattr(txn(m).inputs[0], field, value)
        check(m, "input binding or datatype")
    m = supplier_model()
    txn(m).inputs[0].ClearField("input_cache_address")
    validate_artifact(m.SerializeToString())  # a software model may omit it
    m = supplier_model(backend=1)
    txn(m).inputs[0].ClearField("input_cache_address")
    check(m, "input binding or datatype")
    m = supplier_model()
    txn(m).readbacks[0].output_cache_address = 8
    check(m, "readback binding, array length or datatype")
    m = supplier_model()
    del txn(m).readbacks[0].test_core[2]
    check(m, "readback binding, array length or datatype")
    m = supplier_model()
    txn(m).readbacks[0].route[3] = 2
    check(m, "readback binding, array length or datatype")
    m = supplier_model()
    del txn(m).inputs[3]
    check(m, "incomplete work bindings")
    m = supplier_model()
    txn(m).inputs[2].data_type = mf.BF16
    check(m, "inconsistent work datatypes")


def find_packet(m, kind, group=0):
    for i, p in enumerate(txn(m).packets):
        if p.kind == kind and p.group_id == group:
            return i
    raise AssertionError(kind)


CONTROL, WEIGHT, EXPONENT, WORK, INPUT, RETURN, READ = range(1, 8)


def test_packet_checks():
    cases = [
        (lambda p: setattr(p[find_packet_m(p, WEIGHT)], "kind", 0),
         "packet enum, missing field or array/address"),
        (lambda p: setattr(p[find_packet_m(p, WEIGHT)], "kind", 8),
         "packet enum, missing field or array/address"),
        (lambda p: p[find_packet_m(p, WEIGHT)].ClearField("cache_address"),
         "packet enum, missing field or array/address"),
        (lambda p: setattr(p[find_packet_m(p, WEIGHT)], "cache_address", 8),
         "packet enum, missing field or array/address"),
        (lambda p: p[find_packet_m(p, WEIGHT)].test_core.pop(),
         "packet enum, missing field or array/address"),
        (lambda p: setattr(p[find_packet_m(p, WEIGHT)], "data_type", mf.FP32),
         "packet enum, missing field or array/address"),
        (lambda p: (setattr(p[find_packet_m(p, WEIGHT)], "work_id", -1),
                    setattr(p[find_packet_m(p, WEIGHT)], "group_id", 42)),
         "packet references unknown group"),
        (lambda p: setattr(p[find_packet_m(p, WEIGHT)], "work_id", 5),
         "packet references unknown work/placement"),
        (lambda p: setattr(p[find_packet_m(p, WEIGHT)], "work_id", -1),
         "packet missing work binding"),
        (lambda p: setattr(p[find_packet_m(p, WEIGHT)], "data_type", mf.BF16),
         "packet datatype differs from work"),
        (lambda p: p[find_packet_m(p, INPUT)].route.__setitem__(0, 3),
         "packet route differs from binding"),
        (lambda p: p[find_packet_m(p, RETURN)].test_core.__setitem__(0, 1),
         "packet test core differs from readback"),
        (lambda p: setattr(p[find_packet_m(p, READ)], "cache_address", 5),
         "packet readback address differs from binding"),
        (lambda p: setattr(p[find_packet_m(p, RETURN) + 1], "kind", WEIGHT),
         "inconsistent readback packet sequence"),
        (lambda p: setattr(p[find_packet_m(p, RETURN) + 2], "macro_slot", -1),
         "inconsistent readback packet sequence"),
        (lambda p: p.__delitem__(slice(find_packet_m(p, READ, 7), None)),
         "incomplete readback packet sequence"),
        (lambda p: p.__delitem__(find_packet_m(p, WEIGHT)),
         "work binding has no matching packet"),
    ]
    for mutate, text in cases:
        m = supplier_model()
        mutate(txn(m).packets)
        check(m, text)
    # A WORK packet needs a group; CONTROL may stand alone (-1 bindings).
    m = supplier_model()
    txn(m).packets.add(kind=CONTROL, route=[0] * 6, group_id=-1, work_id=-1, macro_slot=-1,
                       cache_address=-1, test_core=[0] * 3, data_type=mf.INT8)
    validate_artifact(m.SerializeToString())
    m = supplier_model()
    txn(m).packets.add(kind=WORK, route=[0] * 6, group_id=-1, work_id=-1, macro_slot=-1,
                       cache_address=-1, test_core=[0] * 3, data_type=mf.INT8)
    check(m, "work packet missing group")
    m = bf16_model()
    del txn(m).packets[find_packet(m, EXPONENT)]
    check(m, "BF16 weight binding has no exponent packet")


def find_packet_m(packets, kind, group=0):
    for i, p in enumerate(packets):
        if p.kind == kind and p.group_id == group:
            return i
    raise AssertionError(kind)


def test_loader_errors_before_any_device_work(tmp_path):
    lib = native.lib()
    err = native._err()
    assert lib.cim22_cuda_model_load_shared(str(tmp_path / "absent.so").encode(), 0, err,
                                            len(err)) is None
    assert "absent.so" in err.value.decode()
    assert lib.cim22_cuda_model_load_shared(None, 0, err, len(err)) is None
    assert err.value == b"missing model library path"
    no_model = mf.build_library_without_descriptor(tmp_path)
    with pytest.raises(RuntimeError, match="^incompatible CIM22 model ABI$"):
        Session(no_model)
    data = supplier_model().SerializeToString()
    v2 = mf.build_model_library(tmp_path, "abi2", data, mf.INT8_BODY, abi_version=2, ROWS=8)
    with pytest.raises(RuntimeError, match="^incompatible CIM22 model ABI$"):
        Session(v2)
    bad = copy.deepcopy(supplier_model())
    txn(bad).target_profile = "other"
    lib_bad = mf.build_model_library(tmp_path, "bad", bad.SerializeToString(), mf.INT8_BODY,
                                     ROWS=8)
    with pytest.raises(RuntimeError) as info:
        Session(lib_bad)
    assert str(info.value) == reason("unsupported transaction profile")
    with pytest.raises(ValueError, match="compiled .so model"):
        Session(tmp_path / "model.bin")
    with pytest.raises(FileNotFoundError):
        Session(tmp_path / "missing.so")


def test_null_model_accessors():
    lib = native.lib()
    assert lib.cim22_cuda_model_num_inputs(None) == -1
    assert lib.cim22_cuda_model_num_outputs(None) == -1
    assert lib.cim22_cuda_model_rank(None, 0) == -1
    assert lib.cim22_cuda_model_dim(None, 0, 0) == -1
    assert lib.cim22_cuda_model_dtype(None, 0) == -1
    assert lib.cim22_cuda_model_num_transactions(None) == -1
    assert lib.cim22_cuda_model_dispatch_count(None) == 0
    assert lib.cim22_cuda_model_error(None) == b"null session"
    assert lib.cim22_cuda_model_invoke(None, None, None, 0) == 1
