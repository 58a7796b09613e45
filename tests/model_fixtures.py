"""Compiled-model fixtures: Protobuf artifacts and model libraries.

The artifact schema is schema/cim22_model.proto of mlir-cim22 (package
cim22.artifact.v1). It is declared here as a FileDescriptorProto so that the
official protobuf runtime serializes the test artifacts: the CUDA runtime's
own wire decoder is then checked against real Protobuf output, not against a
second hand-written encoder.

A model library is what the reference compiler emits: a shared object that
exports ``cim22_model_v1()`` (include/CIM22/Runtime/ModelABI.h) with the
artifact bytes and an MLIR packed-argument entry point, whose body calls the
``_mlir_ciface_cim22_dispatch*`` tile ABI. The fixtures compile a small C
body with gcc into such a library.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

from cim22_b200.abi import DATA_BF16, TransactionSpec

_F = descriptor_pb2.FieldDescriptorProto
_OPT, _REP = _F.LABEL_OPTIONAL, _F.LABEL_REPEATED

# (name, number, type, label, type_name, proto3_optional, packed)
_MESSAGES = {
    "ModelArtifact": [
        ("schema_version", 1, _F.TYPE_UINT32, _OPT, None, False, False),
        ("inputs", 2, _F.TYPE_MESSAGE, _REP, "TensorSignature", False, False),
        ("outputs", 3, _F.TYPE_MESSAGE, _REP, "TensorSignature", False, False),
        ("kernels", 4, _F.TYPE_MESSAGE, _REP, "Kernel", False, False),
        ("backend", 5, _F.TYPE_ENUM, _OPT, "RuntimeBackend", False, False),
    ],
    "TensorSignature": [
        ("dimensions", 1, _F.TYPE_INT64, _REP, None, False, True),
        ("data_type", 2, _F.TYPE_ENUM, _OPT, "DataType", False, False),
    ],
    "Kernel": [
        ("kernel_name", 1, _F.TYPE_STRING, _OPT, None, False, False),
        ("transaction", 2, _F.TYPE_MESSAGE, _OPT, "Transaction", False, False),
    ],
    "Transaction": [
        ("target_profile", 1, _F.TYPE_STRING, _OPT, None, False, False),
        ("groups", 2, _F.TYPE_MESSAGE, _REP, "Group", False, False),
        ("weights", 3, _F.TYPE_MESSAGE, _REP, "StaticWeight", False, False),
        ("packets", 4, _F.TYPE_MESSAGE, _REP, "Packet", False, False),
        ("inputs", 5, _F.TYPE_MESSAGE, _REP, "InputBinding", False, False),
        ("readbacks", 6, _F.TYPE_MESSAGE, _REP, "ReadbackBinding", False, False),
        ("flits", 7, _F.TYPE_FIXED64, _REP, None, False, True),
    ],
    "Group": [
        ("group_id", 1, _F.TYPE_INT64, _OPT, None, True, False),
        ("works", 2, _F.TYPE_MESSAGE, _REP, "Work", False, False),
    ],
    "Work": [
        ("work_id", 1, _F.TYPE_INT64, _OPT, None, True, False),
        ("core_slot", 2, _F.TYPE_INT64, _OPT, None, True, False),
        ("macro_slot", 3, _F.TYPE_INT64, _OPT, None, True, False),
        ("route", 4, _F.TYPE_SFIXED32, _REP, None, False, True),
    ],
    "StaticWeight": [
        ("group_id", 1, _F.TYPE_INT64, _OPT, None, True, False),
        ("work_id", 2, _F.TYPE_INT64, _OPT, None, True, False),
        ("core_slot", 3, _F.TYPE_INT64, _OPT, None, True, False),
        ("macro_slot", 4, _F.TYPE_INT64, _OPT, None, True, False),
        ("resource", 5, _F.TYPE_STRING, _OPT, None, False, False),
        ("route", 6, _F.TYPE_SFIXED32, _REP, None, False, True),
        ("words", 7, _F.TYPE_SFIXED32, _REP, None, False, True),
        ("values", 8, _F.TYPE_BYTES, _OPT, None, False, False),
        ("exponents", 9, _F.TYPE_BYTES, _OPT, None, False, False),
        ("data_type", 10, _F.TYPE_ENUM, _OPT, "DataType", False, False),
    ],
    "Packet": [
        ("kind", 1, _F.TYPE_ENUM, _OPT, "PacketKind", False, False),
        ("route", 2, _F.TYPE_SFIXED32, _REP, None, False, True),
        ("group_id", 3, _F.TYPE_INT64, _OPT, None, True, False),
        ("work_id", 4, _F.TYPE_INT64, _OPT, None, True, False),
        ("macro_slot", 5, _F.TYPE_INT64, _OPT, None, True, False),
        ("cache_address", 6, _F.TYPE_INT64, _OPT, None, True, False),
        ("test_core", 7, _F.TYPE_SFIXED32, _REP, None, False, True),
        ("data_type", 8, _F.TYPE_ENUM, _OPT, "DataType", False, False),
    ],
    "InputBinding": [
        ("group_id", 1, _F.TYPE_INT64, _OPT, None, True, False),
        ("work_id", 2, _F.TYPE_INT64, _OPT, None, True, False),
        ("macro_slot", 3, _F.TYPE_INT64, _OPT, None, True, False),
        ("input_slot", 4, _F.TYPE_INT64, _OPT, None, True, False),
        ("data_type", 5, _F.TYPE_ENUM, _OPT, "DataType", False, False),
        ("input_cache_address", 6, _F.TYPE_INT64, _OPT, None, True, False),
    ],
    "ReadbackBinding": [
        ("group_id", 1, _F.TYPE_INT64, _OPT, None, True, False),
        ("work_id", 2, _F.TYPE_INT64, _OPT, None, True, False),
        ("macro_slot", 3, _F.TYPE_INT64, _OPT, None, True, False),
        ("output_cache_address", 4, _F.TYPE_INT64, _OPT, None, True, False),
        ("route", 5, _F.TYPE_SFIXED32, _REP, None, False, True),
        ("test_core", 6, _F.TYPE_SFIXED32, _REP, None, False, True),
        ("data_type", 7, _F.TYPE_ENUM, _OPT, "DataType", False, False),
    ],
}
_ENUMS = {
    "RuntimeBackend": [("SOFTWARE", 0), ("USB", 1)],
    "DataType": [("UNSPECIFIED", 0), ("INT8", 1), ("BF16", 2), ("FP32", 3), ("INT32", 4)],
    "PacketKind": [("PACKET_KIND_UNSPECIFIED", 0), ("CONTROL", 1), ("WEIGHT", 2),
                   ("WEIGHT_EXPONENT", 3), ("WORK", 4), ("INPUT_CACHE_WRITE", 5),
                   ("RETURN_ROUTE", 6), ("OUTPUT_CACHE_READ", 7)],
}
_PACKAGE = "cim22.artifact.v1"

# Artifact DataType values of the boundary tensors.
INT8, BF16, FP32, INT32 = 1, 2, 3, 4


def _file_descriptor() -> descriptor_pb2.FileDescriptorProto:
    fd = descriptor_pb2.FileDescriptorProto(name="cim22_model_test.proto", package=_PACKAGE,
                                            syntax="proto3")
    for name, values in _ENUMS.items():
        e = fd.enum_type.add(name=name)
        for vname, number in values:
            e.value.add(name=vname, number=number)
    for name, fields in _MESSAGES.items():
        m = fd.message_type.add(name=name)
        for fname, number, ftype, label, tname, optional, packed in fields:
            f = m.field.add(name=fname, number=number, type=ftype, label=label)
            if tname:
                f.type_name = f".{_PACKAGE}.{tname}"
            if packed:
                f.options.packed = True
            if optional:
                f.proto3_optional = True
                f.oneof_index = len(m.oneof_decl)
                m.oneof_decl.add(name=f"_{fname}")
    return fd


_pool = descriptor_pool.DescriptorPool()
_pool.Add(_file_descriptor())
_CLASSES = {name: message_factory.GetMessageClass(_pool.FindMessageTypeByName(
    f"{_PACKAGE}.{name}")) for name in _MESSAGES}
ModelArtifact = _CLASSES["ModelArtifact"]


def _kind(kind: int) -> int:
    return kind + 1  # native CIM22_PACKET_CONTROL = 0 is proto CONTROL = 1


def _dtype(data_type: int) -> int:
    return BF16 if data_type == DATA_BF16 else INT8


def transaction_message(spec: TransactionSpec, msg) -> None:
    """Fill a Transaction message from a TransactionSpec, as the compiler's
    encodeTransaction does (runtime/src/ModelArtifact.cpp:291-336)."""
    msg.target_profile = spec.target_profile
    for g in spec.groups:
        group = msg.groups.add(group_id=g.group_id)
        for work_id, core, macro in g.works:
            group.works.add(work_id=work_id, core_slot=core, macro_slot=macro,
                            route=[0] * 6)
    for w in spec.weights:
        words = list(w.words) if len(w.words) else [0] * 256
        msg.weights.add(group_id=w.group_id, work_id=w.work_id, core_slot=w.core_slot,
                        macro_slot=w.macro_slot, resource=f"weight_{w.group_id}_{w.work_id}",
                        route=list(w.route), words=words,
                        values=np.ascontiguousarray(w.values, np.int8).tobytes(),
                        exponents=np.ascontiguousarray(w.exponents, np.uint8).tobytes(),
                        data_type=_dtype(w.data_type))
    for p in spec.packets:
        msg.packets.add(kind=_kind(p.kind), route=list(p.route), group_id=p.group_id,
                        work_id=p.work_id, macro_slot=p.macro_slot,
                        cache_address=p.cache_address, test_core=list(p.test_core),
                        data_type=_dtype(p.data_type))
    for b in spec.inputs:
        msg.inputs.add(group_id=b.group_id, work_id=b.work_id, macro_slot=b.macro_slot,
                       input_slot=b.input_slot, data_type=_dtype(b.data_type),
                       input_cache_address=b.input_cache_address)
    for b in spec.readbacks:
        msg.readbacks.add(group_id=b.group_id, work_id=b.work_id, macro_slot=b.macro_slot,
                          output_cache_address=b.output_cache_address, route=list(b.route),
                          test_core=list(b.test_core), data_type=_dtype(b.data_type))
    msg.flits.append(0x0123456789ABCDEF)


def artifact(kernels, inputs, outputs, backend: int = 0):
    """A ModelArtifact message: kernels is [(name, TransactionSpec)], inputs and
    outputs are [(dims, data_type)]."""
    model = ModelArtifact(schema_version=1, backend=backend)
    for dims, dtype in inputs:
        model.inputs.add(dimensions=list(dims), data_type=dtype)
    for dims, dtype in outputs:
        model.outputs.add(dimensions=list(dims), data_type=dtype)
    for name, spec in kernels:
        kernel = model.kernels.add(kernel_name=name)
        transaction_message(spec, kernel.transaction)
    return model


# Entry point bodies. `args[i]` points at a pointer to argument i's MLIR ranked
# descriptor {allocated, aligned, offset, sizes[r], strides[r]}, inputs first.
MODEL_C = r"""
#include <stdint.h>
#include <string.h>

typedef struct { void *allocated, *aligned; int64_t offset, sizes[2], strides[2]; } memref2d;
typedef struct {
  uint64_t abi_version;
  const uint8_t *data;
  uint64_t data_size;
  void (*invoke)(void **);
} CIM22ModelV1;

void _mlir_ciface_cim22_dispatch(int64_t, memref2d *, memref2d *);
void _mlir_ciface_cim22_dispatch_sign_split(int64_t, memref2d *, memref2d *);
void _mlir_ciface_cim22_dispatch_legacy(int64_t, memref2d *, memref2d *);
void _mlir_ciface_cim22_dispatch_int8(int64_t, memref2d *, memref2d *);

static const uint8_t artifact[] = {ARTIFACT_BYTES};

static void *data_of(void **args, int i) {
  int64_t *desc = *(int64_t **)args[i];
  void *aligned;
  memcpy(&aligned, desc + 1, sizeof aligned);
  return aligned;
}

static memref2d tile(void *data, int64_t rows, int64_t cols) {
  memref2d m = {data, data, 0, {rows, cols}, {cols, 1}};
  return m;
}

static void invoke(void **args) {
BODY
}

static const CIM22ModelV1 model = {ABI_VERSION, artifact, sizeof artifact, invoke};
const CIM22ModelV1 *cim22_model_v1(void) { return &model; }
"""

# One INT8 kernel over [rows, 64] -> [rows, 16]: input 0 -> output 1.
INT8_BODY = """
  memref2d in = tile(data_of(args, 0), ROWS, 64), out = tile(data_of(args, 1), ROWS, 16);
  _mlir_ciface_cim22_dispatch_int8(0, &in, &out);
"""

# Two INT8 kernels over the same input: input 0 -> outputs 1 and 2.
TWO_KERNEL_BODY = """
  memref2d in = tile(data_of(args, 0), ROWS, 64);
  memref2d a = tile(data_of(args, 1), ROWS, 16), b = tile(data_of(args, 2), ROWS, 16);
  _mlir_ciface_cim22_dispatch_int8(0, &in, &a);
  _mlir_ciface_cim22_dispatch_int8(1, &in, &b);
"""

# One sign-split BF16 kernel with the compiler's Host glue around it: FP32
# [rows, 64] rounded to BF16 (nearest-even), the tile call, BF16 widened back
# to FP32 [rows, 16].
BF16_BODY = """
  const float *x = (const float *)data_of(args, 0);
  float *y = (float *)data_of(args, 1);
  uint16_t in_bits[ROWS * 64], out_bits[ROWS * 16];
  for (int i = 0; i < ROWS * 64; ++i) {
    uint32_t u;
    memcpy(&u, &x[i], 4);
    in_bits[i] = (uint16_t)((u + 0x7fff + ((u >> 16) & 1)) >> 16);
  }
  memref2d in = tile(in_bits, ROWS, 64), out = tile(out_bits, ROWS, 16);
  DISPATCH(0, &in, &out);
  for (int i = 0; i < ROWS * 16; ++i) {
    uint32_t u = (uint32_t)out_bits[i] << 16;
    memcpy(&y[i], &u, 4);
  }
"""


def build_model_library(directory: Path, name: str, data: bytes, body: str,
                        abi_version: int = 1, **macros) -> Path:
    """Compile a model library exporting cim22_model_v1 with gcc."""
    text = MODEL_C.replace("ARTIFACT_BYTES", ",".join(str(b) for b in data) or "0")
    text = text.replace("ABI_VERSION", str(abi_version)).replace("BODY", body)
    for key, value in macros.items():
        text = text.replace(key, str(value))
    src = Path(directory) / f"{name}.c"
    out = Path(directory) / f"{name}.so"
    src.write_text(text)
    subprocess.run(["gcc", "-O1", "-shared", "-fPIC", "-o", str(out), str(src)], check=True)
    return out


def build_library_without_descriptor(directory: Path) -> Path:
    src = Path(directory) / "no_model.c"
    out = Path(directory) / "no_model.so"
    src.write_text("int not_a_model(void) { return 0; }\n")
    subprocess.run(["gcc", "-shared", "-fPIC", "-o", str(out), str(src)], check=True)
    return out
