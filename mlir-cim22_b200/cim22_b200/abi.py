"""ctypes mirror of the plain-C data structures in include/cim22_cuda.h.

The transaction structures carry the data of the reference's
``cim22::execution::CIMTransaction`` (include/CIM22/Execution/CIMExecutable.h
of mlir-cim22); the library reports the C sizes of each structure through
``cim22_cuda_abi_sizes`` so the layout here is checked against the compiler's.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

DATA_INT8 = 0
DATA_BF16 = 1

PACKET_CONTROL = 0
PACKET_WEIGHT = 1
PACKET_WEIGHT_EXPONENT = 2
PACKET_WORK = 3
PACKET_INPUT_CACHE_WRITE = 4
PACKET_RETURN_ROUTE = 5
PACKET_OUTPUT_CACHE_READ = 6

BF16_NONE = 0
BF16_LEGACY = 1
BF16_SIGN_SPLIT = 2

COMPENSATION = {"none": BF16_NONE, "legacy": BF16_LEGACY, "sign-split": BF16_SIGN_SPLIT}

TRACE_BEGIN_RUN = 0
TRACE_CONFIGURE_WEIGHT = 1
TRACE_CONFIGURE_INPUT = 2
TRACE_SELECT_MACRO = 3
TRACE_START_WORK = 4
TRACE_CONFIGURE_RETURN_ROUTE = 5
TRACE_READ_OUTPUT = 6
TRACE_COMPLETE = 7
TRACE_ERROR = 8

I32x6 = ctypes.c_int32 * 6
I32x3 = ctypes.c_int32 * 3


class FramePacket(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("route", I32x6),
        ("group_id", ctypes.c_int64),
        ("work_id", ctypes.c_int64),
        ("macro_slot", ctypes.c_int64),
        ("cache_address", ctypes.c_int64),
        ("test_core", I32x3),
        ("data_type", ctypes.c_int32),
    ]


class StaticWeight(ctypes.Structure):
    _fields_ = [
        ("group_id", ctypes.c_int64),
        ("work_id", ctypes.c_int64),
        ("core_slot", ctypes.c_int64),
        ("macro_slot", ctypes.c_int64),
        ("route", I32x6),
        ("words", ctypes.POINTER(ctypes.c_int32)),
        ("num_words", ctypes.c_int64),
        ("values", ctypes.c_int8 * 1024),
        ("exponents", ctypes.c_uint8 * 16),
        ("data_type", ctypes.c_int32),
    ]


class InputBinding(ctypes.Structure):
    _fields_ = [
        ("group_id", ctypes.c_int64),
        ("work_id", ctypes.c_int64),
        ("macro_slot", ctypes.c_int64),
        ("input_slot", ctypes.c_int64),
        ("data_type", ctypes.c_int32),
        ("input_cache_address", ctypes.c_int64),
    ]


class ReadbackBinding(ctypes.Structure):
    _fields_ = [
        ("group_id", ctypes.c_int64),
        ("work_id", ctypes.c_int64),
        ("macro_slot", ctypes.c_int64),
        ("output_cache_address", ctypes.c_int64),
        ("route", I32x6),
        ("test_core", I32x3),
        ("data_type", ctypes.c_int32),
    ]


class Work(ctypes.Structure):
    _fields_ = [
        ("work_id", ctypes.c_int64),
        ("core_slot", ctypes.c_int64),
        ("macro_slot", ctypes.c_int64),
        ("route", I32x6),
    ]


class Group(ctypes.Structure):
    _fields_ = [
        ("group_id", ctypes.c_int64),
        ("works", ctypes.POINTER(Work)),
        ("num_works", ctypes.c_int64),
    ]


class Transaction(ctypes.Structure):
    _fields_ = [
        ("target_profile", ctypes.c_char_p),
        ("target_profile_version", ctypes.c_int64),
        ("execution_plan_version", ctypes.c_int64),
        ("groups", ctypes.POINTER(Group)),
        ("num_groups", ctypes.c_int64),
        ("weights", ctypes.POINTER(StaticWeight)),
        ("num_weights", ctypes.c_int64),
        ("packets", ctypes.POINTER(FramePacket)),
        ("num_packets", ctypes.c_int64),
        ("inputs", ctypes.POINTER(InputBinding)),
        ("num_inputs", ctypes.c_int64),
        ("readbacks", ctypes.POINTER(ReadbackBinding)),
        ("num_readbacks", ctypes.c_int64),
    ]


class TraceEvent(ctypes.Structure):
    _fields_ = [
        ("sequence", ctypes.c_uint64),
        ("kind", ctypes.c_int32),
        ("group_id", ctypes.c_int64),
        ("work_id", ctypes.c_int64),
        ("macro_slot", ctypes.c_int64),
        ("packet_index", ctypes.c_int64),
        ("cache_row_or_address", ctypes.c_int64),
    ]


TraceCallback = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.POINTER(TraceEvent))


class Memref2D(ctypes.Structure):
    _fields_ = [
        ("allocated", ctypes.c_void_p),
        ("aligned", ctypes.c_void_p),
        ("offset", ctypes.c_int64),
        ("sizes", ctypes.c_int64 * 2),
        ("strides", ctypes.c_int64 * 2),
    ]


class Gather(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("channels", ctypes.c_int32),
        ("height", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("kernel_h", ctypes.c_int32),
        ("kernel_w", ctypes.c_int32),
        ("stride_h", ctypes.c_int32),
        ("stride_w", ctypes.c_int32),
        ("pad_h", ctypes.c_int32),
        ("pad_w", ctypes.c_int32),
        ("out_h", ctypes.c_int32),
        ("out_w", ctypes.c_int32),
        ("pool_kernel", ctypes.c_int32),
        ("pool_stride", ctypes.c_int32),
        ("pool_src_h", ctypes.c_int32),
        ("pool_src_w", ctypes.c_int32),
    ]


GATHER_ROWS = 0
GATHER_CONV_NCHW = 1
GATHER_CONV_NHWC = 2

# cim22_cuda_binary operations (include/cim22_cuda.h).
(BINARY_ADD, BINARY_SUB, BINARY_MUL, BINARY_DIV, BINARY_GE, BINARY_GT, BINARY_LE, BINARY_LT,
 BINARY_EQ, BINARY_NE, BINARY_MAX, BINARY_MIN) = range(12)


class ChainLayer(ctypes.Structure):
    """cim22_chain_layer: one layer of cim22_cuda_chain_forward."""

    _fields_ = [
        ("kind", ctypes.c_int32),
        ("layer", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("channels", ctypes.c_int32),
        ("height", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("kernel_h", ctypes.c_int32),
        ("kernel_w", ctypes.c_int32),
        ("stride", ctypes.c_int32),
        ("pad", ctypes.c_int32),
        ("branches", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("pool", ctypes.c_int32),
    ]


CHAIN_LINEAR = 0
CHAIN_CONV = 1

MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class PeerOutputs(ctypes.Structure):
    """cim22_peer_outputs: each rank's full [rows][row_stride] output as mapped
    on this device, and this rank's lane block within a row."""
    _fields_ = [
        ("out", ctypes.c_void_p * MAX_PEERS),
        ("ranks", ctypes.c_int32),
        ("row_stride", ctypes.c_int64),
        ("lane_offset", ctypes.c_int64),
        ("lanes", ctypes.c_int64),
    ]


class PeerFlags(ctypes.Structure):
    """cim22_peer_flags: each rank's barrier words (ranks + 1 int32) as mapped
    on this device, the world size and this rank."""
    _fields_ = [
        ("flags", ctypes.c_void_p * MAX_PEERS),
        ("ranks", ctypes.c_int32),
        ("rank", ctypes.c_int32),
    ]


ABI_STRUCTS = (
    FramePacket,
    StaticWeight,
    InputBinding,
    ReadbackBinding,
    Work,
    Group,
    Transaction,
    TraceEvent,
    Memref2D,
    Gather,
    ChainLayer,
    PeerOutputs,
    PeerFlags,
)


# ---------------------------------------------------------------------------
# Python-side transaction description, converted to the C structures on demand.


@dataclass
class TxnWeight:
    group_id: int
    work_id: int
    core_slot: int
    macro_slot: int
    values: np.ndarray  # int8 [16, 64]
    exponents: np.ndarray = field(default_factory=lambda: np.zeros(16, np.uint8))
    data_type: int = DATA_INT8
    route: Sequence[int] = (0,) * 6
    words: Sequence[int] = ()


@dataclass
class TxnPacket:
    kind: int
    group_id: int = -1
    work_id: int = -1
    macro_slot: int = -1
    cache_address: int = -1
    data_type: int = DATA_INT8
    route: Sequence[int] = (0,) * 6
    test_core: Sequence[int] = (0, 0, 0)


@dataclass
class TxnReadback:
    group_id: int
    work_id: int
    macro_slot: int
    output_cache_address: int
    data_type: int = DATA_INT8
    route: Sequence[int] = (0,) * 6
    test_core: Sequence[int] = (0, 0, 0)


@dataclass
class TxnInput:
    group_id: int
    work_id: int
    macro_slot: int
    input_slot: int
    data_type: int = DATA_INT8
    input_cache_address: int = 0


@dataclass
class TxnGroup:
    group_id: int
    works: list  # list of (work_id, core_slot, macro_slot)


@dataclass
class TransactionSpec:
    groups: list
    weights: list
    packets: list
    inputs: list
    readbacks: list
    target_profile: str = "cim22-4x5-v1"
    target_profile_version: int = 1
    execution_plan_version: int = 1

    def to_c(self) -> "CTransaction":
        return CTransaction(self)


class CTransaction:
    """Owns the ctypes arrays behind one ``Transaction`` structure."""

    def __init__(self, spec: TransactionSpec) -> None:
        self._keep = []
        groups = (Group * max(1, len(spec.groups)))()
        for gi, group in enumerate(spec.groups):
            works = (Work * max(1, len(group.works)))()
            for wi, (work_id, core, macro) in enumerate(group.works):
                works[wi].work_id = work_id
                works[wi].core_slot = core
                works[wi].macro_slot = macro
            self._keep.append(works)
            groups[gi].group_id = group.group_id
            groups[gi].works = ctypes.cast(works, ctypes.POINTER(Work))
            groups[gi].num_works = len(group.works)
        weights = (StaticWeight * max(1, len(spec.weights)))()
        for i, w in enumerate(spec.weights):
            c = weights[i]
            c.group_id, c.work_id = w.group_id, w.work_id
            c.core_slot, c.macro_slot = w.core_slot, w.macro_slot
            c.route[:] = list(w.route)
            values = np.ascontiguousarray(w.values, dtype=np.int8).reshape(-1)
            ctypes.memmove(c.values, values.ctypes.data, 1024)
            exps = np.ascontiguousarray(w.exponents, dtype=np.uint8).reshape(-1)
            ctypes.memmove(c.exponents, exps.ctypes.data, 16)
            c.data_type = w.data_type
            if len(w.words):
                words = (ctypes.c_int32 * len(w.words))(*w.words)
                self._keep.append(words)
                c.words = ctypes.cast(words, ctypes.POINTER(ctypes.c_int32))
                c.num_words = len(w.words)
        packets = (FramePacket * max(1, len(spec.packets)))()
        for i, p in enumerate(spec.packets):
            c = packets[i]
            c.kind = p.kind
            c.route[:] = list(p.route)
            c.group_id, c.work_id, c.macro_slot = p.group_id, p.work_id, p.macro_slot
            c.cache_address = p.cache_address
            c.test_core[:] = list(p.test_core)
            c.data_type = p.data_type
        inputs = (InputBinding * max(1, len(spec.inputs)))()
        for i, b in enumerate(spec.inputs):
            c = inputs[i]
            c.group_id, c.work_id, c.macro_slot = b.group_id, b.work_id, b.macro_slot
            c.input_slot, c.data_type = b.input_slot, b.data_type
            c.input_cache_address = b.input_cache_address
        readbacks = (ReadbackBinding * max(1, len(spec.readbacks)))()
        for i, b in enumerate(spec.readbacks):
            c = readbacks[i]
            c.group_id, c.work_id, c.macro_slot = b.group_id, b.work_id, b.macro_slot
            c.output_cache_address = b.output_cache_address
            c.route[:] = list(b.route)
            c.test_core[:] = list(b.test_core)
            c.data_type = b.data_type
        self._profile = spec.target_profile.encode()
        self._keep += [groups, weights, packets, inputs, readbacks]
        self.struct = Transaction(
            self._profile,
            spec.target_profile_version,
            spec.execution_plan_version,
            ctypes.cast(groups, ctypes.POINTER(Group)),
            len(spec.groups),
            ctypes.cast(weights, ctypes.POINTER(StaticWeight)),
            len(spec.weights),
            ctypes.cast(packets, ctypes.POINTER(FramePacket)),
            len(spec.packets),
            ctypes.cast(inputs, ctypes.POINTER(InputBinding)),
            len(spec.inputs),
            ctypes.cast(readbacks, ctypes.POINTER(ReadbackBinding)),
            len(spec.readbacks),
        )

    @property
    def pointer(self):
        return ctypes.byref(self.struct)
