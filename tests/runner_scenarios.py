"""Runner scenarios restated from the reference's unit test.

Every function restates one check of
test/Unit/Execution/CIMSoftwareRunnerTest.cpp (mlir-cim22) and takes a runner
factory, so the same known answers pin both the oracle runner (CPU) and the
CUDA runner (GPU). A runner exposes
``run(spec, mode, inputs, outputs, batch=, residency=, trace=) -> error|None``,
``stats`` and ``clear()``.
"""

from __future__ import annotations

import numpy as np

import txn_fixtures as fx
from cim22_b200.abi import (
    BF16_LEGACY,
    BF16_NONE,
    BF16_SIGN_SPLIT,
    DATA_BF16,
    DATA_INT8,
    TRACE_BEGIN_RUN,
    TRACE_COMPLETE,
    TRACE_CONFIGURE_INPUT,
    TRACE_CONFIGURE_WEIGHT,
    TRACE_ERROR,
    TRACE_READ_OUTPUT,
    TRACE_SELECT_MACRO,
    TRACE_START_WORK,
    TxnInput,
    TxnWeight,
)


def _bf16_io(n_out: int = 1):
    inp = np.zeros(64, np.uint16)
    outs = [np.zeros(16, np.uint16) for _ in range(n_out)]
    return inp, outs


def check_bf16_nonnegative_correction(make_runner, prealign_tile) -> None:
    """:748-873."""
    runner = make_runner()
    inp, (out,) = _bf16_io()
    weight = fx.bf16_weight(0, 127)

    def set_weight(mantissa, exponent):
        weight.values = np.full((16, 64), mantissa, np.int8)
        weight.exponents = np.full(16, exponent, np.uint8)

    def run():
        return runner.run(fx.make_bf16_executable(True, 0, weight), BF16_SIGN_SPLIT, [inp], [out])

    def check(expected):
        before = inp.copy()
        err = run()
        assert err is None, err
        assert np.all(out == expected), (out, hex(expected))
        assert np.array_equal(inp, before)

    set_weight(64, 126)
    inp[:] = 0x3F80
    check(0x4200)
    inp[:] = 0
    inp[0], inp[1] = 0x3F80, 0x3F00
    check(0x3F40)
    set_weight(2, 127)
    inp[1] = 0
    check(0x3D00)
    set_weight(0, 127)
    weight.values[0, 0] = 64
    weight.values[1, 1] = 64
    weight.values[3, 2] = 64
    inp[1] = 0x3B80
    assert run() is None
    assert out[0] == 0x3F80 and np.all(out[1:] == 0)
    set_weight(64, 127)
    inp[:] = 0
    check(0)
    inp[:] = 0x8000
    check(0)
    inp[:] = 0
    for bits in (1, 0x007F, 0x0080, 0x3F00, 0x7F00):
        inp[0] = bits
        check(bits)
    inp[0], inp[1] = 0x3F80, 1
    check(0x3F80)
    inp[:] = 0
    inp[0] = inp[63] = 0x3F80
    set_weight(0, 127)
    weight.values[15, 63] = 64
    assert run() is None
    assert np.all(out[:15] == 0) and out[15] == 0x3F80
    inp[:] = 0
    inp[0], inp[1] = 1, 0
    set_weight(1, 127)
    check(0)
    set_weight(64, 254)
    inp[0] = 0x4000
    assert run() == "CIM BF16 compensated tile exceeds BF16"
    set_weight(64, 127)
    inp[0], inp[1] = 0x3F80, 0xBF80
    assert run() == "CIM nonnegative BF16 mode rejects negative inputs"
    inp[1] = 0x8001
    assert run() == "CIM nonnegative BF16 mode rejects negative inputs"
    for bits in (0x7F80, 0x7FC1, 0xFF80):
        inp[1] = bits
        assert run() == "CIM BF16 input does not support NaN or infinity"
    inp[:] = 0
    weight.values[15, 63] = -1
    assert run() == "CIM nonnegative BF16 mode rejects negative prepared weights"
    set_weight(64, 255)
    assert run() == "CIM nonnegative BF16 weight exponent is not finite"
    set_weight(64, 127)
    inp[0] = 0x3F80
    check(0x3F80)


def check_bf16_legacy_compensation(make_runner, prealign_tile) -> None:
    """:680-746."""
    runner = make_runner()
    inp, (out,) = _bf16_io()
    lane = np.zeros(64, np.uint16)

    def run(mode):
        values, exps = prealign_tile(np.tile(lane, (16, 1)))
        weight = TxnWeight(0, 0, 0, 0, values, exps, DATA_BF16)
        return runner.run(fx.make_bf16_executable(True, 0, weight), mode, [inp], [out])

    def check(mode, expected):
        before = inp.copy()
        err = run(mode)
        assert err is None, err
        assert np.array_equal(inp, before)
        assert np.all(out == expected), (mode, out, hex(expected))

    inp[:] = 0x3F80
    lane[:] = 0x3F00
    check(BF16_LEGACY, 0x4200)
    lane[:] = 0x3F08
    check(BF16_NONE, 0x7F88)
    check(BF16_LEGACY, 0x4208)
    inp[:] = 0
    lane[:] = 0
    inp[0] = inp[1] = 0x3F80
    lane[0], lane[1] = 0x3F80, 0xBF00
    check(BF16_LEGACY, 0xBF00)
    lane[0] = lane[1] = 0x3F00
    inp[1] = 0xBF00
    check(BF16_LEGACY, 0xBE80)
    inp[1] = 0xBF80
    check(BF16_LEGACY, 0x3C80)
    inp[0] = 0x3F84
    check(BF16_LEGACY, 0x3C80)
    inp[:] = 0
    lane[:] = 0
    inp[0] = 0x7880
    lane[0] = 0x3F00
    check(BF16_LEGACY, 0x7800)
    inp[0] = 1
    lane[0] = 0x3F80
    check(BF16_LEGACY, 0)
    inp[0] = 0x7F80
    assert run(BF16_LEGACY) is not None
    inp[0] = 0x7FC1
    assert run(BF16_LEGACY) is not None
    inp[0] = inp[1] = 0x7F7F
    lane[0] = lane[1] = 0x3F80
    assert run(BF16_LEGACY) == "CIM BF16 compensated tile exceeds BF16"


def _int8_rows(n=4):
    rows = np.zeros((n, 64), np.int8)
    for i in range(n):
        for k in range(64):
            rows[i, k] = (i * 3 + k) % 15 - 7
    return rows


def _expected(spec, rows):
    out = []
    for b in spec.readbacks:
        w = next(x for x in spec.weights if x.group_id == b.group_id and x.work_id == b.work_id)
        out.append(w.values.astype(np.int32) @ rows[b.work_id].astype(np.int32))
    return out


def check_run(make_runner, trace_expected: bool = True) -> None:
    """checkRun + main (:249-279, :890-907): values and the 26-event trace."""
    runner = make_runner()
    spec = fx.make_executable()
    rows = _int8_rows()
    outs = [np.zeros(16, np.int32) for _ in range(4)]
    trace = []
    assert runner.run(spec, BF16_NONE, list(rows), outs, trace=trace) is None
    for o, e in zip(outs, _expected(spec, rows)):
        assert np.array_equal(o, e)
    assert len(trace) == 26
    assert [e[0] for e in trace] == list(range(26))
    kinds = [e[1] for e in trace]
    assert kinds[0] == TRACE_BEGIN_RUN and kinds[-1] == TRACE_COMPLETE
    assert kinds[1:5] == [TRACE_CONFIGURE_INPUT, TRACE_CONFIGURE_WEIGHT, TRACE_SELECT_MACRO,
                          TRACE_START_WORK]
    assert trace[9][2] == 0 and trace[9][3] == 0
    assert trace[10][6] == 0
    assert trace[13][2] == 1 and trace[13][3] == 2
    outs2 = [np.zeros(16, np.int32) for _ in range(4)]
    assert runner.run(spec, BF16_NONE, list(rows), outs2) is None
    for a, b in zip(outs, outs2):
        assert np.array_equal(a, b)
    # Wrong view counts (:909-914).
    bad = [np.zeros(16, np.int32) for _ in range(4)]
    assert runner.run(spec, BF16_NONE, [], bad) == \
        "CIM input count does not match executable bindings"


def check_faults(make_runner) -> None:
    """Fault fixtures (:916-936)."""
    messages = {
        "missing_input": "CIM input binding has no input Cache packet",
        "missing_weight": "CIM weight section has no weight packet",
        "missing_readback": "CIM readback is missing 1010/control/0101 sequence",
        "route_mismatch": "CIM readback is missing 1010/control/0101 sequence",
        "invalid_address": "CIM readback binding is outside the target profile",
        "overflow": "CIM software result exceeds signed i21 range",
    }
    for fault, message in messages.items():
        runner = make_runner()
        spec = fx.make_executable(fault)
        rows = np.zeros((4, 64), np.int8)
        if fault == "overflow":
            rows[:] = -128
        outs = [np.zeros(16, np.int32) for _ in range(4)]
        assert runner.run(spec, BF16_NONE, list(rows), outs) == message, fault


def check_independent_readback_batches(make_runner) -> None:
    """:281-298."""
    runner = make_runner()
    spec = fx.make_executable(distinct_cores=True)
    rows = _int8_rows()
    outs = [np.zeros(16, np.int32) for _ in range(4)]
    trace = []
    assert runner.run(spec, BF16_NONE, list(rows), outs, batch=True, trace=trace) is None
    for o, e in zip(outs, _expected(spec, rows)):
        assert np.array_equal(o, e)
    started = 0
    packets = []
    for e in trace:
        if e[1] == TRACE_START_WORK:
            started += 1
        if e[1] == TRACE_READ_OUTPUT:
            assert started == 4
            packets.append(e[5])
    assert packets == [4, 14, 9, 19]


def check_aliased_bf16_views(make_runner) -> None:
    """:300-353: group 0 publishes before group 1 reads the aliased row."""
    runner = make_runner()
    spec = fx.make_aliased_bf16()
    for overlap in (False, True):
        first = np.zeros(64, np.uint16)
        second = np.zeros(64, np.uint16)
        final = np.zeros(16, np.uint16)
        first[0] = 0x3F80
        second[0] = 0x4000
        first_out = final if overlap else second[:16]
        err = runner.run(spec, BF16_SIGN_SPLIT, [first, second], [first_out, final])
        assert err is None, err
        assert final[0] == (0x4000 if overlap else 0x3F80)


def check_int8_weight_residency(make_runner) -> None:
    """:379-421."""
    runner = make_runner()
    spec = fx.make_executable(distinct_cores=True)
    rows = np.zeros((4, 64), np.int8)
    outs = [np.zeros(16, np.int32) for _ in range(4)]
    for value in (3, -2):
        rows[:, 0] = value
        trace = []
        assert runner.run(spec, BF16_NONE, list(rows), outs, residency=True, trace=trace) is None
        writes = sum(1 for e in trace if e[1] == TRACE_CONFIGURE_WEIGHT)
        assert writes == (4 if value == 3 else 0)
        for i, o in enumerate(outs):
            assert np.all(o == value * (i // 2 + i % 2 + 1))
    assert runner.stats == (4, 4)
    assert runner.run(spec, BF16_NONE, [], outs, residency=True) is not None
    assert runner.run(spec, BF16_NONE, list(rows), outs, residency=True) is None
    assert runner.stats == (8, 4)


def check_bf16_weight_residency(make_runner) -> None:
    """:423-475."""
    runner = make_runner()
    weight = TxnWeight(0, 0, 0, 0, np.full((16, 64), 64, np.int8),
                       np.full(16, 126, np.uint8), DATA_BF16)
    first = fx.make_bf16_executable(True, 0, weight, 7)
    second = fx.make_bf16_executable(True, 0, weight, 0, 7)
    inp = np.zeros(64, np.uint16)
    out = [np.zeros(16, np.uint16) for _ in range(2)]
    inp[:] = 0x3F80
    assert runner.run(first, BF16_SIGN_SPLIT, [inp], out[:1], residency=True) is None
    assert np.all(out[0] == 0x4200)
    inp[:] = 0
    inp[0], inp[1] = 0x3F80, 0x3F00
    assert runner.run(second, BF16_SIGN_SPLIT, [inp], out, residency=True) is None
    assert runner.stats == (1, 1)
    assert np.all(out[0] == 0x3F40)
    assert np.all(out[1] == 0)
    inp[:] = 0x3F80
    assert runner.run(first, BF16_LEGACY, [inp], out[:1], residency=True) is None
    assert runner.stats == (2, 1)
    assert np.all(out[0] == 0x4200)
    inp[0] = 0x7F80
    assert runner.run(first, BF16_LEGACY, [inp], out[:1], residency=True) is not None
    assert runner.stats == (2, 1)


def check_all_macro_caches(make_runner) -> None:
    """:479-567."""
    runner = make_runner()
    spec = fx.make_all_macro_caches()
    rows = np.zeros((80, 64), np.int8)
    outs = [np.zeros(16, np.int32) for _ in range(82)]
    for value in (2, -3):
        rows[:, 0] = value
        for o in outs:
            o[:] = 123456
        trace = []
        assert runner.run(spec, BF16_NONE, list(rows), outs, batch=True, trace=trace) is None
        packets, started = [], 0
        for e in trace:
            if e[1] == TRACE_START_WORK:
                started += 1
            if e[1] != TRACE_READ_OUTPUT:
                continue
            assert started == (40 if e[2] == 0 else 80)
            packets.append(e[5])
        expected = []
        for group in (0, 1):
            for macro in (0, 1):
                expected += [4 + 5 * (40 * group + s) for s in range(macro, 40, 2)]
                if group == 1 and macro == 0:
                    expected += [402, 405]
        assert packets == expected
        for i, o in enumerate(outs):
            factor = i + 1 if i < 80 else (1 if i == 80 else 0)
            assert np.all(o == factor * value), (i, o)


def check_int8_numeric_model(make_runner, full: bool = True) -> None:
    """:571-678: signed byte products, extremes, cancellation, overflow."""
    runner = make_runner()
    inp = np.zeros(64, np.int8)
    out = np.zeros(16, np.int32)
    values = np.zeros((16, 64), np.int8)

    def check(spec, expected):
        before = inp.copy()
        out[:] = 77
        err = runner.run(spec, BF16_NONE, [inp], [out])
        assert err is None, err
        assert np.array_equal(out.astype(np.int64), np.asarray(expected, np.int64))
        assert np.array_equal(inp, before)

    positions = (0, 31, 32, 63) if full else (0, 63)
    bases = range(-128, 128, 16) if full else (-128, 112)
    for k in positions:
        inp[:] = 0
        for base in bases:
            values[:] = 0
            values[np.arange(16), k] = (base + np.arange(16)).astype(np.int8)
            spec = fx.make_int8_single(values)
            for a in (range(-128, 128) if full else (-128, -1, 0, 1, 127)):
                inp[k] = a
                check(spec, a * (base + np.arange(16)))
    for k in range(64):
        inp[:] = 0
        inp[k] = -128
        values[:] = 0
        values[np.arange(16), k] = np.arange(16) - 8
        check(fx.make_int8_single(values), -128 * (np.arange(16) - 8))
    inp[:] = -128
    values[:] = -128
    values[:, 63] = -127
    check(fx.make_int8_single(values), np.full(16, 1048448))
    values[:] = 127
    negative = fx.make_int8_single(values)
    check(negative, np.full(16, -1040384))
    inp[:] = 0
    check(negative, np.zeros(16))
    inp[:] = -128
    check(negative, np.full(16, -1040384))
    inp[:] = 127
    values[:] = np.where(np.arange(64) % 2, -127, 127).astype(np.int8)
    check(fx.make_int8_single(values), np.zeros(16))
    inp[:] = -128
    values[:] = 127
    values[15, :] = -128
    out[:] = 77
    trace = []
    err = runner.run(fx.make_int8_single(values), BF16_NONE, [inp], [out], trace=trace)
    assert err == "CIM software result exceeds signed i21 range"
    assert np.all(out == 77)
    assert trace[-1][1] == TRACE_ERROR
    assert all(e[1] != TRACE_COMPLETE for e in trace)
    check(negative, np.full(16, -1040384))


def check_bf16_none_mode(make_runner) -> None:
    """Tail of main (:938-995): None-mode raw converter bits and rejections."""
    runner = make_runner()
    inp = np.full(64, 0x3F80, np.uint16)
    out = np.zeros(16, np.uint16)

    def run(spec, mode=BF16_NONE):
        return runner.run(spec, mode, [inp], [out])

    assert run(fx.make_bf16_executable()) is None
    assert np.all(out == 0x7F80)
    assert run(fx.make_bf16_executable(True, 64)) is None
    assert np.all(out == 0x7F80)
    assert run(fx.make_bf16_executable(True, -64)) is None
    assert np.all(out == 0xFF80)
    inp[:] = 0x8000
    assert run(fx.make_bf16_executable(True, -128)) == \
        "CIM software result exceeds signed i21 range"
    assert run(fx.make_bf16_executable(True, -127)) is None
    assert np.all(out == 0x467E)
    inp[:] = 0xBFFF
    assert run(fx.make_bf16_executable(True, -127)) is None
    assert np.all(out == 0x7FFE)
    inp[:] = 0x3F80
    inp[0] = 0x7F80
    assert run(fx.make_bf16_executable()) == "CIM BF16 input does not support NaN or infinity"
    inp[0] = 0x7FC1
    assert run(fx.make_bf16_executable()) == "CIM BF16 input does not support NaN or infinity"
    inp[0] = 0x3F80
    assert run(fx.make_bf16_executable(False)) == \
        "CIM BF16 weight section has no Weight_EXP packet"
    mixed = fx.make_bf16_executable()
    mixed.inputs = [TxnInput(0, 0, 0, 0, DATA_INT8)]
    assert run(mixed) is not None


ALL = (
    check_bf16_nonnegative_correction,
    check_bf16_legacy_compensation,
    check_run,
    check_faults,
    check_independent_readback_batches,
    check_aliased_bf16_views,
    check_int8_weight_residency,
    check_bf16_weight_residency,
    check_all_macro_caches,
    check_int8_numeric_model,
    check_bf16_none_mode,
)
