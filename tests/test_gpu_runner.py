"""CUDA transaction runner: reference known answers and bit parity with the oracle."""

import json
from pathlib import Path

import numpy as np
import pytest

import oracle
import runner_scenarios as rs
import txn_fixtures as fx
from cim22_b200.abi import (
    BF16_LEGACY,
    BF16_NONE,
    BF16_SIGN_SPLIT,
    DATA_BF16,
    TxnWeight,
)

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def cuda_runner_factory():
    from cim22_b200.native import CudaRunner

    return lambda: CudaRunner(0)


@pytest.mark.parametrize("scenario", rs.ALL, ids=lambda f: f.__name__)
def test_reference_scenarios_on_gpu(scenario, cuda_runner_factory):
    if scenario in (rs.check_bf16_nonnegative_correction, rs.check_bf16_legacy_compensation):
        scenario(cuda_runner_factory, oracle.prealign_tile)
    elif scenario is rs.check_int8_numeric_model:
        scenario(cuda_runner_factory, full=False)
    else:
        scenario(cuda_runner_factory)


def test_supplier_int8_fixtures_on_gpu(cuda_runner_factory):
    data = json.loads((GOLDEN / "supplier_int8.json").read_text())
    runner = cuda_runner_factory()
    for case in data["cases"]:
        weight = np.array(case["weight"], np.int8)
        inputs = np.array(case["inputs"], np.int8)
        outs = [np.zeros(16, np.int32) for _ in range(8)]
        assert runner.run(fx.make_supplier_case(weight), BF16_NONE, list(inputs), outs) is None
        np.testing.assert_array_equal(np.stack(outs), np.array(case["expected"]))


def _random_bf16_row(rng, kind):
    if kind == "signed":
        exp = np.clip(127 - rng.integers(0, 10, 64), 1, 254)
        row = ((rng.random(64) < 0.5).astype(np.uint16) << 15) | (exp.astype(np.uint16) << 7) \
            | rng.integers(0, 128, 64).astype(np.uint16)
    elif kind == "positive":
        exp = np.clip(rng.integers(1, 255) - rng.integers(0, 14, 64), 0, 254)
        row = (exp.astype(np.uint16) << 7) | rng.integers(0, 128, 64).astype(np.uint16)
        row[rng.random(64) < 0.3] = 0
    elif kind == "tiny":
        row = rng.integers(0, 128, 64).astype(np.uint16)
    else:  # wild: any finite pattern
        row = rng.integers(0, 1 << 16, 64).astype(np.uint16)
        bad = ((row >> 7) & 0xFF) == 0xFF
        row[bad] &= 0x807F
    return row.astype(np.uint16)


@pytest.mark.parametrize("mode", [BF16_NONE, BF16_LEGACY, BF16_SIGN_SPLIT])
def test_random_bf16_transactions_match_oracle(mode, cuda_runner_factory):
    rng = np.random.default_rng(100 + mode)
    runner = cuda_runner_factory()
    ref = oracle.Runner()
    kinds = ("signed", "positive", "tiny", "wild")
    for trial in range(60):
        kind = kinds[trial % 4] if mode != BF16_SIGN_SPLIT else ("positive", "tiny")[trial % 2]
        weight_bits = np.zeros((16, 64), np.uint16)
        for lane in range(16):
            weight_bits[lane] = _random_bf16_row(rng, "positive" if mode == BF16_SIGN_SPLIT
                                                 else kind)
        values, exps = oracle.prealign_tile(weight_bits)
        spec = fx.make_bf16_executable(True, 0, TxnWeight(0, 0, 0, 0, values, exps, DATA_BF16))
        row = _random_bf16_row(rng, kind)
        out_gpu, out_cpu = np.zeros(16, np.uint16), np.zeros(16, np.uint16)
        tg, tc = [], []
        eg = runner.run(spec, mode, [row], [out_gpu], trace=tg)
        ec = ref.run(spec, mode, [row], [out_cpu], trace=tc)
        assert eg == ec, (trial, eg, ec)
        np.testing.assert_array_equal(out_gpu, out_cpu, err_msg=f"trial {trial}")
        assert tg == tc


def test_random_int8_multiwave_transactions_match_oracle(cuda_runner_factory):
    rng = np.random.default_rng(7)
    runner = cuda_runner_factory()
    ref = oracle.Runner()
    for trial in range(20):
        spec = fx.make_all_macro_caches()
        for w in spec.weights:
            w.values = rng.integers(-128, 128, (16, 64)).astype(np.int8) // (1 + trial % 3)
        rows = rng.integers(-128, 128, (80, 64)).astype(np.int8)
        og = [np.zeros(16, np.int32) for _ in range(82)]
        oc = [np.zeros(16, np.int32) for _ in range(82)]
        tg, tc = [], []
        batch = bool(trial % 2)
        eg = runner.run(spec, BF16_NONE, list(rows), og, batch=batch, residency=True, trace=tg)
        ec = ref.run(spec, BF16_NONE, list(rows), oc, batch=batch, residency=True, trace=tc)
        assert eg == ec
        for a, b in zip(og, oc):
            np.testing.assert_array_equal(a, b)
        assert tg == tc
        assert runner.stats == ref.stats


def test_session_dispatch_abi(cuda_runner_factory):
    from cim22_b200.native import CudaSession, dispatch

    session = CudaSession(0)
    weight = fx.bf16_weight(64, 126)
    tid = session.add(fx.make_bf16_executable(True, 0, weight), "__cim_kernel_7")
    assert tid == 0 and session.num_transactions == 1
    inputs = np.full((1, 64), 0x3F80, np.uint16)
    outputs = np.full((1, 16), 0xFFFF, np.uint16)
    session.begin()
    dispatch("sign-split", tid, inputs, outputs)
    assert session.end() == 0
    assert session.dispatch_count == 1
    assert np.all(outputs == 0x4200)
    # Descriptor and type errors follow runtime/Runtime.cpp:131-153.
    session.begin()
    dispatch("int8", tid, np.zeros((1, 64), np.int8), np.zeros((1, 16), np.int32))
    assert session.end() == 1
    assert session.error == "native CIM dispatch transaction type or count mismatch"
    session.begin()
    dispatch("sign-split", tid, np.zeros((2, 64), np.uint16), outputs)
    assert session.end() == 1
    assert session.error == "native CIM dispatch transaction type or count mismatch"
    session.begin()
    dispatch("sign-split", 5, inputs, outputs)
    assert session.end() == 1
    assert session.error == "invalid native CIM dispatch descriptor"
    # Runner errors carry the kernel name; outputs were zero-filled first.
    inputs[0, 0] = 0x7F80
    outputs[:] = 0xFFFF
    session.begin()
    dispatch("sign-split", tid, inputs, outputs)
    assert session.end() == 1
    assert session.error == "__cim_kernel_7: CIM BF16 input does not support NaN or infinity"
    assert np.all(outputs == 0)
    session.close()
