"""The reference's own software runner, compiled unmodified into oracle/_ref
(lib/Execution/CIMSoftwareRunner.cpp, BF16Compensation.cpp, BF16Support.cpp
against the clean-room LLVM support subset in oracle/llvm_shim), checked
against the restated oracle: its own unit test passed at build time, random
transactions in all three compensation modes give the same outputs and
error texts, and a runner-driven BF16 layer gives the oracle layer's bits.
These pin the oracle to the reference's code rather than only to its known
answers; the benchmark's CPU baseline runs this runner."""

import numpy as np
import pytest

import oracle
import txn_fixtures as fx
from cim22_b200.abi import BF16_LEGACY, BF16_NONE, BF16_SIGN_SPLIT, DATA_BF16, TxnWeight

pytestmark = pytest.mark.skipif(not oracle.reference_runner_available(),
                                reason="oracle/_ref was not built (no mlir-cim22 source tree)")


def test_reference_unit_test_passed():
    log = (oracle.HERE / "_ref" / "runner_test.log").read_text()
    assert (oracle.HERE / "_ref" / "runner_test.passed").exists()
    assert "PASS nonnegative BF16 correction" in log
    assert "PASS INT8 software model" in log


def _row(rng, kind):
    if kind == "signed":
        e = rng.integers(100, 140, 64)
        row = (rng.integers(0, 2, 64) << 15) | (e << 7) | rng.integers(0, 128, 64)
    elif kind == "positive":
        e = rng.integers(100, 140, 64)
        row = (e << 7) | rng.integers(0, 128, 64)
        row[rng.random(64) < 0.3] = 0
    elif kind == "tiny":
        row = rng.integers(0, 128, 64)
    else:  # any finite pattern
        row = rng.integers(0, 1 << 16, 64)
        bad = ((row >> 7) & 0xFF) == 0xFF
        row[bad] &= 0x807F
    return np.asarray(row, np.uint16)


@pytest.mark.parametrize("mode", [BF16_NONE, BF16_LEGACY, BF16_SIGN_SPLIT])
def test_random_bf16_transactions_match_oracle(mode):
    rng = np.random.default_rng(300 + mode)
    ref = oracle.RefRunner(mode)
    port = oracle.Runner()
    kinds = ("signed", "positive", "tiny", "wild")
    for trial in range(200):
        kind = kinds[trial % 4] if mode != BF16_SIGN_SPLIT else ("positive", "tiny")[trial % 2]
        weight_bits = np.stack([_row(rng, "positive" if mode == BF16_SIGN_SPLIT else kind)
                                for _ in range(16)])
        values, exps = oracle.prealign_tile(weight_bits)
        spec = fx.make_bf16_executable(True, 0, TxnWeight(0, 0, 0, 0, values, exps, DATA_BF16))
        row = _row(rng, kind)
        out_ref, out_port = np.zeros(16, np.uint16), np.zeros(16, np.uint16)
        e_ref = ref.run(spec, [row], [out_ref])
        e_port = port.run(spec, mode, [row], [out_port])
        assert e_ref == e_port, (trial, e_ref, e_port)
        np.testing.assert_array_equal(out_ref, out_port, err_msg=f"trial {trial}")


def test_random_int8_multiwave_transactions_match_oracle():
    rng = np.random.default_rng(11)
    ref = oracle.RefRunner(BF16_NONE)
    port = oracle.Runner()
    for trial in range(20):
        spec = fx.make_all_macro_caches()
        for w in spec.weights:
            w.values[:] = rng.integers(-127, 128, w.values.shape)
        rows = [rng.integers(-128, 128, 64).astype(np.int8) for _ in spec.inputs]
        o_ref = [np.zeros(16, np.int32) for _ in spec.readbacks]
        o_port = [np.zeros(16, np.int32) for _ in spec.readbacks]
        for batch in (False, True):
            e_ref = ref.run(spec, rows, o_ref, batch=batch, residency=True)
            e_port = port.run(spec, 0, rows, o_port, batch=batch, residency=True)
            assert e_ref == e_port
            for a, b in zip(o_ref, o_port):
                np.testing.assert_array_equal(a, b)
    # The i21 overflow gate gives the same error text.
    spec = fx.make_executable("overflow")
    rows = [np.full(64, -128, np.int8) for _ in spec.inputs]
    o = [np.zeros(16, np.int32) for _ in spec.readbacks]
    assert ref.run(spec, rows, o) == port.run(spec, 0, rows, o) is not None


@pytest.mark.parametrize("m,k,n,branches,scale", [
    (9, 150, 37, 4, 1.0), (7, 64, 16, 2, 1.0), (5, 200, 20, 4, 1e-36), (6, 130, 33, 4, 1e30)])
def test_reference_runner_layer_matches_oracle(m, k, n, branches, scale):
    rng = np.random.default_rng(m + k + n)
    x = (rng.standard_normal((m, k)) * scale).astype(np.float32)
    if branches == 2:
        x = np.maximum(x, 0)
    x[rng.random(x.shape) < 0.15] = 0
    x[0, :64] = 0  # an all-zero group
    w = (rng.standard_normal((n, k)) * 0.1).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    try:
        expected = oracle.linear_bf16(x, w, b, branches=branches)
    except oracle.OracleError as e:
        with pytest.raises(oracle.OracleError, match=str(e)):
            oracle.linear_bf16(x, w, b, branches=branches, via_runner="reference")
        return
    got = oracle.linear_bf16(x, w, b, branches=branches, threads=2, via_runner="reference")
    np.testing.assert_array_equal(got.view(np.uint32), expected.view(np.uint32))


def test_reference_runner_forward_matches_oracle_forward():
    from cim22_b200 import workloads

    model, x = workloads.build("lenet", 3)
    a = oracle.cim_forward(model, x.numpy(), branches="reference", threads=2,
                           via_runner="reference")
    b = oracle.cim_forward(model, x.numpy(), branches=4)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
