"""Generate the committed golden vectors under tests/golden/.

Run in a container that has the mlir-cim22 source tree, naming it by the
CIM22_REFERENCE environment variable or the first argument:

    CIM22_REFERENCE=<mlir-cim22 checkout> python tests/golden/make_golden.py
    python tests/golden/make_golden.py <mlir-cim22 checkout>

Outputs:
  supplier_int8.json   The four supplier INT8 tile fixtures
                       (test/Inputs/CIM22/*/{cim_w,cache_in_int8,output_int8}.txt),
                       decoded with the reference's own NumPy model
                       (test/python/CIM22/int8_reference.py:89-150) and checked
                       with its replay (supplier_fixture_replay.py:142-180):
                       8x64 int8 inputs, a 16x64 int8 weight tile and the
                       8x16 signed-INT21 outputs.
  bf16_support_ref.npz Outputs of the reference's lib/Support/BF16Support.cpp,
                       compiled unmodified into oracle/_ref by oracle/Makefile:
                       prealignBF16Vector on seeded random and edge-case rows,
                       and int21ToBF16 on seeded (value, Ew, Ei) triples.
  int8_conv_ref.npz    INT8 Conv / MatMulInteger + bias cases of the
                       reference's ONNX corpus (test/python/ONNX/
                       generate_conv_integer_onnx.py, generate_integer_bias_onnx.py:
                       the same shapes, seeds and weight draws) and of
                       python/tests/test_compile_tool.py:153-258, with outputs
                       computed by the reference's own lowering helpers
                       (test/python/ONNX/int8_lowering.py: conv_to_matrix,
                       fold_bias, wrap_i32), the folded and unfolded forms
                       checked equal as verify_integer_bias.py does.
"""

from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REFERENCE = Path(sys.argv[1] if len(sys.argv) > 1 and not sys.argv[1].startswith("-")
                 else os.environ.get("CIM22_REFERENCE", ""))


def supplier_int8() -> dict:
    sys.path.insert(0, str(REFERENCE / "test/python/CIM22"))
    import int8_reference as reference  # noqa: E402
    import supplier_fixture_replay as replay  # noqa: E402

    manifest_path = REFERENCE / "test/Inputs/CIM22/fixtures.json"
    # The reference's own replay must pass before its data is exported.
    summary = replay.replay(manifest_path)
    manifest = json.loads(manifest_path.read_text(encoding="ascii"))
    root = manifest_path.parent
    cases = []
    for case in replay.validate_manifest(manifest):
        files = case["files"]
        words = replay._parse_weight(replay._checked_path(root, files["weight"]))
        weight = reference.decode_int8_weight_words(words)
        inputs = reference.decode_int8_cache_lines(
            replay._parse_addressed_bits(
                replay._checked_path(root, files["input"]),
                reference.CACHE_ROWS,
                reference.CACHE_LINE_BITS,
            )
        )
        expected = replay._parse_expected(replay._checked_path(root, files["output"]))
        cases.append(
            {
                "case_id": case["case_id"],
                "weight": weight.astype(int).tolist(),
                "inputs": inputs.astype(int).tolist(),
                "expected": expected.astype(int).tolist(),
            }
        )
    return {"source": "test/Inputs/CIM22/fixtures.json", "replay": summary, "cases": cases}


def edge_rows(rng: np.random.Generator) -> np.ndarray:
    rows = []
    # Random BF16 bit patterns without NaN/Inf, signed and unsigned.
    for _ in range(600):
        bits = rng.integers(0, 1 << 16, 64, dtype=np.uint32).astype(np.uint16)
        exp = (bits >> 7) & 0xFF
        bits[exp == 0xFF] &= 0x807F
        rows.append(bits)
    # Narrow exponent spread around a random centre (realistic activations).
    for _ in range(600):
        centre = int(rng.integers(1, 250))
        exp = np.clip(centre - rng.integers(0, 12, 64), 0, 254).astype(np.uint16)
        mant = rng.integers(0, 128, 64).astype(np.uint16)
        sign = (rng.random(64) < 0.5).astype(np.uint16) << 15
        rows.append(sign | (exp << 7) | mant)
    # Sparse rows, zeros, negative zeros and subnormal-only rows.
    for _ in range(300):
        row = np.zeros(64, np.uint16)
        idx = rng.integers(0, 64, int(rng.integers(0, 6)))
        row[idx] = rng.integers(0, 1 << 16, idx.size).astype(np.uint16) & 0xBFFF
        if rng.random() < 0.3:
            row[rng.integers(0, 64, 3)] = 0x8000
        if rng.random() < 0.3:
            row[:] = rng.integers(0, 128, 64).astype(np.uint16) | (
                (rng.random(64) < 0.5).astype(np.uint16) << 15)
        rows.append(row)
    return np.stack(rows)


def bf16_support_ref() -> dict:
    subprocess.run(["make", "-s", "-C", str(REPO / "oracle"), "ref"], check=True,
                   env={**os.environ, "REFERENCE": str(REFERENCE)})
    ref = ctypes.CDLL(str(REPO / "oracle/_ref/libref_bf16support.so"))
    ref.ref_int21_to_bf16.restype = ctypes.c_uint16
    ref.ref_int21_to_bf16.argtypes = [ctypes.c_int32, ctypes.c_uint8, ctypes.c_uint8]
    ref.ref_prealign.argtypes = [ctypes.c_void_p] * 3
    rng = np.random.default_rng(20261201)
    rows = np.ascontiguousarray(edge_rows(rng))
    exps = np.zeros(len(rows), np.uint8)
    mants = np.zeros((len(rows), 64), np.int8)
    for i, row in enumerate(rows):
        e = ctypes.c_uint8()
        out = np.zeros(64, np.int8)
        ref.ref_prealign(row.ctypes.data, ctypes.byref(e), out.ctypes.data)
        exps[i] = e.value
        mants[i] = out
    values = np.concatenate([
        rng.integers(-(1 << 20), 1 << 20, 8000),
        np.arange(-300, 301),
        np.array([0, 1, -1, 127, 128, 255, 256, (1 << 20) - 1, -(1 << 20)]),
    ]).astype(np.int32)
    we = rng.integers(0, 256, values.size).astype(np.uint8)
    ie = rng.integers(0, 256, values.size).astype(np.uint8)
    bits = np.array([ref.ref_int21_to_bf16(int(v), int(a), int(b))
                     for v, a, b in zip(values, we, ie)], np.uint16)
    return {"rows": rows, "prealign_exponent": exps, "prealign_mantissas": mants,
            "int21_values": values, "int21_we": we, "int21_ie": ie, "int21_bits": bits}


def int8_conv_ref() -> dict:
    sys.path.insert(0, str(REFERENCE / "test/python/ONNX"))
    import int8_lowering as lowering  # noqa: E402

    out = {}

    def conv_case(name, x, weight, bias, strides, pads, foldable=False):
        f, c, kh, kw = weight.shape
        patches = lowering.conv_to_matrix(x, (kh, kw), strides, pads)
        core = weight.reshape(f, -1).astype(np.int64) @ patches.astype(np.int64)
        total = core + (0 if bias is None else bias.astype(np.int64).reshape(-1, 1))
        y = lowering.wrap_i32(total)
        if foldable:
            exact_k = (c * kh * kw) % 64 == 0
            fw, fx = lowering.fold_bias(weight.reshape(f, -1), patches, bias, exact_k)
            folded = lowering.wrap_i32(fw.astype(np.int64) @ fx.astype(np.int64))
            assert np.array_equal(folded, y)
        oh = (x.shape[2] + pads[0] + pads[2] - kh) // strides[0] + 1
        ow = (x.shape[3] + pads[1] + pads[3] - kw) // strides[1] + 1
        out[f"{name}.x"] = x
        out[f"{name}.w"] = weight
        if bias is not None:
            out[f"{name}.bias"] = bias.astype(np.int32)
        out[f"{name}.geom"] = np.array([*strides, *pads], np.int64)
        out[f"{name}.y"] = y.reshape(1, f, oh, ow)

    def corpus_input(shape):
        return (np.arange(np.prod(shape), dtype=np.int32) % 17 - 8).astype(np.int8).reshape(shape)

    # generate_conv_integer_onnx.py: (C, H, W, F, seed, kernel, strides, pads).
    for name, (c, h, w, f, seed, kernel, strides, pads) in {
        "canonical": (8, 8, 8, 19, 2201, (3, 3), (1, 1), (1, 1, 1, 1)),
        "odd": (1, 3, 3, 1, 2202, (3, 3), (1, 1), (1, 1, 1, 1)),
        "pointwise": (3, 5, 7, 5, 2203, (1, 1), (2, 2), (0, 0, 0, 0)),
        "rectangular": (2, 5, 6, 17, 2204, (2, 3), (2, 2), (1, 0, 0, 1)),
    }.items():
        weight = np.random.default_rng(seed).integers(-7, 8, size=(f, c, *kernel), dtype=np.int8)
        conv_case(name, corpus_input((1, c, h, w)), weight, None, strides, pads)

    # generate_integer_bias_onnx.py conv cases (bias broadcast [1, 17, 1, 1]).
    for name, foldable, exact_k in (("conv_bias", False, False), ("conv_bias_fold", True, False),
                                    ("conv_bias_exact", True, True)):
        rng = np.random.default_rng(2602 if foldable else 2502)
        if exact_k:
            wshape, xshape, pads, strides = (17, 1, 8, 8), (1, 1, 8, 8), (0, 0, 0, 0), (1, 1)
        else:
            wshape, xshape, pads, strides = (17, 2, 2, 3), (1, 2, 5, 6), (1, 0, 0, 1), (2, 2)
        weight = rng.integers(-7, 8, size=wshape, dtype=np.int8)
        if foldable:
            bias = ((np.arange(17, dtype=np.int32) * 31 + 5) % 256 - 128).astype(np.int32)
            bias[:2] = [-128, 127]
        else:
            bias = (np.arange(17, dtype=np.int64) * 104729 - 700000).astype(np.int32)
            bias[::3] *= -1
        conv_case(name, corpus_input(xshape), weight, bias, strides, pads, foldable)

    # generate_integer_bias_onnx.py linear cases: MatMulInteger [B, K] x [K, 17] + bias.
    for name, foldable, exact_k in (("linear_bias", False, False),
                                    ("linear_bias_fold", True, False),
                                    ("linear_bias_exact", True, True)):
        reduction = 64 if exact_k else 65
        batch = 1 if exact_k else 2
        rng = np.random.default_rng(2601 if foldable else 2501)
        weight = rng.integers(-7, 8, size=(reduction, 17), dtype=np.int8)
        weight[:, 0] = 1
        if foldable:
            bias = ((np.arange(17, dtype=np.int32) * 29 + 3) % 256 - 128).astype(np.int32)
            bias[:2] = [-128, 127]
            x = (np.arange(batch * reduction, dtype=np.int32) % 23 - 11).astype(np.int8)
            x = x.reshape(batch, reduction)
        else:
            bias = (np.arange(17, dtype=np.int64) * 7919 - 50000).astype(np.int32)
            bias[0] = np.iinfo(np.int32).max
            x = np.stack([np.ones(reduction, np.int8), -np.ones(reduction, np.int8)])
        y = lowering.wrap_i32(x.astype(np.int64) @ weight.astype(np.int64) + bias)
        if foldable:
            fw, fx = lowering.fold_bias(weight.T, x.T, bias, exact_k)
            assert np.array_equal(lowering.wrap_i32(fw.astype(np.int64) @ fx.astype(np.int64)).T,
                                  y)
        else:
            assert y[0, 0] == -(2**31) + 64
        out[f"{name}.x"] = x
        out[f"{name}.w"] = weight
        out[f"{name}.bias"] = bias
        out[f"{name}.y"] = y

    # python/tests/test_compile_tool.py:153-258: 1x2x8x8 input, 17x2x6x6 weights.
    weight = (np.arange(17 * 2 * 6 * 6).reshape(17, 2, 6, 6) % 15 - 7).astype(np.int8)
    value = (np.arange(128).reshape(1, 2, 8, 8) * 13 % 256 - 128).astype(np.int8)
    for i, x in enumerate((value, np.flip(value, axis=3).copy())):
        conv_case(f"compile_tool{i}", x, weight, None, (1, 1), (0, 0, 0, 0))
    return out


def main() -> None:
    if not (REFERENCE / "lib").is_dir():
        raise SystemExit("name the mlir-cim22 source tree: CIM22_REFERENCE=<dir> or "
                         "make_golden.py <dir>")
    data = supplier_int8()
    (HERE / "supplier_int8.json").write_text(json.dumps(data) + "\n", encoding="ascii")
    np.savez_compressed(HERE / "bf16_support_ref.npz", **bf16_support_ref())
    np.savez_compressed(HERE / "int8_conv_ref.npz", **int8_conv_ref())
    print("wrote", HERE / "supplier_int8.json", HERE / "bf16_support_ref.npz",
          HERE / "int8_conv_ref.npz")


if __name__ == "__main__":
    main()
