"""The CPU oracle (oracle/intconv_oracle.c) pinned to the reference.

1. Golden fixtures (tests/golden/intconv_golden.json), generated from the
   reference's own run_cpu and det_math compiled from its sources: every
   scalar function, the weight quantiser and 29 whole programs must match.
2. The reference conformance suite's known-answer checks, restated
   (reference tests/deterministic_executor_tests.cpp:75-214, 221-313).
3. When the reference build is present (this container), the oracle against
   the live reference on further programs.
"""
from __future__ import annotations

import hashlib
import json
import math
from pathlib import Path

import numpy as np
import pytest

from nvcr_b200.program import OpKind, Program, SeededStream
from oracle.oracle import canonical_digest, count_differing, same_bits
from tests.golden.cases import program_cases, scalar_inputs, weight_cases
from tests.programs import (CONV_CASES, conv_program, data_movement_program, op_program, staged_chain_program,
                            staged_depthwise_program)

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "intconv_golden.json").read_text())


def digest_bytes(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


# ---------------------------------------------------------------- golden fixtures

def test_golden_scalar_inputs_regenerate():
    s = scalar_inputs()
    for key, value in s.items():
        assert digest_bytes(value) == GOLDEN["scalars"]["inputs_sha256"][key], key


def test_golden_scalars(oracle):
    s = scalar_inputs()
    lib = oracle.lib
    g = GOLDEN["scalars"]
    assert canonical_digest(np.array([lib.or_exp(float(v)) for v in s["floats"]], np.float32)) == g["det_exp"]
    assert canonical_digest(np.array([lib.or_sigmoid(float(v)) for v in s["floats"]], np.float32)) == g["det_sigmoid"]
    assert digest_bytes(np.array([lib.or_float_to_half(float(v)) for v in s["floats"]], np.uint16)) == \
        g["det_float_to_half_bits"]
    assert canonical_digest(np.array([lib.or_half_to_float(int(h)) for h in s["halves"]], np.float32)) == \
        g["det_half_bits_to_float"]
    assert canonical_digest(np.array([lib.or_ldexp(float(v), int(e))
                                      for v, e in zip(s["ldexp_values"], s["ldexp_exponents"])], np.float32)) == \
        g["det_ldexp"]
    for bits in (8, 16):
        assert digest_bytes(np.array([lib.or_int_exponent(float(m), bits) for m in s["maxima"]], np.int32)) == \
            g[f"det_int_exponent_{bits}"]
        assert digest_bytes(np.array([lib.or_int_quantize(float(v), int(e), bits)
                                      for v, e in zip(s["q_values"], s["q_exponents"])], np.int32)) == \
            g[f"det_int_quantize_{bits}"]
    assert canonical_digest(np.array([lib.or_int_output(int(a), float(sc), int(e), float(b))
                                      for a, sc, e, b in zip(s["acc"], s["acc_scale"], s["acc_exponent"],
                                                             s["acc_bias"])], np.float32)) == g["det_int_output"]


def test_golden_quantize_weights(oracle):
    for name, matrix, bits in weight_cases():
        values, scales = oracle.quantize_weights(matrix, bits)
        assert digest_bytes(values) == GOLDEN["quantize_weights"][name]["values"], name
        assert canonical_digest(scales) == GOLDEN["quantize_weights"][name]["scales"], name


CASES = {case.name: case for case in program_cases()}


@pytest.mark.parametrize("entry", GOLDEN["programs"], ids=lambda e: e["name"])
def test_golden_programs(oracle, entry):
    case = CASES[entry["name"]]
    for x, expected in zip(case.inputs, entry["inputs_sha256"]):
        assert digest_bytes(np.ascontiguousarray(x, np.float32)) == expected, "inputs did not regenerate"
    weights = case.program.fp16_weights() if case.fp16_weights else case.program.weights
    outputs = oracle.run(case.program, case.inputs, weights=weights)
    assert len(outputs) == len(entry["outputs"])
    for out, golden in zip(outputs, entry["outputs"]):
        assert list(out.shape) == golden["shape"]
        assert canonical_digest(out) == golden["sha256"], f"{entry['name']}: output differs from the reference"


def test_checker_catches_a_planted_one_ulp_error(oracle):
    """A one-ulp change in one oracle output must break the digest and be counted."""
    case = CASES["config1"]
    out = oracle.run(case.program, case.inputs)[0]
    planted = out.copy()
    planted.view(np.uint32)[0, 3, 5] ^= 1
    assert canonical_digest(planted) != GOLDEN["programs"][[p["name"] for p in GOLDEN["programs"]].index("config1")][
        "outputs"][0]["sha256"]
    assert count_differing(out, planted) == 1
    assert not same_bits(out, planted)


# ---------------------------------------------------------------- reference known-answer checks

def test_exp_accuracy_and_edges(oracle):
    """det_exp within 5e-7 relative of exp over [-87, 88) in 0.0137 steps; its
    cut-offs, NaN, sigmoid saturation; exact half widening (tests/...:75-93)."""
    lib = oracle.lib
    worst = 0.0
    x = np.float32(-87.0)
    step = np.float32(0.0137)
    while x < np.float32(88.0):
        expected = math.exp(float(x))
        worst = max(worst, abs(lib.or_exp(float(x)) - expected) / expected)
        x = np.float32(x + step)
    assert worst < 5e-7
    assert lib.or_exp(-87.5) == 0.0
    assert math.isinf(lib.or_exp(88.0))
    assert math.isnan(lib.or_exp(float("nan")))
    assert lib.or_sigmoid(-200.0) == 0.0 and lib.or_sigmoid(200.0) == 1.0
    assert lib.or_half_to_float(0x3C00) == 1.0
    assert lib.or_half_to_float(0xC000) == -2.0
    assert lib.or_half_to_float(0x0001) == math.ldexp(1.0, -24)
    assert lib.or_half_to_float(0x7BFF) == 65504.0


def test_cpu_pointwise_close_to_double_and_deterministic(oracle):
    """The 16-bit integer pointwise conv stays within 2e-3 of an independent
    double-precision dot product, and repeated runs give the same bits (tests/...:181-214)."""
    stream = SeededStream(7)
    program = op_program(stream)
    x = stream.tensor(70, 11, 18, 2.0)
    outputs = oracle.run(program, [x], weights=program.weights)
    pointwise = outputs[1]
    node = program.nodes[0]
    w = program.weights[node.weight_offset: node.weight_offset + 133 * 70].astype(np.float64).reshape(133, 70)
    b = program.weights[node.bias_offset: node.bias_offset + 133].astype(np.float64)
    exact = w @ x.reshape(70, -1).astype(np.float64) + b[:, None]
    worst = 0.0
    for out in range(0, 133, 17):
        for position in range(0, 11 * 18, 13):
            worst = max(worst, abs(exact[out, position] - pointwise.reshape(133, -1)[out, position]))
    assert worst < 2e-3
    assert outputs[0].shape == (9, 10, 18)
    again = oracle.run(program, [x], weights=program.weights)
    assert all(same_bits(a, b) for a, b in zip(outputs, again))


def test_data_movement_against_direct_indexing(oracle):
    """space_to_depth in PixelUnshuffle order; scale_channels, concat, crop and
    clamp composed by hand (tests/...:265-309)."""
    stream = SeededStream(41)
    inputs = [stream.tensor(5, 12, 20, 1.5), stream.tensor(20, 1, 1, 2.0), stream.tensor(1, 5, 7, 1.0)]
    f, a = oracle.run(data_movement_program(), inputs)
    x, s, _ = inputs
    assert a.shape == (20, 6, 10) and f.shape == (40, 5, 7)
    for c in range(20):
        source, i, j = c // 4, (c // 2) % 2, c % 2
        assert same_bits(a[c], x[source, i::2, j::2])
    for c in range(40):
        channel = c % 20
        value = a[channel, :5, :7]
        if c < 20:
            value = (value * s[channel, 0, 0]).astype(np.float32)
        value = np.where(value < -0.5, np.float32(-0.5), np.where(value > 0.75, np.float32(0.75), value))
        assert same_bits(f[c], value)


# ---------------------------------------------------------------- live reference

@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: f"{c[0]}to{c[1]}k{c[2][0]}x{c[2][1]}s{c[3][0]}")
@pytest.mark.parametrize("bits", [(16, 16), (8, 16), (16, 8), (8, 8)], ids=lambda b: f"w{b[0]}a{b[1]}")
def test_oracle_matches_live_reference(oracle, reference, tmp_path, case, bits):
    cin, cout, kernel, stride, pads, h, w = case
    stream = SeededStream(3000 + cin * 7 + cout)
    program = conv_program(stream, cin, cout, kernel, stride, pads, bits, wsilu=cout % 2 == 0)
    x = stream.tensor(cin, h, w, 5.0)
    path = program.write(tmp_path)
    for weights in (None, program.weights):
        expected = reference.run(path, [x], weights=weights)
        got = oracle.run(program, [x], weights=weights)
        assert all(count_differing(a, b) == 0 for a, b in zip(expected, got))


@pytest.mark.parametrize("bits", [(16, 16), (8, 8)], ids=["w16a16", "w8a8"])
@pytest.mark.parametrize("which", ["chain", "depthwise120", "depthwise250"])
def test_oracle_matches_live_reference_on_chains(oracle, reference, tmp_path, bits, which):
    """The chains behind the staged-intermediate GPU tests (1x1 -> 3x3 -> WSiLU
    chunk-add -> residual; WSiLU -> depthwise 3x3 -> 1x1), with NaN, inf and zero
    inputs, agree with the reference bit for bit (NaN equals NaN)."""
    stream = SeededStream(9100 + bits[0])
    if which == "chain":
        program = staged_chain_program(stream, bits)
    else:
        program = staged_depthwise_program(stream, int(which[len("depthwise"):]), bits)
    x = stream.tensor(24, 9, 13, 2.0)
    x[3, 4, 5] = np.nan
    x[7, 2, 11] = np.inf
    x[:, 6, 12] = 0.0
    path = program.write(tmp_path)
    expected = reference.run(path, [x])
    got = oracle.run(program, [x])
    assert all(count_differing(a, b) == 0 for a, b in zip(expected, got))


def test_reference_output_extents(reference, tmp_path):
    """infer_output_extents of the op program, and its refusal of a wrong channel count."""
    stream = SeededStream(1)
    program = op_program(stream)
    path = program.write(tmp_path)
    code, extents = reference.infer_extents(path, [(70, 33, 47)])
    assert code == 0 and extents == [(9, 32, 46), (133, 33, 47)]
    code, message = reference.infer_extents(path, [(71, 33, 47)])
    assert code == 1 and "unexpected shape" in message  # invalid_argument
