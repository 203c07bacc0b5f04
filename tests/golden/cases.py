"""The cases of the golden fixtures (tests/golden/intconv_golden.json): scalar
arguments of the profile's arithmetic, weight matrices for the quantiser, and
whole programs with seeded inputs. Shared by make_golden.py (which ran them on
the reference) and tests/test_oracle.py (which runs them on the oracle)."""
from __future__ import annotations

import dataclasses

import numpy as np

from nvcr_b200.program import Program, SeededStream
from nvcr_b200.workloads import config1, layer_input
from tests.programs import (CONV_CASES, conv_program, data_movement_program, edge_value_input, op_program,
                            sigmoid_program, sigmoid_sweep_values)

WIDTHS = [(16, 16), (8, 16), (16, 8), (8, 8)]


def scalar_inputs() -> dict:
    """Arguments for det_exp/sigmoid/ldexp/frexp/quantize/output and the FP16 conversions."""
    stream = SeededStream(2024)
    sweep = np.arange(0, 2**32, 65521, dtype=np.uint64).astype(np.uint32)
    specials = np.array([0x00000000, 0x80000000, 0x00000001, 0x807FFFFF, 0x7F800000, 0xFF800000, 0x7FC00000,
                         0x7F7FFFFF, 0xFF7FFFFF, 0x42B00000, 0xC2AE0000, 0xC2AEFFFF, 0x42AFFFFF, 0x38800000,
                         0x33800000, 0x33000000, 0x477FE000, 0x477FF000, 0x477FEFFF], np.uint32)
    floats = np.concatenate([specials, sweep]).view(np.float32)
    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ldexp_values = np.concatenate([stream.uniform(-4, 4, 200), np.array([2.0 ** -149, -(2.0 ** -140), 3.0e38,
                                                                          1.5, -1.5, 0.0, -0.0], np.float32)])
    ldexp_exponents = np.concatenate([stream.integers(-300, 300, 200), np.array([150, 170, -1, -150, -149, 10, 10])])
    maxima = np.concatenate([np.abs(stream.uniform(-100, 100, 100)),
                             np.array([0.0, 2.0 ** -149, 2.0 ** -126, 1.0, 127.0, 128.0, 65504.0, 3.4e38],
                                      np.float32)]).astype(np.float32)
    q_values = np.concatenate([stream.uniform(-200, 200, 300),
                               np.array([0.5, 1.5, 2.5, -0.5, -2.5, 127.5, -127.5, 200.0, 1e-40], np.float32)])
    q_exponents = np.concatenate([stream.integers(-20, 20, 300), np.array([0, 0, 0, 0, 0, 0, 0, 0, -140])])
    acc = np.concatenate([stream.integers(-(2**40), 2**40, 200), np.array([2**53 + 1, -(2**31), 2**31 - 1, 0])])
    acc_scale = np.concatenate([stream.uniform(0, 1e-3, 200), np.array([1.0, 0.5, 3.0, 1.0], np.float32)])
    acc_exponent = np.concatenate([stream.integers(-160, 120, 200), np.array([0, -130, 5, 0])])
    acc_bias = np.concatenate([stream.uniform(-1, 1, 200), np.array([0.25, -0.0, 1e-30, 0.0], np.float32)])
    return {"floats": floats, "halves": halves, "ldexp_values": ldexp_values.astype(np.float32),
            "ldexp_exponents": ldexp_exponents.astype(np.int64), "maxima": maxima,
            "q_values": q_values.astype(np.float32), "q_exponents": q_exponents.astype(np.int64),
            "acc": acc.astype(np.int64), "acc_scale": acc_scale.astype(np.float32),
            "acc_exponent": acc_exponent.astype(np.int64), "acc_bias": acc_bias.astype(np.float32)}


def weight_cases():
    stream = SeededStream(99)
    w = stream.uniform(-0.5, 0.5, 40 * 70).reshape(40, 70)
    w[0] = 0.0
    w[1, :3] = [65504.0, -65504.0, 1e-7]
    w[2] = np.float32(2.0 ** -24)
    cases = []
    for bits in (8, 16):
        cases.append((f"mixed_w{bits}", w.copy(), bits))
    ints = stream.integers(-127, 127, 16 * 27).astype(np.float32).reshape(16, 27) * np.float32(2.0 ** -10)
    cases.append(("int8_scaled_w8", ints, 8))
    return cases


@dataclasses.dataclass
class Case:
    name: str
    program: Program
    inputs: list
    fp16_weights: bool = False


def program_cases() -> list[Case]:
    cases = []
    for bits in WIDTHS:
        for h, w in [(11, 18), (2, 64)]:
            stream = SeededStream(11)
            program = op_program(stream).with_widths(*bits)
            cases.append(Case(f"ops_w{bits[0]}a{bits[1]}_{h}x{w}", program, [stream.tensor(70, h, w, 3.0)]))
    stream = SeededStream(7)
    program = op_program(stream).with_widths(16, 16)
    cases.append(Case("ops_fp16_weights_11x18", program, [stream.tensor(70, 11, 18, 2.0)], fp16_weights=True))
    stream = SeededStream(41)
    cases.append(Case("data_movement", data_movement_program(),
                      [stream.tensor(5, 12, 20, 1.5), stream.tensor(20, 1, 1, 2.0), stream.tensor(1, 5, 7, 1.0)]))
    cases.append(Case("sigmoid_sweep_65521", sigmoid_program(), [sigmoid_sweep_values(65521).reshape(1, 1, -1)]))
    layer = config1()
    cases.append(Case("config1", layer.program, [layer_input(layer, seed=1)], fp16_weights=True))
    for case in CONV_CASES[:6]:
        cin, cout, kernel, stride, pads, h, w = case
        for bits in ((8, 8), (16, 16)):
            stream = SeededStream(1000 + cin + cout)
            program = conv_program(stream, cin, cout, kernel, stride, pads, bits)
            cases.append(Case(f"conv_{cin}to{cout}_k{kernel[0]}x{kernel[1]}s{stride[0]}_w{bits[0]}a{bits[1]}",
                              program, [stream.tensor(cin, h, w, 2.0)]))
    for bits in WIDTHS:
        stream = SeededStream(5)
        x = edge_value_input(stream, 40)
        program = conv_program(stream, 40, 72, (3, 3), (1, 1), (1, 1, 1, 1), bits)
        cases.append(Case(f"edge_values_w{bits[0]}a{bits[1]}", program, [x]))
    stream = SeededStream(77)
    program = conv_program(stream, 96, 192, (1, 1), (1, 1), (0, 0, 0, 0), (16, 8), wsilu=True, chunk_add=True,
                           residual=True)
    cases.append(Case("fusion_wsilu_chunk_residual_w16a8", program, [stream.tensor(96, 13, 29, 3.0)]))
    return cases
