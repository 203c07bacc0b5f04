"""Programs the reference's conformance suite runs, rebuilt with this repo's
program model (reference tests/deterministic_executor_tests.cpp)."""
from __future__ import annotations

import numpy as np

from nvcr_b200.program import OpKind, Program, SeededStream


def op_program(stream: SeededStream) -> Program:
    """Every op on awkward, non-tile-multiple shapes (tests/...:95-179): integer
    pointwise 70->133 + WSiLU, depthwise 3x3, slice 3..131, FP32 dense 3x3
    128->36, FP32 2x2 stride 2, depth_to_space 2, add. Weights in the same
    draw order as the reference test (weights then bias per conv)."""
    p = Program(name="ops")

    def conv(source, cin, cout, depthwise, kernel, stride, pads, name):
        per_output = (1 if depthwise else cin) * kernel[0] * kernel[1]
        w = stream.uniform(-0.3, 0.3, cout * per_output)
        b = stream.uniform(-0.1, 0.1, cout)
        return p.conv(source, cout, w, b, name, depthwise=depthwise, kernel=kernel, stride=stride,
                      pads=pads)

    x = p.add_input("x", 70)
    pointwise = conv(x, 70, 133, False, (1, 1), (1, 1), (0, 0, 0, 0), "pointwise")
    scaled = p.unary(OpKind.mul_scalar, pointwise, "scaled", scalar=4.0)
    gate = p.unary(OpKind.sigmoid, scaled, "gate")
    product = p.binary(OpKind.mul, gate, pointwise, "product")
    depthwise = conv(product, 133, 133, True, (3, 3), (1, 1), (1, 1, 1, 1), "depthwise")
    sliced = p.unary(OpKind.slice_channels, depthwise, "slice", begin=3, end=131)
    dense = conv(sliced, 128, 36, False, (3, 3), (1, 1), (1, 1, 1, 1), "dense")
    strided = conv(dense, 36, 36, False, (2, 2), (2, 2), (0, 0, 0, 0), "strided")
    shuffle = p.unary(OpKind.depth_to_space, strided, "shuffle", block=2)
    total = p.binary(OpKind.add, shuffle, shuffle, "sum")
    return p.finish([total, pointwise])


def data_movement_program() -> Program:
    """scale_channels, clamp, concat, crop, space_to_depth (tests/...:223-263)."""
    p = Program(name="data_movement")
    x = p.add_input("x", 5)
    s = p.add_input("s", 20)
    r = p.add_input("r", 1)
    a = p.unary(OpKind.space_to_depth, x, "a", block=2)
    b = p.binary(OpKind.scale_channels, a, s, "b")
    c = p.binary(OpKind.concat, b, a, "c")
    d = p.binary(OpKind.crop, c, r, "d", axis=2)
    e = p.binary(OpKind.crop, d, r, "e", axis=3)
    f = p.unary(OpKind.clamp, e, "f", minimum=-0.5, maximum=0.75)
    return p.finish([f, a])


def sigmoid_program() -> Program:
    p = Program(name="sigmoid")
    x = p.add_input("x", 1)
    y = p.unary(OpKind.sigmoid, x, "y")
    return p.finish([y])


def sigmoid_sweep_values(step: int = 1021) -> np.ndarray:
    """Every `step`-th float bit pattern plus zeros, denormals, infinities, NaN
    and the exp cut-offs (tests/...:377-410)."""
    patterns = [0x00000000, 0x80000000, 0x00000001, 0x807FFFFF, 0x7F800000, 0xFF800000,
                0x7FC00000, 0x7F7FFFFF, 0xFF7FFFFF]
    sweep = np.arange(0, 2**32, step, dtype=np.uint64).astype(np.uint32)
    bits = np.concatenate([np.array(patterns, np.uint32), sweep])
    values = bits.view(np.float32)
    edges = np.array([-88.0, -87.0, -86.99999, 87.0, 87.99999, 88.0], np.float32)
    return np.concatenate([values, edges])
