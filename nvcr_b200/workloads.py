"""Synthetic intconv.v1 workloads at the benchmark's shapes.

All values come from seeded std::mt19937 streams (SeededStream), so the GPU
path, the oracle and the reference see identical inputs on every platform.
Integer values stand in for the int8 tensors the benchmark names. The profile
carries FP16 at stage boundaries, so the int8 weights are stored times 2^-10
(exact in FP16): each row quantises back to exactly the same int8 values with
scale max|w| / 127, so the integer GEMM is the benchmark's int8 x int8 product,
and the FP16 outputs stay finite instead of saturating at 65504.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from .program import OpKind, Program, SeededStream


WEIGHT_SCALE = 2.0 ** -10


@dataclasses.dataclass
class Layer:
    name: str
    program: Program
    input_shape: tuple[int, int, int]
    ops: float  # 2 * C_in * kh * kw * C_out * P (one MAC = 2 ops)


def _int_tensor(stream: SeededStream, count: int, low: int = -127, high: int = 127) -> np.ndarray:
    return stream.integers(low, high, count).astype(np.float32)


def conv_layer(name: str, cin: int, cout: int, height: int, width: int, *, kernel=(3, 3), stride=(1, 1),
               pads=(1, 1, 1, 1), d2s: int = 0, bits=(8, 8), seed: int = 0,
               bias_range: tuple[int, int] = (-127, 127)) -> Layer:
    """One integer conv as the exporter lowers it (im2col + pointwise), with an
    optional depth_to_space after it. Weights and bias are drawn from `seed`."""
    stream = SeededStream(seed)
    p = Program(name=name)
    x = p.add_input("x", cin)
    taps = kernel[0] * kernel[1]
    w = _int_tensor(stream, cout * cin * taps) * np.float32(WEIGHT_SCALE)
    b = _int_tensor(stream, cout, *bias_range)
    y = p.dense_conv(x, cout, w, b, "y" if not d2s else "conv", kernel=kernel, stride=stride, pads=pads, bits=bits)
    if d2s:
        y = p.unary(OpKind.depth_to_space, y, "y", block=d2s)
    p.finish([y])
    out_h = (height + pads[0] + pads[2] - kernel[0]) // stride[0] + 1
    out_w = (width + pads[1] + pads[3] - kernel[1]) // stride[1] + 1
    ops = 2.0 * cin * taps * cout * out_h * out_w
    return Layer(name, p, (cin, height, width), ops)


def config1() -> Layer:
    """3x3 s1 p1 conv 64->64 on a 36x44 input, w8a8,
    weights and input in [-127, 127], bias in [-2^15, 2^15], seed 0 (draw
    order: weights, bias; the input comes from seed 1)."""
    return conv_layer("config1", 64, 64, 36, 44, seed=0, bias_range=(-(2**15), 2**15))


def config2() -> list[Layer]:
    """the 1920x1088 layer sweep, w8a8, every value in
    [-127, 127]; layer i's weights come from seed 100 + i."""
    return [
        conv_layer("L1_3x3s2_3to64", 3, 64, 1088, 1920, stride=(2, 2), seed=101),
        conv_layer("L2_3x3_64to64", 64, 64, 544, 960, seed=102),
        conv_layer("L3_1x1_128to256", 128, 256, 272, 480, kernel=(1, 1), pads=(0, 0, 0, 0), seed=103),
        conv_layer("L4_3x3_256to256", 256, 256, 136, 240, seed=104),
        conv_layer("L5_3x3_256to1024_d2s", 256, 1024, 68, 120, d2s=2, seed=105),
    ]


def layer_input(layer: Layer, seed: int, height: int | None = None) -> np.ndarray:
    """The layer's seeded int8-valued input (optionally only its first `height` rows)."""
    c, h, w = layer.input_shape
    h = h if height is None else height
    return _int_tensor(SeededStream(seed), c * h * w).reshape(c, h, w)
