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


def conv_program(stream: SeededStream, cin, cout, kernel, stride, pads, bits, *, wsilu=False,
                         chunk_add=False, residual=False, name="conv") -> Program:
    p = Program(name=name)
    x = p.add_input("x", cin)
    r = None
    if residual:
        # An earlier tensor of the output's shape (produced before the conv, so
        # the add folds into the conv's epilogue): a 1x1 FP32 depthwise of x, sliced.
        out_c = cout // 2 if chunk_add else cout
        if out_c > cin:
            raise ValueError("residual needs out channels <= in channels")
        r = p.conv(x, cin, stream.uniform(-1, 1, cin), stream.uniform(-1, 1, cin), "r_dw", depthwise=True)
        if out_c < cin:
            r = p.unary(OpKind.slice_channels, r, "r", begin=0, end=out_c)
    taps = kernel[0] * kernel[1]
    w = stream.uniform(-0.5, 0.5, cout * cin * taps)
    b = stream.uniform(-0.2, 0.2, cout)
    y = p.dense_conv(x, cout, w, b, "c", kernel=kernel, stride=stride, pads=pads, bits=bits)
    if wsilu:
        s = p.unary(OpKind.mul_scalar, y, "s", scalar=4.0)
        g = p.unary(OpKind.sigmoid, s, "g")
        y = p.binary(OpKind.mul, y, g, "w")
    if chunk_add:
        a = p.unary(OpKind.slice_channels, y, "a", begin=0, end=cout // 2)
        b2 = p.unary(OpKind.slice_channels, y, "b", begin=cout // 2, end=cout)
        y = p.binary(OpKind.add, a, b2, "ca")
    if residual:
        y = p.binary(OpKind.add, y, r, "res")
    return p.finish([y])


CONV_CASES = [
    # cin, cout, kernel, stride, pads, height, width
    (64, 64, (3, 3), (1, 1), (1, 1, 1, 1), 36, 44),      # config-1 shape
    (3, 64, (3, 3), (2, 2), (1, 1, 1, 1), 40, 70),       # config-2 L1 shape (K = 27)
    (128, 256, (1, 1), (1, 1), (0, 0, 0, 0), 17, 30),    # pointwise, one full N tile
    (70, 133, (1, 1), (1, 1), (0, 0, 0, 0), 11, 18),     # ragged N, K
    (96, 300, (1, 1), (1, 1), (0, 0, 0, 0), 9, 15),      # two N tiles
    (32, 520, (3, 3), (1, 1), (1, 1, 1, 1), 8, 9),       # three N tiles
    (16, 24, (2, 2), (2, 2), (0, 0, 0, 0), 10, 14),      # 2x2 stride 2
    (20, 40, (3, 5), (1, 2), (2, 0, 1, 3), 13, 21),      # asymmetric window and pads
    (200, 48, (3, 3), (1, 1), (1, 1, 1, 1), 5, 7),       # K = 1800, ragged
    # few channels: the receptive field of a position staged as one record
    (1, 24, (3, 3), (1, 1), (1, 1, 1, 1), 19, 33),      # K = 9
    (7, 40, (3, 3), (2, 2), (1, 1, 1, 1), 23, 37),      # K = 63
    (2, 32, (5, 5), (2, 1), (2, 2, 2, 2), 17, 26),      # K = 50
    (3, 33, (3, 5), (1, 2), (2, 0, 1, 3), 13, 21),      # K = 45, asymmetric
]


def edge_value_input(stream: SeededStream, cin: int = 40) -> np.ndarray:
    """All-zero positions (e = 0), NaN/inf positions (NaN out), maxima in the
    subnormal range (exponents below -126: the wide ldexp path), subnormal
    steps, large magnitudes, values on rounding ties and a near-FLT_MAX value."""
    h, w = 6, 50
    x = stream.tensor(cin, h, w, 1.0)
    x[:, 0, 0] = 0.0
    x[3, 0, 1] = np.nan
    x[7, 0, 2] = np.inf
    x[8, 0, 3] = -np.inf
    x[:, 1, :] *= np.float32(2.0 ** -130)
    x[:, 2, :10] = np.float32(2.0 ** -149) * np.arange(1, cin + 1, dtype=np.float32)[:, None]
    x[:, 3, :] *= np.float32(60000.0)
    x[:, 4, :] = (np.round(x[:, 4, :] * 64) + 0.5) / 64
    x[0, 5, :] = np.float32(3.4e38)
    return x


def staged_chain_program(stream: SeededStream, bits) -> Program:
    """Intermediates that only integer convs read (stored channel-innermost by
    the producing epilogue): 1x1 40->48 (read by a 3x3 conv and, later, as a
    residual), 3x3 48->40, 1x1 40->96 + WSiLU + chunk-add -> 48, 1x1 48->48 +
    residual of the first conv's output; ragged channel counts so the padding
    channels of the staged records matter."""
    p = Program(name="staged_chain")
    x = p.add_input("x", 24)

    def conv(src, cin, cout, name, kernel=(1, 1), pads=(0, 0, 0, 0)):
        taps = kernel[0] * kernel[1]
        w = stream.uniform(-0.5, 0.5, cout * cin * taps)
        b = stream.uniform(-0.2, 0.2, cout)
        return p.dense_conv(src, cout, w, b, name, kernel=kernel, stride=(1, 1), pads=pads, bits=bits)

    a = conv(x, 24, 48, "a")
    t = conv(a, 48, 40, "t", kernel=(3, 3), pads=(1, 1, 1, 1))
    u = conv(t, 40, 96, "u")
    s = p.unary(OpKind.mul_scalar, u, "us", scalar=4.0)
    g = p.unary(OpKind.sigmoid, s, "ug")
    u = p.binary(OpKind.mul, u, g, "uw")
    h1 = p.unary(OpKind.slice_channels, u, "u0", begin=0, end=48)
    h2 = p.unary(OpKind.slice_channels, u, "u1", begin=48, end=96)
    v = p.binary(OpKind.add, h1, h2, "v")
    y = conv(v, 48, 48, "y")
    y = p.binary(OpKind.add, y, a, "out")
    return p.finish([y])


def staged_depthwise_program(stream: SeededStream, channels: int, bits) -> Program:
    """1x1 24->C + WSiLU -> depthwise 3x3 -> 1x1 C->40: the WSiLU conv's output and
    the depthwise output are read only by the depthwise and the last conv, so both
    stay channel-innermost and the depthwise runs on that layout."""
    p = Program(name="staged_depthwise")
    x = p.add_input("x", 24)
    t = p.dense_conv(x, channels, stream.uniform(-0.5, 0.5, channels * 24), stream.uniform(-0.2, 0.2, channels),
                     "t", kernel=(1, 1), stride=(1, 1), pads=(0, 0, 0, 0), bits=bits)
    s = p.unary(OpKind.mul_scalar, t, "ts", scalar=4.0)
    g = p.unary(OpKind.sigmoid, s, "tg")
    t = p.binary(OpKind.mul, t, g, "tw")
    d = p.conv(t, channels, stream.uniform(-0.5, 0.5, channels * 9), stream.uniform(-0.2, 0.2, channels), "d",
               depthwise=True, kernel=(3, 3), pads=(1, 1, 1, 1))
    y = p.dense_conv(d, 40, stream.uniform(-0.5, 0.5, 40 * channels), stream.uniform(-0.2, 0.2, 40), "y",
                     kernel=(1, 1), stride=(1, 1), pads=(0, 0, 0, 0), bits=bits)
    return p.finish([y])
