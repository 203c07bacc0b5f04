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


# ---------------------------------------------------------------- DCVC-RT-style stacks

# The reference pins the intra decoder's block topology by layer name
# (i.dec.dec_1.0 = upsample + DepthConvBlock, i.dec.dec_1.1..12 = DepthConvBlocks,
# i.dec.dec_2 = DepthConvBlock with an adaptor; configs/numerics/dcvcrt-fx.json)
# and the DepthConvBlock structure (scripts/backends/dcvc_fx.py:178-188), but not
# the upstream channel widths or weights. The stacks below use that topology with
# widths chosen here (256 channels at 1/8 resolution) and seeded weights.

DECODER_CHANNELS = 256
DECODER_BLOCKS = 12
WSILU_SCALE = 4.0


class _StackBuilder:
    """Appends DCVC-RT-style blocks to a Program, with seeded weights."""

    def __init__(self, p: Program, stream: SeededStream, bits=(8, 8)) -> None:
        self.p = p
        self.stream = stream
        self.bits = bits
        self.ops = 0.0  # integer-conv MACs x 2 per output position (scaled by positions at the end)

    def weights(self, count: int, fan_in: int) -> np.ndarray:
        bound = 1.0 / np.sqrt(fan_in)
        return self.stream.uniform(-bound, bound, count).astype(np.float16).astype(np.float32)

    def bias(self, count: int) -> np.ndarray:
        return self.stream.uniform(-0.05, 0.05, count).astype(np.float16).astype(np.float32)

    def pointwise(self, x: int, cout: int, name: str) -> int:
        cin = self.p.tensor_channels[x]
        self.ops += 2.0 * cin * cout
        return self.p.conv(x, cout, self.weights(cout * cin, cin), self.bias(cout), name, bits=self.bits)

    def wsilu(self, y: int, name: str) -> int:
        s = self.p.unary(OpKind.mul_scalar, y, f"{name}.scaled", scalar=WSILU_SCALE)
        g = self.p.unary(OpKind.sigmoid, s, f"{name}.gate")
        return self.p.binary(OpKind.mul, y, g, f"{name}.wsilu")

    def chunk_add(self, y: int, name: str) -> int:
        c = self.p.tensor_channels[y]
        a = self.p.unary(OpKind.slice_channels, y, f"{name}.low", begin=0, end=c // 2)
        b = self.p.unary(OpKind.slice_channels, y, f"{name}.high", begin=c // 2, end=c)
        return self.p.binary(OpKind.add, a, b, f"{name}.sum")

    def depthwise(self, x: int, name: str) -> int:
        c = self.p.tensor_channels[x]
        return self.p.conv(x, c, self.weights(c * 9, 9), self.bias(c), name, depthwise=True, kernel=(3, 3),
                           pads=(1, 1, 1, 1))

    def depth_conv_block(self, x: int, channels: int, name: str, *, adaptor: bool = False,
                         shortcut: bool = False) -> int:
        """adaptor 1x1 -> 1x1 + WSiLU -> depthwise 3x3 -> 1x1 + residual -> 1x1 + WSiLU
        chunk-add -> 1x1 + residual (+ the block input when `shortcut`)."""
        if adaptor:
            x = self.pointwise(x, channels, f"{name}.adaptor")
        t = self.wsilu(self.pointwise(x, channels, f"{name}.dc.0"), f"{name}.dc.1")
        t = self.depthwise(t, f"{name}.dc.2")
        out = self.p.binary(OpKind.add, self.pointwise(t, channels, f"{name}.dc.3"), x, f"{name}.dc.res")
        t = self.pointwise(out, 4 * channels, f"{name}.ffn.0")
        t = self.chunk_add(self.wsilu(t, f"{name}.ffn.1"), f"{name}.ffn.1")
        y = self.p.binary(OpKind.add, self.pointwise(t, channels, f"{name}.ffn.2"), out, f"{name}.ffn.res")
        if shortcut:
            y = self.p.binary(OpKind.add, y, x, f"{name}.shortcut")
        return y

    def subpel_up(self, x: int, channels: int, name: str) -> int:
        """SubpelConv2x: 1x1 conv to 4x the channels, then depth_to_space(2)."""
        y = self.pointwise(x, 4 * channels, f"{name}.conv.0")
        return self.p.unary(OpKind.depth_to_space, y, f"{name}.shuffle", block=2)


@dataclasses.dataclass
class Stack:
    name: str
    program: Program
    input_shapes: list[tuple[int, int, int]]
    ops: float          # algorithmic integer-conv ops per run (2 per MAC)


def intra_decoder(latent_hw: tuple[int, int] = (68, 120), *, channels: int = DECODER_CHANNELS,
                  blocks: int = DECODER_BLOCKS, bits=(8, 8), seed: int = 300,
                  every_tensor: bool = False, feature_channels: int = 0) -> Stack:
    """a DCVC-RT-architecture intra decoder. y_hat
    [256, h, w] (1/16 of the frame) -> dec_1.0 (SubpelConv2x up + DepthConvBlock)
    -> dec_1.1..blocks (DepthConvBlocks at 1/8) -> dec_2 (DepthConvBlock with an
    adaptor) -> 1x1 head to 3 x 8 x 8 channels -> depth_to_space(8): the
    3 x 16h x 16w frame. `every_tensor` makes every block's output a program
    output (for parity tests)."""
    stream = SeededStream(seed)
    p = Program(name="intra_decoder")
    b = _StackBuilder(p, stream, bits)
    y_hat = p.add_input("y_hat", 256)
    taps = []
    x = b.subpel_up(y_hat, channels, "i.dec.dec_1.0.up")
    up_ops = b.ops  # at the latent resolution
    b.ops = 0.0
    x = b.depth_conv_block(x, channels, "i.dec.dec_1.0.conv")
    taps.append(x)
    for i in range(1, blocks + 1):
        x = b.depth_conv_block(x, channels, f"i.dec.dec_1.{i}")
        taps.append(x)
    x = b.depth_conv_block(x, channels, "i.dec.dec_2", adaptor=True)
    taps.append(x)
    head = b.pointwise(x, 3 * 64, "i.dec.head")
    frame = p.unary(OpKind.depth_to_space, head, "frame", block=8)
    outputs = (taps + [frame]) if every_tensor else [frame]
    if feature_channels:
        # The reconstructed feature a following P-frame takes as temporal context.
        outputs.append(b.pointwise(x, feature_channels, "feature"))
    p.finish(outputs)
    h, w = latent_hw
    ops = up_ops * h * w + b.ops * (2 * h) * (2 * w)
    return Stack("config3_intra_decoder", p, [(256, h, w)], ops)


def inter_decoder(latent_hw: tuple[int, int] = (48, 80), *, channels: int = DECODER_CHANNELS,
                  context_channels: int = 64, blocks: int = 4, bits=(8, 8), seed: int = 400,
                  every_tensor: bool = False) -> Stack:
    """BASELINE config 4's P-frame decoder, synthetic with the reference's P-side
    names (p.decoder.*, p.recon_generation_net.*, p.feature_adaptor_p): y_hat
    [256, h, w] -> SubpelConv2x up to 1/8 -> concat the previous frame's feature
    [64, 2h, 2w] (temporal context) -> DepthConvBlock with an adaptor -> `blocks`
    DepthConvBlocks -> the next feature (1x1 to 64) and the frame (1x1 head,
    depth_to_space(8))."""
    stream = SeededStream(seed)
    p = Program(name="inter_decoder")
    b = _StackBuilder(p, stream, bits)
    y_hat = p.add_input("y_hat", 256)
    context = p.add_input("context", context_channels)
    x = b.subpel_up(y_hat, channels, "p.decoder.up")
    up_ops = b.ops
    b.ops = 0.0
    x = p.binary(OpKind.concat, x, context, "p.decoder.context")
    taps = []
    x = b.depth_conv_block(x, channels, "p.decoder.conv1.0", adaptor=True)
    taps.append(x)
    for i in range(blocks):
        x = b.depth_conv_block(x, channels, f"p.recon_generation_net.conv.{i}")
        taps.append(x)
    feature = b.pointwise(x, context_channels, "feature")
    head = b.pointwise(x, 3 * 64, "p.recon_generation_net.head")
    frame = p.unary(OpKind.depth_to_space, head, "frame", block=8)
    p.finish((taps + [frame, feature]) if every_tensor else [frame, feature])
    h, w = latent_hw
    ops = up_ops * h * w + b.ops * (2 * h) * (2 * w)
    return Stack("config4_inter_decoder", p, [(256, h, w), (context_channels, 2 * h, 2 * w)], ops)


def laplace_latent(stream: SeededStream, shape: tuple[int, int, int], scale: float = 4.0) -> np.ndarray:
    """Integer latents: Laplace(0, scale) by inverse CDF of the stream's uniforms,
    rounded to nearest and clamped to [-127, 127]."""
    count = int(np.prod(shape))
    u = stream.uniform(-0.5, 0.5, count).astype(np.float64)
    u = np.clip(u, -0.5 + 1e-12, 0.5 - 1e-12)
    x = -scale * np.sign(u) * np.log1p(-2.0 * np.abs(u))
    return np.clip(np.rint(x), -127, 127).astype(np.float32).reshape(shape)


def half_digest(values) -> str:
    """SHA-256 of an FP16 tensor's bytes (C order) with every NaN stored as
    0x7e00, so digests compare under the profile's rule that any NaN equals any
    NaN. Accepts FP16 arrays, or FP32 arrays, which are first rounded to FP16
    (round to nearest even, as at a stage boundary)."""
    import hashlib

    array = np.ascontiguousarray(values)
    if array.dtype != np.float16:
        array = array.astype(np.float32).astype(np.float16)
    bits = array.view(np.uint16).copy()
    bits[((bits & 0x7C00) == 0x7C00) & ((bits & 0x03FF) != 0)] = 0x7E00
    return hashlib.sha256(bits.tobytes()).hexdigest()
