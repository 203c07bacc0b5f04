"""CUDA path == CPU oracle, bit for bit (NaN equals NaN), through the C ABI.

The programs are the reference's own conformance programs
(tests/deterministic_executor_tests.cpp:95-410) rebuilt here, the BASELINE
configs, and integer-conv cases aimed at the sm_100a kernels' edges: every
width pair, K and positions off the 128 tiles, multiple N tiles, chunk-add,
WSiLU and residual fusion, strided and padded windows, non-finite, tiny and
huge activations.
"""
from __future__ import annotations

import numpy as np
import pytest

from nvcr_b200.executor import CudaExecutor, reciprocal_mismatches
from nvcr_b200.program import OpKind, Program, SeededStream
from nvcr_b200.workloads import config1, layer_input
from oracle.oracle import count_differing, same_bits
from tests.programs import (CONV_CASES, conv_program, data_movement_program, edge_value_input, op_program,
                            staged_chain_program, staged_depthwise_program,
                            sigmoid_program, sigmoid_sweep_values)

pytestmark = pytest.mark.gpu

WIDTHS = [(16, 16), (8, 16), (16, 8), (8, 8)]


def run_gpu(program: Program, inputs, fp16_weights=False):
    with CudaExecutor.from_program(program, fp16_weights=fp16_weights) as executor:
        outputs = executor.run(inputs)
        executor.synchronize()
    return outputs


def assert_parity(program, inputs, oracle, label, fp16_weights=False):
    weights = program.fp16_weights() if fp16_weights else program.weights
    expected = oracle.run(program, inputs, weights=weights)
    got = run_gpu(program, inputs, fp16_weights=fp16_weights)
    assert len(got) == len(expected)
    for index, (g, e) in enumerate(zip(got, expected)):
        assert g.shape == e.shape, f"{label} output {index}: shape {g.shape} != {e.shape}"
        bad = count_differing(g, e)
        assert bad == 0, f"{label} output {index}: {bad} of {e.size} elements differ"


@pytest.mark.parametrize("height,width", [(11, 18), (2, 64), (33, 47)])
@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
def test_op_program(cuda, oracle, height, width, bits):
    stream = SeededStream(11)
    program = op_program(stream).with_widths(*bits)
    x = stream.tensor(70, height, width, 3.0)
    assert_parity(program, [x], oracle, f"ops {height}x{width} w{bits[0]}a{bits[1]}")


def test_data_movement(cuda, oracle):
    stream = SeededStream(41)
    inputs = [stream.tensor(5, 12, 20, 1.5), stream.tensor(20, 1, 1, 2.0), stream.tensor(1, 5, 7, 1.0)]
    assert_parity(data_movement_program(), inputs, oracle, "data movement")


def test_sigmoid_sweep(cuda, oracle):
    values = sigmoid_sweep_values()
    x = values.reshape(1, 1, -1)
    assert_parity(sigmoid_program(), [x], oracle, "sigmoid sweep")


def test_half_boundary_exhaustive(cuda, oracle):
    """Every binary16 pattern widens exactly and rounds back unchanged (mul by 1)."""
    import torch

    p = Program(name="identity")
    x = p.add_input("x", 1)
    y = p.unary(OpKind.mul_scalar, x, "y", scalar=1.0)
    p.finish([y])
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    with CudaExecutor.from_program(p) as executor:
        xh = torch.from_numpy(bits.view(np.float16).copy()).cuda().reshape(1, 1, -1)
        yh = torch.empty_like(xh)
        executor.run_half({"x": xh}, {"y": yh})
        executor.synchronize()
        got = yh.cpu().numpy().reshape(-1).view(np.uint16)
    nan = (bits & 0x7C00) == 0x7C00
    nan &= (bits & 0x03FF) != 0
    assert np.array_equal(got[~nan], bits[~nan])
    assert np.all(((got[nan] & 0x7C00) == 0x7C00) & ((got[nan] & 0x3FF) != 0))


def test_float_to_half_rounding(cuda, oracle):
    """FP32 -> FP16 at the stage boundary rounds to nearest even (subnormals,
    ties, overflow to inf), like the reference's det_float_to_half_bits: every
    binary16 input times 2^-11, 3 and 1.5 gives FP32 values that need rounding."""
    import torch

    p = Program(name="round")
    x = p.add_input("x", 1)
    outs = [p.unary(OpKind.mul_scalar, x, f"y{i}", scalar=s) for i, s in enumerate((2.0 ** -11, 3.0, 1.5))]
    p.finish(outs)
    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    with CudaExecutor.from_program(p) as executor:
        xh = torch.from_numpy(halves.copy()).cuda().reshape(1, 1, -1)
        ys = {f"y{i}": torch.empty_like(xh) for i in range(3)}
        executor.run_half({"x": xh}, ys)
        executor.synchronize()
        got = [ys[f"y{i}"].cpu().numpy().reshape(-1).view(np.uint16) for i in range(3)]
    widened = halves.astype(np.float32)
    for g, s in zip(got, (2.0 ** -11, 3.0, 1.5)):
        products = widened * np.float32(s)
        expected = np.array([oracle.lib.or_float_to_half(float(v)) for v in products], np.uint16)
        nan = np.isnan(products)
        assert np.array_equal(g[~nan], expected[~nan]), f"scale {s}"
        assert np.all((g[nan] & 0x7C00) == 0x7C00)


def test_config1_half(cuda, oracle):
    """BASELINE config 1 through run_half (FP16 stage boundary)."""
    import torch

    layer = config1()
    x = layer_input(layer, seed=1)
    expected = oracle.run(layer.program, [x])[0].astype(np.float16)
    with CudaExecutor.from_program(layer.program) as executor:
        xh = torch.from_numpy(x.astype(np.float16)).cuda()
        yh = torch.empty(expected.shape, dtype=torch.float16, device="cuda")
        executor.run_half({"x": xh}, {"y": yh})
        executor.synchronize()
        got = yh.cpu().numpy()
    assert count_differing(got.astype(np.float32), expected.astype(np.float32)) == 0




@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: f"{c[0]}to{c[1]}k{c[2][0]}x{c[2][1]}s{c[3][0]}")
@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
def test_integer_conv(cuda, oracle, case, bits):
    cin, cout, kernel, stride, pads, h, w = case
    stream = SeededStream(1000 + cin + cout)
    program = conv_program(stream, cin, cout, kernel, stride, pads, bits)
    x = stream.tensor(cin, h, w, 2.0)
    assert_parity(program, [x], oracle, f"conv {case} w{bits[0]}a{bits[1]}")


@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
@pytest.mark.parametrize("fusion", ["wsilu", "chunk", "wsilu_chunk_residual", "residual"])
def test_epilogue_fusions(cuda, oracle, bits, fusion):
    stream = SeededStream(77)
    cin, cout = (96, 192) if "chunk" in fusion else (96, 64)
    program = conv_program(stream, cin, cout, (1, 1), (1, 1), (0, 0, 0, 0), bits,
                                   wsilu="wsilu" in fusion, chunk_add="chunk" in fusion,
                                   residual="residual" in fusion)
    x = stream.tensor(cin, 13, 29, 3.0)
    assert_parity(program, [x], oracle, f"fusion {fusion}")


def test_chunk_add_many_tiles(cuda, oracle):
    stream = SeededStream(78)
    program = conv_program(stream, 64, 1040, (1, 1), (1, 1), (0, 0, 0, 0), (8, 8), chunk_add=True)
    x = stream.tensor(64, 7, 23, 2.0)
    assert_parity(program, [x], oracle, "chunk-add over several tiles")


@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
def test_activation_edge_values(cuda, oracle, bits):
    """All-zero positions (e = 0), NaN/inf positions (NaN out), subnormal and
    tiny inputs (exponents below -126: the wide ldexp path), huge inputs, and
    values on rounding ties."""
    stream = SeededStream(5)
    cin = 40
    x = edge_value_input(stream, cin)
    program = conv_program(stream, cin, 72, (3, 3), (1, 1), (1, 1, 1, 1), bits)
    assert_parity(program, [x], oracle, f"edge values w{bits[0]}a{bits[1]}")
    program = conv_program(stream, cin, 72, (1, 1), (1, 1), (0, 0, 0, 0), bits)
    assert_parity(program, [x], oracle, f"edge values pointwise w{bits[0]}a{bits[1]}")


@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
def test_receptive_field_edge_values(cuda, oracle, bits, half):
    """The few-channel path (whole receptive field per staged record): NaN and
    inf in a field, all-zero fields, subnormal and huge maxima, ties."""
    stream = SeededStream(6)
    x = np.ascontiguousarray(edge_value_input(stream, 9)[[0, 3, 7, 8]])
    if half:
        x = x.astype(np.float16).astype(np.float32)
    for kernel, stride, pads in (((3, 3), (1, 1), (1, 1, 1, 1)), ((3, 3), (2, 2), (0, 1, 1, 0))):
        program = conv_program(stream, 4, 40, kernel, stride, pads, bits)
        label = f"fields {kernel} s{stride[0]} w{bits[0]}a{bits[1]}"
        if half:
            assert_half_parity(program, [x], oracle, label)
        else:
            assert_parity(program, [x], oracle, label)


@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
@pytest.mark.parametrize("cin,h,w", [(40, 8, 16), (96, 12, 20), (200, 8, 8), (64, 3, 136)])
def test_wide_record_staging(cuda, oracle, half, cin, h, w):
    """Wide-record staging (48..208 padded channels: one or several channel
    slabs, full and ragged last pixel blocks) with NaN, inf, huge and
    subnormal values in the planes; the pixel maxima come from integer maxima
    of the |x| bit patterns."""
    stream = SeededStream(7000 + cin + h)
    x = stream.tensor(cin, h, w, 2.0)
    x[cin // 3, 0, 3] = np.nan
    x[cin - 1, h - 1, w - 1] = np.inf
    x[cin // 2, h // 2, :] = np.float32(60000.0)
    x[:, 1, 5] *= np.float32(2.0 ** -20)
    program = conv_program(stream, cin, 48, (3, 3), (1, 1), (1, 1, 1, 1), (8, 8))
    if half:
        assert_half_parity(program, [x], oracle, f"wide staging half {cin}x{h}x{w}")
    else:
        assert_parity(program, [x], oracle, f"wide staging {cin}x{h}x{w}")


@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
def test_staged_intermediates(cuda, oracle, bits, half):
    """Chains whose intermediates skip the staging prepass, with NaN, inf and
    all-zero positions propagating through the staged maxima."""
    stream = SeededStream(8100)
    program = staged_chain_program(stream, bits)
    x = stream.tensor(24, 19, 37, 2.0)
    x[3, 4, 5] = np.nan
    x[7, 10, 20] = np.inf
    x[:, 15, 30] = 0.0
    if half:
        assert_half_parity(program, [x], oracle, f"staged chain half w{bits[0]}a{bits[1]}")
    else:
        assert_parity(program, [x], oracle, f"staged chain w{bits[0]}a{bits[1]}")


@pytest.mark.parametrize("bits", [(8, 8), (16, 16)], ids=["w8a8", "w16a16"])
@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
@pytest.mark.parametrize("channels", [120, 250])
def test_staged_depthwise(cuda, oracle, bits, half, channels):
    """The channel-innermost depthwise between integer convs (128 and 256 padded
    channels, ragged real counts), with NaN, inf and zero inputs."""
    stream = SeededStream(8200 + channels)
    program = staged_depthwise_program(stream, channels, bits)
    x = stream.tensor(24, 17, 29, 2.0)
    x[3, 4, 5] = np.nan
    x[7, 10, 20] = np.inf
    x[:, 15, 28] = 0.0
    label = f"staged depthwise {channels} w{bits[0]}a{bits[1]}"
    if half:
        assert_half_parity(program, [x], oracle, label + " half")
    else:
        assert_parity(program, [x], oracle, label)


def test_weight_edge_values(cuda, oracle):
    """A zero weight row (scale 1), FP16-subnormal weights, +-65504 weights."""
    stream = SeededStream(9)
    p = Program(name="weights")
    x = p.add_input("x", 48)
    w = stream.uniform(-1, 1, 32 * 48).reshape(32, 48)
    w[0] = 0.0
    w[1] = np.float32(2.0 ** -24) * np.arange(48)
    w[2, :5] = [65504.0, -65504.0, 1.0, -1.0, 0.5]
    b = stream.uniform(-1, 1, 32)
    y = p.conv(x, 32, w, b, "y", bits=(16, 16))
    p.finish([y])
    xs = stream.tensor(48, 9, 9, 4.0)
    for bits in WIDTHS:
        assert_parity(p.with_widths(*bits), [xs], oracle, f"weight edges w{bits[0]}a{bits[1]}", fp16_weights=True)


def test_bit_stable_repeats(cuda, oracle):
    """Sixty runs of one executor give identical bits (no scheduling-dependent results)."""
    stream = SeededStream(3)
    program = op_program(stream).with_widths(16, 16)
    x = stream.tensor(70, 33, 47, 3.0)
    with CudaExecutor.from_program(program) as executor:
        first = executor.run([x])
        for _ in range(59):
            again = executor.run([x])
            assert all(same_bits(a, b) for a, b in zip(first, again))


def test_one_executor_many_extents(cuda, oracle):
    """Plans are cached per input extent; alternating extents reuse them."""
    stream = SeededStream(4)
    program = op_program(stream).with_widths(8, 16)
    xs = [stream.tensor(70, h, w, 2.0) for h, w in [(11, 18), (33, 47), (11, 18), (5, 200)]]
    with CudaExecutor.from_program(program) as executor:
        for x in xs:
            got = executor.run([x])
            expected = oracle.run(program, [x])
            assert all(count_differing(g, e) == 0 for g, e in zip(got, expected))


@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
def test_many_tiles_per_cta(cuda, oracle, bits):
    """More tiles than SMs, so each persistent CTA walks several tiles and every
    ring (halo, A, B, TMEM, per-tile info) wraps around many times."""
    stream = SeededStream(90)
    program = conv_program(stream, 64, 64, (3, 3), (1, 1), (1, 1, 1, 1), bits)
    x = stream.tensor(64, 288, 288, 2.0)  # 648 tiles: four or five per CTA
    assert_parity(program, [x], oracle, f"many tiles w{bits[0]}a{bits[1]}")


def test_many_tiles_with_fusions_and_groups(cuda, oracle):
    """Several channel groups per tile (C = 256), chunk-add and residual, many tiles."""
    stream = SeededStream(91)
    program = conv_program(stream, 256, 128, (3, 3), (1, 1), (1, 1, 1, 1), (16, 16), chunk_add=True, residual=True)
    x = stream.tensor(256, 96, 224, 2.0)  # 168 tiles of 128 positions
    assert_parity(program, [x], oracle, "many tiles, groups, fusions")


def run_half_gpu(program: Program, inputs):
    """FP16 device tensors in and out (run_half): integer convs stage FP16
    program inputs directly and store outputs nothing else reads directly."""
    import torch

    with CudaExecutor.from_program(program) as executor:
        extents = executor.infer_output_extents([x.shape for x in inputs])
        ins = {name: torch.from_numpy(x.astype(np.float16)).cuda() for name, x in zip(executor.input_names, inputs)}
        outs = {name: torch.empty(tuple(e), dtype=torch.float16, device="cuda")
                for name, e in zip(executor.output_names, extents)}
        executor.run_half(ins, outs)
        executor.synchronize()
        return [outs[name].float().cpu().numpy() for name in executor.output_names]


def assert_half_parity(program, inputs, oracle, label):
    rounded = [x.astype(np.float16).astype(np.float32) for x in inputs]
    expected = [e.astype(np.float16).astype(np.float32) for e in oracle.run(program, rounded)]
    got = run_half_gpu(program, inputs)
    for index, (g, e) in enumerate(zip(got, expected)):
        assert g.shape == e.shape, f"{label} output {index}: shape {g.shape} != {e.shape}"
        bad = count_differing(g, e)
        assert bad == 0, f"{label} output {index}: {bad} of {e.size} elements differ"


@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: f"{c[0]}to{c[1]}k{c[2][0]}x{c[2][1]}s{c[3][0]}")
@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
def test_integer_conv_half(cuda, oracle, case, bits):
    """The FP16 source path: channel counts 3..200 cover every halo record
    width (16-128 bytes, each swizzle) for FP16 sources, as the FP32 runs do
    for FP32 sources."""
    cin, cout, kernel, stride, pads, h, w = case
    stream = SeededStream(2000 + cin + cout)
    program = conv_program(stream, cin, cout, kernel, stride, pads, bits)
    x = stream.tensor(cin, h, w, 2.0)
    assert_half_parity(program, [x], oracle, f"half conv {case} w{bits[0]}a{bits[1]}")


def clamp_and_tiny_input(stream: SeededStream, cin: int, h: int, w: int) -> np.ndarray:
    """FP16-exact values: maxima whose scaled value rounds past 127 (the clamp
    path: 127.5 and 127.75 times a power of two), maxima below 2^-8 (exponents
    under -15, so no FP16 scale), FP16 subnormals, and ordinary positions."""
    x = stream.tensor(cin, h, w, 1.0).astype(np.float16).astype(np.float32)
    x[0, 0, :] = 127.75
    x[1, 1, :] = -127.5
    x[2, 2, :] = np.float32(127.75 * 2.0 ** -6)
    x[:, 3, :] *= np.float32(2.0 ** -12)
    x[:, 4, :] = np.float32(2.0 ** -24) * (np.arange(cin, dtype=np.float32)[:, None] - cin / 2)
    x[5 % cin, 5, 3:9] = -np.float32(127.5 * 2.0 ** 3)
    return x.astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
def test_quantisation_modes(cuda, oracle, bits, half):
    """Positions on the clamp path, below the FP16-scale range and on the
    paired-FP16 path, in one tile (a warp takes several paths at once)."""
    stream = SeededStream(31)
    cin = 24
    x = clamp_and_tiny_input(stream, cin, 8, 40)
    for kernel, pads in (((3, 3), (1, 1, 1, 1)), ((1, 1), (0, 0, 0, 0))):
        program = conv_program(stream, cin, 40, kernel, (1, 1), pads, bits)
        if half:
            assert_half_parity(program, [x], oracle, f"modes half {kernel} w{bits[0]}a{bits[1]}")
        else:
            assert_parity(program, [x], oracle, f"modes {kernel} w{bits[0]}a{bits[1]}")


def d2s_program(stream: SeededStream, cin, cout, block, bits) -> Program:
    p = Program(name="conv_d2s")
    x = p.add_input("x", cin)
    w = stream.uniform(-0.5, 0.5, cout * cin * 9)
    b = stream.uniform(-0.2, 0.2, cout)
    y = p.dense_conv(x, cout, w, b, "c", kernel=(3, 3), stride=(1, 1), pads=(1, 1, 1, 1), bits=bits)
    z = p.unary(OpKind.depth_to_space, y, "z", block=block)
    return p.finish([z])


@pytest.mark.parametrize("block", [2, 3])
@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
def test_depth_to_space_fold(cuda, oracle, block, half):
    """conv -> depth_to_space folds into the conv's store (config-2 L5's shape, smaller)."""
    stream = SeededStream(40 + block)
    program = d2s_program(stream, 32, 36 * block, block, (8, 8))
    x = stream.tensor(32, 19, 45, 2.0)
    if half:
        assert_half_parity(program, [x], oracle, f"d2s {block} half")
    else:
        assert_parity(program, [x], oracle, f"d2s {block}")


def test_half_input_shared_with_other_ops(cuda, oracle):
    """An FP16 program input read by a conv and by a generic op, and a conv
    output that a later op reads: the conv stages the caller's FP16 buffer, the
    other readers see the converted FP32 copy, the read output goes through
    the arena."""
    stream = SeededStream(44)
    p = Program(name="shared")
    x = p.add_input("x", 48)
    y = p.dense_conv(x, 48, stream.uniform(-0.5, 0.5, 48 * 48 * 9), stream.uniform(-0.2, 0.2, 48), "y",
                     bits=(8, 8))
    s = p.binary(OpKind.add, y, x, "s")
    p.finish([s, y])
    xs = stream.tensor(48, 21, 37, 2.0)
    assert_half_parity(p, [xs], oracle, "shared input")


@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
def test_many_tiles_pointwise_and_strided(cuda, oracle, half):
    """Several tiles per CTA on the pointwise and stride-2 shapes of config 2
    (L1, L3), so every ring and the per-tile info buffers wrap many times."""
    stream = SeededStream(92)
    for cin, cout, kernel, stride, pads, h, w in ((3, 64, (3, 3), (2, 2), (1, 1, 1, 1), 260, 300),
                                                  (128, 256, (1, 1), (1, 1), (0, 0, 0, 0), 72, 200)):
        program = conv_program(stream, cin, cout, kernel, stride, pads, (8, 8))
        x = stream.tensor(cin, h, w, 2.0)
        if half:
            assert_half_parity(program, [x], oracle, f"many tiles {cin}->{cout} half")
        else:
            assert_parity(program, [x], oracle, f"many tiles {cin}->{cout}")


@pytest.mark.parametrize("bits", [(8, 8), (16, 16)], ids=["w8a8", "w16a16"])
def test_intra_decoder_stack(cuda, oracle, bits):
    """BASELINE config 3's stack (synthetic DCVC-RT intra decoder: subpel
    upsample, 14 DepthConvBlocks with WSiLU, depthwise 3x3, residuals and
    chunk-add, a depth_to_space(8) head) on a small latent; every block's output
    is compared bit for bit. w8a8 is BASELINE's; w16a16 is the reference width
    map's default for the decoder layers."""
    from nvcr_b200.workloads import intra_decoder, laplace_latent

    stack = intra_decoder((3, 5), bits=bits, every_tensor=True)
    y_hat = laplace_latent(SeededStream(7), stack.input_shapes[0])
    assert_parity(stack.program, [y_hat], oracle, f"intra decoder {bits}")


def test_intra_decoder_stack_half(cuda, oracle):
    """The same stack through run_half (FP16 latent in, FP16 tensors out)."""
    from nvcr_b200.workloads import intra_decoder, laplace_latent

    stack = intra_decoder((4, 6), every_tensor=True)
    y_hat = laplace_latent(SeededStream(8), stack.input_shapes[0])
    assert_half_parity(stack.program, [y_hat], oracle, "intra decoder half")


def chained_convs_program(stream: SeededStream, bits) -> Program:
    """Integer convs feeding integer convs: the producer's epilogue writes the
    consumer's staged source (64 and 32 channels), including through chunk-add
    and a residual; a 40-channel source (not a multiple of 16) is staged by the
    prepass instead."""
    p = Program(name="chained")
    x = p.add_input("x", 48)

    def w(cout, cin, taps):
        return stream.uniform(-0.3, 0.3, cout * cin * taps), stream.uniform(-0.1, 0.1, cout)

    a = p.dense_conv(x, 64, *w(64, 48, 9), "a", bits=bits)
    b = p.conv(a, 128, *w(128, 64, 1), "b", bits=bits)
    lo = p.unary(OpKind.slice_channels, b, "b.lo", begin=0, end=64)
    hi = p.unary(OpKind.slice_channels, b, "b.hi", begin=64, end=128)
    c = p.binary(OpKind.add, lo, hi, "c")
    d = p.conv(c, 32, *w(32, 64, 1), "d", bits=bits)
    e = p.binary(OpKind.add, d, p.unary(OpKind.slice_channels, c, "c32", begin=0, end=32), "e")
    f = p.conv(e, 40, *w(40, 32, 1), "f", bits=bits)
    g = p.dense_conv(f, 16, *w(16, 40, 9), "g", bits=bits)
    return p.finish([g, c])


@pytest.mark.parametrize("bits", WIDTHS, ids=lambda b: f"w{b[0]}a{b[1]}")
@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
def test_chained_integer_convs(cuda, oracle, bits, half):
    stream = SeededStream(55)
    program = chained_convs_program(stream, bits)
    x = stream.tensor(48, 37, 70, 2.0)
    if half:
        assert_half_parity(program, [x], oracle, f"chained w{bits[0]}a{bits[1]} half")
    else:
        assert_parity(program, [x], oracle, f"chained w{bits[0]}a{bits[1]}")


def test_p_frame_sequence(cuda, oracle):
    """BASELINE config 4's shape of work, small: an I-frame (intra decoder with a
    feature output) then P-frames whose temporal context is the previous frame's
    feature, each P-frame's every block output compared; one executor per mode
    reused across frames (its plans and scratch stay)."""
    from nvcr_b200.workloads import inter_decoder, intra_decoder, laplace_latent

    intra = intra_decoder((3, 5), feature_channels=64)
    inter = inter_decoder((3, 5), every_tensor=True)
    latents = [laplace_latent(SeededStream(60 + f), (256, 3, 5)) for f in range(4)]
    with CudaExecutor.from_program(intra.program) as first, CudaExecutor.from_program(inter.program) as rest:
        got = first.run([latents[0]])
        want = oracle.run(intra.program, [latents[0]])
        assert all(count_differing(g, e) == 0 for g, e in zip(got, want))
        context_got, context_want = got[-1], want[-1]
        for f in range(1, 4):
            got = rest.run([latents[f], context_got])
            want = oracle.run(inter.program, [latents[f], context_want])
            for index, (g, e) in enumerate(zip(got, want)):
                assert count_differing(g, e) == 0, f"P-frame {f} output {index}"
            context_got, context_want = got[-1], want[-1]


def test_p_frame_sequence_half(cuda, oracle):
    """The same through run_half: the feature crosses each stage boundary in FP16."""
    from nvcr_b200.workloads import inter_decoder, laplace_latent

    inter = inter_decoder((4, 6), every_tensor=True)
    stream = SeededStream(70)
    context = stream.tensor(64, 8, 12, 2.0).astype(np.float16).astype(np.float32)
    for f in range(2):
        latent = laplace_latent(SeededStream(80 + f), (256, 4, 6))
        assert_half_parity(inter.program, [latent, context], oracle, f"P-frame {f} half")
        context = run_half_gpu(inter.program, [latent, context])[-1]


def test_graph_replay_half(cuda, oracle):
    """Device-boundary runs are captured into a CUDA graph on the second call with
    the same plan and tensors and replayed after: new contents in the same
    buffers must give new, bit-exact outputs on every call."""
    import torch

    stream = SeededStream(88)
    program = conv_program(stream, 64, 96, (3, 3), (1, 1), (1, 1, 1, 1), (8, 8), wsilu=True)
    with CudaExecutor.from_program(program) as executor:
        (c, h, w), = executor.infer_output_extents([(64, 21, 50)])
        xh = torch.empty((64, 21, 50), dtype=torch.float16, device="cuda")
        yh = torch.empty((c, h, w), dtype=torch.float16, device="cuda")
        for call in range(5):
            x = stream.tensor(64, 21, 50, 2.0).astype(np.float16)
            xh.copy_(torch.from_numpy(x))
            executor.run_half({"x": xh}, {executor.output_names[0]: yh})
            executor.synchronize()
            expected = oracle.run(program, [x.astype(np.float32)])[0].astype(np.float16).astype(np.float32)
            assert count_differing(yh.float().cpu().numpy(), expected) == 0, f"call {call}"


def test_sigmoid_reciprocal_exhaustive(cuda):
    """The sigmoid's 1 / (1 + exp(-x)) takes a refined hardware reciprocal for
    denominators in [1, 2^126): every float there gives the IEEE division's bits."""
    first, end = 0x3F800000, 0x7E800000  # 1.0 and 2^126
    assert reciprocal_mismatches(first, end - first) == 0


def test_fallback_in_captured_runs(cuda, oracle):
    """A w8a8 3x3 conv run repeatedly on the same device tensors: the first run
    is launched directly, later ones are captured into a CUDA graph and
    replayed, where the quantise-on-load fallback is a conditional node that the
    conv sets only when a window mixes exponents. Inputs alternate between
    windows that never mix (every pixel's largest value is 100) and windows
    that do (some pixels scaled down), so replays must both skip and take the
    fallback, and every run must equal the oracle."""
    import torch

    stream = SeededStream(95)
    program = conv_program(stream, 64, 64, (3, 3), (1, 1), (1, 1, 1, 1), (8, 8))
    base = np.clip(np.rint(stream.tensor(64, 40, 72, 30.0)), -50, 50).astype(np.float32)
    base[0] = 100.0  # one channel sets every pixel's maximum: one exponent everywhere
    mixed = base.copy()
    mixed[:, 5:9, 10:13] *= 0.125  # pixels whose exponent is lower by three
    mixed[:, 30, 60] *= 0.25
    with CudaExecutor.from_program(program) as executor:
        (c, h, w), = executor.infer_output_extents([base.shape])
        xh = torch.empty(base.shape, dtype=torch.float16, device=cuda)
        yh = torch.empty((c, h, w), dtype=torch.float16, device=cuda)
        for run, x in enumerate([base, mixed, base, mixed, mixed, base, mixed]):
            xh.copy_(torch.from_numpy(x.astype(np.float16)))
            yh.fill_(float("nan"))
            executor.run_half({executor.input_names[0]: xh}, {executor.output_names[0]: yh})
            executor.synchronize()
            expected = oracle.run(program, [x])[0].astype(np.float16).astype(np.float32)
            bad = count_differing(yh.float().cpu().numpy(), expected)
            assert bad == 0, f"run {run}: {bad} of {expected.size} values differ"


@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
@pytest.mark.parametrize("width", [64, 50, 72])
@pytest.mark.parametrize("stride", [1, 2])
def test_three_channel_fields(cuda, oracle, half, width, stride):
    """The compile-time receptive-field prepass (3 channels, 3x3 windows, w8a8):
    widths that allow 16-byte row loads (64, 72) and one that does not (50),
    rows and columns past the image, and positions whose fields are all zero,
    non-finite, subnormal, huge or on rounding ties (the general quantisation)."""
    stream = SeededStream(97 + width + stride)
    x = np.ascontiguousarray(np.tile(edge_value_input(stream, 9)[[0, 3, 7]], (1, 3, 2))[:, :17, :width])
    x[:, 9:, :] = np.rint(stream.tensor(3, 8, width, 60.0))  # ordinary values: the one-fma path
    if half:
        x = x.astype(np.float16).astype(np.float32)
    program = conv_program(stream, 3, 40, (3, 3), (stride, stride), (1, 1, 1, 1), (8, 8))
    label = f"3-channel fields w{width} s{stride}"
    if half:
        assert_half_parity(program, [x], oracle, label)
    else:
        assert_parity(program, [x], oracle, label)


@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
@pytest.mark.parametrize("shape", [(128, 256, 33, 47, None), (256, 256, 12, 90, None), (128, 512, 9, 200, None),
                                   (128, 512, 20, 45, 2)],
                         ids=["128to256", "256to256", "two_n_tiles", "d2s"])
def test_paired_tiles(cuda, oracle, half, shape):
    """Deep-K w8a8 3x3 convs with 128-byte K blocks and few tiles: the planner
    pairs two patches per tile, sharing each weight block between two
    accumulators. Ragged patch counts leave the last pair half empty; the
    inputs mix magnitudes (mixed windows: the fallback writes those
    positions), zeros and non-finite values."""
    cin, cout, h, w, block = shape
    stream = SeededStream(300 + cin + cout + h)
    program = d2s_program(stream, cin, cout, block, (8, 8)) if block else \
        conv_program(stream, cin, cout, (3, 3), (1, 1), (1, 1, 1, 1), (8, 8))
    x = stream.tensor(cin, h, w, 2.0)
    x[:, h // 3, :] *= np.float32(0.01)   # rows of much smaller pixels: mixed windows around them
    x[:, :, 5] = 0.0                      # an all-zero column
    x[3, 2, 7] = np.inf                   # one non-finite pixel: NaN rows around it
    label = f"paired {cin}->{cout} {h}x{w}"
    if half:
        assert_half_parity(program, [x], oracle, label)
    else:
        assert_parity(program, [x], oracle, label)


def uniform_window_input(stream: SeededStream, cin: int, h: int, w: int) -> np.ndarray:
    """Values in +-100 with channel 0 at 120 at every pixel, so each pixel's
    max is 120 and its exponent that of its block's scale: blocks of 8 rows x
    32 columns scaled by 2^k for k from -24 to 9 (FP16-representable), so
    every window inside a block has one exponent (the direct conv's result)
    and windows across a block edge mix exponents (the fallback's)."""
    x = stream.tensor(cin, h, w, 100.0)
    x[0] = 120.0
    rows, cols = np.meshgrid(np.arange(h), np.arange(w), indexing="ij")
    exponents = ((rows // 8) * 17 + (cols // 32) * 5) % 34 - 24
    return (x * np.ldexp(np.float32(1.0), exponents).astype(np.float32)[None, :, :]).astype(np.float32)


@pytest.mark.parametrize("weight_scale", [1.0, 2.0 ** -100], ids=["ordinary", "tiny_weights"])
@pytest.mark.parametrize("shape", [(16, 72, (3, 3), 21, 64), (64, 64, (3, 3), 19, 48), (128, 256, (1, 1), 13, 56),
                                   (256, 256, (3, 3), 12, 96)],
                         ids=["small_acc", "wide_acc", "pointwise", "paired"])
def test_vector_stores(cuda, oracle, shape, weight_scale):
    """FP16 outputs of the direct conv written as 16-byte runs of one channel
    (widths multiples of 8) over inputs whose windows mostly share one
    exponent: accumulators below 2^22 (converted by integer addition) and
    above it, window exponents from -24 to 9, a channel count that is not a
    multiple of 16, patches past the bottom and right edges, paired patches,
    and, with tiny weights (scales near 2^-108), window exponents outside the
    range where the power-of-two scale and the bias add fuse exactly, which
    the per-channel stores take."""
    cin, cout, kernel, h, w = shape
    stream = SeededStream(700 + cin + cout + h)
    p = Program(name="vector")
    x_in = p.add_input("x", cin)
    weights = stream.uniform(-0.5, 0.5, cout * cin * kernel[0] * kernel[1]) * np.float32(weight_scale)
    bias = stream.uniform(-0.2, 0.2, cout)
    pads = (1, 1, 1, 1) if kernel == (3, 3) else (0, 0, 0, 0)
    y = p.dense_conv(x_in, cout, weights.astype(np.float32), bias, "c", kernel=kernel, stride=(1, 1), pads=pads,
                     bits=(8, 8))
    program = p.finish([y])
    x = uniform_window_input(stream, cin, h, w)
    assert_half_parity(program, [x], oracle, f"vector stores {shape} x{weight_scale}")


@pytest.mark.parametrize("half", [False, True], ids=["f32", "f16"])
@pytest.mark.parametrize("shape", [(128, 256, 9, 120, None), (256, 256, 7, 240, None), (128, 128, 5, 256, None),
                                   (128, 64, 11, 250, None), (256, 512, 6, 120, 2), (128, 256, 3, 360, None),
                                   (64, 64, 10, 240, None), (64, 96, 9, 120, None), (192, 64, 5, 128, None),
                                   (40, 48, 6, 128, None)],
                         ids=["120", "240", "256", "250_narrow_n", "d2s", "360_three_patches", "k64_240",
                              "k64_ragged_n", "k64_three_blocks", "k64_40_channels"])
def test_row_halos(cuda, oracle, half, shape):
    """Row-halo direct convs: 3x3 windows over 128-byte channel blocks on
    widths within 1/8 of a multiple of 128, whose patches are single output
    rows of 128 positions and whose A stages are one input row of 130 pixels
    read by three K blocks starting 0, 1 and 2 rows in (64-byte channel blocks,
    the k64 cases, take per-tap boxes on the same widths). The inputs' windows
    mostly share one exponent (the direct conv's results) with block edges
    that mix exponents (the fallback's), an all-zero column and one non-finite
    pixel; patches past the right edge, one to three patches per row, one and
    two N tiles, one to three channel blocks and a depth_to_space output."""
    cin, cout, h, w, block = shape
    stream = SeededStream(900 + cin + cout + w)
    program = d2s_program(stream, cin, cout, block, (8, 8)) if block else \
        conv_program(stream, cin, cout, (3, 3), (1, 1), (1, 1, 1, 1), (8, 8))
    x = uniform_window_input(stream, cin, h, w)
    x[:, :, 7] = 0.0
    x[5, 1, 11] = np.inf
    label = f"row halos {cin}->{cout} {h}x{w}"
    if half:
        assert_half_parity(program, [x], oracle, label)
    else:
        assert_parity(program, [x], oracle, label)
