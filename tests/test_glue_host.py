"""DCVC-RT inter-stage glue (no GPU): the element functions the kernels in
nvcr_b200/csrc/k_glue.cu run, compiled for the host (tests/glue_host.cpp),
bit for bit against the reference's own host ops (src/dcvcrt/host_ops.cpp and
scale_index.hpp, compiled from its sources into oracle/_ref): the FP16
conversions on every half and on every rounding boundary, the exact
scale-to-table index on every threshold and its neighbours, the decode and
encode index builds on every half scale, the four- and two-way masks on every
stage, and the restore on seeded halves with specials; the generated threshold
table against the reference's. FP16 outputs are compared bit for bit, with NaN
equal to NaN: the sign and payload of a NaN that arithmetic makes from two NaN
operands depend on the instruction's operand order on x86 and are canonical on
the GPU, and the library leaves them unspecified, as it does for the conv."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def ptr(array: np.ndarray):
    return array.ctypes.data_as(ctypes.c_void_p)


def same_halves(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit-identical FP16 patterns, any NaN equal to any NaN."""
    a = np.asarray(a).view(np.uint16)
    b = np.asarray(b).view(np.uint16)
    nan_a = (a & 0x7c00) == 0x7c00
    nan_a &= (a & 0x03ff) != 0
    nan_b = (b & 0x7c00) == 0x7c00
    nan_b &= (b & 0x03ff) != 0
    return bool(np.array_equal(nan_a, nan_b) and np.array_equal(a[~nan_a], b[~nan_b]))


@pytest.fixture(scope="module")
def sides(reference):
    from tests.glue_host import load

    mine = load()
    theirs = reference.lib
    for lib, prefix in ((mine, "gh"), (theirs, "ref_glue")):
        for name in ("to_half", "to_float", "exact_scale_indexes"):
            getattr(lib, f"{prefix}_{name}").restype = None
            getattr(lib, f"{prefix}_{name}").argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        getattr(lib, f"{prefix}_decode_indexes").argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                                             ctypes.c_float]
        getattr(lib, f"{prefix}_encode_indexes").argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                             ctypes.c_size_t, ctypes.c_float]
    mine.gh_mask.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 6
    theirs.ref_glue_mask.argtypes = [ctypes.c_void_p, ctypes.c_size_t] + [ctypes.c_int] * 6
    mine.gh_restore.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5
    mine.gh_process.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_size_t, ctypes.c_float]
    theirs.ref_glue_process.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_size_t, ctypes.c_float]
    mine.gh_reduce.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5
    theirs.ref_glue_reduce.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_size_t] + [ctypes.c_int] * 5
    theirs.ref_glue_restore.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_size_t] + [ctypes.c_int] * 5
    return mine, theirs


def test_generated_thresholds_equal_the_reference_table():
    """nvcr_b200/csrc/make_scale_thresholds.py derives the table from its
    definition; the reference ships it as constants (read here as text)."""
    from oracle.oracle import REFERENCE_SOURCES

    header = REFERENCE_SOURCES / "src" / "dcvcrt" / "scale_index.hpp"
    if not header.exists():
        pytest.skip("reference sources not present")
    ref = re.findall(r"(0x[0-9a-f.]+p[+-]?\d+)F", header.read_text())
    mine = [line.strip().rstrip("f,") for line in (ROOT / "nvcr_b200" / "csrc" / "scale_thresholds.inc").read_text()
            .splitlines() if line.startswith("0x")]
    assert len(mine) == 127 and [float.fromhex(v) for v in mine] == [float.fromhex(v) for v in ref]


def test_half_to_float_every_pattern(sides):
    mine, theirs = sides
    halves = np.arange(65536, dtype=np.uint16)
    a = np.zeros(65536, np.float32)
    b = np.zeros(65536, np.float32)
    mine.gh_to_float(ptr(halves), ptr(a), 65536)
    theirs.ref_glue_to_float(ptr(halves), ptr(b), 65536)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_float_to_half_on_every_boundary(sides):
    mine, theirs = sides
    halves = np.arange(0, 0x7c01, dtype=np.uint32)  # every finite magnitude and infinity
    as_float = np.zeros(halves.size, np.float32)
    mine.gh_to_float(ptr(halves.astype(np.uint16)), ptr(as_float), halves.size)
    bits = as_float.view(np.uint32)
    # each half, the midpoints to its neighbours and one float ulp either side of them
    midpoints = ((as_float[:-1].astype(np.float64) + as_float[1:].astype(np.float64)) / 2).astype(np.float32)
    mid_bits = midpoints.view(np.uint32)
    candidates = np.concatenate([bits, bits + 1, bits - 1, mid_bits, mid_bits + 1, mid_bits - 1,
                                 np.array([0x7f800000, 0x7fc00000, 0x7f800001, 0x477fefff, 0x477ff000, 0x477ff001,
                                           0x33000000, 0x33000001, 0x32ffffff, 0x38800000, 0x387fffff],
                                          np.uint32)])
    rng = np.random.default_rng(3)
    candidates = np.concatenate([candidates, rng.integers(0, 2 ** 31, 200000, dtype=np.uint32)])
    candidates = np.concatenate([candidates, candidates | np.uint32(0x80000000)]).astype(np.uint32)
    values = candidates.view(np.float32)
    a = np.zeros(values.size, np.uint16)
    b = np.zeros(values.size, np.uint16)
    mine.gh_to_half(ptr(values), ptr(a), values.size)
    theirs.ref_glue_to_half(ptr(values), ptr(b), values.size)
    assert np.array_equal(a, b)


def test_exact_scale_index_on_every_threshold(sides):
    mine, theirs = sides
    thresholds = np.array([float.fromhex(line.strip().rstrip("f,")) for line in
                           (ROOT / "nvcr_b200" / "csrc" / "scale_thresholds.inc").read_text().splitlines()
                           if line.startswith("0x")], np.float32)
    bits = thresholds.view(np.uint32)
    specials = np.array([0.0, -0.0, -1.0, 0.11, 0.10999999, 16.0, 16.000002, 1e30, np.inf, -np.inf, np.nan],
                        np.float32)
    rng = np.random.default_rng(4)
    scales = np.concatenate([thresholds, (bits + 1).view(np.float32), (bits - 1).view(np.float32), specials,
                             rng.uniform(0.05, 20.0, 100000).astype(np.float32)]).astype(np.float32)
    a = np.zeros(scales.size, np.uint8)
    b = np.zeros(scales.size, np.uint8)
    mine.gh_exact_scale_indexes(ptr(scales), ptr(a), scales.size)
    theirs.ref_glue_exact_scale_indexes(ptr(scales), ptr(b), scales.size)
    assert np.array_equal(a, b)
    assert set(a.tolist()) == set(range(128))


@pytest.mark.parametrize("force_zero", [0.0, 0.11, 0.5, -1.0])
def test_index_builds_on_every_half_scale(sides, force_zero):
    mine, theirs = sides
    scales = np.arange(65536, dtype=np.uint16)
    a = np.zeros(65536, np.uint8)
    b = np.zeros(65536, np.uint8)
    assert mine.gh_decode_indexes(ptr(scales), ptr(a), 65536, force_zero) == 1
    assert theirs.ref_glue_decode_indexes(ptr(scales), ptr(b), 65536, force_zero) == 1
    assert np.array_equal(a, b)
    rng = np.random.default_rng(5)
    symbol_halves = np.zeros(65536, np.uint16)
    values = rng.integers(-128, 128, 65536).astype(np.float32)
    mine.gh_to_half(ptr(values), ptr(symbol_halves), 65536)  # symbols: integers in [-128, 127] as FP16
    ea = np.zeros(65536, np.int16)
    eb = np.zeros(65536, np.int16)
    assert mine.gh_encode_indexes(ptr(symbol_halves), ptr(scales), ptr(ea), 65536, force_zero) == 1
    assert theirs.ref_glue_encode_indexes(ptr(symbol_halves), ptr(scales), ptr(eb), 65536, force_zero) == 1
    assert np.array_equal(ea, eb)


def test_masks_on_every_stage(sides):
    mine, theirs = sides
    for ways in (4, 2):
        for batch, channels, height, width in ((1, 4, 1, 1), (1, 8, 3, 5), (2, 12, 4, 4), (1, 4, 7, 2), (2, 2, 2, 3)):
            for stage in range(-1, ways + 1):
                count = batch * channels * height * width
                a = np.full(count, 0x1234, np.uint16)
                b = np.full(count, 0x1234, np.uint16)
                ok_a = mine.gh_mask(ptr(a), batch, channels, height, width, ways, stage)
                ok_b = theirs.ref_glue_mask(ptr(b), count, batch, channels, height, width, ways, stage)
                assert ok_a == ok_b, (ways, batch, channels, height, width, stage)
                if ok_a:
                    assert np.array_equal(a, b)
    for shape in ((0, 4, 2, 2), (1, 6, 2, 2), (1, 4, 0, 2), (1, 4, 2, -1)):
        a = np.zeros(64, np.uint16)
        assert mine.gh_mask(ptr(a), *shape, 4, 0) == theirs.ref_glue_mask(ptr(a), 64, *shape, 4, 0) == 0


def test_restore_on_seeded_halves(sides):
    mine, theirs = sides
    rng = np.random.default_rng(6)
    specials = np.array([0x7c00, 0xfc00, 0x7e00, 0x7c01, 0x0000, 0x8000, 0x0001, 0x7bff, 0xfbff, 0x3c00], np.uint16)
    for ways in (4, 2):
        for batch, channels, height, width in ((1, 4, 2, 3), (2, 8, 5, 5), (1, 12, 1, 7)):
            count = batch * channels * height * width
            part = count // ways
            symbols = rng.integers(0, 65536, part, dtype=np.uint16)
            means = rng.integers(0, 65536, count, dtype=np.uint16)
            mask = rng.choice(np.array([0x0000, 0x3c00], np.uint16), count)
            symbols[: min(part, specials.size)] = specials[: min(part, specials.size)]
            means[: specials.size] = specials[::-1]
            a = np.zeros(count, np.uint16)
            b = np.zeros(count, np.uint16)
            assert mine.gh_restore(ptr(symbols), ptr(means), ptr(mask), ptr(a), batch, channels, height, width,
                                   ways) == 1
            assert theirs.ref_glue_restore(ptr(symbols), ptr(means), ptr(mask), ptr(b), count, batch, channels,
                                           height, width, ways) == 1
            assert same_halves(a, b)


def random_halves(rng, count: int) -> np.ndarray:
    """Seeded FP16 patterns: mostly moderate values, with specials mixed in."""
    values = rng.normal(0.0, 40.0, count).astype(np.float16).view(np.uint16)
    specials = np.array([0x7c00, 0xfc00, 0x7e00, 0xfe00, 0x7c01, 0xfc01, 0x7d55, 0xfdff, 0x7fff, 0x0000, 0x8000,
                         0x0001, 0x8001, 0x03ff, 0x7bff, 0xfbff, 0x3800, 0xb800, 0x3e00, 0xbe00], np.uint16)
    values[rng.integers(0, count, count // 20)] = rng.choice(specials, count // 20)
    return values


@pytest.mark.parametrize("force_zero", [0.0, 0.11, 2.0])
def test_process_with_mask(sides, force_zero):
    """Ties of the rounding (x.5 residuals), the clamp at -128 / 127, NaN and
    infinities, with and without the residual output."""
    mine, theirs = sides
    rng = np.random.default_rng(7)
    count = 40000
    values = random_halves(rng, count)
    values[:200] = (np.arange(200, dtype=np.float32) / 2 - 50).astype(np.float16).view(np.uint16)
    scales = np.abs(rng.normal(0.0, 3.0, count)).astype(np.float16).view(np.uint16)
    means = random_halves(rng, count)
    mask = rng.choice(np.array([0x0000, 0x3c00], np.uint16), count)
    for with_residual in (True, False):
        outs = [[np.zeros(count, np.uint16) for _ in range(4)] for _ in range(2)]
        for lib, name, out in ((mine, "gh_process", outs[0]), (theirs, "ref_glue_process", outs[1])):
            residual = ptr(out[0]) if with_residual else None
            assert getattr(lib, name)(ptr(values), ptr(scales), ptr(means), ptr(mask), residual, ptr(out[1]),
                                      ptr(out[2]), ptr(out[3]), count, force_zero) == 1
        for a, b in zip(*outs):
            assert same_halves(a, b)


def test_reductions(sides):
    mine, theirs = sides
    rng = np.random.default_rng(8)
    for ways in (4, 2):
        for batch, channels, height, width in ((1, 4, 3, 5), (2, 8, 4, 4), (1, 12, 1, 9)):
            count = batch * channels * height * width
            source = random_halves(rng, count)
            mask = rng.choice(np.array([0x0000, 0x3c00], np.uint16), count)
            for masked in (False, True):
                a = np.zeros(count // ways, np.uint16)
                b = np.zeros(count // ways, np.uint16)
                m = ptr(mask) if masked else None
                assert mine.gh_reduce(ptr(source), m, ptr(a), batch, channels, height, width, ways) == 1
                assert theirs.ref_glue_reduce(ptr(source), m, ptr(b), count, batch, channels, height, width, ways) == 1
                assert same_halves(a, b)
    bad = np.zeros(16, np.uint16)
    assert mine.gh_reduce(ptr(bad), None, ptr(bad), 1, 6, 1, 1, 4) == theirs.ref_glue_reduce(ptr(bad), None, ptr(bad), 16, 1, 6, 1, 1, 4) == 0


POINTWISE = {"round_to_int8": 0, "int8_to_half": 1, "clamp_min": 2, "clamp_reciprocal_with_quant": 3,
             "add_in_place": 4, "multiply_broadcast": 5, "add_and_multiply": 6}


@pytest.mark.parametrize("op", sorted(POINTWISE))
def test_pointwise_steps(sides, op):
    """Each elementwise step on seeded halves with specials (ties of the
    rounding, values that overflow FP16, NaN, infinities, subnormals)."""
    mine, theirs = sides
    for lib, name in ((mine, "gh_pointwise"), (theirs, "ref_glue_pointwise")):
        getattr(lib, name).argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_size_t, ctypes.c_float,
                                                                                  ctypes.c_size_t]
    rng = np.random.default_rng(10 + POINTWISE[op])
    spatial, channels = 257, 7
    count = spatial * channels
    base = [random_halves(rng, count) for _ in range(3)]
    base[0][:64] = (np.arange(64, dtype=np.float32) / 2 - 16).astype(np.float16).view(np.uint16)  # .5 ties
    q = rng.integers(-128, 128, count).astype(np.int8)
    for scalar in (0.0, 0.11, -3.0):
        runs = []
        for lib, name in ((mine, "gh_pointwise"), (theirs, "ref_glue_pointwise")):
            a, b, c, qq = base[0].copy(), base[1].copy(), base[2].copy(), q.copy()
            assert getattr(lib, name)(POINTWISE[op], ptr(a), ptr(b), ptr(c), ptr(qq), count, scalar, spatial) == 1
            runs.append((a, b, qq))
        for x, y in zip(*runs):
            assert (np.array_equal(x, y) if x.dtype == np.int8 else same_halves(x, y)), op


def test_replicate_pad_and_crop(sides):
    mine, theirs = sides
    mine.gh_pad_or_crop.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 7
    theirs.ref_glue_pad_or_crop.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_size_t] + [ctypes.c_int] * 7
    rng = np.random.default_rng(11)
    for batch, channels, height, width in ((1, 3, 5, 7), (2, 2, 1, 1), (1, 1, 4, 3)):
        source = rng.integers(0, 65536, batch * channels * height * width, dtype=np.uint16)
        for pad, out_h, out_w in ((1, height, width), (1, height + 3, width + 5), (1, height - 1, width),
                                  (0, height, width), (0, 1, 1), (0, height, max(1, width - 2)), (0, height + 1, width),
                                  (0, 0, width)):
            capacity = batch * channels * max(out_h, 1) * max(out_w, 1)
            a = np.zeros(capacity, np.uint16)
            b = np.zeros(capacity, np.uint16)
            ok_a = mine.gh_pad_or_crop(ptr(source), ptr(a), batch, channels, height, width, out_h, out_w, pad)
            ok_b = theirs.ref_glue_pad_or_crop(ptr(source), ptr(b), capacity, batch, channels, height, width, out_h,
                                               out_w, pad)
            assert ok_a == ok_b, (pad, out_h, out_w)
            if ok_a:
                assert np.array_equal(a, b)


def test_picture_conversions(sides):
    """RGB24 and YUV 4:2:0 into padded YCbCr (every 8-bit value, odd and even
    sizes, padding), and YCbCr back to YUV 4:2:0 from seeded halves with
    values outside [0, 1] and specials; refusals of odd or oversized pictures."""
    mine, theirs = sides
    mine.gh_to_ycbcr.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int] * 3
    theirs.ref_glue_to_ycbcr.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_size_t] + [ctypes.c_int] * 3
    mine.gh_to_yuv.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p]
    theirs.ref_glue_to_yuv.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_size_t]
    rng = np.random.default_rng(13)
    for yuv in (0, 1):
        for width, height, padded_h, padded_w in ((16, 16, 16, 16), (24, 10, 16, 32), (7, 5, 8, 8), (2, 2, 4, 6),
                                                  (3, 4, 2, 4)):
            size = width * height * 3 if not yuv else width * height + 2 * ((width // 2) * (height // 2))
            picture = rng.integers(0, 256, size, dtype=np.uint8)
            picture[: min(size, 256)] = np.arange(min(size, 256), dtype=np.uint8)
            capacity = 3 * max(padded_h, 1) * max(padded_w, 1)
            a = np.zeros(capacity, np.uint16)
            b = np.zeros(capacity, np.uint16)
            ok_a = mine.gh_to_ycbcr(ptr(picture), width, height, ptr(a), padded_h, padded_w, yuv)
            ok_b = theirs.ref_glue_to_ycbcr(ptr(picture), size, width, height, ptr(b), capacity, padded_h, padded_w,
                                            yuv)
            assert ok_a == ok_b, (yuv, width, height, padded_h, padded_w)
            if ok_a:
                assert np.array_equal(a, b)
    for height, width, visible_w, visible_h in ((16, 16, 16, 16), (10, 24, 20, 8), (9, 9, 8, 8), (8, 8, 7, 8),
                                                (8, 8, 10, 8)):
        source = random_halves(rng, 3 * height * width)
        source[: 3 * height * width // 2] = rng.uniform(-0.2, 1.2, 3 * height * width // 2).astype(np.float16) \
            .view(np.uint16)
        capacity = visible_w * visible_h + 2 * (visible_w // 2) * (visible_h // 2) + 8
        a = np.zeros(capacity, np.uint8)
        b = np.zeros(capacity, np.uint8)
        ok_a = mine.gh_to_yuv(ptr(source), 1, 3, height, width, visible_w, visible_h, ptr(a))
        ok_b = theirs.ref_glue_to_yuv(ptr(source), 1, 3, height, width, visible_w, visible_h, ptr(b), capacity)
        assert ok_a == ok_b, (height, width, visible_w, visible_h)
        if ok_a:
            assert np.array_equal(a, b)
