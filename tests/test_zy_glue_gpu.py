"""DCVC-RT inter-stage glue on the GPU (nvcr_sm100_dcvc_*) against the same
element functions compiled for the host (tests/glue_host.cpp), which
tests/test_glue_host.py pins bit for bit to the reference's host ops: index
builds on every half scale, masks on every stage, restore on seeded halves."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def ptr(tensor):
    return ctypes.c_void_p(tensor.data_ptr())


@pytest.fixture(scope="module")
def host():
    from tests.glue_host import load

    lib = load()
    lib.gh_decode_indexes.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float]
    lib.gh_encode_indexes.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.c_float]
    lib.gh_mask.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 6
    lib.gh_restore.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5
    lib.gh_process.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_size_t, ctypes.c_float]
    lib.gh_reduce.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5
    return lib


def test_index_builds(cuda, host):
    import torch

    from nvcr_b200.executor import _check, library

    scales = np.arange(65536, dtype=np.uint16)
    symbols = np.random.default_rng(5).integers(-128, 128, 65536).astype(np.float16).view(np.uint16)
    for force_zero in (0.0, 0.11, 0.5):
        expected = np.zeros(65536, np.uint8)
        host.gh_decode_indexes(scales.ctypes.data, expected.ctypes.data, 65536, force_zero)
        device_scales = torch.from_numpy(scales.view(np.int16)).cuda()
        out = torch.zeros(65536, dtype=torch.uint8, device="cuda")
        _check(library().nvcr_sm100_dcvc_build_decode_indexes(ptr(device_scales), ptr(out), 65536, force_zero, None))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), expected)
        expected_encode = np.zeros(65536, np.int16)
        host.gh_encode_indexes(symbols.ctypes.data, scales.ctypes.data, expected_encode.ctypes.data, 65536, force_zero)
        device_symbols = torch.from_numpy(symbols.view(np.int16)).cuda()
        encoded = torch.zeros(65536, dtype=torch.int16, device="cuda")
        _check(library().nvcr_sm100_dcvc_build_encode_indexes(ptr(device_symbols), ptr(device_scales), ptr(encoded),
                                                              65536, force_zero, None))
        torch.cuda.synchronize()
        assert np.array_equal(encoded.cpu().numpy(), expected_encode)


def test_masks_and_restore(cuda, host):
    import torch

    from nvcr_b200.executor import _check, library
    from tests.test_glue_host import same_halves

    rng = np.random.default_rng(6)
    for ways in (4, 2):
        for batch, channels, height, width in ((1, 4, 3, 5), (2, 128, 68, 120)):
            count = batch * channels * height * width
            for stage in range(ways):
                expected = np.zeros(count, np.uint16)
                assert host.gh_mask(expected.ctypes.data, batch, channels, height, width, ways, stage) == 1
                mask = torch.zeros(count, dtype=torch.int16, device="cuda")
                _check(library().nvcr_sm100_dcvc_make_mask(ptr(mask), batch, channels, height, width, ways, stage,
                                                           None))
                torch.cuda.synchronize()
                assert np.array_equal(mask.cpu().numpy().view(np.uint16), expected)
            symbols = rng.integers(0, 65536, count // ways, dtype=np.uint16)
            means = rng.integers(0, 65536, count, dtype=np.uint16)
            expected = np.zeros(count, np.uint16)
            host_mask = mask.cpu().numpy().view(np.uint16).copy()
            host.gh_restore(symbols.ctypes.data, means.ctypes.data, host_mask.ctypes.data, expected.ctypes.data,
                            batch, channels, height, width, ways)
            device_symbols = torch.from_numpy(symbols.view(np.int16)).cuda()
            device_means = torch.from_numpy(means.view(np.int16)).cuda()
            out = torch.zeros(count, dtype=torch.int16, device="cuda")
            _check(library().nvcr_sm100_dcvc_restore(ptr(device_symbols), ptr(device_means), ptr(mask), ptr(out),
                                                     batch, channels, height, width, ways, None))
            torch.cuda.synchronize()
            # Restore adds a mean to a symbol: a NaN result's sign follows x86
            # operand order on the host and is canonical on the GPU, so NaN
            # equals NaN here (the profile's rule).
            assert same_halves(out.cpu().numpy().view(np.uint16), expected)


def test_process_and_reduce(cuda, host):
    import torch

    from nvcr_b200.executor import _check, library

    rng = np.random.default_rng(9)
    batch, channels, height, width = 1, 128, 68, 120
    count = batch * channels * height * width
    values = rng.normal(0.0, 40.0, count).astype(np.float16).view(np.uint16)
    scales = np.abs(rng.normal(0.0, 3.0, count)).astype(np.float16).view(np.uint16)
    means = rng.normal(0.0, 10.0, count).astype(np.float16).view(np.uint16)
    mask = rng.choice(np.array([0x0000, 0x3c00], np.uint16), count)
    expected = [np.zeros(count, np.uint16) for _ in range(4)]
    host.gh_process(values.ctypes.data, scales.ctypes.data, means.ctypes.data, mask.ctypes.data,
                    *[e.ctypes.data for e in expected], count, 0.11)
    device = [torch.from_numpy(a.view(np.int16)).cuda() for a in (values, scales, means, mask)]
    outs = [torch.zeros(count, dtype=torch.int16, device="cuda") for _ in range(4)]
    _check(library().nvcr_sm100_dcvc_process_with_mask(*[ptr(t) for t in device], *[ptr(t) for t in outs], count,
                                                       0.11, None))
    torch.cuda.synchronize()
    for out, want in zip(outs, expected):
        assert np.array_equal(out.cpu().numpy().view(np.uint16), want)
    for ways in (4, 2):
        for masked in (False, True):
            want = np.zeros(count // ways, np.uint16)
            host.gh_reduce(values.ctypes.data, mask.ctypes.data if masked else None, want.ctypes.data, batch, channels,
                           height, width, ways)
            out = torch.zeros(count // ways, dtype=torch.int16, device="cuda")
            _check(library().nvcr_sm100_dcvc_reduce(ptr(device[0]), ptr(device[3]) if masked else None, ptr(out),
                                                    batch, channels, height, width, ways, None))
            torch.cuda.synchronize()
            assert np.array_equal(out.cpu().numpy().view(np.uint16), want)


def test_pointwise_steps(cuda, host):
    """Each elementwise step on the device against the host build (NaN equal to NaN)."""
    import torch

    from nvcr_b200.executor import _check, library
    from tests.test_glue_host import POINTWISE, random_halves, same_halves

    host.gh_pointwise.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_size_t, ctypes.c_float,
                                                                           ctypes.c_size_t]
    rng = np.random.default_rng(12)
    spatial, channels = 8160, 16
    count = spatial * channels
    base = [random_halves(rng, count) for _ in range(3)]
    q = rng.integers(-128, 128, count).astype(np.int8)
    lib = library()
    for op, code in POINTWISE.items():
        a, b, c, qq = base[0].copy(), base[1].copy(), base[2].copy(), q.copy()
        assert host.gh_pointwise(code, a.ctypes.data, b.ctypes.data, c.ctypes.data, qq.ctypes.data, count, 0.11,
                                 spatial) == 1
        da, db, dc = (torch.from_numpy(x.view(np.int16).copy()).cuda() for x in base)
        dq = torch.from_numpy(q.copy()).cuda()
        calls = {
            "round_to_int8": lambda: lib.nvcr_sm100_dcvc_round_to_int8(ptr(da), ptr(dq), count, None),
            "int8_to_half": lambda: lib.nvcr_sm100_dcvc_int8_to_half(ptr(dq), ptr(da), count, None),
            "clamp_min": lambda: lib.nvcr_sm100_dcvc_clamp_min(ptr(da), count, 0.11, None),
            "clamp_reciprocal_with_quant": lambda: lib.nvcr_sm100_dcvc_clamp_reciprocal_with_quant(ptr(da), ptr(db),
                                                                                                  count, None),
            "add_in_place": lambda: lib.nvcr_sm100_dcvc_add_in_place(ptr(da), ptr(db), count, None),
            "multiply_broadcast": lambda: lib.nvcr_sm100_dcvc_multiply_broadcast(ptr(da), ptr(db), spatial, channels,
                                                                                 None),
            "add_and_multiply": lambda: lib.nvcr_sm100_dcvc_add_and_multiply(ptr(da), ptr(db), ptr(dc), count, None),
        }
        _check(calls[op]())
        torch.cuda.synchronize()
        assert same_halves(da.cpu().numpy(), a), op
        assert same_halves(db.cpu().numpy(), b), op
        assert np.array_equal(dq.cpu().numpy(), qq), op


def test_picture_conversions(cuda, host):
    import torch

    from nvcr_b200.executor import _check, library

    host.gh_to_ycbcr.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int] * 3
    host.gh_to_yuv.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p]
    rng = np.random.default_rng(14)
    width, height, padded_h, padded_w = 1920, 1080, 1088, 1920
    lib = library()
    for yuv in (0, 1):
        size = width * height * 3 if not yuv else width * height * 3 // 2
        picture = rng.integers(0, 256, size, dtype=np.uint8)
        expected = np.zeros(3 * padded_h * padded_w, np.uint16)
        assert host.gh_to_ycbcr(picture.ctypes.data, width, height, expected.ctypes.data, padded_h, padded_w, yuv) == 1
        device_picture = torch.from_numpy(picture).cuda()
        out = torch.zeros(3 * padded_h * padded_w, dtype=torch.int16, device="cuda")
        convert = lib.nvcr_sm100_dcvc_yuv420p8_to_ycbcr_padded if yuv else lib.nvcr_sm100_dcvc_rgb24_to_ycbcr_padded
        _check(convert(ptr(device_picture), width, height, ptr(out), padded_h, padded_w, None))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint16), expected)
    back = np.zeros(width * height * 3 // 2, np.uint8)
    assert host.gh_to_yuv(expected.ctypes.data, 1, 3, padded_h, padded_w, width, height, back.ctypes.data) == 1
    device_back = torch.zeros(width * height * 3 // 2, dtype=torch.uint8, device="cuda")
    _check(lib.nvcr_sm100_dcvc_ycbcr_padded_to_yuv420p8(ptr(out), 1, 3, padded_h, padded_w, width, height,
                                                        ptr(device_back), None))
    torch.cuda.synchronize()
    assert np.array_equal(device_back.cpu().numpy(), back)
