"""The DCVC-RT glue entry points of the C ABI (no GPU): each refuses, with
NVCR_SM100_INVALID_ARGUMENT and before any launch, the shapes and arguments
the reference's host ops refuse (src/dcvcrt/host_ops.cpp), case by case with
the reference compiled into oracle/_ref. Only refused cases reach the C ABI
here: the buffers are host memory, which an accepted call would hand to a
kernel; that every case the reference refuses is refused, and every case the
host build accepts is computed like the reference's, is checked in
tests/test_glue_host.py."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

INVALID = 1  # NVCR_SM100_INVALID_ARGUMENT


@pytest.fixture(scope="module")
def lib(built_library):
    from nvcr_b200.executor import library

    return library()


def buffer(count: int, dtype=np.uint16) -> np.ndarray:
    return np.zeros(max(count, 1), dtype)


def ptr(array: np.ndarray):
    return ctypes.c_void_p(array.ctypes.data)


SHAPES = [(1, 4, 2, 2), (0, 4, 2, 2), (1, 0, 2, 2), (1, 6, 2, 2), (1, 4, 0, 2), (1, 4, 2, -1), (2, 8, 1, 1),
          (1, 2, 3, 3)]


def test_mask_restore_reduce_refusals_match_reference(lib, reference):
    ref = reference.lib
    ref.ref_glue_mask.argtypes = [ctypes.c_void_p, ctypes.c_size_t] + [ctypes.c_int] * 6
    ref.ref_glue_restore.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_size_t] + [ctypes.c_int] * 5
    ref.ref_glue_reduce.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_size_t] + [ctypes.c_int] * 5
    for ways in (4, 2, 3):
        for shape in SHAPES:
            count = int(np.prod([max(v, 0) for v in shape]))
            a, b, c, d = (buffer(count) for _ in range(4))
            for stage in (-1, 0, ways - 1, ways):
                if ways not in (2, 4) or ref.ref_glue_mask(ptr(a), count, *shape, ways, stage) == 0:
                    assert lib.nvcr_sm100_dcvc_make_mask(ptr(a), *shape, ways, stage, None) == INVALID
            if ways not in (2, 4) or ref.ref_glue_restore(ptr(a), ptr(b), ptr(c), ptr(d), count, *shape, ways) == 0:
                assert lib.nvcr_sm100_dcvc_restore(ptr(a), ptr(b), ptr(c), ptr(d), *shape, ways, None) == INVALID
            if ways not in (2, 4) or ref.ref_glue_reduce(ptr(a), None, ptr(b), count, *shape, ways) == 0:
                assert lib.nvcr_sm100_dcvc_reduce(ptr(a), None, ptr(b), *shape, ways, None) == INVALID


def test_picture_and_resize_refusals_match_reference(lib, reference):
    ref = reference.lib
    ref.ref_glue_pad_or_crop.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_size_t] + [ctypes.c_int] * 7
    ref.ref_glue_to_ycbcr.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_size_t] + [ctypes.c_int] * 3
    ref.ref_glue_to_yuv.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_size_t]
    source = buffer(4096)
    target = buffer(4096)
    for batch, channels, height, width in ((1, 3, 4, 4), (0, 3, 4, 4), (1, 3, -1, 4)):
        for out_h, out_w in ((4, 4), (6, 5), (3, 4), (0, 4), (5, 4)):
            for pad, entry in ((1, lib.nvcr_sm100_dcvc_replicate_pad), (0, lib.nvcr_sm100_dcvc_crop_spatial)):
                if ref.ref_glue_pad_or_crop(ptr(source), ptr(target), 4096, batch, channels, height, width, out_h,
                                            out_w, pad) == 0:
                    assert entry(ptr(source), ptr(target), batch, channels, height, width, out_h, out_w,
                                 None) == INVALID
    picture = buffer(4096, np.uint8)
    for width, height, padded_h, padded_w in ((8, 8, 8, 8), (7, 8, 8, 8), (8, 7, 8, 8), (8, 8, 6, 8), (0, 8, 8, 8)):
        for yuv, entry in ((0, lib.nvcr_sm100_dcvc_rgb24_to_ycbcr_padded),
                           (1, lib.nvcr_sm100_dcvc_yuv420p8_to_ycbcr_padded)):
            if ref.ref_glue_to_ycbcr(ptr(picture), 4096, width, height, ptr(target), 4096, padded_h, padded_w,
                                     yuv) == 0:
                assert entry(ptr(picture), width, height, ptr(target), padded_h, padded_w, None) == INVALID
    for shape, visible in (((1, 3, 8, 8), (8, 8)), ((1, 3, 8, 8), (7, 8)), ((1, 2, 8, 8), (8, 8)),
                           ((2, 3, 8, 8), (8, 8)), ((1, 3, 8, 8), (10, 8))):
        if ref.ref_glue_to_yuv(ptr(source), *shape, *visible, ptr(picture), 4096) == 0:
            assert lib.nvcr_sm100_dcvc_ycbcr_padded_to_yuv420p8(ptr(source), *shape, *visible, ptr(picture),
                                                                None) == INVALID


def test_empty_and_null_are_refused(lib):
    a = buffer(8)
    assert lib.nvcr_sm100_dcvc_build_decode_indexes(ptr(a), ptr(a), 0, 0.0, None) == INVALID
    assert lib.nvcr_sm100_dcvc_build_encode_indexes(None, ptr(a), ptr(a), 4, 0.0, None) == INVALID
    assert lib.nvcr_sm100_dcvc_clamp_min(ptr(a), 0, 0.0, None) == INVALID
    assert lib.nvcr_sm100_dcvc_add_in_place(ptr(a), None, 4, None) == INVALID
    assert lib.nvcr_sm100_dcvc_multiply_broadcast(ptr(a), ptr(a), 4, 0, None) == INVALID
    assert lib.nvcr_sm100_dcvc_add_and_multiply(ptr(a), ptr(a), None, 4, None) == INVALID
    assert lib.nvcr_sm100_dcvc_round_to_int8(ptr(a), None, 4, None) == INVALID
    assert lib.nvcr_sm100_dcvc_process_with_mask(ptr(a), ptr(a), ptr(a), ptr(a), None, ptr(a), ptr(a), None, 4, 0.0,
                                                 None) == INVALID
