"""Builds and calls tests/fx_host.cpp: the product's nvcr.fx.v1 executor and
kernel element functions compiled for the host (TEST INFRASTRUCTURE; see the
header of fx_host.cpp for what this can and cannot check)."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
SOURCES = [ROOT / "tests" / "fx_host.cpp"] + [ROOT / "nvcr_b200" / "csrc" / name for name in
                                              ("fx_executor.cpp", "fx_program.cpp", "json.cpp", "sha256.cpp")]
HEADERS = [ROOT / "nvcr_b200" / "csrc" / name for name in
           ("fx_elements.cuh", "fx_kernels.hpp", "fx_executor.hpp", "fx_program.hpp", "json.hpp", "sha256.hpp",
            "status.hpp")]
LIBRARY = ROOT / "tests" / "_build" / "libfx_host.so"
CUDA_INCLUDE = Path("/usr/local/cuda/include")

_i32p = ctypes.POINTER(ctypes.c_int32)


def build() -> Path:
    newest = max(path.stat().st_mtime for path in SOURCES + HEADERS)
    if LIBRARY.exists() and LIBRARY.stat().st_mtime >= newest:
        return LIBRARY
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-x", "c++", "-Wno-unknown-pragmas",
                    f"-I{ROOT / 'nvcr_b200' / 'csrc'}", f"-I{CUDA_INCLUDE}", *map(str, SOURCES), "-o", str(LIBRARY)],
                   check=True)
    return LIBRARY


class FxHost:
    def __init__(self) -> None:
        lib = ctypes.CDLL(str(build()))
        lib.fxh_run.restype = ctypes.c_int
        lib.fxh_run.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, _i32p, ctypes.POINTER(_i32p),
                                ctypes.c_int, _i32p, ctypes.POINTER(_i32p), ctypes.c_char_p, ctypes.c_size_t,
                                ctypes.c_int]
        lib.fxh_free.argtypes = [ctypes.c_void_p]
        self.lib = lib

    def run(self, directory, stage: str, inputs, capacity: int = 16, device_memory=True):
        """(status, outputs, message): status 0 or ErrorCode + 1; device_memory
        picks the executor's branch (both run on host memory here), or "both"
        for the device branch then the host branch twice on one executor."""
        keep = [np.ascontiguousarray(x, np.int32) for x in inputs]
        extents = np.array([d for x in keep for d in x.shape] or [0], np.int32)
        pointers = (_i32p * max(1, len(keep)))(*[x.ctypes.data_as(_i32p) for x in keep])
        out_extents = np.zeros(3 * capacity, np.int32)
        outputs = (_i32p * capacity)()
        message = ctypes.create_string_buffer(512)
        status = self.lib.fxh_run(str(directory).encode(), stage.encode(), len(keep),
                                  extents.ctypes.data_as(_i32p), pointers, capacity,
                                  out_extents.ctypes.data_as(_i32p), outputs, message, 512,
                                  2 if device_memory == "both" else 1 if device_memory else 0)
        result = []
        for index in range(capacity):
            if not outputs[index]:
                break
            c, h, w = (int(v) for v in out_extents[3 * index:3 * index + 3])
            if status == 0:
                values = np.ctypeslib.as_array(outputs[index], shape=(max(1, c * h * w),))[:c * h * w].copy()
                result.append(values.reshape(c, h, w))
            self.lib.fxh_free(outputs[index])
        return status, result, message.value.decode()
