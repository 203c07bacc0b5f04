"""Builds and loads tests/provider_harness.cpp (TEST INFRASTRUCTURE): C entry
points over the sm_100a provider session of nvcr_b200/provider, which is built
against the reference's provider headers. Both libraries are built only where
the reference checkout is; elsewhere the prebuilt ones are used if present."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
SOURCE = ROOT / "tests" / "provider_harness.cpp"
LIBRARY = ROOT / "tests" / "_build" / "libprovider_harness.so"


def load() -> ctypes.CDLL | None:
    from nvcr_b200.provider import build as provider

    library = provider.build()
    if library is None:
        return None
    if provider.available():
        inputs = [SOURCE, library, provider.HERE / "sm100_session.hpp"]
        if not LIBRARY.exists() or LIBRARY.stat().st_mtime < max(p.stat().st_mtime for p in inputs):
            LIBRARY.parent.mkdir(parents=True, exist_ok=True)
            subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", *provider.include_flags(
                provider.reference_root()), str(SOURCE), "-o", str(LIBRARY), f"-L{library.parent}",
                "-lnvcr_sm100_provider", f"-Wl,-rpath,{library.parent}",
                f"-L{provider.CUDA_HOME / 'lib64'}", "-lcudart"], check=True)
    if not LIBRARY.exists():
        return None
    lib = ctypes.CDLL(str(LIBRARY))
    cp, sz, i32p = ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32)
    u8p = ctypes.POINTER(ctypes.c_ubyte)
    lib.ph_supports.restype = ctypes.c_int
    lib.ph_supports.argtypes = [cp]
    lib.ph_load.restype = ctypes.c_int
    lib.ph_load.argtypes = [cp, cp, u8p, cp, cp, sz]
    lib.ph_registry.restype = ctypes.c_int
    lib.ph_registry.argtypes = [cp, sz]
    lib.ph_run.restype = ctypes.c_int
    lib.ph_run.argtypes = [cp, cp, u8p, ctypes.c_int, ctypes.POINTER(cp), i32p, ctypes.POINTER(ctypes.c_void_p),
                           ctypes.c_int, ctypes.POINTER(cp), i32p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                           ctypes.c_int, cp, sz]
    return lib
