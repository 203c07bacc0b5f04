"""Builds the sm_100a provider session (sm100_session.cpp) against the
reference's provider headers, with the reference sources it needs (the error
type, src/common/error.cpp, the registry, src/runtime/registry.cpp, and what
the registry calls, src/artifacts/resolver.cpp and
src/configuration/configuration.cpp),
into nvcr_b200/provider/_build/libnvcr_sm100_provider.so. It links
libnvcr_sm100.so (the C ABI) and the CUDA runtime.

The provider is reference-side code: it is built only where the reference
checkout is (NVCR_REFERENCE, else a directory named `reference` beside this
repository); the built library travels with the repository like the other
built libraries.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
BUILD = HERE / "_build"
LIBRARY = BUILD / "libnvcr_sm100_provider.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def reference_root() -> Path:
    return Path(os.environ.get("NVCR_REFERENCE", ROOT.parent / "reference"))


def reference_sources(ref: Path) -> list[Path]:
    # The registry's runtime services resolve artifacts and normalise the
    # runtime configuration, so the resolver and the configuration come along.
    return [ref / "src" / "common" / "error.cpp", ref / "src" / "runtime" / "registry.cpp",
            ref / "src" / "artifacts" / "resolver.cpp", ref / "src" / "configuration" / "configuration.cpp"]


def versions_header(ref: Path) -> Path:
    """The reference's generated versions.hpp (zero versions), from its template."""
    out = BUILD / "gen" / "nvcr" / "common" / "versions.hpp"
    template = ref / "include" / "nvcr" / "common" / "versions.hpp.in"
    if not out.exists() or out.stat().st_mtime < template.stat().st_mtime:
        out.parent.mkdir(parents=True, exist_ok=True)
        text = template.read_text()
        for key, value in (("@PROJECT_VERSION_MAJOR@", "0"), ("@PROJECT_VERSION_MINOR@", "0"),
                           ("@PROJECT_VERSION_PATCH@", "0"), ("@PROJECT_VERSION@", "0.0.0")):
            text = text.replace(key, value)
        out.write_text(text)
    return out


def include_flags(ref: Path) -> list[str]:
    return [f"-I{HERE}", f"-I{ROOT / 'include'}", f"-I{ref / 'include'}", f"-I{BUILD / 'gen'}",
            f"-I{ref / 'src'}", f"-I{CUDA_HOME / 'include'}"]


def available() -> bool:
    return (reference_root() / "include" / "nvcr" / "provider" / "experimental" / "session.hpp").exists()


def build(verbose: bool = False) -> Path | None:
    """Builds the provider library when the reference headers exist; returns its
    path, or None when they do not (the prebuilt library, if any, is kept)."""
    if not available():
        return LIBRARY if LIBRARY.exists() else None
    from nvcr_b200.build import build as build_library

    core = build_library()
    ref = reference_root()
    BUILD.mkdir(parents=True, exist_ok=True)
    versions_header(ref)
    sources = [HERE / "sm100_session.cpp", *reference_sources(ref)]
    inputs = sources + [HERE / "sm100_session.hpp", ROOT / "include" / "nvcr_sm100.h", core]
    if LIBRARY.exists() and LIBRARY.stat().st_mtime >= max(p.stat().st_mtime for p in inputs):
        return LIBRARY
    cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-Wl,--no-undefined",
           *include_flags(ref), *map(str, sources), "-o", str(LIBRARY),
           f"-L{core.parent}", "-lnvcr_sm100", f"-Wl,-rpath,$ORIGIN/../../_build",
           f"-L{CUDA_HOME / 'lib64'}", "-lcudart", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"provider build failed: {' '.join(cmd)}\n{result.stderr}")
    if verbose:
        print(f"built {LIBRARY}")
    return LIBRARY


if __name__ == "__main__":
    build(verbose=True)
