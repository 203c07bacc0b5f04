"""Builds libnvcr_sm100.so in-tree (nvcr_b200/_build/) for sm_100a.

CUDA sources: nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
-fmad=false (no FP contraction; denormals kept, IEEE division) and no fast
math. Host sources: g++ -ffp-contract=off -fno-fast-math, as the profile's
host arithmetic requires. The CUDA runtime is linked statically and the driver
is reached through cudaGetDriverEntryPointByVersion, so the library loads on a
machine without a GPU driver (symbols can be listed; compute calls fail).
"""
from __future__ import annotations

import concurrent.futures
import os
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
SOURCE = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIBRARY = BUILD / "libnvcr_sm100.so"
INCLUDE = PACKAGE.parent / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-std=c++20", "-O3", "-lineinfo", "-fmad=false", "-prec-div=true", "-prec-sqrt=true",
                     "-ftz=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
                     f"-I{INCLUDE}", f"-I{SOURCE}"]
CXX_FLAGS = ["-std=c++20", "-O2", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-Wall", "-Wextra",
             "-Wno-unused-parameter", f"-I{CUDA_HOME / 'include'}", f"-I{INCLUDE}", f"-I{SOURCE}"]


def _sources() -> list[Path]:
    return sorted(list(SOURCE.glob("*.cu")) + list(SOURCE.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(SOURCE.glob("*.hpp")) + list(SOURCE.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _compile(source: Path) -> Path:
    obj = BUILD / (source.name + ".o")
    newest_dep = max([source.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    if source.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(source), "-o", str(obj)]
    else:
        cmd = ["g++", *CXX_FLAGS, "-c", str(source), "-o", str(obj)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{result.stdout}\n{result.stderr}")
    return obj


def build(verbose: bool = False) -> Path:
    """Compiles every source (incrementally) and links the shared library."""
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(_compile, sources))
    newest = max(o.stat().st_mtime for o in objects)
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIBRARY), *map(str, objects)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{result.stdout}\n{result.stderr}")
        if verbose:
            print(f"built {LIBRARY}")
    return LIBRARY


if __name__ == "__main__":
    build(verbose=True)
