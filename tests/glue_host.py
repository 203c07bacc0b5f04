"""Builds and calls tests/glue_host.cpp: the DCVC-RT glue element functions the
kernels in nvcr_b200/csrc/k_glue.cu run, compiled for the host (TEST
INFRASTRUCTURE)."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "nvcr_b200" / "csrc"
SOURCES = [ROOT / "tests" / "glue_host.cpp", CSRC / "glue_elements.cuh", CSRC / "scale_thresholds.inc"]
LIBRARY = ROOT / "tests" / "_build" / "libglue_host.so"


def load() -> ctypes.CDLL:
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < max(p.stat().st_mtime for p in SOURCES):
        LIBRARY.parent.mkdir(parents=True, exist_ok=True)
        subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
                        f"-I{CSRC}", str(SOURCES[0]), "-o", str(LIBRARY)], check=True)
    return ctypes.CDLL(str(LIBRARY))
