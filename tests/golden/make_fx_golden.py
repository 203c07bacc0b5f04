#!/usr/bin/env python3
"""Generates tests/golden/fx_golden.json from the REFERENCE's own nvcr.fx.v1
CPU arithmetic (src/deterministic/fx.cpp and fx_program.cpp, compiled from
its sources into oracle/_ref by oracle/Makefile), reached through its own
program loader. The reference ships per-op hand vectors but no whole-program
vectors, so these pin the oracle (oracle/fx_oracle.c, oracle/fx.py) to the
reference's outputs where the reference is not at hand.

Programs and inputs are not stored: each case regenerates them from a seeded
numpy Generator (tests/fx_programs.py), and the fixture records the SHA-256 of
the written program files and of the inputs, so a drift in generation is
caught. Outputs are stored as the SHA-256 of their int32 bytes plus shapes and
the first values; a failing case stores the reference's status and message.

Run from the repository root where the reference sources exist:
    python tests/golden/make_fx_golden.py
"""
from __future__ import annotations

import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.fx import FxReference  # noqa: E402
from oracle.oracle import build  # noqa: E402
from tests.fx_programs import decoder_like, decoder_like_inputs, write_program  # noqa: E402

HERE = Path(__file__).resolve().parent

# (seed, tight, height, width): decoder-like programs that use every op.
CASES = [(seed, seed % 3 == 2, 2 + (seed * 5) % 13, 3 + (seed * 7) % 11) for seed in range(16)]


def case_program(seed: int, tight: bool, height: int, width: int):
    rng = np.random.default_rng(1000 + seed)
    program = decoder_like(rng, tight=tight)
    return program, decoder_like_inputs(rng, program, height, width)


def files_digest(directory: Path, stage: str) -> str:
    digest = hashlib.sha256()
    for suffix in (".fxprog.json", ".fxw"):
        digest.update((directory / f"{stage}{suffix}").read_bytes())
    return digest.hexdigest()


def arrays_digest(arrays) -> str:
    digest = hashlib.sha256()
    for array in arrays:
        digest.update(np.ascontiguousarray(array, np.int32).tobytes())
    return digest.hexdigest()


def main() -> None:
    build(reference=True)
    reference = FxReference()
    entries = []
    with tempfile.TemporaryDirectory() as scratch:
        directory = Path(scratch)
        for seed, tight, height, width in CASES:
            program, inputs = case_program(seed, tight, height, width)
            write_program(directory, "g", program)
            status, outputs, message = reference.run(directory, "g", inputs)
            entries.append({
                "seed": seed, "tight": tight, "height": height, "width": width,
                "program_sha256": files_digest(directory, "g"), "inputs_sha256": arrays_digest(inputs),
                "status": status, "message": message,
                "outputs": [{"shape": list(y.shape), "sha256": arrays_digest([y]), "head": y.reshape(-1)[:6].tolist()}
                            for y in outputs]})
    path = HERE / "fx_golden.json"
    path.write_text(json.dumps({"generator": "tests/golden/make_fx_golden.py", "cases": entries}, indent=1) + "\n")
    print(f"wrote {path} ({len(entries)} cases)")


if __name__ == "__main__":
    main()
