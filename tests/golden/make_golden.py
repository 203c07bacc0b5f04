#!/usr/bin/env python3
"""Generates the golden fixtures in this directory from the REFERENCE's own CPU
executor (run_cpu and det_math, compiled from its sources into oracle/_ref by
oracle/Makefile). The reference ships no golden vectors for intconv.v1, so
these pin the oracle (oracle/intconv_oracle.c) to the reference's outputs.

Inputs are not stored: every case regenerates them from a seeded std::mt19937
stream (nvcr_b200.program.SeededStream), and the fixture records the SHA-256 of
the regenerated inputs so a drift in generation is caught. Outputs are stored
as SHA-256 digests of their FP32 bytes (every NaN made the canonical quiet NaN,
the profile's NaN rule) plus the first values in hex for readability.

Run from the repository root where the reference sources exist:
    python tests/golden/make_golden.py
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

from oracle.oracle import Reference, build, canonical_digest  # noqa: E402
from tests.golden.cases import program_cases, scalar_inputs, weight_cases  # noqa: E402

HERE = Path(__file__).resolve().parent


def digest_bytes(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def head(array: np.ndarray, count: int = 6) -> list[str]:
    return [f"{int(v):08x}" for v in np.ascontiguousarray(array, np.float32).reshape(-1)[:count].view(np.uint32)]


def main() -> int:
    build(reference=True)
    reference = Reference()
    lib = reference.lib

    # ---- scalar arithmetic ----
    scalars: dict = {}
    s = scalar_inputs()
    exp_out = np.array([lib.ref_det_exp(float(v)) for v in s["floats"]], np.float32)
    sig_out = np.array([lib.ref_det_sigmoid(float(v)) for v in s["floats"]], np.float32)
    f2h_out = np.array([lib.ref_float_to_half(float(v)) for v in s["floats"]], np.uint16)
    h2f_out = np.array([lib.ref_half_to_float(int(h)) for h in s["halves"]], np.float32)
    ldexp_out = np.array([lib.ref_det_ldexp(float(v), int(e)) for v, e in zip(s["ldexp_values"], s["ldexp_exponents"])],
                         np.float32)
    exp8 = np.array([lib.ref_det_int_exponent(float(m), 8) for m in s["maxima"]], np.int32)
    exp16 = np.array([lib.ref_det_int_exponent(float(m), 16) for m in s["maxima"]], np.int32)
    q8 = np.array([lib.ref_det_int_quantize(float(v), int(e), 8) for v, e in zip(s["q_values"], s["q_exponents"])],
                  np.int32)
    q16 = np.array([lib.ref_det_int_quantize(float(v), int(e), 16)
                    for v, e in zip(s["q_values"], s["q_exponents"])], np.int32)
    out = np.array([lib.ref_det_int_output(int(a), float(sc), int(e), float(b))
                    for a, sc, e, b in zip(s["acc"], s["acc_scale"], s["acc_exponent"], s["acc_bias"])], np.float32)
    scalars = {
        "inputs_sha256": {k: digest_bytes(v) for k, v in s.items()},
        "det_exp": canonical_digest(exp_out),
        "det_sigmoid": canonical_digest(sig_out),
        "det_float_to_half_bits": digest_bytes(f2h_out),
        "det_half_bits_to_float": canonical_digest(h2f_out),
        "det_ldexp": canonical_digest(ldexp_out),
        "det_int_exponent_8": digest_bytes(exp8),
        "det_int_exponent_16": digest_bytes(exp16),
        "det_int_quantize_8": digest_bytes(q8),
        "det_int_quantize_16": digest_bytes(q16),
        "det_int_output": canonical_digest(out),
        "det_exp_head": head(exp_out),
        "det_sigmoid_head": head(sig_out),
    }
    weights = {}
    for name, matrix, bits in weight_cases():
        values, scales = reference.quantize_weights(matrix, bits)
        weights[name] = {"values": digest_bytes(values), "scales": canonical_digest(scales),
                         "scales_head": head(scales)}

    # ---- whole programs through run_cpu ----
    programs = []
    with tempfile.TemporaryDirectory() as directory:
        for case in program_cases():
            path = case.program.write(Path(directory) / case.name, case.program.name)
            weights_arg = None if case.fp16_weights else case.program.weights
            outputs = reference.run(path, case.inputs, weights=weights_arg)
            programs.append({
                "name": case.name,
                "fp16_weights": case.fp16_weights,
                "inputs_sha256": [digest_bytes(np.ascontiguousarray(x, np.float32)) for x in case.inputs],
                "outputs": [{"shape": list(o.shape), "sha256": canonical_digest(o), "head": head(o)}
                            for o in outputs],
            })
            print(f"{case.name}: {[o.shape for o in outputs]}")

    document = {
        "generator": "tests/golden/make_golden.py",
        "source": "reference run_cpu / det_math compiled from its sources (oracle/_ref/libnvcr_ref.so)",
        "nan_rule": "digests canonicalise every NaN to 0x7fc00000 (NaN payloads are unspecified)",
        "scalars": scalars,
        "quantize_weights": weights,
        "programs": programs,
    }
    (HERE / "intconv_golden.json").write_text(json.dumps(document, indent=1) + "\n")
    print(f"wrote {HERE / 'intconv_golden.json'}: {len(programs)} programs")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
