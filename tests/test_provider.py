"""The sm_100a provider session on the reference's provider boundary
(IProviderSession, include/nvcr/provider/experimental/session.hpp:132-166),
compiled against the reference's headers (nvcr_b200/provider) and reached
through tests/provider_harness.cpp.

Refusals as the reference's exact-stage providers give them
(src/provider/tensorrt/session.cpp:1526-1547, src/provider/onnxruntime/
session.cpp:425-448, contract tests tests/contract_tests.cpp:437-472): a native
stage and a profile other than nvcr.intconv.v1 are incompatible_precision, a
program whose SHA-256 differs from the descriptor's is digest_mismatch, an
absent one missing_artifact. On a GPU, a stage loaded from files written by
Program.write runs through submit() on FP16 tensors in host, pinned-host and
device buffers of the session, bit-exact against the oracle.
"""
from __future__ import annotations

import ctypes
import hashlib

import numpy as np
import pytest

from nvcr_b200 import executor as ex
from nvcr_b200.program import SeededStream
from nvcr_b200.workloads import config1, layer_input
from oracle.oracle import count_differing
from tests.programs import op_program

INCOMPATIBLE_PRECISION = int(ex.ErrorCode.incompatible_precision) + 1


@pytest.fixture(scope="module")
def harness():
    from tests.provider_host import load

    lib = load()
    if lib is None:
        pytest.skip("the provider is built against the reference's headers, which are not here")
    return lib


def digest_of(path) -> ctypes.Array:
    raw = hashlib.sha256(path.read_bytes()).digest()
    return (ctypes.c_ubyte * 32)(*raw)


def load(harness, directory, component, digest, profile):
    message = ctypes.create_string_buffer(512)
    code = harness.ph_load(str(directory).encode(), component.encode(), digest, profile.encode(), message, 512)
    return code, message.value.decode()


def test_registered_with_a_session_factory(harness):
    message = ctypes.create_string_buffer(256)
    assert harness.ph_registry(message, 256) == 0, message.value
    assert b"nvcr.intconv.v1" in message.value


def test_profile_claims_match_the_library(harness, built_library):
    for profile in ("nvcr.intconv.v1", "nvcr.fx.v1", "", "native"):
        assert harness.ph_supports(profile.encode()) == int(ex.supports_numerics_profile(profile)), profile


def test_native_and_foreign_stages_are_refused(harness, tmp_path):
    path = config1().program.write(tmp_path, "stage")
    for profile in ("", "nvcr.fx.v1", "nvcr.intconv.v2", "native"):
        code, message = load(harness, tmp_path, "stage", digest_of(path), profile)
        assert code == INCOMPATIBLE_PRECISION, (profile, message)


def test_exact_stage_without_an_sm100_device_is_refused(harness, tmp_path):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    path = config1().program.write(tmp_path, "stage")
    code, message = load(harness, tmp_path, "stage", digest_of(path), "nvcr.intconv.v1")
    assert code == INCOMPATIBLE_PRECISION, message


@pytest.mark.gpu
def test_digest_and_presence_refusals(harness, cuda, tmp_path):
    path = config1().program.write(tmp_path, "stage")
    assert load(harness, tmp_path, "stage", digest_of(path), "nvcr.intconv.v1")[0] == 0
    wrong = (ctypes.c_ubyte * 32)(*([0] * 32))
    code, message = load(harness, tmp_path, "stage", wrong, "nvcr.intconv.v1")
    assert code == int(ex.ErrorCode.digest_mismatch) + 1, message
    code, message = load(harness, tmp_path, "absent", digest_of(path), "nvcr.intconv.v1")
    assert code == int(ex.ErrorCode.missing_artifact) + 1, message


def run(harness, directory, component, digest, inputs: dict, outputs: dict, domain: int, repeats: int = 2):
    """outputs: name -> (c, h, w); returns name -> FP16 array."""
    keep = {k: np.ascontiguousarray(v, np.float32).astype(np.float16) for k, v in inputs.items()}
    in_names = (ctypes.c_char_p * len(keep))(*[k.encode() for k in keep])
    in_shapes = (ctypes.c_int32 * (3 * len(keep)))(*[d for v in keep.values() for d in v.shape])
    in_data = (ctypes.c_void_p * len(keep))(*[v.ctypes.data for v in keep.values()])
    results = {k: np.zeros(shape, np.float16) for k, shape in outputs.items()}
    out_names = (ctypes.c_char_p * len(results))(*[k.encode() for k in results])
    out_shapes = (ctypes.c_int32 * (3 * len(results)))(*[d for v in results.values() for d in v.shape])
    out_data = (ctypes.c_void_p * len(results))(*[v.ctypes.data for v in results.values()])
    message = ctypes.create_string_buffer(512)
    code = harness.ph_run(str(directory).encode(), component.encode(), digest, len(keep), in_names, in_shapes,
                          in_data, len(results), out_names, out_shapes, out_data, domain, repeats, message, 512)
    assert code == 0, message.value.decode()
    return results


@pytest.mark.gpu
@pytest.mark.parametrize("domain", [0, 1, 2], ids=["host", "pinned", "device"])
@pytest.mark.parametrize("case", ["config1", "ops_w16a16", "ops_w8a8"])
def test_submit_is_bit_exact(harness, cuda, oracle, tmp_path, domain, case):
    if case == "config1":
        layer = config1()
        program, inputs = layer.program, {"x": layer_input(layer, seed=1)}
    else:
        stream = SeededStream(17)
        program = op_program(stream).with_widths(*((16, 16) if case == "ops_w16a16" else (8, 8)))
        inputs = {"x": stream.tensor(70, 13, 21, 3.0)}
    path = program.write(tmp_path, "stage")
    rounded = [np.asarray(v, np.float32).astype(np.float16).astype(np.float32) for v in inputs.values()]
    expected = oracle.run(program, rounded)
    names = [program.tensor_names[i] for i in program.outputs]
    got = run(harness, tmp_path, "stage", digest_of(path), inputs,
              {n: e.shape for n, e in zip(names, expected)}, domain)
    for name, e in zip(names, expected):
        bad = count_differing(got[name].astype(np.float32), e.astype(np.float16).astype(np.float32))
        assert bad == 0, f"{case} {name}: {bad} of {e.size} values differ"
