"""CPU-side checks of the product library and its host logic (no GPU needed):
the C ABI loads and exports every function include/nvcr_sm100.h declares, the
profile negotiation answers as the reference's, and program files are accepted
or refused exactly as the reference's loader does."""
from __future__ import annotations

import json
import re
from pathlib import Path

import numpy as np
import pytest

from nvcr_b200 import executor as ex
from nvcr_b200.program import OpKind, Program, SeededStream
from tests.programs import data_movement_program, op_program

HEADER = Path(__file__).resolve().parent.parent / "include" / "nvcr_sm100.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(nvcr_sm100_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_function(built_library):
    lib = ex.library()
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} is declared but not exported"
    assert set(names) == set(ex.EXPORTS)
    assert lib.nvcr_sm100_abi_version() == 1


def test_is_normative_matches_reference_rule(built_library):
    assert ex.is_normative("") is False
    assert ex.is_normative("nvcr.intconv.v1") is True
    with pytest.raises(ex.ExecutorError) as error:
        ex.is_normative("nvcr.fx.v1")
    assert error.value.code == ex.ErrorCode.incompatible_precision


def test_supports_profile_refuses_other_profiles(built_library):
    assert ex.supports_numerics_profile("nvcr.fx.v1") is False
    assert ex.supports_numerics_profile("native") is False


def _write_variants(tmp_path: Path):
    """A valid program, then malformed variants of its JSON and weights."""
    stream = SeededStream(7)
    program = op_program(stream).with_widths(8, 16)
    good = program.write(tmp_path / "good", "ops")
    base = json.loads(good.read_text())
    variants = {"good": good}

    def variant(name, mutate, weights=None):
        directory = tmp_path / name
        directory.mkdir()
        document = json.loads(json.dumps(base))
        mutate(document)
        blob = (tmp_path / "good" / "ops.detw").read_bytes() if weights is None else weights
        (directory / "ops.detw").write_bytes(blob)
        path = directory / "ops.detprog.json"
        path.write_text(json.dumps(document))
        variants[name] = path

    variant("wrong_format", lambda d: d.update(format="other"))
    variant("wrong_version", lambda d: d.update(version=2))
    variant("fx_profile", lambda d: d.update(numerics="nvcr.fx.v1"))
    variant("digest", lambda d: d["weights"].update(sha256="0" * 64))
    variant("weights_path", lambda d: d["weights"].update(file="../ops.detw"))
    variant("unknown_op", lambda d: d["nodes"][1].update(op="gelu"))
    variant("undefined_tensor", lambda d: d["nodes"][1].update(input="nope"))
    variant("duplicate_output", lambda d: d["nodes"][2].update(output=d["nodes"][1]["output"]))
    variant("bad_widths", lambda d: d["nodes"][0].update(integer={"weight_bits": 4, "activation_bits": 8}))
    variant("widths_on_sigmoid", lambda d: d["nodes"][2].update(integer={"weight_bits": 8, "activation_bits": 8}))
    variant("inexact_scalar", lambda d: d["nodes"][1].update(value=0.1))
    variant("weights_overflow", lambda d: d["nodes"][0].update(weight_offset=10 ** 9))
    variant("bad_block", lambda d: d["nodes"][8].update(block=0))
    variant("depthwise_mismatch", lambda d: d["nodes"][4].update(out_channels=5))
    variant("float_channels", lambda d: d["nodes"][0].update(in_channels=70.0))
    variant("missing_output", lambda d: d["outputs"].append({"name": "ghost"}))
    variant("short_weights", lambda d: d["weights"].update(count=d["weights"]["count"] + 1))
    return variants


def test_loader_accepts_and_refuses_like_the_reference(built_library, reference, tmp_path):
    """Without a GPU, creation reaches the device check only after the program
    loaded; a refused program fails earlier with the loader's code."""
    loader_codes = {ex.ErrorCode.invalid_argument, ex.ErrorCode.io_error, ex.ErrorCode.digest_mismatch}
    for name, path in _write_variants(tmp_path).items():
        ref_code, ref_message = reference.load_check(path)
        try:
            executor = ex.CudaExecutor.create(path)
            ours = None
            executor.close()
        except ex.ExecutorError as error:
            ours = error.code if error.code in loader_codes else None
        expected = None if ref_code == 0 else ex.ErrorCode(ref_code - 1)
        assert ours == expected, f"{name}: reference {expected} ({ref_message}), ours {ours}"


def test_load_normative_checks_presence_and_digest(built_library, tmp_path):
    stream = SeededStream(7)
    path = data_movement_program().write(tmp_path, "stage")
    with pytest.raises(ex.ExecutorError) as error:
        ex.CudaExecutor.load_normative(tmp_path, "absent", "0" * 64)
    assert error.value.code == ex.ErrorCode.missing_artifact
    with pytest.raises(ex.ExecutorError) as error:
        ex.CudaExecutor.load_normative(tmp_path, "stage", "0" * 64)
    assert error.value.code == ex.ErrorCode.digest_mismatch
    with pytest.raises(ex.ExecutorError) as error:
        ex.CudaExecutor.load_normative(tmp_path, "stage", "")
    assert error.value.code == ex.ErrorCode.invalid_argument


def test_program_handle_infers_extents_like_the_reference(built_library, reference, tmp_path):
    """Shape inference needs no GPU; it must agree with the reference's
    infer_output_extents, errors included."""
    stream = SeededStream(3)
    program = op_program(stream)
    path = program.write(tmp_path)
    loaded = ex.LoadedProgram.load(path)
    assert loaded.input_names == ["x"] and loaded.output_names == ["sum", "pointwise"]
    for extent in [(70, 33, 47), (70, 2, 64), (70, 11, 18), (70, 1, 1), (70, 4, 2), (71, 5, 5), (70, 0, 4),
                   (70, 5, -1)]:
        ref_code, ref_value = reference.infer_extents(path, [extent])
        try:
            ours = loaded.infer_output_extents([extent])
            assert ref_code == 0, f"{extent}: reference refused ({ref_value}), ours accepted"
            assert ours == ref_value, extent
        except ex.ExecutorError as error:
            assert ref_code == int(error.code) + 1, f"{extent}: reference {ref_code}, ours {error}"
    data = data_movement_program().write(tmp_path / "dm")
    loaded = ex.LoadedProgram.load(data)
    for extents in [[(5, 12, 20), (20, 1, 1), (1, 5, 7)], [(5, 12, 20), (20, 1, 2), (1, 5, 7)],
                    [(5, 11, 20), (20, 1, 1), (1, 5, 7)], [(5, 12, 20), (20, 1, 1), (1, 7, 7)]]:
        ref_code, ref_value = reference.infer_extents(data, extents)
        try:
            assert loaded.infer_output_extents(extents) == ref_value and ref_code == 0, extents
        except ex.ExecutorError as error:
            assert ref_code == int(error.code) + 1, f"{extents}: reference {ref_code}, ours {error}"


def test_program_handle_without_gpu_refuses_executor(built_library, tmp_path):
    """Creating an executor needs an sm_100 device: on a host without one the
    call fails cleanly with a backend or target error, never a crash."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    loaded = ex.LoadedProgram.from_program(data_movement_program())
    with pytest.raises(ex.ExecutorError) as error:
        loaded.executor()
    assert error.value.code in (ex.ErrorCode.backend_error, ex.ErrorCode.incompatible_target)


def test_stack_profile_report_folds_blocks():
    """The per-op report folds DepthConvBlock indices and sums per run."""
    from nvcr_b200.stack_profile import report

    segments = [
        {"label": "integer_conv:i.dec.dec_1.3.ffn.1.sum", "kernel": "integer_conv", "ms": 0.1, "ops": 1e10, "bytes": 1e8},
        {"label": "integer_conv:i.dec.dec_1.4.ffn.1.sum", "kernel": "integer_conv", "ms": 0.1, "ops": 1e10, "bytes": 1e8},
        {"label": "conv:i.dec.dec_1.4.dc.2", "kernel": "conv", "ms": 0.05, "ops": 0.0, "bytes": 5e7},
    ]
    text = report(segments, 1.0)
    assert "total 0.250 ms per run" in text
    assert "| integer_conv:i.dec.dec_1.ffn.1.sum | 2 | 0.200 | 100.0 | 1000 |" in text
    assert "| conv:i.dec.dec_1.dc.2 | 1 | 0.050 | 0.0 | 1000 |" in text


def _corruption_value(rng):
    return rng.choice([0, -1, 1, 2, 3, 16, 64, 65, 70, 1 << 20, 1 << 40, -(1 << 31), 0.5, 1.0, 0.1, 1e39, "x",
                       "x_in", None, [], {}, [1, 1], [3, 3], [0, 1], [1, 1, 1, 1], [-1, 0, 0, 0], [1, 2, 3], True,
                       False, {"weight_bits": 8, "activation_bits": 8}, {"weight_bits": 16}])


def test_random_corruptions_load_like_the_reference(built_library, reference, tmp_path):
    """Seeded random edits of a valid program's JSON (a node field set to an odd
    value or removed, a top-level member replaced): every edit is accepted or
    refused with the reference loader's code, and an accepted program infers the
    reference's output extents."""
    import random

    rng = random.Random(2027)
    stream = SeededStream(5)
    program = op_program(stream).with_widths(8, 16)
    base_path = program.write(tmp_path / "base", "ops")
    base = json.loads(base_path.read_text())
    blob = (tmp_path / "base" / "ops.detw").read_bytes()
    directory = tmp_path / "edit"
    directory.mkdir()
    (directory / "ops.detw").write_bytes(blob)
    outcomes = {}
    for trial in range(400):
        document = json.loads(json.dumps(base))
        for _ in range(rng.randint(1, 2)):
            if rng.random() < 0.2:
                key = rng.choice(["inputs", "outputs", "nodes", "name", "numerics", "version", "weights"])
                if rng.random() < 0.3:
                    document.pop(key, None)
                else:
                    document[key] = _corruption_value(rng)
                continue
            nodes = document.get("nodes")
            if not isinstance(nodes, list) or not nodes or not isinstance(nodes[0], dict):
                continue
            node = rng.choice([n for n in nodes if isinstance(n, dict)])
            key = rng.choice(sorted(node.keys()) + ["integer", "inputs", "input", "depthwise"])
            if rng.random() < 0.2:
                node.pop(key, None)
            else:
                node[key] = _corruption_value(rng)
        path = directory / "ops.detprog.json"
        path.write_text(json.dumps(document))
        ref_code, ref_message = reference.load_check(path)
        try:
            loaded = ex.LoadedProgram.load(path)
            ours = 0
        except ex.ExecutorError as error:
            ours = int(error.code) + 1
            loaded = None
        assert ours == ref_code, f"trial {trial}: reference {ref_code} ({ref_message}), ours {ours}"
        outcomes[ours] = outcomes.get(ours, 0) + 1
        if loaded is not None:
            for extent in [(70, 11, 18), (70, 3, 5)]:
                if len(loaded.input_names) != 1:
                    break
                code, value = reference.infer_extents(path, [extent])
                try:
                    ours_extents = loaded.infer_output_extents([extent])
                except ex.ExecutorError as error:
                    assert code == int(error.code) + 1, (trial, extent, code, str(error))
                else:
                    assert code == 0 and ours_extents == value, (trial, extent, code, value)
            loaded.close()
    assert outcomes.get(0, 0) > 20 and outcomes.get(int(ex.ErrorCode.invalid_argument) + 1, 0) > 150, outcomes
