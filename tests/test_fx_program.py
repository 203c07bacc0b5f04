"""nvcr.fx-program.v1 loading through the C ABI (no GPU): the behaviours of the
reference's own tests/fx_program_tests.cpp, and the same accept/refuse decision
and error code as the reference's fx::load_program (compiled into oracle/_ref)
on seeded valid programs and on targeted and random corruptions of them."""
from __future__ import annotations

import hashlib
import json
import random

import numpy as np
import pytest

from nvcr_b200.executor import ErrorCode, ExecutorError
from nvcr_b200.fx import load_program, program_digest
from tests.fx_programs import decoder_like, write_program
from tests.test_fx_oracle import one_op_program, reference_program_test_program


def load_status(directory, stage: str) -> int:
    try:
        load_program(directory, stage).close()
        return 0
    except ExecutorError as error:
        return int(error.code) + 1


def same_decision(fx_reference, directory, stage: str) -> int:
    expected, message = fx_reference.load_check(directory, stage)
    got = load_status(directory, stage)
    assert got == expected, message
    return got


def test_reference_program_test_behaviours(tmp_path):
    """tests/fx_program_tests.cpp:66-105 on this loader."""
    write_program(tmp_path, "t", reference_program_test_program(2))
    program = load_program(tmp_path, "t")
    assert [n.op for n in program.nodes] == ["im2col", "gemm", "pixel_shuffle", "pixel_unshuffle"]
    assert (program.tensor_count, program.input_count, program.output_count) == (6, 2, 2)
    digest = program_digest(tmp_path, "t")
    assert digest == program.digest == hashlib.sha256((tmp_path / "t.fxprog.json").read_bytes()).hexdigest()
    write_program(tmp_path, "t", reference_program_test_program(3))
    assert program_digest(tmp_path, "t") != digest  # the digest covers the weights

    bad_weight = reference_program_test_program(2)
    bad_weight["nodes"][1]["weights"] = bad_weight["nodes"][1]["weights"].astype(np.int32)
    bad_weight["nodes"][1]["weights"][0, 4] = 32640
    write_program(tmp_path, "t", bad_weight)
    assert load_status(tmp_path, "t") == ErrorCode.invalid_argument + 1
    bad_shift = reference_program_test_program(2)
    bad_shift["nodes"][1]["shift"] = np.array([32, 32], np.int32)
    write_program(tmp_path, "t", bad_shift)
    assert load_status(tmp_path, "t") == ErrorCode.invalid_argument + 1

    write_program(tmp_path, "t", reference_program_test_program(2))
    with open(tmp_path / "t.fxw", "ab") as data:
        data.write(b"x")
    assert load_status(tmp_path, "t") == ErrorCode.digest_mismatch + 1
    assert load_status(tmp_path, "absent") == ErrorCode.missing_artifact + 1
    (tmp_path / "t.fxw").unlink()
    assert load_status(tmp_path, "t") == ErrorCode.io_error + 1


def test_valid_programs_load_like_the_reference(fx_reference, tmp_path):
    for seed in range(12):
        program = decoder_like(np.random.default_rng(seed), channels=4 * (1 + seed % 3))
        write_program(tmp_path, "v", program)
        assert same_decision(fx_reference, tmp_path, "v") == 0
        loaded = load_program(tmp_path, "v")
        assert [n.op for n in loaded.nodes] == [n["op"] for n in program["nodes"]]
        assert [n.output for n in loaded.nodes] == [n["output"] for n in program["nodes"]]
        assert loaded.inputs == [program["tensors"][i] for i in program["inputs"]]
        assert loaded.outputs == [program["tensors"][i] for i in program["outputs"]]
        status, digest = fx_reference.program_digest(tmp_path, "v")
        assert status == 0 and loaded.digest == digest


def set_path(document: dict, path: tuple, value) -> None:
    target = document
    for key in path[:-1]:
        target = target[key]
    if value is _DELETE:
        if isinstance(target, list):
            del target[path[-1]]
        else:
            target.pop(path[-1], None)
    else:
        target[path[-1]] = value


_DELETE = object()


def node_index(document: dict, op: str) -> int:
    return next(i for i, n in enumerate(document["nodes"]) if n["op"] == op)


# (label, edit of the JSON document): each is compared with the reference.
TARGETED = [
    ("format", lambda d: set_path(d, ("format",), "nvcr.fx-program.v2")),
    ("profile", lambda d: set_path(d, ("profile",), "nvcr.intconv.v1")),
    ("no data", lambda d: set_path(d, ("data",), _DELETE)),
    ("slash in file", lambda d: set_path(d, ("data", "file"), "../x.fxw")),
    ("sha", lambda d: set_path(d, ("data", "sha256"), "0" * 64)),
    ("fa 25", lambda d: set_path(d, ("fa",), 25)),
    ("fa float", lambda d: set_path(d, ("fa",), 14.0)),
    ("no tensors", lambda d: set_path(d, ("tensors",), [])),
    ("channels 0", lambda d: set_path(d, ("tensors", 0, "channels"), 0)),
    ("channels 2^20+1", lambda d: set_path(d, ("tensors", 0, "channels"), (1 << 20) + 1)),
    ("tensor without name", lambda d: set_path(d, ("tensors", 1, "name"), _DELETE)),
    ("numeric name", lambda d: set_path(d, ("tensors", 1, "name"), 7)),
    ("inputs empty", lambda d: set_path(d, ("inputs",), [])),
    ("input out of range", lambda d: set_path(d, ("inputs", 0), 999)),
    ("output negative", lambda d: set_path(d, ("outputs", 0), -1)),
    ("delta h negative", lambda d: set_path(d, ("delta_tables", 0, "h"), -1)),
    ("delta shift 31", lambda d: set_path(d, ("delta_tables", 0, "shift"), 31)),
    ("delta dc count", lambda d: set_path(d, ("delta_tables", 0, "dc", 1), d["delta_tables"][0]["dc"][1] + 1)),
    ("dc outside data", lambda d: set_path(d, ("delta_tables", 0, "dc", 0), 1 << 40)),
    ("no nodes", lambda d: set_path(d, ("nodes",), [])),
    ("unknown op", lambda d: set_path(d, ("nodes", 0, "op"), "conv")),
    ("node without inputs", lambda d: set_path(d, ("nodes", 0, "inputs"), _DELETE)),
    ("too many inputs", lambda d: set_path(d, ("nodes", 1, "inputs"), [0, 2, 2])),
    ("gemm three residuals", lambda d: d["nodes"][node_index(d, "gemm")]["inputs"].extend([5, 5, 5])),
    ("gemm group 3", lambda d: set_path(d, ("nodes", node_index(d, "gemm"), "group"), 3)),
    ("gemm group 5", lambda d: set_path(d, ("nodes", node_index(d, "gemm"), "group"), 5)),
    ("gemm input shift 31", lambda d: set_path(d, ("nodes", node_index(d, "gemm"), "input_shift"), 31)),
    ("gemm table 9", lambda d: set_path(d, ("nodes", node_index(d, "gemm"), "delta_table"), 9)),
    ("gemm weights count", lambda d: set_path(d, ("nodes", node_index(d, "gemm"), "weights", 1), 3)),
    ("gemm bias offset", lambda d: set_path(d, ("nodes", node_index(d, "gemm"), "bias", 0), -8)),
    ("depthwise shift count", lambda d: set_path(d, ("nodes", node_index(d, "depthwise3x3"), "shift", 1), 1)),
    ("mul shift 32", lambda d: set_path(d, ("nodes", 1, "shift"), 32)),
    ("mul factor channels", lambda d: set_path(d, ("nodes", 1, "inputs"), [0, 4])),
    ("affine alpha", lambda d: set_path(d, ("nodes", node_index(d, "affine"), "alpha"), (1 << 24) + 1)),
    ("affine beta", lambda d: set_path(d, ("nodes", node_index(d, "affine"), "beta"), -(1 << 52) - 1)),
    ("affine beta ok", lambda d: set_path(d, ("nodes", node_index(d, "affine"), "beta"), 1 << 52)),
    ("sat_table odd", lambda d: set_path(d, ("nodes", node_index(d, "sat_table"), "table", 1),
                                         d["nodes"][node_index(d, "sat_table")]["table"][1] - 1)),
    ("sat_table top", lambda d: set_path(d, ("nodes", node_index(d, "sat_table"), "top"), 1 << 31)),
    ("delta node table -1", lambda d: set_path(d, ("nodes", node_index(d, "delta"), "delta_table"), -1)),
    ("clamp lo > hi", lambda d: set_path(d, ("nodes", node_index(d, "clamp"), "lo"), (1 << 21))),
    ("clamp hi int32", lambda d: set_path(d, ("nodes", node_index(d, "clamp"), "hi"), 1 << 31)),
    ("slice end", lambda d: set_path(d, ("nodes", node_index(d, "slice"), "end"), 999)),
    ("slice begin = end", lambda d: set_path(d, ("nodes", node_index(d, "slice"), "begin"),
                                             d["nodes"][node_index(d, "slice")]["end"])),
    ("shuffle factor 1", lambda d: set_path(d, ("nodes", node_index(d, "pixel_shuffle"), "factor"), 1)),
    ("shuffle factor 17", lambda d: set_path(d, ("nodes", node_index(d, "pixel_shuffle"), "factor"), 17)),
    ("im2col 2x2 stride 1", lambda d: set_path(d, ("nodes", node_index(d, "im2col"), "kernel"), 2)),
    ("im2col kernel 4", lambda d: set_path(d, ("nodes", node_index(d, "im2col"), "kernel"), 4)),
    ("param_row input", lambda d: set_path(d, ("nodes", 0, "inputs"), [0])),
    ("output out of range", lambda d: set_path(d, ("nodes", 0, "output"), 999)),
]


@pytest.mark.parametrize("label,edit", TARGETED, ids=[label for label, _ in TARGETED])
def test_targeted_refusals_match_reference(fx_reference, tmp_path, label, edit):
    program = decoder_like(np.random.default_rng(3))
    write_program(tmp_path, "m", program, mutate=edit)
    same_decision(fx_reference, tmp_path, "m")


def test_out_of_bound_arrays_match_reference(fx_reference, tmp_path):
    """Weight, bias, shift and table values one past each load-time bound."""
    base = decoder_like(np.random.default_rng(5))
    gemm = next(i for i, n in enumerate(base["nodes"]) if n["op"] == "gemm")
    depthwise = next(i for i, n in enumerate(base["nodes"]) if n["op"] == "depthwise3x3")
    edits = [
        (gemm, "weights", np.int16, -32640), (gemm, "weights", np.int16, 32639), (gemm, "weights", np.int16, -32639),
        (gemm, "bias", np.int64, (1 << 52) + 1), (gemm, "bias", np.int64, -(1 << 52)),
        (gemm, "shift", np.int32, 0), (gemm, "shift", np.int32, 31),
        (depthwise, "weights", np.int32, (1 << 24) + 1), (depthwise, "weights", np.int32, -(1 << 24)),
        (depthwise, "shift", np.int32, 0), (depthwise, "shift", np.int32, 32),
        (depthwise, "bias", np.int64, -(1 << 52) - 1),
        (0, "rows", np.int64, (1 << 24) + 1), (0, "rows", np.int64, -(1 << 24)),
    ]
    outcomes = set()
    for index, (node, field, dtype, value) in enumerate(edits):
        program = {**base, "nodes": [dict(n) for n in base["nodes"]]}
        array = np.array(program["nodes"][node][field], dtype=np.int64).astype(dtype)
        array.reshape(-1)[index % array.size] = value
        program["nodes"][node][field] = array
        write_program(tmp_path, "b", program)
        outcomes.add(same_decision(fx_reference, tmp_path, "b"))
    assert outcomes == {0, ErrorCode.invalid_argument + 1}


def random_value(rng: random.Random):
    return rng.choice([0, -1, 1, 2, 3, 31, 32, 1 << 20, (1 << 20) + 1, 1 << 31, -(1 << 40), 1.5, "x", None, [], {},
                       [0, 1], [0, 1 << 40], True])


def test_random_corruptions_match_reference(fx_reference, tmp_path):
    rng = random.Random(4242)
    program = decoder_like(np.random.default_rng(11))
    write_program(tmp_path, "base", program)
    document = json.loads((tmp_path / "base.fxprog.json").read_text())
    outcomes = {}
    for trial in range(300):
        edited = json.loads(json.dumps(document))
        for _ in range(rng.randint(1, 2)):
            def entries(key):
                value = edited.get(key)
                return [e for e in value if isinstance(e, dict) and e] if isinstance(value, list) else []

            nodes, others = entries("nodes"), entries("tensors") + entries("delta_tables")
            if rng.random() < 0.25 or not (nodes or others):
                target = edited
                key = rng.choice(["fa", "tensors", "inputs", "outputs", "delta_tables", "nodes", "format"])
            else:
                target = rng.choice(nodes if (rng.random() < 0.6 and nodes) or not others else others)
                key = rng.choice(sorted(target.keys()))
            if rng.random() < 0.15:
                target.pop(key, None)
            else:
                target[key] = random_value(rng)
        (tmp_path / "r.fxw").write_bytes((tmp_path / "base.fxw").read_bytes())
        edited["data"]["file"] = "r.fxw"
        (tmp_path / "r.fxprog.json").write_text(json.dumps(edited))
        status = same_decision(fx_reference, tmp_path, "r")
        outcomes[status] = outcomes.get(status, 0) + 1
    assert outcomes.get(ErrorCode.invalid_argument + 1, 0) > 100  # most corruptions are refused


def test_malformed_json_matches_reference(fx_reference, tmp_path):
    rng = random.Random(99)
    program = one_op_program({"op": "add"}, [1, 1], 1)
    write_program(tmp_path, "j", program)
    text = (tmp_path / "j.fxprog.json").read_text()
    for trial in range(120):
        cut = rng.randrange(len(text))
        broken = text[:cut] + rng.choice(["", "}", "{", ",", "\"", "]", "nul", "1e999"]) + text[cut + rng.randint(0, 3):]
        (tmp_path / "k.fxprog.json").write_text(broken)
        same_decision(fx_reference, tmp_path, "k")


def test_executor_extents_match_oracle_shapes(fx_oracle, tmp_path):
    """The executor's host planning (no GPU): output extents equal the oracle's
    output shapes on seeded single ops and whole programs, and inputs the
    oracle refuses for their shapes are refused the same way."""
    from nvcr_b200.fx import FxExecutor
    from tests.fx_programs import decoder_like_inputs
    from tests.test_fx_oracle import random_single_op

    rng = np.random.default_rng(2026)
    cases = []
    for _ in range(300):
        op, ins, out, inputs, tables = random_single_op(rng)
        cases.append((one_op_program(op, ins, out, tables), inputs))
    for seed in range(20):
        generator = np.random.default_rng(seed)
        program = decoder_like(generator, channels=4 * (1 + seed % 4))
        cases.append((program, decoder_like_inputs(generator, program, 1 + seed % 9, 2 + seed % 5)))
    cases.append((one_op_program({"op": "add"}, [2, 2], 2),
                  [np.zeros((2, 2, 2), np.int32), np.zeros((2, 2, 3), np.int32)]))
    cases.append((one_op_program({"op": "pixel_unshuffle", "factor": 2}, [1], 4), [np.zeros((1, 3, 4), np.int32)]))
    for index, (program, inputs) in enumerate(cases):
        write_program(tmp_path, f"e{index % 5}", program)
        status, outputs, _ = fx_oracle.run(program, inputs)
        with load_program(tmp_path, f"e{index % 5}") as loaded, FxExecutor(loaded) as executor:
            try:
                extents = executor.infer_output_extents([x.shape for x in inputs])
            except ExecutorError as error:
                assert status == ErrorCode.invalid_argument + 1 and error.code == ErrorCode.invalid_argument
                continue
            if status == 0:
                assert extents == [y.shape for y in outputs]
            else:
                assert status != ErrorCode.invalid_argument + 1  # only value-dependent failures remain
