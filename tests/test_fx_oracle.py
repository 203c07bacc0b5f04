"""The nvcr.fx.v1 oracle (no GPU): pinned to the hand-computed vectors of the
reference's own tests (tests/fx_reference_tests.cpp, tests/fx_program_tests.cpp)
and, integer for integer and failure for failure, to the reference's fx.cpp and
fx_program.cpp compiled from its sources into oracle/_ref: the conformance
suite's per-op edge vectors (docs/spec/numerics-fx-v1.md section 7.1), single-op
programs on seeded random shapes, and seeded whole programs that use every op."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.fx import DIGIT2_MAX, GEMM_LIMIT, INVALID, STAGE_FAILURE, STORED_MAX
from tests.fx_programs import decoder_like, decoder_like_inputs, delta_table, gemm_node, write_program


def rsr(a: int, s: int) -> int:
    """The spec's rsr on Python integers (floor division is exact here)."""
    return a if s == 0 else (a + (1 << (s - 1))) >> s


def pixel(*channels: int) -> np.ndarray:
    return np.array(channels, np.int32).reshape(len(channels), 1, 1)


def one_op_program(op: dict, in_channels: list[int], out_channels: int, tables=()) -> dict:
    """A program of one node reading tensors 0..k-1 and writing tensor k."""
    names = [(f"in{i}", c) for i, c in enumerate(in_channels)] + [("out", out_channels)]
    node = dict(op)
    node["inputs"] = list(range(len(in_channels)))
    node["output"] = len(in_channels)
    return {"fa": 14, "tensors": names, "inputs": list(range(len(in_channels))), "outputs": [len(in_channels)],
            "delta_tables": list(tables), "nodes": [node]}


def agree(fx_oracle, fx_reference, tmp_path, program: dict, inputs, stage: str = "t"):
    """Runs both sides; asserts they agree and returns (status, outputs, reason)."""
    write_program(tmp_path, stage, program)
    loaded, message = fx_reference.load_check(tmp_path, stage)
    assert loaded == 0, message
    ours = fx_oracle.run(program, inputs)
    theirs = fx_reference.run(tmp_path, stage, inputs)
    assert ours[0] == theirs[0], (ours[2], theirs[2])
    if ours[0] == 0:
        assert len(ours[1]) == len(theirs[1])
        for mine, expected in zip(ours[1], theirs[1]):
            assert mine.shape == expected.shape
            assert np.array_equal(mine, expected)
    else:
        assert ours[2] in theirs[2], (ours[2], theirs[2])
    return ours


# -- the reference's hand-computed vectors -------------------------------------

def test_reference_rounding_and_table_vectors(fx_oracle):
    """tests/fx_reference_tests.cpp:30-51."""
    assert fx_oracle.rsr(5, 1) == 3 and fx_oracle.rsr(-5, 1) == -2
    assert fx_oracle.rsr(-6, 2) == -1 and fx_oracle.rsr(7, 0) == 7
    table = {"h": 4, "shift": 1, "dc": [10, 20, 30, 40, 50]}
    expected = {-5: 0, -4: 10, -3: 10, -2: 20, 0: 30, 4: 54, 5: 5}
    assert {r: fx_oracle.delta_act(r, table) for r in expected} == expected
    y = fx_oracle.sat_table(pixel(-3, -2, 1, 2), [1, 2, 3, 4], 99)
    assert y.ravel().tolist() == [0, 1, 4, 99]


def test_reference_gemm_vectors(fx_oracle):
    """tests/fx_reference_tests.cpp:54-80."""
    op = {"in_channels": 1, "out_channels": 1, "group": 1, "input_shift": 1, "weights": [[3]], "bias": [0],
          "shift": [1]}
    assert fx_oracle.gemm(op, pixel(5)).item() == 5
    op.update(weights=[[1]], input_shift=0)
    assert fx_oracle.gemm(op, pixel(1 << 20)).item() == 16320
    op.update(in_channels=2, weights=[[DIGIT2_MAX, DIGIT2_MAX]])
    status, _, reason = fx_oracle.run(one_op_program(dict(op, op="gemm", delta_table=-1), [2], 1),
                                      [pixel(DIGIT2_MAX, DIGIT2_MAX)])
    assert status == STAGE_FAILURE and reason == "gemm pre-activation out of range"
    op.update(in_channels=1, out_channels=2, weights=[[1], [2]], bias=[0, 0], shift=[1, 1], group=2)
    assert fx_oracle.gemm(op, pixel(4), [pixel(10)]).item() == 16


def test_reference_elementwise_vectors(fx_oracle):
    """tests/fx_reference_tests.cpp:83-96."""
    dw = {"weights": [[0, 0, 0, 0, 4, 0, 0, 0, 0]], "bias": [2], "shift": [1]}
    assert fx_oracle.depthwise3x3(dw, pixel(3)).item() == 7
    assert fx_oracle.mul(pixel(3, 5), pixel(2), 1).ravel().tolist() == [3, 5]
    plane = np.array([[[3, 5]]], np.int32)
    assert fx_oracle.mul(plane, pixel(4), 2).ravel().tolist() == [3, 5]
    assert fx_oracle.affine(pixel(1 << 14), 3, 1 << 14, 1).item() == 1 << 15
    assert fx_oracle.add(pixel(1 << 30), pixel(0)).item() == 1 << 30
    status, _, reason = fx_oracle.run(one_op_program({"op": "add"}, [1, 1], 1), [pixel(1 << 30), pixel(1)])
    assert status == STAGE_FAILURE and reason == "add output out of range"


def reference_program_test_program(weight: int) -> dict:
    """The program of tests/fx_program_tests.cpp:38-63: im2col 3x3 -> gemm
    (centre tap `weight`, 2 rows summed, delta table h 2) and a
    pixel_shuffle / pixel_unshuffle round trip."""
    w = np.zeros((2, 9), np.int16)
    w[0, 4] = weight
    w[1, 4] = 1
    return {"fa": 14, "tensors": [("x", 1), ("cols", 9), ("y", 1), ("q", 4), ("up", 1), ("z", 4)],
            "inputs": [0, 3], "outputs": [2, 5],
            "delta_tables": [{"h": 2, "shift": 1, "dc": np.array([7, 7, 7], np.int16)}],
            "nodes": [{"op": "im2col", "inputs": [0], "output": 1, "kernel": 3, "stride": 1},
                      {"op": "gemm", "inputs": [1], "output": 2, "in_channels": 9, "out_channels": 2, "group": 2,
                       "input_shift": 0, "delta_table": 0, "weights": w, "bias": np.zeros(2, np.int64),
                       "shift": np.array([1, 1], np.int32)},
                      {"op": "pixel_shuffle", "inputs": [3], "output": 4, "factor": 2},
                      {"op": "pixel_unshuffle", "inputs": [4], "output": 5, "factor": 2}]}


def test_reference_program_vectors(fx_oracle, fx_reference, tmp_path):
    """tests/fx_program_tests.cpp:66-87: the values, and the same on the live reference."""
    program = reference_program_test_program(2)
    q = pixel(1, 2, 3, 4)
    status, outputs, _ = agree(fx_oracle, fx_reference, tmp_path, program, [pixel(5), q])
    assert status == 0 and outputs[0].item() == 8 and np.array_equal(outputs[1], q)
    status, _, reason = agree(fx_oracle, fx_reference, tmp_path, program, [pixel((1 << 30) + 1), q])
    assert status == STAGE_FAILURE and reason == "input value out of range"


# -- scalar rules against the live reference ------------------------------------

def test_rsr_matches_reference_on_ties_and_extremes(fx_oracle, fx_reference):
    values = set()
    for s in range(0, 32):
        half = 1 << max(0, s - 1)
        for base in (0, 1 << s, 3 << s, -(1 << s), -(5 << s), 1 << 52, -(1 << 52)):
            for delta in (-half - 1, -half, -half + 1, -1, 0, 1, half - 1, half, half + 1):
                values.add((base + delta, s))
    rng = np.random.default_rng(7)
    for a, s in zip(rng.integers(-(1 << 60), 1 << 60, 2000), rng.integers(0, 32, 2000)):
        values.add((int(a), int(s)))
    for a, s in values:
        assert fx_oracle.rsr(a, s) == fx_reference.rsr(a, s) == rsr(a, s), (a, s)


@pytest.mark.parametrize("h,shift", [(0, 0), (1, 0), (4, 1), (13, 2), (108544, 3), (1000, 5)])
def test_delta_table_edges_match_reference(fx_oracle, fx_reference, h, shift):
    table = delta_table(np.random.default_rng(h + shift), h, shift) if h else {"h": 0, "shift": 0, "dc": [123]}
    points = {-h - 2, -h - 1, -h, -h + 1, -1, 0, 1, h - 1, h, h + 1, h + 2, 1 << 29, -(1 << 29)}
    for edge in range(-h, h + 1, max(1, 1 << shift)):  # bin boundaries
        points.update({edge - 1, edge, edge + (1 << shift) - 1})
    for r in sorted(points):
        assert fx_oracle.delta_act(r, table) == fx_reference.delta_act(r, table), r


# -- the conformance suite's per-op edge vectors (spec 7.1), through programs ----

def gemm_1x1(bias: int, shift: int = 1, input_shift: int = 0, weight: int = 1, table: int = -1) -> dict:
    return {"op": "gemm", "in_channels": 1, "out_channels": 1, "group": 1, "input_shift": input_shift,
            "delta_table": table, "weights": np.array([[weight]], np.int16), "bias": np.array([bias], np.int64),
            "shift": np.array([shift], np.int32)}


def test_gemm_pre_activation_threshold(fx_oracle, fx_reference, tmp_path):
    """|r| = 2^29 - 2 passes, |r| = 2^29 - 1 fails, on both signs."""
    for bias in (2 * GEMM_LIMIT - 2, 2 * GEMM_LIMIT, -(2 * GEMM_LIMIT - 2), -(2 * GEMM_LIMIT), 2 * GEMM_LIMIT - 1,
                 -(2 * GEMM_LIMIT) + 1):
        r = rsr(bias, 1)
        status, outputs, reason = agree(fx_oracle, fx_reference, tmp_path,
                                        one_op_program(gemm_1x1(bias), [1], 1), [pixel(0)])
        if abs(r) >= GEMM_LIMIT:
            assert status == STAGE_FAILURE and reason == "gemm pre-activation out of range", bias
        else:
            assert status == 0 and outputs[0].item() == r, bias


def test_gemm_input_saturation_edges(fx_oracle, fx_reference, tmp_path):
    """Inputs whose rounded value is +-D2 and +-(D2 + 1), at input shifts 0 and 3."""
    for input_shift in (0, 3):
        for value in (DIGIT2_MAX, DIGIT2_MAX + 1, -DIGIT2_MAX, -DIGIT2_MAX - 1):
            for tie in (0, -(1 << input_shift) // 2, (1 << input_shift) // 2 - 1):
                x = (value << input_shift) + tie if input_shift else value
                status, outputs, _ = agree(fx_oracle, fx_reference, tmp_path,
                                           one_op_program(gemm_1x1(0, shift=1, input_shift=input_shift), [1], 1),
                                           [pixel(x)])
                clamped = max(-DIGIT2_MAX, min(DIGIT2_MAX, rsr(x, input_shift)))
                assert status == 0 and outputs[0].item() == rsr(clamped, 1)


def test_stored_bound_threshold_in_every_writing_op(fx_oracle, fx_reference, tmp_path):
    """2^30 is stored, 2^30 + 1 (and -2^30 - 1) fail: gemm (through a residual),
    depthwise, mul, affine and add."""
    top = STORED_MAX
    cases = [
        # (op, input channels, output channels, inputs, failing?)
        (gemm_1x1(0), [1, 1], 1, [pixel(0), pixel(top)], False),
        (gemm_1x1(2), [1, 1], 1, [pixel(0), pixel(top)], True),
        (gemm_1x1(-2), [1, 1], 1, [pixel(0), pixel(-top)], True),
        ({"op": "depthwise3x3", "weights": np.array([[0, 0, 0, 0, 1, 0, 0, 0, 0]], np.int32),
          "bias": np.array([top], np.int64), "shift": np.array([0], np.int32)}, [1], 1, [pixel(0)], False),
        ({"op": "depthwise3x3", "weights": np.array([[0, 0, 0, 0, 1, 0, 0, 0, 0]], np.int32),
          "bias": np.array([top], np.int64), "shift": np.array([0], np.int32)}, [1], 1, [pixel(1)], True),
        ({"op": "mul", "shift": 1}, [1, 1], 1, [pixel(top), pixel(2)], False),
        ({"op": "mul", "shift": 1}, [1, 1], 1, [pixel(top), pixel(3)], True),
        ({"op": "mul", "shift": 0}, [1, 1], 1, [pixel(-top), pixel(-1)], False),
        ({"op": "affine", "alpha": 2, "beta": 1, "shift": 1}, [1], 1, [pixel(top - 1)], False),
        ({"op": "affine", "alpha": 2, "beta": 2, "shift": 1}, [1], 1, [pixel(top)], True),
        ({"op": "affine", "alpha": -1, "beta": -1, "shift": 0}, [1], 1, [pixel(top)], True),
        ({"op": "add"}, [1, 1], 1, [pixel(-top), pixel(0)], False),
        ({"op": "add"}, [1, 1], 1, [pixel(-top), pixel(-1)], True),
    ]
    for op, ins, out, inputs, failing in cases:
        status, _, reason = agree(fx_oracle, fx_reference, tmp_path, one_op_program(op, ins, out), inputs)
        assert (status == STAGE_FAILURE) == failing, (op["op"], reason)
        if failing:
            assert reason.endswith("output out of range")


def test_sat_table_and_param_row_edges(fx_oracle, fx_reference, tmp_path):
    n = 5
    table = np.arange(100, 100 + 2 * n, dtype=np.int32)
    xs = pixel(-n - 1, -n, -n + 1, -1, 0, n - 1, n, n + 1, -(1 << 30), 1 << 30)
    status, outputs, _ = agree(fx_oracle, fx_reference, tmp_path,
                               one_op_program({"op": "sat_table", "table": table, "top": -7}, [10], 10), [xs])
    assert status == 0 and outputs[0].ravel().tolist() == [0, 100, 101, 104, 105, 109, -7, -7, 0, -7]
    rows = np.arange(12, dtype=np.int64).reshape(4, 3) - 6
    program = one_op_program({"op": "param_row", "rows": rows}, [1], 3)
    for q in (-1, 0, 3, 4, 1 << 30):
        status, outputs, reason = agree(fx_oracle, fx_reference, tmp_path, program, [pixel(q)])
        if 0 <= q < 4:
            assert status == 0 and outputs[0].ravel().tolist() == rows[q].tolist()
        else:
            assert status == STAGE_FAILURE and reason == "qp outside the parameter table"


def test_im2col_of_thin_inputs_matches_reference(fx_oracle, fx_reference, tmp_path):
    """Output sizes use C++ truncating division: a 2x2 stride-2 im2col of a
    1-pixel-high or -wide input keeps one row or column."""
    rng = np.random.default_rng(5)
    for k, stride in ((2, 2), (3, 2), (3, 1)):
        for h, w in ((1, 1), (1, 5), (4, 1), (2, 3), (3, 3)):
            x = rng.integers(-100, 100, (2, h, w)).astype(np.int32)
            status, outputs, _ = agree(fx_oracle, fx_reference, tmp_path,
                                       one_op_program({"op": "im2col", "kernel": k, "stride": stride}, [2], 2 * k * k),
                                       [x], stage=f"i{k}{stride}{h}{w}")
            assert status == 0 and outputs[0].shape[1:] == (int((h + 2 * (k == 3) - k) / stride) + 1,
                                                            int((w + 2 * (k == 3) - k) / stride) + 1)


def test_run_time_refusals_match_reference(fx_oracle, fx_reference, tmp_path):
    """Shapes a valid program cannot run on: both sides refuse (invalid_argument)."""
    cases = [
        (one_op_program({"op": "add"}, [2, 2], 2), [np.zeros((2, 2, 2), np.int32), np.zeros((2, 2, 3), np.int32)]),
        (one_op_program({"op": "add"}, [2, 2], 2), [np.zeros((2, 2, 2), np.int32)]),
        (one_op_program({"op": "add"}, [2, 2], 2), [np.zeros((3, 2, 2), np.int32), np.zeros((2, 2, 2), np.int32)]),
        (one_op_program({"op": "crop_like"}, [1, 1], 1), [np.zeros((1, 2, 2), np.int32), np.zeros((1, 3, 2), np.int32)]),
        (one_op_program({"op": "pixel_unshuffle", "factor": 2}, [1], 4), [np.zeros((1, 3, 4), np.int32)]),
        (one_op_program({"op": "mul", "shift": 0}, [2, 1], 2), [np.zeros((2, 2, 2), np.int32), np.zeros((1, 2, 1), np.int32)]),
        (one_op_program({"op": "slice", "begin": 0, "end": 1}, [2], 2), [np.zeros((2, 1, 1), np.int32)]),
    ]
    for index, (program, inputs) in enumerate(cases):
        status, _, _ = agree(fx_oracle, fx_reference, tmp_path, program, inputs, stage=f"r{index}")
        assert status == INVALID, index


# -- seeded random programs ------------------------------------------------------

def random_single_op(rng: np.random.Generator):
    """One node of a random kind on a random (ragged, possibly 1-pixel) shape."""
    c = int(rng.choice([1, 2, 3, 4, 8, 12]))
    h, w = int(rng.integers(1, 9)), int(rng.integers(1, 9))
    big = 1 << int(rng.integers(8, 31))

    def tensor(channels, height=h, width=w):
        return rng.integers(-big, big + 1, (channels, height, width)).astype(np.int32)

    kind = rng.choice(["gemm", "depthwise3x3", "mul", "affine", "add", "sat_table", "delta", "clamp", "concat",
                       "slice", "pixel_shuffle", "pixel_unshuffle", "im2col", "crop_like"])
    tables = []
    if kind == "gemm":
        group = int(rng.choice([1, 2, 4]))
        residuals = int(rng.integers(0, 3))
        table = -1
        if rng.random() < 0.5:
            tables = [delta_table(rng, int(rng.integers(0, 1 << 14)), int(rng.integers(0, 4)))]
            table = 0
        op = gemm_node(rng, [], 0, c, group * int(rng.integers(1, 5)), group=group,
                       input_shift=int(rng.integers(0, 8)), table=table, shift=(int(rng.integers(1, 10)), 24),
                       bias_max=1 << int(rng.integers(0, 53)))
        rows = op["out_channels"] // group
        return op, [c] + [rows] * residuals, rows, [tensor(c)] + [tensor(rows) for _ in range(residuals)], tables
    if kind == "depthwise3x3":
        op = {"op": kind, "weights": rng.integers(-(1 << 24), (1 << 24) + 1, (c, 3, 3)).astype(np.int32),
              "bias": rng.integers(-(1 << 52), (1 << 52) + 1, c).astype(np.int64),
              "shift": rng.integers(0, 32, c).astype(np.int32)}
        return op, [c], c, [tensor(c)], tables
    if kind == "mul":
        bc = int(rng.choice([1, c]))
        bh, bw = (1, 1) if rng.random() < 0.5 else (h, w)
        return {"op": kind, "shift": int(rng.integers(0, 32))}, [c, bc], c, [tensor(c), tensor(bc, bh, bw)], tables
    if kind == "affine":
        op = {"op": kind, "alpha": int(rng.integers(-(1 << 24), (1 << 24) + 1)),
              "beta": int(rng.integers(-(1 << 52), (1 << 52) + 1)), "shift": int(rng.integers(0, 32))}
        return op, [c], c, [tensor(c)], tables
    if kind == "add":
        return {"op": kind}, [c, c], c, [tensor(c), tensor(c)], tables
    if kind == "sat_table":
        n = int(rng.integers(1, 64))
        op = {"op": kind, "table": rng.integers(-(1 << 31), (1 << 31) - 1, 2 * n).astype(np.int32),
              "top": int(rng.integers(-(1 << 31), (1 << 31) - 1))}
        x = rng.integers(-n - 3, n + 3, (c, h, w)).astype(np.int32)
        return op, [c], c, [x], tables
    if kind == "delta":
        tables = [delta_table(rng, int(rng.integers(0, 200)), int(rng.integers(0, 4)))]
        x = rng.integers(-220, 220, (c, h, w)).astype(np.int32)
        return {"op": kind, "delta_table": 0}, [c], c, [x], tables
    if kind == "clamp":
        lo = int(rng.integers(-big, big))
        return {"op": kind, "lo": lo, "hi": int(rng.integers(lo, big + 1))}, [c], c, [tensor(c)], tables
    if kind == "concat":
        c2 = int(rng.integers(1, 5))
        return {"op": kind}, [c, c2], c + c2, [tensor(c), tensor(c2)], tables
    if kind == "slice":
        begin = int(rng.integers(0, c))
        end = int(rng.integers(begin + 1, c + 1))
        return {"op": kind, "begin": begin, "end": end}, [c], end - begin, [tensor(c)], tables
    if kind == "pixel_shuffle":
        r = int(rng.choice([2, 3]))
        return {"op": kind, "factor": r}, [c * r * r], c, [tensor(c * r * r)], tables
    if kind == "pixel_unshuffle":
        r = int(rng.choice([2, 3]))
        return {"op": kind, "factor": r}, [c], c * r * r, [tensor(c, h * r, w * r)], tables
    if kind == "im2col":
        k, stride = [(3, 1), (3, 2), (2, 2)][int(rng.integers(0, 3))]
        return {"op": kind, "kernel": k, "stride": stride}, [c], c * k * k, [tensor(c)], tables
    crop = (int(rng.integers(1, h + 1)), int(rng.integers(1, w + 1)))
    return {"op": "crop_like"}, [c, 1], c, [tensor(c), tensor(1, *crop)], tables


def test_single_ops_match_reference(fx_oracle, fx_reference, tmp_path):
    rng = np.random.default_rng(2026)
    seen = {}
    for index in range(400):
        op, ins, out, inputs, tables = random_single_op(rng)
        program = one_op_program(op, ins, out, tables)
        status, _, reason = agree(fx_oracle, fx_reference, tmp_path, program, inputs, stage=f"op{index % 4}")
        seen[(op["op"], status)] = seen.get((op["op"], status), 0) + 1
    for kind in ("gemm", "depthwise3x3", "mul", "affine", "add", "sat_table", "delta", "clamp", "concat", "slice",
                 "pixel_shuffle", "pixel_unshuffle", "im2col", "crop_like"):
        assert seen.get((kind, 0), 0) > 0, kind  # every op also succeeds on some draws
    for kind in ("gemm", "depthwise3x3", "mul", "affine", "add"):
        assert seen.get((kind, STAGE_FAILURE), 0) > 0, kind  # and every writing op fails on some


def test_whole_programs_match_reference(fx_oracle, fx_reference, tmp_path):
    outcomes = {}
    for seed in range(40):
        rng = np.random.default_rng(seed)
        program = decoder_like(rng, tight=seed % 2 == 1)
        inputs = decoder_like_inputs(rng, program, 2 + seed % 9, 2 + (seed * 7) % 11)
        status, _, reason = agree(fx_oracle, fx_reference, tmp_path, program, inputs, stage=f"p{seed % 3}")
        outcomes[(status, reason)] = outcomes.get((status, reason), 0) + 1
    assert outcomes.get((0, ""), 0) >= 10  # most untightened programs run through
    assert sum(count for (status, _), count in outcomes.items() if status == STAGE_FAILURE) >= 5


# -- committed golden fixtures (no reference needed) -------------------------------

def _golden_cases():
    import json
    from pathlib import Path

    return json.loads((Path(__file__).resolve().parent / "golden" / "fx_golden.json").read_text())["cases"]


@pytest.mark.parametrize("entry", _golden_cases(), ids=lambda e: f"seed{e['seed']}")
def test_golden_fx_programs(fx_oracle, tmp_path, entry):
    """tests/golden/fx_golden.json, written by tests/golden/make_fx_golden.py from
    the reference's own fx::run."""
    from tests.golden.make_fx_golden import arrays_digest, case_program, files_digest

    program, inputs = case_program(entry["seed"], entry["tight"], entry["height"], entry["width"])
    write_program(tmp_path, "g", program)
    assert files_digest(tmp_path, "g") == entry["program_sha256"], "program generation drifted"
    assert arrays_digest(inputs) == entry["inputs_sha256"], "input generation drifted"
    status, outputs, reason = fx_oracle.run(program, inputs)
    assert status == entry["status"]
    if status:
        assert reason in entry["message"]
        return
    assert [list(y.shape) for y in outputs] == [o["shape"] for o in entry["outputs"]]
    for y, golden in zip(outputs, entry["outputs"]):
        assert y.reshape(-1)[:6].tolist() == golden["head"]
        assert arrays_digest([y]) == golden["sha256"]


def empty_and_thin_cases():
    """(program, inputs): each op on zero-height, zero-width and 1-pixel tensors."""
    rng = np.random.default_rng(1)
    ops = [
        ({"op": "im2col", "kernel": 3, "stride": 1}, [2], 18),
        ({"op": "im2col", "kernel": 3, "stride": 2}, [2], 18),
        ({"op": "im2col", "kernel": 2, "stride": 2}, [2], 8),
        ({"op": "depthwise3x3", "weights": np.ones((2, 3, 3), np.int32), "bias": np.ones(2, np.int64),
          "shift": np.ones(2, np.int32)}, [2], 2),
        ({"op": "affine", "alpha": 3, "beta": 1, "shift": 1}, [2], 2),
        ({"op": "pixel_shuffle", "factor": 2}, [8], 2),
        ({"op": "pixel_unshuffle", "factor": 2}, [2], 8),
        ({"op": "slice", "begin": 1, "end": 2}, [2], 1),
        ({"op": "concat"}, [2, 2], 4),
        ({"op": "add"}, [2, 2], 2),
        ({"op": "mul", "shift": 2}, [2, 1], 2),
        ({"op": "crop_like"}, [2, 1], 2),
        (dict(gemm_1x1(5), in_channels=2, out_channels=2, weights=np.ones((2, 2), np.int16),
              bias=np.ones(2, np.int64), shift=np.ones(2, np.int32)), [2], 2),
        ({"op": "param_row", "rows": np.arange(6, dtype=np.int64).reshape(3, 2)}, [1], 2),
    ]
    cases = []
    for op, ins, out in ops:
        for height, width in ((0, 0), (0, 3), (3, 0), (1, 1), (1, 2), (2, 1), (0, 1)):
            inputs = []
            for index, channels in enumerate(ins):
                h, w = height, width
                if op["op"] == "crop_like" and index == 1:
                    h, w = min(height, 1), min(width, 1)
                if op["op"] == "mul" and index == 1:
                    h, w = 1, 1
                inputs.append(rng.integers(-5, 5, (channels, h, w)).astype(np.int32))
            cases.append((one_op_program(op, ins, out), inputs))
    return cases


def test_empty_and_thin_tensors_match_reference(fx_oracle, fx_reference, tmp_path):
    """Zero-size images run (im2col of an empty image can still have a row:
    sizes use truncating division); a param_row on an empty input fails."""
    for index, (program, inputs) in enumerate(empty_and_thin_cases()):
        agree(fx_oracle, fx_reference, tmp_path, program, inputs, stage=f"z{index % 3}")
