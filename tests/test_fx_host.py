"""The nvcr.fx.v1 device path's own code, compiled for the host (tests/fx_host.cpp:
the product's fx executor and the element functions its kernels run), against
the oracle (oracle/fx.py, pinned to the reference by tests/test_fx_oracle.py),
on CPU: the same int32 outputs and, on failing inputs, the same failure, on the
cases tests/test_zy_fx_gpu.py runs on a B200. It checks the arithmetic, the
index formulas, the failure-word order and the executor's orchestration; it
does not check launch geometry or anything about the GPU itself."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.fx import INVALID, STAGE_FAILURE
from tests.fx_programs import decoder_like, decoder_like_inputs, gemm_node, write_program
from tests.test_fx_oracle import (gemm_1x1, one_op_program, pixel, random_single_op,
                                  reference_program_test_program)


@pytest.fixture(scope="module")
def fx_host():
    from tests.fx_host import FxHost

    return FxHost()


def matches_oracle(fx_host, fx_oracle, tmp_path, program, inputs, stage="h"):
    write_program(tmp_path, stage, program)
    expected = fx_oracle.run(program, inputs)
    got = fx_host.run(tmp_path, stage, inputs, device_memory=True)
    host_branch = fx_host.run(tmp_path, stage, inputs, device_memory=False)
    assert host_branch[0] == got[0] and host_branch[2] == got[2]
    assert all(np.array_equal(a, b) for a, b in zip(host_branch[1], got[1]))
    assert got[0] == expected[0], (got[2], expected[2])
    if expected[0] == 0:
        assert len(got[1]) == len(expected[1])
        for mine, oracle_output in zip(got[1], expected[1]):
            assert mine.shape == oracle_output.shape
            assert np.array_equal(mine, oracle_output)
    else:
        assert expected[2] in got[2], (got[2], expected[2])
    return got


def test_reference_program_vectors(fx_host, fx_oracle, tmp_path):
    """tests/fx_program_tests.cpp:66-87."""
    program = reference_program_test_program(2)
    q = pixel(1, 2, 3, 4)
    status, outputs, _ = matches_oracle(fx_host, fx_oracle, tmp_path, program, [pixel(5), q])
    assert status == 0 and outputs[0].item() == 8 and np.array_equal(outputs[1], q)
    status, _, message = matches_oracle(fx_host, fx_oracle, tmp_path, program, [pixel((1 << 30) + 1), q])
    assert status == STAGE_FAILURE and "input value out of range" in message


def test_failure_thresholds(fx_host, fx_oracle, tmp_path):
    for bias in ((1 << 30) - 4, (1 << 30) - 2, -((1 << 30) - 4), -((1 << 30) - 2)):
        matches_oracle(fx_host, fx_oracle, tmp_path, one_op_program(gemm_1x1(bias), [1], 1), [pixel(0)])
    top = 1 << 30
    for residual, bias in ((top, 0), (top, 2), (-top, -2)):
        matches_oracle(fx_host, fx_oracle, tmp_path, one_op_program(gemm_1x1(bias), [1, 1], 1),
                       [pixel(0), pixel(residual)])
    for a, b in ((top, 0), (top, 1), (-top, -1)):
        matches_oracle(fx_host, fx_oracle, tmp_path, one_op_program({"op": "add"}, [1, 1], 1), [pixel(a), pixel(b)])
    rows = np.arange(12, dtype=np.int64).reshape(4, 3)
    for q in (-1, 0, 3, 4):
        matches_oracle(fx_host, fx_oracle, tmp_path, one_op_program({"op": "param_row", "rows": rows}, [1], 3),
                       [pixel(q)])


def test_first_failure_in_reference_order(fx_host, fx_oracle, tmp_path):
    """Several failures in one node, and in several nodes: the one reported is
    the first in the reference's order (node, then its loop position, then the
    gemm's pre-activation rule before its stored bound)."""
    x = np.zeros((1, 1, 4), np.int32)
    residual = np.zeros((1, 1, 4), np.int32)
    residual[0, 0, 1] = 1 << 30
    x[0, 0, 1] = 2  # pixel 1: r = 1, output 2^30 + 1 fails the stored bound
    x[0, 0, 3] = 1 << 20  # pixel 3: a larger pre-activation, still inside its limit
    _, _, message = matches_oracle(fx_host, fx_oracle, tmp_path, one_op_program(gemm_1x1(0, shift=1), [1, 1], 1),
                                   [x, residual])
    assert "gemm output out of range" in message
    _, _, message = matches_oracle(fx_host, fx_oracle, tmp_path,
                                   one_op_program(gemm_1x1((1 << 30) - 2, shift=1), [1, 1], 1), [x, residual])
    assert "gemm pre-activation out of range" in message  # pixel 0 fails the pre-activation rule first
    two = {"fa": 14, "tensors": [("x", 1), ("y", 1), ("z", 1)], "inputs": [0], "outputs": [2], "delta_tables": [],
           "nodes": [{"op": "affine", "inputs": [0], "output": 1, "alpha": 2, "beta": 0, "shift": 0},
                     {"op": "add", "inputs": [1, 1], "output": 2}]}
    _, _, message = matches_oracle(fx_host, fx_oracle, tmp_path, two, [np.array([[[1, 1 << 29]]], np.int32)])
    assert "add output out of range" in message
    _, _, message = matches_oracle(fx_host, fx_oracle, tmp_path, two, [np.array([[[1 << 30, 1 << 29]]], np.int32)])
    assert "affine output out of range" in message


def test_single_ops_match_oracle(fx_host, fx_oracle, tmp_path):
    rng = np.random.default_rng(2026)
    for index in range(300):
        op, ins, out, inputs, tables = random_single_op(rng)
        matches_oracle(fx_host, fx_oracle, tmp_path, one_op_program(op, ins, out, tables), inputs,
                       stage=f"op{index % 4}")


def test_whole_programs_match_oracle(fx_host, fx_oracle, tmp_path):
    outcomes = {}
    for seed in range(40):
        rng = np.random.default_rng(seed)
        program = decoder_like(rng, channels=4 * (1 + seed % 4), tight=seed % 2 == 1)
        inputs = decoder_like_inputs(rng, program, 2 + seed % 17, 2 + (seed * 7) % 23)
        status, _, _ = matches_oracle(fx_host, fx_oracle, tmp_path, program, inputs, stage=f"p{seed % 3}")
        outcomes[status] = outcomes.get(status, 0) + 1
    assert outcomes.get(0, 0) >= 10 and outcomes.get(STAGE_FAILURE, 0) >= 5


def test_wide_gemm_tiles(fx_host, fx_oracle, tmp_path):
    """Row counts that are not a multiple of the four-group tile, each group size."""
    rng = np.random.default_rng(31)
    for group, rows in ((1, 7), (2, 10), (4, 20), (1, 1), (4, 4)):
        node = gemm_node(rng, [0], 1, 13, rows, group=group, input_shift=1, table=0, shift=(12, 16))
        program = {"fa": 14, "tensors": [("x", 13), ("y", rows // group)], "inputs": [0], "outputs": [1],
                   "delta_tables": [{"h": 1 << 12, "shift": 2,
                                     "dc": rng.integers(-100, 100, ((2 << 12) >> 2) + 1).astype(np.int16)}],
                   "nodes": [node]}
        x = rng.integers(-(1 << 18), 1 << 18, (13, 5, 9)).astype(np.int32)
        status, _, _ = matches_oracle(fx_host, fx_oracle, tmp_path, program, [x], stage=f"w{group}{rows}")
        assert status == 0


def test_stage_failure_before_a_shape_refusal(fx_host, fx_oracle, tmp_path):
    program = {"fa": 14, "tensors": [("x", 1), ("y", 1), ("z", 1), ("w", 1)], "inputs": [0, 1], "outputs": [3],
               "delta_tables": [],
               "nodes": [{"op": "affine", "inputs": [0], "output": 2, "alpha": 2, "beta": 0, "shift": 0},
                         {"op": "add", "inputs": [2, 1], "output": 3}]}
    wide = np.zeros((1, 1, 2), np.int32)
    for value, expected in ((1 << 30, STAGE_FAILURE), (1, INVALID)):
        status, _, _ = matches_oracle(fx_host, fx_oracle, tmp_path, program, [pixel(value), wide])
        assert status == expected


def test_empty_and_thin_tensors(fx_host, fx_oracle, tmp_path):
    from tests.test_fx_oracle import empty_and_thin_cases

    for index, (program, inputs) in enumerate(empty_and_thin_cases()):
        matches_oracle(fx_host, fx_oracle, tmp_path, program, inputs, stage=f"z{index % 3}")


def test_cached_plan_across_both_branches(fx_host, fx_oracle, tmp_path):
    """One executor: a device-memory run, then host-memory runs that reuse its
    plan (input buffers made late); all equal the oracle."""
    for seed in range(8):
        rng = np.random.default_rng(100 + seed)
        program = decoder_like(rng, channels=8)
        inputs = decoder_like_inputs(rng, program, 3 + seed, 4 + seed)
        write_program(tmp_path, "c", program)
        expected = fx_oracle.run(program, inputs)
        got = fx_host.run(tmp_path, "c", inputs, device_memory="both")
        assert got[0] == expected[0], got[2]
        for mine, want in zip(got[1], expected[1]):
            assert np.array_equal(mine, want)
