"""nvcr.fx.v1 on the GPU (nvcr_sm100_fx_run) against the oracle (oracle/fx.py),
which tests/test_fx_oracle.py pins to the reference's fx.cpp: the same int32
outputs, and on failing inputs the same failure, on the reference's own
vectors, the conformance edges, seeded single-op programs on ragged shapes and
seeded whole programs that use every op, through host and device memory."""
from __future__ import annotations

import numpy as np
import pytest

from nvcr_b200 import fx
from nvcr_b200.executor import ErrorCode, ExecutorError
from oracle.fx import INVALID, STAGE_FAILURE
from tests.fx_programs import decoder_like, decoder_like_inputs, write_program
from tests.test_fx_oracle import (gemm_1x1, one_op_program, pixel, random_single_op,
                                  reference_program_test_program)

pytestmark = pytest.mark.gpu


def device_run(tmp_path, program: dict, inputs, stage: str = "g", device_memory: bool = False):
    """(status, outputs, message) of the GPU path, status as 0 or ErrorCode + 1."""
    write_program(tmp_path, stage, program)
    with fx.load_program(tmp_path, stage) as loaded, fx.FxExecutor(loaded) as executor:
        try:
            if device_memory:
                import torch

                outputs = executor.run_device([torch.from_numpy(np.ascontiguousarray(x, np.int32)).cuda()
                                               for x in inputs])
                return 0, [y.cpu().numpy() for y in outputs], ""
            return 0, executor.run(inputs), ""
        except ExecutorError as error:
            return int(error.code) + 1, [], str(error)


def matches_oracle(fx_oracle, tmp_path, program, inputs, stage="g", device_memory=False):
    expected = fx_oracle.run(program, inputs)
    got = device_run(tmp_path, program, inputs, stage, device_memory)
    assert got[0] == expected[0], (got[2], expected[2])
    if expected[0] == 0:
        assert len(got[1]) == len(expected[1])
        for mine, oracle_output in zip(got[1], expected[1]):
            assert mine.shape == oracle_output.shape
            assert np.array_equal(mine, oracle_output)
    else:
        assert expected[2] in got[2], (got[2], expected[2])
    return got


def test_reference_program_vectors(cuda, fx_oracle, tmp_path):
    """tests/fx_program_tests.cpp:66-87 on the GPU."""
    program = reference_program_test_program(2)
    q = pixel(1, 2, 3, 4)
    status, outputs, _ = matches_oracle(fx_oracle, tmp_path, program, [pixel(5), q])
    assert status == 0 and outputs[0].item() == 8 and np.array_equal(outputs[1], q)
    status, _, message = matches_oracle(fx_oracle, tmp_path, program, [pixel((1 << 30) + 1), q])
    assert status == STAGE_FAILURE and "input value out of range" in message


def test_failure_thresholds(cuda, fx_oracle, tmp_path):
    for bias in ((1 << 30) - 4, (1 << 30) - 2, -((1 << 30) - 4), -((1 << 30) - 2)):
        matches_oracle(fx_oracle, tmp_path, one_op_program(gemm_1x1(bias), [1], 1), [pixel(0)])
    top = 1 << 30
    for residual, bias in ((top, 0), (top, 2), (-top, -2)):
        matches_oracle(fx_oracle, tmp_path, one_op_program(gemm_1x1(bias), [1, 1], 1), [pixel(0), pixel(residual)])
    for a, b in ((top, 0), (top, 1), (-top, -1)):
        matches_oracle(fx_oracle, tmp_path, one_op_program({"op": "add"}, [1, 1], 1), [pixel(a), pixel(b)])
    rows = np.arange(12, dtype=np.int64).reshape(4, 3)
    for q in (-1, 0, 3, 4):
        matches_oracle(fx_oracle, tmp_path, one_op_program({"op": "param_row", "rows": rows}, [1], 3), [pixel(q)])


def test_first_failure_in_reference_order(cuda, fx_oracle, tmp_path):
    """Both gemm rules fail in one node: the reported one is the first in the
    reference's loop order (pixel, then group)."""
    program = one_op_program(gemm_1x1(0, shift=1), [1, 1], 1)
    x = np.zeros((1, 1, 4), np.int32)
    residual = np.zeros((1, 1, 4), np.int32)
    residual[0, 0, 1] = 1 << 30
    x[0, 0, 1] = 2  # pixel 1: r = 1, output 2^30 + 1 fails the stored bound
    program["nodes"][0]["bias"] = np.array([0], np.int64)
    matches_oracle(fx_oracle, tmp_path, program, [x, residual])
    big = one_op_program(gemm_1x1((1 << 30) - 2, shift=1), [1, 1], 1)
    matches_oracle(fx_oracle, tmp_path, big, [x, residual])


def test_single_ops_match_oracle(cuda, fx_oracle, tmp_path):
    rng = np.random.default_rng(2026)
    for index in range(300):
        op, ins, out, inputs, tables = random_single_op(rng)
        matches_oracle(fx_oracle, tmp_path, one_op_program(op, ins, out, tables), inputs, stage=f"op{index % 4}",
                       device_memory=index % 3 == 0)


def test_whole_programs_match_oracle(cuda, fx_oracle, tmp_path):
    outcomes = {}
    for seed in range(40):
        rng = np.random.default_rng(seed)
        program = decoder_like(rng, channels=4 * (1 + seed % 4), tight=seed % 2 == 1)
        inputs = decoder_like_inputs(rng, program, 2 + seed % 17, 2 + (seed * 7) % 23)
        status, _, _ = matches_oracle(fx_oracle, tmp_path, program, inputs, stage=f"p{seed % 3}",
                                      device_memory=seed % 2 == 0)
        outcomes[status] = outcomes.get(status, 0) + 1
    assert outcomes.get(0, 0) >= 10 and outcomes.get(STAGE_FAILURE, 0) >= 5


def test_large_gemm_and_repeated_runs(cuda, fx_oracle, tmp_path):
    """A 1x1 gemm at 120 x 68 x 4 pixels with 96 -> 2 x 64 rows, run three times
    on one executor (cached plan), device memory."""
    import torch

    rng = np.random.default_rng(77)
    from tests.fx_programs import gemm_node

    node = gemm_node(rng, [0], 1, 96, 128, group=2, input_shift=2, shift=(14, 18))
    program = {"fa": 14, "tensors": [("x", 96), ("y", 64)], "inputs": [0], "outputs": [1], "delta_tables": [],
               "nodes": [node]}
    x = rng.integers(-(1 << 20), 1 << 20, (96, 136, 240)).astype(np.int32)
    expected = fx_oracle.run(program, [x])
    assert expected[0] == 0
    write_program(tmp_path, "big", program)
    with fx.load_program(tmp_path, "big") as loaded, fx.FxExecutor(loaded) as executor:
        device_x = torch.from_numpy(x).cuda()
        for _ in range(3):
            (y,) = executor.run_device([device_x])
            assert np.array_equal(y.cpu().numpy(), expected[1][0])
        assert executor.last_launch_count == 2  # the input check and the gemm


def test_shape_refusals_on_gpu(cuda, fx_oracle, tmp_path):
    program = one_op_program({"op": "add"}, [2, 2], 2)
    status, _, _ = device_run(tmp_path, program, [np.zeros((2, 2, 2), np.int32), np.zeros((2, 2, 3), np.int32)])
    assert status == INVALID == ErrorCode.invalid_argument + 1


def test_stage_failure_before_a_shape_refusal(cuda, fx_oracle, tmp_path):
    """The reference stops at the first problem in node order: a stage failure
    in an earlier node wins over a later node's shape refusal, and without it
    the refusal is reported."""
    program = {"fa": 14, "tensors": [("x", 1), ("y", 1), ("z", 1), ("w", 1)], "inputs": [0, 1], "outputs": [3],
               "delta_tables": [],
               "nodes": [{"op": "affine", "inputs": [0], "output": 2, "alpha": 2, "beta": 0, "shift": 0},
                         {"op": "add", "inputs": [2, 1], "output": 3}]}
    wide = np.zeros((1, 1, 2), np.int32)
    for value, expected in ((1 << 30, STAGE_FAILURE), (1, INVALID)):
        status, _, _ = matches_oracle(fx_oracle, tmp_path, program, [pixel(value), wide])
        assert status == expected


def test_empty_and_thin_tensors(cuda, fx_oracle, tmp_path):
    from tests.test_fx_oracle import empty_and_thin_cases

    for index, (program, inputs) in enumerate(empty_and_thin_cases()):
        matches_oracle(fx_oracle, tmp_path, program, inputs, stage=f"z{index % 3}", device_memory=index % 2 == 0)
