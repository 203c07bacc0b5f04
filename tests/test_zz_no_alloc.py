"""nvcr_sm100_run_half_static, the entry point that allocates no device memory.

Some hosts cannot call cudaMalloc while they run: a provider whose enqueue runs
inside a framework that owns every device allocation, or a real-time decode
thread that must not block on the driver's allocator. They create the executor
at set-up and then run through nvcr_sm100_run_half_static, which keeps every
scratch tensor in the library's fixed static device array. This file checks,
through the C ABI, that two calls in a row give the same bits as the ordinary
nvcr_sm100_run_half (the suite's tolerance: bit-exact, any NaN equals any NaN),
that an executor which only ever runs this way gets no workspace of its own and
leaves the device's free memory unchanged, that a run too large for the array
is refused, and that a call made with another device current is refused. It is
named to be collected last and passes alone in a fresh process or after the
other tests.
"""
from __future__ import annotations

import numpy as np
import pytest

from nvcr_b200.executor import CudaExecutor, ErrorCode, ExecutorError
from nvcr_b200.program import SeededStream
from nvcr_b200.workloads import config1, config2, layer_input
from oracle.oracle import count_differing
from tests.programs import op_program

pytestmark = pytest.mark.gpu


def _half_tensors(torch, arrays: dict, device):
    return {name: torch.from_numpy(np.ascontiguousarray(a, np.float16)).to(device) for name, a in arrays.items()}


@pytest.mark.parametrize("case", ["ops_w16a16", "ops_w8a8", "config1"])
def test_static_run_matches_run_half_on_two_calls(cuda, case):
    import torch

    if case == "config1":
        layer = config1()
        program, inputs = layer.program, {"x": layer_input(layer, seed=1)}
    else:
        stream = SeededStream(31)
        bits = (16, 16) if case == "ops_w16a16" else (8, 8)
        program = op_program(stream).with_widths(*bits)
        inputs = {"x": stream.tensor(70, 33, 47, 3.0)}
    with CudaExecutor.from_program(program) as executor:
        extents = executor.infer_output_extents([a.shape for a in inputs.values()])
        ins = _half_tensors(torch, inputs, cuda)

        def fresh_outputs():
            return {name: torch.full(e, float("nan"), dtype=torch.float16, device=cuda)
                    for name, e in zip(executor.output_names, extents)}

        expected = fresh_outputs()
        executor.run_half(ins, expected)
        executor.synchronize()
        for call in range(2):
            got = fresh_outputs()
            executor.run_half_static(ins, got)
            executor.synchronize()
            for name in executor.output_names:
                bad = count_differing(got[name].float().cpu().numpy(), expected[name].float().cpu().numpy())
                assert bad == 0, f"{case} call {call + 1}: {bad} elements of {name} differ from run_half"


def test_static_run_refuses_a_plan_larger_than_the_array(cuda):
    import torch

    layer = config2()[1]  # 3x3 64->64 at 544x960: its plan needs far more than 64 MiB
    with CudaExecutor.from_program(layer.program) as executor:
        (c, h, w), = executor.infer_output_extents([layer.input_shape])
        x = torch.zeros(layer.input_shape, dtype=torch.float16, device=cuda)
        y = torch.zeros((c, h, w), dtype=torch.float16, device=cuda)
        with pytest.raises(ExecutorError) as error:
            executor.run_half_static({"x": x}, {"y": y})
        assert error.value.code == ErrorCode.invalid_argument
        assert "bytes of workspace" in error.value.message


def test_static_only_executor_allocates_nothing(cuda):
    """An executor that never calls run_half: after two static calls it has no
    workspace of its own, and the second call leaves the free device memory as
    it found it; both calls give run_half's bits (from a second executor)."""
    import torch

    layer = config1()
    x = layer_input(layer, seed=1)
    with CudaExecutor.from_program(layer.program) as reference, CudaExecutor.from_program(layer.program) as executor:
        (c, h, w), = executor.infer_output_extents([x.shape])
        ins = _half_tensors(torch, {"x": x}, cuda)
        expected = torch.empty((c, h, w), dtype=torch.float16, device=cuda)
        reference.run_half(ins, {"y": expected})
        reference.synchronize()
        outputs = [torch.full((c, h, w), float("nan"), dtype=torch.float16, device=cuda) for _ in range(2)]
        torch.cuda.synchronize()
        executor.run_half_static(ins, {"y": outputs[0]})
        executor.synchronize()
        free_before, _ = torch.cuda.mem_get_info(cuda)
        executor.run_half_static(ins, {"y": outputs[1]})
        executor.synchronize()
        free_after, _ = torch.cuda.mem_get_info(cuda)
        assert executor.workspace_bytes == 0
        assert free_after == free_before
        for call, got in enumerate(outputs):
            bad = count_differing(got.float().cpu().numpy(), expected.float().cpu().numpy())
            assert bad == 0, f"static call {call + 1}: {bad} elements differ from run_half"


def test_static_run_refuses_another_current_device(cuda):
    """The array is looked up for the current device, and the executor's work
    belongs to its own: with another device current the call is refused and
    nothing runs."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    layer = config1()
    x = layer_input(layer, seed=1)
    with CudaExecutor.from_program(layer.program) as executor:
        (c, h, w), = executor.infer_output_extents([x.shape])
        ins = _half_tensors(torch, {"x": x}, cuda)
        y = torch.zeros((c, h, w), dtype=torch.float16, device=cuda)
        torch.cuda.synchronize()
        with torch.cuda.device(1):
            with pytest.raises(ExecutorError) as error:
                executor.run_half_static(ins, {"y": y})
        assert error.value.code == ErrorCode.invalid_state
        assert float(y.abs().max()) == 0.0
