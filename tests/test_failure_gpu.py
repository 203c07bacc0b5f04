"""Failure detection without a GPU fault: every device wait in the kernels is
bounded by the global timer and, when it runs out, sets the executor's status
word and returns. Here a self-test kernel waits on a barrier that nothing
completes (limit 20 ms); synchronize() must report it, clear it, and the same
executor must then run bit-exact again."""
from __future__ import annotations

import pytest

from nvcr_b200.executor import CudaExecutor, ErrorCode, ExecutorError
from nvcr_b200.workloads import config1, layer_input
from oracle.oracle import count_differing

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_recovers(cuda, oracle):
    layer = config1()
    x = layer_input(layer, seed=1)
    with CudaExecutor.from_program(layer.program) as executor:
        executor.test_wait_timeout(20)
        with pytest.raises(ExecutorError) as failure:
            executor.synchronize()
        assert failure.value.code == ErrorCode.backend_error
        assert "gave up" in failure.value.message
        executor.synchronize()  # the status word was cleared
        got = executor.run([x])
    expected = oracle.run(layer.program, [x])
    assert count_differing(got[0], expected[0]) == 0


def test_wait_limit_is_checked(cuda):
    layer = config1()
    with CudaExecutor.from_program(layer.program) as executor:
        for bad in (0, 4001):
            with pytest.raises(ExecutorError) as failure:
                executor.test_wait_timeout(bad)
            assert failure.value.code == ErrorCode.invalid_argument
