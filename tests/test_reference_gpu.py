"""The GPU comparator: the reference's own CUDA executor (CudaExecutor, built
for sm_100a into oracle/_ref/libnvcr_ref_cuda.so) on the same B200.

Before its times mean anything it must compute the profile: its outputs equal
the reference's run_cpu, which is the reference's own claim
(tests/deterministic_executor_tests.cpp:316-343, compare_cpu_cuda). And the
new path's outputs equal its outputs, on the same FP16 device tensors.
"""
from __future__ import annotations

import numpy as np
import pytest

from nvcr_b200.executor import CudaExecutor
from nvcr_b200.program import SeededStream
from nvcr_b200.workloads import config1, config2, intra_decoder, laplace_latent, layer_input
from oracle.oracle import ReferenceGpu, count_differing
from tests.programs import op_program

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comparator():
    if not ReferenceGpu.available():
        pytest.skip("the reference's CUDA executor (oracle/_ref/libnvcr_ref_cuda.so) is not built here")
    return ReferenceGpu


def cases():
    layer = config1()
    yield "config1", layer.program, {"x": layer_input(layer, seed=1)}
    for bits in ((8, 8), (16, 16)):
        stream = SeededStream(11)
        program = op_program(stream).with_widths(*bits)
        yield f"ops_w{bits[0]}a{bits[1]}", program, {"x": stream.tensor(70, 33, 47, 3.0)}
    decoder = intra_decoder((3, 5))
    yield "intra_decoder_3x5", decoder.program, {"y_hat": laplace_latent(SeededStream(7), (256, 3, 5))}
    layer = config2()[3]
    yield "config2_L4_rows", layer.program, {"x": layer_input(layer, seed=203, height=24)}


@pytest.mark.parametrize("case", list(cases()), ids=lambda c: c[0])
def test_comparator_equals_run_cpu_and_new_path(cuda, comparator, reference, tmp_path, case):
    import torch

    name, program, inputs = case
    path = program.write(tmp_path, name)
    half_inputs = {k: np.asarray(v, np.float32).astype(np.float16) for k, v in inputs.items()}
    expected = reference.run(path, [half_inputs[k].astype(np.float32) for k in half_inputs])
    device_inputs = {k: torch.from_numpy(v).to(cuda) for k, v in half_inputs.items()}
    with CudaExecutor.from_program(program) as ours, comparator(path) as theirs:
        extents = ours.infer_output_extents([v.shape for v in half_inputs.values()])
        outs_ours = {n: torch.full(e, float("nan"), dtype=torch.float16, device=cuda)
                     for n, e in zip(ours.output_names, extents)}
        outs_theirs = {n: torch.full(e, float("nan"), dtype=torch.float16, device=cuda)
                       for n, e in zip(ours.output_names, extents)}
        ours.run_half(device_inputs, outs_ours)
        ours.synchronize()
        theirs.run_half(device_inputs, outs_theirs)
        torch.cuda.synchronize()
        for index, n in enumerate(ours.output_names):
            e = expected[index].astype(np.float16).astype(np.float32)
            t = outs_theirs[n].float().cpu().numpy()
            o = outs_ours[n].float().cpu().numpy()
            assert count_differing(t, e) == 0, f"{name}/{n}: the reference's CUDA executor differs from run_cpu"
            assert count_differing(o, t) == 0, f"{name}/{n}: the new path differs from the reference's CUDA executor"
