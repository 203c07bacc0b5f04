"""Bit-exactness at the benchmark's full sizes, through the C ABI with FP16
stage boundaries (run_half), against the reference's own CPU executor.

Two checkers, both from the reference's run_cpu (compiled from its sources into
oracle/_ref): elementwise against a live run of it on the same inputs, when
oracle/_ref is present, and always against tests/golden/fullsize_digests.json,
which tests/golden/make_fullsize_digests.py wrote from it (SHA-256 of the FP16
outputs, NaN stored as 0x7e00). Equality is the reference's rule
(tests/deterministic_executor_tests.cpp:54-60): bitwise, any NaN equals any NaN.

  config 2  each of the five 1920x1088 layers, as the benchmark runs them;
  config 3  one 1080p intra-decoder frame with every block's output compared,
            and the frame of every config-5 stream (the decoder the benchmark
            times, frame output only);
  config 4  the whole GOP-30 720p sequence (I-frame then 29 P-frames, the
            feature carried frame to frame in FP16), every frame and feature,
            the first three frames also elementwise.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from nvcr_b200.executor import CudaExecutor
from nvcr_b200.program import SeededStream
from nvcr_b200.workloads import (config2, half_digest, inter_decoder, intra_decoder, laplace_latent,
                                 layer_input)
from oracle.oracle import Reference, count_differing

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "fullsize_digests.json").read_text())


def live_reference():
    if not Reference.available():
        return None
    from oracle.oracle import build

    build(reference=True)
    return Reference()


def to_device(torch, array, device):
    return torch.from_numpy(np.ascontiguousarray(array, np.float32).astype(np.float16)).to(device)


def assert_same(got_half: np.ndarray, expected_fp32: np.ndarray, label: str) -> None:
    expected = np.asarray(expected_fp32, np.float32).astype(np.float16).astype(np.float32)
    got = np.asarray(got_half, np.float16).astype(np.float32)
    assert got.shape == expected.shape, f"{label}: shape {got.shape} != {expected.shape}"
    bad = count_differing(got, expected)
    assert bad == 0, f"{label}: {bad} of {got.size} values differ from the reference"


@pytest.mark.parametrize("index", range(5), ids=[layer.name for layer in config2()])
def test_config2_layer_full_size(cuda, tmp_path, index):
    import torch

    layer = config2()[index]
    x = layer_input(layer, seed=200 + index)
    with CudaExecutor.from_program(layer.program) as executor:
        (c, h, w), = executor.infer_output_extents([x.shape])
        y = torch.full((c, h, w), float("nan"), dtype=torch.float16, device=cuda)
        executor.run_half({"x": to_device(torch, x, cuda)}, {"y": y})
        executor.synchronize()
        got = y.cpu().numpy()
    assert half_digest(got) == GOLDEN["config2"][layer.name]["digest"], f"{layer.name}: digest differs"
    reference = live_reference()
    if reference is not None:
        expected, = reference.run(layer.program.write(tmp_path, layer.name), [x])
        assert_same(got, expected, layer.name)


def test_config3_full_frame_every_tensor(cuda, tmp_path):
    """One 1080p frame (config 5's stream 0) with every block's output a stage
    output: the 14 DepthConvBlock outputs and the frame."""
    import torch

    stack = intra_decoder(every_tensor=True)
    latent = laplace_latent(SeededStream(5000), stack.input_shapes[0])
    with CudaExecutor.from_program(stack.program) as executor:
        extents = executor.infer_output_extents(stack.input_shapes)
        outputs = {name: torch.full(e, float("nan"), dtype=torch.float16, device=cuda)
                   for name, e in zip(executor.output_names, extents)}
        executor.run_half({"y_hat": to_device(torch, latent, cuda)}, outputs)
        executor.synchronize()
        got = {name: t.cpu().numpy() for name, t in outputs.items()}
        names = list(executor.output_names)
    assert half_digest(got["frame"]) == GOLDEN["config3"]["0"]["digest"]
    reference = live_reference()
    if reference is None:
        pytest.skip("elementwise check of the intermediates needs oracle/_ref")
    expected = reference.run(stack.program.write(tmp_path, "intra_every"), [latent], max_outputs=len(names))
    assert len(expected) == len(names)
    for name, e in zip(names, expected):
        assert_same(got[name], e, name)


def test_config3_frame_of_every_stream(cuda):
    """The frame the benchmark decodes for each of config 5's 64 streams."""
    import torch

    stack = intra_decoder()
    with CudaExecutor.from_program(stack.program) as executor:
        (c, h, w), = executor.infer_output_extents(stack.input_shapes)
        frame = torch.empty((c, h, w), dtype=torch.float16, device=cuda)
        wrong = []
        for stream, entry in sorted(GOLDEN["config3"].items(), key=lambda kv: int(kv[0])):
            latent = laplace_latent(SeededStream(entry["latent_seed"]), stack.input_shapes[0])
            frame.fill_(float("nan"))
            executor.run_half({"y_hat": to_device(torch, latent, cuda)}, {"frame": frame})
            executor.synchronize()
            if half_digest(frame.cpu().numpy()) != entry["digest"]:
                wrong.append(stream)
    assert len(GOLDEN["config3"]) == 64
    assert not wrong, f"streams whose frame differs from the reference: {wrong}"


def test_config4_gop30_full_size(cuda, tmp_path):
    """The benchmark's GOP-30 sequence at 768x1280: every frame and feature
    against the reference's digests; the I-frame and two P-frames also
    elementwise against a live reference run chained on its own outputs."""
    import torch

    intra = intra_decoder((48, 80), feature_channels=64)
    inter = inter_decoder((48, 80))
    reference = live_reference()
    paths = None
    if reference is not None:
        paths = (intra.program.write(tmp_path, "intra_720p"), inter.program.write(tmp_path, "inter_720p"))
    golden = GOLDEN["config4"]
    assert len(golden) == 30
    with CudaExecutor.from_program(intra.program) as first, CudaExecutor.from_program(inter.program) as rest:
        frame = torch.empty((3, 768, 1280), dtype=torch.float16, device=cuda)
        features = [torch.empty((64, 96, 160), dtype=torch.float16, device=cuda) for _ in range(2)]
        reference_feature = None
        for f, entry in enumerate(golden):
            latent = laplace_latent(SeededStream(entry["latent_seed"]), (256, 48, 80))
            y_hat = to_device(torch, latent, cuda)
            frame.fill_(float("nan"))
            if f == 0:
                first.run_half({"y_hat": y_hat}, {"frame": frame, "feature": features[0]})
                first.synchronize()
            else:
                rest.run_half({"y_hat": y_hat, "context": features[(f - 1) % 2]},
                              {"frame": frame, "feature": features[f % 2]})
                rest.synchronize()
            got_frame = frame.cpu().numpy()
            got_feature = features[f % 2].cpu().numpy()
            assert half_digest(got_frame) == entry["frame"], f"frame {f}"
            assert half_digest(got_feature) == entry["feature"], f"feature {f}"
            if reference is not None and f < 3:
                if f == 0:
                    e_frame, e_feature = reference.run(paths[0], [latent])
                else:
                    e_frame, e_feature = reference.run(paths[1], [latent, reference_feature])
                reference_feature = e_feature.astype(np.float16).astype(np.float32)
                assert_same(got_frame, e_frame, f"frame {f}")
                assert_same(got_feature, e_feature, f"feature {f}")
