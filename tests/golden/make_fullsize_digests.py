#!/usr/bin/env python3
"""Generates tests/golden/fullsize_digests.json from the REFERENCE's own CPU
executor (run_cpu, compiled from its sources into oracle/_ref by
oracle/Makefile) at the benchmark's full sizes, so that the benchmark can check
every output it produces, on every rank, without running the reference.

Each digest is nvcr_b200.workloads.half_digest of an FP16 stage output: the
reference's FP32 output rounded to FP16 (round to nearest even, what
run_half_cpu does at the stage boundary), SHA-256 over its bytes with every
NaN stored as 0x7e00. Inputs are the benchmark's own seeded inputs:

  config2  the five layers of the 1920x1088 sweep, input seed 200 + layer index;
  config3  the 1080p intra decoder's frame for config 5's 64 streams, latent
           Laplace(4) from seed 5000 + stream (stream 0 is config 3's frame);
  config4  the GOP-30 720p sequence (I-frame then 29 P-frames, each P-frame's
           context the previous frame's FP16 feature), latents seed 6000 + frame:
           the frame and the feature of every frame.

Run from the repository root where the reference sources exist (about 1.5 h
on 8 cores; configs 2 and 3 are saved item by item and a rerun resumes):
    python tests/golden/make_fullsize_digests.py [config2|config3|config4 ...]
"""
from __future__ import annotations

import json
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from nvcr_b200.program import SeededStream  # noqa: E402
from nvcr_b200.workloads import (config2, half_digest, inter_decoder, intra_decoder, laplace_latent,  # noqa: E402
                                 layer_input)
from oracle.oracle import Reference, build  # noqa: E402

OUT = Path(__file__).resolve().parent / "fullsize_digests.json"
STREAMS = 64
GOP = 30


def half_round(x: np.ndarray) -> np.ndarray:
    """A stage-boundary FP16 value widened back to FP32."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def load() -> dict:
    return json.loads(OUT.read_text()) if OUT.exists() else {}


def save(document: dict) -> None:
    partial = OUT.with_suffix(".partial")
    partial.write_text(json.dumps(document, indent=1, sort_keys=True) + "\n")
    partial.replace(OUT)  # atomic: readers never see a half-written file


def main(sections: list[str]) -> None:
    build(reference=True)
    reference = Reference()
    document = load()
    document["format"] = ("half_digest: SHA-256 of the FP16 output bytes (C order, NaN stored as 0x7e00), "
                          "from the reference's run_cpu rounded to FP16")
    with tempfile.TemporaryDirectory() as directory:
        if "config2" in sections:
            entries = document.setdefault("config2", {})
            for index, layer in enumerate(config2()):
                if layer.name in entries:
                    continue
                path = layer.program.write(directory, layer.name)
                x = half_round(layer_input(layer, seed=200 + index))
                start = time.time()
                y, = reference.run(path, [x])
                entries[layer.name] = {"input_seed": 200 + index, "shape": list(y.shape), "digest": half_digest(y)}
                save(document)
                print(f"config2 {layer.name}: {time.time() - start:.1f} s", flush=True)
        if "config3" in sections:
            stack = intra_decoder()
            path = stack.program.write(directory, "intra_1080p")
            entries = document.setdefault("config3", {})
            for stream in range(STREAMS):
                key = str(stream)
                if key in entries:
                    continue
                latent = half_round(laplace_latent(SeededStream(5000 + stream), stack.input_shapes[0]))
                start = time.time()
                frame, = reference.run(path, [latent])
                entries[key] = {"latent_seed": 5000 + stream, "shape": list(frame.shape), "digest": half_digest(frame)}
                save(document)
                print(f"config3 stream {stream}: {time.time() - start:.1f} s", flush=True)
        if "config4" in sections:
            intra = intra_decoder((48, 80), feature_channels=64)
            inter = inter_decoder((48, 80))
            intra_path = intra.program.write(directory, "intra_720p")
            inter_path = inter.program.write(directory, "inter_720p")
            if len(document.get("config4", [])) < GOP:
                entries = []
                feature = None
                for f in range(GOP):
                    latent = half_round(laplace_latent(SeededStream(6000 + f), (256, 48, 80)))
                    start = time.time()
                    if f == 0:
                        frame, out_feature = reference.run(intra_path, [latent])
                    else:
                        frame, out_feature = reference.run(inter_path, [latent, feature])
                    feature = half_round(out_feature)  # the next P-frame's FP16 context
                    entries.append({"latent_seed": 6000 + f, "frame": half_digest(frame),
                                    "feature": half_digest(out_feature), "frame_shape": list(frame.shape),
                                    "feature_shape": list(out_feature.shape)})
                    print(f"config4 frame {f}: {time.time() - start:.1f} s", flush=True)
                document["config4"] = entries
                save(document)


if __name__ == "__main__":
    main(sys.argv[1:] or ["config2", "config4", "config3"])
