"""Per-op device times of one decoder stack run, from the executor's profiling
segments (CUDA events around each launch on the executor's stream).

    python -m nvcr_b200.stack_profile --stack intra --latent 68 120 --runs 5

prints, per kernel family, the time and launches per run, then the ops (block
indices folded together) by time with their algorithmic TOPS and GB/s. The
stacks are the synthetic BASELINE config 3 (intra) and config 4 (inter)
decoders with seeded weights; inputs are seeded integer latents (and, for the
inter decoder, a seeded temporal context), passed as FP16 device tensors.
Profiling adds one event pair per launch and disables graph replay, so the
per-run total is above the bench's frame time.
"""
from __future__ import annotations

import argparse
import collections
import re

import numpy as np


def profile_stack(stack, runs: int, warmup: int) -> tuple[list[dict], float]:
    import torch

    from .executor import CudaExecutor
    from .program import SeededStream
    from .workloads import laplace_latent

    with CudaExecutor.from_program(stack.program) as executor:
        stream = SeededStream(1)
        inputs = {}
        for index, (name, shape) in enumerate(zip(executor.input_names, stack.input_shapes)):
            values = laplace_latent(stream, shape) if index == 0 else stream.tensor(*shape, 1.0)
            inputs[name] = torch.from_numpy(values.astype(np.float16)).cuda()
        outputs = {}
        for name, shape in zip(executor.output_names, executor.infer_output_extents(stack.input_shapes)):
            outputs[name] = torch.empty(shape, dtype=torch.float16, device="cuda")
        for _ in range(warmup):
            executor.run_half(inputs, outputs)
        executor.synchronize()
        executor.profile()
        executor.set_profiling(True)
        for _ in range(runs):
            executor.run_half(inputs, outputs)
        executor.synchronize()
        segments = executor.profile()
        executor.set_profiling(False)
    return segments, float(runs)


def report(segments: list[dict], runs: float) -> str:
    by_kernel = collections.defaultdict(lambda: [0, 0.0])
    by_op = collections.defaultdict(lambda: [0, 0.0, 0.0, 0.0])
    for s in segments:
        by_kernel[s["kernel"]][0] += 1
        by_kernel[s["kernel"]][1] += s["ms"]
        # Fold the block index in front of a DepthConvBlock's parts (dec_1.7.ffn.1 -> dec_1.ffn.1).
        op = re.sub(r"\.\d+\.(?=(dc|ffn|conv|adaptor|up|shortcut)\b)", ".", s["label"])
        entry = by_op[op]
        entry[0] += 1
        entry[1] += s["ms"]
        entry[2] += s["ops"]
        entry[3] += s["bytes"]
    total = sum(v[1] for v in by_kernel.values()) / runs
    lines = [f"total {total:.3f} ms per run", "", "| kernel | ms per run | share | launches per run |",
             "|---|---:|---:|---:|"]
    for kernel, (count, ms) in sorted(by_kernel.items(), key=lambda kv: -kv[1][1]):
        lines.append(f"| {kernel} | {ms / runs:.3f} | {100 * ms / runs / total:.1f}% | {count / runs:.0f} |")
    lines += ["", "| op (block indices folded) | launches per run | ms per run | TOPS | GB/s |", "|---|---:|---:|---:|---:|"]
    for op, (count, ms, ops, nbytes) in sorted(by_op.items(), key=lambda kv: -kv[1][1]):
        seconds = ms / 1e3
        tops = ops / seconds / 1e12 if seconds > 0 else 0.0
        gbs = nbytes / seconds / 1e9 if seconds > 0 else 0.0
        lines.append(f"| {op} | {count / runs:.0f} | {ms / runs:.3f} | {tops:.1f} | {gbs:.0f} |")
    return "\n".join(lines)


def main() -> None:
    from .workloads import inter_decoder, intra_decoder

    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("--stack", choices=["intra", "inter"], default="intra")
    parser.add_argument("--latent", type=int, nargs=2, default=None, metavar=("H", "W"),
                        help="latent height and width (default 68 120, a 1088 x 1920 frame, for the intra "
                             "decoder; 48 80, a 768 x 1280 frame, for the inter decoder)")
    parser.add_argument("--runs", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    args = parser.parse_args()
    if args.stack == "intra":
        stack = intra_decoder(tuple(args.latent) if args.latent else (68, 120))
    else:
        stack = inter_decoder(tuple(args.latent) if args.latent else (48, 80))
    segments, runs = profile_stack(stack, args.runs, args.warmup)
    print(report(segments, runs))


if __name__ == "__main__":
    main()
