"""Measures the dense int8 tensor-core rate of this GPU through the vendor
library, as the denominator for the integer conv's roofline fraction.

    python -m nvcr_b200.peak [--size 8192] [--seconds 4]

torch._int_mm (cuBLASLt, int8 x int8 -> int32) on square matrices: the best of
10 launches timed alone with CUDA events (burst), then back-to-back launches
for `--seconds` (sustained, under the power cap), with nvidia-smi clocks sampled
during the sustained loop. The same for a bf16 matmul, for the ratio to the
driver's measured bf16 figure. Prints one JSON line. Measurement only: nothing
in the library uses it.
"""
from __future__ import annotations

import argparse
import json
import subprocess
import time


def rate(run, ops: float, seconds: float) -> dict:
    import torch

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        run()
        end.record()
        torch.cuda.synchronize()
        best = min(best, start.elapsed_time(end) / 1000.0)
    sampler = subprocess.Popen(["nvidia-smi", "--query-gpu=index,clocks.sm,power.draw,clocks_event_reasons.active",
                                "--format=csv,noheader,nounits", "-i", "0", "-lms", "200"],
                               stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    count = 0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall = time.time()
    start.record()
    while time.time() - wall < seconds:
        for _ in range(20):
            run()
        count += 20
        torch.cuda.synchronize()
    end.record()
    torch.cuda.synchronize()
    sustained = start.elapsed_time(end) / 1000.0 / count
    sampler.terminate()
    lines = sampler.communicate(timeout=5)[0].splitlines()
    clocks = sorted(float(line.split(",")[1]) for line in lines if line.count(",") >= 3)
    return {"burst": ops / best / 1e12, "sustained": ops / sustained / 1e12,
            "sm_mhz_median": clocks[len(clocks) // 2] if clocks else None, "launches": count}


def main() -> None:
    import torch

    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--size", type=int, default=8192)
    parser.add_argument("--seconds", type=float, default=4.0)
    args = parser.parse_args()
    n = args.size
    ops = 2.0 * n * n * n
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()  # column-major operand
    int8 = rate(lambda: torch._int_mm(a, b), ops, args.seconds)
    x = torch.randn((n, n), dtype=torch.bfloat16, device="cuda")
    y = torch.randn((n, n), dtype=torch.bfloat16, device="cuda")
    bf16 = rate(lambda: torch.matmul(x, y), ops, args.seconds)
    print(json.dumps({"gpu": torch.cuda.get_device_name(0), "size": n, "int8_tops": int8, "bf16_tflops": bf16,
                      "int8_over_bf16_burst": int8["burst"] / bf16["burst"],
                      "how": "torch._int_mm int8 (cuBLASLt) and torch.matmul bf16, 2 N^3 ops, best of 10 "
                             "(burst) and back to back (sustained)"}), flush=True)


if __name__ == "__main__":
    main()
