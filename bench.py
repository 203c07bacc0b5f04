#!/usr/bin/env python3
"""Benchmark of the nvcr.intconv.v1 exact-convolution path on B200.

Workload: the 1920x1088 layer sweep, w8a8 integer convs
lowered as the reference's exporter lowers them (im2col + pointwise conv), FP16
at the stage boundary, every value an int8 in [-127, 127] from a seeded
std::mt19937 stream:
  L1 3x3 s2 3->64 at 1088x1920, L2 3x3 64->64 at 544x960, L3 1x1 128->256 at
  272x480, L4 3x3 256->256 at 136x240, L5 3x3 256->1024 at 68x120 + depth_to_space 2.
A step runs the five layers once (125.9 G algorithmic int8 ops, one MAC = 2 ops;
limb expansion and padding are not counted). The step touches about 1 GB, far
more than the 126 MB L2, so no L2 flush is inserted.

  value  whole-job int8 TOPS with inputs resident in HBM (device FP16 tensors);
  e2e    the same through the C ABI with pinned host FP16 buffers, every
         step's host->device input copies and device->host output copies inside
         the timing (uploads, runs and downloads of different layers overlap on
         three streams);
  roofline  the fused conv kernel (CUDA events on its stream, timed region).

N > 1 (torchrun): every rank runs the same sweep on its own GPU (independent
replicas, no collective on the data path); value = all ranks' ops / max time.
`--impl reference` times the reference's own CPU executor (run_cpu, compiled
from its sources into oracle/_ref) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MEASURED_PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
CPU_BASELINE_FRACTION = 2   # cpu_baseline leg: the first half of each layer's output rows
REFERENCE_ARM_FRACTION = 32  # --impl reference: 1/32 per step, so K + W steps end in minutes


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-cpu-baseline", action="store_true", help="skip the reference CPU timing")
    parser.add_argument("--layers", type=str, default="", help="comma-separated layer indices (default: all)")
    parser.add_argument("--no-decoder", action="store_true", help="skip the config 3-5 decoder measurements")
    parser.add_argument("--no-reference-gpu", action="store_true",
                        help="skip timing the reference's own CUDA executor (the GPU comparator)")
    return parser.parse_args()


GOLDEN = ROOT / "tests" / "golden" / "fullsize_digests.json"


def golden_digests() -> dict:
    """The reference run_cpu's digests of the benchmark's outputs at full size
    (tests/golden/make_fullsize_digests.py); empty when the file is absent."""
    return json.loads(GOLDEN.read_text()) if GOLDEN.exists() else {}


INT8_PEAK = ROOT / "profiles" / "int8_peak_cublaslt.json"


def int8_peak_tops(bf16: float, source: str) -> tuple[float, str]:
    """The dense int8 rate measured on this pool (cuBLASLt int8 GEMM burst,
    profiles/int8_peak_cublaslt.md), else twice the bf16 figure."""
    if INT8_PEAK.exists():
        data = json.loads(INT8_PEAK.read_text())
        return data["int8_tops_burst"], f"measured: cuBLASLt int8 8192^3 burst ({INT8_PEAK.name})"
    return 2.0 * bf16, f"2 x bf16 dense ({source} MEASURED_PEAKS bf16_tflops={bf16})"


def peaks():
    if MEASURED_PEAKS.exists():
        data = json.loads(MEASURED_PEAKS.read_text())
        return data["hbm_gbs"], data["bf16_tflops"], "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None) -> None:
        self.uuid = uuid
        self.process = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.process = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.process.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.process is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.process.terminate()
        try:
            self.process.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.process.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, sm_max, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            if self.uuid and parts[1] != self.uuid:
                continue
            try:
                sm.append(float(parts[2]))
                sm_max.append(float(parts[3]))
                power.append(float(parts[4]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[6:10]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(sm_max), "power_w_max": max(power),
                "samples": len(sm), "reasons": sorted(reasons)}


def distributed():
    from nvcr_b200.replicas import rank_environment

    env = rank_environment()
    return env.world, env.rank, env.local


def select_layers(spec: str):
    from nvcr_b200.workloads import config2

    layers = config2()
    if spec:
        layers = [layers[int(i)] for i in spec.split(",")]
    return layers


def input_seed(layer) -> int:
    """Config 2 layer i's input comes from seed 200 + i, whichever layers run."""
    from nvcr_b200.workloads import config2

    return 200 + [candidate.name for candidate in config2()].index(layer.name)


def reference_sample(layers, directory: Path, fraction: int, repeats: int = 1):
    """Times the reference's run_cpu on the first 1/`fraction` of each layer's
    output rows (the input rows that feed them); returns (TOPS, seconds, ops, sample text)."""
    import numpy as np

    from nvcr_b200.workloads import layer_input
    from oracle.oracle import Reference

    reference = Reference()
    total_ops = 0.0
    total_seconds = 0.0
    parts = []
    for index, layer in enumerate(layers):
        c, h, w = layer.input_shape
        node = [n for n in layer.program.nodes if n.kind.name == "im2col"]
        stride = node[0].stride[0] if node else 1
        kernel = node[0].kernel[0] if node else 1
        out_h = (h + (2 if node else 0) - kernel) // stride + 1
        rows_out = max(1, out_h // fraction)
        rows_in = min(h, rows_out * stride + (kernel - 1))
        x = layer_input(layer, seed=input_seed(layer), height=rows_in)
        path = layer.program.write(directory, layer.name)
        seconds = reference.time_run(path, [x], repeats=repeats)
        sample_out_h = (rows_in + (2 if node else 0) - kernel) // stride + 1
        ops = layer.ops * sample_out_h / out_h
        total_ops += ops
        total_seconds += seconds
        parts.append(f"{layer.name}: {rows_in}/{h} input rows")
    tops = total_ops / total_seconds / 1e12
    return tops, total_seconds, total_ops, "; ".join(parts)


def run_reference_arm(args):
    world, rank, _ = distributed()
    if rank != 0:
        return 0
    layers = select_layers(args.layers)
    threads = min(os.cpu_count() or 1, 16)
    with tempfile.TemporaryDirectory() as directory:
        for _ in range(args.warmup):
            reference_sample(layers, Path(directory), REFERENCE_ARM_FRACTION)
        times = []
        ops = 0.0
        sample = ""
        for _ in range(args.steps):
            tops, seconds, ops, sample = reference_sample(layers, Path(directory), REFERENCE_ARM_FRACTION)
            times.append(seconds)
    total = sum(times)
    value = ops * args.steps / total / 1e12
    line = {
        "impl": "reference", "metric": "int8 conv TOPS (config 2 layer sweep, bit-exact intconv.v1)",
        "value": value, "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded mt19937 int8 values)",
        "config": {"workload": "config2: 1920x1088 layer sweep L1-L5, w8a8, FP16 stage boundary",
                   "parallelism": "reference CPU run_cpu, rank 0 only"},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": "reference",
                         "sample": f"reference run_cpu (oracle/_ref) on {sample}"},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)

    import numpy as np
    import torch

    from nvcr_b200.replicas import Group, rank_environment

    env = rank_environment()
    world, rank, local = env.world, env.rank, env.local
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = Group(env, "nccl", device)

    from nvcr_b200.executor import CudaExecutor
    from nvcr_b200.workloads import layer_input

    layers = select_layers(args.layers)
    stream = torch.cuda.Stream(device=device)
    executors, inputs, outputs, pinned_in, pinned_out = [], [], [], [], []
    for index, layer in enumerate(layers):
        executor = CudaExecutor.from_program(layer.program, stream=stream.cuda_stream)
        x = layer_input(layer, seed=input_seed(layer))
        (c, h, w), = executor.infer_output_extents([x.shape])
        xh = torch.from_numpy(x.astype(np.float16)).to(device)
        yh = torch.empty((c, h, w), dtype=torch.float16, device=device)
        executors.append(executor)
        inputs.append(xh)
        outputs.append(yh)
        pinned_in.append(torch.from_numpy(x.astype(np.float16)).pin_memory())
        pinned_out.append(torch.empty((c, h, w), dtype=torch.float16).pin_memory())
    ops_per_step = sum(layer.ops for layer in layers)

    def step():
        for executor, xh, yh in zip(executors, inputs, outputs):
            executor.run_half({"x": xh}, {"y": yh})

    # End to end: each layer's host input is copied in on one stream, run on the
    # executors' stream and its result copied back on a third, ordered by events,
    # so one layer's upload, another's compute and another's download overlap
    # (PCIe moves both directions at once). Events also order the reuse of each
    # layer's device buffers across steps.
    copy_in = torch.cuda.Stream(device=device)
    copy_out = torch.cuda.Stream(device=device)
    in_done = [torch.cuda.Event() for _ in layers]
    run_done = [torch.cuda.Event() for _ in layers]
    out_done = [torch.cuda.Event() for _ in layers]
    for events in (run_done, out_done):
        for event in events:
            event.record(stream)

    def step_e2e():
        for i, (executor, xh, yh, hi, ho) in enumerate(zip(executors, inputs, outputs, pinned_in, pinned_out)):
            copy_in.wait_event(run_done[i])      # the previous step's run has read xh
            with torch.cuda.stream(copy_in):
                xh.copy_(hi, non_blocking=True)
            in_done[i].record(copy_in)
            stream.wait_event(in_done[i])
            stream.wait_event(out_done[i])       # the previous step's download has read yh
            executor.run_half({"x": xh}, {"y": yh})
            run_done[i].record(stream)
            copy_out.wait_event(run_done[i])
            with torch.cuda.stream(copy_out):
                ho.copy_(yh, non_blocking=True)
            out_done[i].record(copy_out)

    barrier = group.barrier
    max_over_ranks = group.max

    def timed(function, steps, profile=False):
        for executor in executors:
            executor.set_profiling(profile)
        barrier()
        torch.cuda.synchronize(device)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        copy_in.wait_event(start)
        copy_out.wait_event(start)
        for _ in range(steps):
            function()
        # The region ends when all three streams are done.
        stream.wait_stream(copy_in)
        stream.wait_stream(copy_out)
        end.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        for executor in executors:
            executor.synchronize()
        return start.elapsed_time(end)

    # Warm-up (plans, arenas, TMA maps), then the timed region.
    for _ in range(max(args.warmup, 3)):
        step()
    for executor in executors:
        executor.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid).start()
    time.sleep(0.3)
    elapsed_ms = timed(step, args.steps)
    clocks = sampler.stop()
    launches = sum(e.launches for e in executors) * args.steps
    elapsed_ms = max_over_ranks(elapsed_ms)
    # Per-kernel CUDA events over a second timed region of the same steps
    # (profiling records events between kernels, so these runs are not replayed
    # from CUDA graphs).
    timed(step, args.steps, profile=True)
    per_layer_segments = [e.profile() for e in executors]
    value = world * ops_per_step * args.steps / (elapsed_ms / 1000.0) / 1e12

    # End to end through the C ABI with host buffers.
    for _ in range(2):
        step_e2e()
    e2e_ms = max_over_ranks(timed(step_e2e, args.steps))
    e2e_value = world * ops_per_step * args.steps / (e2e_ms / 1000.0) / 1e12
    h2d = sum(t.numel() * 2 for t in pinned_in)
    d2h = sum(t.numel() * 2 for t in pinned_out)

    # Parity at full size: every layer's output as the last end-to-end step left
    # it in host memory, against the reference's digest of the same layer.
    from nvcr_b200.workloads import half_digest

    golden = golden_digests()
    expected = golden.get("config2", {})
    unchecked = [layer.name for layer in layers if layer.name not in expected]
    differing = [layer.name for layer, host in zip(layers, pinned_out)
                 if layer.name in expected and half_digest(host.numpy()) != expected[layer.name]["digest"]]
    parity = {"checker": "SHA-256 of each FP16 output against the reference run_cpu's (tests/golden/"
                         "fullsize_digests.json, NaN as 0x7e00), every rank",
              "config2": {"outputs_checked": int(group.sum(len(layers) - len(unchecked))),
                          "differing": int(group.sum(len(differing))), "differing_here": differing,
                          "unchecked": unchecked}}

    # Roofline of the integer conv kernel and per-layer bounds. A layer's time is
    # the kernels a timed (graph-replayed) run launches: activation quantisation
    # or staging and the conv; its algorithmic bytes are the FP16 input once, the
    # int8 weights once and the FP16 output once.
    hbm, bf16, source = peaks()
    int8_peak, int8_source = int8_peak_tops(bf16, source)
    ridge = int8_peak * 1e12 / (hbm * 1e9)  # ops per byte
    kernel_ms: dict[str, float] = {}
    for segments in per_layer_segments:
        for seg in segments:
            kernel_ms[seg["kernel"]] = kernel_ms.get(seg["kernel"], 0.0) + seg["ms"]
    total_ms = sum(kernel_ms.values())
    shares = {k: round(v / total_ms, 3) for k, v in sorted(kernel_ms.items(), key=lambda kv: -kv[1])} \
        if total_ms else {}
    layer_rows = []
    tensor_ops = tensor_ms = all_ops = all_ms = 0.0
    for layer, segments, yh in zip(layers, per_layer_segments, outputs):
        gemms = [seg for seg in segments if seg["kernel"] == "integer_conv"]
        if not gemms:
            continue
        runs = len(gemms)
        conv_ms = sum(seg["ms"] for seg in gemms) / runs
        prep_ms = sum(seg["ms"] for seg in segments if seg["kernel"] in ("quantise", "stage_source")) / runs
        # The gated fallback launches of a direct conv appear only in these
        # profiled runs (launched directly); the timed runs replay CUDA graphs in
        # which the fallback is a conditional node that no mixed window set.
        fallback_ms = sum(seg["ms"] for seg in segments if seg["kernel"] == "fallback") / runs
        layer_ms = conv_ms + prep_ms
        ops = gemms[0]["ops"]
        cin, h, w = layer.input_shape
        pointwise = [n for n in layer.program.nodes if n.kind.name == "conv"][0]  # K = cin * taps inputs
        algorithmic = 2.0 * cin * h * w + pointwise.in_channels * pointwise.out_channels + 2.0 * yh.numel()
        bound = "tensor" if ops / algorithmic > ridge else "hbm"
        conv_tops = ops / (conv_ms / 1000.0) / 1e12
        layer_tops = ops / (layer_ms / 1000.0) / 1e12
        layer_gbs = algorithmic / (layer_ms / 1000.0) / 1e9
        layer_rows.append({"layer": layer.name, "conv_ms": round(conv_ms, 4), "prep_ms": round(prep_ms, 4),
                           "fallback_gated_ms": round(fallback_ms, 4), "layer_ms": round(layer_ms, 4),
                           "conv_tops": round(conv_tops, 1), "layer_tops": round(layer_tops, 1),
                           "algorithmic_bytes": algorithmic, "layer_gbs": round(layer_gbs, 1), "bound": bound,
                           "frac": round(conv_tops / int8_peak if bound == "tensor" else layer_gbs / hbm, 3),
                           "frac_basis": ("conv kernel ops / int8 peak" if bound == "tensor"
                                          else "whole-layer algorithmic bytes / HBM peak")})
        all_ops += ops
        all_ms += conv_ms
        if bound == "tensor":
            tensor_ops += ops
            tensor_ms += conv_ms
    if tensor_ms > 0:
        achieved = tensor_ops / (tensor_ms / 1000.0) / 1e12
    else:
        achieved = all_ops / (all_ms / 1000.0) / 1e12 if all_ms else 0.0
    traffic = None
    traffic_file = ROOT / "profiles" / "direct_conv_traffic.json"
    if traffic_file.exists():
        traffic = json.loads(traffic_file.read_text()).get("bytes_per_launch")
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1), "unit": "TOPS",
                "frac": round(achieved / int8_peak, 4), "traffic": traffic,
                "kernel": "direct_conv_kernel on the tensor-bound layers (L4, L5): tcgen05 kind::i8 over the int8 "
                          "per-pixel copy, row-halo A stages; traffic: one L4 launch (profiles/direct_conv_traffic.json)",
                "peak_source": int8_source,
                "time_share": shares,
                "layers": layer_rows}

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            with tempfile.TemporaryDirectory() as directory:
                tops, seconds, _, sample = reference_sample(layers, Path(directory), CPU_BASELINE_FRACTION)
            cpu_baseline = {"value": tops, "unit": "TOPS", "cores": min(os.cpu_count() or 1, 16),
                            "kind": "reference", "seconds": round(seconds, 2),
                            "sample": f"reference run_cpu (oracle/_ref) on {sample}"}
        except Exception as error:  # the reference build may be absent
            cpu_baseline = {"value": None, "unit": "TOPS", "cores": 0, "kind": "reference",
                            "sample": f"unavailable: {error}"}

    reference_gpu = None
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        try:
            reference_gpu = reference_gpu_leg(layers, device, golden, args.no_decoder)
        except Exception as error:  # the comparator build may be absent
            reference_gpu = {"unavailable": str(error)}

    decoder = None
    if not args.no_decoder:
        decoder = decoder_throughput(args, device, rank, world, group, golden)
        parity.update(decoder.pop("parity"))

    if rank == 0:
        line = {
            "metric": "int8 conv TOPS (config 2 layer sweep, bit-exact intconv.v1)",
            "value": round(value, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded mt19937 int8 values)",
            "config": {"workload": "config2: 1920x1088 layer sweep L1-L5, w8a8, FP16 stage boundary",
                       "layers": [layer.name for layer in layers], "ops_per_step": ops_per_step,
                       "l2": "inputs larger than L2 (about 1 GB touched per step), no flush",
                       "parallelism": f"replicas x{world}"},
            "e2e": {"value": round(e2e_value, 2), "unit": "TOPS", "ms_per_step": round(e2e_ms / args.steps, 4),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": roofline,
            "cpu_baseline": cpu_baseline,
            "clocks": clocks,
            "gpu_launches": launches,
            "parity": parity,
            "decoder": decoder,
            "reference_gpu": reference_gpu,
        }
        print(json.dumps(line), flush=True)
    for executor in executors:
        executor.close()
    group.close()
    return 0


def reference_gpu_leg(layers, device, golden, skip_decoder: bool) -> dict:
    """The GPU comparator: the reference's own CUDA executor (CudaExecutor, its
    cuda_executor.cu built for sm_100a with its flags into
    oracle/_ref/libnvcr_ref_cuda.so) through its public run_half, on the same
    device-resident FP16 inputs as this path, timed with CUDA events on its
    stream after warm-up: the config-2 layers one by one and one config-3
    frame. Its outputs are checked against the reference run_cpu's digests."""
    import numpy as np
    import torch

    from nvcr_b200.program import SeededStream
    from nvcr_b200.workloads import half_digest, intra_decoder, laplace_latent, layer_input
    from oracle.oracle import ReferenceGpu

    if not ReferenceGpu.available():
        return {"unavailable": "oracle/_ref/libnvcr_ref_cuda.so is not built"}
    stream = torch.cuda.Stream(device=device)

    def time_runs(run, count):
        for _ in range(2):
            run()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(count):
            run()
        end.record(stream)
        torch.cuda.synchronize(device)
        return start.elapsed_time(end) / count

    rows = []
    total_ms = total_ops = 0.0
    differing = []
    with tempfile.TemporaryDirectory() as directory:
        for layer in layers:
            x = layer_input(layer, seed=input_seed(layer))
            path = layer.program.write(directory, layer.name)
            shape = tuple(golden.get("config2", {}).get(layer.name, {}).get("shape", ()))
            with ReferenceGpu(path, stream.cuda_stream) as executor:
                xh = torch.from_numpy(x.astype(np.float16)).to(device)
                if not shape:
                    continue
                yh = torch.empty(shape, dtype=torch.float16, device=device)
                ms = time_runs(lambda: executor.run_half({"x": xh}, {"y": yh}), 3)
                if half_digest(yh.cpu().numpy()) != golden["config2"][layer.name]["digest"]:
                    differing.append(layer.name)
            rows.append({"layer": layer.name, "ms": round(ms, 4), "tops": round(layer.ops / (ms / 1000.0) / 1e12, 2)})
            total_ms += ms
            total_ops += layer.ops
        result = {"what": "reference CudaExecutor::run_half (sm_80-style mma.sync int8 kernels) on this B200",
                  "config2": {"tops": round(total_ops / (total_ms / 1000.0) / 1e12, 2) if total_ms else None,
                              "ms_per_step": round(total_ms, 3), "layers": rows, "differing": differing}}
        if not skip_decoder:
            stack = intra_decoder()
            path = stack.program.write(directory, "intra_1080p")
            latent = torch.from_numpy(laplace_latent(SeededStream(5000), stack.input_shapes[0])
                                      .astype(np.float16)).to(device)
            frame = torch.empty((3, 1088, 1920), dtype=torch.float16, device=device)
            with ReferenceGpu(path, stream.cuda_stream) as executor:
                ms = time_runs(lambda: executor.run_half({"y_hat": latent}, {"frame": frame}), 3)
                same = half_digest(frame.cpu().numpy()) == golden.get("config3", {}).get("0", {}).get("digest")
            result["config3"] = {"ms_per_frame": round(ms, 3), "frames_per_s": round(1000.0 / ms, 2),
                                 "tops": round(stack.ops / (ms / 1000.0) / 1e12, 2), "matches_reference_cpu": same}
    return result


def decoder_throughput(args, device, rank, world, group, golden) -> dict:
    """BASELINE configs 3 and 5 on the synthetic DCVC-RT intra decoder (1080p:
    y_hat [256, 68, 120] -> frame [3, 1088, 1920], FP16 boundary).

    Config 3: one stream's frame time with the latent resident on the device,
    at w8a8 (BASELINE) and at w16a16 (the reference width map's default for the
    intra decoder). Config 5: 64 independent streams x 16 GOP-1 frames, stream
    s on rank s mod world, aggregate frames/s over the max-over-ranks device
    time (strong scaling: the 1024 frames are fixed); once with the latents
    resident on the device, and once end to end: every frame's latent copied in
    from pinned host memory and its frame copied back out inside the timing
    (copies and decodes of different frames overlap on three streams). Parity:
    every stream's frame, as the end-to-end run left it in host memory, against
    the reference's digest; config 3's frame likewise."""
    import numpy as np
    import torch

    from nvcr_b200.executor import CudaExecutor
    from nvcr_b200.program import SeededStream
    from nvcr_b200.replicas import streams_of
    from nvcr_b200.workloads import half_digest, intra_decoder, laplace_latent

    barrier = group.barrier
    stack = intra_decoder()
    streams, frames = 64, 16
    mine = streams_of(rank, world, streams)
    torch_stream = torch.cuda.Stream(device=device)
    copy_in = torch.cuda.Stream(device=device)
    copy_out = torch.cuda.Stream(device=device)
    expected = golden.get("config3", {})

    def timed(count, work, executors=()):
        barrier()
        torch.cuda.synchronize(device)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(torch_stream)
        copy_in.wait_event(start)
        copy_out.wait_event(start)
        for i in range(count):
            work(i)
        torch_stream.wait_stream(copy_in)
        torch_stream.wait_stream(copy_out)
        end.record(torch_stream)
        torch.cuda.synchronize(device)
        for e in executors:
            e.synchronize()
        barrier()
        return start.elapsed_time(end)

    with CudaExecutor.from_program(stack.program, stream=torch_stream.cuda_stream) as executor:
        host_latents = [torch.from_numpy(laplace_latent(SeededStream(5000 + s), stack.input_shapes[0])
                                         .astype(np.float16)).pin_memory() for s in mine]
        latents = [h.to(device) for h in host_latents]
        (c, h, w), = executor.infer_output_extents(stack.input_shapes)
        frame = torch.empty((c, h, w), dtype=torch.float16, device=device)

        def decode(latent, out=frame):
            executor.run_half({"y_hat": latent}, {"frame": out})

        for _ in range(3):
            decode(latents[0])
        executor.synchronize()
        single = 10
        frame_ms = timed(single, lambda i: decode(latents[0]), (executor,)) / single
        config3_checked = str(mine[0]) in expected
        config3_ok = not config3_checked or half_digest(frame.cpu().numpy()) == expected[str(mine[0])]["digest"]
        shard_ms = group.max(timed(len(mine) * frames, lambda i: decode(latents[i // frames]), (executor,)))
        launches = executor.launches

        # End to end: two device latent/frame slots; frame i uses slot i % 2.
        slots = 2
        latent_slots = [torch.empty_like(latents[0]) for _ in range(slots)]
        frame_slots = [torch.empty_like(frame) for _ in range(slots)]
        host_frames = [torch.empty((c, h, w), dtype=torch.float16).pin_memory() for _ in mine]
        in_done = [torch.cuda.Event() for _ in range(slots)]
        run_done = [torch.cuda.Event() for _ in range(slots)]
        out_done = [torch.cuda.Event() for _ in range(slots)]
        for events in (run_done, out_done):
            for event in events:
                event.record(torch_stream)

        def decode_e2e(i):
            k = i % slots
            s = i // frames
            copy_in.wait_event(run_done[k])      # the decode that read this slot is done
            with torch.cuda.stream(copy_in):
                latent_slots[k].copy_(host_latents[s], non_blocking=True)
            in_done[k].record(copy_in)
            torch_stream.wait_event(in_done[k])
            torch_stream.wait_event(out_done[k])  # the download from this slot is done
            decode(latent_slots[k], frame_slots[k])
            run_done[k].record(torch_stream)
            copy_out.wait_event(run_done[k])
            with torch.cuda.stream(copy_out):
                host_frames[s].copy_(frame_slots[k], non_blocking=True)
            out_done[k].record(copy_out)

        for i in range(2 * slots):
            decode_e2e(i)
        e2e_ms = group.max(timed(len(mine) * frames, decode_e2e, (executor,)))
        differing = [s for s, host in zip(mine, host_frames)
                     if str(s) in expected and half_digest(host.numpy()) != expected[str(s)]["digest"]]
        h2d = host_latents[0].numel() * 2
        d2h = c * h * w * 2

    # w16a16, the width the reference's width map gives the intra decoder.
    stack16 = intra_decoder(bits=(16, 16))
    with CudaExecutor.from_program(stack16.program, stream=torch_stream.cuda_stream) as executor16:
        for _ in range(3):
            executor16.run_half({"y_hat": latents[0]}, {"frame": frame})
        executor16.synchronize()
        frame16_ms = timed(single, lambda i: executor16.run_half({"y_hat": latents[0]}, {"frame": frame}),
                           (executor16,)) / single

    p_frames, p_parity = p_frame_sequence(device, torch_stream, timed, golden)
    checked5 = sum(1 for s in mine if str(s) in expected)
    parity = {
        "config3": {"outputs_checked": int(group.sum(1 if config3_checked else 0)),
                    "differing": int(group.sum(0 if config3_ok else 1))},
        "config4": p_parity,
        "config5": {"outputs_checked": int(group.sum(checked5)), "differing": int(group.sum(len(differing))),
                    "differing_here": differing, "what": "each stream's frame as the end-to-end run left it "
                                                         "in host memory"},
    }
    return {
        "workload": "synthetic DCVC-RT intra decoder (i.dec topology: subpel up + 14 DepthConvBlocks at "
                    "256 ch, 1/8 res + d2s(8) head), 1088x1920 frame, FP16 boundary",
        "ops_per_frame": stack.ops,
        "config3": {"ms_per_frame": round(frame_ms, 3), "frames_per_s": round(1000.0 / frame_ms, 1),
                    "tops": round(stack.ops / (frame_ms / 1000.0) / 1e12, 1), "gpu_launches_per_frame": launches,
                    "widths": "w8a8"},
        "config3_w16a16": {"ms_per_frame": round(frame16_ms, 3), "frames_per_s": round(1000.0 / frame16_ms, 1),
                           "tops": round(stack.ops / (frame16_ms / 1000.0) / 1e12, 1),
                           "widths": "w16a16 (the reference width map's default)"},
        "config4": p_frames,
        "config5": {"streams": streams, "frames_per_stream": frames, "n_gpus": world, "ms": round(shard_ms, 2),
                    "frames_per_s": round(streams * frames / (shard_ms / 1000.0), 1),
                    "tops_per_gpu": round(streams * frames * stack.ops / world / (shard_ms / 1000.0) / 1e12, 1),
                    "scaling": "strong (1024 frames split round-robin by stream)",
                    "e2e": {"ms": round(e2e_ms, 2), "frames_per_s": round(streams * frames / (e2e_ms / 1000.0), 1),
                            "h2d_bytes_per_frame": h2d, "d2h_bytes_per_frame": d2h}},
        "parity": parity,
    }


def p_frame_sequence(device, torch_stream, timed, golden) -> tuple[dict, dict]:
    """BASELINE config 4 on the synthetic stacks: 1280x720 (padded to 768x1280), GOP
    30 = one I-frame (intra decoder with a 64-channel feature output) and 29
    P-frames whose temporal context is the previous frame's feature, run in order
    on one GPU with one executor per mode (plans and scratch reused); FP16 stage
    boundary, everything device-resident. After the timing the sequence runs
    once more and every frame and feature is checked against the reference's
    digests."""
    import numpy as np
    import torch

    from nvcr_b200.executor import CudaExecutor
    from nvcr_b200.program import SeededStream
    from nvcr_b200.workloads import half_digest, inter_decoder, intra_decoder, laplace_latent

    intra = intra_decoder((48, 80), feature_channels=64)
    inter = inter_decoder((48, 80))
    gop = 30
    expected = golden.get("config4", [])
    with CudaExecutor.from_program(intra.program, stream=torch_stream.cuda_stream) as first, \
            CudaExecutor.from_program(inter.program, stream=torch_stream.cuda_stream) as rest:
        latents = [torch.from_numpy(laplace_latent(SeededStream(6000 + f), (256, 48, 80)).astype(np.float16))
                   .to(device) for f in range(gop)]
        frame = torch.empty((3, 768, 1280), dtype=torch.float16, device=device)
        features = [torch.empty((64, 96, 160), dtype=torch.float16, device=device) for _ in range(2)]

        def decode(f):
            if f == 0:
                first.run_half({"y_hat": latents[0]}, {"frame": frame, "feature": features[0]})
            else:
                rest.run_half({"y_hat": latents[f], "context": features[(f - 1) % 2]},
                              {"frame": frame, "feature": features[f % 2]})

        for f in range(3):
            decode(f)
        ms = timed(gop, decode, (first, rest))
        differing = []
        for f in range(gop if len(expected) == gop else 0):
            decode(f)
            torch.cuda.synchronize(device)
            if half_digest(frame.cpu().numpy()) != expected[f]["frame"]:
                differing.append(f"frame {f}")
            if half_digest(features[f % 2].cpu().numpy()) != expected[f]["feature"]:
                differing.append(f"feature {f}")
    ops = intra.ops + (gop - 1) * inter.ops
    result = {"frames": gop, "resolution": "768x1280 (720p padded to x64)", "ms": round(ms, 3),
              "frames_per_s": round(gop / (ms / 1000.0), 1), "tops": round(ops / (ms / 1000.0) / 1e12, 1)}
    parity = {"outputs_checked": 2 * gop if len(expected) == gop else 0, "differing": len(differing),
              "differing_here": differing, "what": "every frame and feature of the GOP (rank 0's run)"}
    return result, parity


if __name__ == "__main__":
    sys.exit(main())
