"""nvcr.intconv.v1 programs on the host: the in-memory form and the on-disk form.

Mirrors the reference's program model (0elghati/nvcr
src/deterministic/program.hpp:57-136: ``OpKind``, ``Node``, ``Program``) and
writes the on-disk format its loader reads (program.cpp:537-626) and its
exporter writes (scripts/backends/dcvcrt/export_deterministic_program.py:449-484):
``<name>.detprog.json`` plus ``<name>.detw``, raw little-endian FP16 weights
whose SHA-256 the JSON pins.

The arithmetic contract of the profile (program.hpp:1-44):
  * every pointwise dense conv (1x1, stride 1, no padding) is an exact integer
    conv at the node's weight/activation widths (8 or 16 bits, default 16);
  * every other op is FP32 with a fixed operation order;
  * a dense spatial conv reaches the executor as ``im2col`` + pointwise conv.
"""
from __future__ import annotations

import dataclasses
import enum
import hashlib
import json
from pathlib import Path
from typing import Iterable, Sequence

import numpy as np

FORMAT = "nvcr.deterministic-program"
VERSION = 1
INTCONV_PROFILE = "nvcr.intconv.v1"


class OpKind(enum.IntEnum):
    """Op set in the reference's enum order (program.hpp:57-71)."""

    conv = 0
    mul = 1
    add = 2
    mul_scalar = 3
    sigmoid = 4
    slice_channels = 5
    depth_to_space = 6
    scale_channels = 7
    clamp = 8
    concat = 9
    crop = 10
    space_to_depth = 11
    im2col = 12


BINARY_OPS = {OpKind.mul, OpKind.add, OpKind.scale_channels, OpKind.concat, OpKind.crop}


@dataclasses.dataclass
class Node:
    """One program node (program.hpp:73-103); unused fields keep their defaults."""

    kind: OpKind = OpKind.conv
    inputs: tuple[int, int] = (0, 0)
    input_count: int = 1
    output: int = 0
    in_channels: int = 0
    out_channels: int = 0
    depthwise: bool = False
    kernel: tuple[int, int] = (1, 1)
    stride: tuple[int, int] = (1, 1)
    pads: tuple[int, int, int, int] = (0, 0, 0, 0)  # top, left, bottom, right
    weight_offset: int = 0
    bias_offset: int = 0
    scalar: float = 0.0
    begin: int = 0
    end: int = 0
    block: int = 1
    axis: int = 2
    minimum: float = 0.0
    maximum: float = 0.0
    weight_bits: int = 16
    activation_bits: int = 16

    def is_integer_pointwise(self) -> bool:
        """is_integer_pointwise (program.cpp:502-507)."""
        return (self.kind == OpKind.conv and not self.depthwise and tuple(self.kernel) == (1, 1)
                and tuple(self.stride) == (1, 1) and tuple(self.pads) == (0, 0, 0, 0))


@dataclasses.dataclass
class Program:
    """An intconv.v1 program: tensors by id, nodes in execution order, FP32 weights."""

    name: str = "program"
    numerics: str = INTCONV_PROFILE
    tensor_names: list[str] = dataclasses.field(default_factory=list)
    tensor_channels: list[int] = dataclasses.field(default_factory=list)
    inputs: list[int] = dataclasses.field(default_factory=list)
    outputs: list[int] = dataclasses.field(default_factory=list)
    nodes: list[Node] = dataclasses.field(default_factory=list)
    weights: np.ndarray = dataclasses.field(default_factory=lambda: np.zeros(0, np.float32))

    # ---- construction helpers (the reference tests build programs this way) ----
    def define(self, name: str, channels: int) -> int:
        self.tensor_names.append(name)
        self.tensor_channels.append(int(channels))
        return len(self.tensor_names) - 1

    def add_input(self, name: str, channels: int) -> int:
        tid = self.define(name, channels)
        self.inputs.append(tid)
        return tid

    def add_weights(self, values: np.ndarray) -> int:
        offset = int(self.weights.size)
        self.weights = np.concatenate([self.weights, np.asarray(values, np.float32).reshape(-1)])
        return offset

    def conv(self, source: int, out_channels: int, weights: np.ndarray, bias: np.ndarray, name: str,
             *, depthwise: bool = False, kernel=(1, 1), stride=(1, 1), pads=(0, 0, 0, 0),
             bits: tuple[int, int] | None = None) -> int:
        in_channels = self.tensor_channels[source]
        node = Node(kind=OpKind.conv, inputs=(source, 0), in_channels=in_channels,
                    out_channels=out_channels, depthwise=depthwise, kernel=tuple(kernel),
                    stride=tuple(stride), pads=tuple(pads))
        per_output = (1 if depthwise else in_channels) * kernel[0] * kernel[1]
        weights = np.asarray(weights, np.float32).reshape(-1)
        if weights.size != out_channels * per_output or np.asarray(bias).size != out_channels:
            raise ValueError("conv weight or bias count does not match its geometry")
        node.weight_offset = self.add_weights(weights)
        node.bias_offset = self.add_weights(bias)
        if bits is not None:
            node.weight_bits, node.activation_bits = bits
        node.output = self.define(name, out_channels)
        self.nodes.append(node)
        return node.output

    def unary(self, kind: OpKind, source: int, name: str, **fields) -> int:
        node = Node(kind=kind, inputs=(source, 0), **fields)
        node.output = self.define(name, self._channels_of(node, source, None))
        self.nodes.append(node)
        return node.output

    def binary(self, kind: OpKind, first: int, second: int, name: str, **fields) -> int:
        node = Node(kind=kind, inputs=(first, second), input_count=2, **fields)
        node.output = self.define(name, self._channels_of(node, first, second))
        self.nodes.append(node)
        return node.output

    def _channels_of(self, node: Node, first: int, second: int | None) -> int:
        c = self.tensor_channels[first]
        if node.kind == OpKind.slice_channels:
            return node.end - node.begin
        if node.kind == OpKind.depth_to_space:
            return c // (node.block * node.block)
        if node.kind == OpKind.space_to_depth:
            return c * node.block * node.block
        if node.kind == OpKind.im2col:
            return c * node.kernel[0] * node.kernel[1]
        if node.kind == OpKind.concat:
            return c + self.tensor_channels[second]
        return c

    def dense_conv(self, source: int, out_channels: int, weights: np.ndarray, bias: np.ndarray,
                   name: str, *, kernel=(3, 3), stride=(1, 1), pads=(1, 1, 1, 1),
                   bits: tuple[int, int] | None = None) -> int:
        """A dense spatial conv as the exporter lowers it: im2col + pointwise
        (export_deterministic_program.py:326-336)."""
        if tuple(kernel) == (1, 1) and tuple(stride) == (1, 1) and tuple(pads) == (0, 0, 0, 0):
            return self.conv(source, out_channels, weights, bias, name, bits=bits)
        columns = self.unary(OpKind.im2col, source, f"{name}::im2col", kernel=tuple(kernel),
                             stride=tuple(stride), pads=tuple(pads))
        return self.conv(columns, out_channels, weights, bias, name, bits=bits)

    def finish(self, outputs: Iterable[int]) -> "Program":
        self.outputs = list(outputs)
        return self

    def last_use(self) -> list[int]:
        """Index of the last node reading each tensor; outputs read at len(nodes)."""
        use = [0] * len(self.tensor_names)
        for index, node in enumerate(self.nodes):
            for slot in range(node.input_count):
                use[node.inputs[slot]] = index
        for tid in self.outputs:
            use[tid] = len(self.nodes)
        return use

    def with_widths(self, weight_bits: int, activation_bits: int) -> "Program":
        """Copy with every integer pointwise conv set to the given widths."""
        clone = dataclasses.replace(self, nodes=[dataclasses.replace(n) for n in self.nodes],
                                    weights=self.weights.copy())
        for node in clone.nodes:
            if node.is_integer_pointwise():
                node.weight_bits, node.activation_bits = weight_bits, activation_bits
        return clone

    # ---- on-disk form ----
    def to_json(self, weights_file: str, weights_sha256: str) -> dict:
        nodes = []
        for node in self.nodes:
            entry: dict = {"op": node.kind.name}
            if node.kind in BINARY_OPS:
                entry["inputs"] = [self.tensor_names[node.inputs[0]], self.tensor_names[node.inputs[1]]]
            else:
                entry["input"] = self.tensor_names[node.inputs[0]]
            entry["output"] = self.tensor_names[node.output]
            if node.kind == OpKind.conv:
                entry.update(in_channels=node.in_channels, out_channels=node.out_channels,
                             depthwise=bool(node.depthwise), kernel=list(node.kernel),
                             stride=list(node.stride), pads=list(node.pads),
                             weight_offset=node.weight_offset, bias_offset=node.bias_offset)
                if node.is_integer_pointwise():
                    entry["integer"] = {"weight_bits": node.weight_bits,
                                        "activation_bits": node.activation_bits}
            elif node.kind == OpKind.mul_scalar:
                entry["value"] = float(np.float32(node.scalar))
            elif node.kind == OpKind.slice_channels:
                entry.update(begin=node.begin, end=node.end)
            elif node.kind in (OpKind.depth_to_space, OpKind.space_to_depth):
                entry["block"] = node.block
            elif node.kind == OpKind.clamp:
                entry.update(min=float(np.float32(node.minimum)), max=float(np.float32(node.maximum)))
            elif node.kind == OpKind.im2col:
                entry.update(kernel=list(node.kernel), stride=list(node.stride), pads=list(node.pads))
            elif node.kind == OpKind.crop:
                entry["axis"] = node.axis
            nodes.append(entry)
        return {
            "format": FORMAT,
            "version": VERSION,
            "numerics": self.numerics,
            "name": self.name,
            "weights": {"file": weights_file, "dtype": "float16", "count": int(self.weights.size),
                        "sha256": weights_sha256},
            "inputs": [{"name": self.tensor_names[t], "channels": self.tensor_channels[t]}
                       for t in self.inputs],
            "outputs": [{"name": self.tensor_names[t], "channels": self.tensor_channels[t]}
                        for t in self.outputs],
            "nodes": nodes,
        }

    def write(self, directory: str | Path, name: str | None = None) -> Path:
        """Writes <name>.detprog.json and <name>.detw; returns the JSON path.
        Weights are stored as FP16 (round to nearest even), as the exporter does."""
        directory = Path(directory)
        directory.mkdir(parents=True, exist_ok=True)
        name = name or self.name
        blob = self.weights.astype("<f2").tobytes()
        weights_path = directory / f"{name}.detw"
        weights_path.write_bytes(blob)
        document = self.to_json(weights_path.name, hashlib.sha256(blob).hexdigest())
        path = directory / f"{name}.detprog.json"
        path.write_text(json.dumps(document, indent=1) + "\n", encoding="utf-8")
        return path

    def fp16_weights(self) -> np.ndarray:
        """The weights exactly as a loaded program holds them (FP16 widened)."""
        return self.weights.astype(np.float16).astype(np.float32)


def sha256_hex(path: str | Path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


# ---- platform-stable seeded inputs ----

class SeededStream:
    """std::mt19937 with the reference tests' float construction
    (tests/deterministic_executor_tests.cpp:40-44): unit = (raw >> 8) / 2^24,
    value = low + (high - low) * unit in binary32. numpy's legacy RandomState
    seeds MT19937 exactly as std::mt19937(seed) does."""

    def __init__(self, seed: int) -> None:
        self._state = np.random.RandomState(seed)

    def raw(self, count: int) -> np.ndarray:
        """The next `count` raw 32-bit engine outputs."""
        if count == 0:
            return np.zeros(0, np.uint32)
        return np.asarray(self._state._bit_generator.random_raw(count), dtype=np.uint64).astype(np.uint32)

    def uniform(self, low: float, high: float, count: int) -> np.ndarray:
        unit = (self.raw(count) >> np.uint32(8)).astype(np.float32) / np.float32(1 << 24)
        return np.float32(low) + np.float32(np.float32(high) - np.float32(low)) * unit

    def tensor(self, channels: int, height: int, width: int, scale: float) -> np.ndarray:
        return self.uniform(-scale, scale, channels * height * width).reshape(channels, height, width)

    def integers(self, low: int, high: int, count: int) -> np.ndarray:
        """Uniform integers in [low, high] (raw % span; the bias is < 2^-20)."""
        span = np.uint64(high - low + 1)
        return (self.raw(count).astype(np.uint64) % span).astype(np.int64) + low
