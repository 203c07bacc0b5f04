"""nvcr.fx.v1 stage programs through the C ABI: the host-side mirror of the
reference's ``fx::load_program`` and ``fx::program_digest``
(src/deterministic/fx_program.hpp:70-75). Loading applies the profile's
load-time refusals and raises ``ExecutorError`` with the reference's error code
(missing_artifact, io_error, digest_mismatch, invalid_argument).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

from .executor import ErrorCode, ExecutorError, _check, library


@dataclass(frozen=True)
class FxNodeInfo:
    op: str
    input_count: int
    output: int


class FxProgram:
    """A loaded nvcr.fx-program.v1 program (owns the C handle)."""

    def __init__(self, handle: ctypes.c_void_p) -> None:
        self._handle = handle
        lib = library()
        counts = [ctypes.c_size_t(0) for _ in range(4)]
        digest = ctypes.create_string_buffer(65)
        _check(lib.nvcr_sm100_fx_program_summary(handle, *[ctypes.byref(c) for c in counts], digest))
        self.tensor_count, self.node_count, self.input_count, self.output_count = (c.value for c in counts)
        self.digest = digest.value.decode()
        nodes = []
        for index in range(self.node_count):
            op = ctypes.c_char_p()
            inputs = ctypes.c_size_t(0)
            output = ctypes.c_uint32(0)
            _check(lib.nvcr_sm100_fx_program_node(handle, index, ctypes.byref(op), ctypes.byref(inputs),
                                                  ctypes.byref(output)))
            nodes.append(FxNodeInfo(op.value.decode(), inputs.value, output.value))
        self.nodes = nodes
        self.inputs = self._tensors(0, self.input_count)
        self.outputs = self._tensors(1, self.output_count)

    def _tensors(self, is_output: int, count: int) -> list[tuple[str, int]]:
        """(name, channels) of the program's inputs or outputs, in run order."""
        tensors = []
        for index in range(count):
            name = ctypes.c_char_p()
            channels = ctypes.c_int32(0)
            _check(library().nvcr_sm100_fx_program_tensor(self._handle, is_output, index, ctypes.byref(name),
                                                          ctypes.byref(channels)))
            tensors.append((name.value.decode(), channels.value))
        return tensors

    def close(self) -> None:
        if self._handle:
            library().nvcr_sm100_fx_program_destroy(self._handle)
            self._handle = None

    def __enter__(self) -> "FxProgram":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        self.close()


def load_program(directory: str | Path, stage: str) -> FxProgram:
    """Loads <directory>/<stage>.fxprog.json and its data file."""
    handle = ctypes.c_void_p()
    _check(library().nvcr_sm100_fx_program_load(str(directory).encode(), stage.encode(), ctypes.byref(handle)))
    return FxProgram(handle)


def program_digest(directory: str | Path, stage: str) -> str:
    """Lowercase hex SHA-256 of <directory>/<stage>.fxprog.json."""
    digest = ctypes.create_string_buffer(65)
    _check(library().nvcr_sm100_fx_program_digest(str(directory).encode(), stage.encode(), digest))
    return digest.value.decode()


class FxExecutor:
    """Runs one loaded program on the current CUDA device (the reference's
    ``fx::run``, src/deterministic/fx_program.cpp:468-525): the same int32
    outputs; a stage failure raises ExecutorError(malformed_bitstream), shapes
    the program cannot take raise ExecutorError(invalid_argument). Creating it
    and inferring extents need no GPU; parameters upload at the first run."""

    def __init__(self, program: FxProgram, stream=None) -> None:
        handle = ctypes.c_void_p()
        stream_handle = ctypes.c_void_p(stream.cuda_stream if stream is not None else 0)
        _check(library().nvcr_sm100_fx_executor_create(program._handle, stream_handle, ctypes.byref(handle)))
        self._handle = handle
        self.output_count = program.output_count

    def close(self) -> None:
        if self._handle:
            library().nvcr_sm100_fx_executor_destroy(self._handle)
            self._handle = None

    def __enter__(self) -> "FxExecutor":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        self.close()

    def infer_output_extents(self, extents) -> list[tuple[int, int, int]]:
        flat = (ctypes.c_int32 * max(1, 3 * len(extents)))(*[int(v) for e in extents for v in e])
        out = (ctypes.c_int32 * max(1, 3 * self.output_count))()
        _check(library().nvcr_sm100_fx_infer_output_extents(self._handle, flat, len(extents), out, self.output_count))
        return [tuple(out[3 * i:3 * i + 3]) for i in range(self.output_count)]

    def _run(self, input_pointers, extents, output_pointers, device: bool) -> None:
        flat = (ctypes.c_int32 * max(1, 3 * len(extents)))(*[int(v) for e in extents for v in e])
        ins = (ctypes.c_void_p * max(1, len(input_pointers)))(*input_pointers)
        outs = (ctypes.c_void_p * max(1, len(output_pointers)))(*output_pointers)
        _check(library().nvcr_sm100_fx_run(self._handle, ins, flat, len(input_pointers), outs, len(output_pointers),
                                           1 if device else 0))

    def _shapes_or_run(self, extents, input_pointers, device: bool):
        """Output extents; when the shapes alone are refused, runs anyway so that
        a stage failure the reference meets before that refusal is the error
        raised (the run stops where the reference's does)."""
        try:
            return self.infer_output_extents(extents)
        except ExecutorError as error:
            if error.code != ErrorCode.invalid_argument:
                raise
            self._run(input_pointers, extents, [], device)
            raise

    def run(self, inputs):
        """Host path: [C][H][W] int32 numpy inputs in, numpy outputs out (the
        copies to and from the device are inside the call)."""
        import numpy as np

        keep = [np.ascontiguousarray(x, np.int32) for x in inputs]
        extents = [x.shape for x in keep]
        shapes = self._shapes_or_run(extents, [x.ctypes.data for x in keep], device=False)
        outputs = [np.empty(shape, np.int32) for shape in shapes]
        self._run([x.ctypes.data for x in keep], extents, [y.ctypes.data for y in outputs], device=False)
        return outputs

    def run_device(self, inputs):
        """Device path: int32 CUDA tensors of shape [C][H][W] in, CUDA tensors out."""
        import torch

        keep = [x.contiguous() for x in inputs]
        if any(x.dtype != torch.int32 or not x.is_cuda for x in keep):
            raise ValueError("inputs are int32 CUDA tensors")
        extents = [tuple(x.shape) for x in keep]
        shapes = self._shapes_or_run(extents, [x.data_ptr() for x in keep], device=True)
        outputs = [torch.empty(shape, dtype=torch.int32, device=keep[0].device if keep else "cuda")
                   for shape in shapes]
        self._run([x.data_ptr() for x in keep], extents, [y.data_ptr() for y in outputs], device=True)
        return outputs

    @property
    def last_launch_count(self) -> int:
        return library().nvcr_sm100_fx_last_launch_count(self._handle)


def run(program: FxProgram, inputs):
    """``fx::run(program, inputs)`` on the GPU with host numpy tensors."""
    with FxExecutor(program) as executor:
        return executor.run(inputs)
