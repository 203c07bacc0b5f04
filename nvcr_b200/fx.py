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

from .executor import _check, library


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
