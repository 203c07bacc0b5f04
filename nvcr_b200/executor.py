"""Python host mirror of the reference's CudaExecutor over the C ABI.

Reference interface: src/deterministic/cuda_executor.hpp:26-53
(``CudaExecutor::create``, ``run_half``, ``run``) and
src/deterministic/normative_stage.hpp:28-65 (``is_normative``,
``load_normative_program``, ``infer_output_extents``). Every call goes through
``include/nvcr_sm100.h`` into ``nvcr_b200/_build/libnvcr_sm100.so``; there is
no CPU fallback: without the library (or a B200) the calls raise.
"""
from __future__ import annotations

import ctypes
import enum
import json
from pathlib import Path
from typing import Mapping, Sequence

import numpy as np

from .program import Program

LIBRARY = Path(__file__).resolve().parent / "_build" / "libnvcr_sm100.so"


class ErrorCode(enum.IntEnum):
    """The reference's nvcr::ErrorCode (include/nvcr/common/error.hpp:11-34)."""

    invalid_argument = 0
    invalid_state = 1
    io_error = 2
    malformed_bitstream = 3
    resource_exhausted = 4
    dependency_unavailable = 5
    backend_error = 6
    not_implemented = 7
    internal_error = 8
    try_again = 9
    end_of_stream = 10
    missing_artifact = 11
    missing_codec = 12
    missing_provider = 13
    missing_model_set = 14
    incompatible_target = 15
    incompatible_precision = 16
    incompatible_version = 17
    digest_mismatch = 18
    license_restricted = 19


class ExecutorError(RuntimeError):
    def __init__(self, code: ErrorCode, message: str) -> None:
        super().__init__(f"{code.name}: {message}")
        self.code = code
        self.message = message


class Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("channels", ctypes.c_int32), ("height", ctypes.c_int32),
                ("width", ctypes.c_int32), ("data", ctypes.c_void_p)]


class StepTime(ctypes.Structure):
    _fields_ = [("label", ctypes.c_char * 96), ("kernel", ctypes.c_char * 32), ("milliseconds", ctypes.c_double),
                ("algorithmic_ops", ctypes.c_double), ("algorithmic_bytes", ctypes.c_double)]


EXPORTS = [
    "nvcr_sm100_abi_version", "nvcr_sm100_last_error", "nvcr_sm100_supports_profile", "nvcr_sm100_is_normative",
    "nvcr_sm100_executor_create", "nvcr_sm100_executor_create_from_memory", "nvcr_sm100_load_normative",
    "nvcr_sm100_executor_destroy", "nvcr_sm100_tensor_count", "nvcr_sm100_tensor_info",
    "nvcr_sm100_infer_output_extents", "nvcr_sm100_run_half", "nvcr_sm100_run_float", "nvcr_sm100_run_host",
    "nvcr_sm100_synchronize", "nvcr_sm100_stream", "nvcr_sm100_last_launch_count", "nvcr_sm100_workspace_bytes",
    "nvcr_sm100_set_profiling", "nvcr_sm100_profile", "nvcr_sm100_program_load", "nvcr_sm100_program_load_memory",
    "nvcr_sm100_program_destroy", "nvcr_sm100_program_tensor_count", "nvcr_sm100_program_tensor_info",
    "nvcr_sm100_program_infer_output_extents", "nvcr_sm100_executor_create_from_program",
    "nvcr_sm100_run_half_static", "nvcr_sm100_test_wait_timeout", "nvcr_sm100_test_reciprocal",
    "nvcr_sm100_numerics_identity", "nvcr_sm100_numerics_identity_parse", "nvcr_sm100_fx_program_load",
    "nvcr_sm100_fx_program_destroy", "nvcr_sm100_fx_program_digest", "nvcr_sm100_fx_program_summary",
    "nvcr_sm100_fx_program_node", "nvcr_sm100_fx_program_tensor", "nvcr_sm100_fx_executor_create", "nvcr_sm100_fx_executor_destroy",
    "nvcr_sm100_fx_infer_output_extents", "nvcr_sm100_fx_run", "nvcr_sm100_fx_last_launch_count",
    "nvcr_sm100_dcvc_build_decode_indexes", "nvcr_sm100_dcvc_build_encode_indexes", "nvcr_sm100_dcvc_make_mask",
    "nvcr_sm100_dcvc_restore", "nvcr_sm100_dcvc_process_with_mask", "nvcr_sm100_dcvc_reduce",
    "nvcr_sm100_dcvc_round_to_int8", "nvcr_sm100_dcvc_int8_to_half", "nvcr_sm100_dcvc_clamp_min",
    "nvcr_sm100_dcvc_clamp_reciprocal_with_quant", "nvcr_sm100_dcvc_add_in_place", "nvcr_sm100_dcvc_multiply_broadcast",
    "nvcr_sm100_dcvc_add_and_multiply", "nvcr_sm100_dcvc_replicate_pad", "nvcr_sm100_dcvc_crop_spatial",
    "nvcr_sm100_dcvc_rgb24_to_ycbcr_padded", "nvcr_sm100_dcvc_yuv420p8_to_ycbcr_padded",
    "nvcr_sm100_dcvc_ycbcr_padded_to_yuv420p8",
]

_lib: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """Loads the in-tree C-ABI library (raises if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise FileNotFoundError(f"{LIBRARY} is not built; run nvcr_b200.build.build()")
    lib = ctypes.CDLL(str(LIBRARY))
    vp, sz, i32p = ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32)
    tp = ctypes.POINTER(Tensor)
    handle_out = ctypes.POINTER(ctypes.c_void_p)
    signatures = {
        "nvcr_sm100_abi_version": (ctypes.c_int, []),
        "nvcr_sm100_last_error": (sz, [ctypes.c_char_p, sz]),
        "nvcr_sm100_supports_profile": (ctypes.c_int, [ctypes.c_char_p]),
        "nvcr_sm100_is_normative": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]),
        "nvcr_sm100_executor_create": (ctypes.c_int, [ctypes.c_char_p, vp, handle_out]),
        "nvcr_sm100_executor_create_from_memory": (ctypes.c_int, [ctypes.c_char_p, sz,
                                                                  ctypes.POINTER(ctypes.c_float), sz, vp,
                                                                  handle_out]),
        "nvcr_sm100_load_normative": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, vp,
                                                     handle_out]),
        "nvcr_sm100_executor_destroy": (None, [vp]),
        "nvcr_sm100_tensor_count": (ctypes.c_int, [vp, ctypes.c_int, ctypes.POINTER(sz)]),
        "nvcr_sm100_tensor_info": (ctypes.c_int, [vp, ctypes.c_int, sz, ctypes.POINTER(ctypes.c_char_p), i32p]),
        "nvcr_sm100_infer_output_extents": (ctypes.c_int, [vp, tp, sz, tp, sz]),
        "nvcr_sm100_run_half": (ctypes.c_int, [vp, tp, sz, tp, sz]),
        "nvcr_sm100_run_float": (ctypes.c_int, [vp, tp, sz, tp, sz]),
        "nvcr_sm100_run_host": (ctypes.c_int, [vp, tp, sz, tp, sz]),
        "nvcr_sm100_synchronize": (ctypes.c_int, [vp]),
        "nvcr_sm100_test_wait_timeout": (ctypes.c_int, [vp, ctypes.c_uint]),
        "nvcr_sm100_test_reciprocal": (ctypes.c_int, [ctypes.c_uint, ctypes.c_uint, ctypes.POINTER(ctypes.c_ulonglong)]),
        "nvcr_sm100_numerics_identity": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), ctypes.c_char_p,
                                                         ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t,
                                                         ctypes.POINTER(ctypes.c_size_t)]),
        "nvcr_sm100_numerics_identity_parse": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                                               ctypes.c_size_t, ctypes.c_char_p]),
        "nvcr_sm100_stream": (vp, [vp]),
        "nvcr_sm100_last_launch_count": (ctypes.c_int, [vp]),
        "nvcr_sm100_workspace_bytes": (sz, [vp]),
        "nvcr_sm100_set_profiling": (ctypes.c_int, [vp, ctypes.c_int]),
        "nvcr_sm100_profile": (ctypes.c_int, [vp, ctypes.POINTER(StepTime), sz, ctypes.POINTER(sz)]),
        "nvcr_sm100_program_load": (ctypes.c_int, [ctypes.c_char_p, handle_out]),
        "nvcr_sm100_program_load_memory": (ctypes.c_int, [ctypes.c_char_p, sz, ctypes.POINTER(ctypes.c_float), sz,
                                                          handle_out]),
        "nvcr_sm100_program_destroy": (None, [vp]),
        "nvcr_sm100_program_tensor_count": (ctypes.c_int, [vp, ctypes.c_int, ctypes.POINTER(sz)]),
        "nvcr_sm100_program_tensor_info": (ctypes.c_int, [vp, ctypes.c_int, sz, ctypes.POINTER(ctypes.c_char_p),
                                                          i32p]),
        "nvcr_sm100_program_infer_output_extents": (ctypes.c_int, [vp, tp, sz, tp, sz]),
        "nvcr_sm100_executor_create_from_program": (ctypes.c_int, [vp, vp, handle_out]),
        "nvcr_sm100_run_half_static": (ctypes.c_int, [vp, tp, sz, tp, sz]),
        "nvcr_sm100_fx_program_load": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, handle_out]),
        "nvcr_sm100_fx_program_destroy": (None, [vp]),
        "nvcr_sm100_fx_program_digest": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]),
        "nvcr_sm100_fx_program_summary": (ctypes.c_int, [vp, ctypes.POINTER(sz), ctypes.POINTER(sz), ctypes.POINTER(sz),
                                                         ctypes.POINTER(sz), ctypes.c_char_p]),
        "nvcr_sm100_fx_program_node": (ctypes.c_int, [vp, sz, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(sz),
                                                      ctypes.POINTER(ctypes.c_uint32)]),
        "nvcr_sm100_fx_program_tensor": (ctypes.c_int, [vp, ctypes.c_int, sz, ctypes.POINTER(ctypes.c_char_p), i32p]),
        "nvcr_sm100_fx_executor_create": (ctypes.c_int, [vp, vp, handle_out]),
        "nvcr_sm100_fx_executor_destroy": (None, [vp]),
        "nvcr_sm100_fx_infer_output_extents": (ctypes.c_int, [vp, i32p, sz, i32p, sz]),
        "nvcr_sm100_fx_run": (ctypes.c_int, [vp, ctypes.POINTER(vp), i32p, sz, ctypes.POINTER(vp), sz, ctypes.c_int]),
        "nvcr_sm100_fx_last_launch_count": (ctypes.c_int, [vp]),
        "nvcr_sm100_dcvc_build_decode_indexes": (ctypes.c_int, [vp, vp, sz, ctypes.c_float, vp]),
        "nvcr_sm100_dcvc_build_encode_indexes": (ctypes.c_int, [vp, vp, vp, sz, ctypes.c_float, vp]),
        "nvcr_sm100_dcvc_make_mask": (ctypes.c_int, [vp] + [ctypes.c_int32] * 4 + [ctypes.c_int, ctypes.c_int, vp]),
        "nvcr_sm100_dcvc_restore": (ctypes.c_int, [vp] * 4 + [ctypes.c_int32] * 4 + [ctypes.c_int, vp]),
        "nvcr_sm100_dcvc_process_with_mask": (ctypes.c_int, [vp] * 8 + [sz, ctypes.c_float, vp]),
        "nvcr_sm100_dcvc_reduce": (ctypes.c_int, [vp] * 3 + [ctypes.c_int32] * 4 + [ctypes.c_int, vp]),
        "nvcr_sm100_dcvc_round_to_int8": (ctypes.c_int, [vp, vp, sz, vp]),
        "nvcr_sm100_dcvc_int8_to_half": (ctypes.c_int, [vp, vp, sz, vp]),
        "nvcr_sm100_dcvc_clamp_min": (ctypes.c_int, [vp, sz, ctypes.c_float, vp]),
        "nvcr_sm100_dcvc_clamp_reciprocal_with_quant": (ctypes.c_int, [vp, vp, sz, vp]),
        "nvcr_sm100_dcvc_add_in_place": (ctypes.c_int, [vp, vp, sz, vp]),
        "nvcr_sm100_dcvc_multiply_broadcast": (ctypes.c_int, [vp, vp, sz, ctypes.c_int32, vp]),
        "nvcr_sm100_dcvc_add_and_multiply": (ctypes.c_int, [vp, vp, vp, sz, vp]),
        "nvcr_sm100_dcvc_replicate_pad": (ctypes.c_int, [vp, vp] + [ctypes.c_int32] * 6 + [vp]),
        "nvcr_sm100_dcvc_crop_spatial": (ctypes.c_int, [vp, vp] + [ctypes.c_int32] * 6 + [vp]),
        "nvcr_sm100_dcvc_rgb24_to_ycbcr_padded": (ctypes.c_int, [vp, ctypes.c_int32, ctypes.c_int32, vp,
                                                                 ctypes.c_int32, ctypes.c_int32, vp]),
        "nvcr_sm100_dcvc_yuv420p8_to_ycbcr_padded": (ctypes.c_int, [vp, ctypes.c_int32, ctypes.c_int32, vp,
                                                                    ctypes.c_int32, ctypes.c_int32, vp]),
        "nvcr_sm100_dcvc_ycbcr_padded_to_yuv420p8": (ctypes.c_int, [vp] + [ctypes.c_int32] * 6 + [vp, vp]),
    }
    for name, (restype, argtypes) in signatures.items():
        function = getattr(lib, name)
        function.restype = restype
        function.argtypes = argtypes
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status == 0:
        return
    lib = library()
    buffer = ctypes.create_string_buffer(1024)
    lib.nvcr_sm100_last_error(buffer, 1024)
    raise ExecutorError(ErrorCode(status - 1), buffer.value.decode(errors="replace"))


def supports_numerics_profile(profile: str) -> bool:
    return bool(library().nvcr_sm100_supports_profile(profile.encode()))


def is_normative(profile: str) -> bool:
    """Reference is_normative: False for '', True for nvcr.intconv.v1, else raises incompatible_precision."""
    flag = ctypes.c_int(0)
    _check(library().nvcr_sm100_is_normative(profile.encode(), ctypes.byref(flag)))
    return bool(flag.value)


def _stream_handle(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream"))


class LoadedProgram:
    """A program loaded and validated by the library, without a device
    (reference load_program + infer_output_extents)."""

    def __init__(self, handle: int) -> None:
        self._handle = ctypes.c_void_p(handle)
        lib = library()
        self.input_names, self.output_names = [], []
        for is_output, names in ((0, self.input_names), (1, self.output_names)):
            count = ctypes.c_size_t(0)
            _check(lib.nvcr_sm100_program_tensor_count(self._handle, is_output, ctypes.byref(count)))
            for index in range(count.value):
                name = ctypes.c_char_p()
                channels = ctypes.c_int32()
                _check(lib.nvcr_sm100_program_tensor_info(self._handle, is_output, index, ctypes.byref(name),
                                                          ctypes.byref(channels)))
                names.append(name.value.decode())

    @classmethod
    def load(cls, program_json: str | Path) -> "LoadedProgram":
        handle = ctypes.c_void_p()
        _check(library().nvcr_sm100_program_load(str(program_json).encode(), ctypes.byref(handle)))
        return cls(handle.value)

    @classmethod
    def from_program(cls, program: Program, fp16_weights: bool = True) -> "LoadedProgram":
        weights = np.ascontiguousarray(program.fp16_weights() if fp16_weights else program.weights, np.float32)
        text = json.dumps(program.to_json(f"{program.name}.detw", "0" * 64)).encode()
        handle = ctypes.c_void_p()
        _check(library().nvcr_sm100_program_load_memory(text, len(text),
                                                        weights.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                                        weights.size, ctypes.byref(handle)))
        return cls(handle.value)

    def infer_output_extents(self, extents: Sequence[tuple[int, int, int]]) -> list[tuple[int, int, int]]:
        ins = (Tensor * max(1, len(extents)))()
        for i, (c, h, w) in enumerate(extents):
            ins[i] = Tensor(None, c, h, w, None)
        outs = (Tensor * max(1, len(self.output_names)))()
        _check(library().nvcr_sm100_program_infer_output_extents(self._handle, ins, len(extents), outs,
                                                                 len(self.output_names)))
        return [(outs[i].channels, outs[i].height, outs[i].width) for i in range(len(self.output_names))]

    def executor(self, stream=None) -> "CudaExecutor":
        handle = ctypes.c_void_p()
        _check(library().nvcr_sm100_executor_create_from_program(self._handle, _stream_handle(stream),
                                                                 ctypes.byref(handle)))
        return CudaExecutor(handle.value, None)

    def close(self) -> None:
        if self._handle:
            library().nvcr_sm100_program_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


class CudaExecutor:
    """One executor on one stream (reference CudaExecutor)."""

    def __init__(self, handle: int, program: Program | None) -> None:
        self._handle = ctypes.c_void_p(handle)
        self.program = program
        lib = library()
        self.input_names, self.output_names = [], []
        for is_output, names in ((0, self.input_names), (1, self.output_names)):
            count = ctypes.c_size_t(0)
            _check(lib.nvcr_sm100_tensor_count(self._handle, is_output, ctypes.byref(count)))
            for index in range(count.value):
                name = ctypes.c_char_p()
                channels = ctypes.c_int32()
                _check(lib.nvcr_sm100_tensor_info(self._handle, is_output, index, ctypes.byref(name),
                                                  ctypes.byref(channels)))
                names.append(name.value.decode())

    # ---- construction ----
    @classmethod
    def create(cls, program_json: str | Path, stream=None, program: Program | None = None) -> "CudaExecutor":
        """From a .detprog.json file (weights from its .detw, digest-checked)."""
        handle = ctypes.c_void_p()
        _check(library().nvcr_sm100_executor_create(str(program_json).encode(), _stream_handle(stream),
                                                    ctypes.byref(handle)))
        return cls(handle.value, program)

    @classmethod
    def from_program(cls, program: Program, stream=None, fp16_weights: bool = True) -> "CudaExecutor":
        """From an in-memory Program. fp16_weights=True gives the weights a loaded
        program would hold (FP16 widened); False keeps the FP32 values."""
        weights = np.ascontiguousarray(program.fp16_weights() if fp16_weights else program.weights, np.float32)
        text = json.dumps(program.to_json(f"{program.name}.detw", "0" * 64)).encode()
        handle = ctypes.c_void_p()
        _check(library().nvcr_sm100_executor_create_from_memory(
            text, len(text), weights.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), weights.size,
            _stream_handle(stream), ctypes.byref(handle)))
        return cls(handle.value, program)

    @classmethod
    def load_normative(cls, directory: str | Path, component: str, expected_sha256: str,
                       stream=None) -> "CudaExecutor":
        handle = ctypes.c_void_p()
        _check(library().nvcr_sm100_load_normative(str(directory).encode(), component.encode(),
                                                   expected_sha256.encode(), _stream_handle(stream),
                                                   ctypes.byref(handle)))
        return cls(handle.value, None)

    def close(self) -> None:
        if self._handle:
            library().nvcr_sm100_executor_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __enter__(self) -> "CudaExecutor":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    # ---- queries ----
    @property
    def stream(self) -> int:
        return library().nvcr_sm100_stream(self._handle) or 0

    @property
    def launches(self) -> int:
        return library().nvcr_sm100_last_launch_count(self._handle)

    @property
    def workspace_bytes(self) -> int:
        return library().nvcr_sm100_workspace_bytes(self._handle)

    def infer_output_extents(self, extents: Sequence[tuple[int, int, int]]) -> list[tuple[int, int, int]]:
        ins = (Tensor * max(1, len(extents)))()
        for i, (c, h, w) in enumerate(extents):
            ins[i] = Tensor(None, c, h, w, None)
        outs = (Tensor * max(1, len(self.output_names)))()
        _check(library().nvcr_sm100_infer_output_extents(self._handle, ins, len(extents), outs,
                                                         len(self.output_names)))
        return [(outs[i].channels, outs[i].height, outs[i].width) for i in range(len(self.output_names))]

    # ---- execution ----
    @staticmethod
    def _tensors(named: Mapping[str, object]) -> tuple[ctypes.Array, list]:
        keep = []
        array = (Tensor * max(1, len(named)))()
        for i, (name, value) in enumerate(named.items()):
            encoded = name.encode()
            keep.append(encoded)
            if isinstance(value, np.ndarray):
                c, h, w = value.shape
                pointer = value.ctypes.data
            else:  # a torch tensor
                c, h, w = value.shape[-3:]
                pointer = value.data_ptr()
            array[i] = Tensor(encoded, c, h, w, pointer)
        return array, keep

    def run_half(self, inputs: Mapping[str, object], outputs: Mapping[str, object]) -> None:
        """Device FP16 NCHW tensors (torch, batch-1 [1,C,H,W] or [C,H,W]); enqueues only."""
        ins, k1 = self._tensors(inputs)
        outs, k2 = self._tensors(outputs)
        _check(library().nvcr_sm100_run_half(self._handle, ins, len(inputs), outs, len(outputs)))

    def run_half_static(self, inputs: Mapping[str, object], outputs: Mapping[str, object]) -> None:
        """run_half with all scratch in the library's fixed static device array
        (nvcr_sm100_run_half_static): for hosts that cannot allocate device
        memory while running. Calls overlapping on the GPU race on that array."""
        ins, k1 = self._tensors(inputs)
        outs, k2 = self._tensors(outputs)
        _check(library().nvcr_sm100_run_half_static(self._handle, ins, len(inputs), outs, len(outputs)))

    def run_float(self, inputs: Mapping[str, object], outputs: Mapping[str, object]) -> None:
        ins, k1 = self._tensors(inputs)
        outs, k2 = self._tensors(outputs)
        _check(library().nvcr_sm100_run_float(self._handle, ins, len(inputs), outs, len(outputs)))

    def run(self, inputs: Sequence[np.ndarray]) -> list[np.ndarray]:
        """Host FP32 tensors in program input order -> outputs in program order (synchronous)."""
        arrays = [np.ascontiguousarray(x, np.float32) for x in inputs]
        extents = self.infer_output_extents([a.shape for a in arrays])
        outputs = [np.empty(e, np.float32) for e in extents]
        ins, k1 = self._tensors(dict(zip(self.input_names, arrays)))
        outs, k2 = self._tensors(dict(zip(self.output_names, outputs)))
        _check(library().nvcr_sm100_run_host(self._handle, ins, len(arrays), outs, len(outputs)))
        return outputs

    def synchronize(self) -> None:
        _check(library().nvcr_sm100_synchronize(self._handle))

    def test_wait_timeout(self, limit_ms: int) -> None:
        """Enqueues a device wait that gives up after `limit_ms` (failure-detection
        self-test); the next synchronize() raises backend_error."""
        _check(library().nvcr_sm100_test_wait_timeout(self._handle, limit_ms))

    def set_profiling(self, enabled: bool) -> None:
        _check(library().nvcr_sm100_set_profiling(self._handle, int(enabled)))

    def profile(self, capacity: int = 65536) -> list[dict]:
        """Kernel segments of every profiled run since the last call."""
        count = ctypes.c_size_t(0)
        steps = (StepTime * capacity)()
        _check(library().nvcr_sm100_profile(self._handle, steps, capacity, ctypes.byref(count)))
        return [{"label": steps[i].label.decode(), "kernel": steps[i].kernel.decode(),
                 "ms": steps[i].milliseconds, "ops": steps[i].algorithmic_ops,
                 "bytes": steps[i].algorithmic_bytes} for i in range(min(count.value, capacity))]


def reciprocal_mismatches(first_bits: int, count: int) -> int:
    """Floats d with bit patterns first_bits .. first_bits + count - 1 (within
    [1, 2^126)) for which the sigmoid's refined reciprocal differs from the IEEE
    division 1 / d (arithmetic self-test; runs on the current device)."""
    mismatches = ctypes.c_ulonglong(0)
    _check(library().nvcr_sm100_test_reciprocal(first_bits, count, ctypes.byref(mismatches)))
    return int(mismatches.value)


def numerics_identity(profile: str, stages: Sequence[tuple[str, bytes]]) -> bytes:
    """The numerics-identity payload naming `profile` and the normative stages
    (id, 32-byte program SHA-256) in the codec's order; raises ExecutorError
    (invalid_argument) for invalid ids, duplicates or a count outside 1..64."""
    ids = (ctypes.c_char_p * max(1, len(stages)))(*[sid.encode() for sid, _ in stages])
    digests = b"".join(bytes(d) for _, d in stages)
    if any(len(bytes(d)) != 32 for _, d in stages):
        raise ValueError("program digests are 32 bytes")
    payload = ctypes.create_string_buffer(1 + 128 + 32)
    size = ctypes.c_size_t(0)
    _check(library().nvcr_sm100_numerics_identity(profile.encode(), ids, digests, len(stages), payload,
                                                  len(payload), ctypes.byref(size)))
    return payload.raw[:size.value]


def parse_numerics_identity(payload: bytes) -> tuple[str, bytes]:
    """(profile, 32-byte program-set digest) of a numerics-identity payload;
    raises ExecutorError (malformed_bitstream) for a malformed one."""
    profile = ctypes.create_string_buffer(129)
    digest = ctypes.create_string_buffer(32)
    _check(library().nvcr_sm100_numerics_identity_parse(bytes(payload), len(payload), profile, len(profile), digest))
    return profile.value.decode(), digest.raw
