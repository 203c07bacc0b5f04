"""ctypes access to the CPU checkers and the reference's GPU comparator. TEST
AND BENCHMARK INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline, reference and
reference-GPU legs import this module, and only to check or time; the product
never does.

* ``Oracle``: this repo's C restatement (intconv_oracle.c), built into
  oracle/_build/liboracle.so. It is pinned against the reference below and
  against tests/golden/.
* ``Reference``: the reference's own CPU executor (run_cpu,
  src/deterministic/program.cpp:702-820) compiled from its sources into
  oracle/_ref/libnvcr_ref.so, reached through its own program loader.
* ``ReferenceGpu``: the reference's own CUDA executor (CudaExecutor,
  src/deterministic/cuda_executor.cu) built for sm_100a into
  oracle/_ref/libnvcr_ref_cuda.so, the GPU comparator.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path
from typing import Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REFERENCE_LIB = HERE / "_ref" / "libnvcr_ref.so"
# The reference checkout: $NVCR_REFERENCE when set, else a directory named
# `reference` beside this repository.
REFERENCE_SOURCES = Path(os.environ.get("NVCR_REFERENCE", HERE.parent.parent / "reference"))


def build(reference: bool = True) -> None:
    """Builds the C restatement, and the reference shim when its sources exist."""
    targets = ["oracle"]
    if reference and (REFERENCE_SOURCES / "src" / "deterministic" / "program.cpp").exists():
        targets += ["ref", "refgpu"]
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REFERENCE_SOURCES}", *targets], check=True)


class _Node(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "kind", "input0", "input1", "input_count", "output", "in_channels", "out_channels",
        "depthwise", "kernel_h", "kernel_w", "stride_y", "stride_x", "pad_top", "pad_left",
        "pad_bottom", "pad_right")] + [
        ("weight_offset", ctypes.c_int64), ("bias_offset", ctypes.c_int64),
        ("scalar", ctypes.c_float), ("begin", ctypes.c_int32), ("end", ctypes.c_int32),
        ("block", ctypes.c_int32), ("axis", ctypes.c_int32), ("minimum", ctypes.c_float),
        ("maximum", ctypes.c_float), ("weight_bits", ctypes.c_int32),
        ("activation_bits", ctypes.c_int32)]


class _Program(ctypes.Structure):
    _fields_ = [("tensor_count", ctypes.c_int32), ("tensor_channels", ctypes.POINTER(ctypes.c_int32)),
                ("input_count", ctypes.c_int32), ("inputs", ctypes.POINTER(ctypes.c_int32)),
                ("output_count", ctypes.c_int32), ("outputs", ctypes.POINTER(ctypes.c_int32)),
                ("node_count", ctypes.c_int32), ("nodes", ctypes.POINTER(_Node)),
                ("weights", ctypes.POINTER(ctypes.c_float)), ("weight_count", ctypes.c_int64)]


class _Tensor(ctypes.Structure):
    _fields_ = [("channels", ctypes.c_int32), ("height", ctypes.c_int32), ("width", ctypes.c_int32),
                ("values", ctypes.POINTER(ctypes.c_float))]


def _i32(values: Sequence[int]):
    array = (ctypes.c_int32 * max(1, len(values)))(*values)
    return array


class Oracle:
    """The C restatement of run_cpu and the profile's scalar arithmetic."""

    def __init__(self, path: Path = ORACLE_LIB) -> None:
        if not path.exists():
            build(reference=False)
        lib = ctypes.CDLL(str(path))
        self.lib = lib
        lib.or_exp.restype = ctypes.c_float
        lib.or_exp.argtypes = [ctypes.c_float]
        lib.or_sigmoid.restype = ctypes.c_float
        lib.or_sigmoid.argtypes = [ctypes.c_float]
        lib.or_ldexp.restype = ctypes.c_float
        lib.or_ldexp.argtypes = [ctypes.c_float, ctypes.c_int]
        lib.or_half_to_float.restype = ctypes.c_float
        lib.or_half_to_float.argtypes = [ctypes.c_uint16]
        lib.or_float_to_half.restype = ctypes.c_uint16
        lib.or_float_to_half.argtypes = [ctypes.c_float]
        lib.or_int_exponent.restype = ctypes.c_int
        lib.or_int_exponent.argtypes = [ctypes.c_float, ctypes.c_int]
        lib.or_int_quantize.restype = ctypes.c_int
        lib.or_int_quantize.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int]
        lib.or_int_output.restype = ctypes.c_float
        lib.or_int_output.argtypes = [ctypes.c_longlong, ctypes.c_float, ctypes.c_int, ctypes.c_float]
        lib.or_quantize_weights.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_int32,
                                            ctypes.POINTER(ctypes.c_int16), ctypes.POINTER(ctypes.c_float)]
        lib.or_run.restype = ctypes.c_int
        lib.or_run.argtypes = [ctypes.POINTER(_Program), ctypes.POINTER(_Tensor), ctypes.POINTER(_Tensor),
                               ctypes.c_char_p, ctypes.c_size_t]
        lib.or_free.argtypes = [ctypes.c_void_p]

    def quantize_weights(self, weights: np.ndarray, weight_bits: int):
        w = np.ascontiguousarray(weights, np.float32)
        rows, columns = w.shape
        values = np.zeros((rows, columns), np.int16)
        scales = np.zeros(rows, np.float32)
        self.lib.or_quantize_weights(w.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), rows, columns,
                                     weight_bits, values.ctypes.data_as(ctypes.POINTER(ctypes.c_int16)),
                                     scales.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return values, scales

    def run(self, program, inputs: Sequence[np.ndarray], weights: np.ndarray | None = None):
        """run_cpu on FP32 NCHW inputs. `weights` defaults to the program's FP16
        on-disk weights widened (what a loaded program holds); pass
        program.weights to run the in-memory FP32 form."""
        w = np.ascontiguousarray(program.fp16_weights() if weights is None else weights, np.float32)
        nodes = (_Node * max(1, len(program.nodes)))()
        for index, node in enumerate(program.nodes):
            n = nodes[index]
            n.kind = int(node.kind)
            n.input0, n.input1 = node.inputs
            n.input_count, n.output = node.input_count, node.output
            n.in_channels, n.out_channels, n.depthwise = node.in_channels, node.out_channels, int(node.depthwise)
            n.kernel_h, n.kernel_w = node.kernel
            n.stride_y, n.stride_x = node.stride
            n.pad_top, n.pad_left, n.pad_bottom, n.pad_right = node.pads
            n.weight_offset, n.bias_offset = node.weight_offset, node.bias_offset
            n.scalar = node.scalar
            n.begin, n.end, n.block, n.axis = node.begin, node.end, node.block, node.axis
            n.minimum, n.maximum = node.minimum, node.maximum
            n.weight_bits, n.activation_bits = node.weight_bits, node.activation_bits
        channels = _i32(program.tensor_channels)
        ins = _i32(program.inputs)
        outs = _i32(program.outputs)
        prog = _Program(len(program.tensor_channels), channels, len(program.inputs), ins,
                        len(program.outputs), outs, len(program.nodes), nodes,
                        w.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), w.size)
        keep = [np.ascontiguousarray(x, np.float32) for x in inputs]
        tensors = (_Tensor * max(1, len(keep)))()
        for index, x in enumerate(keep):
            c, h, wd = x.shape
            tensors[index] = _Tensor(c, h, wd, x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        results = (_Tensor * max(1, len(program.outputs)))()
        error = ctypes.create_string_buffer(512)
        status = self.lib.or_run(ctypes.byref(prog), tensors, results, error, 512)
        if status != 0:
            raise RuntimeError(f"oracle: {error.value.decode()}")
        outputs = []
        for index in range(len(program.outputs)):
            t = results[index]
            count = t.channels * t.height * t.width
            array = np.ctypeslib.as_array(t.values, shape=(max(count, 1),))[:count].copy()
            outputs.append(array.reshape(t.channels, t.height, t.width))
            self.lib.or_free(ctypes.cast(t.values, ctypes.c_void_p))
        return outputs


class Reference:
    """The reference's own run_cpu, compiled from its sources (oracle/_ref)."""

    def __init__(self, path: Path = REFERENCE_LIB) -> None:
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (needs the reference sources)")
        lib = ctypes.CDLL(str(path))
        self.lib = lib
        f32p = ctypes.POINTER(ctypes.c_float)
        lib.ref_load_check.restype = ctypes.c_int
        lib.ref_load_check.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
        lib.ref_run.restype = ctypes.c_int
        lib.ref_run.argtypes = [ctypes.c_char_p, f32p, ctypes.c_int64, ctypes.c_int,
                                ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(f32p), ctypes.c_int,
                                ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(f32p),
                                ctypes.c_char_p, ctypes.c_size_t]
        lib.ref_time_run.restype = ctypes.c_double
        lib.ref_time_run.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(f32p), ctypes.c_int]
        lib.ref_numerics_identity.restype = ctypes.c_int
        lib.ref_numerics_identity.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), ctypes.c_char_p,
                                              ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t,
                                              ctypes.POINTER(ctypes.c_size_t)]
        lib.ref_numerics_identity_parse.restype = ctypes.c_int
        lib.ref_numerics_identity_parse.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                                    ctypes.c_size_t, ctypes.c_char_p]
        lib.ref_infer_extents.restype = ctypes.c_int
        lib.ref_infer_extents.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
                                          ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
                                          ctypes.c_char_p, ctypes.c_size_t]
        lib.ref_quantize_weights.argtypes = [f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.POINTER(ctypes.c_int16), f32p]
        for name, res, args in [
            ("ref_det_exp", ctypes.c_float, [ctypes.c_float]),
            ("ref_det_sigmoid", ctypes.c_float, [ctypes.c_float]),
            ("ref_det_ldexp", ctypes.c_float, [ctypes.c_float, ctypes.c_int]),
            ("ref_det_int_exponent", ctypes.c_int, [ctypes.c_float, ctypes.c_int]),
            ("ref_det_int_quantize", ctypes.c_int, [ctypes.c_float, ctypes.c_int, ctypes.c_int]),
            ("ref_det_int_output", ctypes.c_float, [ctypes.c_longlong, ctypes.c_float, ctypes.c_int,
                                                    ctypes.c_float]),
            ("ref_half_to_float", ctypes.c_float, [ctypes.c_uint16]),
            ("ref_float_to_half", ctypes.c_uint16, [ctypes.c_float]),
        ]:
            getattr(lib, name).restype = res
            getattr(lib, name).argtypes = args
        lib.ref_free.argtypes = [ctypes.c_void_p]

    @staticmethod
    def available() -> bool:
        return REFERENCE_LIB.exists()

    def load_check(self, program_json) -> tuple[int, str]:
        error = ctypes.create_string_buffer(512)
        code = self.lib.ref_load_check(str(program_json).encode(), error, 512)
        return code, error.value.decode()

    @staticmethod
    def _pack_inputs(inputs):
        keep = [np.ascontiguousarray(x, np.float32) for x in inputs]
        extents = _i32([d for x in keep for d in x.shape])
        f32p = ctypes.POINTER(ctypes.c_float)
        pointers = (f32p * max(1, len(keep)))(*[x.ctypes.data_as(f32p) for x in keep])
        return keep, extents, pointers

    def run(self, program_json, inputs: Sequence[np.ndarray], weights: np.ndarray | None = None,
            max_outputs: int = 16):
        keep, extents, pointers = self._pack_inputs(inputs)
        f32p = ctypes.POINTER(ctypes.c_float)
        w = None if weights is None else np.ascontiguousarray(weights, np.float32)
        out_extents = (ctypes.c_int32 * (3 * max_outputs))()
        outs = (f32p * max_outputs)()
        error = ctypes.create_string_buffer(512)
        status = self.lib.ref_run(str(program_json).encode(),
                                  None if w is None else w.ctypes.data_as(f32p),
                                  0 if w is None else w.size, len(keep), extents, pointers,
                                  max_outputs, out_extents, outs, error, 512)
        if status != 0:
            raise RuntimeError(f"reference run_cpu: {error.value.decode()} (code {status - 1})")
        results = []
        for slot in range(max_outputs):
            if not outs[slot]:
                break
            c, h, wd = out_extents[3 * slot: 3 * slot + 3]
            count = c * h * wd
            array = np.ctypeslib.as_array(outs[slot], shape=(max(count, 1),))[:count].copy()
            results.append(array.reshape(c, h, wd))
            self.lib.ref_free(ctypes.cast(outs[slot], ctypes.c_void_p))
        return results

    def time_run(self, program_json, inputs, repeats: int = 1) -> float:
        keep, extents, pointers = self._pack_inputs(inputs)
        seconds = self.lib.ref_time_run(str(program_json).encode(), len(keep), extents, pointers, repeats)
        if seconds < 0:
            raise RuntimeError("reference run_cpu failed while timing")
        return seconds

    def infer_extents(self, program_json, extents_in, max_outputs: int = 16):
        flat = _i32([d for e in extents_in for d in e])
        out = (ctypes.c_int32 * (3 * max_outputs))()
        error = ctypes.create_string_buffer(512)
        status = self.lib.ref_infer_extents(str(program_json).encode(), len(extents_in), flat,
                                            max_outputs, out, error, 512)
        if status != 0:
            return status, error.value.decode()  # 1 + ErrorCode
        return 0, [tuple(out[3 * i: 3 * i + 3]) for i in range(max_outputs) if out[3 * i] != 0]

    def numerics_identity(self, profile: str, stages):
        """(status, payload): NumericsIdentityIO::make + serialize; status 0 or 1 + ErrorCode."""
        ids = (ctypes.c_char_p * max(1, len(stages)))(*[sid.encode() for sid, _ in stages])
        digests = b"".join(bytes(d) for _, d in stages)
        payload = ctypes.create_string_buffer(256)
        size = ctypes.c_size_t(0)
        status = self.lib.ref_numerics_identity(profile.encode(), ids, digests, len(stages), payload, len(payload),
                                                ctypes.byref(size))
        return status, payload.raw[:size.value] if status == 0 else b""

    def parse_numerics_identity(self, payload: bytes):
        """(status, profile, digest): NumericsIdentityIO::deserialize."""
        profile = ctypes.create_string_buffer(256)
        digest = ctypes.create_string_buffer(32)
        status = self.lib.ref_numerics_identity_parse(bytes(payload), len(payload), profile, len(profile), digest)
        return (status, profile.value.decode(), digest.raw) if status == 0 else (status, "", b"")

    def quantize_weights(self, weights: np.ndarray, weight_bits: int):
        w = np.ascontiguousarray(weights, np.float32)
        rows, columns = w.shape
        values = np.zeros((rows, columns), np.int16)
        scales = np.zeros(rows, np.float32)
        f32p = ctypes.POINTER(ctypes.c_float)
        self.lib.ref_quantize_weights(w.ctypes.data_as(f32p), rows, columns, weight_bits,
                                      values.ctypes.data_as(ctypes.POINTER(ctypes.c_int16)),
                                      scales.ctypes.data_as(f32p))
        return values, scales


def same_bits(left: np.ndarray, right: np.ndarray) -> bool:
    """The profile's equality: bitwise, except that every NaN equals every NaN
    (reference tests/deterministic_executor_tests.cpp:54-60)."""
    left = np.asarray(left, np.float32)
    right = np.asarray(right, np.float32)
    if left.shape != right.shape:
        return False
    ln, rn = np.isnan(left), np.isnan(right)
    if not np.array_equal(ln, rn):
        return False
    return np.array_equal(left.view(np.uint32)[~ln], right.view(np.uint32)[~rn])


def count_differing(left: np.ndarray, right: np.ndarray) -> int:
    left = np.asarray(left, np.float32).reshape(-1)
    right = np.asarray(right, np.float32).reshape(-1)
    if left.shape != right.shape:
        return max(left.size, right.size)
    ln, rn = np.isnan(left), np.isnan(right)
    bits_differ = left.view(np.uint32) != right.view(np.uint32)
    return int(np.count_nonzero((ln != rn) | (bits_differ & ~(ln & rn))))


def canonical_digest(array: np.ndarray) -> str:
    """SHA-256 of the FP32 bytes with every NaN made the canonical quiet NaN."""
    import hashlib
    a = np.ascontiguousarray(array, np.float32).copy()
    a[np.isnan(a)] = np.float32("nan")
    bits = a.view(np.uint32)
    bits[np.isnan(a)] = 0x7FC00000
    return hashlib.sha256(bits.tobytes()).hexdigest()


REFERENCE_GPU_LIB = HERE / "_ref" / "libnvcr_ref_cuda.so"


class ReferenceGpu:
    """The reference's own CUDA executor (CudaExecutor, src/deterministic/
    cuda_executor.cu) built for sm_100a with its kernel flags into
    oracle/_ref/libnvcr_ref_cuda.so: the GPU comparator, timed beside the new
    path in the benchmark. One executor per program, on a given CUDA stream."""

    _lib = None

    @classmethod
    def available(cls) -> bool:
        return REFERENCE_GPU_LIB.exists()

    @classmethod
    def library(cls):
        if cls._lib is None:
            lib = ctypes.CDLL(str(REFERENCE_GPU_LIB))
            vp, cp = ctypes.c_void_p, ctypes.c_char_p
            i32p = ctypes.POINTER(ctypes.c_int32)
            lib.refgpu_create.restype = ctypes.c_int
            lib.refgpu_create.argtypes = [cp, vp, ctypes.POINTER(vp), cp, ctypes.c_size_t]
            lib.refgpu_run_half.restype = ctypes.c_int
            lib.refgpu_run_half.argtypes = [vp, ctypes.c_int, ctypes.POINTER(cp), i32p, ctypes.POINTER(vp),
                                            ctypes.c_int, ctypes.POINTER(cp), i32p, ctypes.POINTER(vp), cp,
                                            ctypes.c_size_t]
            lib.refgpu_destroy.argtypes = [vp]
            cls._lib = lib
        return cls._lib

    def __init__(self, program_json, stream: int | None = None) -> None:
        lib = self.library()
        handle = ctypes.c_void_p()
        error = ctypes.create_string_buffer(512)
        status = lib.refgpu_create(str(program_json).encode(), stream, ctypes.byref(handle), error, 512)
        if status != 0:
            raise RuntimeError(f"reference CudaExecutor::create: {error.value.decode()} (code {status - 1})")
        self._handle = handle

    @staticmethod
    def _pack(named):
        names = list(named)
        name_array = (ctypes.c_char_p * max(1, len(names)))(*[n.encode() for n in names])
        extents = _i32([d for n in names for d in tuple(named[n].shape)])
        data = (ctypes.c_void_p * max(1, len(names)))(*[named[n].data_ptr() for n in names])
        return len(names), name_array, extents, data

    def run_half(self, inputs, outputs) -> None:
        """CudaExecutor::run_half on dicts name -> contiguous FP16 CUDA tensor (c, h, w)."""
        error = ctypes.create_string_buffer(512)
        status = self.library().refgpu_run_half(self._handle, *self._pack(inputs), *self._pack(outputs), error, 512)
        if status != 0:
            raise RuntimeError(f"reference CudaExecutor::run_half: {error.value.decode()} (code {status - 1})")

    def close(self) -> None:
        if self._handle:
            self.library().refgpu_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
