"""ctypes access to the nvcr.fx.v1 checkers. TEST INFRASTRUCTURE ONLY.

Only tests/ import this module, and only to check; the product never does.

* ``FxOracle``: this repo's C restatement of the profile's integer ops
  (fx_oracle.c, built into oracle/_build/liboracle.so) and a program runner
  over it. The runner follows the reference's ``fx::run``
  (src/deterministic/fx_program.cpp:468-525): the same run-time shape checks,
  the same stage failures, nodes in program order; the exact data-movement
  nodes (concat, slice, crop_like, pixel_(un)shuffle, im2col, param_row) are
  numpy index arithmetic as the spec defines them
  (docs/spec/numerics-fx-v1.md section 4.7).
* ``FxReference``: the reference's own fx.cpp and fx_program.cpp compiled
  from its sources into oracle/_ref/libnvcr_ref.so, reached through its own
  program loader (``fx::load_program``) from the files the tests write.

Programs are dicts in the shape of ``<stage>.fxprog.json`` (section 6), with
the data-file arrays inline as numpy arrays of the field's element type:
``{"fa", "tensors": [(name, channels)], "inputs", "outputs",
"delta_tables": [{"h", "shift", "dc"}], "nodes": [{"op", "inputs", "output",
...fields}]}``.

Results are ``(status, outputs, reason)``: status 0, or the reference's
ErrorCode value plus one (1 invalid_argument for a program that cannot run on
these inputs, 4 malformed_bitstream for a stage failure); ``reason`` names
the rule that failed in the reference's words, so a test can check that both
sides failed for the same reason.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Sequence

import numpy as np

from .oracle import ORACLE_LIB, REFERENCE_LIB

INVALID = 1       # ErrorCode::invalid_argument + 1
STAGE_FAILURE = 4  # ErrorCode::malformed_bitstream + 1

DIGIT2_MAX = 32639
STORED_MAX = 1 << 30
GEMM_LIMIT = (1 << 29) - 1

_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i16p = ctypes.POINTER(ctypes.c_int16)

_OP_FAILURES = {"gemm": {1: "gemm pre-activation out of range", 2: "gemm output out of range"},
                "depthwise3x3": {2: "depthwise output out of range"},
                "mul": {2: "mul output out of range"},
                "affine": {2: "affine output out of range"},
                "add": {2: "add output out of range"}}


def _ptr(array: np.ndarray, kind):
    return array.ctypes.data_as(kind)


class FxFailure(Exception):
    def __init__(self, status: int, reason: str) -> None:
        super().__init__(reason)
        self.status = status
        self.reason = reason


class FxOracle:
    """The C restatement (fx_oracle.c) and a program runner over it."""

    def __init__(self, path: Path = ORACLE_LIB) -> None:
        lib = ctypes.CDLL(str(path))
        self.lib = lib
        lib.fx_rsr.restype = ctypes.c_int64
        lib.fx_rsr.argtypes = [ctypes.c_int64, ctypes.c_int]
        lib.fx_delta_act.restype = ctypes.c_int64
        lib.fx_delta_act.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _i16p]
        lib.fx_gemm.restype = ctypes.c_int
        lib.fx_gemm.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int, ctypes.c_int, _i32p, _i64p, _i32p,
                                ctypes.c_int64, ctypes.c_int, _i16p, _i32p, ctypes.c_size_t, ctypes.c_int,
                                ctypes.POINTER(_i32p), _i32p]
        lib.fx_depthwise3x3.restype = ctypes.c_int
        lib.fx_depthwise3x3.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _i32p, _i64p, _i32p,
                                        _i32p, _i32p]
        lib.fx_mul.restype = ctypes.c_int
        lib.fx_mul.argtypes = [_i32p, ctypes.c_int32, ctypes.c_size_t, _i32p, ctypes.c_int32, ctypes.c_size_t,
                               ctypes.c_int, _i32p]
        lib.fx_affine.restype = ctypes.c_int
        lib.fx_affine.argtypes = [_i32p, ctypes.c_size_t, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _i32p]
        lib.fx_add.restype = ctypes.c_int
        lib.fx_add.argtypes = [_i32p, _i32p, ctypes.c_size_t, _i32p]
        lib.fx_sat_table.restype = None
        lib.fx_sat_table.argtypes = [_i32p, ctypes.c_size_t, _i32p, ctypes.c_size_t, ctypes.c_int32, _i32p]
        lib.fx_delta.restype = None
        lib.fx_delta.argtypes = [_i32p, ctypes.c_size_t, ctypes.c_int64, ctypes.c_int, _i16p, _i32p]
        lib.fx_clamp.restype = None
        lib.fx_clamp.argtypes = [_i32p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int32, _i32p]

    # -- scalar rules -------------------------------------------------------
    def rsr(self, a: int, s: int) -> int:
        return self.lib.fx_rsr(a, s)

    def delta_act(self, r: int, table: dict) -> int:
        dc = np.ascontiguousarray(table["dc"], np.int16)
        return self.lib.fx_delta_act(r, table["h"], table["shift"], _ptr(dc, _i16p))

    # -- ops on [C][H][W] int32 arrays; each raises FxFailure on a stage failure
    @staticmethod
    def _check(op: str, status: int) -> None:
        if status != 0:
            raise FxFailure(STAGE_FAILURE, _OP_FAILURES[op][status])

    def gemm(self, node: dict, x: np.ndarray, residuals: Sequence[np.ndarray] = (), table: dict | None = None):
        x = np.ascontiguousarray(x, np.int32)
        _, height, width = x.shape
        rows = node["out_channels"] // node["group"]
        weights = np.ascontiguousarray(node["weights"], np.int32)
        bias = np.ascontiguousarray(node["bias"], np.int64)
        shift = np.ascontiguousarray(node["shift"], np.int32)
        keep = [np.ascontiguousarray(r, np.int32) for r in residuals]
        residual_ptrs = (_i32p * max(1, len(keep)))(*[_ptr(r, _i32p) for r in keep])
        dc = np.ascontiguousarray(table["dc"], np.int16) if table is not None else None
        y = np.zeros((rows, height, width), np.int32)
        status = self.lib.fx_gemm(node["in_channels"], node["out_channels"], node["group"], node["input_shift"],
                                  _ptr(weights, _i32p), _ptr(bias, _i64p), _ptr(shift, _i32p),
                                  table["h"] if table else 0, table["shift"] if table else 0,
                                  _ptr(dc, _i16p) if dc is not None else None,
                                  _ptr(x, _i32p), height * width, len(keep), residual_ptrs, _ptr(y, _i32p))
        self._check("gemm", status)
        return y

    def depthwise3x3(self, node: dict, x: np.ndarray):
        x = np.ascontiguousarray(x, np.int32)
        weights = np.ascontiguousarray(node["weights"], np.int32)
        bias = np.ascontiguousarray(node["bias"], np.int64)
        shift = np.ascontiguousarray(node["shift"], np.int32)
        y = np.zeros_like(x)
        self._check("depthwise3x3", self.lib.fx_depthwise3x3(*x.shape, _ptr(weights, _i32p), _ptr(bias, _i64p),
                                                             _ptr(shift, _i32p), _ptr(x, _i32p), _ptr(y, _i32p)))
        return y

    def mul(self, a: np.ndarray, b: np.ndarray, shift: int):
        a = np.ascontiguousarray(a, np.int32)
        b = np.ascontiguousarray(b, np.int32)
        y = np.zeros_like(a)
        self._check("mul", self.lib.fx_mul(_ptr(a, _i32p), a.shape[0], a.shape[1] * a.shape[2], _ptr(b, _i32p),
                                           b.shape[0], b.shape[1] * b.shape[2], shift, _ptr(y, _i32p)))
        return y

    def affine(self, x: np.ndarray, alpha: int, beta: int, shift: int):
        x = np.ascontiguousarray(x, np.int32)
        y = np.zeros_like(x)
        self._check("affine", self.lib.fx_affine(_ptr(x, _i32p), x.size, alpha, beta, shift, _ptr(y, _i32p)))
        return y

    def add(self, a: np.ndarray, b: np.ndarray):
        a = np.ascontiguousarray(a, np.int32)
        b = np.ascontiguousarray(b, np.int32)
        y = np.zeros_like(a)
        self._check("add", self.lib.fx_add(_ptr(a, _i32p), _ptr(b, _i32p), a.size, _ptr(y, _i32p)))
        return y

    def sat_table(self, x: np.ndarray, table: np.ndarray, top: int):
        x = np.ascontiguousarray(x, np.int32)
        t = np.ascontiguousarray(table, np.int32)
        y = np.zeros_like(x)
        self.lib.fx_sat_table(_ptr(x, _i32p), x.size, _ptr(t, _i32p), t.size, top, _ptr(y, _i32p))
        return y

    def delta(self, x: np.ndarray, table: dict):
        x = np.ascontiguousarray(x, np.int32)
        dc = np.ascontiguousarray(table["dc"], np.int16)
        y = np.zeros_like(x)
        self.lib.fx_delta(_ptr(x, _i32p), x.size, table["h"], table["shift"], _ptr(dc, _i16p), _ptr(y, _i32p))
        return y

    def clamp(self, x: np.ndarray, lo: int, hi: int):
        x = np.ascontiguousarray(x, np.int32)
        y = np.zeros_like(x)
        self.lib.fx_clamp(_ptr(x, _i32p), x.size, lo, hi, _ptr(y, _i32p))
        return y

    # -- exact data movement (spec 4.7) --------------------------------------
    @staticmethod
    def pixel_shuffle(x: np.ndarray, r: int) -> np.ndarray:
        c, h, w = x.shape
        return x.reshape(c // (r * r), r, r, h, w).transpose(0, 3, 1, 4, 2).reshape(c // (r * r), h * r, w * r)

    @staticmethod
    def pixel_unshuffle(x: np.ndarray, r: int) -> np.ndarray:
        c, h, w = x.shape
        return x.reshape(c, h // r, r, w // r, r).transpose(0, 2, 4, 1, 3).reshape(c * r * r, h // r, w // r)

    @staticmethod
    def im2col(x: np.ndarray, k: int, stride: int) -> np.ndarray:
        pad = 1 if k == 3 else 0
        c, h, w = x.shape
        # The reference sizes the output with C++ integer division, which truncates
        # toward zero: a 2x2 stride-2 im2col of a 1-pixel-high input has one row.
        out_h = int((h + 2 * pad - k) / stride) + 1
        out_w = int((w + 2 * pad - k) / stride) + 1
        padded = np.zeros((c, h + 2 * pad + stride, w + 2 * pad + stride), np.int32)
        padded[:, pad:pad + h, pad:pad + w] = x
        y = np.zeros((c, k, k, out_h, out_w), np.int32)
        for i in range(k):
            for j in range(k):
                y[:, i, j] = padded[:, i:i + stride * out_h:stride, j:j + stride * out_w:stride]
        return y.reshape(c * k * k, out_h, out_w)

    # -- whole programs (fx::run) -------------------------------------------
    def run(self, program: dict, inputs: Sequence[np.ndarray]):
        """(status, outputs, reason) for the program on [C][H][W] int32 inputs."""
        try:
            return 0, self._run(program, inputs), ""
        except FxFailure as failure:
            return failure.status, [], failure.reason

    def _run(self, program: dict, inputs: Sequence[np.ndarray]) -> list[np.ndarray]:
        channels = [c for _, c in program["tensors"]]
        if len(inputs) != len(program["inputs"]):
            raise FxFailure(INVALID, "wrong number of inputs")
        tensors: list[np.ndarray | None] = [None] * len(channels)
        for slot, tensor_id in enumerate(program["inputs"]):
            x = np.asarray(inputs[slot], np.int32)
            if x.ndim != 3 or x.shape[0] != channels[tensor_id]:
                raise FxFailure(INVALID, "has the wrong shape")
            if x.size and (int(x.max()) > STORED_MAX or int(x.min()) < -STORED_MAX):
                raise FxFailure(STAGE_FAILURE, "input value out of range")
            tensors[tensor_id] = x
        tables = program.get("delta_tables", [])
        for node in program["nodes"]:
            ins = []
            for tensor_id in node["inputs"]:
                if tensors[tensor_id] is None:
                    raise FxFailure(INVALID, "tensor read before it is written")
                ins.append(tensors[tensor_id])
            x = ins[0]
            op = node["op"]
            if op in ("gemm", "add", "concat") and any(t.shape[1:] != x.shape[1:] for t in ins):
                raise FxFailure(INVALID, "node inputs differ in size")
            y = self._node(program, node, op, ins, tables)
            if y.shape[0] != channels[node["output"]]:
                raise FxFailure(INVALID, "node output has the wrong channel count")
            tensors[node["output"]] = y
        outputs = []
        for tensor_id in program["outputs"]:
            if tensors[tensor_id] is None:
                raise FxFailure(INVALID, "output not produced")
            outputs.append(tensors[tensor_id])
        return outputs

    def _node(self, program: dict, node: dict, op: str, ins: list[np.ndarray], tables: list[dict]) -> np.ndarray:
        x = ins[0]
        if op == "gemm":
            if x.shape[0] != node["in_channels"]:
                raise FxFailure(INVALID, "gemm input channels")
            rows = node["out_channels"] // node["group"]
            if any(r.shape[0] != rows for r in ins[1:]):
                raise FxFailure(INVALID, "residual channels")
            table = tables[node["delta_table"]] if node["delta_table"] >= 0 else None
            return self.gemm(node, x, ins[1:], table)
        if op == "depthwise3x3":
            return self.depthwise3x3(node, x)
        if op == "mul":
            b = ins[1]
            if b.shape[1] * b.shape[2] != 1 and b.shape[1:] != x.shape[1:]:
                raise FxFailure(INVALID, "mul factor size")
            return self.mul(x, b, node["shift"])
        if op == "param_row":
            out_channels = program["tensors"][node["output"]][1]
            rows = np.asarray(node["rows"], np.int64).reshape(-1)
            if x.size != 1 or int(x.flat[0]) < 0 or int(x.flat[0]) >= rows.size // out_channels:
                raise FxFailure(STAGE_FAILURE, "qp outside the parameter table")
            q = int(x.flat[0])
            return rows[q * out_channels:(q + 1) * out_channels].astype(np.int32).reshape(out_channels, 1, 1)
        if op == "crop_like":
            ref = ins[1]
            if ref.shape[1] > x.shape[1] or ref.shape[2] > x.shape[2]:
                raise FxFailure(INVALID, "crop larger than input")
            return np.ascontiguousarray(x[:, :ref.shape[1], :ref.shape[2]])
        if op == "affine":
            return self.affine(x, node["alpha"], node["beta"], node["shift"])
        if op == "add":
            if ins[1].shape[0] != x.shape[0]:
                raise FxFailure(INVALID, "add channels")
            return self.add(x, ins[1])
        if op == "sat_table":
            return self.sat_table(x, node["table"], node["top"])
        if op == "delta":
            return self.delta(x, tables[node["delta_table"]])
        if op == "clamp":
            return self.clamp(x, node["lo"], node["hi"])
        if op == "concat":
            return np.concatenate([x, ins[1]], axis=0)
        if op == "slice":
            return np.ascontiguousarray(x[node["begin"]:node["end"]])
        if op in ("pixel_shuffle", "pixel_unshuffle"):
            r = node["factor"]
            up = op == "pixel_shuffle"
            if (x.shape[0] % (r * r) != 0) if up else (x.shape[1] % r != 0 or x.shape[2] % r != 0):
                raise FxFailure(INVALID, "pixel shuffle size")
            return self.pixel_shuffle(x, r) if up else self.pixel_unshuffle(x, r)
        if op == "im2col":
            return self.im2col(x, node["kernel"], node["stride"])
        raise ValueError(f"unknown op {op}")


class FxReference:
    """The reference's fx.cpp / fx_program.cpp, compiled from its sources (oracle/_ref)."""

    def __init__(self, path: Path = REFERENCE_LIB) -> None:
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (needs the reference sources)")
        lib = ctypes.CDLL(str(path))
        self.lib = lib
        lib.ref_fx_rsr.restype = ctypes.c_int64
        lib.ref_fx_rsr.argtypes = [ctypes.c_int64, ctypes.c_int]
        lib.ref_fx_delta_act.restype = ctypes.c_int64
        lib.ref_fx_delta_act.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _i16p, ctypes.c_size_t]
        lib.ref_fx_load_check.restype = ctypes.c_int
        lib.ref_fx_load_check.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
        lib.ref_fx_program_digest.restype = ctypes.c_int
        lib.ref_fx_program_digest.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]
        lib.ref_fx_run.restype = ctypes.c_int
        lib.ref_fx_run.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, _i32p, ctypes.POINTER(_i32p),
                                   ctypes.c_int, _i32p, ctypes.POINTER(_i32p), ctypes.c_char_p, ctypes.c_size_t]
        lib.ref_free.argtypes = [ctypes.c_void_p]

    def rsr(self, a: int, s: int) -> int:
        return self.lib.ref_fx_rsr(a, s)

    def delta_act(self, r: int, table: dict) -> int:
        dc = np.ascontiguousarray(table["dc"], np.int16)
        return self.lib.ref_fx_delta_act(r, table["h"], table["shift"], _ptr(dc, _i16p), dc.size)

    def load_check(self, directory: Path, stage: str) -> tuple[int, str]:
        error = ctypes.create_string_buffer(512)
        status = self.lib.ref_fx_load_check(str(directory).encode(), stage.encode(), error, 512)
        return status, error.value.decode()

    def program_digest(self, directory: Path, stage: str) -> tuple[int, str]:
        digest = ctypes.create_string_buffer(65)
        status = self.lib.ref_fx_program_digest(str(directory).encode(), stage.encode(), digest)
        return status, digest.value.decode() if status == 0 else ""

    def run(self, directory: Path, stage: str, inputs: Sequence[np.ndarray], max_outputs: int = 16):
        """(status, outputs, message) from fx::load_program + fx::run."""
        keep = [np.ascontiguousarray(x, np.int32) for x in inputs]
        extents = np.array([d for x in keep for d in x.shape] or [0], np.int32)
        pointers = (_i32p * max(1, len(keep)))(*[_ptr(x, _i32p) for x in keep])
        out_extents = np.zeros(3 * max_outputs, np.int32)
        outputs = (_i32p * max_outputs)()
        error = ctypes.create_string_buffer(512)
        status = self.lib.ref_fx_run(str(directory).encode(), stage.encode(), len(keep), _ptr(extents, _i32p),
                                     pointers, max_outputs, _ptr(out_extents, _i32p), outputs, error, 512)
        if status != 0:
            return status, [], error.value.decode()
        result = []
        for index in range(max_outputs):
            if not outputs[index]:
                break
            c, h, w = (int(v) for v in out_extents[3 * index:3 * index + 3])
            values = np.ctypeslib.as_array(outputs[index], shape=(max(1, c * h * w),))[:c * h * w].copy()
            result.append(values.reshape(c, h, w))
            self.lib.ref_free(outputs[index])
        return 0, result, ""
