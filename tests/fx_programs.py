"""nvcr.fx.v1 programs for the tests: the on-disk writer (format
nvcr.fx-program.v1, docs/spec/numerics-fx-v1.md section 6) and seeded
program generators.

A program is a dict in the shape of ``<stage>.fxprog.json`` with the
data-file arrays inline as numpy arrays (the form ``oracle/fx.py`` runs).
``write_program`` lays those arrays out in ``<stage>.fxw`` (little-endian,
each field's element type fixed by the spec's node table) and writes the JSON
with the data file's SHA-256, so the reference's own loader reads exactly
what the oracle runs.
"""
from __future__ import annotations

import copy
import hashlib
import json
from pathlib import Path

import numpy as np

# Element type of each array field (spec section 6, node table).
ARRAY_FIELDS = {
    "gemm": {"weights": np.int16, "bias": np.int64, "shift": np.int32},
    "depthwise3x3": {"weights": np.int32, "bias": np.int64, "shift": np.int32},
    "param_row": {"rows": np.int64},
    "sat_table": {"table": np.int32},
}


def write_program(directory: Path, stage: str, program: dict, mutate=None) -> Path:
    """Writes <stage>.fxprog.json and <stage>.fxw; ``mutate(json_dict)`` may
    edit the JSON before it is written (for load-time refusal tests)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    blob = bytearray()

    def place(values, dtype) -> list[int]:
        array = np.ascontiguousarray(values, dtype=np.dtype(dtype).newbyteorder("<"))
        offset = len(blob)
        blob.extend(array.tobytes())
        return [offset, int(array.size)]

    document = {"format": "nvcr.fx-program.v1", "profile": "nvcr.fx.v1", "fa": program.get("fa", 14),
                "data": {"file": f"{stage}.fxw", "sha256": ""},
                "tensors": [{"name": name, "channels": channels} for name, channels in program["tensors"]],
                "inputs": list(program["inputs"]), "outputs": list(program["outputs"]),
                "delta_tables": [{"h": t["h"], "shift": t["shift"], "dc": place(t["dc"], np.int16)}
                                 for t in program.get("delta_tables", [])],
                "nodes": []}
    for node in program["nodes"]:
        entry = {}
        arrays = ARRAY_FIELDS.get(node["op"], {})
        for key, value in node.items():
            entry[key] = place(value, arrays[key]) if key in arrays else value
        document["nodes"].append(entry)
    data_path = directory / f"{stage}.fxw"
    data_path.write_bytes(bytes(blob))
    document["data"]["sha256"] = hashlib.sha256(bytes(blob)).hexdigest()
    if mutate is not None:
        mutate(document)
    path = directory / f"{stage}.fxprog.json"
    path.write_text(json.dumps(document))
    return path


def delta_table(rng: np.random.Generator, h: int, shift: int) -> dict:
    return {"h": h, "shift": shift, "dc": rng.integers(-(1 << 15) + 1, 1 << 15, ((2 * h) >> shift) + 1).astype(np.int16)}


def gemm_node(rng, inputs, output, in_channels, out_channels, group=1, input_shift=0, table=-1,
              weight_max=32639, shift=(8, 16), bias_max=1 << 20) -> dict:
    return {"op": "gemm", "inputs": list(inputs), "output": output, "in_channels": in_channels,
            "out_channels": out_channels, "group": group, "input_shift": input_shift, "delta_table": table,
            "weights": rng.integers(-weight_max, weight_max + 1, (out_channels, in_channels)).astype(np.int16),
            "bias": rng.integers(-bias_max, bias_max + 1, out_channels).astype(np.int64),
            "shift": rng.integers(shift[0], shift[1] + 1, out_channels).astype(np.int32)}


def decoder_like(rng: np.random.Generator, channels: int = 8, qps: int = 4, tight: bool = False) -> dict:
    """A seeded program that uses every op of the profile once or more, in the
    order a DCVC-style decoder block would (per-QP scale, im2col + gemm with a
    delta activation and grouping, depthwise, gemm with a residual, delta,
    sigmoid table, quant-step affine, products, add, clamp, shuffles, slice,
    concat, strided im2cols, crop). ``tight`` picks smaller shifts, so that
    more programs hit the gemm and stored-bound failures."""
    c = channels
    o = 2 * c
    shift = (1, 4) if tight else (9, 14)
    tables = [delta_table(rng, int(rng.integers(1, 1 << 16)), int(rng.integers(0, 5))),
              delta_table(rng, int(rng.integers(1, 1 << 12)), int(rng.integers(0, 3)))]
    n = int(rng.integers(1, 4096))
    names = [("x", c), ("q", 1), ("scale", c), ("xs", c), ("cols", 9 * c), ("h", c), ("d", c), ("e", c),
             ("e2", c), ("s", c), ("a", c), ("m", c), ("s2", c), ("cl", c), ("up", c // 4), ("back", c),
             ("sl", c // 2), ("cc", c + c // 2), ("down", 4 * (c + c // 2)), ("g2", c), ("cols2", 9 * c),
             ("crop", c), ("ref", 1), ("one", 1), ("e_scaled", c)]
    ids = {name: index for index, (name, _) in enumerate(names)}
    nodes = [
        {"op": "param_row", "inputs": [ids["q"]], "output": ids["scale"],
         "rows": rng.integers(-(1 << 24), (1 << 24) + 1, (qps, c)).astype(np.int64)},
        {"op": "mul", "inputs": [ids["x"], ids["scale"]], "output": ids["xs"], "shift": 18},
        {"op": "im2col", "inputs": [ids["xs"]], "output": ids["cols"], "kernel": 3, "stride": 1},
        gemm_node(rng, [ids["cols"]], ids["h"], 9 * c, o, group=2, input_shift=int(rng.integers(0, 4)),
                  table=0, shift=(shift[0] + 4, shift[1] + 4)),
        {"op": "depthwise3x3", "inputs": [ids["h"]], "output": ids["d"],
         "weights": rng.integers(-(1 << 12), (1 << 12) + 1, (c, 3, 3)).astype(np.int32),
         "bias": rng.integers(-(1 << 40), (1 << 40) + 1, c).astype(np.int64),
         "shift": rng.integers(shift[0] + 2, shift[1] + 4, c).astype(np.int32)},
        gemm_node(rng, [ids["d"], ids["h"]], ids["e"], c, c, shift=(shift[0] + 6, shift[1] + 6)),
        {"op": "delta", "inputs": [ids["e"]], "output": ids["e2"], "delta_table": 1},
        {"op": "sat_table", "inputs": [ids["e2"]], "output": ids["s"],
         "table": np.sort(rng.integers(0, 1 << 14, 2 * n)).astype(np.int32), "top": 1 << 14},
        {"op": "affine", "inputs": [ids["s"]], "output": ids["a"], "alpha": 3, "beta": 1 << 14, "shift": 1},
        {"op": "mul", "inputs": [ids["e"], ids["a"]], "output": ids["m"], "shift": 14},
        {"op": "add", "inputs": [ids["m"], ids["e2"]], "output": ids["s2"]},
        {"op": "clamp", "inputs": [ids["s2"]], "output": ids["cl"],
         "lo": -int(rng.integers(0, 1 << 20)), "hi": int(rng.integers(0, 1 << 20))},
        {"op": "pixel_shuffle", "inputs": [ids["cl"]], "output": ids["up"], "factor": 2},
        {"op": "pixel_unshuffle", "inputs": [ids["up"]], "output": ids["back"], "factor": 2},
        {"op": "slice", "inputs": [ids["back"]], "output": ids["sl"], "begin": c // 4, "end": c // 4 + c // 2},
        {"op": "concat", "inputs": [ids["back"], ids["sl"]], "output": ids["cc"]},
        {"op": "im2col", "inputs": [ids["cc"]], "output": ids["down"], "kernel": 2, "stride": 2},
        gemm_node(rng, [ids["down"]], ids["g2"], 4 * (c + c // 2), 4 * c, group=4,
                  input_shift=int(rng.integers(0, 3)), shift=shift),
        {"op": "im2col", "inputs": [ids["g2"]], "output": ids["cols2"], "kernel": 3, "stride": 2},
        {"op": "crop_like", "inputs": [ids["e"], ids["ref"]], "output": ids["crop"]},
        {"op": "affine", "inputs": [ids["ref"]], "output": ids["one"], "alpha": -(1 << 10),
         "beta": int(rng.integers(-(1 << 24), 1 << 24)), "shift": int(rng.integers(0, 12))},
        {"op": "mul", "inputs": [ids["crop"], ids["one"]], "output": ids["e_scaled"], "shift": 24},
    ]
    return {"fa": 14, "tensors": names, "inputs": [ids["x"], ids["q"], ids["ref"]],
            "outputs": [ids["g2"], ids["cols2"], ids["e_scaled"], ids["s"]],
            "delta_tables": tables, "nodes": nodes}


def decoder_like_inputs(rng: np.random.Generator, program: dict, height: int, width: int,
                        crop: tuple[int, int] | None = None, qp: int | None = None,
                        magnitude: int = 1 << 16) -> list[np.ndarray]:
    c = program["tensors"][0][1]
    qps = program["nodes"][0]["rows"].shape[0]
    crop = crop or (max(1, height - 1), max(1, width - 2))
    x = rng.integers(-magnitude, magnitude + 1, (c, height, width)).astype(np.int32)
    q = np.array([[[qp if qp is not None else int(rng.integers(0, qps))]]], np.int32)
    ref = rng.integers(-(1 << 10), (1 << 10) + 1, (1, crop[0], crop[1])).astype(np.int32)
    return [x, q, ref]


def program_copy(program: dict) -> dict:
    return copy.deepcopy(program)
