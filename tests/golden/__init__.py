"""Golden fixtures: seeds + reference (run_region) outputs, and the input regenerator."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float values to bfloat16 (nearest-even), returned as float64."""
    f = np.asarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def draw(seed: int, shape, dtype: str, scale: float = 1.0, shift: float = 0.0) -> np.ndarray:
    """scale * N(0,1) + shift from ``default_rng(seed)``, rounded to ``dtype``."""
    a = scale * np.random.default_rng(seed).standard_normal(tuple(shape)) + shift
    if dtype == "f32":
        return a.astype(np.float32).astype(np.float64)
    if dtype == "bf16":
        return round_bf16(a)
    if dtype == "f64":
        return a
    raise ValueError(dtype)


def input_checksum(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float64).tobytes()).hexdigest()[:16]


def load(case: str):
    """-> (spec dict, list of input arrays (f64), list of output arrays (f64))."""
    z = np.load(HERE / f"{case}.npz")
    spec = json.loads(str(z["spec"]))
    ins = [draw(s["seed"], s["shape"], s["dtype"], s.get("scale", 1.0), s.get("shift", 0.0)) for s in spec["inputs"]]
    outs = [z[f"out{i}"] for i in range(len([k for k in z.files if k.startswith("out")]))]
    return spec, ins, outs
