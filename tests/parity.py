"""Shared parity helpers for the tests.

Matmul tolerance (the stated bar: max relative error 1e-3, fp32 with reordered accumulation):
    rel = max_i |y_i - ref_i| / max(|ref_i|, 1e-3 * max_j |ref_j|)  <=  1e-3
The floor keeps the relative error well-posed for outputs near zero; the reference's own f32
rounding against exact arithmetic measures ~4e-4 on this metric at the 6144x2048 shape.
"""
from __future__ import annotations

import json
import os

import numpy as np

MATMUL_TOL = 1e-3
HERE = os.path.dirname(os.path.abspath(__file__))


def rel_err(y, ref) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    floor = 1e-3 * np.abs(ref).max()
    denom = np.maximum(np.abs(ref), floor)
    denom[denom == 0] = 1.0
    return float((np.abs(y - ref) / denom).max())


def normwise_err(y, ref) -> float:
    ref = np.asarray(ref, dtype=np.float64)
    m = np.abs(ref).max() if ref.size else 0.0
    return float(np.abs(np.asarray(y, np.float64) - ref).max() / (m if m else 1.0))


def load_kats():
    with open(os.path.join(HERE, "golden", "reference_kats.json")) as f:
        return json.load(f)["kats"]


def f32_eps() -> float:
    return float(np.finfo(np.float32).eps)


def q8_0_bytes(blocks) -> bytes:
    """Serialise [(f16 scale bits, [32 x i8]), ...] as GGUF Q8_0 blocks (34 bytes each)."""
    out = bytearray()
    for scale_bits, vals in blocks:
        out += int(scale_bits).to_bytes(2, "little")
        out += bytes((v & 0xFF) for v in vals)
    return bytes(out)
