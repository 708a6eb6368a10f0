"""Shared parity helpers for the tests.

Matmul bar (max relative error 1e-3, fp32 with the accumulation reordered), measured as
    rel(y, r) = max_i |y_i - r_i| / max(|r_i|, 1e-3 * max_j |r_j|)
The floor keeps the relative error well-posed for outputs near zero.  Two checks:
  1. rel(y, exact) <= 1e-3, exact = the same quantized products summed in float64;
  2. rel(y, ref)   <= 1e-3 + rel(exact, ref), ref = the oracle's sequential f32 sum.
Reordering is allowed, so the reference's own rounding -- its distance from the exact sum --
is added to the budget of check 2: it measures ~4e-4 at K = 2048 and ~8e-4 at K = 6144, where
no reordering of the f32 sum can do better.
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


def exact_matmul(kind: str, data, scales, block_size: int, N: int, K: int, X) -> np.ndarray:
    """float64 sum of x * q * scale (q and scale exact in float64) -- the exact quantized matmul."""
    X = np.atleast_2d(np.asarray(X, np.float64))
    out = np.empty((X.shape[0], N), np.float64)
    sc = np.asarray(scales, np.float64)
    step = max(1, (1 << 24) // max(K, 1))
    for r0 in range(0, N, step):
        r1 = min(N, r0 + step)
        g = np.arange(r0 * K, r1 * K, dtype=np.int64)
        if kind == "int8":
            q = np.asarray(data, np.int8)[g].astype(np.float64)
        else:
            b = np.asarray(data, np.uint8)[g // 2].astype(np.int64)
            q = np.where(g % 2 == 0, b & 15, b >> 4).astype(np.float64) - 8.0
        w = (q * sc[g // block_size]).reshape(r1 - r0, K)
        out[:, r0:r1] = X @ w.T
    return out


def check_matmul(y, ref, exact) -> None:
    """Both parity checks of the module docstring; raises AssertionError with the numbers."""
    e_exact = rel_err(y, exact)
    e_ref = rel_err(y, ref)
    budget = MATMUL_TOL + rel_err(exact, ref)
    assert e_exact <= MATMUL_TOL and e_ref <= budget, dict(
        vs_exact=e_exact, vs_ref=e_ref, ref_budget=budget, normwise=normwise_err(y, ref))


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


def tie_blocks(amax: float, bs: int = 16) -> np.ndarray:
    """Blocks of bs values whose last element is amax (127 for int8, 7 for int4), so the block's
    scale is exactly 1 and each other value is its own quotient: the rounding ties k + 0.5 of
    f32::round and their f32 neighbours for |k + 0.5| < amax, plus +-0.49999997."""
    lim = int(amax) - 1
    ties = []
    for k in range(-lim - 1, lim + 1):
        c = np.float32(k + 0.5)
        ties += [np.nextafter(c, np.float32(-np.inf)), c, np.nextafter(c, np.float32(np.inf))]
    ties += [np.float32(0.49999997), np.float32(-0.49999997)]
    ties = np.array([t for t in ties if abs(float(t)) < amax], np.float32)
    blocks = []
    for i in range(0, ties.size, bs - 1):
        blk = np.zeros(bs, np.float32)
        part = ties[i:i + bs - 1]
        blk[:part.size] = part
        blk[-1] = np.float32(amax)
        blocks.append(blk)
    return np.concatenate(blocks)
