"""Runs the reference's known-answer tests (tests/golden/reference_kats.json) against an
implementation: the oracle (CPU) or the CUDA path.  Assertions restate the reference tests'."""
from __future__ import annotations

import math

import numpy as np

from parity import f32_eps, q8_0_bytes

EPS = f32_eps()


def _f32(x) -> float:
    return float(np.float32(x))


def _div32(a, b) -> float:
    return float(np.float32(a) / np.float32(b))


def _check_quant(kat, data, scales, qtype):
    e = kat["expect"]
    vals = kat["values"]
    n = len(vals)
    bs = kat["block_size"]
    if "data" in e:
        assert [int(v) for v in data] == e["data"], (kat["name"], list(data))
    if "scales" in e:
        assert [float(s) for s in scales] == e["scales"], (kat["name"], list(scales))
    if "n_scales" in e:
        assert len(scales) == e["n_scales"]
    if "num_elements" in e:
        assert e["num_elements"] == n
    if "scales_close" in e:
        for s, (a, b) in zip(scales, e["scales_close"]):
            assert abs(float(s) - _div32(a, b)) < EPS, (kat["name"], float(s), a, b)
    if "dequant_close" in e:
        if qtype == "int8":
            deq = [float(np.float32(d) * np.float32(scales[i // bs])) for i, d in enumerate(data)]
        else:
            deq = []
            for i in range(n):
                byte = int(data[i // 2])
                nib = (byte & 0x0F) if i % 2 == 0 else ((byte >> 4) & 0x0F)
                deq.append(float((np.float32(nib) - np.float32(8.0)) * np.float32(scales[i // bs])))
        for a, x in zip(deq, vals):
            assert abs(a - x) < e["dequant_close"], (kat["name"], a, x)


def run_kat(kat, impl) -> bool:
    """Returns False when `impl` does not cover the KAT's op (e.g. F32 weights on the GPU)."""
    op = kat["op"]
    if op in ("quantize_int8", "quantize_int4"):
        qt = op.split("_")[1]
        data, scales = impl.quantize(qt, np.asarray(kat["values"], np.float32), kat["block_size"])
        _check_quant(kat, data, scales, qt)
        return True
    if op == "quantize_weights":  # src/model.rs:501-530: int8 block = in_features, int4 block = 32
        qt = kat["qtype"]
        bs = kat["in_features"] if qt == "int8" else 32
        src = np.asarray(kat["bf16"], np.uint16) if "bf16" in kat else np.asarray(kat["values"], np.float32)
        data, scales = impl.quantize(qt, src, bs)
        e = kat["expect"]
        assert len(data) == e["data_len"]
        assert bs == e["block_size"]
        if "scales" in e:
            assert [float(s) for s in scales] == e["scales"]
        if "scales_close" in e:
            for s, (a, b) in zip(scales, e["scales_close"]):
                assert abs(float(s) - _div32(a, b)) < EPS
        if "scales_exact" in e:
            assert [float(s) for s in scales] == [_div32(a, b) for a, b in e["scales_exact"]]
        return True
    if op == "matmul_vs_f32":
        N, K, bs = kat["out_features"], kat["in_features"], kat["block_size"]
        w = np.asarray(kat["weight"], np.float32)
        x = np.asarray(kat["input"], np.float32)
        y = impl.quantized_matmul(kat["qtype"], w, bs, x, N, K)
        ref = [sum(float(np.float32(x[i]) * np.float32(w[n * K + i])) for i in range(K)) for n in range(N)]
        for a, b in zip(y, ref):
            assert abs(float(a) - b) < kat["tol"], (kat["name"], float(a), b)
        return True
    if op == "q8_0":
        blob = q8_0_bytes(kat["blocks"])
        data, scales = impl.q8_0(blob, kat["n"])
        e = kat["expect"]
        if "data" in e:
            assert [int(v) for v in data] == e["data"]
            assert [float(s) for s in scales] == e["scales"]
        if "dequant" in e:
            deq = [float(np.float32(d) * np.float32(scales[i // 32])) for i, d in enumerate(data)]
            assert deq == e["dequant"]
        return True
    if op == "argmax":
        assert impl.argmax(np.asarray(kat["values"], np.float32)) == kat["expect"]
        return True
    if op == "matmul_f32_ones":
        if not hasattr(impl, "matmul_f32"):
            return False
        y = impl.matmul_f32(np.ones(kat["in_features"], np.float32),
                            np.ones(kat["out_features"] * kat["in_features"], np.float32),
                            kat["out_features"], kat["in_features"])
        assert np.all(y == kat["expect_all"])
        return True
    if op == "greedy_f32":
        if not hasattr(impl, "matmul_f32"):
            return False
        logits = impl.matmul_f32(np.asarray(kat["hidden_state"], np.float32),
                                 np.asarray(kat["weight"], np.float32), kat["vocab"], kat["hidden"])
        assert impl.argmax(logits) == kat["expect"]
        return True
    if op == "rmsnorm":
        if not hasattr(impl, "rmsnorm"):
            return False
        y = impl.rmsnorm(kat["x"], kat["weight"], kat["eps"])
        for a, b in zip(y, kat["expect_close"]):
            assert abs(float(a) - b) <= max(kat["tol"], 0.0) + (0.0 if kat["tol"] else 0.0), (kat["name"], a, b)
        return True
    if op == "rope":
        if not hasattr(impl, "rope"):
            return False
        y = impl.rope(kat["x"], kat["head_dim"], kat["pos"], kat["theta"])
        a0, a1 = 1.0, 1.0 / math.sqrt(kat["theta"])
        exp = [math.cos(a0), -math.sin(a1), math.sin(a0), math.cos(a1)]
        for a, b in zip(y, exp):
            assert abs(float(a) - b) < kat["tol"]
        return True
    if op == "silu":
        if not hasattr(impl, "silu"):
            return False
        assert abs(impl.silu(kat["x"]) - kat["expect"]) < kat["tol"]
        return True
    if op == "matmul_f32":
        y = impl.matmul_f32(np.asarray(kat["input"], np.float32), np.asarray(kat["weight"], np.float32),
                            kat["out_features"], kat["in_features"])
        assert len(y) == len(kat["expect"]), (kat["name"], len(y))
        for a, b in zip(y, kat["expect"]):
            if kat["tol"] == 0.0:
                assert float(a) == b, (kat["name"], float(a), b)
            else:
                assert abs(float(a) - b) < kat["tol"], (kat["name"], float(a), b)
        return True
    if op == "bf16_vs_f32":
        if not hasattr(impl, "matmul_bf16"):
            return False
        N, K = kat["out_features"], kat["in_features"]
        x = np.asarray(kat["input"], np.float32)
        wf = np.asarray(kat["weight"], np.float32)
        bits = bf16_truncate(wf)
        y = impl.matmul_bf16(x, bits, N, K)
        ref = sequential_matmul(x, widen_bf16(bits) if kat["against"] == "widened" else wf, N, K)
        for a, b in zip(y, ref):
            assert abs(float(a) - float(b)) < kat["tol"], (kat["name"], float(a), float(b))
        return True
    if op == "formula_matmul":
        if not hasattr(impl, "dense_matmul"):
            return False
        N, K = kat["out_features"], kat["in_features"]
        x, wf = formula_inputs(kat)
        w = bf16_truncate(wf) if kat["dtype"] == "bf16" else wf
        ref = sequential_matmul(x, widen_bf16(w) if kat["dtype"] == "bf16" else w, N, K)
        for via in kat["via"]:
            y = np.asarray(impl.dense_matmul(kat["dtype"], x, w, N, K, via), np.float32).reshape(-1)
            assert y.size == N, (kat["name"], via, y.size)
            err = float(np.abs(y.astype(np.float64) - ref.astype(np.float64)).max())
            assert err < kat["tol"], (kat["name"], via, err)
        return True
    if op == "weights_len":
        if not hasattr(impl, "weights_len"):
            return False
        assert impl.weights_len(kat["kind"], kat["data_len"], kat.get("n_scales", 0), kat.get("block_size", 0),
                                kat.get("num_elements", kat["data_len"])) == kat["expect"]
        return True
    if op == "dense_upload":
        if not hasattr(impl, "dense_upload"):
            return False
        vals = np.asarray(kat["values"], np.float32)
        n, nbytes = impl.dense_upload(kat["dtype"], bf16_truncate(vals) if kat["dtype"] == "bf16" else vals)
        assert n == kat["expect_len"] and nbytes == kat["expect_bytes"], (kat["name"], n, nbytes)
        return True
    raise AssertionError(f"unknown KAT op {op}")


def bf16_truncate(v) -> np.ndarray:
    """`(value.to_bits() >> 16) as u16`, the reference tests' f32 -> bf16."""
    return (np.asarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def widen_bf16(bits) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def sequential_matmul(x, w, N: int, K: int) -> np.ndarray:
    """Each row's f32 products summed one after another in f32 (cpu_matmul_f32's iterator sum)."""
    prod = (np.asarray(w, np.float32).reshape(N, K) * np.asarray(x, np.float32)[None, :]).astype(np.float32)
    return np.cumsum(prod, axis=1, dtype=np.float32)[:, -1]


def formula_inputs(kat):
    """x_i = f32(i) % xm / xd - xs, w_i = f32((i*wa + wb) % wm) / wd - ws, each step in f32."""
    N, K = kat["out_features"], kat["in_features"]
    xm, xd, xs = kat["x"]
    wa, wb, wm, wd, ws = kat["w"]
    i = np.arange(K, dtype=np.int64)
    x = np.fmod(i.astype(np.float32), np.float32(xm)) / np.float32(xd) - np.float32(xs)
    j = np.arange(N * K, dtype=np.int64)
    w = ((j * wa + wb) % wm).astype(np.float32) / np.float32(wd) - np.float32(ws)
    return x.astype(np.float32), w.astype(np.float32)
