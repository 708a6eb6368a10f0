"""The oracle (C restatement of the reference CPU path) against the reference's own known-answer
tests, and against an independent numpy restatement on seeded random inputs.  CPU only."""
import numpy as np
import pytest

import oracle
from kat_check import run_kat
from parity import load_kats, tie_blocks


class OracleImpl:
    def quantize(self, qt, src, bs):
        vals = oracle.bf16_to_f32(src) if src.dtype == np.uint16 else src
        return oracle.quantize_int8(vals, bs) if qt == "int8" else oracle.quantize_int4(vals, bs)

    def quantized_matmul(self, qt, w, bs, x, N, K):
        data, scales = self.quantize(qt, w, bs)
        return oracle.matmul(x, oracle.INT8 if qt == "int8" else oracle.INT4, data, scales, bs, N, K)

    def q8_0(self, blob, n):
        return oracle.q8_0_to_int8(blob, n)

    def argmax(self, v):
        return oracle.argmax(v)

    def matmul_f32(self, x, w, N, K):
        return oracle.matmul(x, oracle.F32, w, None, 1, N, K)

    def matmul_bf16(self, x, bits, N, K):
        return oracle.matmul(x, oracle.BF16, bits, None, 1, N, K)

    def dense_matmul(self, dtype, x, w, N, K, via):  # one CPU path: `via` names the GPU's entry points
        return self.matmul_bf16(x, w, N, K) if dtype == "bf16" else self.matmul_f32(x, w, N, K)

    def rmsnorm(self, x, w, eps):
        return oracle.rmsnorm(x, w, eps)

    def rope(self, x, hd, pos, theta):
        return oracle.apply_rope(x, hd, pos, theta)

    def silu(self, x):
        return oracle.silu(x)


@pytest.mark.parametrize("kat", load_kats(), ids=lambda k: k["name"])
def test_oracle_reference_kat(kat):
    if kat["op"] in ("weights_len", "dense_upload"):  # properties of a device weights handle
        pytest.skip("device weights handle: checked on the CUDA path")
    assert run_kat(kat, OracleImpl())


# ---- an independent numpy restatement of src/weights.rs:94-151 ----------------------------------
def round_half_away(t):
    """f32::round: nearest integer, ties away from zero.  t - trunc(t) is exact in f32, so the tie
    test is exact (floor(|t| + 0.5) is not: 0.49999997 + 0.5 rounds up to 1.0)."""
    t = np.asarray(t, np.float32)
    tr = np.trunc(t)
    with np.errstate(invalid="ignore"):
        frac = np.abs(t - tr)
        return (tr + np.sign(t) * (frac >= np.float32(0.5))).astype(np.float32)


def np_quantize_int8(v, bs):
    v = np.asarray(v, np.float32)
    n = v.size
    nb = -(-n // bs)
    pad = np.zeros(nb * bs, np.float32)
    pad[:n] = np.abs(v)
    absmax = np.nanmax(np.where(np.isnan(pad), 0, pad).reshape(nb, bs), axis=1).astype(np.float32)
    scales = np.where(absmax == 0, np.float32(1.0), absmax / np.float32(127.0)).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        t = (v / np.repeat(scales, bs)[:n]).astype(np.float32)
    r = np.clip(round_half_away(t), -127, 127)
    r = np.where(np.isnan(r), 0, r)
    return r.astype(np.int8), scales


def np_quantize_int4(v, bs):
    v = np.asarray(v, np.float32)
    n = v.size
    nb = -(-n // bs)
    pad = np.zeros(nb * bs, np.float32)
    pad[:n] = np.abs(v)
    absmax = np.max(np.where(np.isnan(pad), 0, pad).reshape(nb, bs), axis=1).astype(np.float32)
    scales = np.where(absmax == 0, np.float32(1.0), absmax / np.float32(7.0)).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        t = (v / np.repeat(scales, bs)[:n]).astype(np.float32)
    r = np.clip(round_half_away(t), -8, 7)
    r = np.where(np.isnan(r), 0, r).astype(np.int64) + 8
    codes = np.full(2 * (-(-n // 2)), 8, np.int64)
    codes[:n] = r
    data = (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8)
    return data, scales


SHAPES = [(1, 1), (3, 2), (7, 5), (33, 3), (64, 32), (257, 100), (4096, 2048), (1000, 7)]


@pytest.mark.parametrize("n,bs", SHAPES)
def test_oracle_quantizers_match_numpy_restatement(n, bs):
    rng = np.random.default_rng(n * 131 + bs)
    v = (rng.standard_normal(n) * 0.02).astype(np.float32)
    v[rng.integers(0, n, size=max(1, n // 50))] = 0.0
    d8, s8 = oracle.quantize_int8(v, bs)
    e8, f8 = np_quantize_int8(v, bs)
    assert np.array_equal(d8, e8) and np.array_equal(s8.view(np.uint32), f8.view(np.uint32))
    d4, s4 = oracle.quantize_int4(v, bs)
    e4, f4 = np_quantize_int4(v, bs)
    assert np.array_equal(d4, e4) and np.array_equal(s4.view(np.uint32), f4.view(np.uint32))


def test_oracle_quantizer_special_values():
    v = np.array([np.nan, 1.0, -np.inf, 0.5, -0.0, 3e-39, np.inf, np.nan, 0.0], np.float32)
    for bs in (1, 2, 3, 9):
        d8, s8 = oracle.quantize_int8(v, bs)
        e8, f8 = np_quantize_int8(v, bs)
        assert np.array_equal(d8, e8), (bs, d8, e8)
        assert np.array_equal(s8.view(np.uint32), f8.view(np.uint32))
        d4, s4 = oracle.quantize_int4(v, bs)
        e4, f4 = np_quantize_int4(v, bs)
        assert np.array_equal(d4, e4), (bs, d4, e4)


def test_oracle_matmul_is_sequential_f32():
    """dot_product_int8_scalar / dot_product_int4 keep the reference's left-to-right f32 order."""
    rng = np.random.default_rng(5)
    N, K = 64, 96
    w = (rng.standard_normal(N * K) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    for qt, kind, q in (("int8", oracle.INT8, oracle.quantize_int8), ("int4", oracle.INT4, oracle.quantize_int4)):
        for bs in (K, 32, 5):
            data, scales = q(w, bs)
            y = oracle.matmul(x, kind, data, scales, bs, N, K, nthreads=3)
            deq = oracle.dequantize(kind, data, scales, bs, N * K).reshape(N, K)
            ref = np.empty(N, np.float32)
            for n in range(N):
                acc = np.float32(-0.0) if qt == "int8" else np.float32(0.0)
                for i in range(K):
                    g = n * K + i
                    if qt == "int8":
                        qv = np.float32(data[g])
                    else:
                        byte = int(data[g // 2])
                        qv = np.float32(((byte & 15) if g % 2 == 0 else (byte >> 4)) - 8)
                    acc = np.float32(acc + np.float32(np.float32(x[i] * qv) * scales[g // bs]))
                ref[n] = acc
            assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), (qt, bs)
            assert np.allclose(deq @ x, y, atol=1e-4)


def test_oracle_matmul_threads_do_not_change_results():
    rng = np.random.default_rng(9)
    N, K = 777, 256
    w = (rng.standard_normal(N * K) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    data, scales = oracle.quantize_int4(w, 32)
    y1 = oracle.matmul(x, oracle.INT4, data, scales, 32, N, K, nthreads=1)
    y8 = oracle.matmul(x, oracle.INT4, data, scales, 32, N, K, nthreads=8)
    assert np.array_equal(y1, y8)


def test_oracle_argmax_first_max_and_nan_rules():
    assert oracle.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert oracle.argmax([np.nan, 3.0, 2.0]) == 0  # values[0] NaN: nothing is > NaN
    assert oracle.argmax([1.0, np.nan, 2.0]) == 2
    assert oracle.argmax([-0.0, 0.0]) == 0
    assert oracle.argmax([-np.inf, -np.inf]) == 0


def test_exact_matmul_helper_agrees_with_oracle():
    """tests/parity.py's float64 reference sum stays within f32 rounding of the oracle."""
    from parity import exact_matmul, rel_err
    rng = np.random.default_rng(11)
    N, K = 37, 96
    w = (rng.standard_normal(N * K) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, K)).astype(np.float32)
    for qt, q, kind in (("int8", oracle.quantize_int8, oracle.INT8), ("int4", oracle.quantize_int4, oracle.INT4)):
        for bs in (K, 32, 7):
            d, s = q(w, bs)
            ref = oracle.matmul(x, kind, d, s, bs, N, K)
            assert rel_err(exact_matmul(qt, d, s, bs, N, K, x), ref) < 1e-4


def test_oracle_f16_widening_over_every_bit_pattern():
    """Q8_0 scales: half 2.7.1's f16::to_f32 (the x86 F16C instruction widens the same way).
    Finite values and infinities are exact (numpy's widening agrees); a NaN keeps its sign and
    payload and gets the quiet bit."""
    L = oracle.lib()
    h = np.arange(65536, dtype=np.uint32)
    got = np.array([L.oracle_f16_to_f32(int(v)) for v in h], np.float32).view(np.uint32)
    is_nan = ((h >> 10) & 0x1F == 0x1F) & (h & 0x3FF != 0)
    want = h.astype(np.uint16).view(np.float16).astype(np.float32).view(np.uint32).copy()
    want[is_nan] = ((h[is_nan] & 0x8000) << 16) | 0x7FC00000 | ((h[is_nan] & 0x3FF) << 13)
    assert np.array_equal(got, want)


def test_oracle_quantizers_round_ties_away_from_zero():
    """Blocks whose scale is exactly 1, so every value is its own quotient: the codes must be
    f32::round of the value, ties away from zero."""
    for qt, amax, quant, ref in (("int8", 127.0, oracle.quantize_int8, np_quantize_int8),
                                 ("int4", 7.0, oracle.quantize_int4, np_quantize_int4)):
        v = tie_blocks(amax, 16)
        d, s = quant(v, 16)
        e, f = ref(v, 16)
        assert np.all(s == 1.0) and np.array_equal(s.view(np.uint32), f.view(np.uint32))
        assert np.array_equal(np.asarray(d).view(np.uint8), np.asarray(e).view(np.uint8)), qt
        if qt == "int8":
            want = [int(np.sign(x) * np.floor(abs(float(x)) + 0.5)) for x in v]  # float64: exact here
            assert list(np.asarray(d, np.int64)) == want


def test_oracle_quantizers_property():
    """Random lengths, block sizes and values including NaN, infinities, subnormals and signed
    zeros: the oracle and the numpy restatement agree bit for bit."""
    hyp = pytest.importorskip("hypothesis")
    from hypothesis import given, settings, strategies as st

    floats = st.floats(width=32, allow_nan=True, allow_infinity=True, allow_subnormal=True)

    @settings(max_examples=300, deadline=None, derandomize=True, database=None)
    @given(st.lists(floats, min_size=1, max_size=200), st.integers(min_value=1, max_value=70))
    def check(values, bs):
        v = np.asarray(values, np.float32)
        for quant, ref in ((oracle.quantize_int8, np_quantize_int8), (oracle.quantize_int4, np_quantize_int4)):
            with np.errstate(all="ignore"):
                d, s = quant(v, bs)
                e, f = ref(v, bs)
            assert np.array_equal(np.asarray(d).view(np.uint8), np.asarray(e).view(np.uint8))
            assert np.array_equal(s.view(np.uint32), f.view(np.uint32))

    check()
