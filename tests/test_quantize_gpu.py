"""On-device quantise + pack, bit-exact with the reference quantizer (src/weights.rs:94-151) as
restated by the oracle.  Packed bytes and f32 scale bit patterns must be identical."""
import numpy as np
import pytest

import oracle
import pyxis_b200 as px
from kat_check import run_kat
from parity import load_kats, tie_blocks

pytestmark = pytest.mark.gpu


class CudaImpl:
    def quantize(self, qt, src, bs):
        w = px.Weights.quantize_int8(src, bs) if qt == "int8" else px.Weights.quantize_int4(src, bs)
        return w.download()

    def quantized_matmul(self, qt, wv, bs, x, N, K):
        w = px.Weights.quantize_int8(wv, bs) if qt == "int8" else px.Weights.quantize_int4(wv, bs)
        return px.matmul(x, w, N, K)

    def q8_0(self, blob, n):
        return px.Weights.from_q8_0(blob, n).download()  # unpacked and widened on the device

    def matmul_f32(self, x, w, N, K):
        return px.matmul(x, px.Weights.from_dense(w), N, K)

    def matmul_bf16(self, x, bits, N, K):
        return px.matmul(x, px.Weights.from_dense(bits), N, K)

    def dense_matmul(self, dtype, x, w, N, K, via):
        wd = px.Weights.from_dense(w)  # np.uint16 bits -> Bf16 rows, np.float32 -> F32 rows
        assert wd.qtype == dtype
        if via == "host":
            return px.matmul(x, wd, N, K)
        import torch
        y = px.matmul_dev(torch.from_numpy(np.ascontiguousarray(x)).cuda().view(1, K), wd, N, K)
        return y.cpu().numpy()

    def weights_len(self, kind, data_len, n_scales, block_size, num_elements):
        if kind in ("f32", "bf16"):
            w = px.Weights.from_dense(np.zeros(data_len, np.float32 if kind == "f32" else np.uint16))
        else:
            w = px.Weights.from_packed(kind, np.zeros(data_len, np.uint8), np.ones(n_scales, np.float32),
                                       block_size, num_elements)
        return w.len()

    def dense_upload(self, dtype, values):
        w = px.Weights.from_dense(values)
        assert w.qtype == dtype
        return w.len(), w.data_bytes

    def argmax(self, v):
        return px.argmax(v)

    # the decode step's row operations, through the device helpers the decode kernels use
    # (pyxis_cuda_row_op)
    def _row_op(self, op, x, w=None, eps=0.0, head_dim=0, pos=0, theta=0.0):
        import ctypes as C
        x = np.ascontiguousarray(np.asarray(x, np.float32))
        wv = None if w is None else np.ascontiguousarray(np.asarray(w, np.float32))
        out = np.empty_like(x)
        ctx = px.get_cuda(0)
        px._native.check(px._native.lib().pyxis_cuda_row_op(
            ctx.handle, op, x.ctypes.data_as(C.c_void_p), x.size,
            None if wv is None else wv.ctypes.data_as(C.c_void_p), eps, head_dim, pos, theta,
            out.ctypes.data_as(C.c_void_p)))
        return out

    def rmsnorm(self, x, w, eps):
        return self._row_op(1, x, w=w, eps=eps)

    def rope(self, x, head_dim, pos, theta):
        return self._row_op(2, x, head_dim=head_dim, pos=pos, theta=theta)

    def silu(self, x):
        return float(self._row_op(3, [x])[0])


@pytest.mark.parametrize("kat", load_kats(), ids=lambda k: k["name"])
def test_cuda_reference_kat(kat):
    if not run_kat(kat, CudaImpl()):
        pytest.skip("op not on the CUDA path")


def _bits(a):
    return np.asarray(a).view(np.uint32)


def _oracle_pack(qt, vals, bs):
    return oracle.quantize_int8(vals, bs) if qt == "int8" else oracle.quantize_int4(vals, bs)


@pytest.mark.parametrize("qt", ["int8", "int4"])
@pytest.mark.parametrize("n,bs", [(1, 1), (2, 32), (3, 2), (5, 4), (31, 32), (33, 32), (1001, 7), (4096, 64),
                                  (2048 * 64, 2048), (6144 * 8, 6144), (100_003, 100_003), (300_000, 70_000),
                                  (65 * 1024, 65 * 1024 + 3)])
def test_quantize_bit_exact_f32(qt, n, bs):
    rng = np.random.default_rng(n + bs)
    v = (rng.standard_normal(n) * 0.02).astype(np.float32)
    v[rng.integers(0, n, size=max(1, n // 97))] = 0.0
    w = px.Weights.quantize_int8(v, bs) if qt == "int8" else px.Weights.quantize_int4(v, bs)
    d, s = w.download()
    od, os_ = _oracle_pack(qt, v, bs)
    assert np.array_equal(d.view(np.uint8), od.view(np.uint8))
    assert np.array_equal(_bits(s), _bits(os_))
    assert w.len() == n and w.num_scales == -(-n // bs)


@pytest.mark.parametrize("qt,bs", [("int8", 2048), ("int4", 32), ("int8", 32)])
def test_quantize_bit_exact_bf16_config_shape(qt, bs):
    """gate_proj 6144 x 2048: bf16 N(0, 0.02) weights, widened with << 16 then quantised."""
    bits = px.synth_normal_bf16(0x6A7E, 6144 * 2048, 0.02)
    w = px.Weights.quantize_int8(bits, bs) if qt == "int8" else px.Weights.quantize_int4(bits, bs)
    d, s = w.download()
    od, os_ = _oracle_pack(qt, oracle.bf16_to_f32(bits), bs)
    assert np.array_equal(d.view(np.uint8), od.view(np.uint8))
    assert np.array_equal(_bits(s), _bits(os_))


def test_quantize_from_device_tensor():
    import torch
    bits = px.synth_normal_bf16(11, 1024 * 512, 0.02)
    t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    w = px.Weights.quantize_int4(t, 32)
    d, s = w.download()
    od, os_ = oracle.quantize_int4(oracle.bf16_to_f32(bits), 32)
    assert np.array_equal(d, od) and np.array_equal(_bits(s), _bits(os_))
    tf = torch.from_numpy(oracle.bf16_to_f32(bits)).cuda()
    w2 = px.Weights.quantize_int8(tf, 512)
    d2, s2 = w2.download()
    od2, os2 = oracle.quantize_int8(oracle.bf16_to_f32(bits), 512)
    assert np.array_equal(d2, od2) and np.array_equal(_bits(s2), _bits(os2))


@pytest.mark.parametrize("qt", ["int8", "int4"])
def test_quantize_special_values(qt):
    v = np.array([np.nan, 1.0, -np.inf, 0.5, -0.0, 3e-39, np.inf, np.nan, 0.0, 1e38, -1e38, 2.5, -2.5, 7.0],
                 np.float32)
    for bs in (1, 2, 3, 5, 14, 100):
        w = px.Weights.quantize_int8(v, bs) if qt == "int8" else px.Weights.quantize_int4(v, bs)
        d, s = w.download()
        od, os_ = _oracle_pack(qt, v, bs)
        assert np.array_equal(d.view(np.uint8), od.view(np.uint8)), (bs, d, od)
        assert np.array_equal(_bits(s), _bits(os_)), (bs, s, os_)


def test_quantize_rejects_zero_block():
    with pytest.raises(px.PyxisError):
        px.Weights.quantize_int8(np.ones(4, np.float32), 0)


def test_upload_download_round_trip():
    rng = np.random.default_rng(3)
    data = rng.integers(0, 256, size=999, dtype=np.uint8)
    scales = rng.standard_normal(63).astype(np.float32)
    w = px.Weights.from_packed("int4", data, scales, 32, 1998)
    d, s = w.download()
    assert np.array_equal(d, data) and np.array_equal(s, scales)


def test_device_source_must_be_this_devices_memory():
    """A host pointer flagged as a device source is refused on the host, before any launch."""
    import ctypes as C
    from pyxis_b200 import _native
    ctx = px.get_cuda(0)
    v = np.ones(1024, np.float32)
    h = C.c_void_p()
    rc = _native.lib().pyxis_cuda_quantize(ctx.handle, v.ctypes.data_as(C.c_void_p), _native.DTYPE_F32, 1, v.size,
                                           32, _native.QTYPE_INT8, C.byref(h))
    assert rc == _native.PYXIS_EINVAL
    assert b"device" in _native.lib().pyxis_cuda_last_error()


def _queue_torch_work(torch):
    """Tens of milliseconds of f32 GEMMs queued on torch's current stream."""
    a = torch.full((4096, 4096), 1e-3, device="cuda")
    for _ in range(8):
        a = a @ a
    return a


def test_device_source_written_just_before_the_call():
    """The library packs on its own non-blocking stream.  A source that torch's stream is still
    writing when the call is made (a copy queued behind other work, read through a strided view
    whose contiguous copy is queued too) must be packed from its final values."""
    import torch
    N, K = 1024, 2048
    bits = px.synth_normal_bf16(13, 2 * N * K, 0.02)
    vals = oracle.bf16_to_f32(bits).reshape(2 * N, K)
    staged = torch.from_numpy(vals).cuda()
    src = torch.zeros_like(staged)
    torch.cuda.synchronize()
    _queue_torch_work(torch)
    src.copy_(staged)
    w = px.Weights.quantize_int4(src[::2], 32)
    d, s = w.download()
    od, os_ = oracle.quantize_int4(np.ascontiguousarray(vals[::2]).reshape(-1), 32)
    assert np.array_equal(d, od) and np.array_equal(_bits(s), _bits(os_))


@pytest.mark.parametrize("qt", ["int8", "int4"])
def test_quantize_rounds_ties_away_from_zero(qt):
    """Blocks whose scale is exactly 1: every code is f32::round of its value (ties away from
    zero, 0.49999997 -> 0), as the oracle's roundf gives."""
    amax = 127.0 if qt == "int8" else 7.0
    v = tie_blocks(amax, 16)
    w = px.Weights.quantize_int8(v, 16) if qt == "int8" else px.Weights.quantize_int4(v, 16)
    d, s = w.download()
    od, os_ = (oracle.quantize_int8 if qt == "int8" else oracle.quantize_int4)(v, 16)
    assert np.array_equal(_bits(s), _bits(os_)) and np.all(s == 1.0)
    assert np.array_equal(np.asarray(d).view(np.uint8), np.asarray(od).view(np.uint8))
