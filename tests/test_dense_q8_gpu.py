"""Weights the reference handles outside its two quantizers:

  * GGUF Q8_0 tensors (read_q8_0_weights, src/gguf.rs:245-271) unpacked on the device by
    pyxis_cuda_weights_upload_q8_0: codes and f32 scale bit patterns identical to the oracle's
    restatement, the scales widened from f16 as half 2.7.1 does (NaN payloads quieted);
  * unquantized rows, Weights::F32 and Weights::Bf16 (src/matmul.rs:99-125, :284-295, the
    arms the Metal backend serves as MetalF32 / MetalBf16), through the same matmul entry points.

Matmul parity is the 1e-3 bar of tests/parity.py against the oracle and the float64 sum."""
import numpy as np
import pytest
import torch

import oracle
import pyxis_b200 as px
from parity import check_matmul, exact_matmul

pytestmark = pytest.mark.gpu

# f16 bit patterns the widening must get right: signed zeros, the smallest and largest
# subnormals, the smallest normal, 1, the largest finite, infinities, signalling and quiet NaNs.
SPECIAL_F16 = np.array([0x0000, 0x8000, 0x0001, 0x8001, 0x03FF, 0x83FF, 0x0400, 0x3C00, 0x7BFF, 0xFBFF,
                        0x7C00, 0xFC00, 0x7C01, 0x7DFF, 0x7E00, 0xFE01, 0xFFFF, 0x3555, 0x2E66], np.uint16)


def _q8_0_blob(rng, n, special=True):
    nb = -(-n // 32)
    scales = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint16)
    if special:
        k = min(nb, SPECIAL_F16.size)
        scales[rng.choice(nb, size=k, replace=False)] = SPECIAL_F16[:k]
    blob = np.empty((nb, 34), np.uint8)
    blob[:, 0:2] = scales.astype("<u2").view(np.uint8).reshape(nb, 2)
    blob[:, 2:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    return blob.tobytes()


@pytest.mark.parametrize("n", [1, 31, 32, 33, 40, 1000, 32 * 4097 + 5, 2048 * 6144])
def test_q8_0_unpack_bit_exact(n):
    rng = np.random.default_rng(n)
    blob = _q8_0_blob(rng, n)
    w = px.Weights.from_q8_0(blob, n)
    assert w.qtype == "int8" and w.block_size == 32 and w.len() == n and w.num_scales == -(-n // 32)
    d, s = w.download()
    od, os_ = oracle.q8_0_to_int8(blob, n)
    assert np.array_equal(d.view(np.uint8), od.view(np.uint8))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))


def test_q8_0_reference_example():
    """tests/gguf.rs:75-108: 40 elements in two blocks (scales 0.25 and 0.5)."""
    blob = bytearray(np.float16(0.25).tobytes()) + bytes(range(32))
    blob += bytearray(np.float16(0.5).tobytes()) + bytes(np.arange(-16, 16, dtype=np.int8).view(np.uint8))
    w = px.Weights.from_q8_0(bytes(blob), 40)
    d, s = w.download()
    assert list(d) == list(range(32)) + list(range(-16, -8))
    assert list(s) == [0.25, 0.5]


def test_q8_0_from_device_memory_at_odd_offsets():
    """Blocks already in HBM (a mapped GGUF file copied up whole): 34-byte blocks start at any
    2-byte boundary, and a tensor inside a file can start at an odd byte."""
    rng = np.random.default_rng(7)
    n = 32 * 1000 + 9
    blob = _q8_0_blob(rng, n)
    host = np.frombuffer(blob, np.uint8)
    dev = torch.zeros(host.size + 1, dtype=torch.uint8, device="cuda")
    dev[1:] = torch.from_numpy(host.copy()).cuda()
    w = px.Weights.from_q8_0(dev[1:], n)
    d, s = w.download()
    od, os_ = oracle.q8_0_to_int8(blob, n)
    assert np.array_equal(d.view(np.uint8), od.view(np.uint8))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))


def test_q8_0_short_tensor_is_rejected():
    blob = _q8_0_blob(np.random.default_rng(1), 64)
    with pytest.raises(px.PyxisError):
        px.Weights.from_q8_0(blob[:-1], 64)


@pytest.mark.parametrize("N,K,M", [(2048, 2048, 1), (1024, 2048, 4), (6144, 2048, 64), (96, 100, 2)])
def test_q8_0_matmul_parity(N, K, M):
    rng = np.random.default_rng(N + K + M)
    blob = _q8_0_blob(rng, N * K, special=False)
    w = px.Weights.from_q8_0(blob, N * K)
    od, os_ = oracle.q8_0_to_int8(blob, N * K)
    X = rng.standard_normal((M, K)).astype(np.float32)
    y = px.matmul(X[0], w, N, K)[None] if M == 1 else px.matmul_batch(X, w, N, K)
    ref = oracle.matmul(X, oracle.INT8, od, os_, 32, N, K)
    check_matmul(y, ref, exact_matmul("int8", od, os_, 32, N, K, X))


def _bf16_bits(v):
    """f32 -> bf16 bits, round to nearest even (checkpoint-like rows)."""
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _dense(rng, dtype, N, K):
    v = (rng.standard_normal(N * K) * 0.02).astype(np.float32)
    if dtype == "f32":
        return px.Weights.from_dense(v), oracle.F32, v, v
    bits = _bf16_bits(v)
    return px.Weights.from_dense(bits), oracle.BF16, bits, oracle.bf16_to_f32(bits)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("N,K", [(1, 32), (7, 96), (2048, 2048), (6144, 2048), (2048, 6144), (33, 100), (5, 3)])
@pytest.mark.parametrize("M", [1, 3, 8, 17])
def test_dense_matmul_parity(dtype, N, K, M):
    rng = np.random.default_rng(N * 7 + K + M)
    w, kind, data, wf = _dense(rng, dtype, N, K)
    assert w.qtype == dtype and w.len() == N * K and w.num_scales == 0
    X = rng.standard_normal((M, K)).astype(np.float32)
    y = px.matmul(X[0], w, N, K)[None] if M == 1 else px.matmul_batch(X, w, N, K)
    ref = oracle.matmul(X, kind, data, None, 1, N, K)
    exact = X.astype(np.float64) @ wf.astype(np.float64).reshape(N, K).T
    check_matmul(y, ref, exact)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_dense_device_path_and_kernels(dtype):
    """matmul_dev on device buffers: the batch GEMV for K % 32 == 0 (any M, 8 rows per launch),
    the generic kernel otherwise; never the tensor-core GEMM (it takes quantized rows only)."""
    rng = np.random.default_rng(3)
    N, K, M = 1024, 2048, 40
    w, kind, data, wf = _dense(rng, dtype, N, K)
    assert px.matmul_kernel_name(w, 1, N, K) == "gemv_batch_kernel"
    assert px.matmul_kernel_name(w, M, N, K) == "gemv_batch_kernel"
    X = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    Y = px.matmul_dev(X, w, N, K)
    torch.cuda.synchronize()
    Xh = X.cpu().numpy()
    check_matmul(Y.cpu().numpy(), oracle.matmul(Xh, kind, data, None, 1, N, K),
                 Xh.astype(np.float64) @ wf.astype(np.float64).reshape(N, K).T)
    w2, *_ = _dense(rng, dtype, 8, 100)
    assert px.matmul_kernel_name(w2, 1, 8, 100) == "gemv_generic_kernel"


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_dense_download_round_trip(dtype):
    rng = np.random.default_rng(11)
    w, kind, data, wf = _dense(rng, dtype, 3, 77)
    d, s = w.download()
    assert s.size == 0 and w.block_size == 0
    assert np.array_equal(d.view(np.uint8), np.asarray(data).view(np.uint8))


def test_dense_shape_assert():
    """matmul's weight.len() == out_features * in_features assert (src/matmul.rs:28)."""
    w = px.Weights.from_dense(np.zeros(64, np.float32))
    with pytest.raises(px.PyxisError):
        px.matmul(np.zeros(8, np.float32), w, 9, 8)


def test_q8_0_device_blocks_written_just_before_the_call():
    """Device blocks that torch's stream is still copying when the upload is called (the copy is
    queued behind other work) are unpacked from their final bytes."""
    rng = np.random.default_rng(9)
    n = 2048 * 2048
    blob = _q8_0_blob(rng, n)
    staged = torch.from_numpy(np.frombuffer(blob, np.uint8).copy()).cuda()
    dev = torch.zeros_like(staged)
    torch.cuda.synchronize()
    a = torch.full((4096, 4096), 1e-3, device="cuda")
    for _ in range(8):  # tens of milliseconds of f32 GEMMs ahead of the copy
        a = a @ a
    dev.copy_(staged)
    w = px.Weights.from_q8_0(dev, n)
    d, s = w.download()
    od, os_ = oracle.q8_0_to_int8(blob, n)
    assert np.array_equal(d.view(np.uint8), od.view(np.uint8))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))
