"""Decode GEMV parity: the CUDA matmul against the oracle's restatement of the reference's
quantized CPU matmul (src/matmul.rs:21-97, :149-173, :297-317) on the same seeded inputs.
Bar: max_i |y_i - ref_i| / max(|ref_i|, 1e-3 max|ref|) <= 1e-3 (tests/parity.py)."""
import numpy as np
import pytest

import oracle
import pyxis_b200 as px
from parity import check_matmul, exact_matmul

pytestmark = pytest.mark.gpu

KIND = {"int8": oracle.INT8, "int4": oracle.INT4}


def make(qt, N, K, bs, seed):
    bits = px.synth_normal_bf16(seed, N * K, 0.02)
    vals = oracle.bf16_to_f32(bits)
    w = px.Weights.quantize_int8(bits, bs) if qt == "int8" else px.Weights.quantize_int4(bits, bs)
    od, os_ = (oracle.quantize_int8 if qt == "int8" else oracle.quantize_int4)(vals, bs)
    return w, od, os_


def ref_matmul(qt, od, os_, bs, X, N, K):
    return oracle.matmul(X, KIND[qt], od, os_, bs, N, K)


# The benchmark shapes: gate_proj int8 per-row (one scale per row, the model's int8 policy), and
# the int4 group-32 sweep (q, kv, gate/up, down).
CONFIG_SHAPES = [
    ("int8", 6144, 2048, 2048),
    ("int4", 2048, 2048, 32),
    ("int4", 1024, 2048, 32),
    ("int4", 6144, 2048, 32),
    ("int4", 2048, 6144, 32),
    ("int8", 2048, 6144, 6144),
    ("int8", 6144, 2048, 32),  # GGUF Q8_0 layout
]


@pytest.mark.parametrize("qt,N,K,bs", CONFIG_SHAPES)
@pytest.mark.parametrize("B", [1, 2, 8])
def test_gemv_matches_oracle(qt, N, K, bs, B):
    w, od, os_ = make(qt, N, K, bs, seed=N * 7 + K + bs)
    X = px.synth_normal_f32(1000 + B, B * K, 1.0).reshape(B, K)
    ref = ref_matmul(qt, od, os_, bs, X, N, K)
    Y = px.matmul_batch(X, w, N, K)
    assert Y.shape == (B, N)
    check_matmul(Y, ref, exact_matmul(qt, od, os_, bs, N, K, X))


def test_lm_head_int8_full_size():
    """lm_head 151936 x 2048, int8 per-row quantised copy of the tied embedding (src/model.rs:219-224)."""
    N, K = 151936, 2048
    w, od, os_ = make("int8", N, K, K, seed=0x11EAD)
    x = px.synth_normal_f32(5, K, 1.0)
    ref = ref_matmul("int8", od, os_, K, x, N, K)
    y = px.matmul(x, w, N, K)
    check_matmul(y, ref, exact_matmul("int8", od, os_, K, N, K, x)[0])
    assert px.argmax(y) == oracle.argmax(ref)


@pytest.mark.parametrize("qt,N,K,bs", [
    ("int8", 2, 3, 3), ("int4", 2, 3, 4),          # the reference's own matmul tests (odd K, straddling blocks)
    ("int8", 1, 1, 1), ("int4", 1, 1, 32), ("int4", 5, 7, 3), ("int8", 17, 100, 7),
    ("int4", 33, 96, 32), ("int8", 100, 48, 16), ("int4", 64, 64, 64), ("int4", 300, 4096, 4096),
    ("int8", 129, 8192, 8192), ("int4", 3, 1024 * 9, 32), ("int8", 7, 160, 32), ("int4", 31, 32 * 5, 160),
])
@pytest.mark.parametrize("B", [1, 3])
def test_gemv_odd_shapes(qt, N, K, bs, B):
    w, od, os_ = make(qt, N, K, bs, seed=N + 31 * K + bs)
    X = px.synth_normal_f32(77 + B, B * K, 1.0).reshape(B, K)
    ref = ref_matmul(qt, od, os_, bs, X, N, K)
    Y = px.matmul_batch(X, w, N, K)
    check_matmul(Y, ref, exact_matmul(qt, od, os_, bs, N, K, X))


def test_matmul_rejects_shape_mismatch():
    w, _, _ = make("int8", 4, 8, 8, seed=1)
    with pytest.raises(px.PyxisError):
        px.matmul(np.zeros(8, np.float32), w, 5, 8)  # weight.len() != out * in (src/matmul.rs:28)
    with pytest.raises(px.PyxisError):
        px.matmul(np.zeros(7, np.float32), w, 4, 8)  # input.len() != in_features (src/matmul.rs:27)


def test_matmul_dev_strided_rows():
    import torch
    N, K = 2048, 2048
    w, od, os_ = make("int4", N, K, 32, seed=21)
    X = torch.from_numpy(px.synth_normal_f32(3, 4 * (K + 64), 1.0).reshape(4, K + 64)).cuda()[:, :K]
    Y = torch.zeros((4, N + 32), device="cuda")[:, :N]
    px.matmul_dev(X, w, N, K, Y=Y)
    torch.cuda.synchronize()
    Xh = X.cpu().numpy()
    ref = ref_matmul("int4", od, os_, 32, Xh, N, K)
    check_matmul(Y.cpu().numpy(), ref, exact_matmul("int4", od, os_, 32, N, K, Xh))


@pytest.mark.parametrize("qt,bs", [("int4", 32), ("int8", 2048)])
def test_matmul_dev_rows_off_16_byte_boundaries(qt, bs):
    """x rows that start one float into a buffer cannot be fetched by TMA or 16-byte loads: the
    calls take the element-wise kernel (also for M >= 16, 8 rows per launch) with the same
    results."""
    import torch
    N, K = 1024, 2048
    w, od, os_ = make(qt, N, K, bs, seed=23)
    for M in (1, 3, 20):
        base = torch.from_numpy(px.synth_normal_f32(40 + M, M * K + 1, 1.0)).cuda()
        X = base[1:].view(M, K)
        assert X.data_ptr() % 16 != 0
        Y = px.matmul_dev(X, w, N, K)
        torch.cuda.synchronize()
        Xh = X.cpu().numpy()
        check_matmul(Y.cpu().numpy(), ref_matmul(qt, od, os_, bs, Xh, N, K), exact_matmul(qt, od, os_, bs, N, K, Xh))


def test_argmax_rules():
    import torch
    assert px.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert px.argmax([np.nan, 3.0, 2.0]) == 0
    assert px.argmax([1.0, np.nan, 2.0]) == 2
    assert px.argmax([-0.0, 0.0]) == 0
    assert px.argmax([-np.inf, -np.inf]) == 0
    rng = np.random.default_rng(0)
    v = rng.standard_normal((5, 151936)).astype(np.float32)
    v[2, 100] = v[2, 90000] = 50.0  # tie: lowest index
    t = torch.from_numpy(v).cuda()
    idx, val = px.argmax_dev(t, index_base=1000)
    torch.cuda.synchronize()
    for r in range(5):
        assert int(idx[r]) == oracle.argmax(v[r]) + 1000
        assert float(val[r]) == float(v[r].max())
    for _ in range(3):  # the single-launch reduction re-arms its scratch every call
        idx2, _ = px.argmax_dev(t)
        torch.cuda.synchronize()
        assert [int(i) for i in idx2] == [oracle.argmax(v[r]) for r in range(5)]


@pytest.mark.parametrize("N,K,B", [
    (1, 2048, 1), (300, 128, 1), (2048, 2048, 1), (1024, 2048, 3), (6144, 2048, 5), (18000, 2048, 8),
    (4096, 4096, 4), (129, 1024, 8), (151936, 2048, 8),
])
def test_int8_row_scale_tensor_core_gemv(N, K, B):
    """int8 with one scale per row at batch 1-8.  From 16384 output rows (the lm_head and its
    vocab shards on up to 8 GPUs) it runs
    tcgen05 kind::i8 with x as int8 digits and stream-K (tiles shared by two CTAs added with exact
    int32 atomics); below that the mma.sync GEMV from 8 MB of codes (4 MB at 4-8 rows) and the
    CUDA-core batch kernel under it, whichever finishes first at the size."""
    w, od, os_ = make("int8", N, K, K, seed=N + K + B)
    mma = N * K >= (8 << 20) or (N * K >= (4 << 20) and B >= 4)
    assert px.matmul_kernel_name(w, B, N, K) == (
        "gemv_tc_i8_kernel" if N >= 16384 else "gemv_mma_kernel" if mma else "gemv_batch_kernel")
    X = px.synth_normal_f32(B * 31 + 7, B * K, 1.0).reshape(B, K)
    X[0, :5] = [0.0, -0.0, 1e-30, -3e4, 2.5]
    for rep in range(2):  # the split-K scratch must be left clean for the next launch
        Y = px.matmul_batch(X, w, N, K)
        ref = ref_matmul("int8", od, os_, K, X, N, K)
        check_matmul(Y, ref, exact_matmul("int8", od, os_, K, N, K, X))
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))


@pytest.mark.parametrize("qt,N,K,bs,B", [
    # K % 128 != 0 keeps group-32 batches of 2-8 rows off the weight-streaming matmul
    ("int4", 2048, 2016, 32, 2), ("int4", 2048, 2016, 32, 5), ("int4", 2048, 6112, 32, 7),
    ("int4", 64, 12256, 32, 2),    # two TMA boxes per token
    ("int4", 10, 9632, 32, 2),     # 301 rows of x: boxes of 152 rows, the last one overhangs
    ("int4", 100, 416, 32, 3),     # 13 rows of x in a 16-row box
    ("int4", 40000, 2016, 32, 4),  # many row-group items per CTA (double-buffered combine)
    ("int4", 1779, 2048, 64, 6),   # N % 4 != 0, 64-value groups (2 chunks per scale)
    ("int8", 6144, 2016, 32, 8),   # GGUF Q8_0 layout at batch 8
    ("int8", 515, 4096, 128, 3),
    ("int4", 300, 4096, 4096, 8),  # int4 with one scale per row
])
def test_batch_kernel(qt, N, K, bs, B):
    """The CUDA-core batch kernel (x staged by TMA, split-K over warps, fixed-order combine): the
    products of 1-8 rows that the mma.sync GEMV does not take (matrices under 4 MB, K not a
    multiple of its weight boxes, scale blocks other than 32 or the whole row)."""
    w, od, os_ = make(qt, N, K, bs, seed=N + 3 * K + bs + B)
    assert px.matmul_kernel_name(w, B, N, K) == "gemv_batch_kernel"
    X = px.synth_normal_f32(B * 13 + 1, B * K, 1.0).reshape(B, K)
    X[B - 1, :4] = [0.0, -0.0, 1e-30, -3e4]
    ref = ref_matmul(qt, od, os_, bs, X, N, K)
    Y1 = px.matmul_batch(X, w, N, K)
    check_matmul(Y1, ref, exact_matmul(qt, od, os_, bs, N, K, X))
    Y2 = px.matmul_batch(X, w, N, K)
    assert np.array_equal(Y1, Y2)  # the combine order is fixed: bit-identical reruns
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))


@pytest.mark.parametrize("qt,N,K,bs,B", [
    ("int4", 6144, 2048, 32, 4), ("int4", 6144, 2048, 32, 5), ("int4", 6144, 2048, 32, 8),
    ("int4", 4100, 2048, 32, 8),    # last row tile partly outside the matrix
    ("int4", 2048, 6144, 32, 8),    # down_proj: 8 K parts of 3 boxes
    ("int4", 700, 12288, 32, 7),    # 8 parts of 6 boxes (the most shared memory)
    ("int4", 32768, 256, 32, 4),    # one box: a single K part, no cluster
    ("int4", 2100, 4096, 4096, 8),  # int4 with one scale per row
    ("int8", 6144, 2048, 2048, 1),  # int8 per row at batch 1
    ("int8", 4100, 2048, 2048, 3),  # int8 per row, partial tile
    ("int8", 4100, 2048, 32, 6),    # GGUF Q8_0 layout
    ("int4", 40000, 2048, 32, 8),   # many row tiles
])
def test_mma_kernel(qt, N, K, bs, B):
    """The mma.sync GEMV (codes from registers into m16n8k16 with x as fp16 hi / lo, K parts added
    in rank order through the cluster's shared memory) against the oracle and the exact sum, with
    zeros, a tiny and an outlying x; reruns are bit-identical."""
    w, od, os_ = make(qt, N, K, bs, seed=N + 5 * K + bs + B)
    assert px.matmul_kernel_name(w, B, N, K) == "gemv_mma_kernel"
    X = px.synth_normal_f32(B * 17 + 3, B * K, 1.0).reshape(B, K)
    X[0, :4] = [0.0, -0.0, 1e-30, -3e4]
    ref = ref_matmul(qt, od, os_, bs, X, N, K)
    Y1 = px.matmul_batch(X, w, N, K)
    check_matmul(Y1, ref, exact_matmul(qt, od, os_, bs, N, K, X))
    Y2 = px.matmul_batch(X, w, N, K)
    assert np.array_equal(Y1, Y2)
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))


def test_host_calls_from_several_threads():
    """pyxis_cuda_matmul from four host threads on one context: the calls share its staging
    buffers and serialise on its lock, so every thread gets its own product, bit for bit the
    single-threaded result (the kernels reduce in a fixed order)."""
    import threading
    jobs = []
    for t in range(4):
        N, K = 1024 + 512 * t, 2048
        w, od, os_ = make("int4", N, K, 32, seed=300 + t)
        x = px.synth_normal_f32(400 + t, K, 1.0)
        y0 = px.matmul(x, w, N, K)
        check_matmul(y0[None], ref_matmul("int4", od, os_, 32, x[None], N, K), exact_matmul("int4", od, os_, 32, N, K, x[None]))
        jobs.append((w, x, y0, N, K))
    bad = []

    def run(i):
        w, x, y0, N, K = jobs[i]
        for _ in range(200):
            y = px.matmul(x, w, N, K)
            if y.shape != y0.shape or not np.array_equal(y.view(np.uint32), y0.view(np.uint32)):
                bad.append(i)
                return

    threads = [threading.Thread(target=run, args=(i,)) for i in range(len(jobs))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not bad, bad


@pytest.mark.parametrize("qt,N,K,bs,B", [
    ("int4", 2048, 2048, 32, 1),      # batch GEMV
    ("int4", 1024, 2048, 32, 8),      # batch GEMV, 8 rows
    ("int4", 6144, 2048, 32, 8),      # mma GEMV
    ("int8", 33000, 2048, 2048, 1),   # tensor-core GEMV
    ("int8", 33000, 2048, 2048, 8),
    ("int4", 5, 7, 3, 3),             # generic GEMV
    ("int4", 2048, 2048, 32, 16),     # weight-streaming matmul: keeps the copy
    ("int8", 512, 1024, 1024, 80),    # prefill GEMM: keeps the copy
])
def test_host_call_into_page_locked_output(qt, N, K, bs, B):
    """pyxis_cuda_matmul_batch with a page-locked output: the GEMV kernels store into it
    directly (torch pinned memory, cudaHostRegister'ed numpy memory, and an output that starts
    4 bytes past an allocation's start), the tensor-core products copy into it; each gives the
    pageable-output result bit for bit, and that result matches the oracle."""
    import ctypes as C
    import torch
    w, od, os_ = make(qt, N, K, bs, seed=N + 3 * K + B)
    X = px.synth_normal_f32(900 + B, B * K, 1.0).reshape(B, K)
    X[0, :2] = [-3e4, -0.0]
    Y0 = px.matmul_batch(X, w, N, K)
    check_matmul(Y0, ref_matmul(qt, od, os_, bs, X, N, K), exact_matmul(qt, od, os_, bs, N, K, X))
    L = px._native.lib()
    xp = torch.from_numpy(X).pin_memory()

    def run(out_ptr):
        px._native.check(L.pyxis_cuda_matmul_batch(w.ctx.handle, C.c_void_p(xp.data_ptr()), B, w.handle, N, K,
                                                   C.c_void_p(out_ptr)))

    pinned = torch.full((B * N + 1,), float("nan"), dtype=torch.float32).pin_memory()
    for off in (0, 1):
        pinned.fill_(float("nan"))
        run(pinned.data_ptr() + 4 * off)
        got = pinned[off:off + B * N].numpy().reshape(B, N)
        assert np.array_equal(got.view(np.uint32), Y0.view(np.uint32)), off
        assert np.isnan(pinned[1 - off if off else B * N].item())  # nothing stored past the output
    reg = np.full((B, N), np.nan, dtype=np.float32)
    cr = torch.cuda.cudart()
    assert int(cr.cudaHostRegister(reg.ctypes.data, reg.nbytes, 0)) == 0
    try:
        run(reg.ctypes.data)
    finally:
        assert int(cr.cudaHostUnregister(reg.ctypes.data)) == 0
    assert np.array_equal(reg.view(np.uint32), Y0.view(np.uint32))
    px._native.check(L.pyxis_cuda_check_device_error(w.ctx.handle))
