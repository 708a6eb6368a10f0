"""The weight-streaming tensor-core matmul (gemm_ws.cu) that takes decode-shaped batches of 9-64
token rows: int4 and int8 weights with a scale per 32 values, int8 with one scale per row.
Parity as for every matmul (tests/parity.py): against the oracle's restatement of the
reference's quantized CPU matmul (src/matmul.rs:21-97, :149-173, :297-317) and the float64 sum of
the same quantized products, max_i |y_i - r_i| / max(|r_i|, 1e-3 max|r|) <= 1e-3; plus bit-identical
reruns, special x values, NaN confined to its token, and split and unsplit K on the same shape."""
import ctypes as C

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


def inputs(M, K, seed):
    X = px.synth_normal_f32(seed, M * K, 1.0).reshape(M, K)
    X[M - 1, :5] = [0.0, -0.0, 1e-30, -3e4, 2.5]  # zeros, a subnormal-scale value, an outlier
    return X


@pytest.mark.parametrize("qt,N,K,bs,M", [
    ("int4", 2048, 2048, 32, 9), ("int4", 2048, 2048, 32, 16), ("int4", 2048, 2048, 32, 17),
    ("int4", 2048, 2048, 32, 33), ("int4", 2048, 2048, 32, 64),       # 16 / 32 / 64 token columns
    ("int4", 1024, 2048, 32, 12), ("int4", 6144, 2048, 32, 16), ("int4", 12288, 2048, 32, 64),
    ("int4", 2048, 6144, 32, 10), ("int4", 2048, 6144, 32, 64),       # down_proj: 48 stages per row
    ("int4", 1779, 2048, 32, 13),                                     # a partial last tile
    ("int4", 100, 128, 32, 11),                                       # one stage per row
    ("int4", 37, 9600, 32, 9),                                        # 75 stages, a lone tile
    ("int8", 6144, 2048, 32, 16), ("int8", 515, 4096, 32, 9),         # GGUF Q8_0 layout
    ("int8", 6144, 2048, 2048, 12), ("int8", 2048, 6144, 6144, 64),   # one scale per row
    ("int8", 4096, 2048, 2048, 40),
])
def test_gemm_ws_matches_oracle(qt, N, K, bs, M):
    w, od, os_ = make(qt, N, K, bs, seed=N * 5 + K + bs + M)
    assert px.matmul_kernel_name(w, M, N, K) == "gemm_ws_kernel"
    X = inputs(M, K, seed=M * 17 + K)
    ref = oracle.matmul(X, KIND[qt], od, os_, bs, N, K)
    Y1 = px.matmul_batch(X, w, N, K)
    check_matmul(Y1, ref, exact_matmul(qt, od, os_, bs, N, K, X))
    Y2 = px.matmul_batch(X, w, N, K)
    assert np.array_equal(Y1, Y2)  # partial sums added in a fixed order: bit-identical reruns
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))


def test_gemm_ws_lm_head_int4_batch():
    """The config-5 head: int4 group-32 lm_head 151936 x 2048 for 16 and 64 sequences' rows
    (1187 tiles: several tiles per CTA, K not split), with the argmax of every row."""
    N, K = 151936, 2048
    w, od, os_ = make("int4", N, K, 32, seed=0x11EAD)
    for M in (16, 64):
        X = px.synth_normal_f32(M + 3, M * K, 1.0).reshape(M, K)
        ref = oracle.matmul(X, oracle.INT4, od, os_, 32, N, K).reshape(M, N)
        Y = px.matmul_batch(X, w, N, K)
        check_matmul(Y, ref, exact_matmul("int4", od, os_, 32, N, K, X))
        for m in range(M):
            assert px.argmax(Y[m]) == oracle.argmax(ref[m])


def test_gemm_ws_nan_stays_in_its_token():
    """A NaN in one token row makes that token's outputs NaN (as the reference's sums do) and
    leaves the other tokens' outputs as they are."""
    N, K, M = 2048, 2048, 10
    w, od, os_ = make("int4", N, K, 32, seed=77)
    X = px.synth_normal_f32(9, M * K, 1.0).reshape(M, K)
    Y0 = px.matmul_batch(X, w, N, K)
    X[2, 100] = np.nan
    Y1 = px.matmul_batch(X, w, N, K)
    assert np.isnan(Y1[2]).all()
    keep = [m for m in range(M) if m != 2]
    assert np.array_equal(Y1[keep], Y0[keep])


def test_gemm_ws_split_and_unsplit_k_agree():
    """The same product with the context's workspace (room for split-K partial sums, so K is
    split over more CTAs) and with a caller workspace of the minimum size (no room: every tile in
    one CTA): both meet the parity bar."""
    import torch

    N, K, M = 2048, 6144, 16
    w, od, os_ = make("int4", N, K, 32, seed=5)
    X = inputs(M, K, seed=6)
    ref = oracle.matmul(X, oracle.INT4, od, os_, 32, N, K)
    exact = exact_matmul("int4", od, os_, 32, N, K, X)
    Xd = torch.from_numpy(X).cuda()
    y_ctx = px.matmul_dev(Xd, w, N, K)
    nbytes = px._native.lib().pyxis_cuda_matmul_workspace_size(M, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    y_min = px.matmul_dev(Xd, w, N, K, workspace=ws)
    torch.cuda.synchronize()
    check_matmul(y_ctx.cpu().numpy(), ref, exact)
    check_matmul(y_min.cpu().numpy(), ref, exact)
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))


def test_gemm_ws_strided_rows():
    """x and y rows that are slices of wider tensors (ldx > K, ldy > N)."""
    import torch

    N, K, M = 1024, 2048, 9
    w, od, os_ = make("int4", N, K, 32, seed=8)
    X = inputs(M, K, seed=10)
    Xw = torch.zeros((M, K + 64), dtype=torch.float32, device="cuda")
    Xw[:, :K] = torch.from_numpy(X).cuda()
    Yw = torch.full((M, N + 32), 7.0, dtype=torch.float32, device="cuda")
    px.matmul_dev(Xw[:, :K], w, N, K, Y=Yw[:, :N])
    torch.cuda.synchronize()
    ref = oracle.matmul(X, oracle.INT4, od, os_, 32, N, K)
    check_matmul(Yw[:, :N].cpu().numpy(), ref, exact_matmul("int4", od, os_, 32, N, K, X))
    assert bool((Yw[:, N:] == 7.0).all())  # nothing written past the rows' ends


def test_reserve_workspace():
    """pyxis_cuda_reserve_workspace grows the context's workspace ahead of use (so a captured
    product allocates nothing)."""
    ctx = px.get_cuda(0)
    px._native.check(px._native.lib().pyxis_cuda_reserve_workspace(ctx.handle, 64 << 20))
    N, K, M = 2048, 2048, 12
    w, od, os_ = make("int4", N, K, 32, seed=12)
    X = inputs(M, K, seed=13)
    check_matmul(px.matmul_batch(X, w, N, K), oracle.matmul(X, oracle.INT4, od, os_, 32, N, K),
                 exact_matmul("int4", od, os_, 32, N, K, X))
