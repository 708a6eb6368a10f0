"""Tensor-core prefill GEMM parity: M token rows through pyxis_cuda_matmul_dev (M >= 16 runs the
tcgen05 kernel) against the oracle's per-position matmul (the reference's prefill calls matmul
once per position, src/attention.rs:74-79).  Bar: tests/parity.py's 1e-3 relative error."""
import numpy as np
import pytest

import oracle
import pyxis_b200 as px
from parity import check_matmul, exact_matmul

pytestmark = pytest.mark.gpu
KIND = {"int8": oracle.INT8, "int4": oracle.INT4}


def make(qt, N, K, bs, seed):
    bits = px.synth_normal_bf16(seed, N * K, 0.02)
    w = px.Weights.quantize_int8(bits, bs) if qt == "int8" else px.Weights.quantize_int4(bits, bs)
    od, os_ = w.download()  # bit-exact with the oracle quantizer (test_quantize_gpu.py)
    return w, od, os_


def run_dev(w, X, N, K, workspace=None):
    import torch
    Xd = torch.from_numpy(X).cuda()
    Y = px.matmul_dev(Xd, w, N, K, workspace=workspace)
    torch.cuda.synchronize()
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))
    return Y.cpu().numpy()


@pytest.mark.parametrize("qt,N,K,bs", [
    ("int8", 6144, 2048, 2048),  # prefill gate_proj, int8 per-row (the model's int8 policy)
    ("int4", 6144, 2048, 32),    # prefill gate_proj, int4 group 32
    ("int8", 2048, 6144, 6144),  # prefill down_proj
    ("int4", 2048, 6144, 32),
])
def test_prefill_gemm_config_shapes(qt, N, K, bs):
    M = 512
    w, od, os_ = make(qt, N, K, bs, seed=N + K + bs)
    X = px.synth_normal_f32(2024, M * K, 1.0).reshape(M, K)
    Y = run_dev(w, X, N, K)
    ref = oracle.matmul(X, KIND[qt], od, os_, bs, N, K)
    check_matmul(Y, ref, exact_matmul(qt, od, os_, bs, N, K, X))


@pytest.mark.parametrize("qt,M,N,K,bs", [
    ("int8", 16, 256, 128, 128), ("int4", 16, 128, 128, 32), ("int8", 17, 1000, 512, 32),  # Q8_0 layout
    ("int4", 130, 300, 256, 64), ("int4", 257, 129, 1024, 128), ("int8", 100, 2048, 2048, 2048),
    ("int4", 33, 1024, 2048, 32),
])
def test_prefill_gemm_edges(qt, M, N, K, bs):
    w, od, os_ = make(qt, N, K, bs, seed=M * 3 + N + K)
    X = px.synth_normal_f32(M + 5, M * K, 1.0).reshape(M, K)
    X[0] *= 1e-20   # tiny row: the per-row power-of-two keeps its precision
    X[-1] *= 1e4
    if M > 2:
        X[1] = 0.0  # all-zero row
    Y = run_dev(w, X, N, K)
    ref = oracle.matmul(X, KIND[qt], od, os_, bs, N, K)
    exact = exact_matmul(qt, od, os_, bs, N, K, X)
    for m in range(M):
        check_matmul(Y[m], ref[m], exact[m])


def test_prefill_gemm_caller_workspace():
    import torch
    qt, M, N, K, bs = "int4", 64, 512, 1024, 32
    w, od, os_ = make(qt, N, K, bs, seed=9)
    need = px._native.lib().pyxis_cuda_matmul_workspace_size(M, K)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    X = px.synth_normal_f32(4, M * K, 1.0).reshape(M, K)
    Y = run_dev(w, X, N, K, workspace=ws)
    ref = oracle.matmul(X, KIND[qt], od, os_, bs, N, K)
    check_matmul(Y, ref, exact_matmul(qt, od, os_, bs, N, K, X))
    with pytest.raises(px.PyxisError):
        px.matmul_dev(torch.from_numpy(X).cuda(), w, N, K, workspace=ws[: need // 2])


def test_batch_rows_route_through_host_api():
    """matmul_batch (host buffers) with M = 40 rows: the tensor-core path behind the host API."""
    qt, M, N, K, bs = "int8", 40, 1536, 2048, 2048
    w, od, os_ = make(qt, N, K, bs, seed=77)
    X = px.synth_normal_f32(8, M * K, 1.0).reshape(M, K)
    Y = px.matmul_batch(X, w, N, K)
    ref = oracle.matmul(X, KIND[qt], od, os_, bs, N, K)
    check_matmul(Y, ref, exact_matmul(qt, od, os_, bs, N, K, X))
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))
