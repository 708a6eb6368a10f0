"""Multi-GPU sharding on real GPUs: runs tests/dist_worker.py under torchrun with 2 ranks (NCCL)
when at least two GPUs are visible."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_row_sharded_and_vocab_parallel_on_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(29600 + os.getpid() % 500),
           os.path.join(HERE, "dist_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0 and "DIST_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_one_process_two_devices():
    """One process, one context per device (the C ABI's multi-GPU model for a single host
    process): the same kernels -- batch GEMV, tensor-core GEMV, tensor-core GEMM, each with more
    than 48 KB of dynamic shared memory -- run on device 0 and then on device 1, whose launches
    need their own function attributes."""
    import numpy as np
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, HERE)
    import oracle
    import pyxis_b200 as px
    from parity import check_matmul, exact_matmul

    for qt, N, K, bs, M in (("int4", 2048, 2048, 32, 4), ("int8", 32768, 2048, 2048, 1), ("int4", 1024, 2048, 32, 64)):
        bits = px.synth_normal_bf16(N + M, N * K, 0.02)
        od, os_ = (oracle.quantize_int8 if qt == "int8" else oracle.quantize_int4)(oracle.bf16_to_f32(bits), bs)
        X = px.synth_normal_f32(M + 5, M * K, 1.0).reshape(M, K)
        ref = oracle.matmul(X, oracle.INT8 if qt == "int8" else oracle.INT4, od, os_, bs, N, K)
        exact = exact_matmul(qt, od, os_, bs, N, K, X)
        for dev in (0, 1):
            q = px.Weights.quantize_int8 if qt == "int8" else px.Weights.quantize_int4
            w = q(bits, bs, device=dev)
            check_matmul(px.matmul_batch(X, w, N, K), ref, exact)
            px._native.check(px._native.lib().pyxis_cuda_check_device_error(w.ctx.handle))
