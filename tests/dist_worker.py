"""One rank of the multi-GPU check (launched by tests/test_dist_gpu.py through torchrun, one
process per GPU, NCCL):
  * row-sharded products all-gathered equal the single-GPU product: bit for bit where the kernel's
    per-row arithmetic does not depend on the row count (the GEMVs), within the matmul bar
    (max_i |y_i - r_i| / max(|r_i|, 1e-3 max|r|) <= 1e-3) where the weight-streaming matmul splits K
    by the number of tiles;
  * the vocab-parallel lm_head's device-side greedy argmax (pyxis_cuda_head_greedy_dev) equals
    the single-GPU argmax, int8 per-row and int4 group-32 heads, 1 to 64 rows, including a NaN at
    index 0, -0.0 against +0.0 and ties across the shard boundary;
  * vocab-parallel batched generation (pyxis_cuda_model_set_vocab_parallel) gives every rank's
    sequences the oracle's greedy tokens (small model) and the tokens of the same model with its
    full head (Qwen3-1.7B shape)."""
import ctypes as C
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import oracle  # noqa: E402
from parity import rel_err  # noqa: E402
import pyxis_b200 as px  # noqa: E402
from pyxis_b200 import _native  # noqa: E402
from pyxis_b200.dist import Comm, RowShardedMatmul, VocabParallelHead, shard_range  # noqa: E402
from pyxis_b200.model import QWEN3_1_7B, Decoder, ModelConfig, SyntheticModel  # noqa: E402

SMALL = ModelConfig(hidden=256, n_layers=2, n_q_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=2048,
                    rope_theta=10000.0)


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    fails = []
    for qt, N, K, bs in (("int4", 6144, 2048, 32), ("int8", 6144, 2048, 2048), ("int8", 2048, 6144, 6144)):
        bits = px.synth_normal_bf16(N + K, N * K, 0.02)
        sh = RowShardedMatmul(bits, N, K, qt, rank, world, local)
        t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
        full = (px.Weights.quantize_int8(t, bs, device=local) if qt == "int8"
                else px.Weights.quantize_int4(t, bs, device=local))
        for B in (1, 8):
            X = torch.from_numpy(px.synth_normal_f32(7 + B, B * K, 1.0)).cuda().view(B, K)
            y_sh = sh.forward_gathered(X)
            y_full = px.matmul_dev(X, full, N, K)
            torch.cuda.synchronize()
            # the same kernel on the shard and on the full matrix adds each row in the same order,
            # unless it splits K by the number of row tiles (the mma GEMV, the weight-streaming
            # matmul); kernels chosen by size differ from one another: within the matmul bar
            k_full = px.matmul_kernel_name(full, B, N, K)
            k_sh = px.matmul_kernel_name(sh.w, B, sh.hi - sh.lo, K)
            if k_full != k_sh or k_full in ("gemm_ws_kernel", "gemv_mma_kernel"):
                err = rel_err(y_sh.cpu().numpy(), y_full.cpu().numpy())
                if err > 1e-3:
                    fails.append(f"row-sharded {qt} {N}x{K} B={B} ({k_sh} / {k_full}): rel err {err}")
            elif not torch.equal(y_sh, y_full):
                fails.append(f"row-sharded {qt} {N}x{K} B={B} differs: {(y_sh - y_full).abs().max().item()}")

    comm = Comm(rank, world, local)
    V, H = 151936, 2048
    bits = px.synth_normal_bf16(0x11EAD, V * H, 0.02)
    t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    for qt, bs in (("int8", H), ("int4", 32)):
        head = VocabParallelHead(bits, V, H, qt, comm, block_size=bs)
        full = px.Weights.quantize_int8(t, bs, device=local) if qt == "int8" else \
            px.Weights.quantize_int4(t, bs, device=local)
        for M in (1, 4, 64):
            h = torch.from_numpy(px.synth_normal_f32(9 + M, M * H, 1.0)).cuda().view(M, H)
            got = head.greedy(h).cpu().numpy()
            want = px.argmax_dev(px.matmul_dev(h, full, V, H))[0].cpu().numpy()
            if list(got) != list(want):
                fails.append(f"vocab-parallel {qt} M={M}: {list(got)} != single-GPU {list(want)}")
        del head, full
    # the argmax rules across shards, through an f32 identity head whose logits are the rows
    # themselves: ties go to the lowest index, -0.0 ties with +0.0
    small_v = 1024
    vals = np.random.default_rng(3).standard_normal((3, small_v)).astype(np.float32)
    lo1 = shard_range(small_v, 1, world)[0] if world > 1 else 10
    vals[1, 7] = vals[1, lo1 + 3] = 40.0
    vals[2, :] = -1.0
    vals[2, small_v - 1] = 0.0
    vals[2, 0] = -0.0
    ident = np.zeros((small_v, small_v), np.float32)
    np.fill_diagonal(ident, 1.0)
    lo, hi = shard_range(small_v, rank, world)
    wsh = px.Weights.from_dense(ident[lo:hi].ravel(), device=local)
    X = torch.from_numpy(vals).cuda()
    tok = torch.empty(3, dtype=torch.int32, device="cuda")
    _native.check(_native.lib().pyxis_cuda_head_greedy_dev(comm.handle, wsh.handle, small_v, lo, hi - lo, small_v,
                                                           C.c_void_p(X.data_ptr()), 3, small_v,
                                                           C.c_void_p(tok.data_ptr()),
                                                           C.c_void_p(px._stream_handle(None, local))))
    got = list(tok.cpu().numpy())
    want = [oracle.argmax(vals[m]) for m in range(3)]
    if got != want:
        fails.append(f"vocab-parallel argmax rules: {got} != {want}")

    # vocab-parallel batched generation, small model: every rank's sequences vs the oracle
    m = SyntheticModel(SMALL, seed=29)
    for qt in ("int8", "int4"):
        dec = Decoder(m, qtype=qt, max_seq=80, device=local, vocab_parallel=comm)
        prompts = px.synth_tokens(0x51 + rank, 2 * 70, SMALL.vocab).reshape(2, 70)
        toks, _ = dec.generate_batch(prompts, 5)
        for s in range(2):
            ref = oracle.greedy_decode(SMALL, m.bf16, qt, list(prompts[s]), 5)
            if not np.array_equal(toks[s], ref):
                fails.append(f"vocab-parallel generate_batch {qt} seq {s}: {toks[s]} != oracle {ref}")
        dec.close()
    # Qwen3-1.7B shape, int4: vocab-parallel head == the same model's full head
    m = SyntheticModel(QWEN3_1_7B, seed=0x5EED)
    dec = Decoder(m, qtype="int4", max_seq=64, device=local, vocab_parallel=comm)
    prompts = px.synth_tokens(0xB1 + rank, 4 * 40, QWEN3_1_7B.vocab).reshape(4, 40)
    toks_vp, _ = dec.generate_batch(prompts, 8)
    dec.set_vocab_parallel(False)
    toks_full, _ = dec.generate_batch(prompts, 8)
    if not np.array_equal(toks_vp, toks_full):
        fails.append(f"vocab-parallel Qwen3-shape tokens differ from the full head: {toks_vp} vs {toks_full}")
    dec.close()
    comm.close()

    for f in fails:
        print(f"rank {rank}: {f}", flush=True)
    flag = torch.tensor([len(fails)], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("DIST_OK" if flag.item() == 0 else "DIST_FAIL", flush=True)
    sys.exit(0 if flag.item() == 0 else 1)


if __name__ == "__main__":
    main()
