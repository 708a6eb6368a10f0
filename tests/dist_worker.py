"""One rank of the multi-GPU check (launched by tests/test_dist_gpu.py through torchrun, one
process per GPU, NCCL): row-sharded GEMVs all-gathered equal the single-GPU product bit for bit,
and the vocab-parallel lm_head's distributed greedy argmax equals the single-GPU argmax."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import pyxis_b200 as px  # noqa: E402
from pyxis_b200.dist import RowShardedMatmul, VocabParallelHead  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ok = True
    for qt, N, K, bs in (("int4", 6144, 2048, 32), ("int8", 6144, 2048, 2048), ("int8", 2048, 6144, 6144)):
        bits = px.synth_normal_bf16(N + K, N * K, 0.02)
        sh = RowShardedMatmul(bits, N, K, qt, rank, world, local)
        t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
        full = (px.Weights.quantize_int8(t, bs, device=local) if qt == "int8"
                else px.Weights.quantize_int4(t, bs, device=local))
        X = torch.from_numpy(px.synth_normal_f32(7, K, 1.0)).cuda().view(1, K)
        y_sh = sh.forward_gathered(X)
        y_full = px.matmul_dev(X, full, N, K)
        torch.cuda.synchronize()
        if not torch.equal(y_sh, y_full):
            print(f"rank {rank}: row-sharded {qt} {N}x{K} differs: {(y_sh - y_full).abs().max().item()}", flush=True)
            ok = False
    V, H = 151936, 2048
    bits = px.synth_normal_bf16(0x11EAD, V * H, 0.02)
    head = VocabParallelHead(bits, V, H, "int8", rank, world, local)
    t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    full = px.Weights.quantize_int8(t, H, device=local)
    h = torch.from_numpy(px.synth_normal_f32(9, 4 * H, 1.0)).cuda().view(4, H)
    got = head.greedy(h)
    logits = px.matmul_dev(h, full, V, H)
    want, _ = px.argmax_dev(logits)
    want = want.cpu().numpy()
    if list(got) != list(want):
        print(f"rank {rank}: vocab-parallel argmax {list(got)} != single-GPU {list(want)}", flush=True)
        ok = False
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("DIST_OK" if flag.item() == 0 else "DIST_FAIL", flush=True)
    sys.exit(0 if flag.item() == 0 else 1)


if __name__ == "__main__":
    main()
