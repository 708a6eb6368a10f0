"""One-rank greedy head (pyxis_cuda_head_greedy_dev with a communicator of one GPU): the int8 head
on the tensor-core GEMV with the argmax keys folded into its epilogue, then the NCCL all-gather
and the device pick.  Run by tests/test_head_gpu.py in its own process (a gloo group of one
rank for the id broadcast).  Prints HEAD_OK when every token equals the single-device argmax
(pyxis_cuda_argmax_dev over the same logits) and the oracle's argmax (src/output_head.rs:30-44)."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

import oracle  # noqa: E402
import pyxis_b200 as px  # noqa: E402
from pyxis_b200.dist import Comm, VocabParallelHead  # noqa: E402


def main():
    port = int(sys.argv[1])
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    comm = Comm(0, 1, 0)
    V, H = 40000, 2048
    bits = px.synth_normal_bf16(0x4EAD, V * H, 0.02).reshape(V, H)
    # rows 5 and 30007 identical and aligned with the all-ones input: an exact tie for the maximum
    bits[5] = bits[30007] = px.synth_normal_bf16(77, H, 0.02)
    head = VocabParallelHead(bits.ravel(), V, H, "int8", comm)
    full = px.Weights.quantize_int8(bits.ravel(), H)
    assert px.matmul_kernel_name(full, 1, V, H) == "gemv_tc_i8_kernel"
    fails = []
    tie_x = oracle.bf16_to_f32(bits[5]).astype(np.float32)
    for M in (1, 3, 8, 1, 12, 2, 8):  # changing row counts: the keys must be left zero by every call
        X = px.synth_normal_f32(100 + M, M * H, 1.0).reshape(M, H)
        X[0] = tie_x * 50.0
        if M >= 3:
            X[1, 17] = np.nan   # every logit NaN: the reference answers index 0
            X[2] = 0.0          # every logit 0: ties, index 0
        h = torch.from_numpy(X).cuda()
        got = head.greedy(h).cpu().numpy()
        logits = px.matmul_dev(h, full, V, H)
        want = px.argmax_dev(logits)[0].cpu().numpy()
        lg = logits.cpu().numpy()
        orc = [oracle.argmax(lg[m]) for m in range(M)]
        if list(got) != list(want) or list(got) != orc:
            fails.append(f"M={M}: head {list(got)} argmax_dev {list(want)} oracle {orc}")
        if got[0] != 5:
            fails.append(f"M={M}: the tie of rows 5 and 30007 went to {got[0]}")
        if M >= 3 and (got[1] != 0 or got[2] != 0):
            fails.append(f"M={M}: NaN / zero rows gave {got[1]}, {got[2]}")
    px._native.check(px._native.lib().pyxis_cuda_check_device_error(full.ctx.handle))
    del head
    comm.close()
    dist.destroy_process_group()
    if fails:
        print("\n".join(fails))
        sys.exit(1)
    print("HEAD_OK")


if __name__ == "__main__":
    main()
