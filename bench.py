#!/usr/bin/env python
"""bench.py -- quantized decode GEMV throughput (HBM GB/s) of the B200 backend.

Workload (one "step"): the int4 group-32 decode-GEMV sweep over Qwen3-1.7B projection shapes --
q_proj 2048x2048, kv_proj 1024x2048, gate_proj and up_proj 6144x2048, down_proj 2048x6144 --
plus the int8 per-row lm_head 151936x2048, each at batch 1 and batch 8: 12 GEMV launches that
stream 0.68 GB of packed weights.  Weights are seeded N(0, 0.02) rounded to bf16 and quantised
on the device by the reference's quantizer rules; x is seeded N(0, 1) f32.  The step's working
set (~680 MB) is 5x the 126 MB L2 and every matrix is re-read only after >= 311 MB of other
traffic, so no L2 flush is needed between steps.

  value  whole-job algorithmic GB/s (weights + scales + x + y bytes per step x steps / time),
         inputs resident in HBM, device time by CUDA events, max over ranks.
  e2e    the same sweep through the C ABI's host-pointer matmul (pinned host x in, host y out,
         one synchronous call per GEMV, as a Rust `matmul()` call would do it).
  --impl reference   the oracle port of the reference's Rayon CPU path, all host threads.

Multi-GPU (torchrun): every rank runs the whole sweep on its own GPU -- independent decode
streams, data-parallel, no collective on the data path ("scaling": "weak").  With N > 1 the line
also carries the sharded legs, each checked against the single-GPU result on the same rank:
  row_split       gate/up/down (int4) and the lm_head (int8) split by output rows: per-rank and
                  aggregate device GB/s, with and without the NCCL all-gather of the outputs
  lm_head_vocab_parallel   the greedy head split by vocabulary rows (device argmax keys + one
                  NCCL all-gather of 8 bytes per row and rank), device time per token
  batch_decode    config 5 with its sequences data-parallel and the lm_head vocab-parallel
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s & quantized GEMV HBM GB/s (% of peak) at 1/2/4/8 B200"
UNIT = "GB/s"
WORKLOAD = "int4 g32 decode GEMV sweep (q 2048x2048, kv 1024x2048, gate/up 6144x2048, down 2048x6144) + int8 per-row lm_head 151936x2048, batch 1 and 8"
SWEEP = [  # name, qtype, N (out_features), K (in_features), block_size
    ("q_proj", "int4", 2048, 2048, 32),
    ("kv_proj", "int4", 1024, 2048, 32),
    ("gate_proj", "int4", 6144, 2048, 32),
    ("up_proj", "int4", 6144, 2048, 32),
    ("down_proj", "int4", 2048, 6144, 32),
    ("lm_head", "int8", 151936, 2048, 2048),
]
BATCHES = (1, 8)
SEED = 0x5EED


def gemv_bytes(qt, N, K, bs, B):
    data = N * K if qt == "int8" else (N * K + 1) // 2
    scales = 4 * math.ceil(N * K / bs)
    return data + scales + 4 * B * (K + N)


def step_bytes():
    return sum(gemv_bytes(qt, N, K, bs, B) for B in BATCHES for (_, qt, N, K, bs) in SWEEP)


def config_dict(n):
    return {"workload": WORKLOAD, "batches": list(BATCHES), "weights": "seeded N(0,0.02) bf16 -> reference quantizer",
            "x": "seeded N(0,1) f32", "l2": "working set 680 MB/step > 126 MB L2; no flush needed",
            "timing": "CUDA events around K replays of the 12-launch step captured once as a CUDA graph",
            "parallelism": f"dp{n} (independent decode streams per GPU)"}


# ---------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.gpu_id = gpu_id
        self.proc = None
        self.out = None

    def start(self):
        cmd = ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "200"]
        if self.gpu_id:
            cmd += ["-i", self.gpu_id]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profiled_traffic(kernel_tag: str):
    """dram bytes per launch of the dominant kernel from its committed ncu summary (the latest
    capture it lists), if any."""
    p = os.path.join(ROOT, "profiles", f"{kernel_tag}.txt")
    found = None
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                found = float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return found


# ---------------------------------------------------------------------------------------------
def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist

        # NCCL's communicator set-up lines (rank counts) go to stdout before the JSON line,
        # which is printed last, after the communicators are destroyed
        os.environ["NCCL_DEBUG"] = "INFO"
        os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist

    # NCCL reduces device tensors; the gloo groups of the CPU tests reduce host tensors
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def gpu_uuid(local):
    try:
        import torch

        u = str(torch.cuda.get_device_properties(local).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


# ---------------------------------------------------------------------------------------------
_CPU_SWEEP_INPUTS = None


def cpu_model() -> str:
    """The host CPU's model name (the CPU baselines run on it)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_sweep_inputs():
    """The sweep's matrices packed by the oracle quantizer and the x rows of every batch size,
    built once per process (the packing takes ~10x longer than one timed sweep)."""
    global _CPU_SWEEP_INPUTS
    if _CPU_SWEEP_INPUTS is None:
        import oracle

        mats = []
        for i, (name, qt, N, K, bs) in enumerate(SWEEP):
            vals = oracle.bf16_to_f32(oracle.synth_normal_bf16(SEED + i, N * K, 0.02))
            d, s = (oracle.quantize_int8 if qt == "int8" else oracle.quantize_int4)(vals, bs)
            del vals
            mats.append((qt, N, K, bs, d, s))
        xs = {B: oracle.synth_normal_f32(SEED + 100 + B, B * 6144, 1.0) for B in BATCHES}
        _CPU_SWEEP_INPUTS = (mats, xs)
    return _CPU_SWEEP_INPUTS


def run_cpu_sweep(nthreads: int, batches=BATCHES):
    """One sweep step through the oracle port (the reference's Rayon CPU matmul, restated in C).
    Returns (seconds, bytes) for the given batches."""
    import oracle

    mats, xs = cpu_sweep_inputs()
    t0 = time.perf_counter()
    nbytes = 0
    for B in batches:
        for (qt, N, K, bs, d, s) in mats:
            X = xs[B][: B * K].reshape(B, K)
            oracle.matmul(X, oracle.INT8 if qt == "int8" else oracle.INT4, d, s, bs, N, K, nthreads=nthreads)
            nbytes += gemv_bytes(qt, N, K, bs, B)
    return time.perf_counter() - t0, nbytes


def reference_arm(args, ws, rank):
    if rank != 0:
        return
    import oracle

    cores = oracle.num_cpus()
    for _ in range(args.warmup):
        run_cpu_sweep(cores, batches=(1,))
    total_t, total_b = 0.0, 0
    for _ in range(args.steps):
        t, b = run_cpu_sweep(cores)
        total_t += t
        total_b += b
    value = total_b / total_t / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_t / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(ws),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "cpu": cpu_model(), "kind": "port",
                             "sample": "each step = the full sweep (12 matvec calls) through the C port of "
                                       "src/matmul.rs (scalar x86 dot products, rows over all host threads)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PREFILL_SHAPES = [  # name, qtype, N, K, block: X [512, K] x W [N, K]^T on the tensor cores
    ("gate_proj int8", "int8", 6144, 2048, 2048), ("gate_proj int4", "int4", 6144, 2048, 32),
    ("down_proj int8", "int8", 2048, 6144, 6144), ("down_proj int4", "int4", 2048, 6144, 32)]
PREFILL_M = 512


def run_vocab_parallel_head(comm, ws, rank, local, steps, lm_full):
    """Greedy next token through the int8 lm_head split by vocabulary rows over the ranks: each
    rank's GEMV over V/ws rows, device argmax keys, the keys exchanged (8 bytes per row and rank,
    over peer memory, or an NCCL all-gather where the GPUs cannot map each other), the pick on the
    device (pyxis_cuda_head_greedy_dev).  Device time per token (CUDA events around replays of a
    CUDA graph of 20 calls, as the decode step runs it; max over ranks), at batch 1 and 8; every
    rank's tokens are checked against the single-GPU matmul + argmax of the full head."""
    import torch

    import pyxis_b200 as px
    from pyxis_b200.dist import VocabParallelHead

    V, H = 151936, 2048
    bits = px.synth_normal_bf16(SEED + 5, V * H, 0.02)  # the sweep's lm_head
    head = VocabParallelHead(bits, V, H, "int8", comm)
    del bits
    out = {"n_gpus": ws, "rows_per_gpu": head.mm.hi - head.mm.lo,
           "kernel": px.matmul_kernel_name(head.mm.w, 1, head.mm.hi - head.mm.lo, H), "batches": []}
    parity = True
    peak, _ = measured_peak_hbm()
    for B in BATCHES:
        h = torch.from_numpy(px.synth_normal_f32(9 + B, B * H, 1.0)).cuda().view(B, H)
        tok = head.greedy(h)
        want = px.argmax_dev(px.matmul_dev(h, lm_full, V, H))[0]
        same = bool(torch.equal(tok, want))
        parity = parity and same
        reps = 20
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                head.greedy(h, tokens=tok, stream=s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
            for _ in range(reps):
                head.greedy(h, tokens=tok, stream=s)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        barrier(ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = max_over_ranks(e0.elapsed_time(e1) * 1e3 / (steps * reps), ws)
        del g
        same = same and bool(torch.equal(tok, want))  # after the replays too
        parity = parity and same
        shard_bytes = gemv_bytes("int8", head.mm.hi - head.mm.lo, H, H, B)
        out["batches"].append({"B": B, "us_per_token": us, "tokens_match_single_gpu": same,
                               "shard_gbs": shard_bytes / us / 1e3, "shard_frac_of_peak": shard_bytes / us / 1e3 / peak,
                               "first_tokens": [int(t) for t in tok[:4].cpu()]})
    out["parity"] = bool(max_over_ranks(0.0 if parity else 1.0, ws) == 0.0)
    out["note"] = ("device time per call: shard GEMV + argmax keys + key exchange + device pick; "
                   "shard_frac_of_peak = the shard's algorithmic bytes / time / one GPU's HBM peak")
    return out


def run_row_split(ws, rank, local, steps, capture, replay_ms, full):
    """gate/up/down (int4 g32) and the lm_head (int8 per row) split by output rows: rank r
    quantises and streams only its rows [r*N/ws, (r+1)*N/ws) of each (pyxis_b200.dist
    RowShardedMatmul), at batch 1 and 8.  Device GB/s per rank (CUDA graph of the shard GEMVs),
    aggregate GB/s over the job, and the same with the NCCL all-gather of every output into the
    full vector; the all-gathered output is checked bit for bit against the full matrix on the
    same rank."""
    import torch

    import pyxis_b200 as px
    from pyxis_b200.dist import RowShardedMatmul, shard_range

    dev = torch.device("cuda", local)
    shards = []
    for i, (name, qt, N, K, bs) in enumerate(SWEEP):
        if name not in ("gate_proj", "up_proj", "down_proj", "lm_head"):
            continue
        bits = px.synth_normal_bf16(SEED + i, N * K, 0.02)
        shards.append((name, qt, N, K, bs, RowShardedMatmul(bits, N, K, qt, rank, ws, local, block_size=bs)))
        del bits
    X = {B: torch.from_numpy(px.synth_normal_f32(SEED + 100 + B, B * 6144, 1.0)).to(dev).view(B, 6144) for B in BATCHES}
    Y = {B: torch.empty((B, 151936), dtype=torch.float32, device=dev) for B in BATCHES}

    def step(st):
        for B in BATCHES:
            for (name, qt, N, K, bs, sh) in shards:
                sh.forward(X[B][:, :K], Y=Y[B][:, :sh.hi - sh.lo], stream=st)

    g = capture(step)
    for _ in range(3):
        g.replay()
    barrier(ws)
    ms = max_over_ranks(replay_ms(g, steps), ws)
    del g
    rank_bytes = sum(gemv_bytes(qt, sh.hi - sh.lo, K, bs, B) for B in BATCHES for (_, qt, N, K, bs, sh) in shards)
    # every rank's algorithmic bytes (its rows' codes and scales, x, its outputs), summed
    job_bytes = sum(gemv_bytes(qt, hi - lo, K, bs, B) for B in BATCHES for (_, qt, N, K, bs, _) in shards
                    for (lo, hi) in (shard_range(N, r, ws) for r in range(ws)))
    peak, peak_kind = measured_peak_hbm()
    # parity: all-gathered shards == the full matrix on this rank: bit for bit, or (where the shard
    # and the full matrix take different kernels by size, or the kernel -- the mma GEMV, the
    # weight-streaming matmul -- splits K by the row count) within the matmul bar
    # max_i |y_i - r_i| / max(|r_i|, 1e-3 max|r|) <= 1e-3
    parity = True
    mismatch, bitwise, max_rel = [], [], 0.0
    for B in BATCHES:
        for (name, qt, N, K, bs, sh) in shards:
            yg = sh.forward_gathered(X[B][:, :K])
            yf = px.matmul_dev(X[B][:, :K], full[name], N, K)
            if torch.equal(yg, yf):
                bitwise.append(f"{name} B={B}")
                continue
            d = (yg.double() - yf.double()).abs()
            den = torch.maximum(yf.double().abs(), 1e-3 * yf.double().abs().max())
            rel = float((d / den).max())
            max_rel = max(max_rel, rel)
            if rel > 1e-3:
                parity = False
                mismatch.append(f"{name} B={B}: {rel:.3g}")
    # with the all-gather: eager, one NCCL all-gather per output (device time on torch's stream)
    for _ in range(2):
        for B in BATCHES:
            for (name, qt, N, K, bs, sh) in shards:
                sh.forward_gathered(X[B][:, :K])
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        for B in BATCHES:
            for (name, qt, N, K, bs, sh) in shards:
                sh.forward_gathered(X[B][:, :K])
    e1.record()
    torch.cuda.synchronize()
    ms_ag = max_over_ranks(e0.elapsed_time(e1), ws)
    cases = [{"matrix": f"{name} {qt} {N}x{K}", "rows_per_gpu": sh.hi - sh.lo,
              "kernel": px.matmul_kernel_name(sh.w, 1, sh.hi - sh.lo, K)} for (name, qt, N, K, bs, sh) in shards]
    agg = job_bytes * steps / (ms / 1e3) / 1e9
    return {"matrices": cases, "batches": list(BATCHES), "ms_per_step": ms / steps,
            "rank_gbs": rank_bytes * steps / (ms / 1e3) / 1e9, "aggregate_gbs": agg,
            "aggregate_frac_of_job_peak": agg / (ws * peak), "peak_per_gpu": peak, "peak_kind": peak_kind,
            "ms_per_step_with_allgather": ms_ag / steps,
            "aggregate_gbs_with_allgather": job_bytes * steps / (ms_ag / 1e3) / 1e9,
            "parity": bool(max_over_ranks(0.0 if parity else 1.0, ws) == 0.0), "mismatch": mismatch,
            "bitwise_equal": bitwise, "max_rel_err_vs_full": max_over_ranks(max_rel, ws),
            "note": "without the all-gather: CUDA graph of the shard GEMVs; with it: eager calls, "
                    "torch NCCL all_gather_into_tensor after every GEMV (latency-bound at these sizes)"}


def px_synth_bits(seed, n):
    import pyxis_b200 as px
    return px.synth_normal_bf16(seed, n, 0.02)


def px_synth_f32(seed, n):
    import pyxis_b200 as px
    return px.synth_normal_f32(seed, n, 1.0)


def run_prefill(local, reps=20):
    """Prefill GEMMs (X f32 [512, K] N(0,1) x quantised W): TFLOP/s counting 2*M*N*K only."""
    import numpy as np
    import torch

    import pyxis_b200 as px

    dev = torch.device("cuda", local)
    out = []
    for i, (name, qt, N, K, bs) in enumerate(PREFILL_SHAPES):
        bits = px.synth_normal_bf16(SEED + 50 + i, N * K, 0.02)
        t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(dev)
        w = px.Weights.quantize_int8(t, bs, device=local) if qt == "int8" else px.Weights.quantize_int4(t, bs, device=local)
        X = torch.from_numpy(px.synth_normal_f32(SEED + 60 + i, PREFILL_M * K, 1.0)).to(dev).view(PREFILL_M, K)
        Y = torch.empty((PREFILL_M, N), dtype=torch.float32, device=dev)
        # the context's own workspace (allocated by the first call, outside the timing): it also
        # holds split-K partials, which a caller workspace of pyxis_cuda_matmul_workspace_size
        # bytes has no room for (down_proj's 64 output tiles would leave most SMs idle)
        for _ in range(3):
            px.matmul_dev(X, w, N, K, Y=Y)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            px.matmul_dev(X, w, N, K, Y=Y)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        flops = 2.0 * PREFILL_M * N * K
        out.append({"shape": f"{name}: X[{PREFILL_M},{K}] x W[{N},{K}]", "us": us, "tflops": flops / us / 1e6,
                    "kernel": px.matmul_kernel_name(w, PREFILL_M, N, K), "l2": "warm (back-to-back launches)"})
        del w, X, Y, t
    return out


DECODE_WORKLOAD = ("Qwen3-1.7B-shape decode, random init, int8 one scale per row: hidden 2048, 28 layers, "
                   "16/8 heads x 128, FFN 6144, vocab 151936, tied lm_head; 16 prompt ids + 128 greedy tokens, batch 1")
DECODE_PROMPT, DECODE_NEW = 16, 128
DECODE_CPU_TOKENS = 16  # the CPU baseline's bounded sample of config 4: weight-bound passes of ~1.7 GB each


def decode_bytes_per_token(cfg, pos):
    """HBM bytes one decode step reads at cache position `pos`: int8 codes + row scales of every
    projection and the lm_head, the KV cache rows 0..pos, the embedding row."""
    per_layer = (cfg.q_dim + 2 * cfg.kv_dim) * cfg.hidden + cfg.hidden * cfg.q_dim + 2 * cfg.ffn * cfg.hidden \
        + cfg.hidden * cfg.ffn
    rows = cfg.q_dim + 2 * cfg.kv_dim + cfg.hidden + 2 * cfg.ffn + cfg.hidden
    w = cfg.n_layers * (per_layer + 4 * rows) + cfg.vocab * cfg.hidden + 4 * cfg.vocab
    kv = cfg.n_layers * 2 * (pos + 1) * cfg.kv_dim * 4
    return w + kv + 2 * cfg.hidden


def run_decode(local, cpu_sample_tokens=0):
    import time as _t

    from pyxis_b200 import synth_tokens
    from pyxis_b200.model import QWEN3_1_7B, Decoder, SyntheticModel

    cfg = QWEN3_1_7B
    m = SyntheticModel(cfg, SEED)
    prompt = synth_tokens(0x9E0, DECODE_PROMPT, cfg.vocab)
    t0 = _t.time()
    dec = Decoder(m, qtype="int8", max_seq=DECODE_PROMPT + DECODE_NEW, device=local)
    setup_s = _t.time() - t0
    dec.generate(prompt, 8)  # warm-up: graph capture + first replays
    toks, (p_ms, d_ms) = dec.generate(prompt, DECODE_NEW)
    dec.close()
    steps = DECODE_NEW - 1
    tps = steps / (d_ms / 1e3)
    avg_bytes = sum(decode_bytes_per_token(cfg, DECODE_PROMPT + i) for i in range(steps)) / steps
    out = {"workload": DECODE_WORKLOAD, "tokens_per_s": tps, "ms_per_token": d_ms / steps, "prompt_ms": p_ms,
           "bytes_per_token": avg_bytes, "achieved_gbs": avg_bytes * tps / 1e9, "model_setup_s": setup_s,
           "first_tokens": [int(t) for t in toks[:8]]}
    if cpu_sample_tokens:
        import oracle
        tm = []
        oracle.greedy_decode(cfg, m.bf16, "int8", prompt[:1], cpu_sample_tokens, timing=tm)
        out["cpu_baseline"] = {"tokens_per_s": cpu_sample_tokens / tm[0], "cores": oracle.num_cpus(), "cpu": cpu_model(),
                               "kind": "port",
                               "sample": f"1 prompt id + {cpu_sample_tokens} greedy tokens ({cpu_sample_tokens} forward "
                                         "passes) through the C port of Model::generate on all host threads; the "
                                         "host-side packing of the weights is outside the timed region"}
    return out


BATCH_SEQS, BATCH_PROMPT, BATCH_NEW = 64, 2048, 256
BATCH_WORKLOAD = ("Qwen3-1.7B-shape batched decode, random init, int4 group 32 (lm_head too): 64 sequences x 2048 "
                  "random prompt ids prefilled, then 256 greedy tokens each; sequences split data-parallel over the "
                  "GPUs")


def batch_step_bytes(cfg, n_seq, pos, head_ranks=1):
    """HBM bytes of one batched int4 step at cache position `pos`: every projection's codes and
    group-32 scales once (GEMMs over the n_seq rows) plus each sequence's KV rows 0..pos; with a
    vocab-parallel head over head_ranks GPUs, this rank's 1/head_ranks of the lm_head."""
    layers = cfg.n_layers * ((cfg.q_dim + 2 * cfg.kv_dim) * cfg.hidden + cfg.hidden * cfg.q_dim
                             + 3 * cfg.ffn * cfg.hidden)
    head = cfg.vocab * cfg.hidden // head_ranks
    w = (layers + head) // 2 + (layers + head) // 32 * 4
    kv = n_seq * cfg.n_layers * 2 * (pos + 1) * cfg.kv_dim * 4
    return w + kv


def prefill_flops(cfg, n_seq, P):
    """Algorithmic flops of the prefill: 2 x params x tokens for the projections, the causal
    attention's QK and PV (2 x 2 x hd per (query, key) pair and head), the lm_head of the last rows."""
    proj = cfg.n_layers * ((cfg.q_dim + 2 * cfg.kv_dim) * cfg.hidden + cfg.hidden * cfg.q_dim
                           + 3 * cfg.ffn * cfg.hidden)
    attn = cfg.n_layers * cfg.n_q_heads * 4 * cfg.head_dim * (P * (P + 1) // 2)
    return n_seq * (2 * proj * P + attn) + 2 * n_seq * cfg.vocab * cfg.hidden


def run_batch_decode(local, ws, rank, n_seq_total=BATCH_SEQS, P=BATCH_PROMPT, n_new=BATCH_NEW, comm=None):
    """64 sequences of 2048 prompt ids then 256 greedy tokens, int4: this rank's share of the
    sequences through pyxis_cuda_model_generate_batch.  With a communicator (N > 1) the lm_head is
    vocab-parallel over the ranks (every rank's final hidden rows all-gathered, its V/N rows of
    the head, the argmax keys all-gathered); its tokens are then checked against the same model's
    full head on this rank for the first two sequences."""
    import zlib

    import numpy as np

    from pyxis_b200 import synth_tokens
    from pyxis_b200.model import QWEN3_1_7B, Decoder, SyntheticModel

    cfg = QWEN3_1_7B
    n_seq = n_seq_total // ws + (1 if rank < n_seq_total % ws else 0)
    first = rank * (n_seq_total // ws) + min(rank, n_seq_total % ws)
    prompts = synth_tokens(0xBA7C, n_seq_total * P, cfg.vocab).reshape(n_seq_total, P)[first:first + n_seq]
    vp = comm if (comm is not None and n_seq_total % ws == 0) else None
    dec = Decoder(SyntheticModel(cfg, SEED), qtype="int4", max_seq=P + n_new, device=local, vocab_parallel=vp)
    dec.generate_batch(prompts[:, :64], 4)  # warm-up: first-use set-up of every kernel
    toks, (pre_ms, dec_ms) = dec.generate_batch(prompts, n_new)
    out = {"workload": BATCH_WORKLOAD, "sequences_this_rank": n_seq, "prefill_ms": pre_ms, "decode_ms": dec_ms,
           "lm_head": f"vocab-parallel over {ws} GPUs (NCCL all-gather of hidden rows and argmax keys)" if vp
           else "full int4 lm_head on each GPU"}
    if vp is not None:
        n_chk = 16
        dec.set_vocab_parallel(False)
        ref, _ = dec.generate_batch(prompts[:2], n_chk)
        out["vocab_parallel_parity"] = bool(np.array_equal(ref, toks[:2, :n_chk]))
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.ascontiguousarray(toks)).cuda()
        allt = torch.empty((ws,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(allt, t)
        toks_all = allt.cpu().numpy().reshape(n_seq_total, n_new)
    else:
        toks_all = toks
    out["tokens_crc32"] = zlib.crc32(np.ascontiguousarray(toks_all, np.int32).tobytes())
    dec.close()
    steps = n_new - 1
    bytes_steps = sum(batch_step_bytes(cfg, n_seq, P + i, ws if vp is not None else 1) for i in range(steps))
    out.update({"decode_tokens_per_s": n_seq * steps / (dec_ms / 1e3),
                "decode_achieved_gbs": bytes_steps / (dec_ms / 1e3) / 1e9,
                "prefill_tokens_per_s": n_seq * P / (pre_ms / 1e3),
                "prefill_tflops": prefill_flops(cfg, n_seq, P) / (pre_ms / 1e3) / 1e12,
                "first_tokens": [int(t) for t in toks[0, :8]]})
    return out


def run_config1(local, capture, replay_ms, with_cpu):
    """One int8 per-row matvec, gate_proj 6144 x 2048, batch 1: device time (graph over rotating
    packed copies, each read from HBM), the host-pointer call (x in, y out), and the oracle port of
    the reference's Rayon matmul on the same shape."""
    import ctypes as C

    import numpy as np
    import torch

    import pyxis_b200 as px
    from pyxis_b200 import _native

    N, K = 6144, 2048
    dev = torch.device("cuda", local)
    bits = px.synth_normal_bf16(SEED + 7, N * K, 0.02)
    t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(dev)
    copies = [px.Weights.quantize_int8(t, K, device=local) for _ in range(24)]  # 24 x 12.6 MB > 2 x L2
    del t
    x = torch.from_numpy(px.synth_normal_f32(SEED + 8, K, 1.0)).to(dev).view(1, K)
    y = torch.empty((1, N), dtype=torch.float32, device=dev)

    def fn(st):
        for w in copies:
            px.matmul_dev(x, w, N, K, Y=y, stream=st)

    g = capture(fn)
    g.replay()
    us = replay_ms(g, 4) / (4 * len(copies)) * 1e3
    del g
    by = gemv_bytes("int8", N, K, K, 1)
    hx = torch.from_numpy(px.synth_normal_f32(SEED + 8, K, 1.0)).pin_memory()
    hy = torch.empty(N, dtype=torch.float32).pin_memory()
    L = _native.lib()
    w0 = copies[0]
    for _ in range(3):
        _native.check(L.pyxis_cuda_matmul(w0.ctx.handle, C.c_void_p(hx.data_ptr()), w0.handle, N, K,
                                          C.c_void_p(hy.data_ptr())))
    t0 = time.perf_counter()
    for _ in range(50):
        _native.check(L.pyxis_cuda_matmul(w0.ctx.handle, C.c_void_p(hx.data_ptr()), w0.handle, N, K,
                                          C.c_void_p(hy.data_ptr())))
    e2e_us = (time.perf_counter() - t0) / 50 * 1e6
    out = {"workload": "int8 per-row matvec, gate_proj 6144 x 2048, batch 1", "kernel": px.matmul_kernel_name(w0, 1, N, K),
           "device_us": round(us, 2), "device_gbs": round(by / us / 1e3, 1), "e2e_us": round(e2e_us, 2),
           "e2e_gbs": round(by / e2e_us / 1e3, 1)}
    if with_cpu:
        import oracle
        vals = oracle.bf16_to_f32(bits)
        d, sc = oracle.quantize_int8(vals, K)
        xs = px.synth_normal_f32(SEED + 8, K, 1.0).reshape(1, K)
        cores = oracle.num_cpus()
        oracle.matmul(xs, oracle.INT8, d, sc, K, N, K, nthreads=cores)
        times = []
        for _ in range(21):
            t0 = time.perf_counter()
            oracle.matmul(xs, oracle.INT8, d, sc, K, N, K, nthreads=cores)
            times.append(time.perf_counter() - t0)
        cpu_us = sorted(times)[len(times) // 2] * 1e6
        out["cpu_baseline"] = {"us": round(cpu_us, 1), "gbs": round(by / cpu_us / 1e3, 2), "cores": cores, "cpu": cpu_model(),
                               "kind": "port", "sample": "median of 21 calls through the C port on all host threads"}
    return out


def pyxis_arm(args, ws, rank, local):
    import numpy as np
    import torch

    import pyxis_b200 as px
    from pyxis_b200 import _native

    torch.cuda.set_device(local)
    ctx = px.get_cuda(local)
    if ctx is None:
        raise SystemExit("bench: no B200 visible: " + _native.lib().pyxis_cuda_last_error().decode())
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)

    weights = []
    for i, (name, qt, N, K, bs) in enumerate(SWEEP):
        bits = px.synth_normal_bf16(SEED + i, N * K, 0.02)
        t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(dev)
        w = px.Weights.quantize_int8(t, bs, device=local) if qt == "int8" else px.Weights.quantize_int4(t, bs, device=local)
        del t
        weights.append((name, qt, N, K, bs, w))
    X = {B: torch.from_numpy(px.synth_normal_f32(SEED + 100 + B, B * 6144, 1.0)).to(dev).view(B, 6144) for B in BATCHES}
    Y = {B: torch.empty((B, 151936), dtype=torch.float32, device=dev) for B in BATCHES}
    torch.cuda.synchronize()

    def step(st):
        for B in BATCHES:
            for (name, qt, N, K, bs, w) in weights:
                px.matmul_dev(X[B][:, :K], w, N, K, Y=Y[B][:, :N], stream=st)

    def capture(fn):
        """fn(stream) recorded once into a CUDA graph: replays run the same kernels with no
        host launch work between them (the decode loop runs its step the same way)."""
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            fn(s)  # first-call set-up (kernel attributes, tensor maps) outside the capture
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
            fn(s)
        torch.cuda.synchronize()
        return g

    def replay_ms(g, n):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(n):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    launches_per_step = len(BATCHES) * len(SWEEP)
    # eager reference result, then the captured step must reproduce it bit for bit
    step(stream)
    torch.cuda.synchronize()
    y_eager = {B: Y[B].clone() for B in BATCHES}
    g_step = capture(step)
    for B in BATCHES:
        Y[B].zero_()
    g_step.replay()
    torch.cuda.synchronize()
    for B in BATCHES:
        if not torch.equal(Y[B], y_eager[B]):
            raise SystemExit("bench: the captured sweep step does not reproduce the eager result")
    for _ in range(max(args.warmup, 3)):
        g_step.replay()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = ClockSampler(gpu_uuid(local))
    clocks.start()
    time.sleep(0.3)
    ms = replay_ms(g_step, args.steps)
    clk = clocks.stop()
    ms_max = max_over_ranks(ms, ws)
    barrier(ws)
    # the same steps launched one call at a time from Python (host-launch-bound at these sizes)
    eager_ms = 0.0
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    eager_ms = e0.elapsed_time(e1)
    eager_ms_max = max_over_ranks(eager_ms, ws)

    sb = step_bytes()
    value = ws * sb * args.steps / (ms_max / 1e3) / 1e9

    # per-case device time: a graph of R launches over enough packed copies of the matrix that
    # each launch reads it from HBM (copies x size > 2 x L2), as in the sweep
    cases = []
    lm_ms = None
    for B in BATCHES:
        for i, (name, qt, N, K, bs, w) in enumerate(weights):
            by = gemv_bytes(qt, N, K, bs, B)
            wbytes = N * K if qt == "int8" else N * K // 2
            ncopy = max(1, min(64, -(-(256 << 20) // wbytes)))
            copies = [w]
            if ncopy > 1:
                bits = px.synth_normal_bf16(SEED + i, N * K, 0.02)
                t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(dev)
                for _ in range(ncopy - 1):
                    copies.append(px.Weights.quantize_int8(t, bs, device=local) if qt == "int8"
                                  else px.Weights.quantize_int4(t, bs, device=local))
                del t
            reps = max(len(copies), 8)

            def case_fn(st, copies=copies, B=B, N=N, K=K, reps=reps):
                for r in range(reps):
                    px.matmul_dev(X[B][:, :K], copies[r % len(copies)], N, K, Y=Y[B][:, :N], stream=st)

            g = capture(case_fn)
            g.replay()
            us = replay_ms(g, 3) / (3 * reps) * 1e3
            del g, copies
            if name == "lm_head" and B == 1:
                lm_ms = us / 1e3
            cases.append({"case": f"{name} {qt} {N}x{K} B={B}", "kernel": px.matmul_kernel_name(w, B, N, K),
                          "us": round(us, 2), "gbs": round(by / us / 1e3, 1)})
    lm_bytes = gemv_bytes("int8", 151936, 2048, 2048, 1)
    peak, peak_kind = measured_peak_hbm()
    achieved = lm_bytes / (lm_ms / 1e3) / 1e9
    del g_step

    # e2e: the same sweep through the host-pointer C ABI (pinned host x in, host y out).
    hx = {B: torch.empty((B, 6144), dtype=torch.float32).pin_memory() for B in BATCHES}
    hy = {B: torch.empty((B, 151936), dtype=torch.float32).pin_memory() for B in BATCHES}
    for B in BATCHES:
        hx[B].copy_(X[B].cpu())
    h2d = sum(4 * B * K for B in BATCHES for (_, _, _, K, _) in SWEEP)
    d2h = sum(4 * B * N for B in BATCHES for (_, _, N, _, _) in SWEEP)
    L = _native.lib()
    import ctypes as C

    # contiguous pinned copies per K so the timed loop does no host-side slicing work
    xin_cache = {}
    for B in BATCHES:
        for K in {k for (_, _, _, k, _) in SWEEP}:
            t = torch.empty((B, K), dtype=torch.float32).pin_memory()
            t.copy_(hx[B][:, :K])
            xin_cache[(B, K)] = t

    def e2e_step_cached():
        for B in BATCHES:
            for (name, qt, N, K, bs, w) in weights:
                _native.check(L.pyxis_cuda_matmul_batch(ctx.handle, C.c_void_p(xin_cache[(B, K)].data_ptr()), B,
                                                        w.handle, N, K, C.c_void_p(hy[B].data_ptr())))

    e2e_step_cached()
    barrier(ws)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step_cached()
    e2e_s = max_over_ranks(time.perf_counter() - t0, ws)
    e2e_value = ws * sb * args.steps / e2e_s / 1e9

    config1 = run_config1(local, capture, replay_ms, rank == 0 and ws == 1 and not args.no_cpu_baseline)

    lm_vp = row_split = comm = comm_info = None
    if ws > 1:
        from pyxis_b200.dist import Comm
        comm = Comm(rank, ws, local)
        nr, rk = C.c_int(), C.c_int()
        _native.check(_native.lib().pyxis_cuda_comm_info(comm.handle, C.byref(nr), C.byref(rk)))
        comm_info = {"nranks": nr.value, "ranks_agree": max_over_ranks(0.0 if nr.value == ws else 1.0, ws) == 0.0,
                     "nccl_debug": os.environ.get("NCCL_DEBUG")}
        full = {name: w for (name, qt, N, K, bs, w) in weights}
        row_split = run_row_split(ws, rank, local, args.steps, capture, replay_ms, full)
        lm_vp = run_vocab_parallel_head(comm, ws, rank, local, args.steps, full["lm_head"])
        del full
    prefill = run_prefill(local)
    peak_tf = 0.0
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        peak_tf = float(pk.get("bf16_tflops", 0.0))
    except (OSError, ValueError):
        peak_tf = 1590.0
    for r in prefill:
        r["frac_of_bf16_peak"] = r["tflops"] / peak_tf if peak_tf else None

    decode = None
    if not args.no_decode:
        del weights, X, Y
        torch.cuda.empty_cache()
        decode = run_decode(local, cpu_sample_tokens=DECODE_CPU_TOKENS if rank == 0 and ws == 1 and
                            not args.no_cpu_baseline else 0)
        dsum = max_over_ranks(-decode["tokens_per_s"], ws)  # the slowest rank bounds the job
        decode["tokens_per_s_min_rank"] = -dsum
        decode["job_tokens_per_s"] = ws * (-dsum)
        peak_d, _ = measured_peak_hbm()
        decode["roofline_tokens_per_s"] = peak_d * 1e9 / decode["bytes_per_token"]
        decode["frac_of_peak"] = decode["achieved_gbs"] / peak_d

    batch = None
    if not args.no_batch_decode:
        torch.cuda.empty_cache()
        batch = run_batch_decode(local, ws, rank, comm=comm)
        if "vocab_parallel_parity" in batch:
            batch["vocab_parallel_parity"] = max_over_ranks(0.0 if batch["vocab_parallel_parity"] else 1.0, ws) == 0.0
        ms = max_over_ranks(batch["prefill_ms"] + batch["decode_ms"], ws)
        dmax = max_over_ranks(batch["decode_ms"], ws)
        pmax = max_over_ranks(batch["prefill_ms"], ws)
        peak_d, _ = measured_peak_hbm()
        batch.update({"job_decode_tokens_per_s": BATCH_SEQS * (BATCH_NEW - 1) / (dmax / 1e3),
                      "job_tokens_per_s": BATCH_SEQS * BATCH_NEW / (ms / 1e3),
                      "job_prefill_ms": pmax, "decode_frac_of_hbm_peak": batch["decode_achieved_gbs"] / peak_d,
                      "prefill_frac_of_bf16_peak": batch["prefill_tflops"] / (peak_tf or 1590.0)})

    if comm is not None:
        comm.close()
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        import oracle

        cores = oracle.num_cpus()
        t, b = run_cpu_sweep(cores)
        cpu = {"value": b / t / 1e9, "unit": UNIT, "cores": cores, "cpu": cpu_model(), "kind": "port",
               "sample": "one full sweep step (12 matvec calls, 6.1 GB of int4/int8 rows incl. batch-8 re-reads) "
                         "through the C port of the reference's Rayon matmul, all host threads"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config_dict(ws),
                "roofline": {"bound": "hbm", "kernel": "gemv_tc_i8_kernel (lm_head int8 151936x2048, batch 1)",
                             "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": profiled_traffic("gemv_tc_i8_lm_head"),
                             "algorithmic_bytes_per_launch": lm_bytes, "avg_launch_us": lm_ms * 1e3},
                "frac_of_peak_step": value / ws / peak,
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "cpu_baseline": cpu, "clocks": clk, "gpu_launches": launches_per_step * args.steps,
                "eager_ms_per_step": eager_ms_max / args.steps,
                "cases": cases,
                "config1": config1,
                "decode": decode,
                "batch_decode": batch,
                "lm_head_vocab_parallel": lm_vp,
                "row_split": row_split,
                "comm": comm_info,
                "parity": None if ws == 1 else {
                    "row_split": row_split["parity"], "vocab_parallel": lm_vp["parity"],
                    "batch_decode_vocab_parallel": None if batch is None else batch.get("vocab_parallel_parity")},
                "prefill": {"M": PREFILL_M, "kernel": "split_x_kernel + gemm_tc_kernel (tcgen05 kind::f16, fp16 hi/lo)",
                            "peak_tflops": peak_tf, "peak_kind": "measured bf16 burst", "shapes": prefill},
                "per_gpu_value": value / ws}
        return line
    return None


def profile_case(args):
    """A single GEMV shape, launched warmup + steps times: the target of the committed ncu
    captures (profiles/*.txt name the exact command)."""
    import numpy as np
    import torch

    import pyxis_b200 as px

    if args.profile_case.startswith("batch"):
        parts = [int(v) for v in args.profile_case.split(":")[1:]]
        n_seq, P, n_new = (parts + [BATCH_SEQS, BATCH_PROMPT, BATCH_NEW][len(parts):])[:3]
        r = run_batch_decode(0, 1, 0, n_seq_total=n_seq, P=P, n_new=n_new)
        print(f"profile case batch: {n_seq} x {P} prompt + {n_new} new: prefill {r['prefill_ms']:.1f} ms "
              f"({r['prefill_tflops']:.1f} TFLOP/s), decode {r['decode_ms']:.1f} ms "
              f"({r['decode_tokens_per_s']:.0f} tok/s, {r['decode_achieved_gbs']:.0f} GB/s)")
        return
    if args.profile_case.startswith("decode"):
        from pyxis_b200 import synth_tokens
        from pyxis_b200.model import QWEN3_1_7B, Decoder, SyntheticModel
        ctx = int(args.profile_case.split(":")[1]) if ":" in args.profile_case else 2  # prompt length
        n = max(2, args.steps + 1)
        dec = Decoder(SyntheticModel(QWEN3_1_7B, SEED), qtype="int8", max_seq=ctx + n + 8)
        prompt = synth_tokens(0x9E0, ctx, QWEN3_1_7B.vocab)
        dec.generate(prompt[:2], 2)
        toks, t = dec.generate(prompt, n)
        print(f"profile case decode: prompt {ctx}, {n - 1} steps, prompt {t[0]:.2f} ms, "
              f"decode {t[1] / (n - 1):.3f} ms/token")
        return
    if args.profile_case == "sweep":
        # the timed step's 12 GEMV launches (every SWEEP matrix at batch 1 and 8), eagerly
        ws_ = {}
        for i, (name, qt, N, K, bs) in enumerate(SWEEP):
            bits = px.synth_normal_bf16(SEED + i, N * K, 0.02)
            t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
            ws_[name] = px.Weights.quantize_int8(t, bs) if qt == "int8" else px.Weights.quantize_int4(t, bs)
            del t
        X = {B: torch.from_numpy(px.synth_normal_f32(SEED + 100 + B, B * 6144, 1.0)).cuda().view(B, 6144)
             for B in BATCHES}
        Y = {B: torch.empty((B, 151936), dtype=torch.float32, device="cuda") for B in BATCHES}
        for _ in range(args.warmup + args.steps):
            for B in BATCHES:
                for (name, qt, N, K, bs) in SWEEP:
                    px.matmul_dev(X[B][:, :K], ws_[name], N, K, Y=Y[B][:, :N])
        torch.cuda.synchronize()
        print(f"profile case sweep: {args.warmup + args.steps} steps of {len(SWEEP) * len(BATCHES)} launches")
        return
    if args.profile_case.startswith("prefill"):
        # one prefill GEMM: prefill:<int8|int4>:<gate|down>:<M>
        _, qt, which, M = args.profile_case.split(":")
        M = int(M)
        (name, _, N, K, bs) = next(s for s in PREFILL_SHAPES if s[0] == f"{which}_proj {qt}")
        bits = px.synth_normal_bf16(SEED + 50, N * K, 0.02)
        t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
        w = px.Weights.quantize_int8(t, bs) if qt == "int8" else px.Weights.quantize_int4(t, bs)
        X = torch.from_numpy(px.synth_normal_f32(SEED + 60, M * K, 1.0)).cuda().view(M, K)
        Y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        for _ in range(args.warmup + args.steps):
            px.matmul_dev(X, w, N, K, Y=Y)
        torch.cuda.synchronize()
        print(f"profile case {name} M={M}: {px.matmul_kernel_name(w, M, N, K)}, {args.warmup + args.steps} launches")
        return
    name, B = args.profile_case.split(":") if ":" in args.profile_case else (args.profile_case, "1")
    B = int(B)
    (_, qt, N, K, bs) = next(m for m in SWEEP if m[0] == name)
    bits = px.synth_normal_bf16(SEED, N * K, 0.02)
    t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    w = px.Weights.quantize_int8(t, bs) if qt == "int8" else px.Weights.quantize_int4(t, bs)
    X = torch.from_numpy(px.synth_normal_f32(SEED + 100 + B, B * K, 1.0)).cuda().view(B, K)
    Y = torch.empty((B, N), dtype=torch.float32, device="cuda")
    for _ in range(args.warmup + args.steps):
        px.matmul_dev(X, w, N, K, Y=Y)
    torch.cuda.synchronize()
    print(f"profile case {name} B={B}: {qt} {N}x{K} block {bs}, {args.warmup + args.steps} launches")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile-case", default=None,
                    help="run one shape only, for ncu: lm_head:1, gate_proj:8, sweep (the timed step's "
                         "12 GEMVs), prefill:int4:gate:512, decode:CTX, batch:SEQS:PROMPT:NEW")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["pyxis", "reference"], default="pyxis")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the Qwen3-1.7B-shape greedy decode measurement")
    ap.add_argument("--no-batch-decode", action="store_true",
                    help="skip the 64-sequence int4 batched decode measurement")
    args = ap.parse_args()
    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        from oracle import build as ob

        ob.build()
        reference_arm(args, ws, rank)
        return
    from pyxis_b200 import build as pb

    pb.build()
    from oracle import build as ob

    ob.build()
    if args.profile_case:
        profile_case(args)
        return
    ws, rank, local = dist_setup()
    line = None
    try:
        line = pyxis_arm(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if line is not None:  # last on stdout, after NCCL's own lines
        sys.stdout.flush()
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
