"""The bench's JSON line is a contract with whoever runs it: one line, fixed keys, the
reference arm on the same metric as the CUDA arm.  These checks run on the CPU: the reference arm (the
oracle port of the reference's Rayon matmul) needs no GPU, and the byte counts behind every
GB/s and roofline figure are plain arithmetic."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _run_reference(env_extra):
    env = dict(os.environ, **env_extra)
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    return [l for l in out.stdout.splitlines() if l.strip()]


def test_reference_arm_prints_one_contract_line():
    lines = _run_reference({"WORLD_SIZE": "1", "RANK": "0"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "GB/s"
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["vs_baseline"] is None
    assert d["config"]["workload"] == bench.WORKLOAD
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"] and cb["cpu"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == "GB/s" and e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    """Under torchrun only rank 0 runs the CPU sweep and prints; the other ranks exit 0 quietly."""
    assert _run_reference({"WORLD_SIZE": "2", "RANK": "1"}) == []


def test_algorithmic_bytes():
    """codes + scales + x + y per GEMV: the numbers the GB/s values and the roofline divide by."""
    # int8 per-row gate_proj 6144 x 2048 at batch 1: N K + 4 N + 4 K + 4 N
    assert bench.gemv_bytes("int8", 6144, 2048, 2048, 1) == 12_640_256
    # the lm_head launch the roofline reports: 151936 x 2048 int8 per row, batch 1
    assert bench.gemv_bytes("int8", 151936, 2048, 2048, 1) == 312_388_608
    # int4 group 32: N K / 2 + 4 N K / 32 + 4 B (K + N)
    assert bench.gemv_bytes("int4", 2048, 2048, 32, 8) == 2048 * 2048 // 2 + 4 * 2048 * 2048 // 32 + 4 * 8 * 4096
    assert bench.step_bytes() == sum(bench.gemv_bytes(qt, N, K, bs, B) for B in bench.BATCHES
                                     for (_, qt, N, K, bs) in bench.SWEEP)
    assert 0.6e9 < bench.step_bytes() < 0.8e9  # "0.68 GB of packed weights" per step


def test_decode_and_batch_step_bytes():
    """The bytes behind the decode GB/s figures, Qwen3-1.7B shape."""
    from pyxis_b200.model import QWEN3_1_7B as c
    layer_int8 = 50_331_648 + 81_920          # 7 projections' codes + one f32 scale per row
    lm_head_int8 = 151936 * 2048 + 151936 * 4
    kv_per_pos = 28 * 2 * 1024 * 4            # f32 K and V rows of every layer: 229,376 B
    for pos in (0, 15, 143):
        # int8 single-sequence step: all weights once, the KV rows 0..pos, one bf16 embedding row
        assert bench.decode_bytes_per_token(c, pos) == 28 * layer_int8 + lm_head_int8 + kv_per_pos * (pos + 1) + 2 * 2048
    weights_int4 = 28 * 31_457_280 + 151936 * 2048 * 5 // 8   # codes + group-32 f32 scales, lm_head int4
    for n_seq, pos in ((1, 0), (64, 2047), (8, 2302)):
        assert bench.batch_step_bytes(c, n_seq, pos) == weights_int4 + n_seq * kv_per_pos * (pos + 1)


def _fake_smi(tmp_path, lines):
    script = tmp_path / "nvidia-smi"
    body = "\n".join(f"echo '{l}'" for l in lines)
    script.write_text(f"#!/bin/bash\nwhile true; do\n{body}\nsleep 0.05\ndone\n")
    script.chmod(0o755)
    return str(tmp_path)


def test_clock_sampler_reads_clocks_and_throttle_reasons(tmp_path, monkeypatch):
    """The clocks record beside every number: median SM clock under load, the maximum, and any
    throttle reason nvidia-smi reports Active (from a stand-in nvidia-smi on PATH)."""
    lines = ["0, 1965, 1965, 700.5, 0x0, Not Active, Not Active, Not Active, Not Active",
             "0, 1800, 1965, 990.1, 0x4, Not Active, Not Active, Not Active, Active",
             "0, 1700, 1965, 1001.0, 0x8, Active, Not Active, Not Active, Active"]
    monkeypatch.setenv("PATH", _fake_smi(tmp_path, lines) + os.pathsep + os.environ["PATH"])
    s = bench.ClockSampler("0")
    s.start()
    import time
    time.sleep(0.5)
    r = s.stop()
    assert r["samples"] >= 3 and r["sm_max_mhz"] == 1965.0
    assert 1700.0 <= r["sm_mhz"] <= 1965.0
    assert r["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    s = bench.ClockSampler(None)
    s.start()
    assert s.stop()["reasons"] == ["nvidia-smi unavailable"]


def _max_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, bench.max_over_ranks(1.5 + rank * 2.25, world)))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_world2():
    """Every rank reports the slowest rank's time: the job's time under torchrun."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_max_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got == {0: 3.75, 1: 3.75}


def test_reference_arm_loads_no_cuda_library():
    """The CPU arm makes its seeded inputs with the oracle's copy of the generator: the CUDA
    library is never mapped into the reference process."""
    code = ("import sys, types; sys.path.insert(0, %r); import bench; "
            "bench.reference_arm(types.SimpleNamespace(steps=1, warmup=0), 1, 0); "
            "maps = open('/proc/self/maps').read(); "
            "print('CUDA_LIB_MAPPED' if 'libpyxis_cuda' in maps else 'CUDA_LIB_ABSENT')") % ROOT
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "CUDA_LIB_ABSENT" in out.stdout, out.stdout[-500:]
