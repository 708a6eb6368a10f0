"""Host logic of the multi-GPU sharding (pyxis_b200/dist.py), on CPU: shard ranges, the global
first-maximum pick across vocab shards (against the oracle's argmax, src/output_head.rs:30-44),
and the all-gather + pick over a world-size-2 gloo group."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from pyxis_b200.dist import bits_rows, gather_pick, pick_global_argmax, shard_range


def shard_argmax(v, lo):
    """What argmax_kernel returns for one shard: first max, NaNs skipped except a NaN at global
    index 0 (only the shard with lo == 0 applies that rule)."""
    if lo == 0 and np.isnan(v[0]):
        return np.nan, 0
    best = None
    for i, x in enumerate(v):
        if np.isnan(x):
            continue
        if best is None or x > best[0]:
            best = (x, i)
    if best is None:
        return np.nan, lo
    return best[0], lo + best[1]


@pytest.mark.parametrize("n,world", [(10, 3), (151936, 8), (7, 7), (1, 1), (100, 2)])
def test_shard_range_partitions(n, world):
    parts = [shard_range(n, r, world) for r in range(world)]
    assert parts[0][0] == 0 and parts[-1][1] == n
    for (a, b), (c, d) in zip(parts, parts[1:]):
        assert b == c and a <= b
    assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_global_pick_matches_reference_argmax(world):
    rng = np.random.default_rng(world)
    for trial in range(200):
        n = int(rng.integers(1, 60))
        v = rng.integers(-3, 4, size=n).astype(np.float32)  # many ties
        if trial % 5 == 0:
            v[rng.integers(0, n)] = np.nan
        if trial % 17 == 0:
            v[0] = np.nan
        if trial % 23 == 0:
            v[:] = np.nan
        pairs = [shard_argmax(v[lo:hi], lo) for lo, hi in (shard_range(n, r, world) for r in range(world)) if hi > lo]
        got = pick_global_argmax([p[0] for p in pairs], [p[1] for p in pairs])
        assert got == oracle.argmax(v), (v, pairs, got)


@pytest.mark.parametrize("qt,N,K,bs", [("int8", 37, 96, 96), ("int4", 37, 96, 32), ("int4", 10, 2048, 32),
                                        ("int8", 300, 64, 64)])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_row_shard_packs_are_slices_of_the_full_pack(qt, N, K, bs, world):
    """A rank quantises only its rows (RowShardedMatmul): with one scale per row, or groups that
    divide the row (K % 32 == 0, K even for int4's two codes per byte), the shard's bytes and
    scales are exactly the rows' slice of the full matrix's pack, so the shards' outputs
    concatenate to the single-GPU result."""
    from pyxis_b200 import synth_normal_bf16
    bits = synth_normal_bf16(N * 31 + K, N * K, 0.02)
    quant = oracle.quantize_int8 if qt == "int8" else oracle.quantize_int4
    full_d, full_s = quant(oracle.bf16_to_f32(bits), bs)
    row_bytes = K if qt == "int8" else K // 2
    for r in range(world):
        lo, hi = shard_range(N, r, world)
        d, s = quant(oracle.bf16_to_f32(bits_rows(bits, K, lo, hi)), bs)
        assert np.array_equal(d.view(np.uint8), full_d.view(np.uint8)[lo * row_bytes:hi * row_bytes])
        spr = K // bs
        assert np.array_equal(s.view(np.uint32), full_s.view(np.uint32)[lo * spr:hi * spr])


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    M, V = 3, 1001
    logits = rng.standard_normal((M, V)).astype(np.float32)
    logits[1, 5] = logits[1, 900] = 50.0  # a tie across the shard boundary: index 5 wins
    lo, hi = shard_range(V, rank, world)
    vals, idxs = zip(*[shard_argmax(logits[m, lo:hi], lo) for m in range(M)])
    got = gather_pick(torch.tensor(vals, dtype=torch.float32), torch.tensor(idxs, dtype=torch.int32), world)
    want = [oracle.argmax(logits[m]) for m in range(M)]
    q.put((rank, list(got), want))
    dist.destroy_process_group()


def test_gather_pick_over_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, want in res:
        assert got == want, (rank, got, want)
