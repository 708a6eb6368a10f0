"""Host logic of the multi-GPU sharding (pyxis_b200/dist.py), on CPU: shard ranges, the
vocab-parallel key scheme (a numpy restatement of the device keys, tests/keys.py) against the
oracle's argmax (src/output_head.rs:30-44), and over a world-size-2 gloo group the communicator-id
exchange and the all-gather + pick of the keys."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from keys import epilogue_key, pick, shard_key
from pyxis_b200.dist import bits_rows, exchange_comm_id, shard_range


@pytest.mark.parametrize("n,world", [(10, 3), (151936, 8), (7, 7), (1, 1), (100, 2)])
def test_shard_range_partitions(n, world):
    parts = [shard_range(n, r, world) for r in range(world)]
    assert parts[0][0] == 0 and parts[-1][1] == n
    for (a, b), (c, d) in zip(parts, parts[1:]):
        assert b == c and a <= b
    assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_key_pick_matches_reference_argmax(world):
    rng = np.random.default_rng(world)
    for trial in range(200):
        n = int(rng.integers(1, 60))
        v = rng.integers(-3, 4, size=n).astype(np.float32)  # many ties
        if trial % 3 == 0:
            v[rng.integers(0, n)] = -0.0 if trial % 2 else 0.0
        if trial % 5 == 0:
            v[rng.integers(0, n)] = np.nan
        if trial % 11 == 0:
            v[rng.integers(0, n)] = np.inf if trial % 2 else -np.inf
        if trial % 17 == 0:
            v[0] = np.nan
        if trial % 23 == 0:
            v[:] = np.nan
        keys = [shard_key(v[lo:hi], lo) for lo, hi in (shard_range(n, r, world) for r in range(world)) if hi > lo]
        assert pick(keys) == oracle.argmax(v), (v, keys)


@pytest.mark.parametrize("world", [1, 2, 5])
def test_epilogue_keys_equal_the_scan_keys(world):
    """The key the tensor-core GEMV's epilogue builds for a shard (every logit's key at its global
    index, max-reduced in any grouping and order into a zeroed slot) equals the scan's shard key
    (launch_argmax_keys: the shard's first maximum, then its global index), so the fused head picks
    the same token: NaN at global index 0, NaNs elsewhere, ties across shards, -0.0 / +0.0."""
    rng = np.random.default_rng(10 + world)
    for trial in range(200):
        n = int(rng.integers(1, 50))
        v = rng.integers(-2, 3, size=n).astype(np.float32)
        if trial % 3 == 0:
            v[rng.integers(0, n)] = -0.0
        if trial % 4 == 0:
            v[rng.integers(0, n)] = np.nan
        if trial % 13 == 0:
            v[0] = np.nan
        if trial % 19 == 0:
            v[:] = np.nan
        shards = [(lo, hi) for lo, hi in (shard_range(n, r, world) for r in range(world)) if hi > lo]
        fused = [epilogue_key(v[lo:hi], lo, rng) for lo, hi in shards]
        scan = [shard_key(v[lo:hi], lo) for lo, hi in shards]
        assert fused == scan, (v, fused, scan)
        assert pick(fused) == oracle.argmax(v)


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
    # the communicator id made on rank 0 reaches every rank unchanged
    uid = exchange_comm_id(rank, make_id=lambda: bytes(range(128)))
    rng = np.random.default_rng(0)
    M, V = 3, 1001
    logits = rng.standard_normal((M, V)).astype(np.float32)
    logits[1, 5] = logits[1, 900] = 50.0  # a tie across the shard boundary: index 5 wins
    logits[2, 0] = np.nan  # NaN at index 0: index 0 wins
    lo, hi = shard_range(V, rank, world)
    # 64-bit keys travel as int64 bit patterns, as the device keys do through NCCL
    mine = torch.from_numpy(np.array([shard_key(logits[m, lo:hi], lo) for m in range(M)], np.uint64).view(np.int64))
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    got = [pick([int(p.numpy().view(np.uint64)[m]) for p in parts]) for m in range(M)]
    want = [oracle.argmax(logits[m]) for m in range(M)]
    q.put((rank, uid == bytes(range(128)), got, want))
    dist.destroy_process_group()


def test_key_gather_pick_over_gloo_world2():
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
    for rank, id_ok, got, want in res:
        assert id_ok, rank
        assert got == want, (rank, got, want)
