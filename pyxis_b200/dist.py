"""Multi-GPU sharding of the quantized matmul path (one process per GPU, torch.distributed).

Only the parts that shard naturally are split; nothing here reduces partial sums:
  * row-sharded matmul: rank r owns output rows [r*N/n, (r+1)*N/n) of a matrix.  With one scale
    per row (int8) or per 32 values (int4, in_features a multiple of 32) a row block's packed bytes
    and scales are exactly that slice of the full pack, so each rank quantises only its rows and
    the outputs concatenate to the single-GPU result (optionally all-gathered, NCCL over NVLink).
  * vocab-parallel lm_head + greedy argmax (src/output_head.rs:21-44): each rank computes the
    logits of its vocab shard, takes their argmax on the device (index offset by the shard start),
    and the ranks all-gather one (value, index) pair each; the winner is the largest value, the
    lowest index on ties -- the first maximum, as the reference's strict `>` scan picks it.
  * independent decode sequences: data-parallel replicas (bench.py), no collective.
"""
from __future__ import annotations

import numpy as np


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [lo, hi) of an n-row matrix that `rank` owns (contiguous, sizes differ by <= 1)."""
    lo = (n * rank) // world
    hi = (n * (rank + 1)) // world
    return lo, hi


def pick_global_argmax(vals, idxs) -> int:
    """The first maximum over the per-shard (value, index) pairs: largest value, lowest index on
    ties.  A NaN value never wins (the reference's `value > max_value` is false for NaN) unless the
    global first element is NaN, which the shard holding index 0 reports as its own answer."""
    vals = np.asarray(vals, np.float64)
    idxs = np.asarray(idxs, np.int64)
    if idxs.size == 0:
        raise ValueError("no shards")
    # index 0 holds NaN: the reference never moves off it
    first = np.argmin(idxs)
    if idxs[first] == 0 and np.isnan(vals[first]):
        return 0
    best = None
    for v, i in zip(vals, idxs):
        if np.isnan(v):
            continue
        if best is None or v > best[0] or (v == best[0] and i < best[1]):
            best = (v, i)
    return int(best[1]) if best is not None else 0


class RowShardedMatmul:
    """One rank's row block of a quantized matrix: ``forward`` gives this rank's outputs, and
    ``forward_gathered`` all-gathers them into the full output on every rank."""

    def __init__(self, bf16_bits: np.ndarray, out_features: int, in_features: int, qtype: str, rank: int,
                 world: int, device: int):
        import torch

        from . import Weights

        self.N, self.K, self.rank, self.world = out_features, in_features, rank, world
        self.lo, self.hi = shard_range(out_features, rank, world)
        rows = bits_rows(bf16_bits, in_features, self.lo, self.hi)
        t = torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(f"cuda:{device}")
        if qtype == "int8":
            self.w = Weights.quantize_int8(t, in_features, device=device)
        else:
            self.w = Weights.quantize_int4(t, 32, device=device)
        self.device = device

    def forward(self, X):
        from . import matmul_dev
        return matmul_dev(X, self.w, self.hi - self.lo, self.K)

    def forward_gathered(self, X, group=None):
        import torch
        import torch.distributed as dist

        local = self.forward(X)
        sizes = [shard_range(self.N, r, self.world) for r in range(self.world)]
        width = max(hi - lo for lo, hi in sizes)
        pad = torch.zeros((local.shape[0], width), dtype=local.dtype, device=local.device)
        pad[:, : local.shape[1]] = local
        parts = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(parts, pad, group=group)
        return torch.cat([p[:, : hi - lo] for p, (lo, hi) in zip(parts, sizes)], dim=1)


def bits_rows(bits: np.ndarray, in_features: int, lo: int, hi: int) -> np.ndarray:
    return np.ascontiguousarray(bits.reshape(-1, in_features)[lo:hi]).ravel()


class VocabParallelHead:
    """The lm_head split by vocabulary rows across the ranks, with the distributed greedy argmax."""

    def __init__(self, bf16_bits: np.ndarray, vocab: int, hidden: int, qtype: str, rank: int, world: int,
                 device: int):
        self.mm = RowShardedMatmul(bf16_bits, vocab, hidden, qtype, rank, world, device)
        self.vocab = vocab

    def greedy(self, h, group=None):
        """Next-token ids [M] on every rank for hidden states h [M, hidden] (device tensor)."""
        from . import argmax_dev

        logits = self.mm.forward(h)
        idx, val = argmax_dev(logits, index_base=self.mm.lo)
        return gather_pick(val, idx, self.mm.world, group)


def gather_pick(val, idx, world: int, group=None) -> np.ndarray:
    """All-gather each rank's per-row (value, index) shard argmax and pick the global first
    maximum on every rank (works for CUDA tensors over NCCL and CPU tensors over gloo)."""
    import torch
    import torch.distributed as dist

    pair = torch.stack([val.to(torch.float64), idx.to(torch.float64)], dim=1)  # [M, 2]
    parts = [torch.empty_like(pair) for _ in range(world)]
    dist.all_gather(parts, pair, group=group)
    allp = torch.stack(parts, dim=0).cpu().numpy()  # [world, M, 2]
    return np.array([pick_global_argmax(allp[:, m, 0], allp[:, m, 1]) for m in range(allp.shape[1])],
                    dtype=np.int64)
