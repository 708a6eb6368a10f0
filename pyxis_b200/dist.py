"""Multi-GPU sharding of the quantized matmul path (one process per GPU, torch.distributed for the
rendezvous, NCCL over NVLink for the data; include/pyxis_comm.h).

Only the parts that shard naturally are split; nothing here reduces partial sums:
  * row-sharded matmul: rank r owns output rows [r*N/n, (r+1)*N/n) of a matrix.  With one scale
    per row (int8) or per 32 values (int4, in_features a multiple of 32) a row block's packed bytes
    and scales are exactly that slice of the full pack, so each rank quantises only its rows and
    the outputs concatenate to the single-GPU result -- bit for bit where the shard takes the full
    matrix's kernel (kernels are chosen by size) -- optionally all-gathered (NCCL over NVLink).
  * vocab-parallel lm_head + greedy argmax (src/output_head.rs:21-44): each rank computes the
    logits of its vocab shard and reduces every row to one 64-bit key on the device
    (order-preserving value bits, then the inverted global index); the ranks all-gather the keys
    and the largest key of a row is the reference's first maximum, so every rank ends with the
    same token, on the device, with no host round trip.
  * independent decode sequences: data-parallel, the lm_head of the batched decode vocab-parallel
    (``Decoder(..., vocab_parallel=comm)``, pyxis_cuda_model_set_vocab_parallel).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native
from ._native import check


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [lo, hi) of an n-row matrix that `rank` owns (contiguous, sizes differ by <= 1)."""
    lo = (n * rank) // world
    hi = (n * (rank + 1)) // world
    return lo, hi


def bits_rows(bits: np.ndarray, in_features: int, lo: int, hi: int) -> np.ndarray:
    return np.ascontiguousarray(bits.reshape(-1, in_features)[lo:hi]).ravel()


def exchange_comm_id(rank: int, make_id=None, group=None) -> bytes:
    """The 128-byte communicator id made on rank 0 (pyxis_cuda_comm_unique_id) and broadcast to
    every rank over the torch.distributed group (gloo or NCCL)."""
    import torch.distributed as dist

    if make_id is None:
        def make_id():
            buf = (C.c_uint8 * 128)()
            check(_native.lib().pyxis_cuda_comm_unique_id(buf))
            return bytes(buf)
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise ValueError("communicator id must be 128 bytes")
    return bytes(uid)


class Comm:
    """A communicator of the library (pyxis_cuda_comm_init) on this rank's context: the ranks of
    the current torch.distributed group, one per GPU."""

    def __init__(self, rank: int, world: int, device: int, group=None):
        from . import _require_cuda

        self.ctx = _require_cuda(device)
        self.rank, self.world, self.device = rank, world, device
        uid = exchange_comm_id(rank, group=group)
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        h = C.c_void_p()
        check(_native.lib().pyxis_cuda_comm_init(self.ctx.handle, buf, world, rank, C.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            _native.lib().pyxis_cuda_comm_free(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


class RowShardedMatmul:
    """One rank's row block of a quantized matrix: ``forward`` gives this rank's outputs, and
    ``forward_gathered`` all-gathers them into the full output on every rank."""

    def __init__(self, bf16_bits: np.ndarray, out_features: int, in_features: int, qtype: str, rank: int,
                 world: int, device: int, block_size: int | None = None):
        import torch

        from . import Weights

        self.N, self.K, self.rank, self.world = out_features, in_features, rank, world
        self.lo, self.hi = shard_range(out_features, rank, world)
        rows = bits_rows(bf16_bits, in_features, self.lo, self.hi)
        t = torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(f"cuda:{device}")
        bs = block_size or (in_features if qtype == "int8" else 32)
        self.w = Weights.quantize_int8(t, bs, device=device) if qtype == "int8" else \
            Weights.quantize_int4(t, bs, device=device)
        self.device = device

    def forward(self, X, Y=None, stream=None):
        from . import matmul_dev
        return matmul_dev(X, self.w, self.hi - self.lo, self.K, Y=Y, stream=stream)

    def forward_gathered(self, X, group=None):
        import torch
        import torch.distributed as dist

        local = self.forward(X)
        sizes = [shard_range(self.N, r, self.world) for r in range(self.world)]
        width = max(hi - lo for lo, hi in sizes)
        pad = torch.zeros((local.shape[0], width), dtype=local.dtype, device=local.device)
        pad[:, : local.shape[1]] = local
        parts = torch.empty((self.world,) + tuple(pad.shape), dtype=pad.dtype, device=pad.device)
        dist.all_gather_into_tensor(parts, pad, group=group)
        return torch.cat([parts[r, :, : hi - lo] for r, (lo, hi) in enumerate(sizes)], dim=1)


class VocabParallelHead:
    """The lm_head split by vocabulary rows across the ranks, with the distributed greedy argmax
    (pyxis_cuda_head_greedy_dev)."""

    def __init__(self, bf16_bits: np.ndarray, vocab: int, hidden: int, qtype: str, comm: Comm,
                 block_size: int | None = None):
        self.comm = comm
        self.mm = RowShardedMatmul(bf16_bits, vocab, hidden, qtype, comm.rank, comm.world, comm.device,
                                   block_size=block_size)
        self.vocab, self.hidden = vocab, hidden

    def greedy(self, h, tokens=None, stream=None):
        """Next-token ids (int32 CUDA tensor [M], the same on every rank) for hidden states h
        [M, hidden] (CUDA f32, the same rows on every rank).  Asynchronous on ``stream``."""
        import torch

        from . import _stream_handle

        if h.dim() == 1:
            h = h.unsqueeze(0)
        M = h.shape[0]
        if tokens is None:
            tokens = torch.empty(M, dtype=torch.int32, device=h.device)
        st = _stream_handle(stream, h.device)
        check(_native.lib().pyxis_cuda_head_greedy_dev(self.comm.handle, self.mm.w.handle, self.vocab, self.mm.lo,
                                                       self.mm.hi - self.mm.lo, self.hidden, C.c_void_p(h.data_ptr()),
                                                       M, h.stride(0), C.c_void_p(tokens.data_ptr()), C.c_void_p(st)))
        return tokens
