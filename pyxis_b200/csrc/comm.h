// comm.h -- the communicator handle behind include/pyxis_comm.h, shared by comm.cu and
// decode_batch.cu.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/pyxis_comm.h"
#include "ctx.h"

struct pyxis_cuda_comm {
    pyxis_cuda_ctx *ctx = nullptr;
    int nranks = 1, rank = 0;
    ncclComm_t nccl = nullptr;
    // head buffers, grown by pyxis::head_reserve: logits [rows][shard rows], this rank's keys
    // [rows] followed by every rank's [nranks][rows]
    float *logits = nullptr;
    size_t logits_cap = 0;
    uint64_t *keys = nullptr;
    size_t keys_cap = 0;
    // peer-memory exchange of the head's keys (comm.cu): this rank's receive buffer (mapped into
    // every peer by CUDA IPC), the peers' mappings, and a device table of the nranks buffers
    bool p2p = false;
    void *xbuf = nullptr;                 // local: keys [2 epochs][nranks][kXMaxRows], flags, epoch
    void *peer_base[8] = {nullptr};       // IPC mappings of the peers' xbuf (nullptr for self)
    void **xtable = nullptr;              // device [nranks] pointers to every rank's xbuf
};

namespace pyxis {
// ncclAllGather of `count` elements (f32 or u64) per rank into recv [nranks][count], on st.
int comm_allgather(pyxis_cuda_comm *c, const void *send, void *recv, size_t count, bool u64, cudaStream_t st);
// Grows the head buffers for M rows of shard_rows logits (allocates: not during capture).
int head_reserve(pyxis_cuda_comm *c, size_t M, size_t shard_rows);
// Enqueues the vocab-parallel head on st for M gathered rows X [M, hidden] (the same on every
// rank): logits of this rank's shard, keys, the keys' all-gather, then tokens[r] for the rows
// [row0, row0 + nrows) of X.  The buffers must already hold M rows (head_reserve).
int head_greedy_enqueue(pyxis_cuda_comm *c, const pyxis_cuda_weights *shard, size_t vocab_lo, size_t shard_rows,
                        size_t hidden, const float *X, size_t M, size_t ldx, int row0, int nrows, int32_t *tokens,
                        void *ws, size_t ws_bytes, cudaStream_t st);
}  // namespace pyxis
