/*
 * pyxis_comm.h -- the multi-GPU part of the quantized path: one process per GPU, NCCL over
 * NVLink / NVSwitch for the one exchange the path has.
 *
 * The reference runs on one device; its lm_head (src/output_head.rs:21-44: logits = matmul of
 * the final hidden state with the [vocab, hidden] head, then argmax) is the path's only step
 * whose work splits across GPUs with an exchange.  Split by vocabulary rows, each rank computes
 * the logits of its rows and their argmax; an exchange of a 64-bit key per (row, rank) and a
 * device-side maximum give every rank the token the single-device argmax picks (the first
 * maximum under strict >, a NaN at index 0 winning as it does in the reference's scan).  The
 * exchange is one kernel over peer memory when the ranks' GPUs can map each other's memory
 * (CUDA IPC, set up by pyxis_cuda_comm_init), else an NCCL all-gather.
 *
 * Row-sharded matmuls and data-parallel sequences need no library support: a rank quantises its
 * own row block with pyxis_cuda_quantize (the block's bytes and scales are exactly that slice of
 * the full pack) and multiplies it with pyxis_cuda_matmul_dev.
 *
 * NCCL is loaded at run time (dlopen of libnccl.so.2: the copy already in the process when
 * there is one); the other entry points of the library work without it.
 */
#ifndef PYXIS_COMM_H
#define PYXIS_COMM_H

#include <stddef.h>
#include <stdint.h>

#include "pyxis_cuda.h"
#include "pyxis_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

#define PYXIS_COMM_ID_BYTES 128

typedef struct pyxis_cuda_comm pyxis_cuda_comm;

/* A new communicator id (ncclGetUniqueId).  One rank makes it and sends the 128 bytes to the
 * others by any host channel (a store, MPI, a file); PYXIS_EUNSUPPORTED if NCCL cannot be
 * loaded. */
int pyxis_cuda_comm_unique_id(uint8_t id[PYXIS_COMM_ID_BYTES]);

/* Joins `nranks` processes (rank 0..nranks-1, one per GPU) into a communicator on ctx's device.
 * Every rank must call it with the same id; it returns when all have joined.  Collectives of the
 * communicator run on the stream each call is given, ordered with the context's kernels. */
int pyxis_cuda_comm_init(pyxis_cuda_ctx *ctx, const uint8_t id[PYXIS_COMM_ID_BYTES], int nranks, int rank,
                         pyxis_cuda_comm **comm);
int pyxis_cuda_comm_info(const pyxis_cuda_comm *comm, int *nranks, int *rank);
/* Frees the communicator.  No collective of it may be pending or held by a CUDA graph. */
int pyxis_cuda_comm_free(pyxis_cuda_comm *comm);

/* Vocab-parallel greedy head, device pointers, asynchronous on `stream` (NULL: the context's).
 * Every rank passes the same M rows of hidden states X [M, hidden] (row stride ldx) and its own
 * shard: rows [vocab_lo, vocab_lo + shard_rows) of the [vocab, hidden] lm_head, quantised like
 * the full head (pyxis_cuda_quantize on those rows).  Writes tokens[M] (int32, device) on every
 * rank: the first index of the row maximum over all vocab rows (src/output_head.rs:30-44).
 * Ranks must call it in the same order with the same M.  M <= 1024; vocab < 2^31.  The logits
 * and keys live in buffers the communicator grows on first use (not during stream capture:
 * call pyxis_cuda_head_reserve first). */
int pyxis_cuda_head_greedy_dev(pyxis_cuda_comm *comm, const pyxis_cuda_weights *shard, size_t vocab,
                               size_t vocab_lo, size_t shard_rows, size_t hidden, const float *X, size_t M,
                               size_t ldx, int32_t *tokens, void *stream);

/* Grows the communicator's head buffers for M rows of shard_rows logits. */
int pyxis_cuda_head_reserve(pyxis_cuda_comm *comm, size_t M, size_t shard_rows);

/* Makes pyxis_cuda_model_generate_batch of this model vocab-parallel over `comm`: each rank runs
 * its own sequences (data-parallel; every rank must pass the same n_seq, n_prompt and n_new), the
 * final hidden rows of all ranks are all-gathered before the head, each rank multiplies them with
 * its lm_head shard (rows [vocab_lo, vocab_lo + shard_rows) of the head, kept by reference) and
 * the ranks agree on every row's token as pyxis_cuda_head_greedy_dev does.  The model then needs
 * no full lm_head (pyxis_cuda_model_set_head may pass NULL for it); pyxis_cuda_model_generate
 * (one sequence) still uses the full head.  comm NULL switches vocab-parallel off. */
int pyxis_cuda_model_set_vocab_parallel(pyxis_cuda_model *m, pyxis_cuda_comm *comm,
                                        const pyxis_cuda_weights *lm_head_shard, size_t vocab_lo,
                                        size_t shard_rows);

#ifdef __cplusplus
}
#endif
#endif
