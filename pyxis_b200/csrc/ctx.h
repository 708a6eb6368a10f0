// ctx.h -- the context and weights handles behind the C ABI, shared by api.cu and decode.cu.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>

#include "argmax.h"

struct pyxis_cuda_ctx {
    int device;
    int num_sms;
    cudaStream_t stream;
    // staging for the host-pointer entry points (grown on demand), guarded by host_mu: host
    // threads that call pyxis_cuda_matmul(_batch) on one context at once run one after another
    std::mutex host_mu;
    float *dx = nullptr;
    size_t dx_cap = 0;
    float *dy = nullptr;
    size_t dy_cap = 0;
    // workspace kept for pyxis_cuda_matmul_dev calls that pass none
    void *ws = nullptr;
    size_t ws_cap = 0;
    // argmax scratch (allocated and zeroed at init)
    pyxis::ArgmaxScratch amax{};
    void *amax_mem = nullptr;
    // device error flag written by kernels whose bounded waits ran out (0 = none)
    int *d_err = nullptr;
    // split-K scratch of the tensor-core GEMV (zeroed at init; the kernel leaves it zeroed)
    void *tcg_scratch = nullptr;
    size_t tcg_scratch_bytes = 0;
    // per-tile tickets of the weight-streaming matmul (zeroed at init; the kernel leaves them zero)
    unsigned *ws_tickets = nullptr;
    size_t ws_tickets_n = 0;
};

struct pyxis_cuda_weights {
    int device;
    int qtype;
    size_t num_elements, block_size;
    size_t data_bytes, num_scales;
    uint8_t *data;   // one allocation: data, padded to 256 B, then scales
    float *scales;
};

namespace pyxis {
// Y[M, N] = X[M, K] W^T for device pointers on `st`: the kernel choice of pyxis_cuda_matmul_dev
// (tensor-core GEMM for M >= 16, otherwise GEMVs 8 rows at a time).  Returns a pyxis_status and
// records the message like every entry point.
int run_matmul(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, const float *X, size_t M, size_t ldx,
               size_t N, size_t K, float *Y, size_t ldy, void *workspace, size_t workspace_bytes, cudaStream_t st);
// The greedy head's vocab shard on the tensor-core GEMV with each row's argmax key folded into its
// epilogue: keys[m] (0 on entry) becomes the key of row m's first maximum, global index
// index_base + n, as launch_argmax_keys would write it.  Returns false and launches nothing when
// the product does not take that kernel (more than 8 rows, a matrix the CUDA-core GEMVs take);
// otherwise *err is the launch's status.
bool head_gemv_keys(pyxis_cuda_ctx *ctx, const pyxis_cuda_weights *w, const float *X, size_t M, size_t ldx, size_t N,
                    size_t K, float *Y, size_t ldy, int64_t index_base, uint64_t *keys, cudaStream_t st,
                    cudaError_t *err);
}  // namespace pyxis
