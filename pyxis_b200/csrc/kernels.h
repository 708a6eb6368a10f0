// kernels.h -- internal launcher interface between the C ABI (api.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace pyxis {

enum { kSrcF32 = 1, kSrcBF16 = 2 };  // == PYXIS_DTYPE_*
enum { kQInt8 = 1, kQInt4 = 2, kQF32 = 3, kQBF16 = 4 };  // == PYXIS_QTYPE_*

// A weight matrix [N, K] in the reference layout (see pyxis_cuda.h); unquantized (kQF32, kQBF16)
// matrices have no scales.
struct QMatrix {
    int qtype;
    const uint8_t *data;
    const float *scales;
    size_t block_size;
    size_t N, K;
};

cudaError_t launch_quantize(const void *src, int src_kind, size_t n, size_t bs, int qtype,
                            void *data, float *scales, int num_sms, cudaStream_t st);

// GGUF Q8_0 blocks (34 bytes: f16 scale, 32 int8) -> int8 codes [n] and f32 scales [ceil(n/32)].
cudaError_t launch_q8_0_unpack(const uint8_t *blocks, size_t n, int8_t *data, float *scales, int num_sms,
                               cudaStream_t st);

// Decode GEMV: Y[b, :] = W X[b, :] for b < B (B = 1..8): the batch kernel where it applies, else
// the generic kernel (gemv.cu).  Every weight layout.
cudaError_t launch_gemv(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y,
                        size_t ldy, int *err, int num_sms, cudaStream_t st);

// 1-8 input rows on the CUDA cores with x staged by TMA and split-K over warps (gemv_batch.cu):
// K % 32 == 0, one scale per row or per block of whole 16-byte chunks, B * K * 4 bytes of x in
// shared memory.
bool gemv_batch_supported(const QMatrix &w, size_t B, int num_sms);
cudaError_t launch_gemv_batch(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y, size_t ldy,
                              int *err, int num_sms, cudaStream_t st);

// 1-8 input rows with the codes fed from registers to mma.sync m16n8k16 (gemv_mma.cu): int4 / int8
// with a scale per group of 32 or per row, K % 256 (int4) or K % 128 (int8) == 0, X 16-byte
// aligned, ldx % 4 == 0.
bool gemv_mma_supported(const QMatrix &w, size_t B, int num_sms);
cudaError_t launch_gemv_mma(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y, size_t ldy, int *err,
                            int num_sms, cudaStream_t st);

// Batch-1 products whose x is computed inside the GEMV from the previous step's outputs:
// kProAddNorm: x' = x + delta (delta may be NULL; CTA 0 stores x' to xout, which must not alias
// x), then RMSNorm with weight w; kProSiluMul: SiLU(x[0:K]) * x[K:2K].  All pointers 16-byte
// aligned.
enum { kProNone = 0, kProAddNorm = 1, kProSiluMul = 2 };
struct GemvPrologue {
    int kind = kProNone;
    const float *x = nullptr, *delta = nullptr, *w = nullptr;
    float *xout = nullptr;
    float eps = 0.f;
};
bool gemv_batch_pro_supported(const QMatrix &w, const GemvPrologue &pro, int num_sms);
cudaError_t launch_gemv_batch_pro(const QMatrix &w, const GemvPrologue &pro, float *Y, int *err, int num_sms,
                                  cudaStream_t st);

// Name of the kernel launch_gemv would pick (for tests and the bench's launch accounting).
const char *gemv_kernel_name(const QMatrix &w, size_t B, int num_sms);

// Tensor-core prefill GEMM (gemm_tc.cu).  Supported when K % 64 == 0 and the scales are one per
// row (block == K) or per group of a multiple of 32 that divides K.
bool gemm_tc_supported(const QMatrix &w);
// Workspace: gemm_tc_workspace_bytes(M, K) is enough; with gemm_tc_workspace_bytes_splitk(...)
// bytes a GEMM with fewer output tiles than SMs also splits K over more CTAs (partials added in a
// fixed order by a second kernel).
size_t gemm_tc_workspace_bytes(size_t M, size_t K);
size_t gemm_tc_workspace_bytes_splitk(size_t M, size_t N, size_t K, int block_size_is_k, size_t block_size,
                                      int num_sms);
cudaError_t launch_gemm_tc(const QMatrix &w, const float *X, size_t M, size_t ldx, float *Y, size_t ldy, void *ws,
                           size_t ws_bytes, int *err, int num_sms, cudaStream_t st);

// int8 per-row GEMV for 1-8 input rows on tcgen05 kind::i8 (gemv_tc.cu).  `scratch` holds the
// partial sums of tiles shared by two or more CTAs (one slot per CTA of a grid of up to
// max_grid); it must be zero before the first launch and the kernel leaves it zero.
bool gemv_tc_supported(const QMatrix &w, size_t B, int num_sms);
size_t gemv_tc_scratch_bytes(int max_grid);
// With `keys` (the greedy head's vocab shard): the epilogue also max-reduces, per input row b,
// the argmax key of every logit at global index key_base + n into keys[b] (atomicMax; keys[0, B)
// must be 0 before the launch), the key launch_argmax_keys would write for the row.
cudaError_t launch_gemv_tc(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y, size_t ldy,
                           void *scratch, size_t scratch_bytes, int *err, int num_sms, cudaStream_t st,
                           uint64_t *keys = nullptr, long long key_base = 0);

// Weight-streaming matmul for 1..64 tokens on tcgen05 (gemm_ws.cu): int4 or int8 codes with a scale
// per group of 32, or int8 with one scale per row; K % 128 == 0.  The workspace holds x's fp16
// hi / lo copies (gemm_ws_workspace_bytes(M, N, K, sms, 0) bytes, 256-byte aligned) and, in what
// is left, the partial sums of tiles split along K; `tickets` (one per 128-row tile) must be zero
// before the first launch and are left zero.
bool gemm_ws_supported(const QMatrix &w, size_t M);
size_t gemm_ws_workspace_bytes(size_t M, size_t N, size_t K, int num_sms, size_t partial_cap);
cudaError_t launch_gemm_ws(const QMatrix &w, const float *X, size_t M, size_t ldx, float *Y, size_t ldy, void *ws,
                           size_t ws_bytes, unsigned *tickets, size_t num_tickets, int *err, int num_sms,
                           cudaStream_t st);

// Records `msg` as the calling thread's pyxis_cuda_last_error() and returns `code` (api.cu).
int record_error(int code, const char *msg);

}  // namespace pyxis
