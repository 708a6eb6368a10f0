// gemv.cu -- decode GEMV over int8 / int4 / f32 / bf16 weights in the reference layout, fp32
// accumulation.
//
// Computes what src/matmul.rs:67-96 computes row by row -- y[n] = sum_i x[i] * q[n,i] *
// scale(n,i) -- for B = 1..8 input rows at once, streaming the packed weights from HBM once.
//
// Kernels (chosen by launch_gemv from the shape, first match):
//   mma    int4 / int8 with a scale per group of 32 or per row, K % 256 (int4) or % 128 (int8),
//          matrices of 4 MB or more at 4-8 input rows, int8 ones of 8 MB or more at any batch
//          (prefer_mma): gemv_mma.cu (weights by TMA, codes from registers into mma.sync with x
//          as fp16 hi / lo, K parts reduced in a cluster).
//   batch  B = 1..8 with K % 32 == 0, whole-chunk scale blocks and x fitting shared memory:
//          gemv_batch.cu (x staged by TMA, every weight load in flight at once, split-K over
//          warps): the smaller and the batch-1 int4 products, f32 / bf16 rows, other block
//          sizes and K, and the decode step's GEMVs whose x is computed in the kernel.
//   generic  any shape the others do not take (K not a multiple of the chunk, blocks that
//          straddle rows, odd K with int4 rows that start mid-byte): one warp per row,
//          element-wise decode with the reference's scales[g / block_size] lookup.
#include "common.cuh"
#include "kernels.h"

namespace pyxis {

// ---------------------------------------------------------------- generic kernel --------------
template <int QT>
__global__ void gemv_generic_kernel(const uint8_t *W, const float *S, size_t bs, const float *X,
                                    size_t ldx, float *Y, size_t ldy, size_t N, size_t K, int B) {
    const size_t row = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= N) return;
    for (int b = 0; b < B; ++b) {
        const float *x = X + (size_t)b * ldx;
        float acc = 0.f;
        for (size_t i = lane; i < K; i += 32) {
            const size_t g = row * K + i;  // flattened index: blocks run over it (src/matmul.rs:70)
            float q;
            if (QT == kQF32) {
                acc += x[i] * reinterpret_cast<const float *>(W)[g];  // dot_product_scalar, :284-287
                continue;
            } else if (QT == kQBF16) {
                const uint32_t bits = reinterpret_cast<const uint16_t *>(W)[g];
                acc += x[i] * __uint_as_float(bits << 16);  // dot_product_bf16_scalar, :289-295
                continue;
            } else if (QT == kQInt8) {
                q = (float)(int8_t)W[g];
            } else {
                const uint8_t byte = W[g / 2];
                q = (float)((g & 1) ? (byte >> 4) : (byte & 0x0f)) - 8.0f;
            }
            acc += (x[i] * q) * S[g / bs];
        }
        acc = warp_sum(acc);
        if (lane == 0) Y[(size_t)b * ldy + row] = acc;
    }
}

// ---------------------------------------------------------------- dispatch --------------------
// Where the mma.sync GEMV finishes first (measured on B200, graph replay of back-to-back launches,
// weights streamed from HBM).  Its CTAs stage the weights in shared memory before waiting on the
// previous kernel and then run about 7 instructions per code at 8 input rows against the batch
// kernel's 6.75, 4.4 against 4.3 at 4 rows and 4.4 against 2.5 at one row (an m16n8k16 costs
// about 8 issue slots on sm_100); its fixed cost (x split, cluster reduction) is ~1.3 us more.
// int4 2048 x 2048: 3.9 / 4.1 / 5.1 us at 1 / 4 / 8 rows vs 2.4 / 3.2 / 4.9 us; int4 6144 x 2048:
// 5.8 / 6.5 / 8.3 vs 4.4 / 6.6 / 10.8 us; int4 2048 x 6144: 6.7 / 7.1 / 9.4 vs 4.3 / 6.8 / 13.2 us;
// int8 6144 x 2048 per row: 5.7 / 5.8 / 7.5 vs 6.3 / 8.4 / 13.0 us.
bool prefer_mma(const QMatrix &w, size_t B, int num_sms) {
    const size_t bytes = w.qtype == kQInt4 ? w.N * w.K / 2 : w.N * w.K;
    const bool big = bytes >= (size_t(8) << 20), mid = bytes >= (size_t(4) << 20);
    if (!(big ? (w.qtype == kQInt8 || B >= 4) : (mid && B >= 4))) return false;
    return gemv_mma_supported(w, B, num_sms);
}

const char *gemv_kernel_name(const QMatrix &w, size_t B, int num_sms) {
    if (prefer_mma(w, B, num_sms)) return "gemv_mma_kernel";
    if (gemv_batch_supported(w, B, num_sms)) return "gemv_batch_kernel";
    return "gemv_generic_kernel";
}

cudaError_t launch_gemv(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y,
                        size_t ldy, int *err, int num_sms, cudaStream_t st) {
    if (w.N == 0 || B == 0) return cudaSuccess;
    const bool x_aligned = (reinterpret_cast<uintptr_t>(X) & 15) == 0;
    if (x_aligned && (B == 1 || ldx % 4 == 0) && prefer_mma(w, B, num_sms))
        return launch_gemv_mma(w, X, B, ldx, Y, ldy, err, num_sms, st);
    if (x_aligned && (B == 1 || ldx % 4 == 0) && gemv_batch_supported(w, B, num_sms))
        return launch_gemv_batch(w, X, B, ldx, Y, ldy, err, num_sms, st);
    const size_t threads = w.N * 32;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    switch (w.qtype) {
    case kQInt8:
        gemv_generic_kernel<kQInt8><<<grid, 256, 0, st>>>(w.data, w.scales, w.block_size, X, ldx, Y, ldy, w.N, w.K, (int)B);
        break;
    case kQInt4:
        gemv_generic_kernel<kQInt4><<<grid, 256, 0, st>>>(w.data, w.scales, w.block_size, X, ldx, Y, ldy, w.N, w.K, (int)B);
        break;
    case kQF32:
        gemv_generic_kernel<kQF32><<<grid, 256, 0, st>>>(w.data, w.scales, 1, X, ldx, Y, ldy, w.N, w.K, (int)B);
        break;
    case kQBF16:
        gemv_generic_kernel<kQBF16><<<grid, 256, 0, st>>>(w.data, w.scales, 1, X, ldx, Y, ldy, w.N, w.K, (int)B);
        break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace pyxis
