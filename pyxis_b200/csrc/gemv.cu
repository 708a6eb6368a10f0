// gemv.cu -- decode GEMV over int8 / int4 / f32 / bf16 weights in the reference layout, fp32
// accumulation.
//
// Computes what src/matmul.rs:67-96 computes row by row -- y[n] = sum_i x[i] * q[n,i] *
// scale(n,i) -- for B = 1..8 input rows at once, streaming the packed weights from HBM once.
//
// Kernels (chosen by launch_gemv from the shape, first match):
//   batch  B = 1..8 with K % 32 == 0, whole-chunk scale blocks and x fitting shared memory:
//          gemv_batch.cu (x staged by TMA, every weight load in flight at once, split-K over
//          warps).  The decode shapes and the benchmark sweep all run here.
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
const char *gemv_kernel_name(const QMatrix &w, size_t B, int num_sms) {
    if (gemv_batch_supported(w, B, num_sms)) return "gemv_batch_kernel";
    return "gemv_generic_kernel";
}

cudaError_t launch_gemv(const QMatrix &w, const float *X, size_t B, size_t ldx, float *Y,
                        size_t ldy, int *err, int num_sms, cudaStream_t st) {
    if (w.N == 0 || B == 0) return cudaSuccess;
    const bool x_aligned = (reinterpret_cast<uintptr_t>(X) & 15) == 0;
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
