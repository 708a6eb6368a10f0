// split_x.cuh -- the x operand of the tensor-core matmuls (gemm_tc.cu, gemm_ws.cu): every token
// row scaled by its power of two and split into fp16 hi + lo (22 significant bits).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace pyxis {
namespace {

// One CTA per token row: e = 15 - exponent(max|x|) so |x 2^e| < 2^15; hi = fp16(x 2^e),
// lo = fp16(x 2^e - hi); inv = 2^-e.  PERM writes each 8-element group in the int4 converter's
// order (e0, e4, e1, e5, e2, e6, e3, e7).  A thread takes whole 8-element groups: two 16-byte
// loads when the row is 16-byte aligned (VEC), one 16-byte store each of hi and lo.
template <bool PERM>
__global__ void __launch_bounds__(512) split_x_rows_kernel(const float *__restrict__ X, long long ldx, int K,
                                                         __half *__restrict__ hi, __half *__restrict__ lo,
                                                         float *__restrict__ inv, int vec) {
    __shared__ float red[16];
    // the matmul that reads this kernel's output may launch at once: it streams and converts its
    // weights before its own griddepcontrol.wait, which still waits for this kernel to finish
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x, n8 = K / 8;
    const float *x = X + (size_t)m * ldx;
    auto load8 = [&](int g, float (&v)[8]) {
        if (vec) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(x + 8 * g));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(x + 8 * g + 4));
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldg(x + 8 * g + j);
        }
    };
    float mx = 0.f;
    for (int g = threadIdx.x; g < n8; g += blockDim.x) {
        float v[8];
        load8(g, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    int e = 0;
    if (mx > 0.f && isfinite(mx)) {
        int ex;
        frexpf(mx, &ex);  // mx = f 2^ex, f in [0.5, 1)
        e = 15 - ex;
        e = e > 120 ? 120 : (e < -120 ? -120 : e);
    }
    const float sc = __int_as_float((127 + e) << 23);  // 2^e, exact
    if (threadIdx.x == 0) inv[m] = __int_as_float((127 - e) << 23);
    __half *hrow = hi + (size_t)m * K, *lrow = lo + (size_t)m * K;
    for (int g = threadIdx.x; g < n8; g += blockDim.x) {
        float v[8];
        load8(g, v);
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            // output pair j: (v[2j], v[2j+1]) in order, (v[j], v[j+4]) permuted
            const float a = (PERM ? v[j] : v[2 * j]) * sc, b = (PERM ? v[j + 4] : v[2 * j + 1]) * sc;
            const __half2 h = __floats2half2_rn(a, b);
            const float2 f = __half22float2(h);
            const __half2 l = __floats2half2_rn(a - f.x, b - f.y);
            hw[j] = *reinterpret_cast<const uint32_t *>(&h);
            lw[j] = *reinterpret_cast<const uint32_t *>(&l);
        }
        *reinterpret_cast<uint4 *>(hrow + 8 * g) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(lrow + 8 * g) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
}

}  // namespace
}  // namespace pyxis
