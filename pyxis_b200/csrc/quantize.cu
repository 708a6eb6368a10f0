// quantize.cu -- on-device quantise + pack, bit-exact with the reference quantizers.
//
// Weights::quantize_int8 (src/weights.rs:94-118) and Weights::quantize_int4 (:120-151), applied
// after dequantize_weights' bf16 -> f32 widening (src/model.rs:535-538).  Two phases:
//   1. one scale per block:  absmax = max(|v|) (fmaxf, NaN operands dropped, as f32::max);
//      scale = absmax == 0 ? 1 : absmax / D   (D = 127 or 7, IEEE division)
//   2. one code per element: q = clamp(roundf(v / scale), lo, hi), NaN -> 0   (Rust `as i8`)
//      int4 packs q + 8 into nibbles, element i in byte i/2 (low nibble when i is even); a
//      missing odd element of the last byte stays 0x8 (the 0x88 pre-fill, :125).
// max is order-independent and the per-element arithmetic is the same IEEE operations, so the
// bytes and scale bits equal the reference's whatever the thread mapping.
#include "common.cuh"
#include "kernels.h"

namespace pyxis {

template <int SRC>
PYXIS_DEVINL float load_src(const void *src, size_t i) {
    if (SRC == kSrcF32) return __ldg(reinterpret_cast<const float *>(src) + i);
    return bf16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short *>(src) + i));
}

PYXIS_DEVINL float scale_from_absmax(float absmax, float divisor) {
    return absmax == 0.0f ? 1.0f : __fdiv_rn(absmax, divisor);
}

// Phase 1, block_size <= 64: one thread per block.
template <int SRC>
__global__ void absmax_thread_kernel(const void *src, size_t n, size_t bs, size_t nblocks,
                                     float divisor, float *scales) {
    size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    size_t s = b * bs, e = s + bs < n ? s + bs : n;
    float m = 0.0f;
    for (size_t i = s; i < e; ++i) m = fmaxf(m, fabsf(load_src<SRC>(src, i)));
    scales[b] = scale_from_absmax(m, divisor);
}

// Phase 1, 64 < block_size <= 65536: one warp per block.
template <int SRC>
__global__ void absmax_warp_kernel(const void *src, size_t n, size_t bs, size_t nblocks,
                                   float divisor, float *scales) {
    size_t b = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (b >= nblocks) return;
    size_t s = b * bs, e = s + bs < n ? s + bs : n;
    float m = 0.0f;
    for (size_t i = s + lane; i < e; i += 32) m = fmaxf(m, fabsf(load_src<SRC>(src, i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) scales[b] = scale_from_absmax(m, divisor);
}

// Phase 1, larger blocks: one CTA per block.
template <int SRC>
__global__ void absmax_cta_kernel(const void *src, size_t n, size_t bs, float divisor,
                                  float *scales) {
    __shared__ float red[32];
    size_t b = blockIdx.x;
    size_t s = b * bs, e = s + bs < n ? s + bs : n;
    float m = 0.0f;
    for (size_t i = s + threadIdx.x; i < e; i += blockDim.x) m = fmaxf(m, fabsf(load_src<SRC>(src, i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) scales[b] = scale_from_absmax(m, divisor);
    }
}

PYXIS_DEVINL int quant_code(float v, float scale, float lo, float hi) {
    float t = roundf(__fdiv_rn(v, scale));  // f32::round: half away from zero
    if (isnan(t)) return 0;                 // `as i8` maps NaN to 0
    t = t < lo ? lo : (t > hi ? hi : t);    // f32::clamp
    return (int)t;
}

// Phase 2, int8: one element per thread-iteration.
template <int SRC>
__global__ void pack_int8_kernel(const void *src, size_t n, size_t bs, const float *scales,
                                 int8_t *out) {
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float sc = scales[i / bs];
        out[i] = (int8_t)quant_code(load_src<SRC>(src, i), sc, -127.0f, 127.0f);
    }
}

// Phase 2, int4: one output byte (elements 2j and 2j+1) per thread-iteration.
template <int SRC>
__global__ void pack_int4_kernel(const void *src, size_t n, size_t bs, const float *scales,
                                 uint8_t *out) {
    size_t nbytes = (n + 1) / 2;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x; j < nbytes; j += stride) {
        size_t g0 = 2 * j, g1 = g0 + 1;
        uint32_t lo = (uint32_t)(quant_code(load_src<SRC>(src, g0), scales[g0 / bs], -8.0f, 7.0f) + 8);
        uint32_t hi = 8;  // 0x88 pre-fill for a missing odd element
        if (g1 < n)
            hi = (uint32_t)(quant_code(load_src<SRC>(src, g1), scales[g1 / bs], -8.0f, 7.0f) + 8);
        out[j] = (uint8_t)((hi << 4) | lo);
    }
}

template <int SRC>
static cudaError_t launch_quantize_t(const void *src, size_t n, size_t bs, int qtype, void *data,
                                     float *scales, int num_sms, cudaStream_t st) {
    size_t nblocks = (n + bs - 1) / bs;
    float divisor = qtype == kQInt8 ? 127.0f : 7.0f;
    if (bs <= 64) {
        unsigned grid = (unsigned)((nblocks + 255) / 256);
        absmax_thread_kernel<SRC><<<grid, 256, 0, st>>>(src, n, bs, nblocks, divisor, scales);
    } else if (bs <= 65536) {
        size_t threads = nblocks * 32;
        unsigned grid = (unsigned)((threads + 255) / 256);
        absmax_warp_kernel<SRC><<<grid, 256, 0, st>>>(src, n, bs, nblocks, divisor, scales);
    } else {
        absmax_cta_kernel<SRC><<<(unsigned)nblocks, 1024, 0, st>>>(src, n, bs, divisor, scales);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    size_t work = qtype == kQInt8 ? n : (n + 1) / 2;
    size_t g = (work + 255) / 256;
    size_t gmax = (size_t)num_sms * 16;
    unsigned grid = (unsigned)(g < gmax ? g : gmax);
    if (grid == 0) grid = 1;
    if (qtype == kQInt8)
        pack_int8_kernel<SRC><<<grid, 256, 0, st>>>(src, n, bs, scales, (int8_t *)data);
    else
        pack_int4_kernel<SRC><<<grid, 256, 0, st>>>(src, n, bs, scales, (uint8_t *)data);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- GGUF Q8_0 ---------------------
// f16 bits -> f32 as half 2.7.1's f16::to_f32 widens (the same as x86 F16C): exact for every
// finite value and for infinities; a NaN keeps its sign and payload and gets the quiet bit.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    if (exp == 0x1fu) return __uint_as_float(sign | 0x7f800000u | (man ? 0x400000u | (man << 13) : 0u));
    if (exp != 0) return __uint_as_float(sign | ((exp + 112u) << 23) | (man << 13));
    // zero or subnormal: man * 2^-24, exact in f32 (man < 2^10, a normal f32 result)
    return __uint_as_float(sign | __float_as_uint(__fmul_rn((float)man, __uint_as_float(0x33800000u))));
}

// One thread per 34-byte block (src/gguf.rs:246-271): scale, then the 32 codes, the codes past
// n (the last block's tail) dropped.  Byte loads: a block starts at any 2-byte boundary, and a
// warp's 32 blocks are 1088 contiguous bytes, so the loads still coalesce.
__global__ void q8_0_unpack_kernel(const uint8_t *__restrict__ blocks, size_t n, size_t nb, int8_t *__restrict__ data,
                                   float *__restrict__ scales) {
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += (size_t)gridDim.x * blockDim.x) {
        const uint8_t *blk = blocks + b * 34;
        scales[b] = f16_bits_to_f32((uint32_t)__ldg(blk) | ((uint32_t)__ldg(blk + 1) << 8));
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            w[i] = (uint32_t)__ldg(blk + 2 + 4 * i) | ((uint32_t)__ldg(blk + 3 + 4 * i) << 8) |
                   ((uint32_t)__ldg(blk + 4 + 4 * i) << 16) | ((uint32_t)__ldg(blk + 5 + 4 * i) << 24);
        const size_t g0 = b * 32;
        if (g0 + 32 <= n) {  // data is 256-byte aligned and g0 a multiple of 32
            uint4 *d = reinterpret_cast<uint4 *>(data + g0);
            d[0] = make_uint4(w[0], w[1], w[2], w[3]);
            d[1] = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
            for (size_t i = 0; g0 + i < n; ++i) data[g0 + i] = (int8_t)((w[i / 4] >> (8 * (i % 4))) & 0xffu);
        }
    }
}

cudaError_t launch_q8_0_unpack(const uint8_t *blocks, size_t n, int8_t *data, float *scales, int num_sms,
                               cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const size_t nb = (n + 31) / 32;
    const size_t g = (nb + 255) / 256, gmax = (size_t)num_sms * 16;
    q8_0_unpack_kernel<<<(unsigned)(g < gmax ? g : gmax), 256, 0, st>>>(blocks, n, nb, data, scales);
    return cudaGetLastError();
}

cudaError_t launch_quantize(const void *src, int src_kind, size_t n, size_t bs, int qtype,
                            void *data, float *scales, int num_sms, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    if (src_kind == kSrcF32) return launch_quantize_t<kSrcF32>(src, n, bs, qtype, data, scales, num_sms, st);
    return launch_quantize_t<kSrcBF16>(src, n, bs, qtype, data, scales, num_sms, st);
}

}  // namespace pyxis
