// fp16_codes.cuh -- quantized codes and f32 values as fp16 tensor-core operands, shared by the
// tensor-core matmuls (gemm_tc.cu, gemm_ws.cu, gemv_mma.cu).
//
// Codes become exact fp16 integers with one mask / byte permute and one paired subtraction per two
// codes; an f32 value becomes an fp16 hi + lo pair carrying 22 significant bits.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace pyxis {

PYXIS_DEVINL uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }
PYXIS_DEVINL __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Four int8 codes (signed bytes) -> exact fp16 pairs (e0,e1) (e2,e3): byte b -> fp16(1024 + (b ^ 0x80))
// - 1152.
PYXIS_DEVINL void i8x4_to_h(uint32_t w, uint32_t &h01, uint32_t &h23) {
    const uint32_t u = w ^ 0x80808080u;
    const __half2 bias = bits_h2(0x64806480u);  // (1152, 1152)
    h01 = h2_bits(__hsub2(bits_h2(__byte_perm(u, 0x64646464u, 0x5140u)), bias));
    h23 = h2_bits(__hsub2(bits_h2(__byte_perm(u, 0x64646464u, 0x5342u)), bias));
}

// Eight int4 codes (q + 8 in nibbles; element 2j = low, 2j+1 = high nibble of byte j) -> exact fp16
// pairs in the order (e0,e4) (e1,e5) (e2,e6) (e3,e7): nibbles i and i+4 of the word land in the two
// halves of (w >> 4i) & 0x000F000F; OR-ing in 1024's exponent makes them 1024 + (q + 8), then - 1032.
// Every consumer lays x out in the same element order.
PYXIS_DEVINL void u4x8_to_h(uint32_t w, uint32_t (&h)[4]) {
    const __half2 bias = bits_h2(0x64086408u);  // (1032, 1032)
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = h2_bits(__hsub2(bits_h2(((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u), bias));
}

// A pair of f32 values v (|v| < 2^15) as fp16 hi + lo pairs: hi is v rounded to 11 significant bits
// by Veltkamp's split (c = v (2^13 + 1), hi = c - (c - v)), so it converts to fp16 exactly (above
// fp16's subnormal range), and lo = v - hi is exact in f32 and rounded once to fp16: 22 bits.
PYXIS_DEVINL void split_pair_f32(float2 v, uint32_t &hi, uint32_t &lo) {
    const float2 m1 = make_float2(-1.f, -1.f);
    const float2 c = __fmul2_rn(v, make_float2(8193.0f, 8193.0f));
    const float2 h = __ffma2_rn(__ffma2_rn(v, m1, c), m1, c);  // c - (c - v)
    const float2 l = __ffma2_rn(h, m1, v);                      // v - h
    hi = h2_bits(__floats2half2_rn(h.x, h.y));
    lo = h2_bits(__floats2half2_rn(l.x, l.y));
}

}  // namespace pyxis
