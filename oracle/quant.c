/*
 * quant.c -- restatement of the reference quantizers and layout conversions (oracle, test-only).
 *
 * Rust semantics reproduced here:
 *   f32::abs / f32::max fold from 0.0      -> fabsf / fmaxf (fmaxf also drops a NaN operand)
 *   f32::round (half away from zero)       -> roundf
 *   f32::clamp(lo, hi) (NaN passes through) -> explicit compares
 *   `as i8` (saturating, NaN -> 0)          -> explicit NaN test; the clamp keeps the range
 */
#include <math.h>
#include <string.h>

#include "pyxis_oracle.h"

static float clamp_f32(float v, float lo, float hi) {
    /* f32::clamp: `if self < min { min } else if self > max { max } else { self }` */
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}

static int8_t f32_as_i8(float v) {
    /* Rust `as i8`: NaN -> 0, otherwise saturating truncation.  Callers clamp first, so the
     * value is an integer within range; the saturation arms only document the semantics. */
    if (isnan(v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return (int8_t)v;
}

/* src/weights.rs:94-118 */
void oracle_quantize_int8(const float *values, size_t n, size_t block_size, int8_t *data,
                          float *scales) {
    size_t nb = 0;
    for (size_t start = 0; start < n; start += block_size, ++nb) {
        size_t end = start + block_size < n ? start + block_size : n;
        float absmax = 0.0f; /* .map(|v| v.abs()).fold(0.0, f32::max) (:103) */
        for (size_t i = start; i < end; ++i) absmax = fmaxf(absmax, fabsf(values[i]));
        float scale = absmax == 0.0f ? 1.0f : absmax / 127.0f; /* :104 */
        scales[nb] = scale;
        for (size_t i = start; i < end; ++i) /* (value / scale).round().clamp(-127,127) as i8 */
            data[i] = f32_as_i8(clamp_f32(roundf(values[i] / scale), -127.0f, 127.0f));
    }
}

/* src/weights.rs:120-151 */
void oracle_quantize_int4(const float *values, size_t n, size_t block_size, uint8_t *data,
                          float *scales) {
    memset(data, 0x88, (n + 1) / 2); /* vec![0x88; num_elements.div_ceil(2)] (:125) */
    size_t nb = 0;
    for (size_t start = 0; start < n; start += block_size, ++nb) {
        size_t end = start + block_size < n ? start + block_size : n;
        float absmax = 0.0f;
        for (size_t i = start; i < end; ++i) absmax = fmaxf(absmax, fabsf(values[i]));
        float scale = absmax == 0.0f ? 1.0f : absmax / 7.0f; /* :130 */
        scales[nb] = scale;
        for (size_t g = start; g < end; ++g) {
            /* ((value / scale).round().clamp(-8.0, 7.0) as i8 + 8) as u8 (:135) */
            uint8_t q = (uint8_t)(f32_as_i8(clamp_f32(roundf(values[g] / scale), -8.0f, 7.0f)) + 8);
            uint8_t *byte = &data[g / 2];
            if (g % 2 == 0)
                *byte = (uint8_t)((*byte & 0xf0) | q); /* :138 */
            else
                *byte = (uint8_t)((*byte & 0x0f) | (q << 4)); /* :140 */
        }
    }
}

/* src/model.rs:535-538 */
void oracle_bf16_to_f32(const uint16_t *src, size_t n, float *dst) {
    for (size_t i = 0; i < n; ++i) {
        uint32_t bits = (uint32_t)src[i] << 16;
        memcpy(&dst[i], &bits, 4);
    }
}

/* src/model.rs:539-548 */
void oracle_dequantize_int8(const int8_t *data, const float *scales, size_t block_size, size_t n,
                            float *dst) {
    for (size_t i = 0; i < n; ++i) dst[i] = (float)data[i] * scales[i / block_size];
}

/* src/model.rs:549-564 */
void oracle_dequantize_int4(const uint8_t *data, const float *scales, size_t block_size, size_t n,
                            float *dst) {
    for (size_t i = 0; i < n; ++i) {
        uint8_t byte = data[i / 2];
        uint8_t nib = (i % 2 == 0) ? (byte & 0x0f) : ((byte >> 4) & 0x0f);
        dst[i] = ((float)nib - 8.0f) * scales[i / block_size];
    }
}

/* half::f16::to_f32 (half 2.7.1; x86 F16C widens the same way): exact for finite values and
 * infinities; a NaN keeps its sign and payload and gets the quiet bit (0x00400000). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; ++e; } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man ? 0x00400000u | (man << 13) : 0u);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* src/gguf.rs:245-271 (read_q8_0_weights): 34-byte blocks, truncate data to n. */
void oracle_q8_0_to_int8(const uint8_t *blocks, size_t n, int8_t *data, float *scales) {
    size_t nb = (n + 31) / 32;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t *blk = blocks + b * 34;
        scales[b] = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (size_t i = 0; i < 32; ++i) {
            size_t g = b * 32 + i;
            if (g < n) data[g] = (int8_t)blk[2 + i];
        }
    }
}
