// attn_tc.h -- the causal prefill attention on the tensor cores (attn_tc.cu): operand layout,
// the scaling rule shared with the kernel that writes the operands, and the launches.
//
// src/attention.rs:107-135 computes, for every query position i of head h, the scores
// (q_i . k_j) / sqrt(hd) over keys j <= i of kv head h / G, their softmax and sum_j p_j v_j, all in
// f32.  The tensor-core form keeps that precision with two fp16 terms per operand: every f32 value
// x of a group (a query row of one head; all keys, or all values, of one kv head of a sequence) is
// scaled by the group's power of two 2^e (max |x| 2^e in [2^14, 2^15)) and split as
// hi = fp16(x 2^e), lo = fp16(x 2^e - hi) -- 22 significant bits -- and each product is taken as
// hi.hi + hi.lo + lo.hi (the lo.lo term is below f32 rounding of the sum).  The probabilities get
// the same split, so q.k, p.v and the normalisation all carry f32-level error.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace pyxis {

// The exponent e of a group whose largest magnitude is `m` (0 for 0, Inf or NaN), in [-64, 64].
__host__ __device__ inline int attn_scale_exp(float m) {
    if (!(m > 0.f) || !(m < 3.0e38f)) return 0;
    int ex;
#ifdef __CUDA_ARCH__
    ex = (int)((__float_as_uint(m) >> 23) & 0xFFu) - 127;  // floor(log2 m) for normal m
#else
    uint32_t u;
    __builtin_memcpy(&u, &m, 4);
    ex = (int)((u >> 23) & 0xFFu) - 127;
#endif
    const int e = 14 - ex;
    return e < -64 ? -64 : (e > 64 ? 64 : e);
}
// 2^e for e in [-126, 127], exactly.
__host__ __device__ inline float attn_pow2(int e) {
    const uint32_t u = (uint32_t)(127 + e) << 23;
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}

// Operand buffers of one prefill chunk of `cs` sequences of P positions, Pp = P rounded up to 128:
//   q  [2][cs][n_q][Pp][hd]   fp16, hi rows then lo rows, written by the QK-norm/RoPE kernel
//   qinv [cs][n_q][Pp]        2^-e of each query row
//   k  [2][cs][n_kv][Pp][hd]  fp16 hi then lo, positions >= P zero
//   vt [2][cs][n_kv][hd][Pp]  fp16 hi then lo, V transposed (keys contiguous), positions >= P zero
//   kvmax [cs][n_kv][2]       max |k|, max |v| of the kv head over the prompt (f32 bits, atomicMax)
struct AttnTcBuffers {
    __half *q = nullptr, *k = nullptr, *vt = nullptr;
    float *qinv = nullptr;
    unsigned *kvmax = nullptr;
};
__host__ __device__ inline int attn_tc_padded(int P) { return (P + 127) / 128 * 128; }
bool attn_tc_supported(int head_dim);

// K and V of the chunk's cache rows (this layer; row j of sequence s at kc / vc + s * cache_stride
// + j * n_kv * hd) -> the fp16 operands, with the scales of kvmax.
cudaError_t launch_attn_prep_kv(const float *kc, const float *vc, long long cache_stride, int cs, int P, int n_kv,
                                int hd, const AttnTcBuffers &b, cudaStream_t st);
// out[(s * P + i) * n_q * hd + h * hd + d]: the attention output of every query row of the chunk.
cudaError_t launch_attention_prefill_tc(int cs, int P, int n_q, int n_kv, int hd, const AttnTcBuffers &b, float *out,
                                        int *err, cudaStream_t st);

}  // namespace pyxis
