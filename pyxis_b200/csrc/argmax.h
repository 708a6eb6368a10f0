// argmax.h -- scratch layout of the single-launch argmax (argmax.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace pyxis {

constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxMaxCtasPerRow = 64;
constexpr int kArgmaxMaxRows = 1024;  // rows per launch the context's scratch holds

// partial: [rows][ctas per row] keys; ticket: [rows] counters that must be 0 before the first
// launch (the kernel leaves them at 0 again).
struct ArgmaxScratch {
    uint64_t *partial;
    unsigned *ticket;
};

inline size_t argmax_scratch_bytes(size_t rows) {
    return rows * kArgmaxMaxCtasPerRow * sizeof(uint64_t) + rows * sizeof(unsigned);
}

int argmax_ctas_per_row(size_t n, int num_sms);

// Prefer the maximum shared-memory carveout (as the GEMV kernels it runs between do).
void set_argmax_carveout_max();

cudaError_t launch_argmax_scratch(const float *values, size_t M, size_t n, size_t ld,
                                  int64_t index_base, int32_t *idx, float *val,
                                  const ArgmaxScratch &s, int num_sms, cudaStream_t st);

// The same scan writing one 64-bit key per row instead of (idx, val): order-preserving value
// bits << 32 | (0xFFFFFFFF - (index_base + first index of the maximum)); 0 for a row of NaNs
// only; all ones for a NaN at global index 0 (index_base 0).  The maximum of several shards' keys
// of one row is the key of the whole row's first maximum.
cudaError_t launch_argmax_keys(const float *values, size_t M, size_t n, size_t ld, int64_t index_base,
                               uint64_t *keys, const ArgmaxScratch &s, int num_sms, cudaStream_t st);

// tokens[r] for r < nrows: the index in the largest key of row row0 + r over keys_all
// [nranks][rows] (0 when every key is 0).  Then zeroes keys_all and zero_keys[0, zero_n) (the
// local keys, which the tensor-core GEMV's epilogue max-reduces into: they must be 0 before it).
cudaError_t launch_pick_keys(uint64_t *keys_all, int nranks, int rows, int row0, int nrows, int32_t *tokens,
                             uint64_t *zero_keys, int zero_n, cudaStream_t st);

#ifdef __CUDACC__
// One element's key: order-preserving float bits << 32 | (0xFFFFFFFF - idx).  A NaN is 0, below
// every number (the reference's `>` never picks one), and -0.0 ties with +0.0.
__device__ __forceinline__ uint64_t argmax_key(float v, uint32_t idx) {
    if (isnan(v)) return 0;
    if (v == 0.0f) v = 0.0f;
    const uint32_t u = __float_as_uint(v);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)ord << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}

// The key of a logit at global vocabulary index g, as the shards' keys are compared: a NaN at
// index 0 wins over everything (nothing is `>` values[0] then), other NaNs lose to everything.
__device__ __forceinline__ uint64_t argmax_key_global(float v, long long g) {
    return (g == 0 && isnan(v)) ? ~0ull : argmax_key(v, (uint32_t)g);
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t other = __shfl_xor_sync(0xffffffffu, k, o);
        k = other > k ? other : k;
    }
    return k;
}
#endif

}  // namespace pyxis
