// argmax.cu -- row-wise argmax with the reference's tie and NaN rules (src/output_head.rs:30-44).
//
// The reference scans left to right and replaces the running maximum only on a strict `>`:
//   - ties go to the lowest index;
//   - a NaN is never `>` anything, so NaNs are skipped -- unless values[0] is NaN, in which case
//     nothing ever beats it and the answer is 0 (for a shard of a longer vector, index_base > 0,
//     that rule belongs to the shard holding index 0, so the shard skips a leading NaN);
//   - +0.0 > -0.0 is false, so the two zeros tie (lowest index wins).
// Here every element becomes a 64-bit key (order-preserving float bits << 32 | ~index), the
// maximum key is the reference's answer, and max is associative, so CTAs reduce their segments
// in any order.  One launch: each CTA writes its segment's key to scratch, and the last CTA to
// finish a row (atomic ticket) reduces the row's keys and re-arms the ticket to 0 for the next
// launch.  Scratch: ArgmaxScratch, zeroed once when it is allocated.
// For a vocab shard of a multi-GPU head the kernel can instead write each row's key with the
// global index in its low word (key_out): the maximum of the shards' keys is then the global
// answer, a NaN at global index 0 being the all-ones key.
#include "argmax.h"
#include "common.cuh"
#include "kernels.h"

namespace pyxis {

// Reduce a CTA's 64-bit keys; result valid in thread 0.
PYXIS_DEVINL uint64_t cta_max_u64(uint64_t k, uint64_t *red) {
    k = warp_max_u64(k);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = k;
    __syncthreads();
    if (warp == 0) {
        k = lane < (int)(blockDim.x >> 5) ? red[lane] : 0;
        k = warp_max_u64(k);
    }
    return k;
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(
    const float *__restrict__ values, size_t n, size_t ld, int64_t index_base,
    int32_t *__restrict__ idx_out, float *__restrict__ val_out, uint64_t *__restrict__ key_out, ArgmaxScratch s) {
    __shared__ uint64_t red[kArgmaxThreads / 32];
    __shared__ bool last;
    pdl_wait();
    pdl_trigger();
    const size_t row = blockIdx.y;
    const float *v = values + row * ld;
    const size_t seg = (n + gridDim.x - 1) / gridDim.x;
    const size_t beg = (size_t)blockIdx.x * seg;
    const size_t end = beg + seg < n ? beg + seg : n;
    uint64_t k = 0;
    for (size_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
        uint64_t c = argmax_key(__ldg(v + i), (uint32_t)i);
        k = c > k ? c : k;
    }
    k = cta_max_u64(k, red);
    if (threadIdx.x == 0) {
        s.partial[row * gridDim.x + blockIdx.x] = k;
        __threadfence();
        const unsigned ticket = atomicAdd(&s.ticket[row], 1u);
        last = ticket == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    uint64_t m = 0;
    for (unsigned c = threadIdx.x; c < gridDim.x; c += blockDim.x) {
        uint64_t p = __ldcg(&s.partial[row * gridDim.x + c]);
        m = p > m ? p : m;
    }
    m = cta_max_u64(m, red);
    if (threadIdx.x == 0) {
        uint32_t i = 0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFu);
        // values[0] NaN wins -- when this row starts the vector (index_base 0); a vocab shard
        // that starts later ignores NaNs like every other position.  All-NaN -> first index.
        const bool nan0 = index_base == 0 && isnan(v[0]);
        if (nan0 || m == 0) i = 0;
        if (key_out) {
            const uint32_t g = (uint32_t)(index_base + (int64_t)i);
            key_out[row] = nan0 ? ~0ull : m == 0 ? 0ull : ((m & 0xFFFFFFFF00000000ull) | (uint64_t)(0xFFFFFFFFu - g));
        } else {
            idx_out[row] = (int32_t)(index_base + (int64_t)i);
            if (val_out) val_out[row] = v[i];
        }
        s.ticket[row] = 0;  // re-arm for the next launch on this scratch
    }
}

void set_argmax_carveout_max() {
    cudaFuncSetAttribute(argmax_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}

int argmax_ctas_per_row(size_t n, int num_sms) {
    size_t c = (n + 4095) / 4096;
    if (c > (size_t)kArgmaxMaxCtasPerRow) c = kArgmaxMaxCtasPerRow;
    if (c > (size_t)num_sms) c = num_sms;
    return c < 1 ? 1 : (int)c;
}

cudaError_t launch_argmax_scratch(const float *values, size_t M, size_t n, size_t ld,
                                  int64_t index_base, int32_t *idx, float *val,
                                  const ArgmaxScratch &s, int num_sms, cudaStream_t st) {
    if (M == 0) return cudaSuccess;
    dim3 grid(argmax_ctas_per_row(n, num_sms), (unsigned)M);
    return launch_kernel(argmax_kernel, grid, dim3(kArgmaxThreads), 0, st, values, n, ld, index_base, idx, val,
                         (uint64_t *)nullptr, s);
}

cudaError_t launch_argmax_keys(const float *values, size_t M, size_t n, size_t ld, int64_t index_base,
                               uint64_t *keys, const ArgmaxScratch &s, int num_sms, cudaStream_t st) {
    if (M == 0) return cudaSuccess;
    dim3 grid(argmax_ctas_per_row(n, num_sms), (unsigned)M);
    return launch_kernel(argmax_kernel, grid, dim3(kArgmaxThreads), 0, st, values, n, ld, index_base,
                         (int32_t *)nullptr, (float *)nullptr, keys, s);
}

// tokens[r] = the index in the largest of the nranks keys of row row0 + r (keys_all [nranks][rows]);
// one CTA, which then zeroes keys_all and zero_keys for the next call.
__global__ void pick_keys_kernel(uint64_t *__restrict__ keys_all, int nranks, int rows, int row0, int nrows,
                                 int32_t *__restrict__ tokens, uint64_t *__restrict__ zero_keys, int zero_n) {
    pdl_wait();
    pdl_trigger();
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
        uint64_t m = 0;
        for (int w = 0; w < nranks; ++w) {
            const uint64_t k = keys_all[(size_t)w * rows + row0 + r];
            m = k > m ? k : m;
        }
        tokens[r] = m == 0 ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFu));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nranks * rows; i += blockDim.x) keys_all[i] = 0;
    for (int i = threadIdx.x; i < zero_n; i += blockDim.x) zero_keys[i] = 0;
}

cudaError_t launch_pick_keys(uint64_t *keys_all, int nranks, int rows, int row0, int nrows, int32_t *tokens,
                             uint64_t *zero_keys, int zero_n, cudaStream_t st) {
    if (nrows <= 0 && zero_n <= 0) return cudaSuccess;
    return launch_kernel(pick_keys_kernel, dim3(1), dim3(256), 0, st, keys_all, nranks, rows, row0, nrows, tokens,
                         zero_keys, zero_n);
}

}  // namespace pyxis

