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

}  // namespace pyxis
