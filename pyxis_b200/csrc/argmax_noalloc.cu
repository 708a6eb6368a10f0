// argmax_noalloc.cu -- the row-wise argmax of argmax.cu for callers that cannot allocate device
// memory: its scratch lives in a fixed array in the library's own device image instead of in a
// context (see pyxis_cuda_argmax_noalloc in include/pyxis_cuda.h).
#include "../../include/pyxis_cuda.h"
#include "argmax.h"
#include "kernels.h"

namespace pyxis {
namespace {

constexpr size_t kNoAllocMaxRows = 64;
constexpr size_t kPartialBytes = kNoAllocMaxRows * kArgmaxMaxCtasPerRow * sizeof(uint64_t);  // 32 KiB
constexpr size_t kScratchBytes = kPartialBytes + kNoAllocMaxRows * sizeof(unsigned);

// The scratch every call shares: per-CTA partial keys, then one ticket counter per row.  Loaded
// (zero-filled) with the library on every device that uses it and kept until the process exits.
// In host code this name is only a stand-in for the symbol: the device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_argmax_scratch[kScratchBytes];

// Device address of g_argmax_scratch on the current device.  Looked up on every call
// (cudaGetSymbolAddress allocates nothing): an address kept from an earlier call would be stale
// after the application resets the device (cudaDeviceReset) and its context is re-created.
cudaError_t scratch_for_current_device(void **out) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_argmax_scratch);
    if (e != cudaSuccess) return e;
    *out = ptr;
    return cudaSuccess;
}

}  // namespace
}  // namespace pyxis

extern "C" int pyxis_cuda_argmax_noalloc(const float *values, size_t M, size_t n, size_t ld, int64_t index_base,
                                         int32_t *idx, float *val, void *stream) {
    using namespace pyxis;
    if (M == 0) return PYXIS_OK;
    if (M > kNoAllocMaxRows)
        return record_error(PYXIS_EINVAL, "pyxis_cuda_argmax_noalloc: more than 64 rows per call (its fixed scratch holds 64)");
    if (n == 0) return record_error(PYXIS_EINVAL, "pyxis_cuda_argmax_noalloc: empty row");
    if (n > 0xFFFFFFFFull) return record_error(PYXIS_EINVAL, "pyxis_cuda_argmax_noalloc: row longer than 2^32 - 1");
    if (M > 1 && ld < n) return record_error(PYXIS_EINVAL, "pyxis_cuda_argmax_noalloc: row stride smaller than the row");
    if (!values || !idx) return record_error(PYXIS_EINVAL, "pyxis_cuda_argmax_noalloc: null values or idx");
    if (index_base < 0 || index_base + (int64_t)n - 1 > (int64_t)INT32_MAX)
        return record_error(PYXIS_EINVAL, "pyxis_cuda_argmax_noalloc: index_base + n - 1 outside [0, 2^31 - 1]");
    void *base = nullptr;
    cudaError_t e = scratch_for_current_device(&base);
    if (e != cudaSuccess) return record_error(PYXIS_ECUDA, cudaGetErrorString(e));
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return record_error(PYXIS_ECUDA, "pyxis_cuda_argmax_noalloc: device query failed");
    ArgmaxScratch s;
    s.partial = reinterpret_cast<uint64_t *>(base);
    s.ticket = reinterpret_cast<unsigned *>(reinterpret_cast<unsigned char *>(base) + kPartialBytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // The tickets must start at zero: clear them on the stream rather than trust the last call.
    e = cudaMemsetAsync(s.ticket, 0, M * sizeof(unsigned), st);
    if (e == cudaSuccess) e = launch_argmax_scratch(values, M, n, ld, index_base, idx, val, s, sms, st);
    if (e != cudaSuccess) return record_error(PYXIS_ECUDA, cudaGetErrorString(e));
    return PYXIS_OK;
}
