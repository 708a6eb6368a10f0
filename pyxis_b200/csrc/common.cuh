// common.cuh -- shared device helpers for the sm_100a kernels of libpyxis_cuda.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include <utility>

#define PYXIS_DEVINL __device__ __forceinline__

namespace pyxis {

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs (the launch code queries the real count)

// 16-byte streaming load of weight bytes: read once per call, so keep it out of L1 and ask L2 to
// fetch the whole 256-byte sector group (the rows are contiguous).
PYXIS_DEVINL uint4 ld_stream_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

PYXIS_DEVINL float ld_nc_f32(const float *p) {
    float r;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
    return r;
}

// --- int8 / int4 -> f32 without the conversion pipe ----------------------------------------
// A byte b placed in the low mantissa byte of 2^23 (0x4B000000) is the float 2^23 + b; one
// byte_perm builds it, one (paired) subtraction removes the offset.  Both exact.

// Signed int8 lanes: bias to unsigned first (x ^ 0x80 == x + 128), offset is 2^23 + 128.
constexpr float kMagicI8 = 8388736.0f;  // 2^23 + 128
// Unsigned nibble lanes holding q + 8: offset 2^23 + 8 gives q directly.
constexpr float kMagicU4 = 8388616.0f;  // 2^23 + 8

PYXIS_DEVINL float byte_to_magic(uint32_t word, int sel) {
    // result bytes: [word.byte(sel), 0x00, 0x00, 0x4B]
    return __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u | (uint32_t)sel));
}

PYXIS_DEVINL float2 f2(float a, float b) { return make_float2(a, b); }

// Runs `setup` (cudaFuncSetAttribute calls) once per device and returns its status.  A kernel's
// attributes belong to each device's copy of the module, so a process that drives several GPUs
// (one context per device) must set them on every device it launches on.  `done` is the call
// site's mask of devices already set up; a failed setup is retried on the next call.
template <typename F>
inline cudaError_t once_per_device(std::atomic<uint64_t> &done, F &&setup) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return setup();
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = setup();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

PYXIS_DEVINL float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
PYXIS_DEVINL float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Four signed int8 of `w` -> (q0,q1), (q2,q3) as exact floats.
PYXIS_DEVINL void i8x4_to_f32(uint32_t w, float2 &lo, float2 &hi) {
    uint32_t u = w ^ 0x80808080u;
    const float2 m = f2(-kMagicI8, -kMagicI8);
    lo = fadd2(f2(byte_to_magic(u, 0), byte_to_magic(u, 1)), m);
    hi = fadd2(f2(byte_to_magic(u, 2), byte_to_magic(u, 3)), m);
}

// Eight nibbles of `w` (element 2j = low nibble of byte j, 2j+1 = high nibble; stored q+8) ->
// e01 = (q0,q1), e23, e45, e67 as exact floats.
PYXIS_DEVINL void u4x8_to_f32(uint32_t w, float2 &e01, float2 &e23, float2 &e45, float2 &e67) {
    uint32_t lo = w & 0x0F0F0F0Fu;         // q0+8, q2+8, q4+8, q6+8
    uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;  // q1+8, q3+8, q5+8, q7+8
    const float2 m = f2(-kMagicU4, -kMagicU4);
    e01 = fadd2(f2(byte_to_magic(lo, 0), byte_to_magic(hi, 0)), m);
    e23 = fadd2(f2(byte_to_magic(lo, 1), byte_to_magic(hi, 1)), m);
    e45 = fadd2(f2(byte_to_magic(lo, 2), byte_to_magic(hi, 2)), m);
    e67 = fadd2(f2(byte_to_magic(lo, 3), byte_to_magic(hi, 3)), m);
}

PYXIS_DEVINL float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

PYXIS_DEVINL float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// ---- the decode step's row arithmetic, one definition for every kernel that applies it --------
// RMSNorm (src/rmsnorm.rs:11-20): factor = 1 / sqrt(sum(x^2) / n + eps), then x * (factor * w).
PYXIS_DEVINL float rms_factor(float sumsq, int n, float eps) {
    return __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(sumsq, (float)n), eps)));
}
PYXIS_DEVINL float rms_scale(float v, float factor, float w) { return __fmul_rn(v, __fmul_rn(factor, w)); }
// SiLU (src/ffn.rs:52-54): x / (1 + exp(-x)).
PYXIS_DEVINL float silu_f(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }
// RoPE (src/attention.rs:144-162) of element i of a head and its partner i +- head_dim / 2 at
// angle pos * theta^(-2i / head_dim): x c - y s for the first half, x c + y s for the second.
PYXIS_DEVINL float rope_rot(float v, float other, float c, float s, bool first_half) {
    return first_half ? __fsub_rn(__fmul_rn(v, c), __fmul_rn(other, s)) : __fadd_rn(__fmul_rn(v, c), __fmul_rn(other, s));
}

// ---- programmatic dependent launch ---------------------------------------------------------
// A kernel launched with programmatic stream serialization may start while its predecessor is
// still running; pdl_wait() blocks until the predecessor has completed and its writes are
// visible.  pdl_trigger() lets this kernel's own dependents start launching.  Both are no-ops
// for a kernel launched normally.
PYXIS_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
PYXIS_DEVINL void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host side: launches issued while a PdlScope is alive on this thread (the decode step's capture)
// carry the programmatic-serialization attribute.
bool pdl_enabled();
struct PdlScope {
    bool prev;
    PdlScope();
    ~PdlScope();
};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace pyxis
