// heads.cuh -- per-head helpers shared by the decode kernels (decode.cu, decode_batch.cu).
#pragma once

#include "common.cuh"

namespace pyxis {

constexpr int kAttnMaxG = 4;  // query heads per kv head the attention kernels take

template <int EPL>
PYXIS_DEVINL void load_head(const float *p, float (&v)[EPL]) {
    if constexpr (EPL == 4) {
        const float4 t = *reinterpret_cast<const float4 *>(p);
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
    } else {
        const float2 t = *reinterpret_cast<const float2 *>(p);
        v[0] = t.x, v[1] = t.y;
    }
}

// This lane's EPL floats of a head row, global -> shared without registers (cp.async: 16 bytes
// bypassing L1, or 8 bytes through it for EPL = 2); complete after cp_async_wait<n>().
template <int EPL>
PYXIS_DEVINL void cp_async_head(float *dst_smem, const float *src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst_smem);
    if constexpr (EPL == 4)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(src) : "memory");
}
PYXIS_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
PYXIS_DEVINL void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// QK RMSNorm (optional) and RoPE of one head held across a warp.
template <int EPL>
PYXIS_DEVINL void norm_rope(float (&v)[EPL], const float *nw, const float *rcos, const float *rsin, int pos,
                            float eps, int lane) {
    constexpr int HD = 32 * EPL, HALF = HD / 2;
    if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int t = 0; t < EPL; ++t) ss = __fadd_rn(ss, __fmul_rn(v[t], v[t]));
        ss = warp_sum(ss);
        const float factor = rms_factor(ss, HD, eps);
#pragma unroll
        for (int t = 0; t < EPL; ++t) v[t] = rms_scale(v[t], factor, nw[lane * EPL + t]);
    }
    const bool lo = lane < 16;
#pragma unroll
    for (int t = 0; t < EPL; ++t) {
        const float other = __shfl_xor_sync(0xffffffffu, v[t], 16);
        const int i = (lane & 15) * EPL + t;  // pair index in [0, HALF)
        const float c = rcos[(size_t)pos * HALF + i], s = rsin[(size_t)pos * HALF + i];
        v[t] = rope_rot(v[t], other, c, s, lo);
    }
}

}  // namespace pyxis
