// decode.cu -- device-resident greedy decode (include/pyxis_decode.h).
//
// One step = one token at position pos through all layers, the lm_head and the argmax, entirely on
// the context's stream; the step reads the position, the input token and the output slot from
// device memory, so it is captured once into a CUDA graph and replayed for every token.  The
// kernels between the projections mirror the reference's f32 expressions (src/rmsnorm.rs:11-20,
// src/attention.rs:107-179, src/ffn.rs:39-54) with explicit round-to-nearest multiplies and adds
// where the reference's operation order is cheap to keep (no FMA contraction); sums of many
// terms are reduced in parallel.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <utility>
#include <vector>

#include "../../include/pyxis_decode.h"
#include "argmax.h"
#include "common.cuh"
#include "ctx.h"
#include "heads.cuh"
#include "kernels.h"
#include "model.h"

namespace pyxis {
namespace {

constexpr int kNormThreads = 1024;

PYXIS_DEVINL float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    __syncthreads();
    return t;
}

// x = widen(embedding[token]) (Embedding::lookup, src/embedding.rs:18-24 over bf16 -> f32).
__global__ void embed_kernel(const uint16_t *__restrict__ emb, const int *__restrict__ token, int vocab, int H,
                             float *__restrict__ x) {
    pdl_wait();
    pdl_trigger();
    int t = *token;
    t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
    const uint16_t *row = emb + (size_t)t * H;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
        x[i] = bf16_bits_to_f32(row[i]);
}

// Optional residual add (x += delta, src/transformer.rs:40-42, :54-59), then
// h = x * (factor * w), factor = 1 / sqrt(mean(x^2) + eps) (src/rmsnorm.rs:11-20).  One CTA of
// kNormThreads; each thread keeps its kNormPer values in registers, so x, delta and w are read in
// one pass (n <= kNormThreads * kNormPer).
constexpr int kNormPer = 8;
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float *__restrict__ x, const float *__restrict__ delta,
                                                                  const float *__restrict__ w, float *__restrict__ h,
                                                                  int n, float eps) {
    __shared__ float red[kNormThreads / 32];
    pdl_wait();
    pdl_trigger();
    float v[kNormPer], wv[kNormPer];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        v[j] = 0.f;
        wv[j] = 0.f;
        if (i < n) {
            v[j] = x[i];
            if (delta) v[j] = __fadd_rn(v[j], delta[i]);
            wv[j] = w[i];
        }
    }
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < n) {
            if (delta) x[i] = v[j];
            ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
        }
    }
    ss = block_sum(ss, red);
    const float factor = rms_factor(ss, n, eps);
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < n) h[i] = rms_scale(v[j], factor, wv[j]);
    }
}

// Attention for the newest position, fused with what precedes it (src/attention.rs:81-135):
// per-head QK RMSNorm (:81-90), RoPE at `pos` from the host-made table (:92-93, :144-162), the
// KV-cache append (:100), then causal GQA attention scores = (q . k_j) / sqrt(hd) for j <= pos,
// softmax (:164-179) and out = sum_j p_j v_j.
// Grid (splits, n_kv): CTA (s, h) handles the G = n_q / n_kv query heads of kv head h over the
// keys [s*len/S, (s+1)*len/S).  Every CTA normalises and rotates its heads' q and the new k itself
// (a few hundred flops), the CTA holding key `pos` writes k and v to the cache, and the newest
// key is taken from shared memory, so no CTA reads a cache row another one is writing.  Within a
// CTA each warp takes every 8th key and streams its K and V rows through its own ring of
// kAttnRing keys in shared memory with cp.async (the first ones before griddepcontrol.wait; data
// in flight holds no registers, so three CTAs of 8 warps keep ~96 KB per SM in flight), and keeps
// a running (max, sum of exp, sum of p v) per query head; the
// warps, then the splits (the last CTA of a kv head, by ticket), are rescaled to a common max and
// added in a fixed order.  The softmax is the reference's up to the order of the f32 sums.
// Lane l of a warp holds head elements [l*EPL, (l+1)*EPL); RoPE pairs element i with i + hd/2,
// which sits in lane l ^ 16.
constexpr int kAttnThreads = 256;
constexpr int kAttnRing = 8;  // keys per warp in its cp.async ring: PF being scored, the rest in flight
template <int EPL>
constexpr size_t attn_ring_bytes() { return (size_t)(kAttnThreads / 32) * kAttnRing * 2 * (32 * EPL) * sizeof(float); }
template <int EPL, int G>
__global__ void __launch_bounds__(kAttnThreads)
    attention_step_kernel(const float *__restrict__ qkv, const float *__restrict__ q_norm,
                          const float *__restrict__ k_norm, const float *__restrict__ rcos,
                          const float *__restrict__ rsin, const int *__restrict__ d_pos, int n_q, int n_kv, float eps,
                          float *__restrict__ kcache, float *__restrict__ vcache, float *__restrict__ part,
                          unsigned *__restrict__ tickets, float *__restrict__ out, long long qkv_stride,
                          long long cache_stride, long long out_stride) {
    constexpr int HD = 32 * EPL, PF = 4;  // keys scored per round
    constexpr int NW = kAttnThreads / 32, R = kAttnRing;
    static_assert(R > PF, "the ring must hold the round being scored and keys in flight");
    __shared__ float qs[G][HD], knew[HD], vnew[HD];
    __shared__ float wpart[NW][G][HD + 2];  // per-warp (max, sum, acc[HD])
    __shared__ int flag;
    extern __shared__ float4 attn_ring_raw[];  // [NW][R][K row | V row]
    const int S = gridDim.x, s = blockIdx.x, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_dim = n_kv * HD, q_dim = n_q * HD;
    {  // sequence blockIdx.z of a batch
        const long long z = blockIdx.z;
        qkv += z * qkv_stride;
        kcache += z * cache_stride;
        vcache += z * cache_stride;
        out += z * out_stride;
        part += z * (long long)n_kv * S * G * (HD + 2);
        tickets += z * n_kv;
    }
    // The position and the cache rows below it were written by earlier steps (earlier graph
    // launches): read them, and this warp's first keys, before waiting on the q|k|v projection.
    const int pos = *d_pos;
    const int len = pos + 1;
    const int j0 = (int)((long long)s * len / S), j1 = (int)((long long)(s + 1) * len / S);
    // this warp's keys j0 + warp + i * NW, i < nk; key i sits in ring slot i % R
    const int nk = j0 + warp < j1 ? (j1 - 1 - (j0 + warp)) / NW + 1 : 0;
    float *ring = reinterpret_cast<float *>(attn_ring_raw) + (size_t)warp * R * 2 * HD + lane * EPL;
    auto issue = [&](int i) {  // one commit group per key (empty past the warp's keys)
        const int j = j0 + warp + i * NW;
        if (i < nk && j < pos) {  // key pos is the new one: taken from shared memory below
            float *slot = ring + (size_t)(i % R) * 2 * HD;
            cp_async_head<EPL>(slot, kcache + (size_t)j * kv_dim + (size_t)h * HD + lane * EPL);
            cp_async_head<EPL>(slot + HD, vcache + (size_t)j * kv_dim + (size_t)h * HD + lane * EPL);
        }
        cp_async_commit();
    };
#pragma unroll
    for (int i = 0; i < R - PF; ++i) issue(i);
    pdl_wait();
    pdl_trigger();

    // heads of this kv group: warps 0..G-1 the q heads, warp G the new k, warp G+1 the new v
    if (warp < G) {
        float v[EPL];
        load_head<EPL>(qkv + (size_t)(h * G + warp) * HD + lane * EPL, v);
        norm_rope<EPL>(v, q_norm, rcos, rsin, pos, eps, lane);
#pragma unroll
        for (int t = 0; t < EPL; ++t) qs[warp][lane * EPL + t] = v[t];
    } else if (warp == G) {
        float v[EPL];
        load_head<EPL>(qkv + q_dim + (size_t)h * HD + lane * EPL, v);
        norm_rope<EPL>(v, k_norm, rcos, rsin, pos, eps, lane);
#pragma unroll
        for (int t = 0; t < EPL; ++t) {
            knew[lane * EPL + t] = v[t];
            if (s == S - 1) kcache[(size_t)pos * kv_dim + (size_t)h * HD + lane * EPL + t] = v[t];
        }
    } else if (warp == G + 1) {
        float v[EPL];
        load_head<EPL>(qkv + q_dim + kv_dim + (size_t)h * HD + lane * EPL, v);
#pragma unroll
        for (int t = 0; t < EPL; ++t) {
            vnew[lane * EPL + t] = v[t];
            if (s == S - 1) vcache[(size_t)pos * kv_dim + (size_t)h * HD + lane * EPL + t] = v[t];
        }
    }
    __syncthreads();

    // this warp's keys j0 + warp, j0 + warp + NW, ...: online softmax per query head
    const float scale = sqrtf((float)HD);
    float qr[G][EPL], acc[G][EPL], m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int t = 0; t < EPL; ++t) {
            acc[g][t] = 0.f;
            qr[g][t] = 0.f;
            if (g < G) qr[g][t] = qs[g][lane * EPL + t];
        }
    }
    // Each round: the copies of the keys R - PF ahead are issued, the round's PF keys are read
    // back from the ring (each lane its own elements, so no warp barrier), scored -- all PF x G
    // dot products reduced together (interleaved shuffles) -- and folded into the running softmax
    // with one rescale per round.
    for (int i0 = 0; i0 < nk; i0 += PF) {
        const int jb = j0 + warp + i0 * NW;
#pragma unroll
        for (int u = 0; u < PF; ++u) issue(i0 + R - PF + u);
        cp_async_wait<R - PF>();  // keys up to i0 + PF - 1 have landed
        float kr[PF][EPL], vr[PF][EPL];
        float dot[PF][G];
#pragma unroll
        for (int u = 0; u < PF; ++u) {
            if (jb + u * NW == pos) {
#pragma unroll
                for (int t = 0; t < EPL; ++t) {
                    kr[u][t] = knew[lane * EPL + t];
                    vr[u][t] = vnew[lane * EPL + t];
                }
            } else if (i0 + u < nk) {
                const float *slot = ring + (size_t)((i0 + u) % R) * 2 * HD;
                load_head<EPL>(slot, kr[u]);
                load_head<EPL>(slot + HD, vr[u]);
            } else {
#pragma unroll
                for (int t = 0; t < EPL; ++t) kr[u][t] = vr[u][t] = 0.f;  // past the split: scored -inf
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                dot[u][g] = 0.f;
#pragma unroll
                for (int t = 0; t < EPL; ++t) dot[u][g] = __fmaf_rn(qr[g][t], kr[u][t], dot[u][g]);  // a sum reduced in parallel: fused
            }
        }
        // The round's PF x G dot products, each reduced over the 32 lanes.  With NP = PF G a power
        // of two, a reduce-scatter (levels xor 16, 8, ... keeping half the values each, then full
        // levels) leaves pair p on the lanes pair_lane(p) + [0, 32 / NP): the same additions in the
        // same tree as a per-value butterfly, with log2-many fewer shuffles.  The division and the
        // exponential of each (key, head) pair, and each head's rescale factor, are then computed
        // once (on the pair's first lane, the factor of head g on pair g's second) and shuffled to
        // every lane: a tenth of the issue, the same operations on the same values.
        constexpr int NP = PF * G;
        constexpr bool RS = (NP & (NP - 1)) == 0 && NP >= 2 && NP <= 16;
        constexpr int LPP = RS ? 32 / NP : 1;  // lanes holding one pair after the reduction
        auto pair_lane = [](int pp) {
            if constexpr (RS) {
                int L = 0;
#pragma unroll
                for (int j = 0, o = 16, w = NP / 2; w >= 1; ++j, o >>= 1, w >>= 1)
                    if (pp & w) L |= o;
                return L;
            } else {
                return pp;
            }
        };
        float dsel = 0.f;
        int pl = lane;  // the pair whose scalars this lane computes
        if constexpr (RS) {
            float v[NP];
#pragma unroll
            for (int u = 0; u < PF; ++u)
#pragma unroll
                for (int g = 0; g < G; ++g) v[u * G + g] = dot[u][g];
            pl = 0;
#pragma unroll
            for (int o = 16, n = NP; n > 1; o >>= 1, n >>= 1) {
                const bool upper = (lane & o) != 0;
                if (upper) pl += n / 2;
#pragma unroll
                for (int i = 0; i < n / 2; ++i) {
                    const float send = upper ? v[i] : v[i + n / 2];
                    const float keep = upper ? v[i + n / 2] : v[i];
                    v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
                }
            }
#pragma unroll
            for (int o = 16 / NP; o > 0; o >>= 1) v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], o));
            dsel = v[0];
        } else {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int u = 0; u < PF; ++u)
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        dot[u][g] = __fadd_rn(dot[u][g], __shfl_xor_sync(0xffffffffu, dot[u][g], o));
#pragma unroll
            for (int u = 0; u < PF; ++u)
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (lane == u * G + g) dsel = dot[u][g];
        }
        const int pu = pl / G;
        const float sc_l = pl < NP && jb + pu * NW < j1 ? __fdiv_rn(dsel, scale) : -INFINITY;
        float sc[PF][G], mn[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mt = -INFINITY;
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                sc[u][g] = __shfl_sync(0xffffffffu, sc_l, pair_lane(u * G + g));
                mt = fmaxf(mt, sc[u][g]);
            }
            mn[g] = fmaxf(m[g], mt);  // finite: the round has >= 1 key
        }
        // exponential arguments: pair pl on its first lane, head g's factor on pair g's second lane
        // (RS) or on lane NP + g
        const int sub = RS ? (lane & (LPP - 1)) : 0;
        const int cg = RS ? (sub == 1 ? pl : -1) : lane - NP;
        float ex_arg = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int u = 0; u < PF; ++u)
                if (sub == 0 && pl == u * G + g) ex_arg = __fsub_rn(sc[u][g], mn[g]);
            if (cg == g) ex_arg = __fsub_rn(m[g], mn[g]);  // -inf on the first round: c = 0
        }
        const float ex_l = expf(ex_arg);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (g >= G) break;
            const float c = __shfl_sync(0xffffffffu, ex_l, RS ? pair_lane(g) + 1 : NP + g);
            float ps = 0.f;
#pragma unroll
            for (int t = 0; t < EPL; ++t) acc[g][t] = __fmul_rn(acc[g][t], c);
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const float pj = __shfl_sync(0xffffffffu, ex_l, pair_lane(u * G + g));
                if (jb + u * NW >= j1) break;  // past the split's end: those rows were never loaded
                ps = __fadd_rn(ps, pj);
#pragma unroll
                for (int t = 0; t < EPL; ++t) acc[g][t] = __fmaf_rn(pj, vr[u][t], acc[g][t]);
            }
            l[g] = __fadd_rn(__fmul_rn(l[g], c), ps);
            m[g] = mn[g];
        }
    }
    cp_async_wait<0>();  // only empty groups can be left: nothing in flight past this point
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (g >= G) break;
        if (lane == 0) {
            wpart[warp][g][0] = m[g];
            wpart[warp][g][1] = l[g];
        }
#pragma unroll
        for (int t = 0; t < EPL; ++t) wpart[warp][g][2 + lane * EPL + t] = acc[g][t];
    }
    __syncthreads();

    // this split: the warps' partials rescaled to their common max and added in warp order
    float *mine = part + ((size_t)h * S + s) * G * (HD + 2);
    for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
        const int g = idx / HD, d = idx - g * HD;
        float M = -INFINITY;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, wpart[w][g][0]);
        float L = 0.f, a = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < NW; ++w) {
                const float mw = wpart[w][g][0];
                if (mw == -INFINITY) continue;  // a warp without keys
                const float c = expf(__fsub_rn(mw, M));
                L = __fadd_rn(L, __fmul_rn(wpart[w][g][1], c));
                a = __fadd_rn(a, __fmul_rn(wpart[w][g][2 + d], c));
            }
        }
        if (S == 1) {
            out[(size_t)(h * G + g) * HD + d] = __fdiv_rn(a, L);
        } else {
            if (d == 0) {
                mine[g * (HD + 2)] = M;
                mine[g * (HD + 2) + 1] = L;
            }
            mine[g * (HD + 2) + 2 + d] = a;
        }
    }
    if (S == 1) return;

    // the last CTA of this kv head combines the splits in order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) flag = atomicAdd(&tickets[h], 1u) == (unsigned)(S - 1);
    __syncthreads();
    if (!flag) return;
    __threadfence();
    const float *all = part + (size_t)h * S * G * (HD + 2);
    for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
        const int g = idx / HD, d = idx - g * HD;
        float M = -INFINITY;
        for (int t = 0; t < S; ++t) M = fmaxf(M, __ldcg(all + ((size_t)t * G + g) * (HD + 2)));
        float L = 0.f, a = 0.f;
        for (int t = 0; t < S; ++t) {
            const float *pt = all + ((size_t)t * G + g) * (HD + 2);
            const float mt = __ldcg(pt);
            if (mt == -INFINITY) continue;  // an empty split
            const float c = expf(__fsub_rn(mt, M));
            L = __fadd_rn(L, __fmul_rn(__ldcg(pt + 1), c));
            a = __fadd_rn(a, __fmul_rn(__ldcg(pt + 2 + d), c));
        }
        out[(size_t)(h * G + g) * HD + d] = __fdiv_rn(a, L);
    }
    if (threadIdx.x == 0) tickets[h] = 0;
}

// act = silu(gate) * up, silu(x) = x / (1 + exp(-x)) (src/ffn.rs:39-41, :52-54).
__global__ void silu_mul_kernel(const float *__restrict__ gu, int ffn, float *__restrict__ act) {
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ffn; i += gridDim.x * blockDim.x) {
        const float g = gu[i];
        act[i] = __fmul_rn(silu_f(g), gu[ffn + i]);
    }
}

// Records the argmax token of this step and advances the position / step counters.
__global__ void advance_kernel(const int *__restrict__ token, int *__restrict__ out, int *pos, int *step) {
    pdl_wait();
    pdl_trigger();
    const int s = *step;
    out[s] = *token;
    *step = s + 1;
    *pos = *pos + 1;
}

}  // namespace
}  // namespace pyxis

cudaError_t pyxis::launch_attention_step(const pyxis_model_config &c, int splits, int n_seq, const float *qkv,
                                         size_t qkv_stride, const float *q_norm, const float *k_norm,
                                         const float *rope_cos, const float *rope_sin, const int *d_pos, float *kc,
                                         float *vc, size_t cache_stride, float *part, unsigned *tickets, float *out,
                                         size_t out_stride, cudaStream_t st) {
    using Kern = void (*)(const float *, const float *, const float *, const float *, const float *, const int *, int,
                          int, float, float *, float *, float *, unsigned *, float *, long long, long long, long long);
    static const Kern k128[] = {attention_step_kernel<4, 1>, attention_step_kernel<4, 2>, attention_step_kernel<4, 3>,
                                attention_step_kernel<4, 4>};
    static const Kern k64[] = {attention_step_kernel<2, 1>, attention_step_kernel<2, 2>, attention_step_kernel<2, 3>,
                               attention_step_kernel<2, 4>};
    const int G = c.n_q_heads / c.n_kv_heads;
    const Kern kern = (c.head_dim == 128 ? k128 : k64)[G - 1];
    const size_t ring = c.head_dim == 128 ? attn_ring_bytes<4>() : attn_ring_bytes<2>();
    static std::atomic<uint64_t> attr_done{0};
    const cudaError_t attr = once_per_device(attr_done, [&] {
        bool ok = true;
        for (int g = 0; g < 4; ++g) {
            ok &= cudaFuncSetAttribute(k128[g], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)attn_ring_bytes<4>()) == cudaSuccess;
            ok &= cudaFuncSetAttribute(k64[g], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)attn_ring_bytes<2>()) == cudaSuccess;
            // all of the SM's L1 as shared memory: three CTAs' rings (~76 KB each) fit only then
            ok &= cudaFuncSetAttribute(k128[g], cudaFuncAttributePreferredSharedMemoryCarveout, 100) == cudaSuccess;
            ok &= cudaFuncSetAttribute(k64[g], cudaFuncAttributePreferredSharedMemoryCarveout, 100) == cudaSuccess;
        }
        return ok ? cudaSuccess : cudaErrorInvalidConfiguration;
    });
    if (attr != cudaSuccess) return attr;
    return launch_kernel(kern, dim3(splits, c.n_kv_heads, n_seq), dim3(kAttnThreads), ring, st, qkv, q_norm, k_norm,
                         rope_cos, rope_sin, d_pos, c.n_q_heads, c.n_kv_heads, c.rms_eps, kc, vc, part, tickets, out,
                         (long long)qkv_stride, (long long)cache_stride, (long long)out_stride);
}

using namespace pyxis;


namespace {

int model_fail(int code, const char *msg) { return record_error(code, msg); }

template <typename T>
cudaError_t dalloc(pyxis_cuda_model *m, T **p, size_t count) {
    void *v = nullptr;
    cudaError_t e = cudaMalloc(&v, count * sizeof(T) + 16);
    if (e == cudaSuccess) {
        m->allocs.push_back(v);
        *p = reinterpret_cast<T *>(v);
    }
    return e;
}

struct Guard {
    int prev = -1;
    explicit Guard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~Guard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

QMatrix qmat(const pyxis_cuda_weights *w, size_t N, size_t K) {
    return QMatrix{w->qtype, w->data, w->scales, w->block_size, N, K};
}

// y = W x' with x' = RMSNorm(x + delta) (CTA 0 of the GEMV stores x + delta to xout), fused into
// the GEMV's x staging when the shape allows, else the separate norm kernel and a plain GEMV.
int norm_gemv(pyxis_cuda_model *m, const pyxis_cuda_weights *w, size_t N, float *x, const float *delta,
              float *xout, const float *nw, float *y, cudaStream_t st) {
    const pyxis_model_config &c = m->cfg;
    const size_t H = c.hidden;
    GemvPrologue pro;
    pro.kind = kProAddNorm;
    pro.x = x;
    pro.delta = delta;
    pro.w = nw;
    pro.xout = xout;
    pro.eps = c.rms_eps;
    const QMatrix q = qmat(w, N, H);
    if (gemv_batch_pro_supported(q, pro, m->ctx->num_sms)) {
        cudaError_t e = launch_gemv_batch_pro(q, pro, y, m->ctx->d_err, m->ctx->num_sms, st);
        return e == cudaSuccess ? PYXIS_OK : model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    }
    // unfused: x + delta written to xout by the norm kernel, h = norm(xout)
    if (delta) {
        cudaError_t e = cudaMemcpyAsync(xout, x, H * sizeof(float), cudaMemcpyDeviceToDevice, st);
        if (e == cudaSuccess)
            e = launch_kernel(add_rmsnorm_kernel, dim3(1), dim3(kNormThreads), 0, st, xout, delta, nw, m->h, (int)H,
                              c.rms_eps);
        if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    } else {
        cudaError_t e = launch_kernel(add_rmsnorm_kernel, dim3(1), dim3(kNormThreads), 0, st, x, (const float *)nullptr,
                                      nw, m->h, (int)H, c.rms_eps);
        if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    }
    return run_matmul(m->ctx, w, m->h, 1, H, N, H, y, N, nullptr, 0, st);
}

// y = Wdown (SiLU(gate) * up) from the stacked [gate; up] output gu.
int silu_gemv(pyxis_cuda_model *m, const pyxis_cuda_weights *w, float *y, cudaStream_t st) {
    const pyxis_model_config &c = m->cfg;
    GemvPrologue pro;
    pro.kind = kProSiluMul;
    pro.x = m->gu;
    const QMatrix q = qmat(w, c.hidden, c.ffn);
    if (gemv_batch_pro_supported(q, pro, m->ctx->num_sms)) {
        cudaError_t e = launch_gemv_batch_pro(q, pro, y, m->ctx->d_err, m->ctx->num_sms, st);
        return e == cudaSuccess ? PYXIS_OK : model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    }
    cudaError_t e = launch_kernel(silu_mul_kernel, dim3((c.ffn + 255) / 256), dim3(256), 0, st, (const float *)m->gu,
                                  c.ffn, m->act);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    return run_matmul(m->ctx, w, m->act, 1, c.ffn, c.hidden, c.ffn, y, c.hidden, nullptr, 0, st);
}

// One decode step on `st` (what the graph holds).
int enqueue_step(pyxis_cuda_model *m, cudaStream_t st) {
    const pyxis_model_config &c = m->cfg;
    const int H = c.hidden;
    const size_t qkv_rows = (size_t)m->q_dim + 2 * m->kv_dim;
    PdlScope pdl;  // kernels of the step may start while their predecessor finishes
    cudaError_t le = launch_kernel(embed_kernel, dim3((H + 255) / 256), dim3(256), 0, st, (const uint16_t *)m->emb,
                                   (const int *)m->d_token, c.vocab, H, m->x);
    if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
    float *xr = m->x, *xw = m->x2;  // residual stream: read xr, the fused norm writes xr + delta to xw
    for (int l = 0; l < c.n_layers; ++l) {
        const auto &L = m->layers[l];
        float *kc = m->kcache + (size_t)l * c.max_seq * m->kv_dim;
        float *vc = m->vcache + (size_t)l * c.max_seq * m->kv_dim;
        // layer input: x (+ the previous layer's FFN output) -> RMSNorm -> q|k|v
        int rc = norm_gemv(m, L.wqkv, qkv_rows, xr, l ? m->tmp : nullptr, xw, L.in_norm, m->qkv, st);
        if (rc) return rc;
        if (l) std::swap(xr, xw);
        le = launch_attention_step(c, m->attn_splits, 1, m->qkv, 0, L.q_norm, L.k_norm, m->rope_cos, m->rope_sin,
                                   m->d_pos, kc, vc, 0, m->part, m->tickets, m->attn, 0, st);
        if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
        rc = run_matmul(m->ctx, L.wo, m->attn, 1, m->q_dim, H, m->q_dim, m->tmp, H, nullptr, 0, st);
        if (rc) return rc;
        // x + attention output -> RMSNorm -> gate|up, then SiLU(gate) * up -> down
        rc = norm_gemv(m, L.wgu, 2 * (size_t)c.ffn, xr, m->tmp, xw, L.post_norm, m->gu, st);
        if (rc) return rc;
        std::swap(xr, xw);
        rc = silu_gemv(m, L.wdown, m->tmp, st);
        if (rc) return rc;
    }
    le = launch_kernel(add_rmsnorm_kernel, dim3(1), dim3(kNormThreads), 0, st, xr, (const float *)m->tmp,
                       (const float *)m->final_norm, m->h, H, c.rms_eps);
    if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
    int rc = run_matmul(m->ctx, m->lm_head, m->h, 1, H, c.vocab, H, m->logits, c.vocab, nullptr, 0, st);
    if (rc) return rc;
    cudaError_t e = launch_argmax_scratch(m->logits, 1, c.vocab, c.vocab, 0, m->d_token, nullptr, m->ctx->amax,
                                          m->ctx->num_sms, st);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    e = launch_kernel(advance_kernel, dim3(1), dim3(1), 0, st, (const int *)m->d_token, m->d_out, m->d_pos, m->d_step);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    return PYXIS_OK;
}

// The decode model takes the quantized layouts (its fused GEMV prologues and the prefill GEMM
// are int8 / int4 kernels); unquantized rows go through pyxis_cuda_matmul*.
bool weights_ok(const pyxis_cuda_weights *w, size_t n, int device) {
    return w && w->num_elements == n && w->device == device &&
           (w->qtype == PYXIS_QTYPE_INT8 || w->qtype == PYXIS_QTYPE_INT4);
}

}  // namespace

extern "C" int pyxis_rope_table(float theta, int head_dim, int max_pos, float *cos_out, float *sin_out) {
    if (head_dim <= 0 || head_dim % 2 || max_pos < 0 || !cos_out || !sin_out)
        return model_fail(PYXIS_EINVAL, "pyxis_rope_table: bad arguments");
    const int half = head_dim / 2;
    std::vector<float> freq(half);
    for (int i = 0; i < half; ++i) freq[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);  // :151
    for (int p = 0; p < max_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const float angle = (float)p * freq[i];  // :152
            cos_out[(size_t)p * half + i] = cosf(angle);
            sin_out[(size_t)p * half + i] = sinf(angle);
        }
    return PYXIS_OK;
}

namespace pyxis {

// One CTA applies one of the decode step's row operations to n values with the device helpers
// the decode kernels use (rms_factor / rms_scale, rope_rot, silu_f): the known-answer checks of
// the device arithmetic.  RMSNorm sums x^2 over a CTA reduction like the row kernels do.
__global__ void row_op_kernel(int op, const float *__restrict__ x, int n, const float *__restrict__ w, float eps,
                              const float *__restrict__ rcos, const float *__restrict__ rsin, int head_dim, int pos,
                              float *__restrict__ out) {
    __shared__ float red[32];
    if (op == PYXIS_ROW_RMSNORM) {
        float ss = 0.f;
        for (int i = threadIdx.x; i < n; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot = __fadd_rn(tot, red[i]);
        const float factor = rms_factor(tot, n, eps);
        for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = rms_scale(x[i], factor, w[i]);
    } else if (op == PYXIS_ROW_ROPE) {
        const int half = head_dim / 2;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const int j = i % head_dim, base = i - j;
            const bool first = j < half;
            const int pair = first ? j : j - half;
            const float other = x[base + (first ? j + half : j - half)];
            out[i] = rope_rot(x[i], other, rcos[(size_t)pos * half + pair], rsin[(size_t)pos * half + pair], first);
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = silu_f(x[i]);
    }
}

}  // namespace pyxis

extern "C" int pyxis_cuda_row_op(pyxis_cuda_ctx *ctx, int op, const float *x, size_t n, const float *w, float eps,
                                 int head_dim, int pos, float theta, float *out) {
    if (!ctx || !x || !out) return model_fail(PYXIS_EINVAL, "null argument");
    if (op != PYXIS_ROW_RMSNORM && op != PYXIS_ROW_ROPE && op != PYXIS_ROW_SILU)
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_row_op: unknown op");
    if (n == 0) return PYXIS_OK;
    if (n > 65536) return model_fail(PYXIS_EINVAL, "pyxis_cuda_row_op: more than 65536 values");
    if (op == PYXIS_ROW_RMSNORM && !w) return model_fail(PYXIS_EINVAL, "pyxis_cuda_row_op: RMSNorm needs a weight");
    if (op == PYXIS_ROW_ROPE && (head_dim <= 0 || head_dim % 2 || n % (size_t)head_dim || pos < 0 || pos > 1 << 20))
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_row_op: RoPE needs whole heads of even head_dim and pos >= 0");
    Guard g(ctx->device);
    const size_t half = op == PYXIS_ROW_ROPE ? (size_t)head_dim / 2 : 0;
    const size_t ntab = (size_t)(pos + 1) * half;
    std::vector<float> cs(ntab), sn(ntab);
    if (op == PYXIS_ROW_ROPE) pyxis_rope_table(theta, head_dim, pos + 1, cs.data(), sn.data());
    float *d = nullptr;
    const size_t total = 3 * n + 2 * ntab;
    cudaError_t e = cudaMalloc(&d, total * sizeof(float));
    if (e != cudaSuccess) return model_fail(PYXIS_ENOMEM, cudaGetErrorString(e));
    float *dx = d, *dw = d + n, *dout = d + 2 * n, *dc = d + 3 * n, *ds = dc + ntab;
    e = cudaMemcpy(dx, x, n * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && op == PYXIS_ROW_RMSNORM) e = cudaMemcpy(dw, w, n * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && ntab) e = cudaMemcpy(dc, cs.data(), ntab * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && ntab) e = cudaMemcpy(ds, sn.data(), ntab * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        pyxis::row_op_kernel<<<1, 256, 0, ctx->stream>>>(op, dx, (int)n, dw, eps, dc, ds, head_dim, pos, dout);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpy(out, dout, n * sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    return PYXIS_OK;
}

extern "C" int pyxis_cuda_model_create(pyxis_cuda_ctx *ctx, const pyxis_model_config *cfg, pyxis_cuda_model **out) {
    if (!ctx || !cfg || !out) return model_fail(PYXIS_EINVAL, "null argument");
    *out = nullptr;
    const pyxis_model_config &c = *cfg;
    if (c.hidden <= 0 || c.n_layers <= 0 || c.n_q_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 || c.ffn <= 0 ||
        c.vocab <= 0 || c.max_seq <= 0 || c.head_dim % 2 || c.head_dim > 1024 || c.n_q_heads % c.n_kv_heads)
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_create: bad config");
    if (c.hidden > 1024 * 8) return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_create: hidden > 8192");
    if (c.head_dim != 64 && c.head_dim != 128)
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_create: the decode attention kernel takes head_dim 64 or 128");
    if (c.n_q_heads / c.n_kv_heads > kAttnMaxG)
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_create: more than 4 query heads per kv head");
    Guard g(ctx->device);
    auto *m = new (std::nothrow) pyxis_cuda_model();
    if (!m) return model_fail(PYXIS_ENOMEM, "host allocation failed");
    m->ctx = ctx;
    m->cfg = c;
    m->q_dim = c.n_q_heads * c.head_dim;
    m->kv_dim = c.n_kv_heads * c.head_dim;
    m->layers.resize(c.n_layers);
    // attention key splits: up to one (kv head, split) CTA per SM, each split of >= 256 keys at the
    // longest context (at short contexts the splits' fixed work -- q/k norm and RoPE in every CTA,
    // the combine through a ticket -- outweighs their keys)
    m->attn_splits = std::max(1, std::min({ctx->num_sms / c.n_kv_heads, (c.max_seq + 255) / 256, 64}));
    const size_t H = c.hidden, half = c.head_dim / 2;
    cudaError_t e = cudaSuccess;
    auto A = [&](auto **p, size_t n) {
        if (e == cudaSuccess) e = dalloc(m, p, n);
    };
    for (auto &L : m->layers) {
        A(&L.in_norm, H);
        A(&L.post_norm, H);
    }
    A(&m->final_norm, H);
    A(&m->emb, (size_t)c.vocab * H);
    A(&m->rope_cos, (size_t)c.max_seq * half);
    A(&m->rope_sin, (size_t)c.max_seq * half);
    A(&m->kcache, (size_t)c.n_layers * c.max_seq * m->kv_dim);
    A(&m->vcache, (size_t)c.n_layers * c.max_seq * m->kv_dim);
    A(&m->x, H);
    A(&m->x2, H);
    A(&m->part, (size_t)c.n_kv_heads * m->attn_splits * (c.n_q_heads / c.n_kv_heads) * (c.head_dim + 2));
    A(&m->tickets, (size_t)c.n_kv_heads);
    A(&m->h, H);
    A(&m->qkv, (size_t)m->q_dim + 2 * m->kv_dim);
    A(&m->q, (size_t)m->q_dim);
    A(&m->attn, (size_t)m->q_dim);
    A(&m->tmp, H);
    A(&m->gu, 2 * (size_t)c.ffn);
    A(&m->act, (size_t)c.ffn);
    A(&m->logits, (size_t)c.vocab);
    A(&m->d_pos, 1);
    A(&m->d_token, 1);
    A(&m->d_step, 1);
    A(&m->d_out, (size_t)c.max_seq + 1);
    if (e != cudaSuccess) {
        pyxis_cuda_model_free(m);
        return model_fail(PYXIS_ENOMEM, cudaGetErrorString(e));
    }
    e = cudaMemset(m->tickets, 0, (size_t)c.n_kv_heads * sizeof(unsigned));
    if (e != cudaSuccess) {
        pyxis_cuda_model_free(m);
        return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    }
    std::vector<float> cs((size_t)c.max_seq * half), sn((size_t)c.max_seq * half);
    pyxis_rope_table(c.rope_theta, c.head_dim, c.max_seq, cs.data(), sn.data());
    e = cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        pyxis_cuda_model_free(m);
        return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    }
    *out = m;
    return PYXIS_OK;
}

extern "C" int pyxis_cuda_model_set_layer(pyxis_cuda_model *m, int layer, const pyxis_cuda_weights *wqkv,
                                          const pyxis_cuda_weights *wo, const pyxis_cuda_weights *wgu,
                                          const pyxis_cuda_weights *wdown, const float *input_norm,
                                          const float *post_norm, const float *q_norm, const float *k_norm) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers) return model_fail(PYXIS_EINVAL, "bad model or layer");
    const pyxis_model_config &c = m->cfg;
    const size_t H = c.hidden, dev = m->ctx->device;
    if (!weights_ok(wqkv, ((size_t)m->q_dim + 2 * m->kv_dim) * H, dev) || !weights_ok(wo, H * m->q_dim, dev) ||
        !weights_ok(wgu, 2 * (size_t)c.ffn * H, dev) || !weights_ok(wdown, H * c.ffn, dev))
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_set_layer: a projection has the wrong length or device");
    if (!input_norm || !post_norm) return model_fail(PYXIS_EINVAL, "null norm weights");
    Guard g(m->ctx->device);
    auto &L = m->layers[layer];
    L.wqkv = wqkv;
    L.wo = wo;
    L.wgu = wgu;
    L.wdown = wdown;
    cudaError_t e = cudaMemcpy(L.in_norm, input_norm, H * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(L.post_norm, post_norm, H * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && q_norm) {
        if (!L.q_norm) e = dalloc(m, &L.q_norm, c.head_dim);
        if (e == cudaSuccess) e = cudaMemcpy(L.q_norm, q_norm, c.head_dim * 4, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && k_norm) {
        if (!L.k_norm) e = dalloc(m, &L.k_norm, c.head_dim);
        if (e == cudaSuccess) e = cudaMemcpy(L.k_norm, k_norm, c.head_dim * 4, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    if (m->exec) {  // weights changed: re-capture on the next generate
        cudaGraphExecDestroy(m->exec);
        m->exec = nullptr;
    }
    return PYXIS_OK;
}

extern "C" int pyxis_cuda_model_set_head(pyxis_cuda_model *m, const uint16_t *embedding_bf16,
                                         const pyxis_cuda_weights *lm_head, const float *final_norm) {
    if (!m || !embedding_bf16 || !final_norm) return model_fail(PYXIS_EINVAL, "null argument");
    const pyxis_model_config &c = m->cfg;
    // NULL lm_head: a vocab-parallel model that holds only its shard (pyxis_comm.h)
    if (lm_head && !weights_ok(lm_head, (size_t)c.vocab * c.hidden, m->ctx->device))
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_set_head: lm_head has the wrong length or device");
    Guard g(m->ctx->device);
    m->lm_head = lm_head;
    cudaError_t e = cudaMemcpy(m->emb, embedding_bf16, (size_t)c.vocab * c.hidden * 2, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(m->final_norm, final_norm, (size_t)c.hidden * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    if (m->exec) {
        cudaGraphExecDestroy(m->exec);
        m->exec = nullptr;
    }
    return PYXIS_OK;
}

extern "C" int pyxis_cuda_model_generate(pyxis_cuda_model *m, const int32_t *prompt, size_t n_prompt, size_t n_new,
                                         int32_t *out_tokens, float *timing_ms) {
    if (!m || !prompt || !out_tokens) return model_fail(PYXIS_EINVAL, "null argument");
    if (n_prompt == 0) return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_generate: empty prompt");
    if (n_new == 0) return PYXIS_OK;
    const pyxis_model_config &c = m->cfg;
    if (n_prompt + n_new - 1 > (size_t)c.max_seq) return model_fail(PYXIS_EINVAL, "prompt + new tokens exceed max_seq");
    for (size_t i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= c.vocab) return model_fail(PYXIS_EINVAL, "token id out of range");
    for (const auto &L : m->layers)
        if (!L.wqkv) return model_fail(PYXIS_EINVAL, "a layer has no weights");
    if (!m->lm_head) return model_fail(PYXIS_EINVAL, "no lm_head");
    Guard g(m->ctx->device);
    cudaStream_t st = m->ctx->stream;
    cudaError_t e = cudaSuccess;
    if (!m->exec) {
        // Every kernel of the step asks for the same (maximum) shared-memory carveout as the
        // GEMV kernels, so the SMs never re-split L1 / shared memory between graph nodes.
        const void *small_kernels[] = {(const void *)embed_kernel, (const void *)add_rmsnorm_kernel,
                                       (const void *)attention_step_kernel<2, 2>, (const void *)attention_step_kernel<4, 2>,
                                       (const void *)silu_mul_kernel, (const void *)advance_kernel};
        for (const void *k : small_kernels) cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        set_argmax_carveout_max();
        // Warm every kernel once outside capture (first-use attribute setting and occupancy
        // queries), then capture the step.
        int zero = 0;
        e = cudaMemcpyAsync(m->d_pos, &zero, 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_step, &zero, 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_token, prompt, 4, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
        int rc = enqueue_step(m, st);
        if (rc) return rc;
        e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
        cudaGraph_t graph = nullptr;
        e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
        rc = enqueue_step(m, st);
        e = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (e == cudaSuccess) e = cudaGraphInstantiate(&m->exec, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    }
    // Reset the cache position and run the prompt, one position per step.
    int zero = 0;
    e = cudaMemcpyAsync(m->d_pos, &zero, 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_step, &zero, 4, cudaMemcpyHostToDevice, st);
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    for (auto &x : ev)
        if (e == cudaSuccess) e = cudaEventCreate(&x);
    if (e == cudaSuccess) e = cudaEventRecord(ev[0], st);
    for (size_t i = 0; i < n_prompt && e == cudaSuccess; ++i) {
        e = cudaMemcpyAsync(m->d_token, prompt + i, 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaGraphLaunch(m->exec, st);
    }
    if (e == cudaSuccess) e = cudaEventRecord(ev[1], st);
    for (size_t i = 1; i < n_new && e == cudaSuccess; ++i) e = cudaGraphLaunch(m->exec, st);
    if (e == cudaSuccess) e = cudaEventRecord(ev[2], st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && timing_ms) {
        e = cudaEventElapsedTime(&timing_ms[0], ev[0], ev[1]);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&timing_ms[1], ev[1], ev[2]);
    }
    if (e == cudaSuccess)
        e = cudaMemcpy(out_tokens, m->d_out + (n_prompt - 1), n_new * sizeof(int32_t), cudaMemcpyDeviceToHost);
    for (auto &x : ev)
        if (x) cudaEventDestroy(x);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    return PYXIS_OK;
}

extern "C" int pyxis_cuda_model_free(pyxis_cuda_model *m) {
    if (!m) return PYXIS_OK;
    Guard g(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    free_batch_state(m->batch);
    for (void *p : m->allocs) cudaFree(p);
    delete m;
    return PYXIS_OK;
}
