// decode_batch.cu -- greedy generation for many independent sequences at once
// (pyxis_cuda_model_generate_batch, include/pyxis_decode.h).
//
// Model::generate (src/model.rs:245-285) with temperature 0, run for n_seq prompts of the same
// length side by side.  Prefill processes whole prompts: the projections of all their positions
// are tensor-core GEMMs (pyxis_cuda_matmul_dev's M >= 16 path), attention is the causal
// tensor-core prefill attention of attn_tc.cu, and the K/V rows go straight into each sequence's
// cache.  Every
// generated token is then one batched step -- the projections are GEMMs over the n_seq rows,
// attention is the fused decode kernel of decode.cu over a (split, kv head, sequence) grid --
// captured once into a CUDA graph and replayed.  The arithmetic between the projections is the
// single-sequence decoder's (decode.cu), row by row.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <tuple>
#include <type_traits>
#include <vector>

#include "../../include/pyxis_decode.h"
#include "argmax.h"
#include "attn_tc.h"
#include "comm.h"
#include "common.cuh"
#include "ctx.h"
#include "heads.cuh"
#include "kernels.h"
#include "model.h"

namespace pyxis {
namespace {

// ------------------------------------------------------------------------------ row kernels --
// x[r] = widen(embedding[tokens[r]]) (src/embedding.rs:18-24); grid (ceil(H / 256), rows).
__global__ void embed_rows_kernel(const uint16_t *__restrict__ emb, const int *__restrict__ tokens, int vocab, int H,
                                  float *__restrict__ x) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.y;
    int t = tokens[r];
    t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
    const uint16_t *row = emb + (size_t)t * H;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < H) x[(size_t)r * H + i] = bf16_bits_to_f32(row[i]);
}

// Output row r from residual row rx = r * row_step + row_off: x[rx] += delta[rx] (optional, in
// place: one CTA owns the row), then h[r] = x[rx] * (factor * w), factor = 1 / sqrt(mean(x^2) + eps)
// (src/transformer.rs:40-42,54-59, src/rmsnorm.rs:11-20).  256 threads, n % 4 == 0, n <= 8192.
constexpr int kRowThreads = 256;
constexpr int kRowQuads = 8;
__global__ void __launch_bounds__(kRowThreads)
    add_rmsnorm_rows_kernel(float *__restrict__ x, const float *__restrict__ delta, const float *__restrict__ w,
                            float *__restrict__ h, int n, float eps, int row_step, int row_off) {
    __shared__ float red[kRowThreads / 32];
    pdl_wait();
    pdl_trigger();
    const size_t rx = (size_t)blockIdx.x * row_step + row_off;
    float4 *xr = reinterpret_cast<float4 *>(x + rx * n);
    const float4 *dr = delta ? reinterpret_cast<const float4 *>(delta + rx * n) : nullptr;
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    const int nq = n / 4;
    float4 v[kRowQuads];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < kRowQuads; ++u) {
        const int k = threadIdx.x + u * kRowThreads;
        if (k < nq) {
            v[u] = xr[k];
            if (dr) {
                const float4 d = dr[k];
                v[u] = make_float4(__fadd_rn(v[u].x, d.x), __fadd_rn(v[u].y, d.y), __fadd_rn(v[u].z, d.z),
                                   __fadd_rn(v[u].w, d.w));
            }
        }
    }
#pragma unroll
    for (int u = 0; u < kRowQuads; ++u) {
        const int k = threadIdx.x + u * kRowThreads;
        if (k < nq) {
            if (dr) xr[k] = v[u];
            ss = __fadd_rn(ss, __fmul_rn(v[u].x, v[u].x));
            ss = __fadd_rn(ss, __fmul_rn(v[u].y, v[u].y));
            ss = __fadd_rn(ss, __fmul_rn(v[u].z, v[u].z));
            ss = __fadd_rn(ss, __fmul_rn(v[u].w, v[u].w));
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < kRowThreads / 32; ++i) tot = __fadd_rn(tot, red[i]);
    const float factor = rms_factor(tot, n, eps);
    float4 *hr = reinterpret_cast<float4 *>(h + (size_t)blockIdx.x * n);
#pragma unroll
    for (int u = 0; u < kRowQuads; ++u) {
        const int k = threadIdx.x + u * kRowThreads;
        if (k < nq) {
            const float4 ww = w4[k];
            hr[k] = make_float4(rms_scale(v[u].x, factor, ww.x), rms_scale(v[u].y, factor, ww.y),
                                rms_scale(v[u].z, factor, ww.z), rms_scale(v[u].w, factor, ww.w));
        }
    }
}

// Prefill row r = (sequence r / P, position pos0 + r % P): per-head QK RMSNorm and RoPE
// (src/attention.rs:81-93), k and v to the sequence's cache row (:100), q as the prefill
// attention's operand: each q head row scaled by its power of two and split into fp16 hi/lo, with
// 2^-e (attn_tc.h).  The largest |k| and |v| of every kv head are folded into tc.kvmax.
// One CTA per row, one warp per head: warps [0, n_q) the q heads, [n_q, n_q + n_kv) the k heads,
// warp n_q + n_kv copies v.
template <int EPL>
__global__ void qk_rope_rows_kernel(const float *__restrict__ qkv, const float *__restrict__ q_norm,
                                    const float *__restrict__ k_norm, const float *__restrict__ rcos,
                                    const float *__restrict__ rsin, int n_q, int n_kv, float eps, int P, int pos0,
                                    float *__restrict__ kcache, float *__restrict__ vcache, long long cache_stride,
                                    AttnTcBuffers tc, int cs) {
    constexpr int HD = 32 * EPL;
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq = r / P, pos = pos0 + r % P;
    const int q_dim = n_q * HD, kv_dim = n_kv * HD;
    const float *row = qkv + (size_t)r * (q_dim + 2 * kv_dim);
    float *kc = kcache + seq * cache_stride + (size_t)pos * kv_dim;
    float *vc = vcache + seq * cache_stride + (size_t)pos * kv_dim;
    if (warp < n_q + n_kv) {
        const bool is_q = warp < n_q;
        const int hh = is_q ? warp : warp - n_q;
        float v[EPL];
        load_head<EPL>(row + (is_q ? 0 : q_dim) + (size_t)hh * HD + lane * EPL, v);
        norm_rope<EPL>(v, is_q ? q_norm : k_norm, rcos, rsin, pos, eps, lane);
        float m = 0.f;
#pragma unroll
        for (int t = 0; t < EPL; ++t) m = fmaxf(m, fabsf(v[t]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (is_q) {
            const int Pp = attn_tc_padded(P);
            const int e = attn_scale_exp(m);
            const float sc = attn_pow2(e);
            const size_t qrow = ((size_t)seq * n_q + hh) * Pp + pos;
            __half *hi = tc.q + qrow * HD + lane * EPL;
            __half *lo = hi + (size_t)cs * n_q * Pp * HD;
#pragma unroll
            for (int t = 0; t < EPL; t += 2) {
                const float x0 = v[t] * sc, x1 = v[t + 1] * sc;
                const __half2 h = __floats2half2_rn(x0, x1);
                const float2 f = __half22float2(h);
                *reinterpret_cast<__half2 *>(hi + t) = h;
                *reinterpret_cast<__half2 *>(lo + t) = __floats2half2_rn(x0 - f.x, x1 - f.y);
            }
            if (lane == 0) tc.qinv[qrow] = attn_pow2(-e);
        } else {
            float *dst = kc + (size_t)hh * HD;
#pragma unroll
            for (int t = 0; t < EPL; ++t) dst[lane * EPL + t] = v[t];
            if (lane == 0) atomicMax(&tc.kvmax[((size_t)seq * n_kv + hh) * 2], __float_as_uint(m));
        }
    } else if (warp == n_q + n_kv) {
        for (int h = 0; h < n_kv; ++h) {
            float m = 0.f;
#pragma unroll
            for (int t = 0; t < EPL; ++t) {
                const int i = h * HD + t * 32 + lane;
                const float x = row[q_dim + kv_dim + i];
                vc[i] = x;
                m = fmaxf(m, fabsf(x));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) atomicMax(&tc.kvmax[((size_t)seq * n_kv + h) * 2 + 1], __float_as_uint(m));
        }
    }
}

// act[r] = SiLU(gu[r][0:ffn]) * gu[r][ffn:2 ffn] (src/ffn.rs:39-41,52-54); grid (ceil(ffn/1024), rows):
// four consecutive elements per thread (16-byte loads and store) when ffn % 4 == 0.
__global__ void silu_rows_kernel(const float *__restrict__ gu, int ffn, float *__restrict__ act) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.y, i = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= ffn) return;
    const float *row = gu + (size_t)r * 2 * ffn;
    float *out = act + (size_t)r * ffn;
    if ((ffn & 3) == 0) {
        const float4 g = __ldg(reinterpret_cast<const float4 *>(row + i));
        const float4 u = __ldg(reinterpret_cast<const float4 *>(row + ffn + i));
        *reinterpret_cast<float4 *>(out + i) = make_float4(__fmul_rn(silu_f(g.x), u.x), __fmul_rn(silu_f(g.y), u.y),
                                                           __fmul_rn(silu_f(g.z), u.z), __fmul_rn(silu_f(g.w), u.w));
    } else {
        for (int j = i; j < i + 4 && j < ffn; ++j) out[j] = __fmul_rn(silu_f(row[j]), row[ffn + j]);
    }
}

// out[b][step] = tokens[b] for every sequence, then step += 1 and pos += 1 (one CTA).
__global__ void advance_rows_kernel(const int *__restrict__ tokens, int n_seq, int n_new, int *__restrict__ out,
                                    int *pos, int *step) {
    pdl_wait();
    pdl_trigger();
    const int s = *step;
    for (int b = threadIdx.x; b < n_seq; b += blockDim.x) out[(size_t)b * n_new + s] = tokens[b];
    __syncthreads();
    if (threadIdx.x == 0) {
        *step = s + 1;
        *pos = *pos + 1;
    }
}

}  // namespace

// ------------------------------------------------------------------------------ host side --
struct BatchState {
    int n_seq = 0, n_prompt = 0, n_new = 0;  // capacity of the buffers below
    int chunk = 0;                           // sequences per prefill pass
    size_t cache_stride = 0;                 // floats per sequence: n_layers * max_seq * kv_dim
    int splits = 1;                          // decode attention key splits
    float *kc = nullptr, *vc = nullptr;      // [n_seq][n_layers][max_seq][kv_dim]
    // prefill rows (chunk * n_prompt)
    float *px = nullptr, *ph = nullptr, *pqkv = nullptr, *pattn = nullptr, *ptmp = nullptr,
          *pgu = nullptr, *pact = nullptr;
    // decode rows (n_seq)
    float *dx = nullptr, *dh = nullptr, *dqkv = nullptr, *dattn = nullptr, *dtmp = nullptr, *dgu = nullptr,
          *dact = nullptr, *dlogits = nullptr;
    // vocab-parallel head: every rank's final hidden rows [nranks][n_seq][hidden]
    float *xall = nullptr;
    int vp_ranks = 0;
    float *part = nullptr;
    unsigned *tickets = nullptr;
    // tensor-core prefill attention operands of one chunk (attn_tc.h); kvmax per layer
    AttnTcBuffers tc{};
    int *d_prompt = nullptr, *d_tokens = nullptr, *d_out = nullptr, *d_pos = nullptr, *d_step = nullptr;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    std::vector<void *> allocs;
};

namespace {

// Keys per decode-attention CTA of a batched step: fewer, longer splits amortise each CTA's fixed
// work (q/k norm + RoPE, the fence and ticket of the split combine) now that its warps stream
// keys through cp.async rings.
constexpr int kKeysPerSplit = 768;

int batch_fail(int code, const char *msg) { return record_error(code, msg); }

int kv_dim_of(const pyxis_model_config &c) { return c.n_kv_heads * c.head_dim; }
int q_dim_of(const pyxis_model_config &c) { return c.n_q_heads * c.head_dim; }

// Buffers for n_seq prompts of n_prompt ids and n_new tokens (grown, never shrunk).
int ensure_state(pyxis_cuda_model *m, int n_seq, int n_prompt, int n_new) {
    BatchState *b = m->batch;
    if (b && b->n_seq >= n_seq && b->n_prompt >= n_prompt && b->n_new >= n_new) return PYXIS_OK;
    const pyxis_model_config &c = m->cfg;
    if (b) {
        n_seq = std::max(n_seq, b->n_seq);
        n_prompt = std::max(n_prompt, b->n_prompt);
        n_new = std::max(n_new, b->n_new);
        free_batch_state(b);
        m->batch = nullptr;
    }
    b = new (std::nothrow) BatchState();
    if (!b) return batch_fail(PYXIS_ENOMEM, "host allocation failed");
    const size_t H = c.hidden, qd = q_dim_of(c), kvd = kv_dim_of(c), ffn = c.ffn;
    const size_t qkv_rows = qd + 2 * kvd;
    b->n_seq = n_seq;
    b->n_prompt = n_prompt;
    b->n_new = n_new;
    b->chunk = std::max(1, std::min(n_seq, 16384 / n_prompt));
    b->cache_stride = (size_t)c.n_layers * c.max_seq * kvd;
    const int G = c.n_q_heads / c.n_kv_heads;
    // attention key splits: at least two CTAs per SM, and at most kKeysPerSplit keys per CTA
    const int want = std::max((2 * m->ctx->num_sms + c.n_kv_heads * n_seq - 1) / (c.n_kv_heads * n_seq),
                              (c.max_seq + kKeysPerSplit - 1) / kKeysPerSplit);
    b->splits = std::max(1, std::min({want, (c.max_seq + 15) / 16, 64}));
    const size_t rows = (size_t)b->chunk * n_prompt;
    const size_t kmax = std::max({H, qd, ffn});
    // split_x space for the largest GEMM, plus split-K partials for the n_seq-row step GEMMs
    size_t ws = gemm_tc_workspace_bytes(std::max(rows, (size_t)n_seq), kmax);
    for (const auto &L : m->layers)
        for (auto [w, N, K] : {std::tuple{L.wqkv, qkv_rows, H}, std::tuple{L.wo, H, qd}, std::tuple{L.wgu, 2 * ffn, H},
                               std::tuple{L.wdown, H, ffn}})
            if (w) {
                ws = std::max(ws, gemm_tc_workspace_bytes_splitk(n_seq, N, K, w->block_size == K, w->block_size,
                                                                 m->ctx->num_sms));
                // the prefill's products over all the chunk's rows (group-scaled weights converted
                // once per product)
                ws = std::max(ws, gemm_tc_workspace_bytes_splitk(rows, N, K, w->block_size == K, w->block_size,
                                                                 m->ctx->num_sms));
            }
    pyxis_cuda_comm *vp = m->vp_comm;
    const size_t head_rows = vp ? (size_t)vp->nranks * n_seq : (size_t)n_seq;
    // the decode step's products of n_seq rows on the weight-streaming matmul: x copies plus room
    // for split-K partial sums
    constexpr size_t kStepPartialCap = 12u << 20;
    for (const auto &L : m->layers)
        for (auto [w, N, K] : {std::tuple{L.wqkv, qkv_rows, H}, std::tuple{L.wo, H, qd}, std::tuple{L.wgu, 2 * ffn, H},
                               std::tuple{L.wdown, H, ffn}})
            if (w) ws = std::max(ws, gemm_ws_workspace_bytes(n_seq, N, K, m->ctx->num_sms, kStepPartialCap));
    ws = std::max(ws, gemm_ws_workspace_bytes(head_rows, vp ? m->vp_rows : (size_t)c.vocab, H, m->ctx->num_sms,
                                              kStepPartialCap));
    if (vp) {
        ws = std::max(ws, gemm_tc_workspace_bytes(head_rows, H));
        ws = std::max(ws, gemm_tc_workspace_bytes_splitk(head_rows, m->vp_rows, H, m->vp_shard->block_size == H,
                                                         m->vp_shard->block_size, m->ctx->num_sms));
    } else if (m->lm_head) {
        ws = std::max(ws, gemm_tc_workspace_bytes_splitk(n_seq, c.vocab, H, m->lm_head->block_size == H,
                                                         m->lm_head->block_size, m->ctx->num_sms));
    }
    b->ws_bytes = ws;
    cudaError_t e = cudaSuccess;
    auto A = [&](auto **p, size_t count) {
        if (e != cudaSuccess) return;
        void *v = nullptr;
        e = cudaMalloc(&v, count * sizeof(**p) + 256);
        if (e == cudaSuccess) {
            b->allocs.push_back(v);
            *p = reinterpret_cast<std::remove_reference_t<decltype(*p)>>(v);
        }
    };
    A(&b->kc, (size_t)n_seq * b->cache_stride);
    A(&b->vc, (size_t)n_seq * b->cache_stride);
    A(&b->px, rows * H);
    A(&b->ph, rows * H);
    A(&b->pqkv, rows * qkv_rows);
    A(&b->pattn, rows * qd);
    A(&b->ptmp, rows * H);
    A(&b->pgu, rows * 2 * ffn);
    A(&b->pact, rows * ffn);
    A(&b->dx, (size_t)n_seq * H);
    A(&b->dh, (size_t)n_seq * H);
    A(&b->dqkv, (size_t)n_seq * qkv_rows);
    A(&b->dattn, (size_t)n_seq * qd);
    A(&b->dtmp, (size_t)n_seq * H);
    A(&b->dgu, (size_t)n_seq * 2 * ffn);
    A(&b->dact, (size_t)n_seq * ffn);
    if (vp) {
        A(&b->xall, head_rows * H);
        b->vp_ranks = vp->nranks;
    } else {
        A(&b->dlogits, (size_t)n_seq * c.vocab);
    }
    {
        const size_t Pp = attn_tc_padded(n_prompt), hd = c.head_dim, cs = b->chunk;
        A(&b->tc.q, 2 * cs * c.n_q_heads * Pp * hd);
        A(&b->tc.qinv, cs * c.n_q_heads * Pp);
        A(&b->tc.k, 2 * cs * c.n_kv_heads * Pp * hd);
        A(&b->tc.vt, 2 * cs * c.n_kv_heads * hd * Pp);
        A(&b->tc.kvmax, (size_t)c.n_layers * cs * c.n_kv_heads * 2);
        if (e == cudaSuccess) e = cudaMemset(b->tc.q, 0, 2 * cs * c.n_q_heads * Pp * hd * sizeof(__half));
        if (e == cudaSuccess) e = cudaMemset(b->tc.qinv, 0, cs * c.n_q_heads * Pp * sizeof(float));
    }
    A(&b->part, (size_t)n_seq * c.n_kv_heads * b->splits * G * (c.head_dim + 2));
    A(&b->tickets, (size_t)n_seq * c.n_kv_heads);
    A(&b->d_prompt, (size_t)n_seq * n_prompt);
    A(&b->d_tokens, (size_t)n_seq);
    A(&b->d_out, (size_t)n_seq * n_new);
    A(&b->d_pos, 1);
    A(&b->d_step, 1);
    if (e == cudaSuccess) {
        void *w = nullptr;
        e = cudaMalloc(&w, b->ws_bytes);
        if (e == cudaSuccess) {
            b->allocs.push_back(w);
            b->ws = w;
        }
    }
    if (e == cudaSuccess) e = cudaMemset(b->tickets, 0, (size_t)n_seq * c.n_kv_heads * sizeof(unsigned));
    if (e != cudaSuccess) {
        free_batch_state(b);
        cudaGetLastError();
        return batch_fail(PYXIS_ENOMEM, cudaGetErrorString(e));
    }
    if (vp) {
        const int rc = head_reserve(vp, head_rows, m->vp_rows);
        if (rc) {
            free_batch_state(b);
            return rc;
        }
    }
    m->batch = b;
    return PYXIS_OK;
}

#define PX_TRY(expr)                                                              \
    do {                                                                          \
        cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) return batch_fail(PYXIS_ECUDA, cudaGetErrorString(e_)); \
    } while (0)

// Next tokens of the n_seq rows of b->dh: the lm_head and argmax on this GPU, or (vocab-parallel)
// every rank's rows all-gathered, this rank's vocab shard, the keys' all-gather and the pick of
// this rank's rows.
int enqueue_head(pyxis_cuda_model *m, int n_seq, cudaStream_t st) {
    const pyxis_model_config &c = m->cfg;
    BatchState *b = m->batch;
    const int H = c.hidden;
    pyxis_cuda_ctx *ctx = m->ctx;
    if (pyxis_cuda_comm *vp = m->vp_comm) {
        int rc = comm_allgather(vp, b->dh, b->xall, (size_t)n_seq * H, false, st);
        if (rc) return rc;
        return head_greedy_enqueue(vp, m->vp_shard, m->vp_lo, m->vp_rows, H, b->xall, (size_t)vp->nranks * n_seq, H,
                                   vp->rank * n_seq, n_seq, b->d_tokens, b->ws, b->ws_bytes, st);
    }
    int rc = run_matmul(ctx, m->lm_head, b->dh, n_seq, H, c.vocab, H, b->dlogits, c.vocab, b->ws, b->ws_bytes, st);
    if (rc) return rc;
    PX_TRY(launch_argmax_scratch(b->dlogits, n_seq, c.vocab, c.vocab, 0, b->d_tokens, nullptr, ctx->amax, ctx->num_sms,
                                 st));
    return PYXIS_OK;
}

// All prompt positions of every sequence: the layers over `chunk` sequences at a time, then the
// lm_head over each sequence's last position and the argmax -> the first generated tokens.
int enqueue_prefill(pyxis_cuda_model *m, int n_seq, int P, cudaStream_t st) {
    const pyxis_model_config &c = m->cfg;
    BatchState *b = m->batch;
    const int H = c.hidden, qd = q_dim_of(c), kvd = kv_dim_of(c), ffn = c.ffn;
    const size_t qkv_rows = (size_t)qd + 2 * kvd;
    const size_t layer_stride = (size_t)c.max_seq * kvd;
    pyxis_cuda_ctx *ctx = m->ctx;
    PdlScope pdl;
    for (int s0 = 0; s0 < n_seq; s0 += b->chunk) {
        const int cs = std::min(b->chunk, n_seq - s0);
        const int M = cs * P;
        PX_TRY(cudaMemsetAsync(b->tc.kvmax, 0, (size_t)c.n_layers * b->chunk * c.n_kv_heads * 2 * sizeof(unsigned),
                                   st));
        PX_TRY(launch_kernel(embed_rows_kernel, dim3((H + 255) / 256, M), dim3(256), 0, st, (const uint16_t *)m->emb,
                             (const int *)(b->d_prompt + (size_t)s0 * P), c.vocab, H, b->px));
        for (int l = 0; l < c.n_layers; ++l) {
            const auto &L = m->layers[l];
            float *kc = b->kc + (size_t)s0 * b->cache_stride + l * layer_stride;
            float *vc = b->vc + (size_t)s0 * b->cache_stride + l * layer_stride;
            PX_TRY(launch_kernel(add_rmsnorm_rows_kernel, dim3(M), dim3(kRowThreads), 0, st, b->px,
                                 (const float *)(l ? b->ptmp : nullptr), (const float *)L.in_norm, b->ph, H, c.rms_eps,
                                 1, 0));
            int rc = run_matmul(ctx, L.wqkv, b->ph, M, H, qkv_rows, H, b->pqkv, qkv_rows, b->ws, b->ws_bytes, st);
            if (rc) return rc;
            AttnTcBuffers t = b->tc;
            t.kvmax += (size_t)l * b->chunk * c.n_kv_heads * 2;
            auto rope = c.head_dim == 128 ? qk_rope_rows_kernel<4> : qk_rope_rows_kernel<2>;
            PX_TRY(launch_kernel(rope, dim3(M), dim3((c.n_q_heads + c.n_kv_heads + 1) * 32), 0, st,
                                 (const float *)b->pqkv, (const float *)L.q_norm, (const float *)L.k_norm,
                                 (const float *)m->rope_cos, (const float *)m->rope_sin, c.n_q_heads, c.n_kv_heads,
                                 c.rms_eps, P, 0, kc, vc, (long long)b->cache_stride, t, cs));
            PX_TRY(launch_attn_prep_kv(kc, vc, (long long)b->cache_stride, cs, P, c.n_kv_heads, c.head_dim, t, st));
            PX_TRY(launch_attention_prefill_tc(cs, P, c.n_q_heads, c.n_kv_heads, c.head_dim, t, b->pattn, ctx->d_err,
                                               st));
            rc = run_matmul(ctx, L.wo, b->pattn, M, qd, H, qd, b->ptmp, H, b->ws, b->ws_bytes, st);
            if (rc) return rc;
            PX_TRY(launch_kernel(add_rmsnorm_rows_kernel, dim3(M), dim3(kRowThreads), 0, st, b->px,
                                 (const float *)b->ptmp, (const float *)L.post_norm, b->ph, H, c.rms_eps, 1, 0));
            rc = run_matmul(ctx, L.wgu, b->ph, M, H, 2 * (size_t)ffn, H, b->pgu, 2 * (size_t)ffn, b->ws, b->ws_bytes, st);
            if (rc) return rc;
            PX_TRY(launch_kernel(silu_rows_kernel, dim3((ffn + 1023) / 1024, M), dim3(256), 0, st, (const float *)b->pgu,
                                 ffn, b->pact));
            rc = run_matmul(ctx, L.wdown, b->pact, M, ffn, H, ffn, b->ptmp, H, b->ws, b->ws_bytes, st);
            if (rc) return rc;
        }
        // final norm of each sequence's last position only
        PX_TRY(launch_kernel(add_rmsnorm_rows_kernel, dim3(cs), dim3(kRowThreads), 0, st, b->px,
                             (const float *)b->ptmp, (const float *)m->final_norm, b->dh + (size_t)s0 * H, H,
                             c.rms_eps, P, P - 1));
    }
    int rc = enqueue_head(m, n_seq, st);
    if (rc) return rc;
    PX_TRY(launch_kernel(advance_rows_kernel, dim3(1), dim3(256), 0, st, (const int *)b->d_tokens, n_seq, b->n_new,
                         b->d_out, b->d_pos, b->d_step));
    return PYXIS_OK;
}

// One generated token for every sequence (what the graph holds): the step of decode.cu over
// n_seq rows, all sequences at position *d_pos.
int enqueue_step(pyxis_cuda_model *m, int n_seq, cudaStream_t st) {
    const pyxis_model_config &c = m->cfg;
    BatchState *b = m->batch;
    const int H = c.hidden, qd = q_dim_of(c), kvd = kv_dim_of(c), ffn = c.ffn;
    const size_t qkv_rows = (size_t)qd + 2 * kvd;
    const size_t layer_stride = (size_t)c.max_seq * kvd;
    pyxis_cuda_ctx *ctx = m->ctx;
    PdlScope pdl;
    PX_TRY(launch_kernel(embed_rows_kernel, dim3((H + 255) / 256, n_seq), dim3(256), 0, st, (const uint16_t *)m->emb,
                         (const int *)b->d_tokens, c.vocab, H, b->dx));
    for (int l = 0; l < c.n_layers; ++l) {
        const auto &L = m->layers[l];
        PX_TRY(launch_kernel(add_rmsnorm_rows_kernel, dim3(n_seq), dim3(kRowThreads), 0, st, b->dx,
                             (const float *)(l ? b->dtmp : nullptr), (const float *)L.in_norm, b->dh, H, c.rms_eps, 1,
                             0));
        int rc = run_matmul(ctx, L.wqkv, b->dh, n_seq, H, qkv_rows, H, b->dqkv, qkv_rows, b->ws, b->ws_bytes, st);
        if (rc) return rc;
        PX_TRY(launch_attention_step(c, b->splits, n_seq, b->dqkv, qkv_rows, L.q_norm, L.k_norm, m->rope_cos,
                                     m->rope_sin, b->d_pos, b->kc + l * layer_stride, b->vc + l * layer_stride,
                                     b->cache_stride, b->part, b->tickets, b->dattn, qd, st));
        rc = run_matmul(ctx, L.wo, b->dattn, n_seq, qd, H, qd, b->dtmp, H, b->ws, b->ws_bytes, st);
        if (rc) return rc;
        PX_TRY(launch_kernel(add_rmsnorm_rows_kernel, dim3(n_seq), dim3(kRowThreads), 0, st, b->dx,
                             (const float *)b->dtmp, (const float *)L.post_norm, b->dh, H, c.rms_eps, 1, 0));
        rc = run_matmul(ctx, L.wgu, b->dh, n_seq, H, 2 * (size_t)ffn, H, b->dgu, 2 * (size_t)ffn, b->ws, b->ws_bytes, st);
        if (rc) return rc;
        PX_TRY(launch_kernel(silu_rows_kernel, dim3((ffn + 1023) / 1024, n_seq), dim3(256), 0, st, (const float *)b->dgu,
                             ffn, b->dact));
        rc = run_matmul(ctx, L.wdown, b->dact, n_seq, ffn, H, ffn, b->dtmp, H, b->ws, b->ws_bytes, st);
        if (rc) return rc;
    }
    PX_TRY(launch_kernel(add_rmsnorm_rows_kernel, dim3(n_seq), dim3(kRowThreads), 0, st, b->dx, (const float *)b->dtmp,
                         (const float *)m->final_norm, b->dh, H, c.rms_eps, 1, 0));
    int rc = enqueue_head(m, n_seq, st);
    if (rc) return rc;
    PX_TRY(launch_kernel(advance_rows_kernel, dim3(1), dim3(256), 0, st, (const int *)b->d_tokens, n_seq, b->n_new,
                         b->d_out, b->d_pos, b->d_step));
    return PYXIS_OK;
}

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DevGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

void free_batch_state(BatchState *b) {
    if (!b) return;
    for (void *p : b->allocs) cudaFree(p);
    delete b;
}

}  // namespace pyxis

using namespace pyxis;

namespace {

// The host-side checks of pyxis_cuda_model_generate_batch (PYXIS_OK or a recorded error).
int check_batch_args(const pyxis_cuda_model *m, const int32_t *prompts, size_t n_seq, size_t n_prompt, size_t n_new) {
    const pyxis_model_config &c = m->cfg;
    if (n_prompt == 0) return batch_fail(PYXIS_EINVAL, "pyxis_cuda_model_generate_batch: empty prompts");
    if (n_prompt + n_new - 1 > (size_t)c.max_seq)
        return batch_fail(PYXIS_EINVAL, "pyxis_cuda_model_generate_batch: prompt + new tokens exceed max_seq");
    if (n_seq > (size_t)kArgmaxMaxRows || n_prompt > 16384)
        return batch_fail(PYXIS_EINVAL, "pyxis_cuda_model_generate_batch: more than 1024 sequences or 16384 prompt ids");
    if (c.hidden % 4 || c.hidden > kRowThreads * kRowQuads * 4 || c.ffn % 4 || c.n_q_heads + c.n_kv_heads + 1 > 32)
        return batch_fail(PYXIS_EINVAL, "pyxis_cuda_model_generate_batch: unsupported model shape");
    for (size_t i = 0; i < n_seq * n_prompt; ++i)
        if (prompts[i] < 0 || prompts[i] >= c.vocab) return batch_fail(PYXIS_EINVAL, "token id out of range");
    for (const auto &L : m->layers)
        if (!L.wqkv) return batch_fail(PYXIS_EINVAL, "a layer has no weights");
    if (!m->lm_head && !m->vp_comm) return batch_fail(PYXIS_EINVAL, "no lm_head");
    if (m->vp_comm && (size_t)m->vp_comm->nranks * n_seq > (size_t)kArgmaxMaxRows)
        return batch_fail(PYXIS_EINVAL, "vocab-parallel generate_batch: more than 1024 sequences over all ranks");
    return PYXIS_OK;
}

// Vocab-parallel mode: the ranks exchange (n_seq, n_prompt, n_new, local verdict) before any other
// collective, so that all of them go on, or all of them return PYXIS_EINVAL, together.
int agree_batch_args(pyxis_cuda_model *m, size_t n_seq, size_t n_prompt, size_t n_new, int local_rc) {
    pyxis_cuda_comm *vp = m->vp_comm;
    const int W = vp->nranks;
    uint64_t *d = nullptr;
    std::vector<uint64_t> all((size_t)W * 4);
    const uint64_t mine[4] = {n_seq, n_prompt, n_new, (uint64_t)local_rc};
    cudaError_t ce = cudaMalloc(&d, (size_t)(W + 1) * 4 * sizeof(uint64_t));
    if (ce != cudaSuccess) return batch_fail(PYXIS_ECUDA, cudaGetErrorString(ce));
    ce = cudaMemcpyAsync(d, mine, sizeof mine, cudaMemcpyHostToDevice, m->ctx->stream);
    int rc = ce == cudaSuccess ? comm_allgather(vp, d, d + 4, 4, true, m->ctx->stream) : PYXIS_ECUDA;
    if (rc == PYXIS_OK) {
        ce = cudaMemcpyAsync(all.data(), d + 4, all.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost, m->ctx->stream);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(m->ctx->stream);
        if (ce != cudaSuccess) rc = PYXIS_ECUDA;
    }
    cudaFree(d);
    if (rc == PYXIS_ECUDA) return batch_fail(PYXIS_ECUDA, cudaGetErrorString(ce));
    if (rc) return rc;
    if (local_rc) return local_rc;  // this rank's own message stays the recorded one
    for (int r = 0; r < W; ++r) {
        const uint64_t *a = &all[(size_t)r * 4];
        if (a[3] != 0)
            return batch_fail(PYXIS_EINVAL, "vocab-parallel generate_batch: another rank's arguments failed its checks");
        if (a[0] != n_seq || a[1] != n_prompt || a[2] != n_new)
            return batch_fail(PYXIS_EINVAL,
                              "vocab-parallel generate_batch: the ranks passed different n_seq, n_prompt or n_new");
    }
    return PYXIS_OK;
}

}  // namespace

extern "C" int pyxis_cuda_model_generate_batch(pyxis_cuda_model *m, const int32_t *prompts, size_t n_seq,
                                               size_t n_prompt, size_t n_new, int32_t *out_tokens, float *timing_ms) {
    if (!m || !prompts || !out_tokens) return batch_fail(PYXIS_EINVAL, "null argument");
    if (n_seq == 0 || n_new == 0) return PYXIS_OK;
    int rc = check_batch_args(m, prompts, n_seq, n_prompt, n_new);
    DevGuard g(m->ctx->device);
    if (m->vp_comm) rc = agree_batch_args(m, n_seq, n_prompt, n_new, rc);
    if (rc) return rc;
    rc = ensure_state(m, (int)n_seq, (int)n_prompt, (int)n_new);
    if (rc) return rc;
    BatchState *b = m->batch;
    cudaStream_t st = m->ctx->stream;
    // prompts (row stride n_prompt capacity == n_prompt here: the prefill reads rows of n_prompt)
    PX_TRY(cudaMemcpyAsync(b->d_prompt, prompts, n_seq * n_prompt * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    const int zero = 0, last = (int)n_prompt - 1;
    PX_TRY(cudaMemcpyAsync(b->d_step, &zero, sizeof(int), cudaMemcpyHostToDevice, st));
    PX_TRY(cudaMemcpyAsync(b->d_pos, &last, sizeof(int), cudaMemcpyHostToDevice, st));
    cudaEvent_t ev[3];
    for (auto &e : ev) PX_TRY(cudaEventCreate(&e));
    struct EvFree {
        cudaEvent_t *e;
        ~EvFree() {
            for (int i = 0; i < 3; ++i) cudaEventDestroy(e[i]);
        }
    } ev_free{ev};
    PX_TRY(cudaEventRecord(ev[0], st));
    rc = enqueue_prefill(m, (int)n_seq, (int)n_prompt, st);
    if (rc) return rc;
    PX_TRY(cudaEventRecord(ev[1], st));
    if (n_new > 1) {
        // the step as a CUDA graph (pointers and shapes are fixed for this call), replayed per token
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        PX_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
        rc = enqueue_step(m, (int)n_seq, st);
        cudaError_t ce = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        PX_TRY(ce);
        ce = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        PX_TRY(ce);
        for (size_t t = 1; t < n_new && ce == cudaSuccess; ++t) ce = cudaGraphLaunch(exec, st);
        cudaGraphExecDestroy(exec);
        PX_TRY(ce);
    }
    PX_TRY(cudaEventRecord(ev[2], st));
    PX_TRY(cudaMemcpy2DAsync(out_tokens, n_new * sizeof(int32_t), b->d_out, (size_t)b->n_new * sizeof(int32_t),
                             n_new * sizeof(int32_t), n_seq, cudaMemcpyDeviceToHost, st));
    PX_TRY(cudaStreamSynchronize(st));
    rc = pyxis_cuda_check_device_error(m->ctx);
    if (rc) return rc;
    if (timing_ms) {
        PX_TRY(cudaEventElapsedTime(&timing_ms[0], ev[0], ev[1]));
        PX_TRY(cudaEventElapsedTime(&timing_ms[1], ev[1], ev[2]));
    }
    return PYXIS_OK;
}

extern "C" int pyxis_cuda_model_prefill_hidden(pyxis_cuda_model *m, const int32_t *prompts, size_t n_seq,
                                               size_t n_prompt, float *hidden_out) {
    if (!m || !prompts || !hidden_out) return batch_fail(PYXIS_EINVAL, "null argument");
    if (n_seq == 0) return PYXIS_OK;
    if (m->vp_comm) return batch_fail(PYXIS_EINVAL, "prefill_hidden: not with a vocab-parallel head");
    int rc = check_batch_args(m, prompts, n_seq, n_prompt, 1);
    if (rc) return rc;
    DevGuard g(m->ctx->device);
    rc = ensure_state(m, (int)n_seq, (int)n_prompt, 1);
    if (rc) return rc;
    BatchState *b = m->batch;
    cudaStream_t st = m->ctx->stream;
    PX_TRY(cudaMemcpyAsync(b->d_prompt, prompts, n_seq * n_prompt * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    const int zero = 0, last = (int)n_prompt - 1;
    PX_TRY(cudaMemcpyAsync(b->d_step, &zero, sizeof(int), cudaMemcpyHostToDevice, st));
    PX_TRY(cudaMemcpyAsync(b->d_pos, &last, sizeof(int), cudaMemcpyHostToDevice, st));
    rc = enqueue_prefill(m, (int)n_seq, (int)n_prompt, st);
    if (rc) return rc;
    PX_TRY(cudaMemcpyAsync(hidden_out, b->dh, n_seq * (size_t)m->cfg.hidden * sizeof(float), cudaMemcpyDeviceToHost,
                           st));
    PX_TRY(cudaStreamSynchronize(st));
    return pyxis_cuda_check_device_error(m->ctx);
}

extern "C" int pyxis_cuda_model_set_vocab_parallel(pyxis_cuda_model *m, pyxis_cuda_comm *comm,
                                                   const pyxis_cuda_weights *lm_head_shard, size_t vocab_lo,
                                                   size_t shard_rows) {
    if (!m) return batch_fail(PYXIS_EINVAL, "null model");
    const pyxis_model_config &c = m->cfg;
    if (comm) {
        if (comm->ctx->device != m->ctx->device)
            return batch_fail(PYXIS_EINVAL, "set_vocab_parallel: communicator and model on different devices");
        if (!lm_head_shard || lm_head_shard->device != m->ctx->device ||
            lm_head_shard->num_elements != shard_rows * (size_t)c.hidden)
            return batch_fail(PYXIS_EINVAL, "set_vocab_parallel: shard length != shard_rows * hidden, or wrong device");
        if (lm_head_shard->qtype != PYXIS_QTYPE_INT8 && lm_head_shard->qtype != PYXIS_QTYPE_INT4)
            return batch_fail(PYXIS_EINVAL, "set_vocab_parallel: the shard must be int8 or int4");
        if (shard_rows == 0 || vocab_lo + shard_rows > (size_t)c.vocab)
            return batch_fail(PYXIS_EINVAL, "set_vocab_parallel: the shard's rows are not inside [0, vocab)");
    }
    DevGuard g(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    free_batch_state(m->batch);  // the head buffers depend on the mode
    m->batch = nullptr;
    m->vp_comm = comm;
    m->vp_shard = comm ? lm_head_shard : nullptr;
    m->vp_lo = comm ? vocab_lo : 0;
    m->vp_rows = comm ? shard_rows : 0;
    return PYXIS_OK;
}
