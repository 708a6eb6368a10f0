// decode.cu -- device-resident greedy decode (include/pyxis_decode.h).
//
// One step = one token at position pos through all layers, the lm_head and the argmax, entirely on
// the context's stream; the step reads the position, the input token and the output slot from
// device memory, so it is captured once into a CUDA graph and replayed for every token.  The
// kernels between the projections mirror the reference's f32 expressions (src/rmsnorm.rs:11-20,
// src/attention.rs:107-179, src/ffn.rs:39-54) with explicit round-to-nearest multiplies and adds
// where the reference's operation order is cheap to keep (no FMA contraction); sums of many
// terms are reduced in parallel.
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/pyxis_decode.h"
#include "argmax.h"
#include "common.cuh"
#include "ctx.h"
#include "kernels.h"

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

PYXIS_DEVINL float block_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = fmaxf(t, red[i]);
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
    const float factor = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < n) h[i] = __fmul_rn(v[j], __fmul_rn(factor, wv[j]));
    }
}

// Per head: QK RMSNorm (src/attention.rs:81-90), RoPE at `pos` from the host-made table
// (:92-93, :144-162), then q -> qout, k and v -> the KV cache row `pos` (cache.append, :100).
// Grid: n_q + n_kv CTAs (one per q or k head) + 1 CTA copying v; head_dim threads.
__global__ void qk_rope_append_kernel(const float *__restrict__ qkv, const float *__restrict__ q_norm,
                                      const float *__restrict__ k_norm, const float *__restrict__ rcos,
                                      const float *__restrict__ rsin, const int *__restrict__ d_pos, int n_q, int n_kv,
                                      int hd, float eps, float *__restrict__ qout, float *__restrict__ kcache,
                                      float *__restrict__ vcache) {
    extern __shared__ float sh[];  // [hd] head values, [32] reduction
    float *hv = sh, *red = sh + hd;
    pdl_wait();
    pdl_trigger();
    const int pos = *d_pos;
    const int kv_dim = n_kv * hd, q_dim = n_q * hd;
    const int b = blockIdx.x, d = threadIdx.x;
    if (b == n_q + n_kv) {  // v row
        for (int i = d; i < kv_dim; i += blockDim.x) vcache[(size_t)pos * kv_dim + i] = qkv[q_dim + kv_dim + i];
        return;
    }
    const bool is_q = b < n_q;
    const float *src = is_q ? qkv + (size_t)b * hd : qkv + q_dim + (size_t)(b - n_q) * hd;
    const float *nw = is_q ? q_norm : k_norm;
    float v = src[d];
    if (nw) {
        float ss = block_sum(__fmul_rn(v, v), red);
        const float factor = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)hd), eps)));
        v = __fmul_rn(v, __fmul_rn(factor, nw[d]));
    }
    hv[d] = v;
    __syncthreads();
    const int half = hd / 2;
    const int i = d < half ? d : d - half;
    const float c = rcos[(size_t)pos * half + i], s = rsin[(size_t)pos * half + i];
    const float x0 = hv[i], x1 = hv[i + half];
    const float r = d < half ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)) : __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    if (is_q) qout[(size_t)b * hd + d] = r;
    else kcache[(size_t)pos * kv_dim + (size_t)(b - n_q) * hd + d] = r;
}

// Causal GQA attention for the newest position (src/attention.rs:107-135): one CTA per q head;
// scores = (q . k_j) / sqrt(hd) for j <= pos, softmax (:164-179), out[d] = sum_j p_j v_j[d]
// accumulated over j in order with separate multiply and add, as the reference does.
__global__ void attention_decode_kernel(const float *__restrict__ q, const float *__restrict__ kcache,
                                        const float *__restrict__ vcache, const int *__restrict__ d_pos, int n_q,
                                        int n_kv, int hd, float *__restrict__ out) {
    extern __shared__ float sc[];  // [pos + 1] scores, then [32] reduction
    pdl_wait();
    pdl_trigger();
    const int pos = *d_pos;
    const int len = pos + 1;
    float *red = sc + len;
    const int qh = blockIdx.x;
    const int kvh = qh * n_kv / n_q;  // src/attention.rs:111
    const int kv_dim = n_kv * hd;
    const float *qh_p = q + (size_t)qh * hd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const float scale = sqrtf((float)hd);
    for (int j = warp; j < len; j += nw) {
        const float *k = kcache + (size_t)j * kv_dim + (size_t)kvh * hd;
        float dot = 0.f;
        for (int e = lane; e < hd; e += 32) dot = __fadd_rn(dot, __fmul_rn(qh_p[e], k[e]));
        dot = warp_sum(dot);
        if (lane == 0) sc[j] = __fdiv_rn(dot, scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int j = threadIdx.x; j < len; j += blockDim.x) m = fmaxf(m, sc[j]);
    m = block_max(m, red);
    float s = 0.f;
    for (int j = threadIdx.x; j < len; j += blockDim.x) {
        const float e = expf(__fsub_rn(sc[j], m));
        sc[j] = e;
        s = __fadd_rn(s, e);
    }
    s = block_sum(s, red);
    for (int j = threadIdx.x; j < len; j += blockDim.x) sc[j] = __fdiv_rn(sc[j], s);
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.f;
        const float *v = vcache + (size_t)kvh * hd + d;
        for (int j = 0; j < len; ++j) acc = __fadd_rn(acc, __fmul_rn(sc[j], v[(size_t)j * kv_dim]));
        out[(size_t)qh * hd + d] = acc;
    }
}

// act = silu(gate) * up, silu(x) = x / (1 + exp(-x)) (src/ffn.rs:39-41, :52-54).
__global__ void silu_mul_kernel(const float *__restrict__ gu, int ffn, float *__restrict__ act) {
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ffn; i += gridDim.x * blockDim.x) {
        const float g = gu[i];
        act[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), gu[ffn + i]);
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

using namespace pyxis;

struct pyxis_cuda_model {
    pyxis_cuda_ctx *ctx = nullptr;
    pyxis_model_config cfg{};
    int q_dim = 0, kv_dim = 0;
    struct Layer {
        const pyxis_cuda_weights *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
        float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    };
    std::vector<Layer> layers;
    uint16_t *emb = nullptr;
    const pyxis_cuda_weights *lm_head = nullptr;
    float *final_norm = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    float *kcache = nullptr, *vcache = nullptr;
    float *x = nullptr, *h = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *tmp = nullptr, *gu = nullptr,
          *act = nullptr, *logits = nullptr;
    int *d_pos = nullptr, *d_token = nullptr, *d_step = nullptr, *d_out = nullptr;
    cudaGraphExec_t exec = nullptr;
    std::vector<void *> allocs;
};

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

// One decode step on `st` (what the graph holds).
int enqueue_step(pyxis_cuda_model *m, cudaStream_t st) {
    const pyxis_model_config &c = m->cfg;
    const int H = c.hidden;
    PdlScope pdl;  // kernels of the step may start while their predecessor finishes
    cudaError_t le = launch_kernel(embed_kernel, dim3((H + 255) / 256), dim3(256), 0, st, (const uint16_t *)m->emb,
                                   (const int *)m->d_token, c.vocab, H, m->x);
    if (le == cudaSuccess)
        le = launch_kernel(add_rmsnorm_kernel, dim3(1), dim3(kNormThreads), 0, st, m->x, (const float *)nullptr,
                           (const float *)m->layers[0].in_norm, m->h, H, c.rms_eps);
    if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
    for (int l = 0; l < c.n_layers; ++l) {
        const auto &L = m->layers[l];
        float *kc = m->kcache + (size_t)l * c.max_seq * m->kv_dim;
        float *vc = m->vcache + (size_t)l * c.max_seq * m->kv_dim;
        int rc = run_matmul(m->ctx, L.wqkv, m->h, 1, H, (size_t)m->q_dim + 2 * m->kv_dim, H, m->qkv,
                            (size_t)m->q_dim + 2 * m->kv_dim, nullptr, 0, st);
        if (rc) return rc;
        le = launch_kernel(qk_rope_append_kernel, dim3(c.n_q_heads + c.n_kv_heads + 1), dim3(c.head_dim),
                           (c.head_dim + 32) * sizeof(float), st, (const float *)m->qkv, (const float *)L.q_norm,
                           (const float *)L.k_norm, (const float *)m->rope_cos, (const float *)m->rope_sin,
                           (const int *)m->d_pos, c.n_q_heads, c.n_kv_heads, c.head_dim, c.rms_eps, m->q, kc, vc);
        if (le == cudaSuccess)
            le = launch_kernel(attention_decode_kernel, dim3(c.n_q_heads), dim3(128), (c.max_seq + 32) * sizeof(float),
                               st, (const float *)m->q, (const float *)kc, (const float *)vc, (const int *)m->d_pos,
                               c.n_q_heads, c.n_kv_heads, c.head_dim, m->attn);
        if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
        rc = run_matmul(m->ctx, L.wo, m->attn, 1, m->q_dim, H, m->q_dim, m->tmp, H, nullptr, 0, st);
        if (rc) return rc;
        le = launch_kernel(add_rmsnorm_kernel, dim3(1), dim3(kNormThreads), 0, st, m->x, (const float *)m->tmp,
                           (const float *)L.post_norm, m->h, H, c.rms_eps);
        if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
        rc = run_matmul(m->ctx, L.wgu, m->h, 1, H, 2 * (size_t)c.ffn, H, m->gu, 2 * (size_t)c.ffn, nullptr, 0, st);
        if (rc) return rc;
        le = launch_kernel(silu_mul_kernel, dim3((c.ffn + 255) / 256), dim3(256), 0, st, (const float *)m->gu, c.ffn,
                           m->act);
        if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
        rc = run_matmul(m->ctx, L.wdown, m->act, 1, c.ffn, H, c.ffn, m->tmp, H, nullptr, 0, st);
        if (rc) return rc;
        const float *next_norm = l + 1 < c.n_layers ? m->layers[l + 1].in_norm : m->final_norm;
        le = launch_kernel(add_rmsnorm_kernel, dim3(1), dim3(kNormThreads), 0, st, m->x, (const float *)m->tmp,
                           next_norm, m->h, H, c.rms_eps);
        if (le != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(le));
    }
    int rc = run_matmul(m->ctx, m->lm_head, m->h, 1, H, c.vocab, H, m->logits, c.vocab, nullptr, 0, st);
    if (rc) return rc;
    cudaError_t e = launch_argmax_scratch(m->logits, 1, c.vocab, c.vocab, 0, m->d_token, nullptr, m->ctx->amax,
                                          m->ctx->num_sms, st);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    e = launch_kernel(advance_kernel, dim3(1), dim3(1), 0, st, (const int *)m->d_token, m->d_out, m->d_pos, m->d_step);
    if (e != cudaSuccess) return model_fail(PYXIS_ECUDA, cudaGetErrorString(e));
    return PYXIS_OK;
}

bool weights_ok(const pyxis_cuda_weights *w, size_t n, int device) {
    return w && w->num_elements == n && w->device == device;
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

extern "C" int pyxis_cuda_model_create(pyxis_cuda_ctx *ctx, const pyxis_model_config *cfg, pyxis_cuda_model **out) {
    if (!ctx || !cfg || !out) return model_fail(PYXIS_EINVAL, "null argument");
    *out = nullptr;
    const pyxis_model_config &c = *cfg;
    if (c.hidden <= 0 || c.n_layers <= 0 || c.n_q_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 || c.ffn <= 0 ||
        c.vocab <= 0 || c.max_seq <= 0 || c.head_dim % 2 || c.head_dim > 1024 || c.n_q_heads % c.n_kv_heads)
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_create: bad config");
    if (c.hidden > 1024 * 8) return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_create: hidden > 8192");
    if ((size_t)c.max_seq * 4 + 256 > 160 * 1024)
        return model_fail(PYXIS_EINVAL, "pyxis_cuda_model_create: max_seq too large for the decode attention kernel");
    Guard g(ctx->device);
    auto *m = new (std::nothrow) pyxis_cuda_model();
    if (!m) return model_fail(PYXIS_ENOMEM, "host allocation failed");
    m->ctx = ctx;
    m->cfg = c;
    m->q_dim = c.n_q_heads * c.head_dim;
    m->kv_dim = c.n_kv_heads * c.head_dim;
    m->layers.resize(c.n_layers);
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
    if (!weights_ok(lm_head, (size_t)c.vocab * c.hidden, m->ctx->device))
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
    if (n_prompt == 0 || n_new == 0) return PYXIS_OK;
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
                                       (const void *)qk_rope_append_kernel, (const void *)attention_decode_kernel,
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
    for (void *p : m->allocs) cudaFree(p);
    delete m;
    return PYXIS_OK;
}
