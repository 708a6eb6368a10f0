/*
 * model.c -- restatement of the reference's decode stack around matmul (oracle, test-only):
 * src/rmsnorm.rs, src/attention.rs, src/ffn.rs, src/transformer.rs, src/kv_cache.rs,
 * src/embedding.rs and the greedy arm of the output head.  Used only to produce the greedy token
 * stream the CUDA decode loop must reproduce.  f32 transcendental functions are glibc's powf,
 * cosf, sinf, expf and sqrtf -- the same libm rustc's f32 methods call on x86-64 Linux.
 */
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "pyxis_oracle.h"

/* src/rmsnorm.rs:11-20 */
void oracle_rmsnorm(float *x, const float *weight, size_t n, float eps) {
    float ss = -0.0f; /* .map(|v| v * v).sum::<f32>() */
    for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float mean_square = ss / (float)n;
    float factor = 1.0f / sqrtf(mean_square + eps);
    for (size_t i = 0; i < n; ++i) x[i] *= factor * weight[i];
}

/* src/attention.rs:144-162 */
void oracle_apply_rope(float *q_or_k, size_t len, size_t head_dim, size_t pos, float theta) {
    size_t half = head_dim / 2;
    for (size_t h = 0; h + head_dim <= len; h += head_dim) {
        float *head = q_or_k + h;
        for (size_t i = 0; i < half; ++i) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
            float angle = (float)pos * freq;
            float c = cosf(angle), s = sinf(angle);
            float x0 = head[i], x1 = head[i + half];
            head[i] = x0 * c - x1 * s;
            head[i + half] = x1 * c + x0 * s;
        }
    }
}

/* src/attention.rs:164-179 */
void oracle_softmax(float *scores, size_t n) {
    float max = -INFINITY;
    for (size_t i = 0; i < n; ++i) max = fmaxf(max, scores[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        scores[i] = expf(scores[i] - max);
        sum += scores[i];
    }
    for (size_t i = 0; i < n; ++i) scores[i] /= sum;
}

/* src/ffn.rs:52-54 */
float oracle_silu(float x) { return x / (1.0f + expf(-x)); }

struct oracle_kv {
    size_t n_layers, kv_dim, max_len;
    size_t *len;
    float *keys, *values; /* [n_layers][max_len][kv_dim] */
};

oracle_kv *oracle_kv_new(const oracle_model *m, size_t max_len) {
    oracle_kv *kv = (oracle_kv *)calloc(1, sizeof(oracle_kv));
    if (!kv) return NULL;
    kv->n_layers = m->n_layers;
    kv->kv_dim = m->n_kv_heads * m->head_dim;
    kv->max_len = max_len;
    kv->len = (size_t *)calloc(m->n_layers, sizeof(size_t));
    size_t sz = m->n_layers * max_len * kv->kv_dim;
    kv->keys = (float *)malloc(sz * sizeof(float));
    kv->values = (float *)malloc(sz * sizeof(float));
    if (!kv->len || !kv->keys || !kv->values) {
        oracle_kv_free(kv);
        return NULL;
    }
    return kv;
}

void oracle_kv_free(oracle_kv *kv) {
    if (!kv) return;
    free(kv->len);
    free(kv->keys);
    free(kv->values);
    free(kv);
}

size_t oracle_kv_len(const oracle_kv *kv, size_t layer) { return kv->len[layer]; }

/* The model's projections.  The value computed for each row is exactly oracle_dot_int8 /
 * oracle_dot_int4 (same operations in the same order, so the same bits); the scale index
 * (o+i)/block is found without a division per element, which only makes the greedy-decode
 * oracle faster.  The timed CPU baseline keeps the reference's own per-element division. */
typedef struct {
    const oracle_weights *w;
    const float *x;
    size_t in, out;
    float *y;
    size_t next;
    pthread_mutex_t mu;
} mm_fast_job;

static void mm_fast_rows(const mm_fast_job *j, size_t r0, size_t r1) {
    const oracle_weights *w = j->w;
    const size_t K = j->in, bs = w->block_size;
    for (size_t r = r0; r < r1; ++r) {
        const size_t o = r * K;
        size_t blk = o / bs, blk_end = (blk + 1) * bs;
        float sc = w->scales[blk];
        if (w->kind == ORACLE_INT8) {
            const int8_t *q = (const int8_t *)w->data;
            float sum = -0.0f;
            for (size_t i = 0; i < K; ++i) {
                if (o + i == blk_end) { ++blk; blk_end += bs; sc = w->scales[blk]; }
                float t = j->x[i] * (float)q[o + i];
                t = t * sc;
                sum += t;
            }
            j->y[r] = sum;
        } else {
            const uint8_t *q = (const uint8_t *)w->data;
            float sum = 0.0f;
            for (size_t i = 0; i < K; ++i) {
                const size_t g = o + i;
                if (g == blk_end) { ++blk; blk_end += bs; sc = w->scales[blk]; }
                const uint8_t byte = q[g / 2];
                const uint8_t nib = (g % 2 == 0) ? (byte & 0x0f) : ((byte >> 4) & 0x0f);
                float t = j->x[i] * ((float)nib - 8.0f);
                t = t * sc;
                sum += t;
            }
            j->y[r] = sum;
        }
    }
}

static void *mm_fast_worker(void *arg) {
    mm_fast_job *j = (mm_fast_job *)arg;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        size_t r0 = j->next;
        j->next += 64;
        pthread_mutex_unlock(&j->mu);
        if (r0 >= j->out) break;
        size_t r1 = r0 + 64 < j->out ? r0 + 64 : j->out;
        mm_fast_rows(j, r0, r1);
    }
    return NULL;
}

static void mm(const oracle_weights *w, const float *x, size_t out, size_t in, float *y, int nt) {
    if (w->kind != ORACLE_INT8 && w->kind != ORACLE_INT4) {
        oracle_matmul(x, w->kind, w->data, w->scales, w->block_size, out, in, y, nt);
        return;
    }
    mm_fast_job j = {w, x, in, out, y, 0, PTHREAD_MUTEX_INITIALIZER};
    int n = nt > 0 ? nt : oracle_num_cpus();
    if (n > 64) n = 64;
    pthread_t th[64];
    int started = 0;
    for (int t = 1; t < n; ++t)
        if (pthread_create(&th[started], NULL, mm_fast_worker, &j) == 0) ++started;
    mm_fast_worker(&j);
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

const float *oracle_kv_keys(const oracle_kv *kv, size_t layer) {
    return kv->keys + layer * kv->max_len * kv->kv_dim;
}

/* Attention::forward (src/attention.rs:57-141).  x: [seq_len, hidden] (already input-normed),
 * out: [seq_len, hidden]. */
int oracle_attention_forward(const oracle_model *m, size_t layer, const float *x, size_t seq_len,
                             size_t start_pos, oracle_kv *kv, float *out, int nt) {
    size_t hd = m->head_dim, H = m->hidden;
    size_t q_dim = m->n_q_heads * hd, kv_dim = m->n_kv_heads * hd;
    if (kv->len[layer] != start_pos) return -1; /* assert_eq!(cache.len(), start_pos) (:68) */
    if (start_pos + seq_len > kv->max_len) return -1;
    float *queries = (float *)malloc(seq_len * q_dim * sizeof(float));
    float *scores = (float *)malloc((start_pos + seq_len) * sizeof(float));
    float *attn = (float *)malloc(q_dim * sizeof(float));
    if (!queries || !scores || !attn) {
        free(queries); free(scores); free(attn);
        return -1;
    }
    float *kbase = kv->keys + layer * kv->max_len * kv_dim;
    float *vbase = kv->values + layer * kv->max_len * kv_dim;
    for (size_t pos = 0; pos < seq_len; ++pos) { /* :74-98 */
        const float *in = x + pos * H;
        float *q = queries + pos * q_dim;
        float *k = kbase + (start_pos + pos) * kv_dim; /* cache.append (:100) writes here */
        float *v = vbase + (start_pos + pos) * kv_dim;
        mm(&m->wq[layer], in, q_dim, H, q, nt);
        mm(&m->wk[layer], in, kv_dim, H, k, nt);
        mm(&m->wv[layer], in, kv_dim, H, v, nt);
        if (m->q_norm && m->q_norm[layer])
            for (size_t h = 0; h < m->n_q_heads; ++h)
                oracle_rmsnorm(q + h * hd, m->q_norm[layer], hd, m->rms_eps);
        if (m->k_norm && m->k_norm[layer])
            for (size_t h = 0; h < m->n_kv_heads; ++h)
                oracle_rmsnorm(k + h * hd, m->k_norm[layer], hd, m->rms_eps);
        oracle_apply_rope(q, q_dim, hd, start_pos + pos, m->rope_theta);
        oracle_apply_rope(k, kv_dim, hd, start_pos + pos, m->rope_theta);
    }
    kv->len[layer] += seq_len;
    size_t cached_len = kv->len[layer];
    float scale = sqrtf((float)hd); /* :105 */
    for (size_t pos = 0; pos < seq_len; ++pos) { /* :107-138 */
        for (size_t i = 0; i < q_dim; ++i) attn[i] = 0.0f;
        for (size_t qh = 0; qh < m->n_q_heads; ++qh) {
            size_t kvh = qh * m->n_kv_heads / m->n_q_heads; /* :111 */
            const float *q = queries + pos * q_dim + qh * hd;
            size_t max_key_pos = start_pos + pos;
            for (size_t kp = 0; kp < cached_len; ++kp) scores[kp] = -INFINITY;
            for (size_t kp = 0; kp <= max_key_pos && kp < cached_len; ++kp) {
                const float *k = kbase + kp * kv_dim + kvh * hd;
                float dot = -0.0f;
                for (size_t d = 0; d < hd; ++d) dot += q[d] * k[d];
                scores[kp] = dot / scale;
            }
            oracle_softmax(scores, cached_len);
            float *o = attn + qh * hd;
            for (size_t kp = 0; kp < cached_len; ++kp) {
                const float *v = vbase + kp * kv_dim + kvh * hd;
                for (size_t d = 0; d < hd; ++d) o[d] += scores[kp] * v[d];
            }
        }
        mm(&m->wo[layer], attn, H, q_dim, out + pos * H, nt); /* :136 */
    }
    free(queries);
    free(scores);
    free(attn);
    return 0;
}

/* Ffn::forward (src/ffn.rs:33-50) for one position. */
static void ffn_forward(const oracle_model *m, size_t layer, const float *x, float *out,
                        float *gate, float *up, int nt) {
    mm(&m->wgate[layer], x, m->ffn, m->hidden, gate, nt);
    mm(&m->wup[layer], x, m->ffn, m->hidden, up, nt);
    for (size_t i = 0; i < m->ffn; ++i) gate[i] = oracle_silu(gate[i]) * up[i];
    mm(&m->wdown[layer], gate, m->hidden, m->ffn, out, nt);
}

int oracle_ffn_forward(const oracle_model *m, size_t layer, const float *x, float *out, int nt) {
    float *gate = (float *)malloc(m->ffn * sizeof(float));
    float *up = (float *)malloc(m->ffn * sizeof(float));
    int rc = (gate && up) ? 0 : -1;
    if (rc == 0) ffn_forward(m, layer, x, out, gate, up, nt);
    free(gate);
    free(up);
    return rc;
}

/* TransformerBlock::forward (src/transformer.rs:28-62) for layer l; scratch holds 2 seq_len H +
 * 2 ffn + H floats. */
static int block_forward(const oracle_model *m, size_t l, float *x, size_t seq_len, size_t start_pos,
                         oracle_kv *kv, float *scratch, int nt) {
    size_t H = m->hidden;
    float *residual = scratch, *attn = residual + seq_len * H, *gate = attn + seq_len * H;
    float *up = gate + m->ffn, *fo = up + m->ffn;
    memcpy(residual, x, seq_len * H * sizeof(float));
    for (size_t p = 0; p < seq_len; ++p) oracle_rmsnorm(x + p * H, m->input_norm[l], H, m->rms_eps);
    int rc = oracle_attention_forward(m, l, x, seq_len, start_pos, kv, attn, nt);
    if (rc) return rc;
    for (size_t i = 0; i < seq_len * H; ++i) x[i] = residual[i] + attn[i];
    memcpy(residual, x, seq_len * H * sizeof(float));
    for (size_t p = 0; p < seq_len; ++p) oracle_rmsnorm(x + p * H, m->post_norm[l], H, m->rms_eps);
    for (size_t p = 0; p < seq_len; ++p) {
        ffn_forward(m, l, x + p * H, fo, gate, up, nt);
        for (size_t i = 0; i < H; ++i) x[p * H + i] = residual[p * H + i] + fo[i];
    }
    return 0;
}

static float *block_scratch(const oracle_model *m, size_t seq_len) {
    return (float *)malloc((2 * seq_len * m->hidden + 2 * m->ffn + m->hidden) * sizeof(float));
}

int oracle_block_forward(const oracle_model *m, size_t layer, float *x, size_t seq_len, size_t start_pos,
                         oracle_kv *kv, int nt) {
    float *scratch = block_scratch(m, seq_len);
    int rc = scratch ? block_forward(m, layer, x, seq_len, start_pos, kv, scratch, nt) : -1;
    free(scratch);
    return rc;
}

/* Transformer::forward (src/transformer.rs:80-90): the blocks, then the final norm. */
int oracle_transformer_forward(const oracle_model *m, float *x, size_t seq_len, size_t start_pos,
                               oracle_kv *kv, int nt) {
    size_t H = m->hidden;
    float *scratch = block_scratch(m, seq_len);
    int rc = scratch ? 0 : -1;
    for (size_t l = 0; l < m->n_layers && rc == 0; ++l) rc = block_forward(m, l, x, seq_len, start_pos, kv, scratch, nt);
    if (rc == 0)
        for (size_t p = 0; p < seq_len; ++p) oracle_rmsnorm(x + p * H, m->final_norm, H, m->rms_eps);
    free(scratch);
    return rc;
}

/* Model::generate (src/model.rs:245-285) with the sampler replaced by output_head::argmax. */
int oracle_greedy_decode(const oracle_model *m, const int32_t *prompt, size_t n_prompt,
                         size_t n_new, int32_t *out_tokens, int nt) {
    if (n_prompt == 0 || n_new == 0) return 0;
    size_t H = m->hidden;
    oracle_kv *kv = oracle_kv_new(m, n_prompt + n_new);
    float *x = (float *)malloc(n_prompt * H * sizeof(float));
    float *logits = (float *)malloc(m->vocab * sizeof(float));
    int rc = (kv && x && logits) ? 0 : -1;
    for (size_t p = 0; p < n_prompt && rc == 0; ++p) {
        if (prompt[p] < 0 || (size_t)prompt[p] >= m->vocab) rc = -1; /* embedding.rs:19 */
        else memcpy(x + p * H, m->embedding + (size_t)prompt[p] * H, H * sizeof(float));
    }
    if (rc == 0) rc = oracle_transformer_forward(m, x, n_prompt, 0, kv, nt);
    if (rc == 0) {
        mm(&m->lm_head, x + (n_prompt - 1) * H, m->vocab, H, logits, nt);
        int32_t next = (int32_t)oracle_argmax(logits, m->vocab);
        for (size_t i = 0; i < n_new; ++i) {
            out_tokens[i] = next;
            if (i + 1 == n_new) break;
            memcpy(x, m->embedding + (size_t)next * H, H * sizeof(float));
            rc = oracle_transformer_forward(m, x, 1, n_prompt + i, kv, nt);
            if (rc) break;
            mm(&m->lm_head, x, m->vocab, H, logits, nt);
            next = (int32_t)oracle_argmax(logits, m->vocab);
        }
    }
    oracle_kv_free(kv);
    free(x);
    free(logits);
    return rc;
}

/* The hidden state greedy decoding reads the first token from: the whole prompt through the
 * transformer (src/model.rs:245-262, src/transformer.rs:28-90), then the final RMSNorm of its last
 * position (the row that src/output_head.rs:21-28 multiplies with the lm_head). */
int oracle_prefill_hidden(const oracle_model *m, const int32_t *prompt, size_t n_prompt, float *out_hidden, int nt) {
    if (n_prompt == 0) return -1;
    size_t H = m->hidden;
    oracle_kv *kv = oracle_kv_new(m, n_prompt);
    float *x = (float *)malloc(n_prompt * H * sizeof(float));
    int rc = (kv && x) ? 0 : -1;
    for (size_t p = 0; p < n_prompt && rc == 0; ++p) {
        if (prompt[p] < 0 || (size_t)prompt[p] >= m->vocab) rc = -1;
        else memcpy(x + p * H, m->embedding + (size_t)prompt[p] * H, H * sizeof(float));
    }
    if (rc == 0) rc = oracle_transformer_forward(m, x, n_prompt, 0, kv, nt);
    if (rc == 0) memcpy(out_hidden, x + (n_prompt - 1) * H, H * sizeof(float));
    oracle_kv_free(kv);
    free(x);
    return rc;
}
