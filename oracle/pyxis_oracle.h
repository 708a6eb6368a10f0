/*
 * pyxis_oracle.h -- CPU restatement of the reference (mizzy/pyxis, Rust) hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA path and the timed
 * CPU baseline ("port" of the reference's Rayon path).  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs load it.  The product (pyxis_b200, libpyxis_cuda)
 * never links or calls it.
 *
 * The reference cannot be built here (Rust crate, no cargo/rustc in the image), so every function
 * below restates one reference function in C, keeping its operation order, and cites it.
 * Build: -O2 -ffp-contract=off, no -ffast-math, so each f32 expression rounds exactly as rustc's
 * (x86-64, SSE, no FMA contraction: rustc never contracts a*b+c into an FMA).
 *
 * Parity is pinned by the reference's own known-answer tests (src/weights.rs:202-366,
 * src/matmul.rs:335-489, src/model.rs:627-698, tests/gguf.rs:56-108, src/attention.rs:218-262,
 * src/rmsnorm.rs:34-63, src/output_head.rs:81-89), restated in tests/golden/reference_kats.json.
 */
#ifndef PYXIS_ORACLE_H
#define PYXIS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- src/weights.rs ---------------------------------------------------------------------- */

/* Weights::quantize_int8 (src/weights.rs:94-118).  data: n bytes, scales: ceil(n/block). */
void oracle_quantize_int8(const float *values, size_t n, size_t block_size,
                          int8_t *data, float *scales);

/* Weights::quantize_int4 (src/weights.rs:120-151).  data: ceil(n/2) bytes (pre-filled 0x88),
 * scales: ceil(n/block). */
void oracle_quantize_int4(const float *values, size_t n, size_t block_size,
                          uint8_t *data, float *scales);

/* ---- src/model.rs ------------------------------------------------------------------------ */

/* dequantize_weights, Bf16 arm (src/model.rs:535-538): f32::from_bits((b as u32) << 16). */
void oracle_bf16_to_f32(const uint16_t *src, size_t n, float *dst);

/* dequantize_weights, Int8 / Int4 arms (src/model.rs:539-564). */
void oracle_dequantize_int8(const int8_t *data, const float *scales, size_t block_size,
                            size_t n, float *dst);
void oracle_dequantize_int4(const uint8_t *data, const float *scales, size_t block_size,
                            size_t n, float *dst);

/* ---- src/gguf.rs ------------------------------------------------------------------------- */

/* read_q8_0_weights (src/gguf.rs:245-271): blocks of 34 bytes = f16 scale (LE) + 32 x i8,
 * truncated to n elements.  data: n bytes; scales: ceil(n/32). */
void oracle_q8_0_to_int8(const uint8_t *blocks, size_t n, int8_t *data, float *scales);
/* half::f16 -> f32 (exact). */
float oracle_f16_to_f32(uint16_t h);

/* ---- src/matmul.rs ----------------------------------------------------------------------- */

/* dot_product_int8_scalar (src/matmul.rs:297-317): sum over i of (x[i] * q[o+i] as f32) *
 * scales[(o+i)/bs], Iterator::sum from -0.0, left to right. */
float oracle_dot_int8(const float *x, const int8_t *q, const float *scales, size_t block_size,
                      size_t offset, size_t len);

/* dot_product_int4 (src/matmul.rs:149-173): sum starts at +0.0,
 * sum += (x[i] * (nib - 8.0)) * scale. */
float oracle_dot_int4(const float *x, const uint8_t *packed, const float *scales,
                      size_t block_size, size_t offset, size_t len);

/* dot_product_scalar / dot_product_bf16_scalar (src/matmul.rs:284-295). */
float oracle_dot_f32(const float *a, const float *b, size_t len);
float oracle_dot_bf16(const float *a, const uint16_t *b, size_t len);

/* Weight kinds accepted by oracle_matmul (the enum Weights arms, src/weights.rs:6-21). */
enum oracle_kind { ORACLE_F32 = 0, ORACLE_BF16 = 1, ORACLE_INT8 = 2, ORACLE_INT4 = 3 };

/* matmul (src/matmul.rs:21-97): y[n] = dot(x, W[n,:]) for n in 0..out_features, rows split
 * across nthreads worker threads (the Rayon into_par_iter over output rows, :67-96; the per-row
 * result does not depend on the split).  `data` is f32 / u16 / i8 / packed u8 by kind; `scales`
 * and `block_size` are ignored for F32/BF16.  nthreads <= 0 means one thread per online core.
 * Returns 0, or -1 on a shape error (where the reference asserts, :27-50). */
int oracle_matmul(const float *x, int kind, const void *data, const float *scales,
                  size_t block_size, size_t out_features, size_t in_features, float *y,
                  int nthreads);

/* M independent matmul calls, the way the reference's prefill issues one matmul per position
 * (src/attention.rs:74-79).  X: [M, in], Y: [M, out]. */
int oracle_matmul_batch(const float *X, size_t M, int kind, const void *data,
                        const float *scales, size_t block_size, size_t out_features,
                        size_t in_features, float *Y, int nthreads);

/* output_head::argmax (src/output_head.rs:30-44): first index of the maximum under strict >. */
size_t oracle_argmax(const float *values, size_t n);

/* ---- decode model (src/rmsnorm.rs, src/attention.rs, src/ffn.rs, src/transformer.rs) -------- */

/* RmsNorm::forward (src/rmsnorm.rs:11-20), in place. */
void oracle_rmsnorm(float *x, const float *weight, size_t n, float eps);
/* apply_rope (src/attention.rs:144-162), in place over len/head_dim heads. */
void oracle_apply_rope(float *q_or_k, size_t len, size_t head_dim, size_t pos, float theta);
/* softmax (src/attention.rs:164-179), in place. */
void oracle_softmax(float *scores, size_t n);
/* silu (src/ffn.rs:52-54). */
float oracle_silu(float x);

/* One quantized projection of the model: the kind/data/scales/block of a Weights value. */
typedef struct {
    int kind;
    const void *data;
    const float *scales;
    size_t block_size;
} oracle_weights;

typedef struct {
    size_t hidden, n_layers, n_q_heads, n_kv_heads, head_dim, ffn, vocab;
    float rms_eps, rope_theta;
    const float *embedding;          /* [vocab, hidden] f32 (Embedding, src/embedding.rs:18-24) */
    const float *const *input_norm;  /* [n_layers][hidden] */
    const float *const *post_norm;   /* [n_layers][hidden] */
    const float *const *q_norm;      /* [n_layers][head_dim] or NULL entries */
    const float *const *k_norm;
    const oracle_weights *wq, *wk, *wv, *wo, *wgate, *wup, *wdown; /* [n_layers] */
    const float *final_norm;         /* [hidden] */
    oracle_weights lm_head;          /* [vocab, hidden] */
} oracle_model;

typedef struct oracle_kv oracle_kv;
/* KvCache::new (src/kv_cache.rs:13-17) with room for max_len positions per layer. */
oracle_kv *oracle_kv_new(const oracle_model *m, size_t max_len);
void oracle_kv_free(oracle_kv *kv);
size_t oracle_kv_len(const oracle_kv *kv, size_t layer);

/* The cached keys of one layer, [max_len][n_kv_heads * head_dim] (LayerCache::keys,
 * src/kv_cache.rs:43-45): normalised and rotated as Attention::forward stores them. */
const float *oracle_kv_keys(const oracle_kv *kv, size_t layer);

/* Attention::forward (src/attention.rs:57-141) of one layer over seq_len positions of x
 * [seq_len, hidden] starting at start_pos (== the layer's cache length, :68), appending to kv;
 * out [seq_len, hidden].  Returns 0 or -1. */
int oracle_attention_forward(const oracle_model *m, size_t layer, const float *x, size_t seq_len,
                             size_t start_pos, oracle_kv *kv, float *out, int nthreads);

/* Ffn::forward (src/ffn.rs:33-50) of one layer for one position: out [hidden].  Returns 0 or -1. */
int oracle_ffn_forward(const oracle_model *m, size_t layer, const float *x, float *out, int nthreads);

/* TransformerBlock::forward (src/transformer.rs:28-62) of one layer, in place on x
 * [seq_len, hidden].  Returns 0 or -1. */
int oracle_block_forward(const oracle_model *m, size_t layer, float *x, size_t seq_len, size_t start_pos,
                         oracle_kv *kv, int nthreads);

/* Transformer::forward (src/transformer.rs:80-90) over seq_len positions of x [seq_len, hidden],
 * in place, appending to kv.  Returns 0 or -1 (capacity / shape). */
int oracle_transformer_forward(const oracle_model *m, float *x, size_t seq_len, size_t start_pos,
                               oracle_kv *kv, int nthreads);

/* Greedy decode: prefill `prompt` (n_prompt ids), then n_new tokens, each the argmax of the
 * lm_head logits (output_head.rs:25-27) -- Model::generate (src/model.rs:245-285) with temperature
 * 0 and no repetition penalty.  Writes n_new ids to out_tokens.  Returns 0 or -1. */
/* The final-norm hidden state of the prompt's last position (the first token's lm_head input). */
int oracle_prefill_hidden(const oracle_model *m, const int32_t *prompt, size_t n_prompt, float *out_hidden, int nt);
int oracle_greedy_decode(const oracle_model *m, const int32_t *prompt, size_t n_prompt,
                         size_t n_new, int32_t *out_tokens, int nthreads);

/* Online CPU count (the baseline's thread count when nthreads <= 0). */
int oracle_num_cpus(void);

#ifdef __cplusplus
}
#endif
#endif
