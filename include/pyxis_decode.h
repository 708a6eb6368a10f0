/*
 * pyxis_decode.h -- device-resident greedy decode of the transformer pyxis runs.
 *
 * Replaces Model::generate (src/model.rs:245-285) with temperature-0 sampling (the argmax of
 * src/output_head.rs:25-44) for the Qwen3 layer stack of src/transformer.rs:28-90:
 *   RmsNorm (src/rmsnorm.rs:11-20) -> Attention (src/attention.rs:57-141: q/k/v projections,
 *   per-head QK RMSNorm, RoPE :144-162, causal GQA softmax attention over an f32 KV cache
 *   (src/kv_cache.rs), o projection) -> residual -> RmsNorm -> Ffn (src/ffn.rs:33-54: gate/up,
 *   SiLU, down) -> residual; final RmsNorm; lm_head; argmax.
 * Every projection is a quantized matrix from pyxis_cuda.h, multiplied on the tensor cores or the
 * GEMV kernels; everything between the projections runs as CUDA kernels on the context's stream,
 * and one decode step is captured once into a CUDA graph and replayed per token.  Prompt tokens
 * go through the same step one position at a time, as the reference's prefill does
 * (src/attention.rs:74-98): position p attends to keys 0..p.
 *
 * A model runs on its context's stream and uses the context's scratch, so its calls follow the
 * context's rule: they must not overlap with other work of the same context (another model's
 * generate, a `_dev` call, a host-pointer matmul from another thread).  Use one context per
 * concurrently generating model.
 */
#ifndef PYXIS_DECODE_H
#define PYXIS_DECODE_H

#include <stddef.h>
#include <stdint.h>

#include "pyxis_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ModelConfig (src/model.rs:63-75) plus the KV-cache capacity in positions. */
typedef struct {
    int hidden, n_layers, n_q_heads, n_kv_heads, head_dim, ffn, vocab;
    float rms_eps, rope_theta;
    int max_seq;
} pyxis_model_config;

typedef struct pyxis_cuda_model pyxis_cuda_model;

/* Allocates the KV cache, activations and the RoPE table (computed on the host in f32 with the
 * reference's formula, src/attention.rs:151-154) on the context's device. */
int pyxis_cuda_model_create(pyxis_cuda_ctx *ctx, const pyxis_model_config *cfg, pyxis_cuda_model **m);

/* One layer's weights.  Projections are device handles kept by reference (they must outlive the
 * model): wqkv = rows [q_proj (n_q*hd); k_proj (n_kv*hd); v_proj (n_kv*hd)] x hidden (per-row or
 * per-group quantisation packs the stacked rows exactly as the three matrices), wo = hidden x
 * n_q*hd, wgu = [gate_proj; up_proj] (2*ffn x hidden), wdown = hidden x ffn.  Norm weights are host
 * f32 arrays copied to the device; q_norm / k_norm NULL means the layer has no QK-norm
 * (src/model.rs:118-135). */
int pyxis_cuda_model_set_layer(pyxis_cuda_model *m, int layer, const pyxis_cuda_weights *wqkv,
                               const pyxis_cuda_weights *wo, const pyxis_cuda_weights *wgu,
                               const pyxis_cuda_weights *wdown, const float *input_norm,
                               const float *post_norm, const float *q_norm, const float *k_norm);

/* The token embedding as host bf16 bits [vocab, hidden] (widened exactly on lookup, as
 * tensor_f32 does), the lm_head handle (vocab x hidden; with tied embeddings a quantised copy of
 * the same table, src/model.rs:219-224) and the final norm weight (host f32). */
int pyxis_cuda_model_set_head(pyxis_cuda_model *m, const uint16_t *embedding_bf16,
                              const pyxis_cuda_weights *lm_head, const float *final_norm);

/* Greedy generation: feeds the n_prompt ids, then writes the n_new next tokens to out_tokens.
 * An empty prompt (n_prompt == 0) is PYXIS_EINVAL, as in pyxis_cuda_model_generate_batch; n_new
 * == 0 returns PYXIS_OK with nothing written.  n_prompt + n_new - 1 <= max_seq.  timing_ms (optional, 2 floats): device time of
 * the prompt phase (through the first generated token) and of the remaining n_new - 1 steps. */
int pyxis_cuda_model_generate(pyxis_cuda_model *m, const int32_t *prompt, size_t n_prompt, size_t n_new,
                              int32_t *out_tokens, float *timing_ms);

/* Greedy generation for n_seq independent prompts of n_prompt ids each (row-major
 * [n_seq][n_prompt]) side by side; writes out_tokens [n_seq][n_new].  Each sequence gets exactly
 * the tokens pyxis_cuda_model_generate would give it alone (up to the order of f32 sums: prompts
 * go through tensor-core GEMMs and a causal prefill attention kernel, then every new token is one
 * batched step).  n_prompt + n_new - 1 <= max_seq, n_seq <= 1024, n_prompt <= 16384.  The first call, and any later
 * call with more sequences, a longer prompt or more new tokens, allocates on the context's device
 * a KV cache of n_seq x n_layers x max_seq x 2 x n_kv_heads x head_dim floats and work buffers
 * (prompts are processed up to 16384 positions at a time); they are kept until
 * pyxis_cuda_model_free.  timing_ms (optional, 2 floats): device time of the prefill through the
 * first generated tokens, and of the remaining n_new - 1 steps. */
int pyxis_cuda_model_generate_batch(pyxis_cuda_model *m, const int32_t *prompts, size_t n_seq, size_t n_prompt,
                                    size_t n_new, int32_t *out_tokens, float *timing_ms);

/* Diagnostics, no counterpart in the reference: runs the prefill of pyxis_cuda_model_generate_batch
 * for n_seq prompts of n_prompt ids and writes each sequence's final-norm hidden state of its last
 * prompt position (the row the lm_head multiplies for the first generated token) to hidden_out
 * [n_seq][hidden] (host memory).  Not with a vocab-parallel head. */
int pyxis_cuda_model_prefill_hidden(pyxis_cuda_model *m, const int32_t *prompts, size_t n_seq, size_t n_prompt,
                                    float *hidden_out);

int pyxis_cuda_model_free(pyxis_cuda_model *m);

/* The decode step's row operations, for known-answer checks of the device arithmetic: the same
 * device functions the decode kernels apply, run by one CTA on n host values (n <= 65536),
 * synchronously on the context's stream.
 *   PYXIS_ROW_RMSNORM  out = RmsNorm::forward(x) with weight w and eps (src/rmsnorm.rs:11-20)
 *   PYXIS_ROW_ROPE     out = apply_rope on every head_dim-wide head of x at `pos` with `theta`
 *                      (src/attention.rs:144-162; the table from pyxis_rope_table)
 *   PYXIS_ROW_SILU     out[i] = silu(x[i]) (src/ffn.rs:52-54)
 * Unused arguments are ignored. */
enum { PYXIS_ROW_RMSNORM = 1, PYXIS_ROW_ROPE = 2, PYXIS_ROW_SILU = 3 };
int pyxis_cuda_row_op(pyxis_cuda_ctx *ctx, int op, const float *x, size_t n, const float *w, float eps,
                      int head_dim, int pos, float theta, float *out);

/* The RoPE table the model uses: cos/sin[pos * (head_dim/2) + i] of pos * theta^(-2i/head_dim),
 * computed on the host in f32 exactly as src/attention.rs:151-154 does. */
int pyxis_rope_table(float theta, int head_dim, int max_pos, float *cos_out, float *sin_out);

#ifdef __cplusplus
}
#endif
#endif
