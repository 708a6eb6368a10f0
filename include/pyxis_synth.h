/*
 * pyxis_synth.h -- seeded synthetic inputs for the benchmark workloads and parity tests.
 *
 * The reference is benchmarked on real Qwen3 checkpoints the build does not have, so the
 * workloads use seeded synthetic tensors with the checkpoint's shapes: weights N(0, 0.02)
 * rounded to bf16, activations N(0, 1) in f32, token ids uniform in [0, vocab).  No reference
 * counterpart; this is host code (multi-threaded), so a tensor is identical on every machine.
 *
 * Element i of a tensor with seed s is a pure function of (s, i): Box-Muller (cosine branch,
 * double precision) over the splitmix64 outputs number 2i and 2i+1 of the stream started at s.
 */
#ifndef PYXIS_SYNTH_H
#define PYXIS_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[i] = (float)(sigma * z_i), z_i ~ N(0, 1). */
void pyxis_synth_normal_f32(uint64_t seed, size_t n, float sigma, float *out);

/* The same values rounded to bf16 (round to nearest even), as raw bits. */
void pyxis_synth_normal_bf16(uint64_t seed, size_t n, float sigma, uint16_t *out);

/* out[i] uniform in [0, vocab). */
void pyxis_synth_tokens(uint64_t seed, size_t n, uint32_t vocab, int32_t *out);

#ifdef __cplusplus
}
#endif
#endif
