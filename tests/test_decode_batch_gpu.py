"""Greedy generation for many sequences at once (pyxis_cuda_model_generate_batch): every
sequence must get the tokens the oracle's restatement of Model::generate (src/model.rs:245-285,
argmax sampling) gives it alone, and at the Qwen3-1.7B shape the tokens the single-sequence
device decoder gives it."""
import numpy as np
import pytest

import oracle
from pyxis_b200 import synth_tokens
from pyxis_b200.model import QWEN3_1_7B, Decoder, ModelConfig, SyntheticModel

pytestmark = pytest.mark.gpu

SMALL = ModelConfig(hidden=256, n_layers=3, n_q_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=2048,
                    rope_theta=10000.0)


@pytest.mark.parametrize("qtype", ["int8", "int4"])
def test_small_model_batch_matches_oracle(qtype):
    m = SyntheticModel(SMALL, seed=23)
    dec = Decoder(m, qtype=qtype, max_seq=96)
    # 70 prompt ids: two 64-query tiles and three 32-key tiles in the prefill attention
    prompts = synth_tokens(0x77, 3 * 70, SMALL.vocab).reshape(3, 70)
    toks, (t_pre, t_dec) = dec.generate_batch(prompts, 6)
    assert toks.shape == (3, 6) and t_pre > 0 and t_dec > 0
    for s in range(3):
        ref = oracle.greedy_decode(SMALL, m.bf16, qtype, list(prompts[s]), 6)
        assert np.array_equal(toks[s], ref), (s, toks[s], ref)
    # a second, smaller call reuses the buffers; one token only (no decode step)
    toks2, _ = dec.generate_batch(prompts[:2, :9], 1)
    for s in range(2):
        assert np.array_equal(toks2[s], oracle.greedy_decode(SMALL, m.bf16, qtype, list(prompts[s, :9]), 1))
    dec.close()


def test_small_model_batch_of_17_uses_gemm_steps():
    """17 sequences: the decode-step projections take the tensor-core GEMM (M >= 16)."""
    m = SyntheticModel(SMALL, seed=5)
    dec = Decoder(m, qtype="int4", max_seq=40)
    prompts = synth_tokens(0x99, 17 * 12, SMALL.vocab).reshape(17, 12)
    toks, _ = dec.generate_batch(prompts, 4)
    for s in range(17):
        assert np.array_equal(toks[s], oracle.greedy_decode(SMALL, m.bf16, "int4", list(prompts[s]), 4)), s
    dec.close()


def test_qwen3_shape_batch_matches_single_sequence_decoder():
    m = SyntheticModel(QWEN3_1_7B, seed=0x5EED)
    dec = Decoder(m, qtype="int4", max_seq=80)
    prompts = synth_tokens(0xB0, 3 * 40, QWEN3_1_7B.vocab).reshape(3, 40)
    toks, _ = dec.generate_batch(prompts, 8)
    for s in range(3):
        one, _ = dec.generate(prompts[s], 8)
        assert np.array_equal(toks[s], one), (s, toks[s], one)
    dec.close()


def test_qwen3_shape_batch_of_6_on_the_mma_gemv():
    """Six sequences: the decode steps' 6-row products of the large int4 matrices (qkv, gate|up,
    down, lm_head) take the mma.sync GEMV, the o projection the CUDA-core batch kernel; every
    sequence's greedy tokens equal the single-sequence decoder's (batch-1 GEMVs)."""
    import pyxis_b200 as px
    m = SyntheticModel(QWEN3_1_7B, seed=0x5EE6)
    dec = Decoder(m, qtype="int4", max_seq=48)
    H, F, V = QWEN3_1_7B.hidden, QWEN3_1_7B.ffn, QWEN3_1_7B.vocab
    probe = px.Weights.quantize_int4(px.synth_normal_bf16(1, 2 * F * H, 0.02), 32)  # the gate|up shape
    assert px.matmul_kernel_name(probe, 6, 2 * F, H) == "gemv_mma_kernel"
    del probe
    prompts = synth_tokens(0xB6, 6 * 24, V).reshape(6, 24)
    toks, _ = dec.generate_batch(prompts, 5)
    for s in range(6):
        one, _ = dec.generate(prompts[s], 5)
        assert np.array_equal(toks[s], one), (s, toks[s], one)
    dec.close()


# GQA 16 / 8 x 128 like Qwen3-1.7B, narrow elsewhere so that the oracle's prefill of 2048
# positions takes seconds
GQA_2048 = ModelConfig(hidden=256, n_layers=1, n_q_heads=16, n_kv_heads=8, head_dim=128, ffn=512, vocab=2048,
                       rope_theta=1e6)


def test_prefill_of_2048_positions_matches_oracle():
    """The batched prefill at the config-5 prompt length: 2048 positions, i.e. 16 query tiles of
    128 with up to 16 key tiles of 128 in the tensor-core causal attention (several raises of the
    running maximum per row), with the GQA 16 / 8 x 128 heads.
    Sequence 0's final-norm hidden state (the first token's lm_head input) is held to the matmul
    bar against the oracle's prefill -- rel(y, r) = max_i |y_i - r_i| / max(|r_i|, 1e-3 max|r|)
    <= 1e-3 -- and sequence 1's greedy tokens must equal the oracle's."""
    m = SyntheticModel(GQA_2048, seed=41)
    dec = Decoder(m, qtype="int4", max_seq=2048 + 4)
    prompts = synth_tokens(0x2048, 2 * 2048, GQA_2048.vocab).reshape(2, 2048)
    hid = dec.prefill_hidden(prompts)
    toks, _ = dec.generate_batch(prompts, 4)
    dec.close()
    ref = oracle.prefill_hidden(GQA_2048, m.bf16, "int4", list(prompts[0]))
    r = ref.astype(np.float64)
    err = float((np.abs(hid[0].astype(np.float64) - r) / np.maximum(np.abs(r), 1e-3 * np.abs(r).max())).max())
    assert err <= 1e-3, err
    want = oracle.greedy_decode(GQA_2048, m.bf16, "int4", list(prompts[1]), 4)
    assert np.array_equal(toks[1], want), (toks[1], want)


@pytest.mark.parametrize("hn", [3.0])
def test_prefill_with_sharp_attention_matches_oracle(hn):
    """QK-norm weights of 3 (scores 9x those of unit weights): peaked softmax rows whose running
    maximum is raised at different key tiles for different rows of one warp -- the prefill
    attention's per-row rescaling -- over 640 positions (5 query and key tiles of 128), against
    the oracle: the greedy tokens, and the final-norm hidden state of every sequence within
    max_i |y_i - r_i| <= 1e-5 max|r|.  With scores this large the reference's own f32 softmax is
    the larger error term (about 5e-6 of max |out| against float64, where the tensor-core
    attention measures 2e-6), so the element-wise 1e-3 bar of the test above would measure the
    reference's rounding at the hidden state's near-zero elements; the max-norm bar is twice the
    reference's own error."""
    cfg = GQA_2048
    m = SyntheticModel(cfg, seed=43, head_norm_value=hn)
    hn_w = m.head_norm()
    dec = Decoder(m, qtype="int8", max_seq=640 + 4)
    prompts = synth_tokens(0x640, 2 * 640, cfg.vocab).reshape(2, 640)
    hid = dec.prefill_hidden(prompts)
    toks, _ = dec.generate_batch(prompts, 3)
    dec.close()
    for sq in range(2):
        r = oracle.prefill_hidden(cfg, m.bf16, "int8", list(prompts[sq]), head_norm=hn_w).astype(np.float64)
        d = np.abs(hid[sq].astype(np.float64) - r)
        err_max = float(d.max() / np.abs(r).max())
        err_elem = float((d / np.maximum(np.abs(r), 1e-3 * np.abs(r).max())).max())
        assert err_max <= 1e-5, (sq, err_max, err_elem)
        want = oracle.greedy_decode(cfg, m.bf16, "int8", list(prompts[sq]), 3, head_norm=hn_w)
        assert np.array_equal(toks[sq], want), (sq, toks[sq], want)


def test_batch_rejects_bad_arguments():
    from pyxis_b200._native import PyxisError
    m = SyntheticModel(SMALL, seed=1)
    dec = Decoder(m, qtype="int8", max_seq=16)
    with pytest.raises(PyxisError):
        dec.generate_batch(np.zeros((2, 16), np.int32), 2)  # 16 + 2 - 1 > max_seq
    with pytest.raises(PyxisError):
        dec.generate_batch(np.full((2, 4), SMALL.vocab, np.int32), 2)  # id out of range
    dec.close()
