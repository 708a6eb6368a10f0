"""Device-resident greedy decode (include/pyxis_decode.h) against the oracle's restatement of
Model::generate with argmax sampling (src/model.rs:245-285, src/output_head.rs:25-44): the
token streams must be identical."""
import json
import os

import numpy as np
import pytest

import oracle
from pyxis_b200.model import QWEN3_1_7B, Decoder, ModelConfig, SyntheticModel

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))

SMALL = ModelConfig(hidden=256, n_layers=3, n_q_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=2048,
                    rope_theta=10000.0)


@pytest.mark.parametrize("qtype", ["int8", "int4"])
def test_small_model_greedy_tokens_match_oracle(qtype):
    m = SyntheticModel(SMALL, seed=11)
    prompt = [5, 1999, 42, 7, 1024, 3]
    dec = Decoder(m, qtype=qtype, max_seq=64)
    toks, (t_prompt, t_decode) = dec.generate(prompt, 24)
    ref = oracle.greedy_decode(SMALL, m.bf16, qtype, prompt, 24)
    assert np.array_equal(toks, ref), (toks, ref)
    assert t_prompt > 0 and t_decode > 0
    toks2, _ = dec.generate(prompt, 24)  # the graph replays from a clean cache
    assert np.array_equal(toks2, ref)
    toks3, _ = dec.generate(prompt[:2], 5)
    assert np.array_equal(toks3, oracle.greedy_decode(SMALL, m.bf16, qtype, prompt[:2], 5))
    dec.close()


def test_qwen3_1p7b_shape_int8_greedy_matches_golden():
    """16 prompt ids, 128 greedy tokens on the random-init Qwen3-1.7B-shape int8 model; the
    expected stream comes from the oracle (tests/golden/make_decode_golden.py)."""
    with open(os.path.join(HERE, "golden", "decode_qwen3_1p7b_int8.json")) as f:
        g = json.load(f)
    m = SyntheticModel(QWEN3_1_7B, seed=g["seed"])
    dec = Decoder(m, qtype="int8", max_seq=160)
    toks, (t_prompt, t_decode) = dec.generate(g["prompt"], len(g["tokens"]))
    assert [int(t) for t in toks] == g["tokens"]
    dec.close()


def test_generate_rejects_bad_arguments():
    """Checked on the host before any launch: token ids outside the vocabulary (the embedding
    lookup's bounds assert, src/embedding.rs:18-24) and runs longer than the KV cache."""
    from pyxis_b200._native import PyxisError
    dec = Decoder(SyntheticModel(SMALL, seed=1), qtype="int8", max_seq=16)
    with pytest.raises(PyxisError):
        dec.generate([1, SMALL.vocab], 2)
    with pytest.raises(PyxisError):
        dec.generate([-1], 2)
    with pytest.raises(PyxisError):
        dec.generate(np.zeros(16, np.int32), 2)  # 16 + 2 - 1 > max_seq
    with pytest.raises(PyxisError):
        dec.generate(np.zeros(0, np.int32), 2)  # an empty prompt, as generate_batch rejects it
    toks, _ = dec.generate([1, 2], 2)  # the model still works after the rejections
    assert toks.shape == (2,)
    dec.close()
