"""Writes tests/golden/decode_qwen3_1p7b_int8.json: the greedy token stream of the oracle (the C
restatement of the reference's Model::generate with argmax sampling) on the random-init
Qwen3-1.7B-shape model -- hidden 2048, 28 layers, 16/8 heads, head_dim 128, FFN 6144, vocab
151936, RoPE theta 1e6, tied embeddings, int8 (one scale per row), seeded N(0, 0.02) bf16
weights, RMSNorm weights 1 -- for 16 seeded prompt ids and 128 new tokens.  The GPU decode test
compares the CUDA decoder's tokens with this file.  Runs on the CPU in about a minute."""
from __future__ import annotations

import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from pyxis_b200 import synth_tokens  # noqa: E402
from pyxis_b200.model import QWEN3_1_7B, SyntheticModel  # noqa: E402

OUT = os.path.join(HERE, "decode_qwen3_1p7b_int8.json")
SEED = 0x5EED
PROMPT_SEED = 0x9E0
N_PROMPT, N_NEW = 16, 128


def main():
    m = SyntheticModel(QWEN3_1_7B, SEED)
    prompt = synth_tokens(PROMPT_SEED, N_PROMPT, QWEN3_1_7B.vocab)
    t0 = time.time()
    toks = oracle.greedy_decode(QWEN3_1_7B, m.bf16, "int8", prompt, N_NEW)
    with open(OUT, "w") as f:
        json.dump({"model": "Qwen3-1.7B shape, random init, int8 per-row", "seed": SEED, "prompt_seed": PROMPT_SEED,
                   "prompt": [int(t) for t in prompt], "tokens": [int(t) for t in toks],
                   "generator": "tests/golden/make_decode_golden.py (oracle_greedy_decode)"}, f)
    print(f"wrote {OUT} in {time.time() - t0:.0f} s: {list(toks[:16])} ...", file=sys.stderr)


if __name__ == "__main__":
    main()
