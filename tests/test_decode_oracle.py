"""The oracle's greedy decode (C restatement of Model::generate, argmax sampling) on a tiny
random-init model: runs, is deterministic, and its layer math agrees with a float64 numpy
restatement of src/transformer.rs / attention.rs / ffn.rs to within f32 rounding."""
import numpy as np

import oracle
from pyxis_b200.model import ModelConfig, SyntheticModel

TINY = ModelConfig(hidden=128, n_layers=2, n_q_heads=4, n_kv_heads=2, head_dim=32, ffn=256, vocab=500,
                   rope_theta=10000.0)


def np_forward_tokens(cfg, m, qtype, prompt, n_new):
    """float64 numpy model over the oracle's own quantized weights (dequantized)."""
    def deq(name, in_f):
        vals = oracle.bf16_to_f32(m.bf16(name))
        if qtype == "int8":
            d, s = oracle.quantize_int8(vals, in_f)
            return oracle.dequantize(oracle.INT8, d, s, in_f, vals.size).astype(np.float64).reshape(-1, in_f)
        d, s = oracle.quantize_int4(vals, 32)
        return oracle.dequantize(oracle.INT4, d, s, 32, vals.size).astype(np.float64).reshape(-1, in_f)

    W = {}
    for l in range(cfg.n_layers):
        for k, i in (("q", cfg.hidden), ("k", cfg.hidden), ("v", cfg.hidden), ("o", cfg.q_dim), ("gate", cfg.hidden),
                     ("up", cfg.hidden), ("down", cfg.ffn)):
            W[l, k] = deq(f"layers.{l}.{k}", i)
    emb = oracle.bf16_to_f32(m.bf16("embed")).astype(np.float64).reshape(cfg.vocab, cfg.hidden)
    lm = deq("embed", cfg.hidden)
    hd, half = cfg.head_dim, cfg.head_dim // 2
    freq = 1.0 / cfg.rope_theta ** (np.arange(half) * 2 / hd)

    def rms(x):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + cfg.rms_eps)

    def rope(v, pos):
        v = v.reshape(-1, hd).copy()
        c, s = np.cos(pos * freq), np.sin(pos * freq)
        x0, x1 = v[:, :half].copy(), v[:, half:].copy()
        v[:, :half] = x0 * c - x1 * s
        v[:, half:] = x1 * c + x0 * s
        return v

    K = {l: [] for l in range(cfg.n_layers)}
    V = {l: [] for l in range(cfg.n_layers)}
    out = []
    toks = list(prompt)
    for step in range(len(prompt) + n_new - 1):
        x = emb[toks[step]].copy()
        for l in range(cfg.n_layers):
            h = rms(x)
            qv = (W[l, "q"] @ h).reshape(-1, hd)
            kv = (W[l, "k"] @ h).reshape(-1, hd)
            vv = (W[l, "v"] @ h).reshape(-1, hd)
            qv = rope(rms(qv), step)
            kv = rope(rms(kv), step)
            K[l].append(kv)
            V[l].append(vv)
            Ks, Vs = np.stack(K[l]), np.stack(V[l])
            att = np.empty_like(qv)
            for qh in range(cfg.n_q_heads):
                kh = qh * cfg.n_kv_heads // cfg.n_q_heads
                sc = Ks[:, kh] @ qv[qh] / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                p /= p.sum()
                att[qh] = p @ Vs[:, kh]
            x = x + W[l, "o"] @ att.ravel()
            h = rms(x)
            g, u = W[l, "gate"] @ h, W[l, "up"] @ h
            x = x + W[l, "down"] @ (g / (1 + np.exp(-g)) * u)
        logits = lm @ rms(x)
        nxt = int(np.argmax(logits))
        if step >= len(prompt) - 1:
            out.append(nxt)
            toks.append(nxt)
    return np.array(out)


def test_oracle_greedy_decode_matches_float64_model():
    m = SyntheticModel(TINY, seed=3)
    prompt = [1, 7, 42, 499, 0]
    for qt in ("int8", "int4"):
        a = oracle.greedy_decode(TINY, m.bf16, qt, prompt, 12, nthreads=2)
        b = oracle.greedy_decode(TINY, m.bf16, qt, prompt, 12, nthreads=5)
        assert np.array_equal(a, b)
        ref = np_forward_tokens(TINY, m, qt, prompt, 12)
        assert np.array_equal(a, ref), (qt, a, ref)
