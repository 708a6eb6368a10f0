"""The reference's own unit tests of the decode stack around matmul, re-run on the oracle that
the CUDA decode loop's greedy tokens are checked against: RoPE, softmax, Attention::forward
(causal mask, GQA, q_dim > hidden, QK-norm, incremental KV cache == full), Ffn::forward,
RmsNorm, TransformerBlock / Transformer::forward.  Each test restates the cited reference test's
setup and assertions, with its tolerance (1e-5 absolute)."""
import math

import numpy as np

import oracle

TOL = 1e-5


def close(a, b, tol=TOL):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert np.all(np.abs(a - b) < tol), (a, b)


def identity(n):
    return np.eye(n, dtype=np.float32)


def zeros(r, c):
    return np.zeros((r, c), np.float32)


def attention(hidden, nq, nkv, hd, wq, wk, wv, wo, q_norm=True, k_norm=True, theta=10.0):
    """Attention::new(wq, wk, wv, wo, q_norm, k_norm, hidden, nq, nkv, hd, theta); True = unit
    head norm (RmsNorm of ones, eps 1e-6), None = no QK-norm, else the weight vector."""
    def norm(v):
        return np.ones(hd, np.float32) if v is True else v
    return oracle.Layers(hidden, nq, nkv, hd, wq, wk, wv, wo, q_norm=norm(q_norm), k_norm=norm(k_norm), theta=theta)


# ---- src/attention.rs ------------------------------------------------------------------------
def test_apply_rope_at_position_zero_is_identity():
    """src/attention.rs:219-225"""
    v = np.arange(1, 9, dtype=np.float32)
    close(oracle.apply_rope(v, 4, 0, 10.0), v)


def test_softmax_produces_valid_distribution():
    """src/attention.rs:243-251"""
    s = oracle.softmax([1.0, 2.0, 3.0])
    assert abs(float(s.sum(dtype=np.float32)) - 1.0) < TOL
    assert s[0] < s[1] < s[2]


def test_softmax_handles_large_values():
    """src/attention.rs:254-261"""
    s = oracle.softmax([1000.0, 1001.0, 1002.0])
    assert np.all(np.isfinite(s)) and abs(float(s.sum(dtype=np.float32)) - 1.0) < TOL


def test_forward_single_token_identity_weights():
    """src/attention.rs:264-285: identity projections, one token: the output is the input."""
    a = attention(8, 2, 2, 4, identity(8), identity(8), identity(8), identity(8))
    x = np.arange(1, 9, dtype=np.float32)
    close(a.attention(x, 1, 0, a.cache()), x)


def test_forward_causal_mask():
    """src/attention.rs:288-315: zero q/k projections (uniform scores), identity v/o: position 0
    sees only itself, position 1 the mean of both."""
    a = attention(8, 2, 2, 4, zeros(8, 8), zeros(8, 8), identity(8), identity(8))
    x = np.array([2, 4, 6, 8, 10, 12, 14, 16, 4, 6, 8, 10, 12, 14, 16, 18], np.float32)
    out = a.attention(x, 2, 0, a.cache())
    close(out[:8], x[:8])
    close(out[8:], [3, 5, 7, 9, 11, 13, 15, 17])


def test_forward_with_hidden_dim_smaller_than_q_dim():
    """src/attention.rs:318-353: hidden 4, q_dim = kv_dim = 8."""
    hidden, nq, nkv, hd = 4, 2, 2, 4
    q_dim, kv_dim = nq * hd, nkv * hd
    wv, wo = zeros(kv_dim, hidden), zeros(hidden, q_dim)
    for d in range(hidden):
        wv[d, d] = 1.0
        wo[d, d] = 1.0
    a = attention(hidden, nq, nkv, hd, zeros(q_dim, hidden), zeros(kv_dim, hidden), wv, wo)
    out = a.attention(np.arange(1, 9, dtype=np.float32), 2, 0, a.cache())
    assert out.size == 2 * hidden
    close(out, [1, 2, 3, 4, 3, 4, 5, 6])


def test_forward_gqa_shares_kv_heads():
    """src/attention.rs:356-378: 4 query heads over 2 KV heads, three positions."""
    a = attention(16, 4, 2, 4, zeros(16, 16), zeros(8, 16), zeros(8, 16), zeros(16, 16))
    out = a.attention(np.ones(16 * 3, np.float32), 3, 0, a.cache())
    assert out.size == 16 * 3


def test_forward_without_qk_norm():
    """src/attention.rs:381-403"""
    a = attention(8, 2, 2, 4, identity(8), identity(8), identity(8), identity(8), q_norm=None, k_norm=None)
    out = a.attention([1.0, 0.5, -1.0, 2.0, 0.25, -0.5, 1.5, -2.0], 1, 0, a.cache())
    assert out.size == 8 and np.all(np.isfinite(out))


def test_forward_with_kv_cache_incremental():
    """src/attention.rs:406-434: two positions then one through the cache equals three at once."""
    a = attention(8, 2, 2, 4, identity(8), identity(8), identity(8), identity(8))
    x = np.array([1.0, 0.5, -1.0, 2.0, 0.25, -0.5, 1.5, -2.0, -0.75, 1.25, 0.0, 0.5, 2.0, -1.0, 0.75, -0.25,
                  0.3, -1.5, 1.2, 0.8, -0.4, 2.5, -0.9, 1.1], np.float32)
    full = a.attention(x, 3, 0, a.cache())
    inc = a.cache()
    a.attention(x[:16], 2, 0, inc)
    close(a.attention(x[16:], 1, 2, inc), full[16:])


def test_qk_norm_is_applied_per_head():
    """src/attention.rs:437-483: a larger q_norm weight sharpens the scores, and the cached key is
    the per-head RMS-normed, k_norm-weighted, rotated projection."""
    hd = 4
    x = np.array([1, 0, 0, 0, 0, 0, 0, 0, 3, 1, 0, 0, 0, 0, 0, 0], np.float32)
    k_norm = np.array([1, 2, 3, 4], np.float32)
    base = attention(8, 2, 2, hd, identity(8), identity(8), identity(8), identity(8), q_norm=np.ones(hd, np.float32),
                     k_norm=k_norm)
    scaled = attention(8, 2, 2, hd, identity(8), identity(8), identity(8), identity(8),
                       q_norm=np.full(hd, 2.0, np.float32), k_norm=k_norm)
    base_out = base.attention(x, 2, 0, base.cache())
    cache = scaled.cache()
    scaled_out = scaled.attention(x, 2, 0, cache)
    assert scaled_out[8] > base_out[8] + 0.1
    rms = np.sqrt(np.float32((3.0 * 3.0 + 1.0) / hd) + np.float32(1e-6), dtype=np.float32)
    norm_0, norm_2 = np.float32(3.0) / rms, np.float32(0.0) / rms * np.float32(3.0)
    expected_first = norm_0 * np.float32(math.cos(1.0)) - norm_2 * np.float32(math.sin(1.0))
    assert abs(float(cache.keys()[8]) - float(expected_first)) < TOL


# ---- src/ffn.rs, src/rmsnorm.rs --------------------------------------------------------------
def test_silu_at_zero_is_zero():
    """src/ffn.rs:76-78"""
    assert abs(oracle.silu(0.0)) < TOL


def test_ffn_forward_with_known_weights():
    """src/ffn.rs:91-102: gate [3,2], up [3,2], down [2,3], hidden 2, intermediate 3."""
    f = oracle.Layers(2, 1, 1, 2, None, None, None, None, ffn=3,
                      wgate=[1.0, 0.0, 0.0, 1.0, 1.0, 1.0], wup=[2.0, 0.0, 0.0, -1.0, 0.5, 0.5],
                      wdown=[1.0, 0.0, 0.0, 0.0, 1.0, 1.0])
    close(f.ffn([1.0, 2.0]), [1.4621172, 0.7633953])


def test_rmsnorm_normalizes_uniform_vector():
    """src/rmsnorm.rs:35-44"""
    close(oracle.rmsnorm([1.0, 1.0, 1.0, 1.0], [1.0, 1.0, 1.0, 1.0], 1e-6), [1.0, 1.0, 1.0, 1.0])


# ---- src/transformer.rs (hidden 4, 2 + 2 heads of 2, intermediate 8, eps 1e-6) ----------------
H, NQ, NKV, HD, FFN = 4, 2, 2, 2, 8


def block(attn_weight, n_layers=1):
    w = attn_weight(H)
    return oracle.Layers(H, NQ, NKV, HD, w, w, w, w, q_norm=np.ones(HD, np.float32), k_norm=np.ones(HD, np.float32),
                         ffn=FFN, wgate=zeros(FFN, H), wup=zeros(FFN, H), wdown=zeros(H, FFN), n_layers=n_layers)


def rms_norm_values(x):
    x = np.asarray(x, np.float32)
    ms = np.float32(0.0)
    for v in x:
        ms = np.float32(ms + v * v)
    factor = np.float32(1.0) / np.sqrt(np.float32(ms / np.float32(x.size)) + np.float32(1e-6), dtype=np.float32)
    return x * factor


def test_transformer_block_forward_applies_residual_connections():
    """src/transformer.rs:190-199: a block of zero weights leaves x unchanged."""
    b = block(lambda n: zeros(n, n))
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    close(b.block(x, 1, 0, b.cache()), x)


def test_transformer_block_forward_seq_len_2():
    """src/transformer.rs:202-211"""
    b = block(lambda n: zeros(n, n))
    x = np.array([1.0, 2.0, 3.0, 4.0, -1.0, -2.0, -3.0, -4.0], np.float32)
    close(b.block(x, 2, 0, b.cache()), x)


def test_transformer_forward_stacks_blocks():
    """src/transformer.rs:214-223: two zero blocks, then the final norm."""
    t = block(lambda n: zeros(n, n), n_layers=2)
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    close(t.transformer(x, 1, 0, t.cache()), rms_norm_values(x))


def test_transformer_forward_with_identity_attention():
    """src/transformer.rs:226-243: identity attention adds the normed input to the residual."""
    b = block(identity)
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    out = b.block(x, 1, 0, b.cache())
    assert not np.array_equal(out, x)
    close(out, x + rms_norm_values(x))
