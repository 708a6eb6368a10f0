"""oracle -- ctypes binding of the C restatement of the reference's CPU path (liboracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.  Imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / --impl reference legs, never by the
product package pyxis_b200.  See pyxis_oracle.h for the reference function each entry restates.
"""
from __future__ import annotations

import ctypes as C
import os
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

F32, BF16, INT8, INT4 = 0, 1, 2, 3
_vp, _sz = C.c_void_p, C.c_size_t
_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from . import build as _b
            _b.build()
        L = C.CDLL(LIB_PATH)
        L.oracle_quantize_int8.argtypes = [_vp, _sz, _sz, _vp, _vp]
        L.oracle_quantize_int4.argtypes = [_vp, _sz, _sz, _vp, _vp]
        L.oracle_bf16_to_f32.argtypes = [_vp, _sz, _vp]
        L.oracle_dequantize_int8.argtypes = [_vp, _vp, _sz, _sz, _vp]
        L.oracle_dequantize_int4.argtypes = [_vp, _vp, _sz, _sz, _vp]
        L.oracle_q8_0_to_int8.argtypes = [_vp, _sz, _vp, _vp]
        L.oracle_f16_to_f32.argtypes = [C.c_uint16]
        L.oracle_f16_to_f32.restype = C.c_float
        for n in ("oracle_dot_int8", "oracle_dot_int4"):
            getattr(L, n).argtypes = [_vp, _vp, _vp, _sz, _sz, _sz]
            getattr(L, n).restype = C.c_float
        L.oracle_dot_f32.argtypes = [_vp, _vp, _sz]
        L.oracle_dot_f32.restype = C.c_float
        L.oracle_matmul.argtypes = [_vp, C.c_int, _vp, _vp, _sz, _sz, _sz, _vp, C.c_int]
        L.oracle_matmul_batch.argtypes = [_vp, _sz, C.c_int, _vp, _vp, _sz, _sz, _sz, _vp, C.c_int]
        L.oracle_argmax.argtypes = [_vp, _sz]
        L.oracle_argmax.restype = _sz
        L.oracle_rmsnorm.argtypes = [_vp, _vp, _sz, C.c_float]
        L.oracle_apply_rope.argtypes = [_vp, _sz, _sz, _sz, C.c_float]
        L.oracle_softmax.argtypes = [_vp, _sz]
        L.oracle_silu.argtypes = [C.c_float]
        L.oracle_silu.restype = C.c_float
        L.oracle_greedy_decode.argtypes = [_vp, _vp, _sz, _sz, _vp, C.c_int]
        L.oracle_greedy_decode.restype = C.c_int
        L.oracle_prefill_hidden.argtypes = [_vp, _vp, _sz, _vp, C.c_int]
        L.oracle_prefill_hidden.restype = C.c_int
        L.oracle_kv_new.argtypes = [_vp, _sz]
        L.oracle_kv_new.restype = _vp
        L.oracle_kv_free.argtypes = [_vp]
        L.oracle_kv_len.argtypes = [_vp, _sz]
        L.oracle_kv_len.restype = _sz
        L.oracle_kv_keys.argtypes = [_vp, _sz]
        L.oracle_kv_keys.restype = C.POINTER(C.c_float)
        L.oracle_attention_forward.argtypes = [_vp, _sz, _vp, _sz, _sz, _vp, _vp, C.c_int]
        L.oracle_attention_forward.restype = C.c_int
        L.oracle_ffn_forward.argtypes = [_vp, _sz, _vp, _vp, C.c_int]
        L.oracle_ffn_forward.restype = C.c_int
        L.oracle_block_forward.argtypes = [_vp, _sz, _vp, _sz, _sz, _vp, C.c_int]
        L.oracle_block_forward.restype = C.c_int
        L.oracle_transformer_forward.argtypes = [_vp, _vp, _sz, _sz, _vp, C.c_int]
        L.oracle_transformer_forward.restype = C.c_int
        L.oracle_num_cpus.restype = C.c_int
        L.pyxis_synth_normal_f32.argtypes = [C.c_uint64, _sz, C.c_float, _vp]
        L.pyxis_synth_normal_bf16.argtypes = [C.c_uint64, _sz, C.c_float, _vp]
        L.pyxis_synth_tokens.argtypes = [C.c_uint64, _sz, C.c_uint32, _vp]
        for n in ("pyxis_synth_normal_f32", "pyxis_synth_normal_bf16", "pyxis_synth_tokens"):
            getattr(L, n).restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray) -> C.c_void_p:
    return a.ctypes.data_as(C.c_void_p)


# The seeded generator of include/pyxis_synth.h (the same source as the CUDA library's copy), for
# the CPU baseline, which must not load the CUDA library.
def synth_normal_f32(seed: int, n: int, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().pyxis_synth_normal_f32(seed, n, sigma, _p(out))
    return out


def synth_normal_bf16(seed: int, n: int, sigma: float = 0.02) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().pyxis_synth_normal_bf16(seed, n, sigma, _p(out))
    return out


def synth_tokens(seed: int, n: int, vocab: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().pyxis_synth_tokens(seed, n, vocab, _p(out))
    return out


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def num_cpus() -> int:
    return lib().oracle_num_cpus()


def quantize_int8(values, block_size: int):
    """Weights::quantize_int8 (src/weights.rs:94-118) -> (data i8 [n], scales f32)."""
    v = _f32(values)
    n = v.size
    data = np.empty(n, np.int8)
    scales = np.empty((n + block_size - 1) // block_size, np.float32)
    lib().oracle_quantize_int8(_p(v), n, block_size, _p(data), _p(scales))
    return data, scales


def quantize_int4(values, block_size: int):
    """Weights::quantize_int4 (src/weights.rs:120-151) -> (data u8 [ceil(n/2)], scales f32)."""
    v = _f32(values)
    n = v.size
    data = np.empty((n + 1) // 2, np.uint8)
    scales = np.empty((n + block_size - 1) // block_size, np.float32)
    lib().oracle_quantize_int4(_p(v), n, block_size, _p(data), _p(scales))
    return data, scales


def bf16_to_f32(bits) -> np.ndarray:
    b = np.ascontiguousarray(np.asarray(bits, dtype=np.uint16))
    out = np.empty(b.size, np.float32)
    lib().oracle_bf16_to_f32(_p(b), b.size, _p(out))
    return out


def dequantize(kind: int, data, scales, block_size: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    d = np.ascontiguousarray(data)
    s = _f32(scales)
    if kind == INT8:
        lib().oracle_dequantize_int8(_p(d), _p(s), block_size, n, _p(out))
    else:
        lib().oracle_dequantize_int4(_p(d), _p(s), block_size, n, _p(out))
    return out


def q8_0_to_int8(blocks: bytes, n: int):
    """read_q8_0_weights (src/gguf.rs:245-271) -> (data i8 [n], scales f32 [ceil(n/32)])."""
    b = np.frombuffer(blocks, dtype=np.uint8).copy()
    data = np.empty(n, np.int8)
    scales = np.empty((n + 31) // 32, np.float32)
    lib().oracle_q8_0_to_int8(_p(b), n, _p(data), _p(scales))
    return data, scales


def matmul(x, kind: int, data, scales, block_size: int, out_features: int, in_features: int,
           nthreads: int = 0) -> np.ndarray:
    """matmul (src/matmul.rs:21-97), rows over nthreads threads (0: all cores)."""
    X = _f32(x)
    d = np.ascontiguousarray(data)
    s = _f32(scales) if scales is not None else np.zeros(1, np.float32)
    M = X.size // in_features if in_features else 1
    Y = np.empty((M, out_features), np.float32)
    rc = lib().oracle_matmul_batch(_p(X), M, kind, _p(d), _p(s), block_size, out_features, in_features, _p(Y),
                                   nthreads)
    if rc:
        raise ValueError("oracle_matmul: shape error")
    return Y[0] if np.asarray(x).ndim == 1 else Y


def argmax(values) -> int:
    v = _f32(values)
    return int(lib().oracle_argmax(_p(v), v.size))


def rmsnorm(x, weight, eps: float) -> np.ndarray:
    v = _f32(x).copy()
    w = _f32(weight)
    lib().oracle_rmsnorm(_p(v), _p(w), v.size, eps)
    return v


def apply_rope(x, head_dim: int, pos: int, theta: float) -> np.ndarray:
    v = _f32(x).copy()
    lib().oracle_apply_rope(_p(v), v.size, head_dim, pos, theta)
    return v


def softmax(x) -> np.ndarray:
    v = _f32(x).copy()
    lib().oracle_softmax(_p(v), v.size)
    return v


def silu(x: float) -> float:
    return float(lib().oracle_silu(x))


# ---- greedy decode (oracle_greedy_decode: Model::generate with argmax sampling) ----------------
class OWeights(C.Structure):
    _fields_ = [("kind", C.c_int), ("data", _vp), ("scales", _vp), ("block_size", _sz)]


class OModel(C.Structure):
    _fields_ = [("hidden", _sz), ("n_layers", _sz), ("n_q_heads", _sz), ("n_kv_heads", _sz), ("head_dim", _sz),
                ("ffn", _sz), ("vocab", _sz), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("embedding", _vp), ("input_norm", _vp), ("post_norm", _vp), ("q_norm", _vp), ("k_norm", _vp),
                ("wq", _vp), ("wk", _vp), ("wv", _vp), ("wo", _vp), ("wgate", _vp), ("wup", _vp), ("wdown", _vp),
                ("final_norm", _vp), ("lm_head", OWeights)]


def _model(cfg, bf16, qtype: str, head_norm=None):
    """The oracle_model of a config whose tensors ``bf16(name)`` returns (np.uint16 bits; names
    ``layers.{l}.{q,k,v,o,gate,up,down}`` and ``embed``), quantised by the reference's policy
    (src/model.rs:520-530: int8 one scale per row, int4 one per 32), tied lm_head, RMSNorm
    weights 1, QK-norm when cfg.qk_norm with weights ``head_norm`` (default 1).  Returns (model,
    arrays to keep alive)."""
    keep = []

    def q(bits, in_features):
        vals = bf16_to_f32(bits)
        if qtype == "int8":
            d, s = quantize_int8(vals, in_features)
            w = OWeights(INT8, d.ctypes.data, s.ctypes.data, in_features)
        else:
            d, s = quantize_int4(vals, 32)
            w = OWeights(INT4, d.ctypes.data, s.ctypes.data, 32)
        keep.extend([d, s])
        return w

    nl = cfg.n_layers
    ws = {k: (OWeights * nl)() for k in ("q", "k", "v", "o", "gate", "up", "down")}
    ins = {"q": cfg.hidden, "k": cfg.hidden, "v": cfg.hidden, "o": cfg.q_dim, "gate": cfg.hidden,
           "up": cfg.hidden, "down": cfg.ffn}
    for l in range(nl):
        for k in ws:
            ws[k][l] = q(bf16(f"layers.{l}.{k}"), ins[k])
    ones = np.ones(cfg.hidden, np.float32)
    hones = (np.ones(cfg.head_dim, np.float32) if head_norm is None
             else np.ascontiguousarray(np.asarray(head_norm, np.float32).reshape(cfg.head_dim)))
    norm_arr = (_vp * nl)(*([ones.ctypes.data] * nl))
    hn_arr = (_vp * nl)(*([hones.ctypes.data if cfg.qk_norm else None] * nl))
    emb_bits = bf16("embed")
    emb = bf16_to_f32(emb_bits)
    lm = q(emb_bits, cfg.hidden)
    m = OModel(cfg.hidden, nl, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab, cfg.rms_eps,
               cfg.rope_theta, emb.ctypes.data, C.addressof(norm_arr), C.addressof(norm_arr), C.addressof(hn_arr),
               C.addressof(hn_arr), C.addressof(ws["q"]), C.addressof(ws["k"]), C.addressof(ws["v"]),
               C.addressof(ws["o"]), C.addressof(ws["gate"]), C.addressof(ws["up"]), C.addressof(ws["down"]),
               ones.ctypes.data, lm)
    keep += [ws, ones, hones, norm_arr, hn_arr, emb]
    return m, keep


def greedy_decode(cfg, bf16, qtype: str, prompt, n_new: int, nthreads: int = 0, timing=None, head_norm=None):
    """Greedy tokens (Model::generate with argmax sampling, src/model.rs:245-285) of the model
    ``_model`` builds.  A list passed as ``timing`` receives the seconds of the generation alone
    (the len(prompt) + n_new - 1 forward passes, without the packing)."""
    m, keep = _model(cfg, bf16, qtype, head_norm)
    pr = np.ascontiguousarray(np.asarray(prompt, np.int32))
    out = np.empty(n_new, np.int32)
    t0 = time.perf_counter()
    rc = lib().oracle_greedy_decode(C.addressof(m), pr.ctypes.data, pr.size, n_new, out.ctypes.data, nthreads)
    if timing is not None:
        timing.append(time.perf_counter() - t0)
    if rc:
        raise RuntimeError("oracle_greedy_decode failed")
    return out


def prefill_hidden(cfg, bf16, qtype: str, prompt, nthreads: int = 0, head_norm=None) -> np.ndarray:
    """The final-norm hidden state [hidden] of the prompt's last position: what the first greedy
    token's lm_head product reads."""
    m, keep = _model(cfg, bf16, qtype, head_norm)
    pr = np.ascontiguousarray(np.asarray(prompt, np.int32))
    out = np.empty(cfg.hidden, np.float32)
    if lib().oracle_prefill_hidden(C.addressof(m), pr.ctypes.data, pr.size, out.ctypes.data, nthreads):
        raise RuntimeError("oracle_prefill_hidden failed")
    return out


# ---- layers with f32 weights, as the reference's unit tests build them -------------------------
class Layers:
    """n_layers identical transformer layers with f32 weights (Weights::F32): wq [q_dim, hidden],
    wk / wv [kv_dim, hidden], wo [hidden, q_dim], QK-norm weights [head_dim] or None, FFN
    wgate / wup [ffn, hidden] and wdown [hidden, ffn], RMSNorm weights [hidden] (1 when omitted),
    every norm with eps.  Drives oracle_attention_forward / _ffn_ / _block_ / _transformer_."""

    def __init__(self, hidden, n_q_heads, n_kv_heads, head_dim, wq, wk, wv, wo, q_norm=None, k_norm=None,
                 theta=10.0, eps=1e-6, ffn=0, wgate=None, wup=None, wdown=None, n_layers=1):
        self._keep = []
        self.hidden = hidden

        def arr(a):
            a = np.ascontiguousarray(np.asarray(a, np.float32).ravel())
            self._keep.append(a)
            return a

        def weights(a):
            if a is None:
                return OWeights(F32, None, None, 1)
            return OWeights(F32, arr(a).ctypes.data, None, 1)

        def per_layer(w):
            return (OWeights * n_layers)(*([weights(w)] * n_layers))

        def norm_ptrs(v):
            p = None if v is None else arr(v).ctypes.data
            return (_vp * n_layers)(*([p] * n_layers))

        ones = arr(np.ones(hidden, np.float32))
        self._tabs = [per_layer(w) for w in (wq, wk, wv, wo, wgate, wup, wdown)]
        self._norms = [norm_ptrs(np.ones(hidden, np.float32)), norm_ptrs(np.ones(hidden, np.float32)),
                       norm_ptrs(q_norm), norm_ptrs(k_norm)]
        self.m = OModel(hidden, n_layers, n_q_heads, n_kv_heads, head_dim, ffn, 0, eps, theta, None,
                        C.addressof(self._norms[0]), C.addressof(self._norms[1]), C.addressof(self._norms[2]),
                        C.addressof(self._norms[3]), *[C.addressof(t) for t in self._tabs], ones.ctypes.data,
                        OWeights(F32, None, None, 1))
        self.kv_dim = n_kv_heads * head_dim

    def cache(self, max_len=64):
        return _KV(self, max_len)

    def attention(self, x, seq_len, start_pos, kv, layer=0):
        x = _f32(x).copy()
        out = np.empty(seq_len * self.hidden, np.float32)
        if lib().oracle_attention_forward(C.byref(self.m), layer, _p(x), seq_len, start_pos, kv.h, _p(out), 1):
            raise RuntimeError("oracle_attention_forward failed")
        return out

    def ffn(self, x, layer=0):
        x = _f32(x).copy()
        out = np.empty(self.hidden, np.float32)
        if lib().oracle_ffn_forward(C.byref(self.m), layer, _p(x), _p(out), 1):
            raise RuntimeError("oracle_ffn_forward failed")
        return out

    def block(self, x, seq_len, start_pos, kv, layer=0):
        x = _f32(x).copy()
        if lib().oracle_block_forward(C.byref(self.m), layer, _p(x), seq_len, start_pos, kv.h, 1):
            raise RuntimeError("oracle_block_forward failed")
        return x

    def transformer(self, x, seq_len, start_pos, kv):
        x = _f32(x).copy()
        if lib().oracle_transformer_forward(C.byref(self.m), _p(x), seq_len, start_pos, kv.h, 1):
            raise RuntimeError("oracle_transformer_forward failed")
        return x


class _KV:
    """KvCache for a Layers model (oracle_kv)."""

    def __init__(self, layers: Layers, max_len: int):
        self.layers = layers
        self.max_len = max_len
        self.h = lib().oracle_kv_new(C.byref(layers.m), max_len)
        if not self.h:
            raise MemoryError("oracle_kv_new")

    def __len__(self):
        return int(lib().oracle_kv_len(self.h, 0))

    def keys(self, layer=0) -> np.ndarray:
        """The cached keys so far, [len * kv_dim] (LayerCache::keys)."""
        n = int(lib().oracle_kv_len(self.h, layer)) * self.layers.kv_dim
        return np.ctypeslib.as_array(lib().oracle_kv_keys(self.h, layer), shape=(max(n, 1),))[:n].copy()

    def __del__(self):  # pragma: no cover
        if getattr(self, "h", None):
            lib().oracle_kv_free(self.h)
            self.h = None
