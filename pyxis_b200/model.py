"""Device-resident greedy decode over quantized weights (include/pyxis_decode.h) and the seeded
random-init model it is benchmarked and tested on.

``SyntheticModel`` builds the Qwen3 layer stack of pyxis (src/model.rs:84-239) from seeded
N(0, 0.02) bf16 tensors with RMSNorm weights 1 -- the checkpoint-free stand-in for a real model.
The projections are quantised on the device by the reference's rules (src/model.rs:501-530: int8
one scale per row, int4 one per 32 values); the lm_head is the quantised tied embedding
(src/model.rs:219-224).  ``Decoder`` runs Model::generate with greedy sampling on the GPU.
"""
from __future__ import annotations

import ctypes as C
import zlib
from dataclasses import dataclass

import numpy as np

from . import Weights, _native, _require_cuda
from ._native import check

INT4_BLOCK_SIZE = 32


@dataclass(frozen=True)
class ModelConfig:
    """ModelConfig (src/model.rs:63-75)."""
    hidden: int = 2048
    n_layers: int = 28
    n_q_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 6144
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    qk_norm: bool = True

    @property
    def q_dim(self) -> int:
        return self.n_q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim


QWEN3_1_7B = ModelConfig()


class _CConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_layers", C.c_int), ("n_q_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("rms_eps", C.c_float),
                ("rope_theta", C.c_float), ("max_seq", C.c_int)]


def tensor_seed(base: int, name: str) -> int:
    return (base * 0x100000001B3 ^ zlib.crc32(name.encode())) & 0xFFFFFFFFFFFFFFFF


class SyntheticModel:
    """Seeded bf16 tensors of one model: ``bf16(name)`` -> np.uint16 bits, generated on demand
    (include/pyxis_synth.h), so the oracle and the device see the same values."""

    def __init__(self, cfg: ModelConfig, seed: int = 0x5EED, head_norm_value: float = 1.0):
        """``head_norm_value``: the QK-RMSNorm weight (1 like the other norms; larger values
        sharpen the attention, as trained QK-norm weights do)."""
        self.cfg = cfg
        self.seed = seed
        self.head_norm_value = head_norm_value

    def shape(self, name: str) -> tuple[int, int]:
        c = self.cfg
        kind = name.split(".")[-1]
        return {"q": (c.q_dim, c.hidden), "k": (c.kv_dim, c.hidden), "v": (c.kv_dim, c.hidden),
                "o": (c.hidden, c.q_dim), "gate": (c.ffn, c.hidden), "up": (c.ffn, c.hidden),
                "down": (c.hidden, c.ffn), "embed": (c.vocab, c.hidden)}[kind]

    def bf16(self, name: str) -> np.ndarray:
        from . import synth_normal_bf16
        r, k = self.shape(name)
        return synth_normal_bf16(tensor_seed(self.seed, name), r * k, 0.02)

    def norm(self) -> np.ndarray:
        return np.ones(self.cfg.hidden, np.float32)

    def head_norm(self):
        return np.full(self.cfg.head_dim, self.head_norm_value, np.float32) if self.cfg.qk_norm else None


def _quantize(bits: np.ndarray, qtype: str, in_features: int, device: int):
    """quantize_weights' block policy (src/model.rs:520-530) applied on the device."""
    import torch
    t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(f"cuda:{device}")
    if qtype == "int8":
        return Weights.quantize_int8(t, in_features, device=device)
    return Weights.quantize_int4(t, INT4_BLOCK_SIZE, device=device)


class Decoder:
    """Model::generate (src/model.rs:245-285) with temperature-0 sampling, on one GPU."""

    def __init__(self, model: SyntheticModel, qtype: str = "int8", max_seq: int = 256, device: int = 0,
                 vocab_parallel=None, full_head: bool = True):
        """``vocab_parallel``: a ``pyxis_b200.dist.Comm`` -- generate_batch then runs this rank's
        sequences with the lm_head split by vocabulary rows over the communicator's ranks (this
        rank quantises only its rows).  ``full_head`` False leaves the full lm_head out (generate
        then fails; generate_batch needs the vocab-parallel head)."""
        cfg = model.cfg
        self.cfg = cfg
        self.ctx = _require_cuda(device)
        L = _native.lib()
        cc = _CConfig(cfg.hidden, cfg.n_layers, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                      cfg.rms_eps, cfg.rope_theta, max_seq)
        h = C.c_void_p()
        check(L.pyxis_cuda_model_create(self.ctx.handle, C.addressof(cc), C.byref(h)))
        self.handle = h
        self.max_seq = max_seq
        self._keep = []
        ones = model.norm()
        hn = model.head_norm()
        fp = C.POINTER(C.c_float)

        def p(a):
            return a.ctypes.data_as(fp) if a is not None else None

        for layer in range(cfg.n_layers):
            pre = f"layers.{layer}."
            qkv = np.concatenate([model.bf16(pre + "q"), model.bf16(pre + "k"), model.bf16(pre + "v")])
            wqkv = _quantize(qkv, qtype, cfg.hidden, device)
            wo = _quantize(model.bf16(pre + "o"), qtype, cfg.q_dim, device)
            wgu = _quantize(np.concatenate([model.bf16(pre + "gate"), model.bf16(pre + "up")]), qtype, cfg.hidden,
                            device)
            wd = _quantize(model.bf16(pre + "down"), qtype, cfg.ffn, device)
            self._keep += [wqkv, wo, wgu, wd]
            check(L.pyxis_cuda_model_set_layer(self.handle, layer, wqkv.handle, wo.handle, wgu.handle, wd.handle,
                                               p(ones), p(ones), p(hn), p(hn)))
        emb = model.bf16("embed")
        lm = _quantize(emb, qtype, cfg.hidden, device) if full_head else None
        if lm is not None:
            self._keep.append(lm)
        check(L.pyxis_cuda_model_set_head(self.handle, emb.ctypes.data_as(C.POINTER(C.c_uint16)),
                                          lm.handle if lm is not None else None, p(ones)))
        self.vocab_parallel = None
        if vocab_parallel is not None:
            from .dist import bits_rows, shard_range
            lo, hi = shard_range(cfg.vocab, vocab_parallel.rank, vocab_parallel.world)
            shard = _quantize(bits_rows(emb, cfg.hidden, lo, hi), qtype, cfg.hidden, device)
            self._keep.append(shard)
            check(L.pyxis_cuda_model_set_vocab_parallel(self.handle, vocab_parallel.handle, shard.handle, lo, hi - lo))
            self.vocab_parallel = vocab_parallel
            self._shard = (shard, lo, hi)

    def set_vocab_parallel(self, on: bool) -> None:
        """Switch generate_batch between the vocab-parallel head and this rank's full head."""
        L = _native.lib()
        if on:
            shard, lo, hi = self._shard
            check(L.pyxis_cuda_model_set_vocab_parallel(self.handle, self.vocab_parallel.handle, shard.handle, lo,
                                                        hi - lo))
        else:
            check(L.pyxis_cuda_model_set_vocab_parallel(self.handle, None, None, 0, 0))

    def prefill_hidden(self, prompts) -> np.ndarray:
        """The batched prefill's final-norm hidden state of every prompt's last position
        (pyxis_cuda_model_prefill_hidden): prompts [n_seq, n_prompt] -> [n_seq, hidden] f32."""
        pr = np.ascontiguousarray(np.asarray(prompts, np.int32))
        out = np.empty((pr.shape[0], self.cfg.hidden), np.float32)
        check(_native.lib().pyxis_cuda_model_prefill_hidden(self.handle, pr.ctypes.data_as(C.c_void_p), pr.shape[0],
                                                            pr.shape[1], out.ctypes.data_as(C.c_void_p)))
        return out

    def generate(self, prompt, n_new: int):
        """Returns (tokens [n_new], (prompt_ms, decode_ms)) -- device time of the two phases."""
        pr = np.ascontiguousarray(np.asarray(prompt, np.int32))
        out = np.empty(n_new, np.int32)
        t = (C.c_float * 2)()
        check(_native.lib().pyxis_cuda_model_generate(self.handle, pr.ctypes.data_as(C.c_void_p), pr.size, n_new,
                                                      out.ctypes.data_as(C.c_void_p), t))
        return out, (t[0], t[1])

    def generate_batch(self, prompts, n_new: int):
        """Greedy generation for several prompts of one length side by side
        (pyxis_cuda_model_generate_batch): prompts [n_seq, n_prompt] ids -> (tokens [n_seq, n_new],
        (prefill_ms, decode_ms)), the device time of the prefill through the first generated tokens
        and of the remaining steps."""
        pr = np.ascontiguousarray(np.asarray(prompts, np.int32))
        if pr.ndim != 2:
            raise ValueError("prompts must be [n_seq, n_prompt]")
        out = np.empty((pr.shape[0], n_new), np.int32)
        t = (C.c_float * 2)()
        check(_native.lib().pyxis_cuda_model_generate_batch(self.handle, pr.ctypes.data_as(C.c_void_p), pr.shape[0],
                                                            pr.shape[1], n_new, out.ctypes.data_as(C.c_void_p), t))
        return out, (t[0], t[1])

    def close(self):
        if self.handle:
            _native.lib().pyxis_cuda_model_free(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
