"""The C-ABI library without a GPU: it loads, exports every symbol include/*.h declares, and its
host-side checks answer without touching a device."""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

from pyxis_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(pyxis_\w+)\s*\(", text):
            syms.add(m.group(1))
    return sorted(syms)


def test_headers_declare_the_boundary():
    syms = declared_symbols()
    for s in ("pyxis_cuda_init", "pyxis_cuda_quantize", "pyxis_cuda_matmul", "pyxis_cuda_matmul_dev",
              "pyxis_cuda_weights_upload", "pyxis_cuda_weights_download", "pyxis_cuda_argmax_dev"):
        assert s in syms


@pytest.mark.parametrize("sym", declared_symbols())
def test_library_exports_declared_symbol(sym):
    L = C.CDLL(_native.LIB_PATH)
    assert hasattr(L, sym), f"{sym} declared in include/*.h but not exported"
    assert sym in _native.SIGNATURES, f"{sym} has no ctypes signature in pyxis_b200/_native.py"


def test_abi_version():
    assert _native.lib().pyxis_cuda_abi_version() >> 16 == 1


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device path")
def test_init_without_device_reports_enodev():
    L = _native.lib()
    h = C.c_void_p()
    rc = L.pyxis_cuda_init(0, C.byref(h))
    assert rc == _native.PYXIS_ENODEV
    assert L.pyxis_cuda_last_error()
    import pyxis_b200
    assert pyxis_b200.get_cuda(0) is None
    with pytest.raises(pyxis_b200.PyxisError):
        pyxis_b200.Weights.quantize_int8(np.ones(4, np.float32), 4)


def _construct(px, what):
    from pyxis_b200.model import Decoder, ModelConfig, SyntheticModel
    if what == "quantize_int4":
        return px.Weights.quantize_int4(np.ones(64, np.float32), 32)
    if what == "quantize_int8_bf16":
        return px.Weights.quantize_int8(np.ones(4, np.uint16), 4)
    if what == "from_packed":
        return px.Weights.from_packed("int8", np.zeros(4, np.int8), np.ones(1, np.float32), 4, 4)
    if what == "from_q8_0":
        return px.Weights.from_q8_0(bytes(34), 32)
    if what == "from_dense":
        return px.Weights.from_dense(np.ones(8, np.float32))
    cfg = ModelConfig(hidden=64, n_layers=1, n_q_heads=1, n_kv_heads=1, head_dim=64, ffn=64, vocab=64)
    return Decoder(SyntheticModel(cfg))


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device path")
@pytest.mark.parametrize("what", ["quantize_int4", "quantize_int8_bf16", "from_packed", "from_q8_0", "from_dense",
                                  "decoder"])
def test_every_entry_point_raises_without_a_device(what):
    """No CPU fallback anywhere: without a B200 each constructor raises the library's ENODEV."""
    import pyxis_b200 as px
    with pytest.raises(px.PyxisError) as e:
        _construct(px, what)
    assert e.value.code == _native.PYXIS_ENODEV


def test_null_arguments_are_rejected_on_the_host():
    L = _native.lib()
    assert L.pyxis_cuda_init(0, None) == _native.PYXIS_EINVAL
    assert L.pyxis_cuda_quantize(None, None, 1, 0, 4, 4, 1, None) == _native.PYXIS_EINVAL
    assert L.pyxis_cuda_weights_info(None, None, None, None, None, None) == _native.PYXIS_EINVAL
    assert L.pyxis_cuda_matmul(None, None, None, 1, 1, None) == _native.PYXIS_EINVAL
    assert L.pyxis_cuda_argmax_dev(None, None, 1, 1, 1, 0, None, None, None) == _native.PYXIS_EINVAL
    assert b"null" in L.pyxis_cuda_last_error()
    assert L.pyxis_cuda_weights_free(None) == _native.PYXIS_OK
    assert L.pyxis_cuda_destroy(None) == _native.PYXIS_OK


def test_synth_is_deterministic_and_normal():
    import pyxis_b200 as p
    a = p.synth_normal_f32(123, 200_000, 1.0)
    b = p.synth_normal_f32(123, 200_000, 1.0)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    c = p.synth_normal_f32(124, 1000, 1.0)
    assert not np.array_equal(a[:1000], c)
    w = p.synth_normal_bf16(7, 100_000, 0.02)
    wf = (w.astype(np.uint32) << 16).view(np.float32)
    assert abs(wf.std() - 0.02) < 5e-4
    t = p.synth_tokens(1, 10_000, 151936)
    assert t.min() >= 0 and t.max() < 151936


def _np_synth(seed, n, sigma):
    """numpy restatement of include/pyxis_synth.h (splitmix64 + Box-Muller cosine branch)."""
    M = np.uint64(0xFFFFFFFFFFFFFFFF)
    G = np.uint64(0x9E3779B97F4A7C15)

    def mix(z):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))

    k = np.arange(2 * n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = mix((np.uint64(seed) + (k + np.uint64(1)) * G) & M)
    u1 = ((h[0::2] >> np.uint64(11)).astype(np.float64) + 0.5) / 9007199254740992.0
    u2 = (h[1::2] >> np.uint64(11)).astype(np.float64) / 9007199254740992.0
    return (sigma * (np.sqrt(-2.0 * np.log(u1)) * np.cos(6.283185307179586 * u2))).astype(np.float32)


def test_synth_matches_numpy_restatement():
    import pyxis_b200 as p
    a = p.synth_normal_f32(99, 4096, 0.5)
    b = _np_synth(99, 4096, 0.5)
    assert np.max(np.abs(a - b)) <= 1e-6
