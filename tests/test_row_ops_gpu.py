"""The decode step's row arithmetic on the device (pyxis_cuda_row_op: the rms_factor / rms_scale,
rope_rot and silu_f helpers every decode kernel applies) against the oracle's restatement of
src/rmsnorm.rs:11-20, src/attention.rs:144-162 and src/ffn.rs:52-54 at the model's sizes.
Tolerance: a few ulp of relative error per element (the device sums x^2 in another order and uses
CUDA's expf; RoPE reads the same host-made f32 table)."""
import ctypes as C

import numpy as np
import pytest

import oracle
import pyxis_b200 as px

pytestmark = pytest.mark.gpu


def row_op(op, x, w=None, eps=0.0, head_dim=0, pos=0, theta=0.0):
    x = np.ascontiguousarray(np.asarray(x, np.float32))
    wv = None if w is None else np.ascontiguousarray(np.asarray(w, np.float32))
    out = np.empty_like(x)
    px._native.check(px._native.lib().pyxis_cuda_row_op(
        px.get_cuda(0).handle, op, x.ctypes.data_as(C.c_void_p), x.size,
        None if wv is None else wv.ctypes.data_as(C.c_void_p), eps, head_dim, pos, theta,
        out.ctypes.data_as(C.c_void_p)))
    return out


@pytest.mark.parametrize("n", [2, 128, 2048, 6144])
def test_rmsnorm_matches_oracle(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32) * 3
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    got = row_op(1, x, w=w, eps=1e-6)
    ref = oracle.rmsnorm(x, w, 1e-6)
    np.testing.assert_allclose(got, ref, rtol=4e-7 * np.sqrt(n), atol=1e-30)


@pytest.mark.parametrize("head_dim,pos,theta", [(64, 0, 1e4), (128, 1, 1e6), (128, 2047, 1e6), (128, 2303, 1e6),
                                                (64, 70, 1e4)])
def test_rope_matches_oracle(head_dim, pos, theta):
    rng = np.random.default_rng(pos + head_dim)
    heads = 16
    x = rng.standard_normal(heads * head_dim).astype(np.float32)
    got = row_op(2, x, head_dim=head_dim, pos=pos, theta=theta)
    ref = np.concatenate([oracle.apply_rope(x[h * head_dim:(h + 1) * head_dim], head_dim, pos, theta)
                          for h in range(heads)])
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_silu_matches_oracle():
    x = np.concatenate([np.linspace(-30, 30, 4001), [0.0, -0.0, 1.0, -1.0, 88.0, -88.0]]).astype(np.float32)
    got = row_op(3, x)
    ref = np.array([oracle.silu(float(v)) for v in x], np.float32)
    np.testing.assert_allclose(got, ref, rtol=4e-7, atol=1e-37)
