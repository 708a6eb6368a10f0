"""pyxis_cuda_argmax_noalloc: the argmax for callers that cannot call cudaMalloc (code running
under an allocator it does not own, or a memory-capped pool).  Its scratch is a fixed array in
the library's device image, so the check is that it returns exactly what the context-based
pyxis_cuda_argmax_dev returns -- argmax is integer work, so exactly equal, as the other argmax
tests require -- on two calls in a row (the second call reuses the scratch the first one left),
and that it refuses more rows than its scratch holds.  This file sorts last so a run that stops at
the first failure has run every other test before it."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call_both(values, index_base):
    import torch

    import pyxis_b200 as px
    from pyxis_b200 import _native

    L = _native.lib()
    M, n = values.shape
    ctx = px.get_cuda(values.device.index or 0)
    st = px._stream_handle(None, values.device)
    idx_ref = torch.empty(M, dtype=torch.int32, device=values.device)
    val_ref = torch.empty(M, dtype=torch.float32, device=values.device)
    _native.check(L.pyxis_cuda_argmax_dev(ctx.handle, C.c_void_p(values.data_ptr()), M, n, values.stride(0),
                                          index_base, C.c_void_p(idx_ref.data_ptr()), C.c_void_p(val_ref.data_ptr()),
                                          C.c_void_p(st)))
    out = []
    for _ in range(2):  # two calls in a row on the shared scratch
        idx = torch.full((M,), -1, dtype=torch.int32, device=values.device)
        val = torch.full((M,), np.nan, dtype=torch.float32, device=values.device)
        _native.check(L.pyxis_cuda_argmax_noalloc(C.c_void_p(values.data_ptr()), M, n, values.stride(0), index_base,
                                                  C.c_void_p(idx.data_ptr()), C.c_void_p(val.data_ptr()),
                                                  C.c_void_p(st)))
        torch.cuda.synchronize()
        out.append((idx.cpu().numpy(), val.cpu().numpy()))
    return idx_ref.cpu().numpy(), val_ref.cpu().numpy(), out


@pytest.mark.parametrize("index_base", [0, 123])
@pytest.mark.parametrize("M,n,ld", [(1, 151936, 151936), (5, 151936, 151936), (64, 4096, 4096), (3, 7, 7),
                                    (4, 1000, 1536)])
def test_noalloc_argmax_matches_context_argmax(M, n, ld, index_base):
    """Contiguous rows and rows that are a slice of a wider tensor (ld > n); index_base 0, where
    a NaN at a row's index 0 wins (the reference never moves off values[0]), and 123 (a vocab
    shard that does not hold index 0, where that NaN is skipped)."""
    import torch

    rng = np.random.default_rng(M * 1000 + n + index_base)
    v = rng.standard_normal((M, ld)).astype(np.float32)
    if n > 100:
        v[0, 17] = v[0, n - 3] = 99.0   # a tie: the lowest index wins
        v[-1, 0] = np.nan               # values[0] NaN
        if M > 2:
            v[1, 5] = np.nan            # a NaN elsewhere is skipped
            v[1, n:] = 1e30             # past the row's end (ld > n): never read
    t = torch.from_numpy(v).cuda()[:, :n]
    assert t.stride(0) == ld
    idx_ref, val_ref, calls = _call_both(t, index_base=index_base)
    if n > 100 and index_base == 0:
        assert idx_ref[-1] == 0
    for idx, val in calls:
        assert np.array_equal(idx, idx_ref)
        assert np.array_equal(val.view(np.uint32), val_ref.view(np.uint32))


def test_noalloc_argmax_allocates_nothing():
    """Device memory in use is the same before and after repeated calls (after one warm-up call,
    which loads the kernel)."""
    import torch

    t = torch.from_numpy(np.random.default_rng(1).standard_normal((8, 151936)).astype(np.float32)).cuda()
    _call_both(t, index_base=0)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _call_both(t, index_base=0)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    # the helper's own small torch outputs come from torch's cache, not new device memory
    assert free1 == free0, (free0, free1)


def test_noalloc_argmax_rejects_out_of_range_index_base():
    import torch

    import pyxis_b200 as px  # noqa: F401
    from pyxis_b200 import _native

    L = _native.lib()
    t = torch.zeros((2, 16), dtype=torch.float32, device="cuda")
    idx = torch.empty(2, dtype=torch.int32, device="cuda")
    for base in (-1, 2**31 - 15):  # the last index, base + n - 1, must fit an int32
        rc = L.pyxis_cuda_argmax_noalloc(C.c_void_p(t.data_ptr()), 2, 16, 16, base, C.c_void_p(idx.data_ptr()),
                                         None, None)
        assert rc == _native.PYXIS_EINVAL, base


def test_noalloc_argmax_rejects_more_rows_than_its_scratch():
    import torch

    import pyxis_b200 as px  # noqa: F401
    from pyxis_b200 import _native

    L = _native.lib()
    t = torch.zeros((65, 16), dtype=torch.float32, device="cuda")
    idx = torch.empty(65, dtype=torch.int32, device="cuda")
    rc = L.pyxis_cuda_argmax_noalloc(C.c_void_p(t.data_ptr()), 65, 16, 16, 0, C.c_void_p(idx.data_ptr()), None, None)
    assert rc == _native.PYXIS_EINVAL
    assert b"64 rows" in L.pyxis_cuda_last_error()
