"""ctypes binding of libpyxis_cuda.so (include/pyxis_cuda.h, pyxis_decode.h, pyxis_comm.h,
include/pyxis_synth.h).

The library is built in-tree by ``pyxis_b200.build``.  There is no fallback: if the shared
library is missing or cannot be loaded, importing the CUDA path raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpyxis_cuda.so")

PYXIS_OK = 0
PYXIS_EINVAL = 1
PYXIS_ENODEV = 2
PYXIS_ECUDA = 3
PYXIS_ENOMEM = 4
PYXIS_ETIMEOUT = 5
PYXIS_EUNSUPPORTED = 6
PYXIS_ENCCL = 7

QTYPE_INT8 = 1
QTYPE_INT4 = 2
QTYPE_F32 = 3
QTYPE_BF16 = 4
DTYPE_F32 = 1
DTYPE_BF16 = 2

_vp = C.c_void_p
_sz = C.c_size_t

# name -> (restype, argtypes); every symbol the public headers declare.
SIGNATURES = {
    "pyxis_cuda_last_error": (C.c_char_p, []),
    "pyxis_cuda_abi_version": (C.c_uint32, []),
    "pyxis_cuda_init": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "pyxis_cuda_destroy": (C.c_int, [_vp]),
    "pyxis_cuda_stream": (_vp, [_vp]),
    "pyxis_cuda_synchronize": (C.c_int, [_vp]),
    "pyxis_cuda_quantize": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _sz, _sz, C.c_int, C.POINTER(_vp)]),
    "pyxis_cuda_weights_upload": (C.c_int, [_vp, C.c_int, _vp, _vp, _sz, _sz, C.POINTER(_vp)]),
    "pyxis_cuda_weights_upload_q8_0": (C.c_int, [_vp, _vp, C.c_int, _sz, C.POINTER(_vp)]),
    "pyxis_cuda_weights_info": (C.c_int, [_vp, C.POINTER(C.c_int), C.POINTER(_sz), C.POINTER(_sz),
                                          C.POINTER(_sz), C.POINTER(_sz)]),
    "pyxis_cuda_weights_download": (C.c_int, [_vp, _vp, _vp]),
    "pyxis_cuda_weights_device_ptrs": (C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_vp)]),
    "pyxis_cuda_weights_free": (C.c_int, [_vp]),
    "pyxis_cuda_matmul": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "pyxis_cuda_matmul_batch": (C.c_int, [_vp, _vp, _sz, _vp, _sz, _sz, _vp]),
    "pyxis_cuda_matmul_dev": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp, _sz, _vp, _sz, _vp]),
    "pyxis_cuda_matmul_workspace_size": (_sz, [_sz, _sz]),
    "pyxis_cuda_reserve_workspace": (C.c_int, [_vp, _sz]),
    "pyxis_cuda_check_device_error": (C.c_int, [_vp]),
    "pyxis_cuda_matmul_kernel": (C.c_char_p, [_vp, _vp, C.c_size_t, C.c_size_t, C.c_size_t]),
    "pyxis_cuda_argmax_dev": (C.c_int, [_vp, _vp, _sz, _sz, _sz, C.c_int64, _vp, _vp, _vp]),
    "pyxis_cuda_argmax_noalloc": (C.c_int, [_vp, _sz, _sz, _sz, C.c_int64, _vp, _vp, _vp]),
    "pyxis_cuda_model_create": (C.c_int, [_vp, _vp, C.POINTER(_vp)]),
    "pyxis_cuda_model_set_layer": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "pyxis_cuda_model_set_head": (C.c_int, [_vp, _vp, _vp, _vp]),
    "pyxis_cuda_model_generate": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _vp]),
    "pyxis_cuda_model_generate_batch": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _vp, _vp]),
    "pyxis_cuda_model_free": (C.c_int, [_vp]),
    "pyxis_rope_table": (C.c_int, [C.c_float, C.c_int, C.c_int, _vp, _vp]),
    "pyxis_cuda_row_op": (C.c_int, [_vp, C.c_int, _vp, _sz, _vp, C.c_float, C.c_int, C.c_int, C.c_float, _vp]),
    "pyxis_cuda_model_prefill_hidden": (C.c_int, [_vp, _vp, _sz, _sz, _vp]),
    "pyxis_cuda_comm_unique_id": (C.c_int, [_vp]),
    "pyxis_cuda_comm_init": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.POINTER(_vp)]),
    "pyxis_cuda_comm_info": (C.c_int, [_vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "pyxis_cuda_comm_free": (C.c_int, [_vp]),
    "pyxis_cuda_head_greedy_dev": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _sz, _sz, _vp, _vp]),
    "pyxis_cuda_head_reserve": (C.c_int, [_vp, _sz, _sz]),
    "pyxis_cuda_model_set_vocab_parallel": (C.c_int, [_vp, _vp, _vp, _sz, _sz]),
    "pyxis_synth_normal_f32": (None, [C.c_uint64, _sz, C.c_float, _vp]),
    "pyxis_synth_normal_bf16": (None, [C.c_uint64, _sz, C.c_float, _vp]),
    "pyxis_synth_tokens": (None, [C.c_uint64, _sz, C.c_uint32, _vp]),
}


class PyxisError(RuntimeError):
    """A nonzero pyxis_status; the reference panics on the same conditions."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"pyxis_cuda error {code}: {msg}")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    """Load libpyxis_cuda.so (once).  Raises if it is missing: there is no CPU fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m pyxis_b200.build` "
                              "(the CUDA path has no fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != PYXIS_OK:
        raise PyxisError(rc, lib().pyxis_cuda_last_error().decode(errors="replace"))
