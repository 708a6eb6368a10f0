"""pyxis_b200 -- B200 (sm_100a) backend for pyxis's quantized matmul hot path, host side.

Mirrors the reference's call surface over the C ABI of libpyxis_cuda.so (include/pyxis_cuda.h):

  Weights.quantize_int8(values, block_size)          src/weights.rs:94-118
  Weights.quantize_int4(values, block_size)          src/weights.rs:120-151
  Weights.len() / is_empty()                         src/weights.rs:35-50
  matmul(input, weight, out_features, in_features)   src/matmul.rs:21-97
  argmax(values)                                     src/output_head.rs:30-44
  get_cuda()                                         src/matmul.rs:6-19 (the OnceLock singleton)

A ``Weights`` here is the HBM-resident variant (what ``Weights::CudaInt8 / CudaInt4`` is in the
Rust drop-in): packed once, at load time, on the device.  Errors raise ``PyxisError`` where the
reference panics.  There is no CPU fallback: without the CUDA library or a B200 the calls raise.
"""
from __future__ import annotations

import ctypes as C
import threading
from typing import Optional

import numpy as np

from . import _native
from ._native import PyxisError, QTYPE_BF16, QTYPE_F32, QTYPE_INT4, QTYPE_INT8, DTYPE_BF16, DTYPE_F32, check

__all__ = ["Weights", "CudaMatmul", "get_cuda", "matmul", "matmul_batch", "matmul_dev", "argmax",
           "argmax_dev", "PyxisError", "synth_normal_f32", "synth_normal_bf16", "synth_tokens"]

INT4_BLOCK_SIZE = 32  # src/model.rs:20


class CudaMatmul:
    """One device context (pyxis_cuda_init): the counterpart of MetalMatmul
    (src/metal_matmul.rs:191-219)."""

    def __init__(self, device: int = 0):
        L = _native.lib()
        h = C.c_void_p()
        check(L.pyxis_cuda_init(device, C.byref(h)))
        self.handle = h
        self.device = device
        self._lib = L

    @property
    def stream(self) -> int:
        return self._lib.pyxis_cuda_stream(self.handle) or 0

    def synchronize(self) -> None:
        check(self._lib.pyxis_cuda_synchronize(self.handle))

    def close(self) -> None:
        if self.handle:
            self._lib.pyxis_cuda_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


_CUDA: dict[int, Optional[CudaMatmul]] = {}
_CUDA_LOCK = threading.Lock()


def get_cuda(device: int = 0) -> Optional[CudaMatmul]:
    """Process-wide context per device, created on first use; None when there is no usable
    device (MetalMatmul::new returning None, src/metal_matmul.rs:199-205)."""
    with _CUDA_LOCK:
        if device not in _CUDA:
            try:
                _CUDA[device] = CudaMatmul(device)
            except PyxisError as e:
                if e.code != _native.PYXIS_ENODEV:
                    raise
                _CUDA[device] = None
        return _CUDA[device]


def _require_cuda(device: int = 0) -> CudaMatmul:
    ctx = get_cuda(device)
    if ctx is None:
        raise PyxisError(_native.PYXIS_ENODEV,
                         "CUDA weights require a CUDA device (" + _native.lib().pyxis_cuda_last_error().decode() + ")")
    return ctx


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


_QTYPE_NAMES = {QTYPE_INT8: "int8", QTYPE_INT4: "int4", QTYPE_F32: "f32", QTYPE_BF16: "bf16"}


class Weights:
    """HBM-resident weights in the reference layout (enum Weights, src/weights.rs:6-21).

    ``qtype`` is "int8" or "int4" (packed bytes and scales bit-identical to the reference
    quantizer's; ``download()`` returns them), or "f32" / "bf16" for unquantized rows
    (Weights::F32 / Weights::Bf16, no scales)."""

    def __init__(self, handle: C.c_void_p, ctx: CudaMatmul):
        self.handle = handle
        self.ctx = ctx
        L = _native.lib()
        qt, n, bs, nb, ns = C.c_int(), C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_size_t()
        check(L.pyxis_cuda_weights_info(handle, C.byref(qt), C.byref(n), C.byref(bs), C.byref(nb), C.byref(ns)))
        self.qtype = _QTYPE_NAMES[qt.value]
        self.num_elements = n.value
        self.block_size = bs.value
        self.data_bytes = nb.value
        self.num_scales = ns.value

    # -- constructors mirroring the reference ------------------------------------------------
    @staticmethod
    def _quantize(values, block_size: int, qtype: int, device: int = 0) -> "Weights":
        ctx = _require_cuda(device)
        L = _native.lib()
        h = C.c_void_p()
        try:  # a torch tensor already on the device is quantised in place, no host round trip
            import torch
            is_torch = isinstance(values, torch.Tensor)
        except ImportError:  # pragma: no cover
            is_torch = False
        if is_torch and values.is_cuda:
            if (values.device.index or 0) != device:
                raise PyxisError(_native.PYXIS_EINVAL,
                                 f"source tensor on {values.device}, weights requested on cuda:{device}")
            t = values.contiguous()
            # The library reads the source on its own non-blocking stream: torch's writes of the
            # tensor (and of the contiguous copy) must be complete first.
            torch.cuda.synchronize(device)
            if t.dtype == torch.float32:
                dt = DTYPE_F32
            elif t.dtype == torch.bfloat16:
                dt = DTYPE_BF16
            else:
                raise PyxisError(_native.PYXIS_EINVAL, f"unsupported source dtype {t.dtype}")
            check(L.pyxis_cuda_quantize(ctx.handle, C.c_void_p(t.data_ptr()), dt, 1, t.numel(), block_size,
                                        qtype, C.byref(h)))
            return Weights(h, ctx)
        if is_torch:
            values = values.detach().cpu().numpy() if values.dtype != torch.bfloat16 else \
                values.detach().cpu().view(torch.int16).numpy().view(np.uint16)
        arr = np.asarray(values)
        if arr.dtype == np.uint16:  # raw bf16 bits (Weights::Bf16)
            arr = np.ascontiguousarray(arr)
            dt = DTYPE_BF16
        else:
            arr = _f32(arr)
            dt = DTYPE_F32
        check(L.pyxis_cuda_quantize(ctx.handle, arr.ctypes.data_as(C.c_void_p), dt, 0, arr.size, block_size,
                                    qtype, C.byref(h)))
        return Weights(h, ctx)

    @staticmethod
    def quantize_int8(values, block_size: int, device: int = 0) -> "Weights":
        """Weights::quantize_int8 (src/weights.rs:94-118), packed on the device."""
        return Weights._quantize(values, block_size, QTYPE_INT8, device)

    @staticmethod
    def quantize_int4(values, block_size: int, device: int = 0) -> "Weights":
        """Weights::quantize_int4 (src/weights.rs:120-151), packed on the device."""
        return Weights._quantize(values, block_size, QTYPE_INT4, device)

    @staticmethod
    def from_packed(qtype: str, data, scales, block_size: int, num_elements: int, device: int = 0) -> "Weights":
        """Upload an already-packed Weights::Int8 / Int4 (e.g. a GGUF Q8_0 tensor, src/gguf.rs:245-271)."""
        ctx = _require_cuda(device)
        qt = QTYPE_INT8 if qtype == "int8" else QTYPE_INT4
        d = np.ascontiguousarray(np.asarray(data).view(np.uint8))
        s = _f32(scales)
        h = C.c_void_p()
        check(_native.lib().pyxis_cuda_weights_upload(ctx.handle, qt, d.ctypes.data_as(C.c_void_p),
                                                      s.ctypes.data_as(C.c_void_p), num_elements, block_size,
                                                      C.byref(h)))
        return Weights(h, ctx)

    @staticmethod
    def from_q8_0(blocks, num_elements: int, device: int = 0) -> "Weights":
        """read_q8_0_weights (src/gguf.rs:245-271) on the device: ``blocks`` holds the GGUF Q8_0
        tensor bytes (ceil(n/32) blocks of 34 bytes: f16 scale, 32 int8) on the host, or is a
        CUDA torch uint8 tensor on the weights' device.  Returns int8 weights with block 32."""
        ctx = _require_cuda(device)
        h = C.c_void_p()
        try:
            import torch
            is_dev = isinstance(blocks, torch.Tensor) and blocks.is_cuda
        except ImportError:  # pragma: no cover
            is_dev = False
        nb = (num_elements + 31) // 32
        if is_dev:
            if (blocks.device.index or 0) != device:
                raise PyxisError(_native.PYXIS_EINVAL,
                                 f"q8_0 tensor on {blocks.device}, weights requested on cuda:{device}")
            if blocks.numel() * blocks.element_size() < nb * 34:
                raise PyxisError(_native.PYXIS_EINVAL, "q8_0 tensor shorter than ceil(n/32) * 34 bytes")
            torch.cuda.synchronize(device)  # the upload reads it on the library's own stream
            check(_native.lib().pyxis_cuda_weights_upload_q8_0(ctx.handle, C.c_void_p(blocks.data_ptr()), 1,
                                                               num_elements, C.byref(h)))
            return Weights(h, ctx)
        b = np.frombuffer(bytes(blocks), dtype=np.uint8) if isinstance(blocks, (bytes, bytearray, memoryview)) \
            else np.ascontiguousarray(np.asarray(blocks).view(np.uint8).reshape(-1))
        if b.size < nb * 34:  # tensor_bytes: the data must cover every block (src/gguf.rs:273-287)
            raise PyxisError(_native.PYXIS_EINVAL, "q8_0 tensor shorter than ceil(n/32) * 34 bytes")
        check(_native.lib().pyxis_cuda_weights_upload_q8_0(ctx.handle, b.ctypes.data_as(C.c_void_p), 0,
                                                           num_elements, C.byref(h)))
        return Weights(h, ctx)

    @staticmethod
    def from_dense(values, device: int = 0) -> "Weights":
        """Unquantized rows on the device: Weights::F32 from float values, Weights::Bf16 from raw
        bf16 bit patterns (a np.uint16 array or a torch.bfloat16 tensor)."""
        ctx = _require_cuda(device)
        try:
            import torch
            if isinstance(values, torch.Tensor):
                values = values.detach().cpu()
                values = values.view(torch.int16).numpy().view(np.uint16) if values.dtype == torch.bfloat16 \
                    else values.numpy()
        except ImportError:  # pragma: no cover
            pass
        arr = np.asarray(values)
        if arr.dtype == np.uint16:
            arr, qt = np.ascontiguousarray(arr.reshape(-1)), QTYPE_BF16
        else:
            arr, qt = _f32(arr).reshape(-1), QTYPE_F32
        h = C.c_void_p()
        check(_native.lib().pyxis_cuda_weights_upload(ctx.handle, qt, arr.ctypes.data_as(C.c_void_p), None,
                                                      arr.size, 0, C.byref(h)))
        return Weights(h, ctx)

    # -- accessors ---------------------------------------------------------------------------
    def len(self) -> int:
        return self.num_elements

    def __len__(self) -> int:
        return self.num_elements

    def is_empty(self) -> bool:
        return self.num_elements == 0

    def download(self) -> tuple[np.ndarray, np.ndarray]:
        """(data, scales) on the host: int8 -> np.int8 [n]; int4 -> np.uint8 [ceil(n/2)];
        f32 -> np.float32 [n]; bf16 -> np.uint16 [n] (no scales: an empty array)."""
        dt = {"int8": np.int8, "int4": np.uint8, "f32": np.float32, "bf16": np.uint16}[self.qtype]
        data = np.empty(self.data_bytes // np.dtype(dt).itemsize, dtype=dt)
        scales = np.empty(self.num_scales, dtype=np.float32)
        check(_native.lib().pyxis_cuda_weights_download(self.handle, data.ctypes.data_as(C.c_void_p),
                                                        scales.ctypes.data_as(C.c_void_p)))
        return data, scales

    def device_ptrs(self) -> tuple[int, int]:
        d, s = C.c_void_p(), C.c_void_p()
        check(_native.lib().pyxis_cuda_weights_device_ptrs(self.handle, C.byref(d), C.byref(s)))
        return d.value, s.value

    def free(self) -> None:
        if self.handle:
            _native.lib().pyxis_cuda_weights_free(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.free()
        except Exception:
            pass


def matmul(input, weight: Weights, out_features: int, in_features: int) -> np.ndarray:
    """matmul (src/matmul.rs:21-97) with host buffers: returns y [out_features] f32."""
    x = _f32(input)
    if x.size != in_features:  # assert_eq!(input.len(), in_features) (:27)
        raise PyxisError(_native.PYXIS_EINVAL, f"input.len() = {x.size} != in_features = {in_features}")
    y = np.empty(out_features, dtype=np.float32)
    check(_native.lib().pyxis_cuda_matmul(weight.ctx.handle, x.ctypes.data_as(C.c_void_p), weight.handle,
                                          out_features, in_features, y.ctypes.data_as(C.c_void_p)))
    return y


def matmul_batch(inputs, weight: Weights, out_features: int, in_features: int) -> np.ndarray:
    """M independent matmul rows with host buffers: [M, in] -> [M, out]."""
    X = _f32(inputs).reshape(-1, in_features)
    Y = np.empty((X.shape[0], out_features), dtype=np.float32)
    check(_native.lib().pyxis_cuda_matmul_batch(weight.ctx.handle, X.ctypes.data_as(C.c_void_p), X.shape[0],
                                                weight.handle, out_features, in_features,
                                                Y.ctypes.data_as(C.c_void_p)))
    return Y


CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the legacy default stream, as an explicit handle


def _stream_handle(stream, device) -> int:
    """cudaStream_t for a torch stream.  torch reports its default stream as 0, which the C ABI
    reads as "the context's own stream"; pass the legacy default stream's explicit handle
    instead so work lands on the stream the caller's events and tensors use."""
    import torch

    h = (stream or torch.cuda.current_stream(device)).cuda_stream
    return h if h else CUDA_STREAM_LEGACY


def matmul_dev(X, weight: Weights, out_features: int, in_features: int, Y=None, stream=None, workspace=None):
    """Device-pointer form over torch CUDA tensors: X [M, in] f32 -> Y [M, out] f32, launched
    asynchronously on ``stream`` (a torch.cuda.Stream; default: torch's current stream)."""
    import torch

    if X.dim() == 1:
        X = X.unsqueeze(0)
    if (X.device.index or 0) != weight.ctx.device or (Y is not None and (Y.device.index or 0) != weight.ctx.device):
        raise PyxisError(_native.PYXIS_EINVAL, f"X/Y must be on cuda:{weight.ctx.device}, the weights' device")
    M = X.shape[0]
    if Y is None:
        Y = torch.empty((M, out_features), dtype=torch.float32, device=X.device)
    st = _stream_handle(stream, X.device)
    ws_ptr, ws_bytes = (workspace.data_ptr(), workspace.numel() * workspace.element_size()) if workspace is not None else (None, 0)
    check(_native.lib().pyxis_cuda_matmul_dev(weight.ctx.handle, weight.handle, C.c_void_p(X.data_ptr()), M,
                                              X.stride(0), out_features, in_features, C.c_void_p(Y.data_ptr()),
                                              Y.stride(0), C.c_void_p(ws_ptr), ws_bytes, C.c_void_p(st)))
    return Y


def matmul_kernel_name(weight: Weights, M: int, out_features: int, in_features: int) -> str:
    """The kernel ``matmul_dev`` launches for M contiguous rows of x (diagnostics)."""
    return _native.lib().pyxis_cuda_matmul_kernel(weight.ctx.handle, weight.handle, M, out_features,
                                                   in_features).decode()


def argmax_dev(values, index_base: int = 0, idx=None, val=None, stream=None, device: int = 0):
    """Row-wise argmax of a torch CUDA tensor [M, n] (src/output_head.rs:30-44 per row)."""
    import torch

    if values.dim() == 1:
        values = values.unsqueeze(0)
    M, n = values.shape
    ctx = _require_cuda(values.device.index or 0)
    if idx is None:
        idx = torch.empty(M, dtype=torch.int32, device=values.device)
    if val is None:
        val = torch.empty(M, dtype=torch.float32, device=values.device)
    st = _stream_handle(stream, values.device)
    check(_native.lib().pyxis_cuda_argmax_dev(ctx.handle, C.c_void_p(values.data_ptr()), M, n, values.stride(0),
                                              index_base, C.c_void_p(idx.data_ptr()), C.c_void_p(val.data_ptr()),
                                              C.c_void_p(st)))
    return idx, val


def argmax(values) -> int:
    """output_head::argmax (src/output_head.rs:30-44) of a host vector, computed on the device."""
    import torch

    v = _f32(values)
    if v.size == 0:
        raise PyxisError(_native.PYXIS_EINVAL, "argmax of an empty slice (assert!, src/output_head.rs:31)")
    t = torch.from_numpy(v).cuda()
    idx, _ = argmax_dev(t)
    return int(idx.item())


# -- seeded synthetic inputs (include/pyxis_synth.h) ----------------------------------------------
def synth_normal_f32(seed: int, n: int, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _native.lib().pyxis_synth_normal_f32(seed, n, sigma, out.ctypes.data_as(C.c_void_p))
    return out


def synth_normal_bf16(seed: int, n: int, sigma: float = 0.02) -> np.ndarray:
    """bf16 bit patterns (np.uint16) of N(0, sigma) values rounded to nearest even."""
    out = np.empty(n, dtype=np.uint16)
    _native.lib().pyxis_synth_normal_bf16(seed, n, sigma, out.ctypes.data_as(C.c_void_p))
    return out


def synth_tokens(seed: int, n: int, vocab: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    _native.lib().pyxis_synth_tokens(seed, n, vocab, out.ctypes.data_as(C.c_void_p))
    return out
