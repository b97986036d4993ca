"""telmo_b200: the B200-native (sm_100a) hot path of telmo's speech encoders.

The Python layer mirrors the reference's operator interface for this path -- ``Kernels``,
``PackedWeights``, ``Epilogue``, ``Act``, ``Precision`` (src/kernels/mod.rs, src/quant.rs) and the
model entry points -- over the C ABI of ``libtelmo_b200.so`` (include/telmo_b200.h). Device
buffers are torch CUDA tensors (torch is used for device memory and streams only); every
computation runs in the library's CUDA kernels. There is no CPU fallback: without the library
or a B200 the calls raise.
"""

from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _lib
from ._lib import TelmoError, check

__all__ = ["Act", "Context", "Epilogue", "Kernels", "PackedWeights", "Precision", "TelmoError",
           "DeviceWeights"]


class Precision(enum.IntEnum):
    """How a weight matrix's values are stored (src/quant.rs:22-30)."""
    F32 = 0
    F16 = 1
    BF16 = 2
    INT8 = 3
    Q8_0 = 4


class Act(enum.IntEnum):
    """An activation applied in the matrix product's epilogue (src/kernels/mod.rs:366-373)."""
    NONE = 0
    RELU = 1
    SILU = 2


class DType(enum.IntEnum):
    F32 = 0
    BF16 = 1
    I32_PAIR = 2


@dataclass
class Epilogue:
    """``c = (accumulate ? c : 0) + scale * act(sum + bias)`` (src/kernels/mod.rs:375-398)."""
    bias: Optional[object] = None
    act: Act = Act.NONE
    scale: float = 1.0
    accumulate: bool = False

    @staticmethod
    def with_bias(bias) -> "Epilogue":
        return Epilogue(bias=bias)


Epilogue.PLAIN = Epilogue()


def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return int(t)


def _stream(stream) -> Optional[int]:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


class Context:
    """One GPU. Replaces the reference's Kernels table + thread Pool with CUDA streams."""

    def __init__(self, device: int = 0):
        lib = _lib.load()
        h = ctypes.c_void_p()
        check(lib.telmo_ctx_create(device, ctypes.byref(h)), None)
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    def check(self, stream=None) -> None:
        """Waits for the stream and raises if a kernel gave up on a bounded wait."""
        check(_lib.load().telmo_ctx_check(self._h, _stream(stream)), self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().telmo_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceWeights:
    """A weight matrix uploaded to one context (tensor-core layout)."""

    def __init__(self, ctx: Context, handle, n: int, k: int):
        self.ctx, self._h, self.n, self.k = ctx, handle, n, k

    @property
    def handle(self):
        return self._h

    def free(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().telmo_weights_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class PackedWeights:
    """A weight matrix of ``n`` outputs and ``k`` inputs in the reference's panel layout
    (src/kernels/mod.rs:177-304): 16-output panels of int8 values with one f32 scale per output
    (Int8) or per block of 32 inputs of each output (Q8_0, src/quant.rs:8-13)."""

    def __init__(self, n: int, k: int, precision: Precision, values: np.ndarray,
                 scales: np.ndarray):
        panels = (n + 15) // 16
        if precision not in (Precision.INT8, Precision.Q8_0):
            raise TelmoError(_lib.TELMO_ERR_UNSUPPORTED,
                             f"{precision.name}: this build runs int8 weights (INT8, Q8_0) only")
        if precision == Precision.Q8_0 and k % 32:
            raise TelmoError(_lib.TELMO_ERR_ARGUMENT, "Q8_0 needs inputs in multiples of 32")
        n_scales = panels * 16 * (k // 32 if precision == Precision.Q8_0 else 1)
        if values.size != panels * 16 * k or scales.size != n_scales:
            raise TelmoError(_lib.TELMO_ERR_ARGUMENT, "panel sizes do not match n and k")
        self.n, self.k, self.precision = n, k, precision
        self.values = np.ascontiguousarray(values, dtype=np.int8)
        self.scales = np.ascontiguousarray(scales, dtype=np.float32)

    @staticmethod
    def encode(rows: np.ndarray, n: int, k: int,
               precision: Precision = Precision.INT8) -> "PackedWeights":
        """quant::encode (src/quant.rs:202-269) of a row-major f32 [n, k] matrix."""
        rows = np.ascontiguousarray(rows, dtype=np.float32).reshape(n, k)
        panels = (n + 15) // 16
        values = np.zeros(panels * 16 * k, np.int8)
        if precision == Precision.Q8_0:
            scales = np.zeros(panels * 16 * (k // 32), np.float32)
            encode = _lib.load().telmo_encode_q8_0
        else:
            scales = np.zeros(panels * 16, np.float32)
            encode = _lib.load().telmo_encode_int8
        check(encode(rows.ctypes.data, n, k, values.ctypes.data, scales.ctypes.data))
        return PackedWeights(n, k, precision, values, scales)

    def upload(self, ctx: Context) -> DeviceWeights:
        h = ctypes.c_void_p()
        check(_lib.load().telmo_weights_upload(ctx.handle, int(self.precision), self.n, self.k,
                                               self.values.ctypes.data, self.scales.ctypes.data,
                                               ctypes.byref(h)), ctx.handle)
        return DeviceWeights(ctx, h, self.n, self.k)


class Kernels:
    """The matrix product of src/kernels/mod.rs on the GPU: ``linear`` and ``matmul`` over
    packed int8 weights, with the reference's Epilogue. Tensors are torch CUDA tensors."""

    def __init__(self, ctx: Context):
        self.ctx = ctx

    def linear(self, a, m: int, w: DeviceWeights, c, epi: Epilogue = Epilogue.PLAIN,
               stream=None) -> None:
        """``c = epilogue(a * w^T)`` with ``a`` and ``c`` contiguous (src/kernels/mod.rs:691)."""
        self.matmul(a, w.k, m, w, c, w.n, epi, stream)

    def matmul(self, a, lda: int, m: int, w: DeviceWeights, c, ldc: int,
               epi: Epilogue = Epilogue.PLAIN, stream=None, out_dtype: DType = None) -> None:
        """``c[m, n] = epilogue(a[m, k] * w^T)`` with strides (src/kernels/mod.rs:657)."""
        import torch
        if out_dtype is None:
            out_dtype = DType.BF16 if c.dtype == torch.bfloat16 else \
                DType.I32_PAIR if c.dtype == torch.int32 else DType.F32
        check(_lib.load().telmo_linear(self.ctx.handle, _ptr(a), lda, m, w.handle, _ptr(epi.bias),
                                       int(epi.act), float(epi.scale), int(epi.accumulate),
                                       _ptr(c), int(out_dtype), ldc, _stream(stream)),
              self.ctx.handle)

    def quantize_x2(self, a, lda: int, m: int, k: int, hi, lo, ldq: int, scale,
                    stream=None) -> None:
        check(_lib.load().telmo_quantize_x2(self.ctx.handle, _ptr(a), lda, m, k, _ptr(hi),
                                            _ptr(lo), ldq, _ptr(scale), _stream(stream)),
              self.ctx.handle)

    def conv_module_rows(self, x, frames: int, channels: int, kernel: int, stride: int, w, bias,
                         out, stream=None) -> None:
        """GLU, depthwise convolution and SiLU over one utterance's rows into `out` (f32), the
        reference's glu, dwconv1d_frame and silu kernels (src/kernels/mod.rs:462-470)."""
        check(_lib.load().telmo_conv_module_rows(self.ctx.handle, _ptr(x), frames, channels, kernel,
                                                 stride, _ptr(w), _ptr(bias), _ptr(out),
                                                 _stream(stream)),
              self.ctx.handle)

    def linear_q(self, hi, lo, ldq: int, scale, m: int, w: DeviceWeights, c, ldc: int,
                 epi: Epilogue = Epilogue.PLAIN, out_dtype: DType = DType.F32,
                 stream=None) -> None:
        check(_lib.load().telmo_linear_q(self.ctx.handle, _ptr(hi), _ptr(lo), ldq, _ptr(scale),
                                         m, w.handle, _ptr(epi.bias), int(epi.act),
                                         float(epi.scale), int(epi.accumulate), _ptr(c),
                                         int(out_dtype), ldc, _stream(stream)),
              self.ctx.handle)
