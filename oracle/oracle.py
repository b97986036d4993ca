"""ctypes bindings of the oracle library (liboracle.so), a CPU restatement of telmo's CPU path.

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
use this module as the checker. The product (``telmo_b200``) never imports it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

ACT_NONE, ACT_RELU, ACT_SILU = 0, 1, 2

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t


class GraniteConfig(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in (
        "d_model", "heads", "head_dim", "layers", "ff", "conv_kernel", "conv_channels", "n_mels",
        "context", "max_relative", "n_subsample")] + [
        ("subsample_layers", ctypes.c_int * 8), ("vocab", ctypes.c_int), ("blank", ctypes.c_int)]


def build() -> str:
    """Compiles liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    L = ctypes.CDLL(_LIB_PATH)
    L.oracle_quantize_row_int8.restype = ctypes.c_float
    L.oracle_quantize_row_int8.argtypes = [_f32p, _sz, _i8p]
    L.oracle_encode_int8.argtypes = [_f32p, _sz, _sz, _i8p, _f32p]
    L.oracle_decode_int8.argtypes = [_i8p, _f32p, _sz, _sz, _f32p]
    L.oracle_f32_to_bf16.restype = ctypes.c_uint16
    L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
    L.oracle_f32_to_f16.restype = ctypes.c_uint16
    L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
    L.oracle_f16_to_f32.restype = ctypes.c_float
    L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.oracle_bf16_to_f32.restype = ctypes.c_float
    L.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
    L.oracle_linear_int8.argtypes = [_f32p, _sz, _sz, _i8p, _f32p, _sz, _sz, _f32p, _sz,
                                     ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                     ctypes.c_int]
    L.oracle_linear_q8_0.argtypes = L.oracle_linear_int8.argtypes
    L.oracle_granite_set_matrix_q8_0.restype = ctypes.c_int
    L.oracle_granite_set_matrix_q8_0.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _sz, _sz, _i8p,
                                                 _f32p]
    L.oracle_encode_q8_0.argtypes = [_f32p, _sz, _sz, _i8p, _f32p]
    L.oracle_decode_q8_0.argtypes = [_i8p, _f32p, _sz, _sz, _f32p]
    L.oracle_q8_0_two_level.argtypes = [_i8p, _f32p, _sz, _sz, _i8p, _i8p, _f32p]
    L.oracle_gemm_i8_x2w_acc.argtypes = [_i8p, _i8p, _sz, _sz, _i8p, _i8p, _sz, _sz, _i32p, _i32p]
    L.oracle_matmul_rowmajor.argtypes = [_f32p, _sz, _sz, _f32p, _sz, _sz, _sz, _f32p, _sz,
                                         ctypes.c_void_p, ctypes.c_int, ctypes.c_float,
                                         ctypes.c_int]
    L.oracle_quantize_x2.argtypes = [_f32p, _sz, _sz, _sz, _i8p, _i8p, _sz, _f32p]
    L.oracle_gemm_i8_x2_acc.argtypes = [_i8p, _i8p, _sz, _sz, _i8p, _sz, _sz, _i32p, _i32p]
    L.oracle_epilogue_x2.argtypes = [_i32p, _i32p, _sz, _sz, _f32p, _f32p, ctypes.c_void_p,
                                     ctypes.c_int, ctypes.c_float, ctypes.c_int, _f32p, _sz]
    L.oracle_layer_norm.argtypes = [_f32p, _f32p, _f32p, _f32p, _sz, ctypes.c_float]
    L.oracle_softmax.argtypes = [_f32p, _sz]
    L.oracle_glu.argtypes = [_f32p, _f32p, _f32p, _sz]
    L.oracle_silu.argtypes = [_f32p, _sz]
    L.oracle_dwconv1d_frame.argtypes = [_f32p, _sz, _sz, _sz, _f32p, _sz, _f32p, _f32p]
    L.oracle_real_fft.restype = ctypes.c_int
    L.oracle_real_fft.argtypes = [_f64p, _sz, _f64p]
    L.oracle_granite_rows_for.restype = _sz
    L.oracle_granite_rows_for.argtypes = [_sz]
    L.oracle_granite_features.restype = ctypes.c_int
    L.oracle_granite_features.argtypes = [_f32p, _sz, _sz, _f32p]
    L.oracle_parakeet_features.restype = ctypes.c_int
    L.oracle_parakeet_features.argtypes = [_f32p, _sz, _f32p]
    L.oracle_granite_new.restype = ctypes.c_void_p
    L.oracle_granite_new.argtypes = [ctypes.POINTER(GraniteConfig)]
    L.oracle_granite_free.argtypes = [ctypes.c_void_p]
    L.oracle_granite_set_matrix.restype = ctypes.c_int
    L.oracle_granite_set_matrix.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _sz, _sz, _i8p,
                                            _f32p]
    L.oracle_granite_set_vector.restype = ctypes.c_int
    L.oracle_granite_set_vector.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _sz, _f32p]
    L.oracle_granite_missing.restype = ctypes.c_int
    L.oracle_granite_missing.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _sz]
    L.oracle_granite_frames_for.restype = _sz
    L.oracle_granite_frames_for.argtypes = [ctypes.c_void_p, _sz]
    L.oracle_granite_encode.restype = ctypes.c_long
    L.oracle_granite_encode.argtypes = [ctypes.c_void_p, _f32p, _sz, _f32p, ctypes.c_int,
                                        ctypes.c_int]
    L.oracle_granite_frame_ids.argtypes = [ctypes.c_void_p, _f32p, _sz, _u32p, _f32p,
                                           ctypes.c_int]
    L.oracle_granite_logits.argtypes = [ctypes.c_void_p, _f32p, _sz, _f32p, ctypes.c_int]
    L.oracle_ctc_tokens.restype = _sz
    L.oracle_ctc_tokens.argtypes = [_u32p, _sz, ctypes.c_uint32, _u32p]
    _lib = L
    return L


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---- quant.rs -------------------------------------------------------------------------------

def quantize_row_int8(x):
    x = _c(x, np.float32)
    q = np.zeros(x.size, np.int8)
    d = lib().oracle_quantize_row_int8(x, x.size, q)
    return q, np.float32(d)


def encode_int8(w):
    """Row-major [n, k] f32 -> (panel values int8 [ceil(n/16)*16*k], scales f32)."""
    w = _c(w, np.float32)
    n, k = w.shape
    panels = (n + 15) // 16
    values = np.zeros(panels * 16 * k, np.int8)
    scales = np.zeros(panels * 16, np.float32)
    lib().oracle_encode_int8(w.reshape(-1), n, k, values, scales)
    return values, scales


def decode_int8(values, scales, n, k):
    out = np.zeros((n, k), np.float32)
    lib().oracle_decode_int8(_c(values, np.int8), _c(scales, np.float32), n, k, out.reshape(-1))
    return out


def encode_q8_0(w):
    """Row-major [n, k] f32 (k a multiple of 32) -> Q8_0 panels: (values int8
    [ceil(n/16)*16*k], scales f32 [ceil(n/16)*(k/32)*16])."""
    w = _c(w, np.float32)
    n, k = w.shape
    panels = (n + 15) // 16
    values = np.zeros(panels * 16 * k, np.int8)
    scales = np.zeros(panels * (k // 32) * 16, np.float32)
    lib().oracle_encode_q8_0(w.reshape(-1), n, k, values, scales)
    return values, scales


def decode_q8_0(values, scales, n, k):
    out = np.zeros((n, k), np.float32)
    lib().oracle_decode_q8_0(_c(values, np.int8), _c(scales, np.float32), n, k, out.reshape(-1))
    return out


# ---- the matrix product -----------------------------------------------------------------------

def linear_int8(a, values, scales, n, k, bias=None, act=ACT_NONE, scale=1.0, c=None,
                accumulate=False, threads=1):
    """Kernels::linear with int8 PackedWeights: returns c [m, n] f32."""
    a = _c(a, np.float32)
    m = a.shape[0]
    out = np.zeros((m, n), np.float32) if c is None else np.array(c, np.float32, copy=True)
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_linear_int8(a.reshape(-1) if m else np.zeros(1, np.float32), a.shape[1] if m else k,
                             m, _c(values, np.int8), _c(scales, np.float32), n, k,
                             out.reshape(-1) if m else np.zeros(1, np.float32), n, _ptr(b), act,
                             float(scale), int(accumulate), int(threads))
    return out


def linear_q8_0(a, values, scales, n, k, bias=None, act=ACT_NONE, scale=1.0, c=None,
                accumulate=False, threads=1):
    """Kernels::linear with Q8_0 PackedWeights: returns c [m, n] f32."""
    a = _c(a, np.float32)
    m = a.shape[0]
    out = np.zeros((m, n), np.float32) if c is None else np.array(c, np.float32, copy=True)
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_linear_q8_0(a.reshape(-1), a.shape[1], m, _c(values, np.int8),
                             _c(scales, np.float32), n, k, out.reshape(-1), n, _ptr(b), act,
                             float(scale), int(accumulate), int(threads))
    return out


def q8_0_two_level(values, scales, n, k):
    """The CUDA upload's re-encoding of Q8_0 panels: (w_hi [n, k], w_lo [n, k], w_scale [n])."""
    w_hi = np.zeros((n, k), np.int8)
    w_lo = np.zeros((n, k), np.int8)
    ws = np.zeros(n, np.float32)
    lib().oracle_q8_0_two_level(_c(values, np.int8), _c(scales, np.float32), n, k,
                                w_hi.reshape(-1), w_lo.reshape(-1), ws)
    return w_hi, w_lo, ws


def gemm_i8_x2w_acc(hi, lo, w_hi, w_lo, n, k):
    """Integer sums against two-level weights: (hi . W_hi, lo . W_hi + hi . W_lo)."""
    hi = _c(hi, np.int8)
    lo = _c(lo, np.int8)
    m = hi.shape[0]
    acc_hi = np.zeros((m, n), np.int32)
    acc_lo = np.zeros((m, n), np.int32)
    lib().oracle_gemm_i8_x2w_acc(hi.reshape(-1), lo.reshape(-1), k, m, _c(w_hi, np.int8).reshape(-1),
                                 _c(w_lo, np.int8).reshape(-1), n, k, acc_hi.reshape(-1),
                                 acc_lo.reshape(-1))
    return acc_hi, acc_lo


def linear_x2_q8_0(a, values, scales, n, k, bias=None, act=ACT_NONE, scale=1.0, c=None,
                   accumulate=False):
    """The CUDA linear's exact arithmetic over Q8_0 panels: the two-level re-encoding, split
    activations, i32 sums (lo . W_hi + hi . W_lo into the low sums), the x2 epilogue."""
    w_hi, w_lo, ws = q8_0_two_level(values, scales, n, k)
    hi, lo, s = quantize_x2(a)
    acc_hi, acc_lo = gemm_i8_x2w_acc(hi, lo, w_hi, w_lo, n, k)
    return epilogue_x2(acc_hi, acc_lo, s, ws, bias, act, scale, c, accumulate)


def quantize_x2(x):
    """The CUDA path's split int8 rule: (hi [m, k] int8, lo [m, k] int8, scale [m] f32)."""
    x = _c(x, np.float32)
    m, k = x.shape
    hi = np.zeros((m, k), np.int8)
    lo = np.zeros((m, k), np.int8)
    s = np.zeros(m, np.float32)
    lib().oracle_quantize_x2(x.reshape(-1), m, k, k, hi.reshape(-1), lo.reshape(-1), k, s)
    return hi, lo, s


def gemm_i8_x2_acc(hi, lo, values, n, k):
    hi = _c(hi, np.int8)
    lo = _c(lo, np.int8)
    m = hi.shape[0]
    acc_hi = np.zeros((m, n), np.int32)
    acc_lo = np.zeros((m, n), np.int32)
    lib().oracle_gemm_i8_x2_acc(hi.reshape(-1), lo.reshape(-1), k, m, _c(values, np.int8), n, k,
                                acc_hi.reshape(-1), acc_lo.reshape(-1))
    return acc_hi, acc_lo


def epilogue_x2(acc_hi, acc_lo, row_scale, w_scales, bias=None, act=ACT_NONE, scale=1.0,
                c=None, accumulate=False):
    acc_hi = _c(acc_hi, np.int32)
    acc_lo = _c(acc_lo, np.int32)
    m, n = acc_hi.shape
    out = np.zeros((m, n), np.float32) if c is None else np.array(c, np.float32, copy=True)
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_epilogue_x2(acc_hi.reshape(-1), acc_lo.reshape(-1), m, n,
                             _c(row_scale, np.float32), _c(w_scales, np.float32)[:n].copy(),
                             _ptr(b), act, float(scale), int(accumulate), out.reshape(-1), n)
    return out


def linear_x2(a, values, scales, n, k, bias=None, act=ACT_NONE, scale=1.0, c=None,
              accumulate=False):
    """The CUDA linear's exact arithmetic: split quantization, i32 sums, the x2 epilogue."""
    hi, lo, s = quantize_x2(a)
    acc_hi, acc_lo = gemm_i8_x2_acc(hi, lo, values, n, k)
    return epilogue_x2(acc_hi, acc_lo, s, scales, bias, act, scale, c, accumulate)


# ---- row kernels ------------------------------------------------------------------------------

def layer_norm(x, gamma, beta, eps=1e-5):
    x = _c(x, np.float32)
    out = np.zeros_like(x)
    for r in range(x.shape[0]):
        lib().oracle_layer_norm(x[r].copy(), out[r], _c(gamma, np.float32), _c(beta, np.float32),
                                x.shape[1], eps)
    return out


def softmax(x):
    x = np.array(x, np.float32, copy=True)
    for r in range(x.shape[0]):
        row = x[r].copy()
        lib().oracle_softmax(row, row.size)
        x[r] = row
    return x


def real_fft(x):
    x = _c(x, np.float64)
    out = np.zeros(2 * (x.size // 2 + 1), np.float64)
    if lib().oracle_real_fft(x, x.size, out) != 0:
        raise ValueError("the FFT length must be a power of two of at least 4")
    return out[0::2] + 1j * out[1::2]


# ---- front ends -------------------------------------------------------------------------------

def granite_rows_for(samples):
    return lib().oracle_granite_rows_for(samples)


def granite_features(samples, n_mels=80):
    x = _c(samples, np.float32)
    rows = granite_rows_for(x.size)
    out = np.zeros((max(rows, 1), 4 * n_mels), np.float32)
    if lib().oracle_granite_features(x, x.size, n_mels, out.reshape(-1)) != 0:
        raise ValueError(f"The audio is too short ({x.size} samples). It needs at least 320.")
    return out[:rows]


def parakeet_features(samples):
    x = _c(samples, np.float32)
    frames = x.size // 160
    out = np.zeros((max(frames, 1), 128), np.float32)
    if lib().oracle_parakeet_features(x, x.size, out.reshape(-1)) != 0:
        raise ValueError(f"The audio is too short ({x.size} samples). It needs at least 320.")
    return out[:frames]


# ---- the Granite encoder -----------------------------------------------------------------------

class Granite:
    """The oracle's Granite model, filled from the same named entries as the CUDA model."""

    def __init__(self, config: dict, entries: dict):
        cfg = GraniteConfig()
        for key in ("d_model", "heads", "head_dim", "layers", "ff", "conv_kernel",
                    "conv_channels", "n_mels", "context", "max_relative", "vocab", "blank"):
            setattr(cfg, key, int(config[key]))
        subs = list(config["subsample_layers"])
        cfg.n_subsample = len(subs)
        for i, s in enumerate(subs):
            cfg.subsample_layers[i] = s
        self.config = dict(config)
        self._h = lib().oracle_granite_new(ctypes.byref(cfg))
        if not self._h:
            raise ValueError("the Granite config does not fit together")
        for name, entry in entries.items():
            if isinstance(entry, tuple):
                values, scales, n, k = entry[:4]
                q8 = len(entry) > 4 and entry[4] == "q8_0"
                setter = lib().oracle_granite_set_matrix_q8_0 if q8 else lib().oracle_granite_set_matrix
                rc = setter(self._h, name.encode(), n, k, _c(values, np.int8), _c(scales, np.float32))
            else:
                data = _c(entry, np.float32).reshape(-1)
                rc = lib().oracle_granite_set_vector(self._h, name.encode(), data.size, data)
            if rc != 0:
                raise ValueError(f"bad entry {name}")
        buf = ctypes.create_string_buffer(64)
        if lib().oracle_granite_missing(self._h, buf, 64):
            raise ValueError(f"missing entry {buf.value.decode()}")

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib().oracle_granite_free(self._h)
                self._h = None
        except Exception:
            pass

    def frames_for(self, rows):
        return lib().oracle_granite_frames_for(self._h, rows)

    def encode(self, features, tap_layer=-1, threads=1):
        f = _c(features, np.float32)
        rows = f.shape[0]
        out = np.zeros((max(rows, 1), self.config["d_model"]), np.float32)
        t = lib().oracle_granite_encode(self._h, f.reshape(-1), rows, out.reshape(-1), tap_layer,
                                        threads)
        if t < 0:
            raise ValueError(f"The audio is too short ({rows} feature rows).")
        return out[:t]

    def logits(self, encoded, threads=1):
        e = _c(encoded, np.float32)
        out = np.zeros((e.shape[0], self.config["vocab"]), np.float32)
        lib().oracle_granite_logits(self._h, e.reshape(-1), e.shape[0], out.reshape(-1), threads)
        return out

    def frame_ids(self, encoded, threads=1):
        e = _c(encoded, np.float32)
        ids = np.zeros(e.shape[0], np.uint32)
        margin = np.zeros(e.shape[0], np.float32)
        lib().oracle_granite_frame_ids(self._h, e.reshape(-1), e.shape[0], ids, margin, threads)
        return ids, margin


def ctc_tokens(ids, blank=0):
    ids = _c(ids, np.uint32)
    out = np.zeros(3 * max(ids.size, 1), np.uint32)
    n = lib().oracle_ctc_tokens(ids, ids.size, blank, out)
    return [tuple(int(v) for v in out[3 * i:3 * i + 3]) for i in range(n)]


# ---- the Parakeet TDT model ---------------------------------------------------------------------

def _declare_stream(L):
    if getattr(L, "_stream_declared", False):
        return L
    vp = ctypes.c_void_p
    L.oracle_granite_stream_new.restype = vp
    L.oracle_granite_stream_new.argtypes = [vp]
    L.oracle_granite_stream_free.argtypes = [vp]
    L.oracle_granite_stream_set_freeze_lag.argtypes = [vp, _sz]
    L.oracle_granite_stream_push.restype = ctypes.c_int
    L.oracle_granite_stream_push.argtypes = [vp, _f32p, _sz]
    L.oracle_granite_stream_update.restype = ctypes.c_int
    L.oracle_granite_stream_update.argtypes = [vp, ctypes.c_int, ctypes.c_int]
    for name in ("frames", "first_changed", "frozen", "rows"):
        f = getattr(L, f"oracle_granite_stream_{name}")
        f.restype = _sz
        f.argtypes = [vp]
    L.oracle_granite_stream_frame_ids.argtypes = [vp, _u32p]
    L.oracle_granite_stream_layer_output.restype = _sz
    L.oracle_granite_stream_layer_output.argtypes = [vp, ctypes.c_int, vp]
    L.oracle_granite_stream_features.restype = _sz
    L.oracle_granite_stream_features.argtypes = [vp, vp]
    L._stream_declared = True
    return L


class GraniteStream:
    """GraniteStream (src/granite_stream.rs) over an oracle Granite model: push 16 kHz samples,
    update (finished or not), read frame ids, the first changed frame, the frozen frame, and
    each block's outputs so far."""

    def __init__(self, model: "Granite"):
        self.model = model
        self.L = _declare_stream(lib())
        self._h = self.L.oracle_granite_stream_new(model._h)
        self.d = model.config["d_model"]

    def __del__(self):
        try:
            if self._h:
                self.L.oracle_granite_stream_free(self._h)
                self._h = None
        except Exception:
            pass

    def set_freeze_lag(self, frames):
        self.L.oracle_granite_stream_set_freeze_lag(self._h, frames)

    def push(self, samples):
        x = _c(samples, np.float32).reshape(-1)
        if self.L.oracle_granite_stream_push(self._h, x, x.size) != 0:
            raise ValueError("audio pushed after the stream finished")

    def update(self, finished=False, threads=1):
        if self.L.oracle_granite_stream_update(self._h, int(finished), threads) != 0:
            raise ValueError("the stream already finished")

    def frame_ids(self):
        out = np.zeros(self.L.oracle_granite_stream_frames(self._h), np.uint32)
        self.L.oracle_granite_stream_frame_ids(self._h, out)
        return out

    def first_changed(self):
        return self.L.oracle_granite_stream_first_changed(self._h)

    def frozen(self):
        return self.L.oracle_granite_stream_frozen(self._h)

    def layer_output(self, layer):
        rows = self.L.oracle_granite_stream_layer_output(self._h, layer, None)
        out = np.zeros((rows, self.d), np.float32)
        self.L.oracle_granite_stream_layer_output(self._h, layer, out.ctypes.data)
        return out

    def features(self):
        rows = self.L.oracle_granite_stream_features(self._h, None)
        out = np.zeros((rows, 4 * self.model.config["n_mels"]), np.float32)
        self.L.oracle_granite_stream_features(self._h, out.ctypes.data)
        return out


class ParakeetConfig(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in (
        "d_model", "heads", "layers", "ff", "conv_kernel", "sub_channels", "n_mels",
        "pred_hidden", "pred_layers", "vocab", "blank", "n_durations")] + [
        ("durations", ctypes.c_int * 8), ("max_symbols", ctypes.c_int)]


def _parakeet_lib():
    L = lib()
    if getattr(L, "_parakeet_declared", False):
        return L
    L.oracle_parakeet_new.restype = ctypes.c_void_p
    L.oracle_parakeet_new.argtypes = [ctypes.POINTER(ParakeetConfig)]
    L.oracle_parakeet_free.argtypes = [ctypes.c_void_p]
    L.oracle_parakeet_set_matrix_q8_0.restype = ctypes.c_int
    L.oracle_parakeet_set_matrix_q8_0.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _sz, _sz, _i8p,
                                                  _f32p]
    L.oracle_parakeet_set_matrix.restype = ctypes.c_int
    L.oracle_parakeet_set_matrix.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _sz, _sz, _i8p,
                                             _f32p]
    L.oracle_parakeet_set_vector.restype = ctypes.c_int
    L.oracle_parakeet_set_vector.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _sz, _f32p]
    L.oracle_parakeet_frames_for.restype = _sz
    L.oracle_parakeet_frames_for.argtypes = [_sz]
    L.oracle_parakeet_positions.argtypes = [_sz, _sz, _f32p]
    L.oracle_parakeet_encode.restype = ctypes.c_long
    L.oracle_parakeet_encode.argtypes = [ctypes.c_void_p, _f32p, _sz, _f32p, ctypes.c_int,
                                         ctypes.c_int]
    L.oracle_parakeet_decode.restype = _sz
    L.oracle_parakeet_decode.argtypes = [ctypes.c_void_p, _f32p, _sz, _u32p,
                                         ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    L.oracle_parakeet_decode_sure.restype = _sz
    L.oracle_parakeet_decode_sure.argtypes = [ctypes.c_void_p, _f32p, _sz, _u32p,
                                              ctypes.POINTER(ctypes.c_float), ctypes.c_float,
                                              ctypes.POINTER(_sz), ctypes.c_int]
    L.oracle_tdt_step.restype = ctypes.c_int
    L.oracle_tdt_step.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                  ctypes.c_int, ctypes.c_int, ctypes.POINTER(_sz),
                                  ctypes.POINTER(ctypes.c_int), _u32p]
    L.oracle_parakeet_enc_proj.argtypes = [ctypes.c_void_p, _f32p, _sz, _f32p, ctypes.c_int]
    L.oracle_parakeet_joint.argtypes = [ctypes.c_void_p, _f32p, _f32p, _sz, _f32p]
    L.oracle_parakeet_predict.argtypes = [ctypes.c_void_p, _i32p, _sz, _f32p, _f32p]
    L._parakeet_declared = True
    return L


def tdt_step(logits, vocab, blank, durations, max_symbols, t, on_frame):
    """One greedy TDT step after the joint: (token (id, frame, duration) or None, t, on_frame)."""
    lg = _c(logits, np.float32).reshape(-1)
    durs = (ctypes.c_int * len(durations))(*[int(x) for x in durations])
    tt = _sz(t)
    on = ctypes.c_int(on_frame)
    tok = np.zeros(3, np.uint32)
    emitted = _parakeet_lib().oracle_tdt_step(lg, vocab, blank, durs, len(durations), max_symbols,
                                              ctypes.byref(tt), ctypes.byref(on), tok)
    return (tuple(int(v) for v in tok) if emitted else None), tt.value, on.value


def parakeet_frames_for(feature_frames):
    return _parakeet_lib().oracle_parakeet_frames_for(feature_frames)


def parakeet_positions(t, d):
    out = np.zeros((2 * t - 1, d), np.float32)
    _parakeet_lib().oracle_parakeet_positions(t, d, out.reshape(-1))
    return out


class Parakeet:
    """The oracle's Parakeet TDT model, filled from the same named entries as the CUDA model."""

    def __init__(self, config: dict, entries: dict):
        L = _parakeet_lib()
        cfg = ParakeetConfig()
        for key in ("d_model", "heads", "layers", "ff", "conv_kernel", "sub_channels", "n_mels",
                    "pred_hidden", "pred_layers", "vocab", "blank", "max_symbols"):
            setattr(cfg, key, int(config[key]))
        cfg.n_durations = len(config["durations"])
        for i, v in enumerate(config["durations"]):
            cfg.durations[i] = int(v)
        self.config = dict(config)
        self._h = L.oracle_parakeet_new(ctypes.byref(cfg))
        if not self._h:
            raise ValueError("the Parakeet config does not fit together")
        for name, entry in entries.items():
            if isinstance(entry, tuple):
                values, scales, n, k = entry[:4]
                q8 = len(entry) > 4 and entry[4] == "q8_0"
                setter = L.oracle_parakeet_set_matrix_q8_0 if q8 else L.oracle_parakeet_set_matrix
                rc = setter(self._h, name.encode(), n, k, _c(values, np.int8), _c(scales, np.float32))
            else:
                data = _c(entry, np.float32).reshape(-1)
                rc = L.oracle_parakeet_set_vector(self._h, name.encode(), data.size, data)
            if rc != 0:
                raise ValueError(f"bad entry {name}")

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                _parakeet_lib().oracle_parakeet_free(self._h)
                self._h = None
        except Exception:
            pass

    def encode(self, features, tap_layer=-1, threads=1):
        f = _c(features, np.float32)
        t = parakeet_frames_for(f.shape[0])
        out = np.zeros((max(t, 1), self.config["d_model"]), np.float32)
        got = _parakeet_lib().oracle_parakeet_encode(self._h, f.reshape(-1), f.shape[0],
                                                     out.reshape(-1), tap_layer, threads)
        if got < 0:
            raise ValueError("no feature frames")
        return out[:got]

    def decode(self, encoded, threads=1):
        """Greedy TDT: ([(id, frame, duration), ...], smallest top-2 logit gap)."""
        e = _c(encoded, np.float32)
        frames = e.shape[0]
        cap = frames * (self.config["max_symbols"] + 1) + 1
        out = np.zeros(3 * cap, np.uint32)
        margin = ctypes.c_float()
        n = _parakeet_lib().oracle_parakeet_decode(self._h, e.reshape(-1), frames, out,
                                                   ctypes.byref(margin), threads)
        return [tuple(int(v) for v in out[3 * i:3 * i + 3]) for i in range(n)], margin.value

    def decode_sure(self, encoded, threshold=1e-2, threads=1):
        """Greedy TDT: ([(id, frame, duration), ...], sure), where the first ``sure`` tokens were
        emitted before any joint step whose top-2 logit gap (token or duration) is at or below
        ``threshold``: the prefix a decoder whose logits are that close must reproduce."""
        e = _c(encoded, np.float32)
        frames = e.shape[0]
        cap = frames * (self.config["max_symbols"] + 1) + 1
        out = np.zeros(3 * cap, np.uint32)
        margin = ctypes.c_float()
        sure = _sz()
        n = _parakeet_lib().oracle_parakeet_decode_sure(self._h, e.reshape(-1), frames, out,
                                                        ctypes.byref(margin), threshold,
                                                        ctypes.byref(sure), threads)
        return [tuple(int(v) for v in out[3 * i:3 * i + 3]) for i in range(n)], int(sure.value)

    # The networks the biased beam search reads (src/parakeet.rs:1641-1676).
    def enc_proj(self, encoded, threads=1):
        e = _c(encoded, np.float32)
        out = np.zeros((e.shape[0], self.config["pred_hidden"]), np.float32)
        _parakeet_lib().oracle_parakeet_enc_proj(self._h, e.reshape(-1), e.shape[0], out.reshape(-1),
                                                 threads)
        return out

    def joint(self, enc_row, preds):
        p = _c(preds, np.float32)
        rows = p.shape[0]
        out = np.zeros((rows, self.config["vocab"] + len(self.config["durations"])), np.float32)
        _parakeet_lib().oracle_parakeet_joint(self._h, _c(enc_row, np.float32).reshape(-1),
                                              p.reshape(-1), rows, out.reshape(-1))
        return out

    def predict(self, tokens, states):
        """predict_rows: (new states [rows, layers * 2 * h], preds [rows, h])."""
        t = _c(tokens, np.int32).reshape(-1)
        st = np.array(states, np.float32, copy=True)
        preds = np.zeros((t.size, self.config["pred_hidden"]), np.float32)
        _parakeet_lib().oracle_parakeet_predict(self._h, t, t.size, st.reshape(-1), preds.reshape(-1))
        return st, preds
