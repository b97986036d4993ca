"""Loads libtelmo_b200.so and declares the C ABI of include/telmo_b200.h for ctypes.

There is no fallback: if the library is missing or cannot load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtelmo_b200.so")

TELMO_OK = 0
TELMO_ERR_ARGUMENT = -1
TELMO_ERR_CUDA = -2
TELMO_ERR_DEVICE_TIMEOUT = -3
TELMO_ERR_UNSUPPORTED = -4
TELMO_ERR_MODEL = -5

# Output element types of telmo_linear (TELMO_DTYPE_*).
DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_I32_PAIR = 2

# Weight precisions (include/telmo_b200.h, telmo's Precision).
PRECISIONS = {"f32": 0, "f16": 1, "bf16": 2, "int8": 3, "q8_0": 4}


def precision_code(name: str) -> int:
    try:
        return PRECISIONS[name]
    except KeyError:
        raise ValueError(f"unknown weight precision {name!r}") from None

_c = ctypes
_vp = _c.c_void_p
_sz = _c.c_size_t
_int = _c.c_int
_float = _c.c_float

# The caller's networks of telmo_tdt_beam_search (telmo_tdt_joint_fn, telmo_tdt_predict_fn).
TDT_JOINT_FN = _c.CFUNCTYPE(_int, _vp, _sz, _c.POINTER(_float), _sz, _c.POINTER(_float))
TDT_PREDICT_FN = _c.CFUNCTYPE(_int, _vp, _c.POINTER(_int), _sz, _c.POINTER(_float), _c.POINTER(_float))


class Boost(ctypes.Structure):
    """telmo_boost (include/telmo_b200.h)."""
    _fields_ = [("bonus", ctypes.c_float), ("beam", ctypes.c_int), ("spotting_bonus", ctypes.c_float),
                ("spotting_margin", ctypes.c_float), ("short_word_margin", ctypes.c_float)]


# name -> (restype, argtypes); every function include/telmo_b200.h declares.
SIGNATURES = {
    "telmo_ctx_create": (_int, [_int, _c.POINTER(_vp)]),
    "telmo_ctx_destroy": (None, [_vp]),
    "telmo_last_error": (_c.c_char_p, [_vp]),
    "telmo_ctx_check": (_int, [_vp, _vp]),
    "telmo_ctx_device": (_int, [_vp]),
    "telmo_encode_int8": (_int, [_vp, _sz, _sz, _vp, _vp]),
    "telmo_encode_q8_0": (_int, [_vp, _sz, _sz, _vp, _vp]),
    "telmo_weights_upload": (_int, [_vp, _int, _sz, _sz, _vp, _vp, _c.POINTER(_vp)]),
    "telmo_weights_free": (None, [_vp]),
    "telmo_weights_shape": (_int, [_vp, _c.POINTER(_sz), _c.POINTER(_sz)]),
    "telmo_linear": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _int, _float, _int, _vp, _int, _sz,
                            _vp]),
    "telmo_quantize_x2": (_int, [_vp, _vp, _sz, _sz, _sz, _vp, _vp, _sz, _vp, _vp]),
    "telmo_conv_module_rows": (_int, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _vp, _vp]),
    "telmo_linear_noalloc": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _int, _float, _int, _vp, _int,
                                    _sz, _vp]),
    "telmo_linear_q": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _vp, _vp, _int, _float, _int, _vp,
                              _int, _sz, _vp]),
    "telmo_granite_create": (_int, [_vp, _vp, _c.POINTER(_vp)]),
    "telmo_granite_free": (None, [_vp]),
    "telmo_granite_set_matrix": (_int, [_vp, _c.c_char_p, _int, _sz, _sz, _vp, _vp]),
    "telmo_granite_set_vector": (_int, [_vp, _c.c_char_p, _sz, _vp]),
    "telmo_granite_finalize": (_int, [_vp]),
    "telmo_granite_frames_for": (_sz, [_vp, _sz]),
    "telmo_granite_encode": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _int, _vp]),
    "telmo_granite_logits": (_int, [_vp, _vp, _sz, _vp, _sz, _vp]),
    "telmo_granite_frame_ids": (_int, [_vp, _vp, _sz, _vp, _vp, _vp]),
    "telmo_ctc_tokens": (_int, [_vp, _vp, _vp, _vp, _int, _c.c_uint32, _vp, _vp, _vp]),
    "telmo_logmel_rows": (_sz, [_int, _c.c_int64]),
    "telmo_logmel": (_int, [_vp, _int, _vp, _vp, _int, _vp, _vp, _vp]),
    "telmo_granite_frames_for_samples": (_sz, [_vp, _c.c_int64]),
    "telmo_granite_transcribe": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "telmo_granite_transcribe_device": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "telmo_granite_set_transcribe_group": (_int, [_vp, _c.c_double]),
    "telmo_granite_launches": (_c.c_long, [_vp]),
    "telmo_pack_open": (_c.c_int, [_c.c_char_p, _vp]),
    "telmo_pack_from_bytes": (_c.c_int, [_c.c_char_p, _sz, _vp]),
    "telmo_pack_free": (None, [_vp]),
    "telmo_pack_last_error": (_c.c_char_p, []),
    "telmo_pack_model": (_c.c_char_p, [_vp]),
    "telmo_pack_meta": (_c.c_char_p, [_vp, _c.c_char_p]),
    "telmo_pack_entry_count": (_sz, [_vp]),
    "telmo_pack_entry_info": (_c.c_int, [_vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp]),
    "telmo_pack_bytes": (_c.c_int, [_vp, _c.c_char_p, _vp, _vp]),
    "telmo_pack_to_device": (_c.c_int, [_vp, _vp]),
    "telmo_pack_save": (_c.c_int, [_vp, _c.c_char_p]),
    "telmo_granite_config_from_json": (_c.c_int, [_c.c_char_p, _sz, _vp]),
    "telmo_parakeet_config_from_json": (_c.c_int, [_c.c_char_p, _sz, _vp]),
    "telmo_granite_load_pack": (_c.c_int, [_vp, _vp, _vp]),
    "telmo_parakeet_load_pack": (_c.c_int, [_vp, _vp, _vp]),
    "telmo_granite_stream_create": (_c.c_int, [_vp, _vp]),
    "telmo_granite_stream_free": (None, [_vp]),
    "telmo_granite_stream_set_freeze_lag": (_c.c_int, [_vp, _c.c_int]),
    "telmo_granite_stream_push": (_c.c_int, [_vp, _vp, _sz]),
    "telmo_granite_stream_update": (_c.c_int, [_vp, _c.c_int, _vp]),
    "telmo_granite_stream_frames": (_sz, [_vp]),
    "telmo_granite_stream_first_changed": (_sz, [_vp]),
    "telmo_granite_stream_frozen": (_sz, [_vp]),
    "telmo_granite_stream_frame_ids": (_c.c_int, [_vp, _vp, _sz]),
    "telmo_granite_stream_layer_output": (_c.c_int, [_vp, _c.c_int, _vp, _sz, _vp]),
    "telmo_granite_stream_features": (_c.c_int, [_vp, _vp, _sz, _vp]),
    "telmo_granite_profile": (_int, [_vp, _int]),
    "telmo_granite_profile_read": (_int, [_vp, _vp, _vp, _vp, _vp]),
    "telmo_parakeet_create": (_int, [_vp, _vp, _c.POINTER(_vp)]),
    "telmo_parakeet_free": (None, [_vp]),
    "telmo_parakeet_set_matrix": (_int, [_vp, _c.c_char_p, _int, _sz, _sz, _vp, _vp]),
    "telmo_parakeet_set_vector": (_int, [_vp, _c.c_char_p, _sz, _vp]),
    "telmo_parakeet_finalize": (_int, [_vp]),
    "telmo_parakeet_frames_for": (_sz, [_sz]),
    "telmo_parakeet_frames_for_samples": (_sz, [_c.c_int64]),
    "telmo_parakeet_encode": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _int, _vp]),
    "telmo_parakeet_decode": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "telmo_parakeet_transcribe": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "telmo_parakeet_transcribe_device": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "telmo_parakeet_launches": (_c.c_long, [_vp]),
    "telmo_parakeet_set_decoder": (_c.c_int, [_vp, _c.c_int]),
    "telmo_parakeet_enc_proj": (_c.c_int, [_vp, _vp, _c.c_size_t, _vp, _vp]),
    "telmo_parakeet_joint": (_c.c_int, [_vp, _vp, _vp, _c.c_int, _vp, _c.c_size_t, _vp]),
    "telmo_parakeet_predict": (_c.c_int, [_vp, _vp, _c.c_int, _vp, _vp, _vp]),
    "telmo_parakeet_last_decoder": (_c.c_int, [_vp]),
    "telmo_parakeet_test_barrier_timeout": (_c.c_int, [_vp, _c.c_int]),
    "telmo_parakeet_decoder_profile": (_c.c_int, [_vp, _c.c_void_p, _c.c_void_p]),
    "telmo_parakeet_profile": (_int, [_vp, _int]),
    "telmo_parakeet_profile_read": (_int, [_vp, _vp, _vp, _vp, _vp]),
    "telmo_boost_default": (None, [_vp]),
    "telmo_words_create": (_int, [_sz, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "telmo_words_free": (None, [_vp]),
    "telmo_words_last_error": (_c.c_char_p, []),
    "telmo_words_forms": (_sz, [_vp]),
    "telmo_words_columns": (_sz, [_vp, _vp, _sz]),
    "telmo_words_step": (_int, [_vp, _vp, _c.c_uint32, _vp, _vp]),
    "telmo_words_finish": (_int, [_vp, _vp, _vp]),
    "telmo_spot": (_int, [_vp, _vp, _sz, _vp, _sz, _sz, _vp, _sz, _vp, _vp, _sz, _vp]),
    "telmo_granite_decode_biased": (_int, [_vp, _vp, _sz, _vp, _vp, _sz, _vp, _vp]),
    "telmo_tdt_beam_search": (_int, [_int, _int, _vp, _int, _int, _sz, _sz, TDT_JOINT_FN, TDT_PREDICT_FN, _vp,
                                     _sz, _sz, _sz, _vp, _vp, _vp, _vp, _sz, _vp]),
    "telmo_parakeet_beam_search": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _sz, _vp, _vp]),
}

FRONTEND_GRANITE = 0
FRONTEND_PARAKEET = 1


class GraniteConfig(ctypes.Structure):
    """telmo_granite_config (include/telmo_b200.h)."""
    _fields_ = [(name, ctypes.c_int) for name in (
        "d_model", "heads", "head_dim", "layers", "ff", "conv_kernel", "conv_channels", "n_mels",
        "context", "max_relative", "n_subsample")] + [
        ("subsample_layers", ctypes.c_int * 8), ("vocab", ctypes.c_int), ("blank", ctypes.c_int)]


class ParakeetConfig(ctypes.Structure):
    """telmo_parakeet_config (include/telmo_b200.h)."""
    _fields_ = [(name, ctypes.c_int) for name in (
        "d_model", "heads", "layers", "ff", "conv_kernel", "sub_channels", "n_mels", "pred_hidden",
        "pred_layers", "vocab", "blank", "n_durations")] + [
        ("durations", ctypes.c_int * 8), ("max_symbols", ctypes.c_int)]


_lib = None


class TelmoError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"telmo status {status}: {message}")
        self.status = status


def load():
    """The loaded library. Raises when it is missing: there is no CPU path behind it."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing; build it with `python -m telmo_b200.build` (the CUDA path "
            "has no fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, ctx=None) -> None:
    if status != TELMO_OK:
        msg = load().telmo_last_error(ctx)
        raise TelmoError(status, msg.decode() if msg else "")
