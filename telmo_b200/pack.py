"""The reference's weight file (a pack, src/pack.rs) over the C ABI: open a pack, list its
entries, read config.json, and load Granite or Parakeet models from it onto the GPU."""

from __future__ import annotations

import ctypes
import json
import struct
from typing import List, Optional

import numpy as np

from . import _lib
from ._lib import TelmoError

KINDS = {0: "matrix", 1: "f32", 2: "bytes", 3: "device"}
PRECISIONS = {v: k for k, v in _lib.PRECISIONS.items()}


def _fail(rc: int):
    raise TelmoError(rc, _lib.load().telmo_pack_last_error().decode())


class Pack:
    """Pack::open / Pack::from_bytes (src/pack.rs:78-259): the whole file read into memory and its
    index checked before anything is used."""

    def __init__(self, path: Optional[str] = None, data: Optional[bytes] = None, _handle=None):
        L = _lib.load()
        h = ctypes.c_void_p()
        if _handle is not None:
            self._h = _handle
            return
        if data is not None:
            self._data = bytes(data)
            rc = L.telmo_pack_from_bytes(self._data, len(self._data), ctypes.byref(h))
        else:
            rc = L.telmo_pack_open(str(path).encode(), ctypes.byref(h))
        if rc:
            _fail(rc)
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().telmo_pack_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    @property
    def model(self) -> str:
        return _lib.load().telmo_pack_model(self._h).decode()

    def meta(self, key: str) -> Optional[str]:
        v = _lib.load().telmo_pack_meta(self._h, key.encode())
        return v.decode() if v is not None else None

    def entries(self) -> List[dict]:
        L = _lib.load()
        out = []
        for i in range(L.telmo_pack_entry_count(self._h)):
            name = ctypes.c_char_p()
            kind, prec = ctypes.c_int(), ctypes.c_int()
            n, k, nb = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
            rc = L.telmo_pack_entry_info(self._h, i, ctypes.byref(name), ctypes.byref(kind), ctypes.byref(prec),
                                         ctypes.byref(n), ctypes.byref(k), ctypes.byref(nb))
            if rc:
                _fail(rc)
            e = {"name": name.value.decode(), "kind": KINDS[kind.value], "bytes": nb.value}
            if kind.value in (0, 3):
                e.update(precision=PRECISIONS[prec.value], n=n.value, k=k.value)
            out.append(e)
        return out

    def to_device(self) -> "Pack":
        """The same pack with its Int8 and Q8_0 matrices in the device layout (an extension of the
        reference's format: loading it skips the host-side panel repack). Host only."""
        h = ctypes.c_void_p()
        rc = _lib.load().telmo_pack_to_device(self._h, ctypes.byref(h))
        if rc:
            _fail(rc)
        return Pack(_handle=h)

    def save(self, path) -> None:
        rc = _lib.load().telmo_pack_save(self._h, str(path).encode())
        if rc:
            _fail(rc)

    def bytes(self, name: str) -> bytes:
        data = ctypes.c_void_p()
        n = ctypes.c_size_t()
        rc = _lib.load().telmo_pack_bytes(self._h, name.encode(), ctypes.byref(data), ctypes.byref(n))
        if rc:
            _fail(rc)
        return ctypes.string_at(data.value, n.value) if n.value else b""


def write_pack(model, entries, metadata=None, version=1):
    """A pack file's bytes in the reference's format (FileSink, src/pack.rs:470-620): "TELMOPAK", the
    format version and 4 zero bytes; each entry's data at a multiple of 64 bytes; the JSON index;
    the index's offset and length (u64s) and "TELMOIDX". entries: name -> a matrix in the
    reference's panels as (values, scales, n, k[, "q8_0"]), an f32 array, or bytes."""
    data = bytearray(b"TELMOPAK" + struct.pack("<I", version) + b"\0" * 4)
    index = []

    def put(blob):
        while len(data) % 64:
            data.append(0)
        at = len(data)
        data.extend(blob)
        return at

    for name, e in entries.items():
        if isinstance(e, (bytes, bytearray)):
            at = put(bytes(e))
            index.append({"name": name, "type": "bytes", "offset": at, "bytes": len(e)})
        elif isinstance(e, tuple):
            values, scales, n, k = e[:4]
            precision = e[4] if len(e) > 4 else "int8"
            v = np.ascontiguousarray(values, np.int8).tobytes()
            s = np.ascontiguousarray(scales, np.float32).tobytes()
            at = put(v)
            s_at = put(s)
            index.append({"name": name, "type": "matrix", "precision": precision, "n": n, "k": k,
                          "offset": at, "bytes": len(v), "scales_offset": s_at, "scales_bytes": len(s)})
        else:
            a = np.ascontiguousarray(e, np.float32)
            at = put(a.tobytes())
            index.append({"name": name, "type": "f32", "shape": list(a.shape), "offset": at,
                          "bytes": a.nbytes})
    idx = json.dumps({"model": model, "metadata": metadata or {}, "entries": index}).encode()
    at = len(data)
    data.extend(idx)
    data.extend(struct.pack("<QQ", at, len(idx)) + b"TELMOIDX")
    return bytes(data)



def granite_config_json(c) -> bytes:
    """A Granite config dict as the config.json that Config::from_json (src/granite.rs:60-146) reads."""
    return json.dumps({
        "model_type": "granite_speech5_ctc", "vocab_size": c["vocab"], "pad_token_id": c["blank"],
        "encoder_config": {
            "model_type": "granite_speech5_encoder", "hidden_size": c["d_model"],
            "num_attention_heads": c["heads"], "head_dim": c["head_dim"],
            "num_hidden_layers": c["layers"], "intermediate_size": c["ff"],
            "conv_kernel_size": c["conv_kernel"],
            "conv_expansion_factor": c["conv_channels"] // c["d_model"],
            "num_mel_bins": c["n_mels"], "context_size": c["context"],
            "max_position_embeddings": c["max_relative"], "vocab_size": c["vocab"],
            "subsample_layers": list(c["subsample_layers"])}}).encode()


def parakeet_config_json(c) -> bytes:
    """A Parakeet config dict as the config.json that Config::from_json (src/parakeet.rs:70-141) reads."""
    return json.dumps({
        "model_type": "parakeet_tdt", "hidden_act": "relu", "vocab_size": c["vocab"],
        "blank_token_id": c["blank"], "decoder_hidden_size": c["pred_hidden"],
        "num_decoder_layers": c["pred_layers"], "max_symbols_per_step": c["max_symbols"],
        "durations": list(c["durations"]),
        "encoder_config": {
            "hidden_act": "silu", "attention_bias": False, "convolution_bias": False,
            "scale_input": False, "subsampling_factor": 8, "subsampling_conv_kernel_size": 3,
            "subsampling_conv_stride": 2, "hidden_size": c["d_model"],
            "num_attention_heads": c["heads"], "num_hidden_layers": c["layers"],
            "intermediate_size": c["ff"], "conv_kernel_size": c["conv_kernel"],
            "subsampling_conv_channels": c["sub_channels"], "num_mel_bins": c["n_mels"]}}).encode()


def granite_config_from_json(text) -> dict:
    """Config::from_json (src/granite.rs:60-146) as the config dict Granite takes."""
    raw = text.encode() if isinstance(text, str) else bytes(text)
    cfg = _lib.GraniteConfig()
    rc = _lib.load().telmo_granite_config_from_json(raw, len(raw), ctypes.byref(cfg))
    if rc:
        _fail(rc)
    c = {name: getattr(cfg, name) for name in ("d_model", "heads", "head_dim", "layers", "ff", "conv_kernel",
                                               "conv_channels", "n_mels", "context", "max_relative", "vocab",
                                               "blank")}
    c["subsample_layers"] = [cfg.subsample_layers[i] for i in range(cfg.n_subsample)]
    return c


def parakeet_config_from_json(text) -> dict:
    """Config::from_json (src/parakeet.rs:70-141) as the config dict Parakeet takes."""
    raw = text.encode() if isinstance(text, str) else bytes(text)
    cfg = _lib.ParakeetConfig()
    rc = _lib.load().telmo_parakeet_config_from_json(raw, len(raw), ctypes.byref(cfg))
    if rc:
        _fail(rc)
    c = {name: getattr(cfg, name) for name in ("d_model", "heads", "layers", "ff", "conv_kernel", "sub_channels",
                                               "n_mels", "pred_hidden", "pred_layers", "vocab", "blank",
                                               "max_symbols")}
    c["durations"] = [cfg.durations[i] for i in range(cfg.n_durations)]
    return c
