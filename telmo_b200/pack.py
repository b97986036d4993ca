"""The reference's weight file (a pack, src/pack.rs) over the C ABI: open a pack, list its
entries, read config.json, and load Granite or Parakeet models from it onto the GPU."""

from __future__ import annotations

import ctypes
from typing import List, Optional

from . import _lib
from ._lib import TelmoError

KINDS = {0: "matrix", 1: "f32", 2: "bytes"}
PRECISIONS = {v: k for k, v in _lib.PRECISIONS.items()}


def _fail(rc: int):
    raise TelmoError(rc, _lib.load().telmo_pack_last_error().decode())


class Pack:
    """Pack::open / Pack::from_bytes (src/pack.rs:78-259): the whole file read into memory and its
    index checked before anything is used."""

    def __init__(self, path: Optional[str] = None, data: Optional[bytes] = None):
        L = _lib.load()
        h = ctypes.c_void_p()
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
            if kind.value == 0:
                e.update(precision=PRECISIONS[prec.value], n=n.value, k=k.value)
            out.append(e)
        return out

    def bytes(self, name: str) -> bytes:
        data = ctypes.c_void_p()
        n = ctypes.c_size_t()
        rc = _lib.load().telmo_pack_bytes(self._h, name.encode(), ctypes.byref(data), ctypes.byref(n))
        if rc:
            _fail(rc)
        return ctypes.string_at(data.value, n.value) if n.value else b""


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
