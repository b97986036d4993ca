"""Readers for the reference's golden files (safetensors tensors and 16-bit PCM WAVs).

The reference keeps golden feature tensors for its front ends beside LibriSpeech and FLEURS
clips (tests/goldens/<model>/ in the telmo source tree). They are read in place when a copy of
the telmo source is present: at the path in ``TELMO_REFERENCE``, else in a checkout named
``reference`` beside this repository. Without one the tests that need them skip. The clips are
never copied into this repository.
"""

from __future__ import annotations

import json
import os
import struct
import wave

import numpy as np

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE = os.environ.get("TELMO_REFERENCE") or os.path.join(os.path.dirname(_REPO), "reference")
GOLDENS = os.path.join(REFERENCE, "tests", "goldens")

_DTYPES = {"F32": np.float32, "F64": np.float64, "I64": np.int64, "I32": np.int32,
           "U32": np.uint32, "F16": np.float16, "U8": np.uint8, "I8": np.int8}


def available() -> bool:
    return os.path.isdir(GOLDENS)


def read_safetensors(path: str) -> dict:
    with open(path, "rb") as f:
        raw = f.read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + hlen])
    base = 8 + hlen
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        a, b = info["data_offsets"]
        arr = np.frombuffer(raw[base + a:base + b], dtype=_DTYPES[info["dtype"]])
        out[name] = arr.reshape(info["shape"])
    return out


def read_wav(path: str) -> np.ndarray:
    """16 kHz mono 16-bit PCM as float32 int16/32768 (the reference's wav::read)."""
    with wave.open(path, "rb") as w:
        assert w.getsampwidth() == 2 and w.getnchannels() == 1 and w.getframerate() == 16000
        data = np.frombuffer(w.readframes(w.getnframes()), dtype="<i2")
    return (data.astype(np.float32) / np.float32(32768.0)).astype(np.float32)


def clips(model: str):
    """(id, samples, tensors) for every clip of a golden manifest."""
    d = os.path.join(GOLDENS, model)
    with open(os.path.join(d, "manifest.json")) as f:
        manifest = json.load(f)
    for clip in manifest["clips"]:
        yield clip["id"], read_wav(os.path.normpath(os.path.join(d, clip["wav"]))), \
            read_safetensors(os.path.join(d, clip["tensors"]))
