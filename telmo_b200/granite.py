"""The Granite Speech CTC model on the GPU: the reference's Granite interface (src/granite.rs)
over the C ABI.

``Granite.from_entries`` plays the part of ``Granite::from_pack`` (named pack entries), and
``encode`` / ``frame_ids`` / ``ctc_logits`` / ``ctc_tokens`` / ``transcribe`` mirror the
reference's methods, extended to batches of utterances whose rows are packed one after another.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Sequence

import numpy as np

from . import _lib
from ._lib import TelmoError, check


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


@dataclass
class Token:
    """A CTC token: its id, the frame its run starts on and the run's length (src/parakeet.rs)."""
    id: int
    frame: int
    duration: int


def config_struct(config: dict) -> _lib.GraniteConfig:
    cfg = _lib.GraniteConfig()
    for key in ("d_model", "heads", "head_dim", "layers", "ff", "conv_kernel", "conv_channels",
                "n_mels", "context", "max_relative", "vocab", "blank"):
        setattr(cfg, key, int(config[key]))
    subs = list(config["subsample_layers"])
    if len(subs) > 8:
        raise TelmoError(_lib.TELMO_ERR_MODEL, "too many subsample layers")
    cfg.n_subsample = len(subs)
    for i, s in enumerate(subs):
        cfg.subsample_layers[i] = int(s)
    return cfg


class Granite:
    """A loaded Granite Speech CTC model on one context (src/granite.rs:375-716)."""

    def __init__(self, ctx, config: dict):
        self.ctx = ctx
        self.config = dict(config)
        h = ctypes.c_void_p()
        cfg = config_struct(config)
        check(_lib.load().telmo_granite_create(ctx.handle, ctypes.byref(cfg), ctypes.byref(h)),
              ctx.handle)
        self._h = h

    @staticmethod
    def from_entries(ctx, config: dict, entries: dict) -> "Granite":
        """Builds the model from named pack entries: matrices as (values, scales, n, k) in the
        panel layout (Int8), or (values, scales, n, k, "q8_0") for Q8_0 panels; vectors as f32
        arrays (Granite::from_pack, src/granite.rs:424-500)."""
        g = Granite(ctx, config)
        L = _lib.load()
        for name, entry in entries.items():
            if isinstance(entry, tuple):
                values, scales, n, k = entry[:4]
                precision = _lib.precision_code(entry[4] if len(entry) > 4 else "int8")
                values = np.ascontiguousarray(values, dtype=np.int8)
                scales = np.ascontiguousarray(scales, dtype=np.float32)
                rc = L.telmo_granite_set_matrix(g._h, name.encode(), precision, n, k, values.ctypes.data,
                                                scales.ctypes.data)
            else:
                data = np.ascontiguousarray(entry, dtype=np.float32).reshape(-1)
                rc = L.telmo_granite_set_vector(g._h, name.encode(), data.size, data.ctypes.data)
            check(rc, ctx.handle)
        check(L.telmo_granite_finalize(g._h), ctx.handle)
        return g

    @staticmethod
    def from_pack(ctx, pack) -> "Granite":
        """Granite::from_pack: the config from the pack's config.json, every entry the model knows
        uploaded as it is stored (src/pack.rs, Model::load)."""
        from .pack import granite_config_from_json
        obj = Granite.__new__(Granite)
        obj.ctx = ctx
        obj.config = granite_config_from_json(pack.bytes("config.json"))
        h = ctypes.c_void_p()
        check(_lib.load().telmo_granite_load_pack(ctx.handle, pack.handle, ctypes.byref(h)), ctx.handle)
        obj._h = h
        return obj

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().telmo_granite_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def frames_for(self, rows: int) -> int:
        """Config::frames_for (src/granite.rs:155-158)."""
        return _lib.load().telmo_granite_frames_for(self._h, rows)

    def encode(self, features, rows: Sequence[int], tap_layer: int = -1, stream=None):
        """Granite::encode over a batch. ``features`` is a CUDA f32 tensor [sum(rows), 4 * n_mels];
        returns (encoded CUDA tensor [sum(frames), d_model], frames per utterance)."""
        import torch
        rows_arr = np.ascontiguousarray(rows, dtype=np.int32)
        n = rows_arr.size
        total = sum(self.frames_for(int(r)) for r in rows_arr)
        if tap_layer >= 0:
            total = int(rows_arr.sum())
        out = torch.empty((max(total, 1), self.config["d_model"]), dtype=torch.float32,
                          device=features.device)
        frames = np.zeros(n, np.int32)
        check(_lib.load().telmo_granite_encode(self._h, features.data_ptr(), rows_arr.ctypes.data,
                                               n, out.data_ptr(), frames.ctypes.data, tap_layer,
                                               _stream(stream)), self.ctx.handle)
        return out[:int(frames.sum())], frames

    def ctc_logits(self, encoded, stream=None):
        """Granite::ctc_logits (src/granite.rs:657-673): [frames, vocab]."""
        import torch
        frames = encoded.shape[0]
        ld = (self.config["vocab"] + 3) // 4 * 4
        out = torch.empty((max(frames, 1), ld), dtype=torch.float32, device=encoded.device)
        check(_lib.load().telmo_granite_logits(self._h, encoded.data_ptr(), frames, out.data_ptr(),
                                               ld, _stream(stream)), self.ctx.handle)
        return out[:frames, :self.config["vocab"]]

    def frame_ids(self, encoded, with_margin: bool = False, stream=None):
        """Granite::frame_ids (src/granite.rs:677-716): each frame's first most likely token."""
        import torch
        frames = encoded.shape[0]
        ids = torch.empty(max(frames, 1), dtype=torch.int32, device=encoded.device)
        margin = torch.empty(max(frames, 1), dtype=torch.float32, device=encoded.device) \
            if with_margin else None
        check(_lib.load().telmo_granite_frame_ids(self._h, encoded.data_ptr(), frames,
                                                  ids.data_ptr(),
                                                  margin.data_ptr() if margin is not None else None,
                                                  _stream(stream)), self.ctx.handle)
        if with_margin:
            return ids[:frames], margin[:frames]
        return ids[:frames]

    def ctc_tokens(self, ids, frames: Sequence[int], stream=None) -> List[List[Token]]:
        """ctc_tokens (src/granite.rs:1074-1094) for every utterance of a batch, on the GPU."""
        return ctc_tokens(self.ctx, ids, frames, self.config["blank"], stream)

    def decode_biased(self, encoded, words, stream=None) -> np.ndarray:
        """Granite::decode_biased (src/granite.rs:584-604) up to the text rewrites: greedy CTC
        tokens of one utterance's CUDA encoder output [frames, d_model] with special words
        spotted in (telmo_b200.biasing.Words). Returns (id, frame, duration) tokens [n, 3]."""
        frames = int(encoded.shape[0])
        cap = frames + 16
        out = np.zeros((cap, 3), np.uint32)
        n = ctypes.c_size_t()
        check(_lib.load().telmo_granite_decode_biased(self._h, encoded.data_ptr(), frames, words.handle,
                                                      out.ctypes.data, cap, ctypes.byref(n), _stream(stream)),
              self.ctx.handle)
        return out[:n.value].copy()

    def frames_for_samples(self, samples: int) -> int:
        return _lib.load().telmo_granite_frames_for_samples(self._h, int(samples))

    def transcribe(self, utterances: Sequence[np.ndarray], stream=None) -> List[List[Token]]:
        """Granite::transcribe (src/granite.rs:553-582) up to the token ids, for a batch of 16 kHz
        utterances in host memory."""
        lengths = np.array([len(u) for u in utterances], np.int64)
        samples = np.ascontiguousarray(np.concatenate(utterances), dtype=np.float32)
        return self.transcribe_packed(samples, lengths, stream)

    def transcribe_packed(self, samples: np.ndarray, lengths: np.ndarray, stream=None,
                          tokens_buf: np.ndarray = None):
        """As transcribe, with the utterances already packed one after another (host memory;
        a pinned buffer copies fastest)."""
        tok, counts, frames = self.transcribe_arrays(samples, lengths, stream, tokens_buf)
        out, at = [], 0
        for u in range(len(counts)):
            t = tok[3 * at:3 * at + 3 * counts[u]].reshape(-1, 3)
            out.append([Token(int(a), int(b), int(c)) for a, b, c in t])
            at += int(frames[u])
        return out

    def transcribe_arrays(self, samples, lengths, stream=None, tokens_buf=None):
        """telmo_granite_transcribe as it is: (tokens, counts, frames) host arrays, utterance u's
        counts[u] (id, frame, duration) triples at element 3 * (frames[0] + ... + frames[u-1])
        of tokens."""
        lengths = np.ascontiguousarray(lengths, dtype=np.int64)
        n = lengths.size
        if tokens_buf is not None:  # the caller sized it (3 x the utterances' frames)
            tokens = tokens_buf
        else:
            cap = sum(self.frames_for_samples(int(x)) for x in lengths)
            tokens = np.zeros(3 * max(cap, 1), np.uint32)
        counts = np.zeros(n, np.int32)
        frames = np.zeros(n, np.int32)
        ptr = samples.data_ptr() if hasattr(samples, "data_ptr") else samples.ctypes.data
        tptr = tokens.data_ptr() if hasattr(tokens, "data_ptr") else tokens.ctypes.data
        check(_lib.load().telmo_granite_transcribe(self._h, ptr, lengths.ctypes.data, n, tptr,
                                                   counts.ctypes.data, frames.ctypes.data,
                                                   _stream(stream)), self.ctx.handle)
        tok = tokens if isinstance(tokens, np.ndarray) else tokens.numpy()
        return tok.reshape(-1), counts, frames

    def set_transcribe_group(self, seconds: float):
        """The audio per group of the host-buffer transcription (telmo_granite_transcribe), which
        transcribes one group while the next group's samples are copied to the device."""
        check(_lib.load().telmo_granite_set_transcribe_group(self._h, float(seconds)), self.ctx.handle)

    def transcribe_device(self, samples, lengths, tokens, counts, stream=None):
        """Device-resident variant: samples, tokens [3 * frames] (int32) and counts are CUDA
        tensors; returns the host array of frames per utterance."""
        lengths = np.ascontiguousarray(lengths, dtype=np.int64)
        frames = np.zeros(lengths.size, np.int32)
        check(_lib.load().telmo_granite_transcribe_device(
            self._h, samples.data_ptr(), lengths.ctypes.data, lengths.size, tokens.data_ptr(),
            counts.data_ptr(), frames.ctypes.data, _stream(stream)), self.ctx.handle)
        return frames

    def launches(self) -> int:
        return _lib.load().telmo_granite_launches(self._h)


def logmel(ctx, kind: int, samples, lengths, stream=None):
    """The batched front ends (telmo_logmel): samples a CUDA f32 tensor of every utterance's
    samples one after another; returns (features CUDA tensor, rows per utterance)."""
    import torch
    lengths = np.ascontiguousarray(lengths, dtype=np.int64)
    L = _lib.load()
    rows_total = sum(L.telmo_logmel_rows(kind, int(x)) for x in lengths)
    width = 320 if kind == _lib.FRONTEND_GRANITE else 128
    feats = torch.empty((max(rows_total, 1), width), dtype=torch.float32, device=samples.device)
    rows = np.zeros(lengths.size, np.int32)
    check(L.telmo_logmel(ctx.handle, kind, samples.data_ptr(), lengths.ctypes.data, lengths.size,
                         feats.data_ptr(), rows.ctypes.data, _stream(stream)), ctx.handle)
    return feats[:int(rows.sum())], rows


def ctc_tokens(ctx, ids, frames: Sequence[int], blank: int = 0, stream=None) -> List[List[Token]]:
    import torch
    frames_arr = np.ascontiguousarray(frames, dtype=np.int32)
    first = np.concatenate([[0], np.cumsum(frames_arr)[:-1]]).astype(np.int32)
    n = frames_arr.size
    dev = ids.device
    d_first = torch.from_numpy(first).to(dev)
    d_frames = torch.from_numpy(frames_arr).to(dev)
    tokens = torch.zeros((max(int(frames_arr.sum()), 1), 3), dtype=torch.int32, device=dev)
    counts = torch.zeros(max(n, 1), dtype=torch.int32, device=dev)
    check(_lib.load().telmo_ctc_tokens(ctx.handle, ids.data_ptr(), d_first.data_ptr(),
                                       d_frames.data_ptr(), n, blank, tokens.data_ptr(),
                                       counts.data_ptr(), _stream(stream)), ctx.handle)
    tok = tokens.cpu().numpy()
    cnt = counts.cpu().numpy()
    out = []
    for u in range(n):
        t = tok[first[u]:first[u] + cnt[u]]
        out.append([Token(int(a), int(b), int(c)) for a, b, c in t])
    return out


class GraniteStream:
    """GraniteStream (src/granite_stream.rs) on the GPU: one utterance transcribed while it is
    spoken. ``push`` appends 16 kHz samples, ``update`` encodes what they can change; the frame
    ids so far, the first frame the last update may have changed and the frozen frame follow the
    reference's."""

    def __init__(self, model: "Granite"):
        self.model = model
        self.ctx = model.ctx
        h = ctypes.c_void_p()
        check(_lib.load().telmo_granite_stream_create(model.handle, ctypes.byref(h)), self.ctx.handle)
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().telmo_granite_stream_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_freeze_lag(self, frames: int):
        check(_lib.load().telmo_granite_stream_set_freeze_lag(self._h, int(frames)), self.ctx.handle)

    def push(self, samples):
        x = np.ascontiguousarray(samples, dtype=np.float32).reshape(-1)
        check(_lib.load().telmo_granite_stream_push(self._h, x.ctypes.data, x.size), self.ctx.handle)

    def update(self, finished: bool = False, stream=None):
        check(_lib.load().telmo_granite_stream_update(self._h, int(finished), _stream(stream)),
              self.ctx.handle)

    def frames(self) -> int:
        return _lib.load().telmo_granite_stream_frames(self._h)

    def first_changed(self) -> int:
        return _lib.load().telmo_granite_stream_first_changed(self._h)

    def frozen(self) -> int:
        return _lib.load().telmo_granite_stream_frozen(self._h)

    def frame_ids(self) -> np.ndarray:
        out = np.zeros(self.frames(), np.uint32)
        check(_lib.load().telmo_granite_stream_frame_ids(self._h, out.ctypes.data, out.size),
              self.ctx.handle)
        return out

    def tokens(self) -> List[Token]:
        """The frames so far as CTC tokens (repeats collapsed, blanks dropped; ctc_tokens on the
        GPU)."""
        import torch
        ids = self.frame_ids()
        if ids.size == 0:
            return []
        dev = torch.from_numpy(ids.view(np.int32)).cuda()
        return ctc_tokens(self.ctx, dev, [ids.size], self.model.config["blank"])[0]

    def layer_output(self, layer: int) -> np.ndarray:
        rows = ctypes.c_size_t(0)
        L = _lib.load()
        check(L.telmo_granite_stream_layer_output(self._h, layer, None, 0, ctypes.byref(rows)), self.ctx.handle)
        out = np.zeros((rows.value, self.model.config["d_model"]), np.float32)
        check(L.telmo_granite_stream_layer_output(self._h, layer, out.ctypes.data, rows.value, None),
              self.ctx.handle)
        return out

    def features(self) -> np.ndarray:
        rows = ctypes.c_size_t(0)
        L = _lib.load()
        check(L.telmo_granite_stream_features(self._h, None, 0, ctypes.byref(rows)), self.ctx.handle)
        out = np.zeros((rows.value, 4 * self.model.config["n_mels"]), np.float32)
        check(L.telmo_granite_stream_features(self._h, out.ctypes.data, rows.value, None), self.ctx.handle)
        return out
