"""The Parakeet TDT model on the GPU: the reference's Parakeet interface (src/parakeet.rs) over
the C ABI.

``Parakeet.from_entries`` plays the part of ``Parakeet::from_pack`` (named pack entries), and
``encode`` / ``decode`` / ``transcribe`` mirror the reference's methods, extended to batches of
utterances whose rows are packed one after another.
"""

from __future__ import annotations

import ctypes
from typing import List, Sequence

import numpy as np

from . import _lib
from ._lib import TelmoError, check
from .granite import Token, _stream


def config_struct(config: dict) -> _lib.ParakeetConfig:
    cfg = _lib.ParakeetConfig()
    for key in ("d_model", "heads", "layers", "ff", "conv_kernel", "sub_channels", "n_mels",
                "pred_hidden", "pred_layers", "vocab", "blank", "max_symbols"):
        setattr(cfg, key, int(config[key]))
    durations = list(config["durations"])
    if len(durations) > 8:
        raise TelmoError(_lib.TELMO_ERR_UNSUPPORTED, "more than 8 durations")
    cfg.n_durations = len(durations)
    for i, x in enumerate(durations):
        cfg.durations[i] = int(x)
    return cfg


def frames_for(feature_frames: int) -> int:
    """Encoder frames for a number of feature frames (three stride-2 convolutions)."""
    return _lib.load().telmo_parakeet_frames_for(int(feature_frames))


def frames_for_samples(samples: int) -> int:
    return _lib.load().telmo_parakeet_frames_for_samples(int(samples))


class Parakeet:
    """A loaded Parakeet TDT model on one context (src/parakeet.rs:315-327, :672-1596)."""

    def __init__(self, ctx, config: dict):
        self.ctx = ctx
        self.config = dict(config)
        h = ctypes.c_void_p()
        cfg = config_struct(config)
        check(_lib.load().telmo_parakeet_create(ctx.handle, ctypes.byref(cfg), ctypes.byref(h)),
              ctx.handle)
        self._h = h

    @staticmethod
    def from_entries(ctx, config: dict, entries: dict) -> "Parakeet":
        """Builds the model from named pack entries: matrices as (values, scales, n, k) in the
        panel layout (Int8), or (values, scales, n, k, "q8_0") for Q8_0 panels; vectors as f32
        arrays (Parakeet::from_pack, src/parakeet.rs:691-795)."""
        p = Parakeet(ctx, config)
        L = _lib.load()
        for name, entry in entries.items():
            if isinstance(entry, tuple):
                values, scales, n, k = entry[:4]
                precision = _lib.precision_code(entry[4] if len(entry) > 4 else "int8")
                values = np.ascontiguousarray(values, dtype=np.int8)
                scales = np.ascontiguousarray(scales, dtype=np.float32)
                rc = L.telmo_parakeet_set_matrix(p._h, name.encode(), precision, n, k, values.ctypes.data,
                                                 scales.ctypes.data)
            else:
                data = np.ascontiguousarray(entry, dtype=np.float32).reshape(-1)
                rc = L.telmo_parakeet_set_vector(p._h, name.encode(), data.size, data.ctypes.data)
            check(rc, ctx.handle)
        check(L.telmo_parakeet_finalize(p._h), ctx.handle)
        return p

    @staticmethod
    def from_pack(ctx, pack) -> "Parakeet":
        """Parakeet::from_pack: the config from the pack's config.json, every entry the model knows
        uploaded as it is stored (src/pack.rs, Model::load)."""
        from .pack import parakeet_config_from_json
        obj = Parakeet.__new__(Parakeet)
        obj.ctx = ctx
        obj.config = parakeet_config_from_json(pack.bytes("config.json"))
        h = ctypes.c_void_p()
        check(_lib.load().telmo_parakeet_load_pack(ctx.handle, pack.handle, ctypes.byref(h)), ctx.handle)
        obj._h = h
        return obj

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().telmo_parakeet_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, features, rows: Sequence[int], tap_layer: int = -1, stream=None):
        """Parakeet::encode over a batch. ``features`` is a CUDA f32 tensor [sum(rows), n_mels];
        tap_layer -2 stops after the subsampling, i >= 0 after layer i. Returns (encoded CUDA
        tensor [sum(frames), d_model], frames per utterance)."""
        import torch
        rows_arr = np.ascontiguousarray(rows, dtype=np.int32)
        n = rows_arr.size
        total = sum(frames_for(int(r)) for r in rows_arr)
        out = torch.empty((max(total, 1), self.config["d_model"]), dtype=torch.float32,
                          device=features.device)
        frames = np.zeros(n, np.int32)
        check(_lib.load().telmo_parakeet_encode(self._h, features.data_ptr(), rows_arr.ctypes.data,
                                                n, out.data_ptr(), frames.ctypes.data, tap_layer,
                                                _stream(stream)), self.ctx.handle)
        return out[:int(frames.sum())], frames

    def decode_packed(self, encoded, frames: Sequence[int], stream=None):
        """Greedy TDT decoding (Parakeet::decode, src/parakeet.rs:1285-1296) of a batch of
        encoder outputs packed one after another; returns (tokens CUDA int32 [total, 3], counts
        CUDA int32 [n], total)."""
        import torch
        frames_arr = np.ascontiguousarray(frames, dtype=np.int32)
        n = frames_arr.size
        cap = 3 * self.config["max_symbols"] * int(frames_arr.sum()) + 3
        tokens = torch.zeros(cap, dtype=torch.int32, device=encoded.device)
        counts = torch.zeros(max(n, 1), dtype=torch.int32, device=encoded.device)
        total = ctypes.c_long(0)
        check(_lib.load().telmo_parakeet_decode(self._h, encoded.data_ptr(), frames_arr.ctypes.data,
                                                n, tokens.data_ptr(), counts.data_ptr(),
                                                ctypes.byref(total), _stream(stream)),
              self.ctx.handle)
        return tokens[:3 * total.value].view(-1, 3), counts[:n], total.value

    def decode(self, encoded, frames: Sequence[int], stream=None) -> List[List[Token]]:
        """As decode_packed, split into each utterance's tokens."""
        tokens, counts, _ = self.decode_packed(encoded, frames, stream)
        return _split(tokens.cpu().numpy(), counts.cpu().numpy())

    def transcribe(self, utterances: Sequence[np.ndarray], stream=None) -> List[List[Token]]:
        """Parakeet::transcribe (src/parakeet.rs:842-867) up to the token ids, for a batch of
        16 kHz utterances in host memory."""
        lengths = np.array([len(u) for u in utterances], np.int64)
        samples = np.ascontiguousarray(np.concatenate(utterances), dtype=np.float32)
        return self.transcribe_packed(samples, lengths, stream)

    def transcribe_packed(self, samples, lengths, stream=None, tokens_buf=None):
        """As transcribe, with the utterances packed one after another in host memory (a pinned
        buffer copies fastest)."""
        tok, counts, _ = self.transcribe_arrays(samples, lengths, stream, tokens_buf)
        return _split(tok, counts)

    def transcribe_arrays(self, samples, lengths, stream=None, tokens_buf=None):
        """telmo_parakeet_transcribe as it is: (tokens [total, 3], counts, frames) host arrays,
        the triples packed utterance after utterance."""
        lengths = np.ascontiguousarray(lengths, dtype=np.int64)
        n = lengths.size
        if tokens_buf is not None:  # the caller sized it (3 x max_symbols x the frames, + 3)
            tokens = tokens_buf
        else:
            cap = 3 * self.config["max_symbols"] * sum(frames_for_samples(int(x)) for x in lengths) + 3
            tokens = np.zeros(cap, np.uint32)
        counts = np.zeros(n, np.int32)
        frames = np.zeros(n, np.int32)
        ptr = samples.data_ptr() if hasattr(samples, "data_ptr") else samples.ctypes.data
        tptr = tokens.data_ptr() if hasattr(tokens, "data_ptr") else tokens.ctypes.data
        check(_lib.load().telmo_parakeet_transcribe(self._h, ptr, lengths.ctypes.data, n, tptr,
                                                    counts.ctypes.data, frames.ctypes.data,
                                                    _stream(stream)), self.ctx.handle)
        tok = tokens if isinstance(tokens, np.ndarray) else tokens.numpy()
        return tok.reshape(-1)[:3 * int(counts.sum())].reshape(-1, 3), counts, frames

    def transcribe_device(self, samples, lengths, tokens, counts, stream=None):
        """Device-resident variant: samples, tokens (int32, 3 * max_symbols * frames) and counts
        are CUDA tensors; returns the host array of frames per utterance."""
        lengths = np.ascontiguousarray(lengths, dtype=np.int64)
        frames = np.zeros(lengths.size, np.int32)
        check(_lib.load().telmo_parakeet_transcribe_device(
            self._h, samples.data_ptr(), lengths.ctypes.data, lengths.size, tokens.data_ptr(),
            counts.data_ptr(), frames.ctypes.data, _stream(stream)), self.ctx.handle)
        return frames

    # -- the networks the reference's biased beam search reads (src/parakeet.rs:1641-1676) --------
    def enc_proj(self, encoded, stream=None):
        """The joint's projection of encoder frames: CUDA [frames, d_model] -> [frames, h]."""
        import torch
        out = torch.empty((encoded.shape[0], self.config["pred_hidden"]), dtype=torch.float32,
                          device=encoded.device)
        check(_lib.load().telmo_parakeet_enc_proj(self._h, encoded.data_ptr(), encoded.shape[0],
                                                  out.data_ptr(), _stream(stream)), self.ctx.handle)
        return out

    def joint(self, enc_row, preds, stream=None):
        """TdtNetwork::joint: [rows, vocab + durations] for CUDA preds [rows, h] at one projected
        frame enc_row [h]."""
        import torch
        rows = preds.shape[0]
        outputs = self.config["vocab"] + len(self.config["durations"])
        out = torch.empty((rows, outputs), dtype=torch.float32, device=preds.device)
        check(_lib.load().telmo_parakeet_joint(self._h, enc_row.data_ptr(), preds.data_ptr(), rows,
                                               out.data_ptr(), outputs, _stream(stream)),
              self.ctx.handle)
        return out

    def predict(self, tokens, states, preds, stream=None):
        """TdtNetwork::predict: host tokens [rows]; CUDA states [rows, layers * 2 * h] updated in
        place and preds [rows, h] written."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(_lib.load().telmo_parakeet_predict(self._h, t.ctypes.data, t.size, states.data_ptr(),
                                                 preds.data_ptr(), _stream(stream)), self.ctx.handle)

    def beam_search(self, encoded, words, offset: int = 0, state=None, stream=None) -> np.ndarray:
        """Parakeet::beam_search (src/parakeet.rs:1360-1410) on the GPU networks: the TDT beam
        search that favours special words (telmo_b200.biasing.Words) over one utterance's CUDA
        encoder frames [frames, d_model] (its frames from `offset`). state: None for the decoder
        state before any token, else (lstm, pred, frame, on_frame) with host arrays. Returns (id,
        frame, duration) tokens [n, 3], frames counted from the utterance's start."""
        frames = int(encoded.shape[0])
        cap = frames * int(self.config["max_symbols"]) + 16
        out = np.zeros((cap, 3), np.uint32)
        n = ctypes.c_size_t()
        if state is None:
            lstm = pred = None
            frame = on_frame = 0
        else:
            lstm = np.ascontiguousarray(state[0], np.float32)
            pred = np.ascontiguousarray(state[1], np.float32)
            frame, on_frame = int(state[2]), int(state[3])
        check(_lib.load().telmo_parakeet_beam_search(
            self._h, encoded.data_ptr(), frames, offset, None if lstm is None else lstm.ctypes.data,
            None if pred is None else pred.ctypes.data, frame, on_frame, words.handle, out.ctypes.data, cap,
            ctypes.byref(n), _stream(stream)), self.ctx.handle)
        return out[:n.value].copy()

    def set_decoder(self, persistent: bool):
        """1/True: the persistent decoder kernel (the default); 0/False: per-phase launches."""
        check(_lib.load().telmo_parakeet_set_decoder(self._h, int(persistent)), self.ctx.handle)

    def test_barrier_timeout(self, cta: int = 0):
        """Makes the next persistent decode's first grid barrier run out (CTA `cta` never
        arrives): that decode raises TelmoError with TELMO_ERR_DEVICE_TIMEOUT after about a
        second, and the model and context stay usable. A test of the failure path."""
        check(_lib.load().telmo_parakeet_test_barrier_timeout(self._h, int(cta)), self.ctx.handle)

    def last_decoder(self) -> int:
        """1 if the last decode ran the persistent kernel, 0 per-phase launches, -1 none yet."""
        return _lib.load().telmo_parakeet_last_decoder(self._h)

    def decoder_profile(self):
        """The persistent decoder's clock for the last profiled decode: ({phase: ms}, passes)."""
        ms = (ctypes.c_double * 10)()
        passes = ctypes.c_long(0)
        check(_lib.load().telmo_parakeet_decoder_profile(self._h, ms, ctypes.byref(passes)),
              self.ctx.handle)
        names = ("start", "joint", "decide", "lstm", "cell", "pred", "prepare", "cta0_products",
                 "cta0_waiting", "cta0_epilogue")
        return dict(zip(names, list(ms))), passes.value

    def launches(self) -> int:
        return _lib.load().telmo_parakeet_launches(self._h)

    def profile(self, enable: bool = True):
        check(_lib.load().telmo_parakeet_profile(self._h, int(enable)), self.ctx.handle)

    def profile_read(self):
        """(ms[4], launches[4], gemm_ops, gemm_bytes) since the last read; classes as
        telmo_granite_profile_read reports them."""
        ms = (ctypes.c_double * 4)()
        launches = (ctypes.c_long * 4)()
        ops = ctypes.c_double(0.0)
        byts = ctypes.c_double(0.0)
        check(_lib.load().telmo_parakeet_profile_read(self._h, ms, launches, ctypes.byref(ops),
                                                      ctypes.byref(byts)), self.ctx.handle)
        return list(ms), list(launches), ops.value, byts.value


def _split(tokens: np.ndarray, counts: np.ndarray) -> List[List[Token]]:
    out, at = [], 0
    for c in counts:
        t = tokens[at:at + int(c)]
        out.append([Token(int(a), int(b), int(d)) for a, b, d in t])
        at += int(c)
    return out
