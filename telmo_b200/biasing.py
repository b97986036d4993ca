"""Decoding that favours special words (src/biasing.rs, src/biasing/) over the C ABI: the special
words compiled from their token spellings, Granite's CTC word spotting and Parakeet's TDT beam
search. The search logic runs on the host; the models' networks run on the GPU
(`Granite.decode_biased`, `Parakeet.beam_search`). This library has no tokenizer: callers pass
each spelling already split into the model's tokens, plus two flags per vocabulary token."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from ._lib import TelmoError


def _fail(rc: int):
    raise TelmoError(rc, _lib.load().telmo_words_last_error().decode())


@dataclass
class Boost:
    """Boost (src/biasing.rs:40-150), the reference's defaults."""
    bonus: float = 1.5
    beam: int = 4
    spotting_bonus: float = 4.0
    spotting_margin: float = 2.0
    short_word_margin: float = 3.0

    def _c(self) -> _lib.Boost:
        return _lib.Boost(self.bonus, self.beam, self.spotting_bonus, self.spotting_margin, self.short_word_margin)


def token_flags(pieces: Sequence[str], space: str = "▁") -> Tuple[np.ndarray, np.ndarray]:
    """(boundary, wordlike) for a vocabulary of text pieces written with `space` for a leading space
    (special tokens as None): Tokenizer::is_word_boundary (src/tokenizer.rs:278-286) -- the piece
    starts a word or holds no letter or digit -- and whether it holds a letter or digit."""
    boundary = np.ones(len(pieces), np.uint8)
    wordlike = np.zeros(len(pieces), np.uint8)
    for i, p in enumerate(pieces):
        if p is None:
            continue
        text = p.replace(space, " ")
        alnum = any(ch.isalnum() for ch in text)
        boundary[i] = text.startswith(" ") or not alnum
        wordlike[i] = alnum
    return boundary, wordlike


def letters_of(spelling: str) -> int:
    """Letters and digits of a spelling, which set a short word's extra spotting margin."""
    return sum(1 for ch in spelling if ch.isalnum())


class Words:
    """Special words ready for decoding (Compiled, src/biasing.rs:740-870, without the text
    rewrites). forms: each spelling's tokens (the word, its capitalized form, spoken forms' capitals
    as Compiled::new collects them; repeats count once); letters: letters and digits of each
    spelling; boundary, wordlike: per vocabulary token (see `token_flags`)."""

    def __init__(self, forms: Sequence[Sequence[int]], letters: Sequence[int], boundary, wordlike,
                 boost: Optional[Boost] = None):
        self.boost = boost or Boost()
        L = _lib.load()
        self._boundary = np.ascontiguousarray(boundary, np.uint8)
        self._wordlike = np.ascontiguousarray(wordlike, np.uint8)
        if self._boundary.shape != self._wordlike.shape or self._boundary.ndim != 1:
            raise ValueError("boundary and wordlike must be one flag per vocabulary token")
        flat = np.ascontiguousarray([t for f in forms for t in f], np.uint32)
        lengths = np.ascontiguousarray([len(f) for f in forms], np.uintp)
        lets = np.ascontiguousarray(list(letters), np.uintp)
        if len(lets) != len(lengths):
            raise ValueError("one letter count per form")
        h = ctypes.c_void_p()
        c = self.boost._c()
        rc = L.telmo_words_create(len(self._boundary), self._boundary.ctypes.data, self._wordlike.ctypes.data,
                                  flat.ctypes.data if flat.size else None,
                                  lengths.ctypes.data if lengths.size else None,
                                  lets.ctypes.data if lets.size else None, len(lengths), ctypes.byref(c),
                                  ctypes.byref(h))
        if rc:
            _fail(rc)
        self._h = h

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().telmo_words_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def n_forms(self) -> int:
        return _lib.load().telmo_words_forms(self._h)

    @property
    def columns(self) -> np.ndarray:
        """The sorted distinct tokens of all forms: columns 2.. of the score rows."""
        L = _lib.load()
        n = L.telmo_words_columns(self._h, None, 0)
        out = np.zeros(n, np.uint32)
        L.telmo_words_columns(self._h, out.ctypes.data, n)
        return out

    def step(self, state, token: int):
        """The matcher's state after `token` (a state is (node, covered, half); (0, 0, 0) at the
        start) and the change in bonus (Matcher::step, src/biasing.rs:653-670)."""
        s = np.ascontiguousarray(state, np.uint64)
        nxt = np.zeros(3, np.uint64)
        delta = ctypes.c_float()
        rc = _lib.load().telmo_words_step(self._h, s.ctypes.data, token, nxt.ctypes.data, ctypes.byref(delta))
        if rc:
            raise TelmoError(rc, "the list holds no special words")
        return tuple(int(x) for x in nxt), delta.value

    def finish(self, state) -> float:
        """The change in bonus when the audio ends in `state` (Matcher::finish)."""
        s = np.ascontiguousarray(state, np.uint64)
        delta = ctypes.c_float()
        rc = _lib.load().telmo_words_finish(self._h, s.ctypes.data, ctypes.byref(delta))
        if rc:
            raise TelmoError(rc, "the list holds no special words")
        return delta.value


def score_rows(logits: np.ndarray, blank: int, columns: np.ndarray) -> np.ndarray:
    """score_row (src/biasing/spotting.rs:10-15) of host logits [frames, vocab]: each frame's best
    logit, the blank's and the columns' -- the rows `spot` reads."""
    logits = np.asarray(logits, np.float32)
    return np.concatenate([logits.max(axis=1, keepdims=True), logits[:, blank:blank + 1],
                           logits[:, np.asarray(columns, np.int64)]], axis=1).astype(np.float32)


def _tokens_array(tokens) -> np.ndarray:
    a = np.ascontiguousarray(tokens, np.uint32)
    return a.reshape(-1, 3) if a.size else np.zeros((0, 3), np.uint32)


def spot(words: Words, greedy, scores: np.ndarray, first: int = 0):
    """Word spotting (spot, src/biasing/spotting.rs:95-245) of greedy (id, frame, duration) tokens
    of frames first.. against score rows of every frame from 0. Returns the tokens [n, 3] and
    each spotted word's [begin, end) range of them."""
    g = _tokens_array(greedy)
    sc = np.ascontiguousarray(scores, np.float32)
    frames = sc.shape[0] if sc.ndim == 2 else 0
    L = _lib.load()
    cap = len(g) + 64
    while True:
        out = np.zeros((cap, 3), np.uint32)
        ranges = np.zeros((cap, 2), np.uintp)
        n, nr = ctypes.c_size_t(), ctypes.c_size_t()
        rc = L.telmo_spot(words.handle, g.ctypes.data if len(g) else None, len(g),
                          sc.ctypes.data if sc.size else None, frames, first, out.ctypes.data, cap,
                          ctypes.byref(n), ranges.ctypes.data, cap, ctypes.byref(nr))
        if rc and n.value > cap:
            cap = n.value
            continue
        if rc:
            _fail(rc)
        return out[:n.value].copy(), [(int(a), int(b)) for a, b in ranges[:nr.value]]


def tdt_beam_search(words: Words, joint: Callable, predict: Callable, vocab: int, blank: int,
                    durations: Sequence[int], max_symbols: int, frames: int, start_state, start_pred,
                    start_frame: int = 0, start_on_frame: int = 0) -> np.ndarray:
    """tdt_beam::beam_search (src/biasing/tdt_beam.rs:141-401) over Python networks:
    joint(frame, preds [rows, pred_width]) -> [rows, vocab + len(durations)] and
    predict(tokens [rows], states [rows, state_width]) -> (states, preds). Returns (id, frame,
    duration) tokens [n, 3]."""
    state = np.ascontiguousarray(start_state, np.float32).reshape(-1)
    pred = np.ascontiguousarray(start_pred, np.float32).reshape(-1)
    sw, pw = state.size, pred.size
    outputs = vocab + len(durations)
    errors: List[BaseException] = []

    def joint_cb(_user, frame, preds_p, rows, out_p):
        try:
            p = np.ctypeslib.as_array(preds_p, shape=(rows * pw,)).reshape(rows, pw).copy()
            o = np.asarray(joint(int(frame), p), np.float32).reshape(rows, outputs)
            np.ctypeslib.as_array(out_p, shape=(rows * outputs,))[:] = o.reshape(-1)
            return 0
        except BaseException as e:  # reported after the search ends
            errors.append(e)
            return _lib.TELMO_ERR_ARGUMENT

    def predict_cb(_user, tokens_p, rows, states_p, preds_p):
        try:
            t = np.ctypeslib.as_array(tokens_p, shape=(rows,)).copy()
            st = np.ctypeslib.as_array(states_p, shape=(rows * sw,)).reshape(rows, sw).copy() if sw else \
                np.zeros((rows, 0), np.float32)
            new_states, new_preds = predict(t, st)
            if sw:
                np.ctypeslib.as_array(states_p, shape=(rows * sw,))[:] = np.asarray(new_states, np.float32).reshape(-1)
            np.ctypeslib.as_array(preds_p, shape=(rows * pw,))[:] = np.asarray(new_preds, np.float32).reshape(-1)
            return 0
        except BaseException as e:
            errors.append(e)
            return _lib.TELMO_ERR_ARGUMENT

    jf, pf = _lib.TDT_JOINT_FN(joint_cb), _lib.TDT_PREDICT_FN(predict_cb)
    d = np.ascontiguousarray(durations, np.int32)
    L = _lib.load()
    cap = 4 * max(frames, 1) * max_symbols + 16
    out = np.zeros((cap, 3), np.uint32)
    n = ctypes.c_size_t()
    rc = L.telmo_tdt_beam_search(vocab, blank, d.ctypes.data, len(d), max_symbols, sw, pw, jf, pf, None, frames,
                                 start_frame, start_on_frame, state.ctypes.data if sw else None,
                                 pred.ctypes.data if pw else None, words.handle, out.ctypes.data, cap,
                                 ctypes.byref(n))
    if errors:
        raise errors[0]
    if rc:
        _fail(rc)
    return out[:n.value].copy()
