"""Decoding that favours special words over the models' GPU networks, against the same search run
by the oracle's restatement (oracle/biasing.py) over the oracle's networks (Granite::decode_biased,
src/granite.rs:584-604; Parakeet::beam_search, src/parakeet.rs:1360-1410).

Bars: token (id, frame, duration) lists identical to the oracle's wherever the oracle's greedy
decode has a top-2 logit margin above 1e-2 (the north star's rule for ids), on the conditioned
tiny models; a beam of one without a bonus gives the greedy decoder's tokens.
"""

import numpy as np
import pytest

from oracle import biasing as ob
from telmo_b200 import biasing as tb
from telmo_b200 import synthetic

pytestmark = pytest.mark.gpu

PARAKEET = synthetic.parakeet_config(layers=2, d_model=128, heads=2, ff=256, sub_channels=32,
                                     pred_hidden=64, vocab=65, blank=64)
GRANITE = synthetic.granite_config(d_model=128, heads=2, head_dim=64, layers=4, ff=256, conv_channels=256,
                                   conv_kernel=5, context=16, max_relative=32, vocab=33, n_mels=8)


def _flags(vocab, blank):
    """A synthetic vocabulary: every third token starts a word, every token but the blank holds a
    letter."""
    boundary = np.array([t % 3 == 0 or t == blank for t in range(vocab)], np.uint8)
    wordlike = np.array([t != blank for t in range(vocab)], np.uint8)
    return boundary, wordlike


def _words(forms, vocab, blank, **boost):
    boundary, wordlike = _flags(vocab, blank)
    letters = [2 + 2 * len(f) for f in forms]
    b = tb.Boost(**boost)
    lib = tb.Words(forms, letters, boundary, wordlike, b)
    ora = ob.Words(forms, letters, boundary, wordlike, b.bonus, b.beam, b.spotting_bonus, b.spotting_margin,
                   b.short_word_margin)
    return lib, ora


@pytest.fixture(scope="module")
def parakeet(ctx, oracle_lib):
    from telmo_b200.parakeet import Parakeet
    entries = synthetic.parakeet_entries(PARAKEET, seed=21, scales="conditioned")
    return Parakeet.from_entries(ctx, PARAKEET, entries), oracle_lib.Parakeet(PARAKEET, entries)


@pytest.fixture(scope="module")
def granite(ctx, oracle_lib):
    from telmo_b200.granite import Granite
    entries = synthetic.granite_entries(GRANITE, seed=11)
    return Granite.from_entries(ctx, GRANITE, entries), oracle_lib.Granite(GRANITE, entries)


def _parakeet_forms(greedy, seed):
    """Special words near what the model says: runs of two or three of its tokens with one
    replaced, and one run as said."""
    r = np.random.default_rng(seed)
    ids = [t[0] for t in greedy]
    forms = []
    for _ in range(4):
        if len(ids) < 3:
            break
        at = int(r.integers(0, len(ids) - 2))
        f = ids[at:at + int(r.integers(2, 4))]
        f[int(r.integers(0, len(f)))] = int(r.integers(0, PARAKEET["blank"]))
        forms.append(f)
    if len(ids) >= 2:
        forms.append(ids[:2])
    return forms or [[1, 2]]


def _oracle_beam(ref, enc, ora_words):
    c = PARAKEET
    h, L = c["pred_hidden"], c["pred_layers"]
    ep = ref.enc_proj(enc)
    state, pred = ref.predict([c["blank"]], np.zeros((1, L * 2 * h), np.float32))
    return ob.beam_search(ora_words, lambda f, p: ref.joint(ep[f], p), ref.predict, c["vocab"], c["blank"],
                          c["durations"], c["max_symbols"], enc.shape[0], state[0], pred[0])


@pytest.mark.parametrize("case", range(4))
def test_parakeet_beam_search_matches_the_oracle(parakeet, case):
    import torch
    gpu, ref = parakeet
    rows = [203, 450, 130, 330][case]
    # The first of a few seeded utterances whose greedy decode has no near tie.
    for seed in range(300 + 10 * case, 310 + 10 * case):
        enc = ref.encode(synthetic.rng(seed).standard_normal((rows, 128)).astype(np.float32))
        greedy, margin = ref.decode(enc)
        if margin > 1e-2:
            break
    assert margin > 1e-2
    beam = [1, 2, 4, 8][case]
    lib, ora = _words(_parakeet_forms(greedy, case), PARAKEET["vocab"], PARAKEET["blank"], bonus=2.0, beam=beam)
    got = gpu.beam_search(torch.from_numpy(enc).cuda(), lib)
    gpu.ctx.check()
    want = _oracle_beam(ref, enc, ora)
    assert [tuple(int(x) for x in t) for t in got] == [tuple(t) for t in want]
    assert len(want) > 0


def test_parakeet_beam_of_one_without_a_bonus_decodes_greedily(parakeet):
    # src/biasing/tdt_beam.rs:459-503 on the real networks: the GPU beam search with beam 1 and
    # no bonus gives the GPU greedy decoder's tokens.
    import torch
    gpu, ref = parakeet
    compared = 0
    for i, rows in enumerate([203, 450, 57, 330, 260, 130]):
        enc = ref.encode(synthetic.rng(320 + i).standard_normal((rows, 128)).astype(np.float32))
        want, margin = ref.decode(enc)
        if margin <= 1e-2:
            continue
        lib, _ = _words([[1, 2, 3]], PARAKEET["vocab"], PARAKEET["blank"], bonus=0.0, beam=1)
        e = torch.from_numpy(enc).cuda()
        got = gpu.beam_search(e, lib)
        greedy = gpu.decode(e, [enc.shape[0]])[0]
        gpu.ctx.check()
        assert [tuple(int(x) for x in t) for t in got] == [(t.id, t.frame, t.duration) for t in greedy] == want
        compared += 1
    assert compared >= 2


def test_parakeet_beam_search_continues_from_a_state(parakeet):
    # Parakeet::beam_search from a later frame and offset (the streaming caller's form): the state
    # after the greedy tokens that end by frame 8, the encoder frames from 3 on, token frames
    # counted from the utterance's start.
    import torch
    gpu, ref = parakeet
    c = PARAKEET
    h, L = c["pred_hidden"], c["pred_layers"]
    enc = ref.encode(synthetic.rng(340).standard_normal((330, 128)).astype(np.float32))
    greedy, _ = ref.decode(enc)
    lib, ora = _words(_parakeet_forms(greedy, 9), c["vocab"], c["blank"], bonus=2.0, beam=4)
    state, pred = ref.predict([c["blank"]], np.zeros((1, L * 2 * h), np.float32))
    frame = 0
    for tok, f, d in greedy:
        if frame >= 8:
            break
        state, pred = ref.predict([tok], state)
        frame = f + max(d, 1)
    offset = 3
    assert frame >= offset
    got = gpu.beam_search(torch.from_numpy(enc[offset:]).cuda(), lib, offset=offset,
                          state=(state[0], pred[0], frame, 0))
    gpu.ctx.check()
    ep = ref.enc_proj(enc[offset:])
    want = ob.beam_search(ora, lambda f, p: ref.joint(ep[f], p), ref.predict, c["vocab"], c["blank"], c["durations"],
                          c["max_symbols"], enc.shape[0] - offset, state[0], pred[0], start_frame=frame - offset)
    assert [tuple(int(x) for x in t) for t in got] == [(i, f + offset, d) for i, f, d in want]
    assert all(t[1] >= frame for t in got)


def _granite_forms(logits, seed):
    """Special words near what the model says: the second-best tokens over a few frames, and the
    best tokens with one replaced by the second best."""
    r = np.random.default_rng(seed)
    order = np.argsort(-logits, axis=1)
    forms = []
    for _ in range(4):
        at = int(r.integers(0, logits.shape[0] - 3))
        n = int(r.integers(1, 4))
        f = [int(order[at + i, 1]) for i in range(n)]
        forms.append([t if t != 0 else int(order[at, 2]) for t in f])
    return forms


@pytest.mark.parametrize("case", range(4))
def test_granite_decode_biased_matches_the_oracle(granite, case):
    import torch
    gpu, ref = granite
    rows = [130, 61, 250, 90][case]
    # The first of a few seeded utterances whose greedy ids have no near tie.
    for seed in range(400 + 10 * case, 410 + 10 * case):
        enc = ref.encode(synthetic.rng(seed).standard_normal((rows, 32)).astype(np.float32))
        logits = ref.logits(enc)
        top2 = np.sort(logits, axis=1)[:, -2:]
        if np.min(top2[:, 1] - top2[:, 0]) > 1e-2:
            break
    assert np.min(top2[:, 1] - top2[:, 0]) > 1e-2
    forms = _granite_forms(logits, case)
    lib, ora = _words(forms, GRANITE["vocab"], GRANITE["blank"], spotting_bonus=[2.0, 4.0, 6.0, 8.0][case],
                      spotting_margin=[0.0, 1.0, 2.0, 0.5][case])
    got = gpu.decode_biased(torch.from_numpy(enc).cuda(), lib)
    gpu.ctx.check()
    greedy = ob.ctc_tokens(logits.argmax(axis=1), GRANITE["blank"])
    want, _ = ob.spot(ora, greedy, tb.score_rows(logits, GRANITE["blank"], np.array(ora.tokens)))
    assert [tuple(int(x) for x in t) for t in got] == want


def test_granite_decode_biased_spots_and_keeps_greedy_text_elsewhere(granite):
    # A strong bonus makes spotting replace words; without forms the result is the greedy text.
    import torch
    gpu, ref = granite
    enc = ref.encode(synthetic.rng(420).standard_normal((200, 32)).astype(np.float32))
    logits = ref.logits(enc)
    greedy = ob.ctc_tokens(logits.argmax(axis=1), GRANITE["blank"])
    e = torch.from_numpy(enc).cuda()
    empty, _ = _words([], GRANITE["vocab"], GRANITE["blank"])
    assert [tuple(int(x) for x in t) for t in gpu.decode_biased(e, empty)] == greedy
    lib, ora = _words(_granite_forms(logits, 7), GRANITE["vocab"], GRANITE["blank"], spotting_bonus=10.0,
                      spotting_margin=0.0, short_word_margin=0.0)
    got = gpu.decode_biased(e, lib)
    gpu.ctx.check()
    want, ranges = ob.spot(ora, greedy, tb.score_rows(logits, GRANITE["blank"], np.array(ora.tokens)))
    assert [tuple(int(x) for x in t) for t in got] == want
    assert len(ranges) >= 1 and want != greedy
