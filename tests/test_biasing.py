"""Decoding that favours special words (src/biasing.rs, src/biasing/spotting.rs,
src/biasing/tdt_beam.rs): the reference's own unit tests for the matcher, word spotting and the TDT
beam search, run against the library (telmo_b200.biasing, host code over the C ABI) and against the
oracle's restatement (oracle/biasing.py), then the two compared on random cases. CPU only."""

import numpy as np
import pytest

from oracle import biasing as ob
from telmo_b200 import biasing as tb

# The reference's test vocabulary (src/biasing.rs:1073-1087), id order; id 0 is the blank, a
# special token.
PIECES = [None, "▁ku", "be", "ctl", "▁cube", "▁control", "▁the", ",", "▁Ku", "▁ng", "inx", "▁",
          "k", "u", "b", "e", "c", "t", "l", "K", "n", "g", "i", "x", "o", "r", "h", "▁k", "▁K", "▁n",
          "▁c", "▁t", "ct", "▁co", "▁con", "ro", "▁cu", "nt", "ntro", "ntrol", "in", "▁th",
          "▁New", "▁York", "▁city", "▁Ne", "w", "s", "N", "Y", "▁N", "▁Y", "▁Yo", "▁Yor", "▁ci", "▁cit",
          "y", "C", "▁C", "be.", ".", "—", "'s", "-", "p", "a", "+", "#", "▁p", "▁pl", "▁plu",
          "▁plus", "▁s", "▁sh", "▁sha", "▁shar", "▁sharp", "’s", "U", "m"]
BOUNDARY, WORDLIKE = tb.token_flags(PIECES)

# Each word's spellings as Compiled::new collects them (the word, then its first letter
# capitalized) split by that vocabulary's BPE: the reference's tests give "kubectl" [1, 2, 3],
# "Kubectl" [8, 2, 3], "nginx" [9, 10], "Nginx" [50, 21, 10], "kub" [1, 14]
# (src/biasing.rs:1353-1376, src/biasing/spotting.rs:382-384); "the" has no capitalized spelling
# (the vocabulary has no "T").
SPELLINGS = {
    "kubectl": [([1, 2, 3], "kubectl"), ([8, 2, 3], "Kubectl")],
    "kube": [([1, 2], "kube"), ([8, 2], "Kube")],
    "kub": [([1, 14], "kub"), ([8, 14], "Kub")],
    "nginx": [([9, 10], "nginx"), ([50, 21, 10], "Nginx")],
    "New": [([42], "New")],
    "New York": [([42, 43], "New York")],
    "New York city": [([42, 43, 44], "New York city")],
    "York": [([43], "York")],
    "the": [([6], "the")],
}


def _forms(entries):
    forms = [f for e in entries for f, _ in SPELLINGS[e]]
    letters = [tb.letters_of(s) for e in entries for _, s in SPELLINGS[e]]
    return forms, letters


def lib_words(entries, bonus=1.5, beam=4, spotting_bonus=4.0, spotting_margin=2.0, short_word_margin=3.0):
    forms, letters = _forms(entries)
    return tb.Words(forms, letters, BOUNDARY, WORDLIKE,
                    tb.Boost(bonus, beam, spotting_bonus, spotting_margin, short_word_margin))


def oracle_words(entries, bonus=1.5, beam=4, spotting_bonus=4.0, spotting_margin=2.0, short_word_margin=3.0):
    forms, letters = _forms(entries)
    return ob.Words(forms, letters, BOUNDARY, WORDLIKE, bonus, beam, spotting_bonus, spotting_margin,
                    short_word_margin)


BACKENDS = ["library", "oracle"]


def words(backend, entries, **kw):
    return lib_words(entries, **kw) if backend == "library" else oracle_words(entries, **kw)


# ---- the matcher (src/biasing.rs:1427-1480) -------------------------------------------------------

def _walk(backend, w, tokens, bonus=1.5):
    """(final bonus, bonus held before the end) in bonuses per token."""
    held = np.float32(0)
    if backend == "library":
        s = (0, 0, 0)
        for t in tokens:
            s, d = w.step(s, t)
            held = np.float32(held + np.float32(d))
        fin = w.finish(s)
    else:
        s = (0, 0, 0)
        for t in tokens:
            s, d = w.matcher.step(s, t)
            held = np.float32(held + d)
        fin = w.matcher.finish(s)
    return float(np.float32(held + np.float32(fin)) / bonus), float(held / bonus)


def test_spellings_and_columns():
    # src/biasing.rs:1353-1376: the forms in order and the sorted tokens of all of them.
    w = lib_words(["kubectl", "nginx"])
    assert w.n_forms == 4
    assert list(w.columns) == [1, 2, 3, 8, 9, 10, 21, 50]
    assert oracle_words(["kubectl", "nginx"]).tokens == [1, 2, 3, 8, 9, 10, 21, 50]
    # A repeated spelling counts once.
    assert tb.Words([[1, 2, 3], [1, 2, 3]], [7, 7], BOUNDARY, WORDLIKE).n_forms == 1


@pytest.mark.parametrize("backend", BACKENDS)
def test_the_matcher_pays_each_token_of_a_completed_word_once(backend):
    half = 0.5
    cases = [
        (["kubectl"], [1, 2, 3, 6], 3.0, 3.0),
        (["kubectl"], [1, 2, 3], 3.0, 3.0),
        (["kubectl"], [1, 2, 3, 7, 6], 3.0, 3.0),
        # Left before the end, or the word goes on with letters, so it is taken back.
        (["kubectl"], [1, 2, 6], 0.0, 0.0),
        (["kubectl"], [1, 2], 0.0, 2.0),
        (["kubectl"], [1, 2, 3, 47], 0.0, 0.0),
        # A new special word right where another was left.
        (["kubectl"], [1, 2, 8, 2, 3], 3.0, 3.0),
        # "New" does not block "New York", and the shared token is paid once, fully.
        (["New", "New York"], [42, 43, 6], 2.0, 2.0),
        (["New", "New York"], [42, 6], half, half),
        (["New", "New York"], [42, 43], 2.0, 1.0 + half),
        # A word that ends inside a longer one that dies keeps its own bonus.
        (["New York city", "York"], [42, 43, 6], half, half),
        (["New York city", "York"], [42, 43, 44], 3.0, 2.0 + half),
        (["New York city", "York"], [42, 43], half, 2.0),
        # Two words in a row, and a single-token word.
        (["kubectl", "the"], [1, 2, 3, 6, 7], 3.0 + half, 3.0 + half),
        (["the"], [6, 6, 47], half, half),
    ]
    for entries, tokens, done, held in cases:
        got_done, got_held = _walk(backend, words(backend, entries), tokens)
        assert abs(got_done - done) < 1e-5 and abs(got_held - held) < 1e-5, (entries, tokens, got_done, got_held)


def test_default_steps_match_the_steps_of_ordinary_tokens():
    # src/biasing.rs:1496-1516, on the oracle's matcher (the library's is exercised through the
    # beam search, which compares equal to the oracle's below).
    m = oracle_words(["kubectl", "New York"]).matcher
    for prefix in ([], [1], [1, 2, 3], [42], [42, 43]):
        s = (0, 0, 0)
        for t in prefix:
            s = m.step(s, t)[0]
        special = m.special_tokens(s)
        boundary, other = m.default_steps(s)
        for t in range(len(PIECES)):
            if t in special:
                continue
            want = boundary if m.is_boundary(t) else other
            assert m.step(s, t)[1] == want, (prefix, t)


def test_lists_refuse_what_they_cannot_hold():
    # Boost::new's ranges (src/biasing.rs:80-128) and the forms' limits.
    from telmo_b200 import TelmoError
    for kw in (dict(bonus=10.5), dict(bonus=-1), dict(spotting_bonus=11), dict(beam=0), dict(beam=17),
               dict(spotting_margin=51), dict(short_word_margin=-0.5)):
        with pytest.raises(TelmoError):
            lib_words(["kubectl"], **kw)
    for forms in ([[]], [[1] * 33], [[len(PIECES)]]):
        with pytest.raises(TelmoError):
            tb.Words(forms, [3], BOUNDARY, WORDLIKE)
    assert tb.Words([[1] * 32], [3], BOUNDARY, WORDLIKE).n_forms == 1


# ---- word spotting (src/biasing/spotting.rs:312-433) ----------------------------------------------

def _scores(columns, best, sets):
    """Frames where each frame's best token (or the blank) has logit 0 and every other -10, except
    the (frame, token, logit) in sets."""
    rows = []
    for f, b in enumerate(best):
        logits = np.full(64, -10.0, np.float32)
        logits[b] = 0.0
        for sf, t, l in sets:
            if sf == f:
                logits[t] = l
        rows.append(logits)
    return tb.score_rows(np.stack(rows), 0, columns)


def _spot(backend, w, greedy, scores, first=0):
    if backend == "library":
        out, ranges = tb.spot(w, greedy, scores, first)
        return [tuple(int(x) for x in t) for t in out], ranges
    return ob.spot(w, greedy, scores, first)


def _columns(backend, w):
    return np.asarray(w.columns if backend == "library" else w.tokens)


@pytest.mark.parametrize("backend", BACKENDS)
def test_spotting_replaces_whole_greedy_words_when_the_word_is_close(backend):
    w = words(backend, ["kubectl"])
    # The greedy text is "▁the ▁cube ▁control ,".
    best = [6, 0, 4, 4, 0, 5, 5, 0, 7, 0]
    greedy = ob.ctc_tokens(best, 0)
    close = [(2, 1, -0.5), (3, 2, -0.5), (5, 3, -0.5), (6, 3, -0.5)]
    out, ranges = _spot(backend, w, greedy, _scores(_columns(backend, w), best, close))
    assert [t[0] for t in out] == [6, 1, 2, 3, 7]
    assert ranges == [(1, 4)]
    assert (out[3][1], out[3][2]) == (5, 2)
    # Far from it, the greedy words stay.
    far = [(2, 1, -6.0), (3, 2, -6.0), (5, 3, -6.0), (6, 3, -6.0)]
    assert _spot(backend, w, greedy, _scores(_columns(backend, w), best, far))[0] == greedy
    # Frames before `first` are not touched.
    assert _spot(backend, w, greedy[2:], _scores(_columns(backend, w), best, close), 5)[0] == greedy[2:]


@pytest.mark.parametrize("backend", BACKENDS)
def test_spotting_never_inserts_a_word_into_silence(backend):
    w = words(backend, ["kubectl"])
    best = [6, 0, 0, 0, 0, 0]
    greedy = ob.ctc_tokens(best, 0)
    strong = [(2, 1, 0.0), (3, 2, 0.0), (4, 3, 0.0)]
    assert _spot(backend, w, greedy, _scores(_columns(backend, w), best, strong))[0] == greedy


@pytest.mark.parametrize("backend", BACKENDS)
def test_a_cheap_path_over_blanks_doesnt_hide_a_spot_over_a_word(backend):
    w = words(backend, ["kubectl"])
    # Greedy "▁the ▁cube" then silence; the word's last token fits only frame 6, where the path
    # over the silence alone is cheaper.
    best = [6, 0, 4, 4, 0, 0, 0, 0]
    greedy = ob.ctc_tokens(best, 0)
    sets = [(2, 1, -0.5), (3, 2, -0.5), (4, 1, 0.0), (5, 2, 0.0), (6, 3, -0.5)]
    out, ranges = _spot(backend, w, greedy, _scores(_columns(backend, w), best, sets))
    assert [t[0] for t in out] == [6, 1, 2, 3]
    assert ranges == [(1, 4)]


def test_overlapping_spots_of_one_word_stay_until_the_choice():
    # src/biasing/spotting.rs:360-378, on the oracle's helpers (internal to the library).
    spots = []
    for s in [(0, 0, 3, 1.0), (0, 2, 5, 2.0), (0, 4, 7, 3.0)]:
        ob._keep(spots, 0, s)
    assert len(spots) == 3
    assert [(s[1], s[2]) for s in ob._choose(spots)] == [(0, 3), (4, 7)]
    spots = []
    ob._keep(spots, 0, (0, 0, 7, 1.0))
    ob._keep(spots, 0, (0, 2, 7, 1.5))
    ob._keep(spots, 0, (0, 1, 7, 0.5))
    assert [(s[1], s[2]) for s in spots] == [(2, 7)]


@pytest.mark.parametrize("backend", BACKENDS)
def test_a_short_word_needs_a_larger_margin(backend):
    # "kub" has three letters in two tokens.
    best = [6, 0, 4, 4, 0, 0]
    greedy = ob.ctc_tokens(best, 0)
    sets = [(2, 1, -1.0), (3, 14, -1.0)]

    def spotted(short):
        w = words(backend, ["kub"], short_word_margin=short)
        return len(_spot(backend, w, greedy, _scores(_columns(backend, w), best, sets))[1])

    assert spotted(0.0) == 1
    assert spotted(1.0) == 1
    assert spotted(2.5) == 0


@pytest.mark.parametrize("backend", BACKENDS)
def test_a_spot_of_several_words_comes_back_as_one_range(backend):
    w = words(backend, ["New York city"])
    # Greedy "▁the ▁cube ▁control ▁the"; the phrase fits the middle words.
    best = [6, 0, 4, 0, 5, 0, 6, 0]
    greedy = ob.ctc_tokens(best, 0)
    sets = [(2, 42, -0.3), (3, 43, -0.3), (4, 44, -0.3)]
    out, ranges = _spot(backend, w, greedy, _scores(_columns(backend, w), best, sets))
    assert [t[0] for t in out] == [6, 42, 43, 44, 6]
    assert ranges == [(1, 4)]


# ---- the TDT beam search (src/biasing/tdt_beam.rs:403-562) ----------------------------------------

DURATIONS = [0, 1, 2]
VOCAB = 57
NONE = 0xFFFFFFFF


class Scripted:
    """A network whose joint outputs depend on the frame and the last token, as `script` gives them;
    the state and the prediction output are the last token."""

    def __init__(self, script):
        self.script = script

    def joint(self, frame, preds):
        out = np.full((preds.shape[0], VOCAB + len(DURATIONS)), -20.0, np.float32)
        for r in range(preds.shape[0]):
            last = int(preds[r, 0])
            self.script(frame, NONE if last >= NONE else last, out[r])
        return out

    def predict(self, tokens, states):
        t = np.asarray(tokens, np.float32).reshape(-1, 1)
        return t.copy(), t.copy()


def search(backend, script, frames, entries, bonus, beam):
    net = Scripted(script)
    start = np.array([NONE], np.float32)
    if backend == "library":
        w = lib_words(entries, bonus=bonus, beam=beam)
        out = tb.tdt_beam_search(w, net.joint, net.predict, VOCAB, 0, DURATIONS, 3, frames, start, start)
        return [int(t[0]) for t in out]
    w = oracle_words(entries, bonus=bonus, beam=beam)
    return [t[0] for t in ob.beam_search(w, net.joint, net.predict, VOCAB, 0, DURATIONS, 3, frames, start, start)]


def setrow(row, token, logit, durations):
    row[token] = logit
    row[VOCAB:] = durations


def _index(v):
    best = 0
    for i, x in enumerate(v):
        if x > v[best]:
            best = i
    return best


@pytest.mark.parametrize("backend", BACKENDS)
def test_a_beam_of_one_without_a_bonus_decodes_greedily(backend):
    def script(frame, last, row):
        for i in range(len(row)):
            h = ((frame * 1_000_003 + last * 7919 + i + 1) * 0x9E3779B97F4A7C15) & ((1 << 64) - 1)
            h ^= h >> 29
            row[i] = np.float32(h % 10_000) / np.float32(1000.0)

    frames = 40
    row = np.zeros(VOCAB + len(DURATIONS), np.float32)
    t, on_frame, last, greedy = 0, 0, NONE, []
    while t < frames:
        row.fill(-20.0)
        script(t, last, row)
        token = _index(row[:VOCAB])
        d = DURATIONS[_index(row[VOCAB:])]
        if token == 0:
            t += max(d, 1)
            on_frame = 0
            continue
        greedy.append(token)
        last = token
        if d > 0:
            t += d
            on_frame = 0
        else:
            on_frame += 1
            if on_frame >= 3:
                t += 1
                on_frame = 0
    assert len(greedy) > 5
    assert search(backend, script, frames, ["kubectl"], 0.0, 1) == greedy


@pytest.mark.parametrize("backend", BACKENDS)
def test_the_same_text_at_different_frames_stays_two_states(backend):
    def script(frame, last, row):
        if (frame, last) == (0, NONE):
            setrow(row, 6, 0.0, [-20.0, 0.0, -0.5])
        elif (frame, last) == (1, 6):
            row.fill(-3.0)
        elif (frame, last) == (2, 6):
            setrow(row, 7, 0.0, [-20.0, 0.0, -20.0])
        else:
            setrow(row, 0, 0.0, [-20.0, 0.0, -20.0])

    assert search(backend, script, 3, ["kubectl"], 0.0, 2) == [6, 7]


@pytest.mark.parametrize("backend", BACKENDS)
def test_a_word_boundary_that_keeps_a_bonus_is_expanded(backend):
    def script(frame, last, row):
        if (frame, last) == (0, NONE):
            setrow(row, 1, 0.0, [-20.0, 0.0, -20.0])
        elif (frame, last) == (1, 1):
            setrow(row, 2, 0.0, [-20.0, 0.0, -20.0])
        elif (frame, last) == (2, 2):
            setrow(row, 3, 0.0, [-20.0, 0.0, -20.0])
        elif (frame, last) == (3, 3):
            setrow(row, 47, 0.0, [-20.0, 0.0, -20.0])
            row[6] = -0.5
            row[0] = -5.0
        else:
            setrow(row, 0, 0.0, [-20.0, 0.0, -20.0])

    assert search(backend, script, 5, ["kubectl"], 1.5, 1) == [1, 2, 3, 6]


@pytest.mark.parametrize("backend", BACKENDS)
def test_a_hypothesis_at_the_end_gives_back_an_unfinished_word(backend):
    def script(frame, last, row):
        if (frame, last) == (0, NONE):
            setrow(row, 1, -1.0, [-20.0, -20.0, 0.0])
            row[0] = 0.0
        else:
            setrow(row, 0, 0.0, [-20.0, 0.0, -20.0])

    assert search(backend, script, 2, ["kubectl"], 1.5, 1) == []


@pytest.mark.parametrize("backend", BACKENDS)
def test_an_unfinished_word_at_the_end_doesnt_crowd_out_an_ordinary_token(backend):
    def script(frame, last, row):
        if (frame, last) == (0, NONE):
            setrow(row, 6, 0.0, [-20.0, 0.0, -20.0])
            row[1] = -0.5
        else:
            setrow(row, 0, 0.0, [-20.0, 0.0, -20.0])

    assert search(backend, script, 1, ["kubectl"], 1.5, 1) == [6]


@pytest.mark.parametrize("backend", BACKENDS)
def test_a_token_that_may_land_live_or_at_the_end_keeps_its_live_landing(backend):
    def script(frame, last, row):
        if (frame, last) == (0, NONE):
            setrow(row, 1, 0.0, [-20.0, 0.0, 0.0])
            row[6] = 0.1
        elif (frame, last) == (1, 1):
            setrow(row, 2, 0.0, [-20.0, 0.0, -20.0])
        else:
            setrow(row, 0, 0.0, [-20.0, 0.0, -20.0])

    assert search(backend, script, 2, ["kube"], 1.5, 1) == [1, 2]


# ---- the library against the oracle on random cases ------------------------------------------------

class RandomNet:
    """A joint whose outputs are a fixed random table over (frame, last token), peaked so special
    words compete, and a prediction state that is the last token."""

    def __init__(self, seed, frames, favour):
        r = np.random.default_rng(seed)
        self.table = r.normal(0, 2.0, (frames, VOCAB + 1, VOCAB + len(DURATIONS))).astype(np.float32)
        for f in range(frames):
            for tok in favour[f % len(favour)]:
                self.table[f, :, tok] += np.float32(r.uniform(1.0, 4.0))

    def joint(self, frame, preds):
        rows = [self.table[frame, VOCAB if int(p[0]) >= NONE else int(p[0])] for p in preds]
        return np.stack(rows).astype(np.float32)

    def predict(self, tokens, states):
        t = np.asarray(tokens, np.float32).reshape(-1, 1)
        return t.copy(), t.copy()


@pytest.mark.parametrize("seed", range(12))
def test_the_beam_search_matches_the_oracle_on_random_networks(seed):
    r = np.random.default_rng(100 + seed)
    entries = [["kubectl"], ["kubectl", "New York"], ["New", "New York", "the"], ["kube", "nginx", "York"]][seed % 4]
    bonus = float(r.choice([0.0, 1.5, 4.0]))
    beam = int(r.choice([1, 2, 4, 8]))
    frames = int(r.integers(6, 14))
    favour = [[1, 2, 3], [42, 43], [8, 2], [9, 10, 6]]
    net = RandomNet(seed, frames, favour)
    start = np.array([NONE], np.float32)
    want = ob.beam_search(oracle_words(entries, bonus=bonus, beam=beam), net.joint, net.predict, VOCAB, 0, DURATIONS,
                          3, frames, start, start)
    got = tb.tdt_beam_search(lib_words(entries, bonus=bonus, beam=beam), net.joint, net.predict, VOCAB, 0, DURATIONS,
                             3, frames, start, start)
    assert [tuple(int(x) for x in t) for t in got] == [tuple(t) for t in want]


@pytest.mark.parametrize("seed", range(12))
def test_spotting_matches_the_oracle_on_random_scores(seed):
    r = np.random.default_rng(200 + seed)
    entries = [["kubectl"], ["kubectl", "New York city"], ["kub", "nginx"], ["New", "York", "the"]][seed % 4]
    w_lib = lib_words(entries, spotting_margin=float(r.choice([0.0, 1.0, 2.0])))
    w_or = oracle_words(entries, spotting_margin=w_lib.boost.spotting_margin)
    frames = int(r.integers(10, 40))
    logits = r.normal(0, 3.0, (frames, 64)).astype(np.float32)
    cols = w_lib.columns
    for f in range(frames):  # the words' tokens close behind the best on some frames
        if r.random() < 0.5:
            logits[f, r.choice(cols)] = logits[f].max() - np.float32(r.uniform(0, 1.5))
    ids = logits.argmax(axis=1)
    greedy = ob.ctc_tokens(ids, 0)
    scores = tb.score_rows(logits, 0, cols)
    first = int(r.integers(0, 3))
    kept = [t for t in greedy if t[1] >= first]
    want = ob.spot(w_or, kept, scores, first)
    got, ranges = tb.spot(w_lib, kept, scores, first)
    assert [tuple(int(x) for x in t) for t in got] == want[0]
    assert ranges == want[1]
