"""Test infrastructure only: a pure-Python restatement of the reference's decoding that favours
special words, the checker for telmo_b200's host implementation (csrc/biasing.cu). Nothing in the
product imports it.

  Matcher        src/biasing.rs:470-705 (Aho-Corasick over the forms, committed and provisional
                 bonus)
  spot, align    src/biasing/spotting.rs:95-310 (CTC word spotting)
  beam_search    src/biasing/tdt_beam.rs:141-401 (TDT beam search)

Floats are numpy float32 with the reference's order of operations, so scores match the C++ bit
for bit on the same inputs. Pinned by the reference's own unit tests for these files, restated in
tests/test_biasing.py, which run against both this module and the library.
"""

from __future__ import annotations

import ctypes
import ctypes.util
from collections import deque

import numpy as np

F = np.float32
SINGLE_PIECE_SHARE = F(0.5)
ROOT = 0
NONE = 0xFFFFFFFF


def _mask(depth):
    return (1 << 64) - 1 if depth >= 64 else (1 << depth) - 1


class Matcher:
    """Matcher::new (src/biasing.rs:533-600) and its steps (:600-697). A state is (node, covered,
    half)."""

    def __init__(self, forms, boundary, bonus):
        self.children = [dict()]
        self.fail = [ROOT]
        self.depth = [0]
        self.output = [NONE]
        for form in forms:
            node = ROOT
            for t in form:
                c = self.children[node].get(t)
                if c is None:
                    c = len(self.children)
                    self.children.append(dict())
                    self.fail.append(ROOT)
                    self.depth.append(self.depth[node] + 1)
                    self.output.append(NONE)
                    self.children[node][t] = c
                node = c
            self.output[node] = node
        queue = deque(self.children[ROOT][t] for t in sorted(self.children[ROOT]))
        while queue:
            node = queue.popleft()
            if self.output[node] == NONE:
                self.output[node] = self.output[self.fail[node]]
            for t in sorted(self.children[node]):
                c = self.children[node][t]
                f = self.fail[node]
                while True:
                    nxt = self.children[f].get(t)
                    if nxt is not None and nxt != c:
                        fail = nxt
                        break
                    if f == ROOT:
                        fail = ROOT
                        break
                    f = self.fail[f]
                self.fail[c] = fail
                queue.append(c)
        self.boundary = list(boundary)
        self.bonus = F(bonus)

    def is_boundary(self, t):
        return t >= len(self.boundary) or bool(self.boundary[t])

    def provisional(self, s):
        return F(self.bonus * F(self.depth[s[0]] - bin(s[1]).count("1")))

    def commit(self, s):
        node, covered, half = s
        output = self.output[node]
        if output == NONE:
            return F(0), s
        depth = self.depth[output]
        window = _mask(depth)
        new = window & ~covered
        covered |= window
        if depth == 1:
            half |= new
            return F(F(F(bin(new).count("1")) * self.bonus) * SINGLE_PIECE_SHARE), (node, covered, half)
        upgraded = window & half
        half &= ~window & ((1 << 64) - 1)
        return (F(F(F(bin(new).count("1")) + F(F(bin(upgraded).count("1")) * F(F(1) - SINGLE_PIECE_SHARE)))
                  * self.bonus), (node, covered, half))

    def goto(self, node, t):
        while True:
            c = self.children[node].get(t)
            if c is not None:
                return c
            if node == ROOT:
                return ROOT
            node = self.fail[node]

    def step(self, s, t):
        before = self.provisional(s)
        committed = F(0)
        if self.is_boundary(t):
            committed, s = self.commit(s)
        node = self.goto(s[0], t)
        window = _mask(self.depth[node])
        nxt = (node, (s[1] << 1) & window, (s[2] << 1) & window)
        return nxt, F(F(committed + self.provisional(nxt)) - before)

    def finish(self, s):
        before = self.provisional(s)
        c, _ = self.commit(s)
        return F(c - before)

    def default_steps(self, s):
        before = self.provisional(s)
        c, _ = self.commit(s)
        return F(c - before), F(-before)

    def special_tokens(self, s):
        n = s[0]
        out = []
        while True:
            out.extend(sorted(self.children[n]))
            if n == ROOT:
                return out
            n = self.fail[n]


class Words:
    """Compiled (src/biasing.rs:740-870) of token forms: the matcher, the forms' columns, bonuses
    and margins."""

    def __init__(self, forms, letters, boundary, wordlike, bonus=1.5, beam=4, spotting_bonus=4.0,
                 spotting_margin=2.0, short_word_margin=3.0):
        seen, fs, ls = set(), [], []
        for f, l in zip(forms, letters):
            if tuple(f) not in seen:
                seen.add(tuple(f))
                fs.append(list(f))
                ls.append(l)
        self.boundary, self.wordlike = list(boundary), list(wordlike)
        self.beam = beam
        self.matcher = Matcher(fs, boundary, bonus) if fs else None
        self.tokens = sorted(set(t for f in fs for t in f))
        self.forms = []
        for f, l in zip(fs, ls):
            share = SINGLE_PIECE_SHARE if len(f) == 1 else F(1)
            missing = max(0, 5 - l)
            self.forms.append({
                "tokens": f,
                "columns": [2 + self.tokens.index(t) for t in f],
                "bonus": F(F(F(spotting_bonus) * F(len(f))) * share),
                "margin": F(F(spotting_margin) + F(F(short_word_margin) * F(missing))),
            })

    def is_boundary(self, t):
        return t >= len(self.boundary) or bool(self.boundary[t])


def _column(form, s):
    return 1 if s % 2 == 0 else form["columns"][s // 2]


def _may_skip(form, s):
    return s % 2 == 1 and s >= 3 and form["tokens"][s // 2] != form["tokens"][s // 2 - 1]


def ctc_tokens(ids, blank):
    """ctc_tokens (src/granite.rs:1074-1094)."""
    out, previous = [], None
    for f, i in enumerate(ids):
        i = int(i)
        if i != blank:
            if previous == i:
                if out:
                    out[-1][2] += 1
            else:
                out.append([i, f, 1])
        previous = i
    return [tuple(t) for t in out]


def spot(w: Words, greedy, scores, first=0):
    """spot (src/biasing/spotting.rs:95-245): (tokens, ranges)."""
    scores = np.asarray(scores, F)
    width = 2 + len(w.tokens)
    frames = scores.shape[0] if scores.size else 0
    greedy = [tuple(int(x) for x in t) for t in greedy]
    if not w.forms or first >= frames:
        return greedy, []
    spans = []
    for (i, f, d) in greedy:
        last = f + max(d, 1) - 1
        if spans and not w.is_boundary(i):
            spans[-1][1] = last
        else:
            spans.append([f, last, False])
        spans[-1][2] = spans[-1][2] or (i < len(w.wordlike) and bool(w.wordlike[i]))
    n = frames - first
    may_start, may_end, in_word = [True] * n, [True] * n, [False] * n
    for (sf, sl, hw) in spans:
        if sf < first:
            continue
        end = min(sl, frames - 1)
        for f in range(sf + 1, end + 1):
            may_start[f - first] = False
        for f in range(sf, end):
            may_end[f - first] = False
        if hw:
            for f in range(sf, end + 1):
                in_word[f - first] = True

    def cost(f, c):
        return F(scores[f, 0] - scores[f, c])

    inf = F(np.inf)
    spots = []
    for index, form in enumerate(w.forms):
        states = 2 * len(form["tokens"]) + 1
        cost_of = [[inf, inf] for _ in range(states)]
        start = [[0, 0] for _ in range(states)]
        base = len(spots)
        for f in range(first, frames):
            i = f - first
            nc = [[inf, inf] for _ in range(states)]
            ns = [[0, 0] for _ in range(states)]
            for s in range(states):
                for covered in (0, 1):
                    best = (inf, 0)
                    for fr in (0, 1):
                        if int(bool(fr) or in_word[i]) != covered:
                            continue
                        opts = [(cost_of[s][fr], start[s][fr])] * 3
                        if s >= 1:
                            opts[1] = (cost_of[s - 1][fr], start[s - 1][fr])
                        if _may_skip(form, s):
                            opts[2] = (cost_of[s - 2][fr], start[s - 2][fr])
                        for o in opts:
                            if o[0] < best[0]:
                                best = o
                    if s <= 1 and may_start[i] and covered == int(in_word[i]) and best[0] > 0:
                        best = (F(0), f)
                    nc[s][covered] = F(best[0] + cost(f, _column(form, s)))
                    ns[s][covered] = best[1]
            cost_of, start = nc, ns
            if not may_end[i]:
                continue
            for s in (states - 2, states - 1):
                gain = F(F(form["bonus"] - cost_of[s][1]) - form["margin"])
                if gain > 0:
                    _keep(spots, base, (index, start[s][1], f, gain))
    if not spots:
        return greedy, []
    chosen = _choose(spots)
    out, ranges, nxt, i = [], [], 0, 0
    while i < len(greedy):
        t = greedy[i]
        if nxt < len(chosen) and t[1] >= chosen[nxt][1]:
            s = chosen[nxt]
            at = len(out)
            out.extend(_align(w.forms[s[0]], s[1], s[2], cost))
            ranges.append((at, len(out)))
            while i < len(greedy) and greedy[i][1] <= s[2]:
                i += 1
            nxt += 1
        else:
            out.append(t)
            i += 1
    return out, ranges


def _dominates(a, b):
    return a[3] >= b[3] and b[1] <= a[1] and a[2] <= b[2]


def _keep(spots, base, spot):
    i = len(spots)
    while i > base and spots[i - 1][2] >= spot[1]:
        i -= 1
        if _dominates(spots[i], spot):
            return
    kept = spots[:i] + [s for s in spots[i:] if not _dominates(spot, s)]
    spots[:] = kept + [spot]


def _choose(spots):
    order = sorted(spots, key=lambda s: -float(s[3]))  # stable, best first
    chosen = []
    for s in order:
        if all(not (c[1] <= s[2] and s[1] <= c[2]) for c in chosen):
            chosen.append(s)
    return sorted(chosen, key=lambda s: s[1])


def _align(form, first, last, cost):
    states = 2 * len(form["tokens"]) + 1
    n = last + 1 - first
    inf = F(np.inf)
    cost_of = [inf] * states
    cost_of[0] = cost(first, _column(form, 0))
    cost_of[1] = cost(first, _column(form, 1))
    back = [[0] * states for _ in range(n)]
    for i in range(1, n):
        nxt = [inf] * states
        for s in range(states):
            best = (cost_of[s], 0)
            if s >= 1 and cost_of[s - 1] < best[0]:
                best = (cost_of[s - 1], 1)
            if _may_skip(form, s) and cost_of[s - 2] < best[0]:
                best = (cost_of[s - 2], 2)
            nxt[s] = F(best[0] + cost(first + i, _column(form, s)))
            back[i][s] = best[1]
        cost_of = nxt
    s = states - 2 if cost_of[states - 2] <= cost_of[states - 1] else states - 1
    path = [0] * n
    for i in range(n - 1, -1, -1):
        path[i] = s
        s -= back[i][s]
    toks = []
    for i, s in enumerate(path):
        new_run = i == 0 or path[i - 1] != s
        if s % 2 == 1 and new_run:
            toks.append([form["tokens"][s // 2], first + i, 1])
        elif s % 2 == 1:
            toks[-1][2] += 1
    if toks:
        toks[-1][2] = last + 1 - toks[-1][1]
    return [tuple(t) for t in toks]


_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
_libm.logf.restype = ctypes.c_float
_libm.logf.argtypes = [ctypes.c_float]


def _lse(v):
    """log_sum_exp (src/biasing/tdt_beam.rs:86-89) in f32, with the C library's expf and logf (the
    functions f32::exp and f32::ln call)."""
    v = np.asarray(v, F)
    mx = F(-np.inf)
    for x in v:
        mx = max(mx, x)
    total = F(0)
    for x in v:
        total = F(total + F(_libm.expf(float(F(x - mx)))))
    return F(mx + F(_libm.logf(float(total))))


def beam_search(w: Words, joint, predict, vocab, blank, durations, max_symbols, frames, state, pred,
                start_frame=0, start_on_frame=0):
    """beam_search (src/biasing/tdt_beam.rs:141-401) over Python networks (as
    telmo_b200.biasing.tdt_beam_search takes them). Returns [(id, frame, duration)]."""
    if start_frame >= frames or not w.forms:
        return []
    m = w.matcher
    beam = w.beam
    nd = len(durations)
    start_key = (0, 0, start_frame, start_on_frame, (0, 0, 0))
    hyps = [dict(tokens=[], key=start_key, score=F(0), state=np.asarray(state, F), pred=np.asarray(pred, F))]
    neg = F(-np.inf)

    def land(parent, step, key, score):
        h, ln, fr, of, ms = key
        if fr >= frames:
            score = F(score + m.finish(ms))
            key = (h, ln, frames, 0, (0, 0, 0))
        return dict(parent=parent, step=step, key=key, score=score)

    while True:
        live = [h["key"][2] for h in hyps if h["key"][2] < frames]
        if not live:
            break
        t = min(live)
        group = [i for i, h in enumerate(hyps) if h["key"][2] == t]
        logits = np.asarray(joint(t, np.stack([hyps[i]["pred"] for i in group])), F)
        cands = [dict(parent=i, step=None, key=h["key"], score=h["score"])
                 for i, h in enumerate(hyps) if h["key"][2] != t]
        for g, i in enumerate(group):
            hyp = hyps[i]
            row = logits[g]
            tl, dlse = _lse(row[:vocab]), _lse(row[vocab:])
            hh, ln, fr, of, ms = hyp["key"]
            for j, d in enumerate(durations):
                key = (hh, ln, t + max(d, 1), 0, ms)
                score = F(F(F(F(hyp["score"] + row[blank]) - tl) + row[vocab + j]) - dlse)
                cands.append(land(i, ("blank",), key, score))
            after = []
            for d in durations:
                if d > 0:
                    after.append((t + d, 0))
                elif of + 1 >= max_symbols:
                    after.append((t + 1, 0))
                else:
                    after.append((t, of + 1))
            live_dl, end_dl = neg, neg
            for (f2, _), dl in zip(after, row[vocab:]):
                if f2 >= frames:
                    end_dl = max(end_dl, dl)
                else:
                    live_dl = max(live_dl, dl)
            special = []
            for tok in m.special_tokens(ms):
                if tok < vocab and tok not in special:
                    special.append(tok)
            bstep, ostep = m.default_steps(ms)
            any_dl = max(live_dl, end_dl)
            top = []

            def push(score, tok):
                if len(top) == beam and score <= top[-1][0]:
                    return
                at = 0
                while at < len(top) and top[at][0] >= score:
                    at += 1
                top.insert(at, (score, tok))
                del top[beam:]

            for tok in range(vocab):
                if tok == blank or tok in special:
                    continue
                delta = bstep if m.is_boundary(tok) else ostep
                push(F(F(row[tok] + delta) + any_dl), tok)
            for tok in special:
                if tok != blank:
                    nxt, delta = m.step(ms, tok)
                    landing = max(live_dl, F(end_dl + m.finish(nxt)))
                    push(F(F(row[tok] + delta) + landing), tok)
            for _, tok in top:
                nms, delta = m.step(ms, tok)
                base = F(F(F(hyp["score"] + row[tok]) - tl) + delta)
                hsh = ((hh ^ (tok + 1)) * 0x100000001B3) & ((1 << 64) - 1)
                for j, (d, (f2, of2)) in enumerate(zip(durations, after)):
                    key = (hsh, ln + 1, f2, of2, nms)
                    cands.append(land(i, ("emit", tok, d), key, F(F(base + row[vocab + j]) - dlse)))
        cands.sort(key=lambda c: -float(c["score"]))  # stable, best first

        def ids(c):
            out = [tk[0] for tk in hyps[c["parent"]]["tokens"]]
            if c["step"] and c["step"][0] == "emit":
                out.append(c["step"][1])
            return out

        kept = []
        for c in cands:
            if len(kept) == beam:
                break
            if not any(k["key"] == c["key"] and ids(k) == ids(c) for k in kept):
                kept.append(c)
        nxt_hyps, emitted = [], []
        for c in kept:
            p = hyps[c["parent"]]
            h = dict(tokens=list(p["tokens"]), key=c["key"], score=c["score"], state=p["state"].copy(),
                     pred=p["pred"].copy())
            if c["step"] and c["step"][0] == "emit":
                h["tokens"].append((c["step"][1], t, c["step"][2]))
                if h["key"][2] < frames:
                    emitted.append(len(nxt_hyps))
            nxt_hyps.append(h)
        if emitted:
            toks = np.array([nxt_hyps[i]["tokens"][-1][0] for i in emitted], np.int32)
            states = np.stack([nxt_hyps[i]["state"] for i in emitted])
            new_states, new_preds = predict(toks, states)
            for r, i in enumerate(emitted):
                nxt_hyps[i]["state"] = np.asarray(new_states[r], F)
                nxt_hyps[i]["pred"] = np.asarray(new_preds[r], F)
        hyps = nxt_hyps
    best, best_score = None, None
    for h in hyps:
        s = F(h["score"] / F(len(h["tokens"]) + 1))
        if best is None or s >= best_score:
            best, best_score = h, s
    return best["tokens"] if best else []
