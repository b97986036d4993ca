// biasing.cu -- the decoders that favour special words (host logic over the device networks) and
// the score-row gather that Granite's word spotting reads from the device logits.
//
// Matcher: src/biasing.rs:470-705. Word spotting: src/biasing/spotting.rs. TDT beam search:
// src/biasing/tdt_beam.rs. The rules, the order of every floating-point sum and the tie-breaking
// follow the reference, so the same scores choose the same tokens.
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "biasing.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <deque>
#include <limits>
#include <memory>
#include <new>
#include <string>

namespace telmo {
namespace biasing {

namespace {

uint64_t mask(uint32_t depth) { return depth >= 64 ? ~0ull : (1ull << depth) - 1; }

int popcount(uint64_t v) { return __builtin_popcountll(v); }

// f32::total_cmp as an integer key: the IEEE order with -0 below +0 and NaNs at the ends.
int32_t total_key(float x) {
    int32_t b;
    memcpy(&b, &x, 4);
    return b ^ static_cast<int32_t>(static_cast<uint32_t>(b >> 31) >> 1);
}

constexpr float kInf = std::numeric_limits<float>::infinity();

}  // namespace

// ---- the matcher (src/biasing.rs:533-705) -------------------------------------------------------

uint32_t Matcher::child(uint32_t node, uint32_t token) const {
    const auto& c = nodes_[node].children;
    auto it = std::lower_bound(c.begin(), c.end(), token,
                               [](const std::pair<uint32_t, uint32_t>& a, uint32_t t) { return a.first < t; });
    return it != c.end() && it->first == token ? it->second : kNone;
}

void Matcher::build(const std::vector<std::vector<uint32_t>>& forms, std::vector<uint8_t> boundary, float bonus) {
    nodes_.assign(1, Node());
    for (const auto& form : forms) {
        uint32_t node = kRoot;
        for (uint32_t token : form) {
            uint32_t c = child(node, token);
            if (c == kNone) {
                c = static_cast<uint32_t>(nodes_.size());
                Node fresh;
                fresh.depth = nodes_[node].depth + 1;
                nodes_.push_back(fresh);
                auto& ch = nodes_[node].children;
                auto at = std::lower_bound(ch.begin(), ch.end(), token,
                                           [](const std::pair<uint32_t, uint32_t>& a, uint32_t t) { return a.first < t; });
                ch.insert(at, {token, c});
            }
            node = c;
        }
        nodes_[node].output = node;
    }
    // Failure and output links, breadth first.
    std::deque<uint32_t> queue;
    for (const auto& c : nodes_[kRoot].children) queue.push_back(c.second);
    while (!queue.empty()) {
        const uint32_t node = queue.front();
        queue.pop_front();
        const uint32_t fail_output = nodes_[nodes_[node].fail].output;
        if (nodes_[node].output == kNone) nodes_[node].output = fail_output;
        const auto children = nodes_[node].children;
        for (const auto& tc : children) {
            uint32_t f = nodes_[node].fail, fail;
            for (;;) {
                const uint32_t next = child(f, tc.first);
                if (next != kNone && next != tc.second) {
                    fail = next;
                    break;
                }
                if (f == kRoot) {
                    fail = kRoot;
                    break;
                }
                f = nodes_[f].fail;
            }
            nodes_[tc.second].fail = fail;
            queue.push_back(tc.second);
        }
    }
    boundary_ = std::move(boundary);
    bonus_ = bonus;
}

uint32_t Matcher::go(uint32_t node, uint32_t token) const {
    for (;;) {
        const uint32_t c = child(node, token);
        if (c != kNone) return c;
        if (node == kRoot) return kRoot;
        node = nodes_[node].fail;
    }
}

float Matcher::provisional(const MatchState& s) const {
    return bonus_ * static_cast<float>(static_cast<int>(nodes_[s.node].depth) - popcount(s.covered));
}

float Matcher::commit(MatchState& s) const {
    const uint32_t output = nodes_[s.node].output;
    if (output == kNone) return 0.0f;
    const uint32_t depth = nodes_[output].depth;
    const uint64_t window = mask(depth);
    const uint64_t fresh = window & ~s.covered;
    s.covered |= window;
    if (depth == 1) {
        s.half |= fresh;
        return static_cast<float>(popcount(fresh)) * bonus_ * kSinglePieceShare;
    }
    const uint64_t upgraded = window & s.half;
    s.half &= ~window;
    return (static_cast<float>(popcount(fresh)) + static_cast<float>(popcount(upgraded)) * (1.0f - kSinglePieceShare)) *
           bonus_;
}

std::pair<MatchState, float> Matcher::step(MatchState s, uint32_t token) const {
    const float before = provisional(s);
    const float committed = is_boundary(token) ? commit(s) : 0.0f;
    const uint32_t node = go(s.node, token);
    const uint64_t window = mask(nodes_[node].depth);
    MatchState next;
    next.node = node;
    next.covered = (s.covered << 1) & window;
    next.half = (s.half << 1) & window;
    return {next, committed + provisional(next) - before};
}

float Matcher::finish(MatchState s) const {
    const float before = provisional(s);
    return commit(s) - before;
}

std::pair<float, float> Matcher::default_steps(MatchState s) const {
    const float before = provisional(s);
    MatchState committed = s;
    return {commit(committed) - before, -before};
}

// ---- ctc_tokens (src/granite.rs:1074-1094) -------------------------------------------------------

std::vector<Token> ctc_tokens(const uint32_t* ids, size_t frames, uint32_t blank) {
    std::vector<Token> out;
    bool have_previous = false;
    uint32_t previous = 0;
    for (size_t f = 0; f < frames; ++f) {
        const uint32_t id = ids[f];
        if (id != blank) {
            if (have_previous && previous == id) {
                if (!out.empty()) out.back().duration += 1;
            } else {
                out.push_back({id, static_cast<uint32_t>(f), 1});
            }
        }
        previous = id;
        have_previous = true;
    }
    return out;
}

// ---- word spotting (src/biasing/spotting.rs) -----------------------------------------------------

namespace {

struct Span {
    size_t first, last;
    bool has_word;
};

struct Spot {
    size_t form, first, last;
    float gain;
};

bool overlap(const Spot& a, const Spot& b) { return a.first <= b.last && b.first <= a.last; }

// Whether a has as good a gain over frames inside b's (b can then never win).
bool dominates(const Spot& a, const Spot& b) { return a.gain >= b.gain && b.first <= a.first && a.last <= b.last; }

// Adds spot to spots (whose part from `from` on holds its form's spots in the order their last
// frames came) unless one of them dominates it, and drops those it dominates.
void keep(std::vector<Spot>& spots, size_t from, const Spot& spot) {
    size_t i = spots.size();
    while (i > from && spots[i - 1].last >= spot.first) {
        --i;
        if (dominates(spots[i], spot)) return;
    }
    size_t j = i;
    for (size_t k = i; k < spots.size(); ++k)
        if (!dominates(spot, spots[k])) spots[j++] = spots[k];
    spots.resize(j);
    spots.push_back(spot);
}

// The winners in frame order: the best first, then each next best that overlaps none chosen.
std::vector<Spot> choose(std::vector<Spot> spots) {
    std::stable_sort(spots.begin(), spots.end(),
                     [](const Spot& a, const Spot& b) { return total_key(b.gain) < total_key(a.gain); });
    std::vector<Spot> chosen;
    for (const Spot& s : spots) {
        bool free = true;
        for (const Spot& c : chosen) free = free && !overlap(c, s);
        if (free) chosen.push_back(s);
    }
    std::stable_sort(chosen.begin(), chosen.end(), [](const Spot& a, const Spot& b) { return a.first < b.first; });
    return chosen;
}

// The tokens of the best CTC alignment of form over frames first..=last, each at the frame its
// run starts, the last lasting to `last`.
template <class Cost>
std::vector<Token> align(const Form& form, size_t first, size_t last, const Cost& cost) {
    const size_t states = 2 * form.tokens.size() + 1;
    const size_t n = last + 1 - first;
    std::vector<float> cost_of(states, kInf), next(states);
    cost_of[0] = cost(first, form.column(0));
    cost_of[1] = cost(first, form.column(1));
    std::vector<uint8_t> back(n * states, 0);
    for (size_t i = 1; i < n; ++i) {
        for (size_t s = 0; s < states; ++s) {
            float best = cost_of[s];
            uint8_t from = 0;
            if (s >= 1 && cost_of[s - 1] < best) {
                best = cost_of[s - 1];
                from = 1;
            }
            if (form.may_skip(s) && cost_of[s - 2] < best) {
                best = cost_of[s - 2];
                from = 2;
            }
            next[s] = best + cost(first + i, form.column(s));
            back[i * states + s] = from;
        }
        std::swap(cost_of, next);
    }
    size_t s = cost_of[states - 2] <= cost_of[states - 1] ? states - 2 : states - 1;
    std::vector<size_t> path(n);
    for (size_t i = n; i-- > 0;) {
        path[i] = s;
        s -= back[i * states + s];
    }
    std::vector<Token> tokens;
    for (size_t i = 0; i < n; ++i) {
        const size_t st = path[i];
        const bool new_run = i == 0 || path[i - 1] != st;
        if (st % 2 == 1 && new_run)
            tokens.push_back({form.tokens[st / 2], static_cast<uint32_t>(first + i), 1});
        else if (st % 2 == 1)
            tokens.back().duration += 1;
    }
    if (!tokens.empty()) tokens.back().duration = static_cast<uint32_t>(last) + 1 - tokens.back().frame;
    return tokens;
}

}  // namespace

void spot(const Words& w, const std::vector<Token>& greedy, const float* scores, size_t frames, size_t first,
          std::vector<Token>* out, std::vector<std::pair<size_t, size_t>>* ranges) {
    const size_t width = 2 + w.tokens.size();
    out->clear();
    ranges->clear();
    if (w.forms.empty() || first >= frames) {
        *out = greedy;
        return;
    }
    // Words and punctuation of the greedy text, as spans of frames.
    std::vector<Span> spans;
    for (const Token& t : greedy) {
        const size_t last = t.frame + std::max<uint32_t>(t.duration, 1) - 1;
        if (!spans.empty() && !w.is_boundary(t.id))
            spans.back().last = last;
        else
            spans.push_back({t.frame, last, false});
        spans.back().has_word = spans.back().has_word || w.is_wordlike(t.id);
    }
    // An alignment may start where no span is under way, end where none goes on, and must cover
    // a frame of a word.
    const size_t n = frames - first;
    std::vector<uint8_t> may_start(n, 1), may_end(n, 1), in_word(n, 0);
    for (const Span& s : spans) {
        if (s.first < first) continue;
        const size_t end = std::min(s.last, frames - 1);
        for (size_t f = s.first + 1; f <= end; ++f) may_start[f - first] = 0;
        for (size_t f = s.first; f < end; ++f) may_end[f - first] = 0;
        if (s.has_word)
            for (size_t f = s.first; f <= end; ++f) in_word[f - first] = 1;
    }
    auto cost = [&](size_t f, size_t column) {
        const float* row = scores + f * width;
        return row[0] - row[column];
    };

    std::vector<Spot> spots;
    for (size_t index = 0; index < w.forms.size(); ++index) {
        const Form& form = w.forms[index];
        // The best path to each state, apart for paths that have covered a word's frame and those
        // that haven't, so a cheaper path over blanks cannot hide one that may replace.
        const size_t states = 2 * form.tokens.size() + 1;
        std::vector<float> cost_of(2 * states, kInf), next_cost(2 * states);
        std::vector<size_t> start(2 * states, 0), next_start(2 * states);
        const size_t from_spot = spots.size();
        for (size_t f = first; f < frames; ++f) {
            const size_t i = f - first;
            for (size_t s = 0; s < states; ++s) {
                for (int covered = 0; covered < 2; ++covered) {
                    // Arriving at a word's frame makes a path covered.
                    float best = kInf;
                    size_t best_start = 0;
                    for (int from = 0; from < 2; ++from) {
                        if (static_cast<int>(from || in_word[i]) != covered) continue;
                        const float o0 = cost_of[2 * s + from];
                        const size_t s0 = start[2 * s + from];
                        float o1 = o0, o2 = o0;
                        size_t s1 = s0, s2 = s0;
                        if (s >= 1) {
                            o1 = cost_of[2 * (s - 1) + from];
                            s1 = start[2 * (s - 1) + from];
                        }
                        if (form.may_skip(s)) {
                            o2 = cost_of[2 * (s - 2) + from];
                            s2 = start[2 * (s - 2) + from];
                        }
                        if (o0 < best) best = o0, best_start = s0;
                        if (o1 < best) best = o1, best_start = s1;
                        if (o2 < best) best = o2, best_start = s2;
                    }
                    if (s <= 1 && may_start[i] && covered == in_word[i] && best > 0.0f) {
                        best = 0.0f;
                        best_start = f;
                    }
                    next_cost[2 * s + covered] = best + cost(f, form.column(s));
                    next_start[2 * s + covered] = best_start;
                }
            }
            std::swap(cost_of, next_cost);
            std::swap(start, next_start);
            if (!may_end[i]) continue;
            for (size_t s : {states - 2, states - 1}) {
                const float gain = form.bonus - cost_of[2 * s + 1] - form.margin;
                if (gain > 0.0f) keep(spots, from_spot, {index, start[2 * s + 1], f, gain});
            }
        }
    }
    if (spots.empty()) {
        *out = greedy;
        return;
    }
    const std::vector<Spot> chosen = choose(std::move(spots));
    size_t next = 0, i = 0;
    while (i < greedy.size()) {
        const Token& t = greedy[i];
        if (next < chosen.size() && t.frame >= chosen[next].first) {
            const Spot& s = chosen[next];
            const size_t at = out->size();
            const std::vector<Token> word = align(w.forms[s.form], s.first, s.last, cost);
            out->insert(out->end(), word.begin(), word.end());
            ranges->push_back({at, out->size()});
            while (i < greedy.size() && greedy[i].frame <= s.last) ++i;
            ++next;
        } else {
            out->push_back(t);
            ++i;
        }
    }
}

// ---- TDT beam search (src/biasing/tdt_beam.rs) ----------------------------------------------------

namespace {

// What identifies a search state: equal keys with equal token ids have the same future.
struct Key {
    uint64_t hash = 0;
    size_t len = 0, frame = 0, on_frame = 0;
    MatchState matcher;
    bool operator==(const Key& o) const {
        return hash == o.hash && len == o.len && frame == o.frame && on_frame == o.on_frame && matcher == o.matcher;
    }
};

struct Hyp {
    std::vector<Token> tokens;
    Key key;
    float score = 0.0f;  // log probability plus bonus, provisional until the end of the audio
    std::vector<float> state, pred;
};

enum StepKind { kKeep, kBlank, kEmit };

struct Candidate {
    size_t parent;
    StepKind kind;
    uint32_t id, duration;
    Key key;
    float score;
};

float log_sum_exp(const float* v, size_t n) {
    float mx = -kInf;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, v[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += std::exp(v[i] - mx);
    return mx + std::log(sum);
}

// Keeps the n best (score, token) pairs, best first, earlier ones first among equals.
void push_top(std::vector<std::pair<float, size_t>>& top, size_t n, float score, size_t token) {
    if (top.size() == n && score <= top[n - 1].first) return;
    auto at = std::partition_point(top.begin(), top.end(),
                                   [&](const std::pair<float, size_t>& e) { return e.first >= score; });
    top.insert(at, {score, token});
    if (top.size() > n) top.resize(n);
}

// A candidate landing on key with score; one that reaches the end of the audio cannot emit again,
// so it takes its final score there, and all such with the same text are one state.
Candidate land(const Matcher& m, size_t frames, size_t parent, StepKind kind, uint32_t id, uint32_t duration, Key key,
               float score) {
    if (key.frame >= frames) {
        score += m.finish(key.matcher);
        key.matcher = MatchState();
        key.frame = frames;
        key.on_frame = 0;
    }
    return {parent, kind, id, duration, key, score};
}

// Whether two candidates' texts are the same token ids.
bool same_ids(const std::vector<Hyp>& hyps, const Candidate& a, const Candidate& b) {
    const auto& ta = hyps[a.parent].tokens;
    const auto& tb = hyps[b.parent].tokens;
    const size_t na = ta.size() + (a.kind == kEmit), nb = tb.size() + (b.kind == kEmit);
    if (na != nb) return false;
    for (size_t i = 0; i < na; ++i) {
        const uint32_t x = i < ta.size() ? ta[i].id : a.id;
        const uint32_t y = i < tb.size() ? tb[i].id : b.id;
        if (x != y) return false;
    }
    return true;
}

}  // namespace

int beam_search(TdtNetwork& net, const TdtShape& shape, size_t frames, TdtStart start, const Words& w,
                std::vector<Token>* out) {
    out->clear();
    if (start.frame >= frames || w.forms.empty()) return TELMO_OK;
    const Matcher& m = w.matcher;
    const size_t beam = static_cast<size_t>(w.boost.beam);
    const size_t vocab = static_cast<size_t>(shape.vocab), nd = shape.durations.size();
    const size_t outputs = vocab + nd, pred_width = net.pred_width();
    const size_t blank = static_cast<size_t>(shape.blank);
    if (start.state.size() != net.state_width() || start.pred.size() != pred_width) return TELMO_ERR_ARGUMENT;
    std::vector<Hyp> hyps(1);
    hyps[0].key.frame = start.frame;
    hyps[0].key.on_frame = start.on_frame;
    hyps[0].state = std::move(start.state);
    hyps[0].pred = std::move(start.pred);
    std::vector<float> preds, logits;
    std::vector<Candidate> candidates;
    std::vector<uint8_t> special(vocab, 0);
    std::vector<size_t> marked, group;
    std::vector<std::pair<float, size_t>> top;
    std::vector<std::pair<size_t, size_t>> after(nd);
    for (;;) {
        size_t t = frames;
        for (const Hyp& h : hyps)
            if (h.key.frame < frames) t = std::min(t, h.key.frame);
        if (t >= frames) break;
        group.clear();
        for (size_t i = 0; i < hyps.size(); ++i)
            if (hyps[i].key.frame == t) group.push_back(i);
        preds.clear();
        for (size_t i : group) preds.insert(preds.end(), hyps[i].pred.begin(), hyps[i].pred.end());
        logits.assign(group.size() * outputs, 0.0f);
        if (int rc = net.joint(t, preds.data(), group.size(), logits.data())) return rc;

        candidates.clear();
        for (size_t i = 0; i < hyps.size(); ++i)
            if (hyps[i].key.frame != t) candidates.push_back({i, kKeep, 0, 0, hyps[i].key, hyps[i].score});
        for (size_t g = 0; g < group.size(); ++g) {
            const size_t i = group[g];
            const Hyp& hyp = hyps[i];
            const float* row = logits.data() + g * outputs;
            const float token_lse = log_sum_exp(row, vocab);
            const float duration_lse = log_sum_exp(row + vocab, nd);
            for (size_t j = 0; j < nd; ++j) {
                const size_t d = static_cast<size_t>(shape.durations[j]);
                Key key = hyp.key;
                key.frame = t + std::max<size_t>(d, 1);
                key.on_frame = 0;
                const float score = hyp.score + row[blank] - token_lse + row[vocab + j] - duration_lse;
                candidates.push_back(land(m, frames, i, kBlank, 0, 0, key, score));
            }
            // Where a token lands with each duration: the frame and the tokens on it.
            for (size_t j = 0; j < nd; ++j) {
                const size_t d = static_cast<size_t>(shape.durations[j]);
                if (d > 0)
                    after[j] = {t + d, 0};
                else if (hyp.key.on_frame + 1 >= static_cast<size_t>(shape.max_symbols))
                    after[j] = {t + 1, 0};
                else
                    after[j] = {t, hyp.key.on_frame + 1};
            }
            float live_dl = -kInf, end_dl = -kInf;
            for (size_t j = 0; j < nd; ++j) {
                float& best = after[j].first >= frames ? end_dl : live_dl;
                best = std::fmax(best, row[vocab + j]);
            }
            // The best tokens by the score of their best landing. A token that neither continues
            // nor starts a special word changes the bonus by one of two amounts and has nothing to
            // take back; the matcher lists the rest.
            const MatchState state = hyp.key.matcher;
            m.special_tokens(state, [&](uint32_t tok) {
                if (tok < vocab && !special[tok]) {
                    special[tok] = 1;
                    marked.push_back(tok);
                }
            });
            const std::pair<float, float> steps = m.default_steps(state);
            const float any_dl = std::fmax(live_dl, end_dl);
            top.clear();
            for (size_t tok = 0; tok < vocab; ++tok) {
                if (tok == blank || special[tok]) continue;
                const float delta = m.is_boundary(static_cast<uint32_t>(tok)) ? steps.first : steps.second;
                push_top(top, beam, row[tok] + delta + any_dl, tok);
            }
            for (size_t tok : marked) {
                if (tok != blank) {
                    const auto nx = m.step(state, static_cast<uint32_t>(tok));
                    const float landing = std::fmax(live_dl, end_dl + m.finish(nx.first));
                    push_top(top, beam, row[tok] + nx.second + landing, tok);
                }
                special[tok] = 0;
            }
            marked.clear();
            for (const auto& e : top) {
                const size_t tok = e.second;
                const auto nx = m.step(state, static_cast<uint32_t>(tok));
                const float base = hyp.score + row[tok] - token_lse + nx.second;
                const uint64_t hash = (hyp.key.hash ^ (static_cast<uint64_t>(tok) + 1)) * 0x00000100000001b3ull;
                for (size_t j = 0; j < nd; ++j) {
                    Key key;
                    key.hash = hash;
                    key.len = hyp.key.len + 1;
                    key.frame = after[j].first;
                    key.on_frame = after[j].second;
                    key.matcher = nx.first;
                    candidates.push_back(land(m, frames, i, kEmit, static_cast<uint32_t>(tok),
                                              static_cast<uint32_t>(shape.durations[j]), key,
                                              base + row[vocab + j] - duration_lse));
                }
            }
        }
        // The best distinct states survive.
        std::stable_sort(candidates.begin(), candidates.end(), [](const Candidate& a, const Candidate& b) {
            return total_key(b.score) < total_key(a.score);
        });
        std::vector<const Candidate*> kept;
        for (const Candidate& c : candidates) {
            if (kept.size() == beam) break;
            bool duplicate = false;
            for (const Candidate* k : kept)
                if (k->key == c.key && same_ids(hyps, *k, c)) {
                    duplicate = true;
                    break;
                }
            if (!duplicate) kept.push_back(&c);
        }
        std::vector<Hyp> next;
        next.reserve(kept.size());
        std::vector<size_t> emitted;
        for (const Candidate* c : kept) {
            const Hyp& parent = hyps[c->parent];
            Hyp hyp;
            hyp.tokens = parent.tokens;
            hyp.key = c->key;
            hyp.score = c->score;
            hyp.state = parent.state;
            hyp.pred = parent.pred;
            if (c->kind == kEmit) {
                hyp.tokens.push_back({c->id, static_cast<uint32_t>(t), c->duration});
                if (hyp.key.frame < frames) emitted.push_back(next.size());
            }
            next.push_back(std::move(hyp));
        }
        if (!emitted.empty()) {
            const size_t sw = net.state_width();
            std::vector<int> tokens(emitted.size());
            std::vector<float> states(emitted.size() * sw), new_preds(emitted.size() * pred_width);
            for (size_t r = 0; r < emitted.size(); ++r) {
                const Hyp& h = next[emitted[r]];
                tokens[r] = static_cast<int>(h.tokens.back().id);
                std::copy(h.state.begin(), h.state.end(), states.begin() + r * sw);
            }
            if (int rc = net.predict(tokens.data(), emitted.size(), states.data(), new_preds.data())) return rc;
            for (size_t r = 0; r < emitted.size(); ++r) {
                Hyp& h = next[emitted[r]];
                std::copy(states.begin() + r * sw, states.begin() + (r + 1) * sw, h.state.begin());
                std::copy(new_preds.begin() + r * pred_width, new_preds.begin() + (r + 1) * pred_width, h.pred.begin());
            }
        }
        hyps = std::move(next);
    }
    // The best final score per token (NeMo's choice); the last of equals, as Iterator::max_by.
    const Hyp* best = nullptr;
    float best_score = 0.0f;
    for (const Hyp& h : hyps) {
        const float s = h.score / static_cast<float>(h.tokens.size() + 1);
        if (!best || total_key(s) >= total_key(best_score)) {
            best = &h;
            best_score = s;
        }
    }
    if (best) *out = best->tokens;
    return TELMO_OK;
}

// One warp per frame: the row's largest logit, the blank's, and the logits of the listed tokens.
__global__ void score_rows_kernel(const float* __restrict__ logits, int64_t frames, int vocab, int64_t ld, int blank,
                                  const uint32_t* __restrict__ tokens, int n_tokens, float* __restrict__ out) {
    const int64_t f = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x % 32;
    if (f >= frames) return;
    const float* row = logits + f * ld;
    float mx = -INFINITY;
    for (int i = lane; i < vocab; i += 32) mx = fmaxf(mx, row[i]);
    for (int o = 16; o > 0; o /= 2) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int width = 2 + n_tokens;
    float* dst = out + f * width;
    if (lane == 0) {
        dst[0] = mx;
        dst[1] = row[blank];
    }
    for (int j = lane; j < n_tokens; j += 32) dst[2 + j] = row[tokens[j]];
}

}  // namespace biasing
}  // namespace telmo

// ---- the C ABI -------------------------------------------------------------------------------------

using namespace telmo;
using namespace telmo::biasing;

namespace {

thread_local std::string words_error;

int fail_words(const char* why) { return telmo::words_fail(why); }

bool in_range(float x, float max) { return x >= 0.0f && x <= max; }

}  // namespace

struct telmo_words {
    Words w;
    uint32_t* tokens_dev = nullptr;  // the columns, for score_rows (uploaded on first use)
    int device = -1;
    ~telmo_words() {
        if (tokens_dev) cudaFree(tokens_dev);
    }
};

extern "C" void telmo_boost_default(telmo_boost* b) {
    if (!b) return;
    const Boost d;
    b->bonus = d.bonus;
    b->beam = d.beam;
    b->spotting_bonus = d.spotting_bonus;
    b->spotting_margin = d.spotting_margin;
    b->short_word_margin = d.short_word_margin;
}

extern "C" const char* telmo_words_last_error(void) { return words_error.c_str(); }

extern "C" int telmo_words_create(size_t vocab, const uint8_t* boundary, const uint8_t* wordlike,
                                  const uint32_t* form_tokens, const size_t* form_lengths, const size_t* form_letters,
                                  size_t n_forms, const telmo_boost* boost, telmo_words** out) {
    if (!out || !boost || (n_forms && (!form_tokens || !form_lengths || !form_letters)) || (vocab && (!boundary || !wordlike)))
        return fail_words("A pointer is missing.");
    *out = nullptr;
    if (vocab == 0 || vocab > (1u << 24)) return fail_words("The vocabulary size is out of range.");
    if (n_forms > kMaxForms) return fail_words("There are too many forms.");
    // Boost::new and with_short_word_margin (src/biasing.rs:80-128).
    if (!in_range(boost->bonus, kMaxBonus) || !in_range(boost->spotting_bonus, kMaxBonus))
        return fail_words("A bonus must be from 0 to 10.");
    if (!in_range(boost->spotting_margin, kMaxMargin)) return fail_words("The spotting margin must be from 0 to 50.");
    if (!in_range(boost->short_word_margin, kMaxMargin))
        return fail_words("The short-word margin must be from 0 to 50.");
    if (boost->beam < 1 || boost->beam > kMaxBeam) return fail_words("The beam must be from 1 to 16.");
    std::unique_ptr<telmo_words> h(new (std::nothrow) telmo_words());
    if (!h) return fail_words("Out of host memory.");
    Words& w = h->w;
    w.boost.bonus = boost->bonus;
    w.boost.beam = boost->beam;
    w.boost.spotting_bonus = boost->spotting_bonus;
    w.boost.spotting_margin = boost->spotting_margin;
    w.boost.short_word_margin = boost->short_word_margin;
    w.boundary.assign(boundary, boundary + vocab);
    w.wordlike.assign(wordlike, wordlike + vocab);
    // Forms, each once (the first spelling's letters kept), as Compiled::new collects them.
    std::vector<std::vector<uint32_t>> forms;
    std::vector<size_t> letters;
    size_t at = 0;
    for (size_t i = 0; i < n_forms; ++i) {
        const size_t len = form_lengths[i];
        if (len == 0 || len > kMaxTokens) return fail_words("A form must have 1 to 32 tokens.");
        std::vector<uint32_t> f(form_tokens + at, form_tokens + at + len);
        at += len;
        for (uint32_t t : f)
            if (t >= vocab) return fail_words("A form's token is outside the vocabulary.");
        if (std::find(forms.begin(), forms.end(), f) != forms.end()) continue;
        forms.push_back(std::move(f));
        letters.push_back(form_letters[i]);
    }
    if (!forms.empty()) w.matcher.build(forms, w.boundary, w.boost.bonus);
    for (const auto& f : forms) w.tokens.insert(w.tokens.end(), f.begin(), f.end());
    std::sort(w.tokens.begin(), w.tokens.end());
    w.tokens.erase(std::unique(w.tokens.begin(), w.tokens.end()), w.tokens.end());
    for (size_t i = 0; i < forms.size(); ++i) {
        Form form;
        const float share = forms[i].size() == 1 ? kSinglePieceShare : 1.0f;
        const size_t missing = letters[i] < kShortWordLetters ? kShortWordLetters - letters[i] : 0;
        form.margin = w.boost.spotting_margin + w.boost.short_word_margin * static_cast<float>(missing);
        for (uint32_t t : forms[i])
            form.columns.push_back(2 + static_cast<size_t>(std::lower_bound(w.tokens.begin(), w.tokens.end(), t) -
                                                            w.tokens.begin()));
        form.bonus = w.boost.spotting_bonus * static_cast<float>(forms[i].size()) * share;
        form.tokens = std::move(forms[i]);
        w.forms.push_back(std::move(form));
    }
    *out = h.release();
    return TELMO_OK;
}

extern "C" void telmo_words_free(telmo_words* w) { delete w; }

extern "C" size_t telmo_words_forms(const telmo_words* w) { return w ? w->w.forms.size() : 0; }

extern "C" size_t telmo_words_columns(const telmo_words* w, uint32_t* tokens, size_t cap) {
    if (!w) return 0;
    const size_t n = w->w.tokens.size();
    if (tokens) std::copy(w->w.tokens.begin(), w->w.tokens.begin() + std::min(n, cap), tokens);
    return n;
}

extern "C" int telmo_words_step(const telmo_words* w, const uint64_t* state, uint32_t token, uint64_t* next,
                                float* delta) {
    if (!w || !state || !next || !delta || w->w.forms.empty()) return TELMO_ERR_ARGUMENT;
    MatchState s;
    s.node = static_cast<uint32_t>(state[0]);
    s.covered = state[1];
    s.half = state[2];
    const auto r = w->w.matcher.step(s, token);
    next[0] = r.first.node;
    next[1] = r.first.covered;
    next[2] = r.first.half;
    *delta = r.second;
    return TELMO_OK;
}

extern "C" int telmo_words_finish(const telmo_words* w, const uint64_t* state, float* delta) {
    if (!w || !state || !delta || w->w.forms.empty()) return TELMO_ERR_ARGUMENT;
    MatchState s;
    s.node = static_cast<uint32_t>(state[0]);
    s.covered = state[1];
    s.half = state[2];
    *delta = w->w.matcher.finish(s);
    return TELMO_OK;
}

namespace telmo {

int words_fail(const char* why) {
    words_error = why;
    return TELMO_ERR_ARGUMENT;
}

const Words& words_of(const telmo_words* w) { return w->w; }

int words_spot(const telmo_words* wh, const uint32_t* greedy, size_t n_greedy, const float* scores, size_t frames,
               size_t first, uint32_t* tokens, size_t cap, size_t* n_tokens, size_t* ranges, size_t ranges_cap,
               size_t* n_ranges) {
    if (!wh || (n_greedy && !greedy) || (frames && !scores) || !n_tokens) return fail_words("A pointer is missing.");
    std::vector<Token> in(n_greedy), out;
    for (size_t i = 0; i < n_greedy; ++i) in[i] = {greedy[3 * i], greedy[3 * i + 1], greedy[3 * i + 2]};
    std::vector<std::pair<size_t, size_t>> rs;
    spot(wh->w, in, scores, frames, first, &out, &rs);
    *n_tokens = out.size();
    if (n_ranges) *n_ranges = rs.size();
    if (out.size() > cap || (ranges && rs.size() > ranges_cap)) return TELMO_ERR_ARGUMENT;
    for (size_t i = 0; i < out.size(); ++i) {
        tokens[3 * i] = out[i].id;
        tokens[3 * i + 1] = out[i].frame;
        tokens[3 * i + 2] = out[i].duration;
    }
    if (ranges)
        for (size_t i = 0; i < rs.size(); ++i) {
            ranges[2 * i] = rs[i].first;
            ranges[2 * i + 1] = rs[i].second;
        }
    return TELMO_OK;
}

int words_score_rows(const telmo_words* wh, const float* logits, int64_t frames, int vocab, int64_t ld, int blank,
                     float* out, cudaStream_t stream) {
    auto* w = const_cast<telmo_words*>(wh);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TELMO_ERR_CUDA;
    const size_t n = w->w.tokens.size();
    if (n && (!w->tokens_dev || w->device != dev)) {
        // The columns go to the device once per device (a handle is used from one device).
        if (w->tokens_dev) cudaFree(w->tokens_dev);
        w->tokens_dev = nullptr;
        if (cudaMalloc(&w->tokens_dev, n * sizeof(uint32_t)) != cudaSuccess) return TELMO_ERR_CUDA;
        if (cudaMemcpy(w->tokens_dev, w->w.tokens.data(), n * sizeof(uint32_t), cudaMemcpyHostToDevice) != cudaSuccess)
            return TELMO_ERR_CUDA;
        w->device = dev;
    }
    if (frames == 0) return TELMO_OK;
    const int threads = 256;
    const int64_t blocks = (frames * 32 + threads - 1) / threads;
    score_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(logits, frames, vocab, ld, blank,
                                                                            w->tokens_dev, static_cast<int>(n), out);
    return cudaGetLastError() == cudaSuccess ? TELMO_OK : TELMO_ERR_CUDA;
}

}  // namespace telmo

extern "C" int telmo_spot(const telmo_words* w, const uint32_t* greedy, size_t n_greedy, const float* scores,
                          size_t frames, size_t first, uint32_t* tokens, size_t cap, size_t* n_tokens, size_t* ranges,
                          size_t ranges_cap, size_t* n_ranges) {
    return words_spot(w, greedy, n_greedy, scores, frames, first, tokens, cap, n_tokens, ranges, ranges_cap, n_ranges);
}

namespace {

// A network whose joint and predict are the caller's functions.
class CallbackNetwork : public TdtNetwork {
public:
    CallbackNetwork(size_t sw, size_t pw, telmo_tdt_joint_fn j, telmo_tdt_predict_fn p, void* user)
        : sw_(sw), pw_(pw), joint_(j), predict_(p), user_(user) {}
    size_t state_width() const override { return sw_; }
    size_t pred_width() const override { return pw_; }
    int joint(size_t frame, const float* preds, size_t rows, float* out) override {
        return joint_(user_, frame, preds, rows, out);
    }
    int predict(const int* tokens, size_t rows, float* states, float* preds) override {
        return predict_(user_, tokens, rows, states, preds);
    }

private:
    size_t sw_, pw_;
    telmo_tdt_joint_fn joint_;
    telmo_tdt_predict_fn predict_;
    void* user_;
};

}  // namespace

namespace telmo {

int words_tdt_shape(int vocab, int blank, const int* durations, int n_durations, int max_symbols, TdtShape* shape) {
    if (vocab < 1 || blank < 0 || blank >= vocab || !durations || n_durations < 1 || n_durations > 64 || max_symbols < 1)
        return fail_words("The transducer's shape is invalid.");
    shape->vocab = vocab;
    shape->blank = blank;
    shape->durations.assign(durations, durations + n_durations);
    for (int d : shape->durations)
        if (d < 0) return fail_words("A duration is negative.");
    shape->max_symbols = max_symbols;
    return TELMO_OK;
}

int words_tokens_out(const std::vector<Token>& toks, uint32_t* tokens, size_t cap, size_t* n) {
    *n = toks.size();
    if (toks.size() > cap) return TELMO_ERR_ARGUMENT;
    for (size_t i = 0; i < toks.size(); ++i) {
        tokens[3 * i] = toks[i].id;
        tokens[3 * i + 1] = toks[i].frame;
        tokens[3 * i + 2] = toks[i].duration;
    }
    return TELMO_OK;
}

}  // namespace telmo

extern "C" int telmo_tdt_beam_search(int vocab, int blank, const int* durations, int n_durations, int max_symbols,
                                     size_t state_width, size_t pred_width, telmo_tdt_joint_fn joint,
                                     telmo_tdt_predict_fn predict, void* user, size_t frames, size_t start_frame,
                                     size_t start_on_frame, const float* start_state, const float* start_pred,
                                     const telmo_words* w, uint32_t* tokens, size_t cap, size_t* n_tokens) {
    if (!joint || !predict || !w || !n_tokens || (state_width && !start_state) || (pred_width && !start_pred))
        return fail_words("A pointer is missing.");
    TdtShape shape;
    if (int rc = words_tdt_shape(vocab, blank, durations, n_durations, max_symbols, &shape)) return rc;
    CallbackNetwork net(state_width, pred_width, joint, predict, user);
    TdtStart start;
    start.frame = start_frame;
    start.on_frame = start_on_frame;
    start.state.assign(start_state, start_state + state_width);
    start.pred.assign(start_pred, start_pred + pred_width);
    std::vector<Token> out;
    if (int rc = beam_search(net, shape, frames, std::move(start), w->w, &out)) return rc;
    return words_tokens_out(out, tokens, cap, n_tokens);
}
