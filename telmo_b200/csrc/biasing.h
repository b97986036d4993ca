// biasing.h -- the decoders that favour special words, over this library's networks: the matcher
// of special-word token sequences (src/biasing.rs:470-705), Granite's CTC word spotting
// (src/biasing/spotting.rs) and Parakeet's TDT beam search (src/biasing/tdt_beam.rs). This is
// host logic; the networks they read (Granite's logits, Parakeet's joint and prediction networks)
// run on the device and are reached through TdtNetwork and the score rows.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <utility>
#include <vector>

#include "../../include/telmo_b200.h"

namespace telmo {
namespace biasing {

// Boost (src/biasing.rs:40-150): bonuses and margins in log probability.
struct Boost {
    float bonus = 1.5f;
    int beam = 4;
    float spotting_bonus = 4.0f;
    float spotting_margin = 2.0f;
    float short_word_margin = 3.0f;
};
constexpr float kMaxBonus = 10.0f;
constexpr int kMaxBeam = 16;
constexpr float kMaxMargin = 50.0f;
constexpr size_t kShortWordLetters = 5;
constexpr size_t kMaxTokens = 32;      // tokens of one form (SpecialWords::MAX_TOKENS)
constexpr size_t kMaxForms = 4000;     // two spellings of each of SpecialWords::MAX_WORDS, and room
constexpr float kSinglePieceShare = 0.5f;

// Where a hypothesis stands in the matcher: its last depth(node) tokens are the longest special
// word under way; bit i of covered marks the token i places from the end as inside a completed
// word, bit i of half as paid at a single-token word's share.
struct MatchState {
    uint32_t node = 0;
    uint64_t covered = 0;
    uint64_t half = 0;
    bool operator==(const MatchState& o) const { return node == o.node && covered == o.covered && half == o.half; }
};

// An Aho-Corasick automaton over the forms' token sequences that keeps the committed bonus (each
// token of a completed word paid once, at the word's weight) apart from the provisional bonus
// (the tokens of the longest word under way that no completed word covers, given back when that
// word dies).
class Matcher {
public:
    static constexpr uint32_t kRoot = 0;
    static constexpr uint32_t kNone = 0xffffffffu;

    void build(const std::vector<std::vector<uint32_t>>& forms, std::vector<uint8_t> boundary, float bonus);
    bool is_boundary(uint32_t token) const { return token >= boundary_.size() || boundary_[token]; }
    // The state after token, and the change in the bonus the hypothesis holds.
    std::pair<MatchState, float> step(MatchState s, uint32_t token) const;
    // The change in bonus when the audio ends in state s.
    float finish(MatchState s) const;
    // The change in bonus of every token that neither continues nor starts a special word from s:
    // (word boundaries, other tokens).
    std::pair<float, float> default_steps(MatchState s) const;
    // Calls f(token) for each token that continues a special word from s or starts one.
    template <class F>
    void special_tokens(MatchState s, F f) const {
        uint32_t n = s.node;
        for (;;) {
            for (const auto& c : nodes_[n].children) f(c.first);
            if (n == kRoot) break;
            n = nodes_[n].fail;
        }
    }

private:
    struct Node {
        std::vector<std::pair<uint32_t, uint32_t>> children;  // (token, node), sorted by token
        uint32_t fail = kRoot;
        uint32_t depth = 0;
        uint32_t output = kNone;  // the deepest node on the failure chain where a form ends
    };
    uint32_t child(uint32_t node, uint32_t token) const;
    uint32_t go(uint32_t node, uint32_t token) const;
    float provisional(const MatchState& s) const;
    float commit(MatchState& s) const;

    std::vector<Node> nodes_;
    std::vector<uint8_t> boundary_;
    float bonus_ = 0.0f;
};

// One spelling of a special word, for word spotting.
struct Form {
    std::vector<uint32_t> tokens;
    std::vector<size_t> columns;  // each token's column in the score rows
    float bonus = 0.0f;
    float margin = 0.0f;
    // Alignment state s: even states are blanks (column 1), odd ones the tokens.
    size_t column(size_t s) const { return s % 2 == 0 ? 1 : columns[s / 2]; }
    bool may_skip(size_t s) const { return s % 2 == 1 && s >= 3 && tokens[s / 2] != tokens[s / 2 - 1]; }
};

// Special words split into one model's tokens (Compiled, src/biasing.rs:740-870, without the
// text rewrites): the matcher, the forms, their tokens sorted (the score rows' columns 2..), the
// boost, and per vocabulary token whether a word may end before it and whether it holds a letter
// or digit.
struct Words {
    Matcher matcher;
    std::vector<Form> forms;
    std::vector<uint32_t> tokens;
    Boost boost;
    std::vector<uint8_t> boundary;
    std::vector<uint8_t> wordlike;
    bool is_boundary(uint32_t t) const { return t >= boundary.size() || boundary[t]; }
    bool is_wordlike(uint32_t t) const { return t < wordlike.size() && wordlike[t]; }
};

struct Token {
    uint32_t id = 0, frame = 0, duration = 0;
    bool operator==(const Token& o) const { return id == o.id && frame == o.frame && duration == o.duration; }
};

// spot (src/biasing/spotting.rs:95-245): greedy tokens of frames first.., score rows
// [frames, 2 + words.tokens.size()] from frame 0. Writes the tokens and, for each spotted word,
// the [begin, end) range of them it holds.
void spot(const Words& w, const std::vector<Token>& greedy, const float* scores, size_t frames, size_t first,
          std::vector<Token>* out, std::vector<std::pair<size_t, size_t>>* ranges);

// tdt_beam::TdtNetwork (src/biasing/tdt_beam.rs:15-26). Calls return a status (0 = OK).
class TdtNetwork {
public:
    virtual ~TdtNetwork() = default;
    virtual size_t state_width() const = 0;
    virtual size_t pred_width() const = 0;
    // The joint's outputs at encoder frame `frame` for `rows` prediction rows.
    virtual int joint(size_t frame, const float* preds, size_t rows, float* out) = 0;
    // The prediction network on tokens, updating each row of states and writing each of preds.
    virtual int predict(const int* tokens, size_t rows, float* states, float* preds) = 0;
};

struct TdtShape {
    int vocab = 0;
    int blank = 0;
    std::vector<int> durations;
    int max_symbols = 1;
};

struct TdtStart {
    size_t frame = 0, on_frame = 0;
    std::vector<float> state, pred;
};

// beam_search (src/biasing/tdt_beam.rs:141-401).
int beam_search(TdtNetwork& net, const TdtShape& shape, size_t frames, TdtStart start, const Words& w,
                std::vector<Token>* out);

// ctc_tokens (src/granite.rs:1074-1094): runs of equal ids, blanks dropped.
std::vector<Token> ctc_tokens(const uint32_t* ids, size_t frames, uint32_t blank);

}  // namespace biasing

// Helpers the models' entry points share (biasing.cu). Failures set telmo_words_last_error().
const biasing::Words& words_of(const telmo_words* w);
int words_fail(const char* why);
// Gathers the score rows [frames, 2 + columns] of device logits [frames, ld] on the stream.
int words_score_rows(const telmo_words* w, const float* logits, int64_t frames, int vocab, int64_t ld, int blank,
                     float* out, cudaStream_t stream);
int words_tdt_shape(int vocab, int blank, const int* durations, int n_durations, int max_symbols,
                    biasing::TdtShape* shape);
// Tokens as (id, frame, duration) triples, up to cap; *n is their number.
int words_tokens_out(const std::vector<biasing::Token>& toks, uint32_t* tokens, size_t cap, size_t* n);

}  // namespace telmo
