// granite_internal.h -- the device model behind telmo_granite handles.
#pragma once

#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "kernels.h"

#include <string>
#include <vector>

namespace telmo {

struct DevVec {
    float* p = nullptr;
};
struct Lin {
    DevWeights w;
    DevVec b;
};
struct Norm {
    DevVec g, b;
};
struct FF {
    Norm norm;
    Lin up, down;
};
// One conformer block, as Granite's Block (src/granite.rs:186-206).
struct Block {
    bool strided = false;
    FF ff1, ff2;
    Norm norm_att, norm_conv, norm_out;
    DevWeights qkv, rel;
    void* rel16 = nullptr;  // the relative table as fp16 [2 * ctx - 1, head_dim] (exact)
    Lin out, pw1, pw2;
    DevVec dw_w, dw_b;
};

// Optional timing of every launch with CUDA events on the launching stream, by kernel class.
enum ProfKind { kProfGemm = 0, kProfAttention, kProfRows, kProfFrontEnd, kProfKinds };

struct Profiler {
    bool on = false;
    std::vector<cudaEvent_t> pool;   // free events
    std::vector<cudaEvent_t> start[kProfKinds], stop[kProfKinds];
    double gemm_ops = 0.0, gemm_bytes = 0.0;
    long count[kProfKinds] = {0, 0, 0, 0};

    cudaEvent_t take();
    void begin(int kind, cudaStream_t s);
    void end(int kind, cudaStream_t s);
    // Sums the recorded intervals (ms) per kind, then recycles the events.
    void read(double* ms, long* launches, double* ops, double* bytes);
    ~Profiler();
};

struct Granite {
    Ctx* ctx = nullptr;
    Profiler prof;
    telmo_granite_config c{};
    Lin input, head, mid;
    std::vector<Block> blocks;
    bool finalized = false;
    long launches = 0;  // kernels launched so far (for benchmark accounting)

    // Activation buffers, sized for cap_rows packed rows.
    int cap_rows = 0, tasks_cap = 0;
    float *x = nullptr, *y = nullptr, *big = nullptr, *att = nullptr, *conv = nullptr;
    QuantAct q;
    int* tasks_dev = nullptr;
    int64_t big_ld = 0, vocab_ld = 0;

    // End-to-end buffers (audio in, tokens out), grown on demand.
    float* audio_dev = nullptr;
    size_t audio_cap = 0;
    // The host-buffer transcription's pipeline: each group's audio goes up on copy_stream into
    // one of two device buffers (through one of two pinned buffers when the caller's memory is
    // pageable) while the previous group is transcribed; tokens come back through pinned memory.
    int64_t group_samples = int64_t(2048) * 16000;
    cudaStream_t copy_stream = nullptr;
    float* group_audio[2] = {nullptr, nullptr};
    size_t group_audio_cap = 0;
    float* group_pinned[2] = {nullptr, nullptr};
    size_t group_pinned_cap = 0;
    cudaEvent_t group_copied[2] = {nullptr, nullptr};  // the group's audio is on the device
    cudaEvent_t group_read[2] = {nullptr, nullptr};    // the group's transcription is done with it
    uint32_t* tokens_pinned = nullptr;
    size_t tokens_pinned_cap = 0;
    int* counts_pinned = nullptr;
    size_t counts_pinned_cap = 0;
    // A call's tokens and counts stay on the device until its last group is done, then come back
    // in one copy each.
    uint32_t* call_tokens_dev = nullptr;
    size_t call_tokens_cap = 0;
    int* call_counts_dev = nullptr;
    size_t call_counts_cap = 0;
    float* feats_dev = nullptr;
    float* enc_dev = nullptr;
    uint32_t* ids_dev = nullptr;
    uint32_t* tokens_dev = nullptr;
    int* counts_dev = nullptr;
    int* first_dev = nullptr;
    int e2e_rows_cap = 0, e2e_frames_cap = 0, e2e_utt_cap = 0;

    struct Entry {
        DevWeights* mat = nullptr;
        DevVec* vec = nullptr;
        int n = 0, k = 0, len = 0;
    };

    ~Granite();
    static int validate(const telmo_granite_config& c, std::string& why);
    Entry find(const std::string& name);
    std::string missing() const;
    int fail(int code, const char* msg);
    int ensure(int rows, int tasks);
    void release_buffers();
    int gemm(const QuantAct& a, int m, const Lin& l, float* out, int64_t ldc, int act, float scale, int acc,
             cudaStream_t s);
    int gemm_w(const QuantAct& a, int m, const DevWeights& w, const float* bias, void* out, int64_t ldc, int act,
               float scale, int acc, cudaStream_t s, int out_kind = kOutF32);
    int feed_forward(const FF& f, float* x, int m, cudaStream_t s, bool normed = false);
    // Granite::block_span for one stream (src/granite.rs:795-952): block b over input frames
    // start..end, whose rows x ([t = end - start, d]) end up holding their post-attention
    // states; `window` holds the post-attention states of frames lo..end ([m, d], x's rows its
    // last t) that the convolution reads; the outputs of frames out_start .. out_start + n go to
    // out.
    int span(const Block& b, float* x, int t, const float* window, int m, int lo, int out_start, int n, float* out,
             cudaStream_t s);
    // Self-conditioning (src/granite.rs:1040-1069) of n rows in place: x += mid(softmax(head(x))).
    int self_condition(float* x, int n, cudaStream_t s);
    int encode(const float* feats, const int* rows, int n_utt, float* out, int* frames_out, int tap, cudaStream_t s);
    int logits(const float* encoded, int frames, float* out, int64_t ld, cudaStream_t s);
    int frame_ids(const float* encoded, int frames, uint32_t* ids, float* margin, cudaStream_t s);
    // Audio (device) -> tokens and counts (device); frames_out (host) gets each utterance's
    // encoder frames, whose prefix sums place its tokens.
    int transcribe_device(const float* samples, const int64_t* lengths, int n_utt, uint32_t* tokens, int* counts,
                          int* frames_out, cudaStream_t s);
    int ensure_e2e(int rows, int frames, int n_utt);
    void release_e2e();
    // Host audio -> host tokens in groups of at most group_samples samples, pipelined.
    int transcribe_host(const float* samples, const int64_t* lengths, int n_utt, uint32_t* tokens, int* counts,
                        int* frames, cudaStream_t s);
    void release_pipeline();
};

}  // namespace telmo
