// parakeet.cu -- the Parakeet TDT encoder and batched greedy TDT decoding on the GPU, behind the
// C ABI.
//
// Host orchestration of Parakeet::encode (src/parakeet.rs:880-902), subsample (:904-993),
// layer (:1011-1172) and decode_inner (:1412-1513) for a batch of utterances packed along the
// rows of every activation matrix, as the Granite model packs them: each matrix product runs
// once over all utterances' rows; the subsampling convolutions, attention and the depthwise
// convolution see utterance boundaries through task lists built here.
//
// Two layout choices differ from the reference's and change no result:
//  * "sub.linear" reads the last convolution channel-major (c * freqs + f). Its columns are
//    permuted on upload to read the convolution's [freq][channel] rows in place; the product's
//    integer sums do not depend on the order of k, and the activation quantization is a
//    per-row maximum, so every output is unchanged.
//  * Every utterance's relative position table is a slice of the longest utterance's table
//    (a row depends only on its position), so the positions are built, quantized and projected
//    once per layer for the whole batch.
// Decoding advances every utterance by one joint step per pass, with the prediction network
// run for the utterances that emitted a token; the passes run as a replayed CUDA graph and the
// host polls for completion every kPollSteps passes (passes after an utterance finishes change
// nothing of it).
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "biasing.h"
#include "frontend.h"
#include "granite_internal.h"
#include "kernels.h"
#include "parakeet_kernels.h"
#include "rowops.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace telmo {

namespace {

constexpr int kSubSpan = 8;     // output time steps of the second depthwise convolution per task
constexpr int kPollSteps = 16;  // decoding passes between completion checks

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
int out_len(int n) { return (n - 1) / 2 + 1; }

void free_vec(DevVec& v) {
    if (v.p) cudaFree(v.p);
    v.p = nullptr;
}

// A device region grown on demand and carved into aligned pieces.
struct Arena {
    char* base = nullptr;
    size_t cap = 0, used = 0;

    int reserve(Ctx* ctx, size_t bytes) {
        used = 0;
        if (bytes <= cap) return TELMO_OK;
        cudaDeviceSynchronize();
        if (base) cudaFree(base);
        base = nullptr;
        cap = 0;
        const size_t want = bytes + bytes / 8 + (1 << 20);
        if (cudaMalloc(&base, want) != cudaSuccess) {
            cudaGetLastError();
            return ctx->fail(TELMO_ERR_CUDA, "parakeet: cannot allocate %zu bytes of device buffers", want);
        }
        cap = want;
        return TELMO_OK;
    }
    template <class T>
    T* take(size_t count) {
        T* p = reinterpret_cast<T*>(base + used);
        used += round_up(count * sizeof(T), 256);
        return p;
    }
    ~Arena() {
        if (base) cudaFree(base);
    }
};

// Bytes a take<T>(count) uses.
template <class T>
size_t piece(size_t count) {
    return round_up(count * sizeof(T), 256);
}

QuantAct quant_piece(Arena& a, size_t rows, int64_t ld) {
    QuantAct q;
    q.ld = ld;
    q.hi = a.take<int8_t>(rows * ld);
    q.lo = a.take<int8_t>(rows * ld);
    q.scale = a.take<float>(rows);
    return q;
}
size_t quant_bytes(size_t rows, int64_t ld) { return 2 * piece<int8_t>(rows * ld) + piece<float>(rows); }

// An instantiated CUDA graph, destroyed with its scope.
struct GraphExec {
    cudaGraphExec_t exec = nullptr;
    void reset() {
        if (exec) cudaGraphExecDestroy(exec);
        exec = nullptr;
    }
    ~GraphExec() { reset(); }
};

}  // namespace

// One conformer layer, as Parakeet's Layer (src/parakeet.rs:269-292).
struct PLayer {
    Norm norm_ff1, norm_att, norm_conv, norm_ff2, norm_out;
    DevWeights ff1_in, ff1_out, qkv, pos, out, pw1, pw2, ff2_in, ff2_out;
    DevVec bias_u, bias_v, dw_w, dw_b;
};

struct Parakeet {
    Ctx* ctx = nullptr;
    Profiler prof;
    telmo_parakeet_config c{};
    // Subsampling (src/parakeet.rs:251-267).
    DevVec conv0_w, conv0_b, dw1_w, dw1_b, pw1_b, dw2_w, dw2_b, pw2_b, linear_b;
    DevWeights pw1, pw2, linear;
    std::vector<PLayer> layers;
    // Decoder (src/parakeet.rs:294-313).
    std::vector<DevWeights> lstm;
    std::vector<DevVec> lstm_b;
    DevVec embedding, pred_proj_b, enc_proj_b, joint_b;
    DevWeights pred_proj, enc_proj, joint;
    int* durations_dev = nullptr;
    int* host_words = nullptr;  // pinned: [0] active utterances, [1] total tokens, [2..3] decoder words
    bool finalized = false;
    int decoder = 1;       // 1: the persistent kernel where the model and device allow it; 0: phases
    int last_decoder = -1;  // which one the last decode ran
    int withhold_cta = -1;  // the next persistent decode's barrier test (telmo_parakeet_test_barrier_timeout)
    double phase_ms[kTdtClocks] = {};  // the persistent decoder's clock, last profiled decode
    long phase_passes = 0;
    long launches = 0;

    Arena enc_arena, dec_arena, e2e_arena, net_arena;
    cudaStream_t capture_stream = nullptr;  // records the decoding passes as a graph
    float* audio_dev = nullptr;
    size_t audio_cap = 0;

    struct Entry {
        DevWeights* mat = nullptr;
        DevVec* vec = nullptr;
        int n = 0, k = 0, len = 0;
    };

    ~Parakeet();
    static int validate(const telmo_parakeet_config& c, std::string& why);
    Entry find(const std::string& name);
    std::string missing();
    int gemm(const QuantAct& a, int m, const DevWeights& w, const float* bias, void* out, int64_t ldc, int act,
             float scale, int acc, cudaStream_t s, int out_kind = kOutF32);
    int quant(const float* x, int64_t ldx, int m, int k, const QuantAct& q, cudaStream_t s);
    int encode(const float* feats, const int* rows, int n_utt, float* out, int* frames_out, int tap, cudaStream_t s);
    int decode(const float* encoded, const int* frames, int n_utt, uint32_t* tokens, int* counts, long* total,
               cudaStream_t s);
    int enc_proj_rows(const float* encoded, int64_t frames, float* out, cudaStream_t s);
    int joint_rows(const float* enc_row, const float* preds, int rows, float* out, int64_t ld_out, cudaStream_t s);
    int predict_rows(const int* tokens, int rows, float* states, float* preds, cudaStream_t s);
    int transcribe_device(const float* samples, const int64_t* lengths, int n_utt, uint32_t* tokens, int* counts,
                          int* frames_out, long* total, cudaStream_t s);
};

Parakeet::~Parakeet() {
    cudaSetDevice(ctx->device);
    auto nrm = [](Norm& n) { free_vec(n.g); free_vec(n.b); };
    for (DevVec* v : {&conv0_w, &conv0_b, &dw1_w, &dw1_b, &pw1_b, &dw2_w, &dw2_b, &pw2_b, &linear_b, &embedding,
                      &pred_proj_b, &enc_proj_b, &joint_b})
        free_vec(*v);
    for (DevWeights* w : {&pw1, &pw2, &linear, &pred_proj, &enc_proj, &joint}) free_weights(w);
    for (auto& w : lstm) free_weights(&w);
    for (auto& b : lstm_b) free_vec(b);
    for (auto& L : layers) {
        nrm(L.norm_ff1); nrm(L.norm_att); nrm(L.norm_conv); nrm(L.norm_ff2); nrm(L.norm_out);
        for (DevWeights* w : {&L.ff1_in, &L.ff1_out, &L.qkv, &L.pos, &L.out, &L.pw1, &L.pw2, &L.ff2_in, &L.ff2_out})
            free_weights(w);
        for (DevVec* v : {&L.bias_u, &L.bias_v, &L.dw_w, &L.dw_b}) free_vec(*v);
    }
    if (durations_dev) cudaFree(durations_dev);
    if (host_words) cudaFreeHost(host_words);
    if (audio_dev) cudaFree(audio_dev);
    if (capture_stream) cudaStreamDestroy(capture_stream);
}

// Config::from_json's checks (src/parakeet.rs:131-140), plus the limits of these kernels.
int Parakeet::validate(const telmo_parakeet_config& c, std::string& why) {
    auto bad = [&](const char* m) { why = m; return TELMO_ERR_MODEL; };
    auto unsupported = [&](const char* m) { why = m; return TELMO_ERR_UNSUPPORTED; };
    if (c.heads <= 0 || c.d_model <= 0 || c.layers <= 0 || c.ff <= 0 || c.sub_channels <= 0 || c.pred_hidden <= 0 ||
        c.pred_layers <= 0 || c.vocab <= 0 || c.max_symbols <= 0)
        return bad("a size is not positive");
    if (c.blank + 1 != c.vocab || c.d_model % c.heads || c.n_mels % 8 || c.conv_kernel % 2 == 0 ||
        c.n_durations <= 0)
        return bad("Its sizes don't fit together.");
    if (c.n_durations > 8 || c.pred_layers > 8) return unsupported("more than 8 durations or prediction layers");
    for (int i = 0; i < c.n_durations; ++i)
        if (c.durations[i] < 0) return bad("a duration is negative");
    if (c.d_model % 128 || c.d_model > 2048) return unsupported("d_model must be a multiple of 128 up to 2048");
    const int hd = c.d_model / c.heads;
    if (hd != 32 && hd != 64 && hd != 128) return unsupported("head size must be 32, 64 or 128");
    if (c.conv_kernel != 3 && c.conv_kernel != 5 && c.conv_kernel != 7 && c.conv_kernel != 9 && c.conv_kernel != 15)
        return unsupported("conv_kernel must be 3, 5, 7, 9 or 15");
    return TELMO_OK;
}

Parakeet::Entry Parakeet::find(const std::string& name) {
    const int d = c.d_model, ch = c.sub_channels, h = c.pred_hidden;
    Entry e;
    auto mat = [&](DevWeights* w, int n, int k) { e.mat = w; e.n = n; e.k = k; };
    auto vec = [&](DevVec* v, int len) { e.vec = v; e.len = len; };
    if (name == "sub.conv0.w") vec(&conv0_w, 9 * ch);
    else if (name == "sub.conv0.b") vec(&conv0_b, ch);
    else if (name == "sub.dw1.w") vec(&dw1_w, 9 * ch);
    else if (name == "sub.dw1.b") vec(&dw1_b, ch);
    else if (name == "sub.pw1") mat(&pw1, ch, ch);
    else if (name == "sub.pw1.b") vec(&pw1_b, ch);
    else if (name == "sub.dw2.w") vec(&dw2_w, 9 * ch);
    else if (name == "sub.dw2.b") vec(&dw2_b, ch);
    else if (name == "sub.pw2") mat(&pw2, ch, ch);
    else if (name == "sub.pw2.b") vec(&pw2_b, ch);
    else if (name == "sub.linear") mat(&linear, d, ch * (c.n_mels / 8));
    else if (name == "sub.linear.b") vec(&linear_b, d);
    else if (name == "dec.embedding") vec(&embedding, c.vocab * h);
    else if (name == "dec.pred_proj") mat(&pred_proj, h, h);
    else if (name == "dec.pred_proj.b") vec(&pred_proj_b, h);
    else if (name == "dec.enc_proj") mat(&enc_proj, h, d);
    else if (name == "dec.enc_proj.b") vec(&enc_proj_b, h);
    else if (name == "dec.joint") mat(&joint, c.vocab + c.n_durations, h);
    else if (name == "dec.joint.b") vec(&joint_b, c.vocab + c.n_durations);
    if (e.mat || e.vec) return e;
    int i = -1;
    char rest[64] = {0};
    if (sscanf(name.c_str(), "dec.lstm.%d%63s", &i, rest) >= 1 && i >= 0 && i < c.pred_layers) {
        if (rest[0] == 0) mat(&lstm[i], 4 * h, 2 * h);
        else if (!strcmp(rest, ".b")) vec(&lstm_b[i], 4 * h);
        return e;
    }
    if (sscanf(name.c_str(), "layers.%d.%63s", &i, rest) != 2 || i < 0 || i >= c.layers) return e;
    PLayer& L = layers[i];
    const std::string r(rest);
    if (r == "ff1_in") mat(&L.ff1_in, c.ff, d);
    else if (r == "ff1_out") mat(&L.ff1_out, d, c.ff);
    else if (r == "ff2_in") mat(&L.ff2_in, c.ff, d);
    else if (r == "ff2_out") mat(&L.ff2_out, d, c.ff);
    else if (r == "qkv") mat(&L.qkv, 3 * d, d);
    else if (r == "pos") mat(&L.pos, d, d);
    else if (r == "out") mat(&L.out, d, d);
    else if (r == "pw1") mat(&L.pw1, 2 * d, d);
    else if (r == "pw2") mat(&L.pw2, d, d);
    else if (r == "bias_u") vec(&L.bias_u, d);
    else if (r == "bias_v") vec(&L.bias_v, d);
    else if (r == "dw.w") vec(&L.dw_w, c.conv_kernel * d);
    else if (r == "dw.b") vec(&L.dw_b, d);
    else {
        static const char* norms[] = {"norm_ff1", "norm_att", "norm_conv", "norm_ff2", "norm_out"};
        Norm* ns[] = {&L.norm_ff1, &L.norm_att, &L.norm_conv, &L.norm_ff2, &L.norm_out};
        for (int k = 0; k < 5; ++k) {
            if (r == std::string(norms[k]) + ".w") vec(&ns[k]->g, d);
            if (r == std::string(norms[k]) + ".b") vec(&ns[k]->b, d);
        }
    }
    return e;
}

std::string Parakeet::missing() {
    std::vector<std::string> names = {"sub.conv0.w", "sub.conv0.b", "sub.dw1.w", "sub.dw1.b", "sub.pw1",
                                      "sub.pw1.b", "sub.dw2.w", "sub.dw2.b", "sub.pw2", "sub.pw2.b",
                                      "sub.linear", "sub.linear.b", "dec.embedding", "dec.pred_proj",
                                      "dec.pred_proj.b", "dec.enc_proj", "dec.enc_proj.b", "dec.joint",
                                      "dec.joint.b"};
    for (int l = 0; l < c.pred_layers; ++l) {
        names.push_back("dec.lstm." + std::to_string(l));
        names.push_back("dec.lstm." + std::to_string(l) + ".b");
    }
    static const char* per_layer[] = {"ff1_in", "ff1_out", "ff2_in", "ff2_out", "qkv", "pos", "out", "pw1", "pw2",
                                      "bias_u", "bias_v", "dw.w", "dw.b", "norm_ff1.w", "norm_ff1.b", "norm_att.w",
                                      "norm_att.b", "norm_conv.w", "norm_conv.b", "norm_ff2.w", "norm_ff2.b",
                                      "norm_out.w", "norm_out.b"};
    for (int i = 0; i < c.layers; ++i)
        for (auto n : per_layer) names.push_back("layers." + std::to_string(i) + "." + n);
    for (auto& n : names) {
        Entry e = find(n);
        if ((e.mat && !e.mat->values) || (e.vec && !e.vec->p) || (!e.mat && !e.vec)) return n;
    }
    return "";
}

int Parakeet::gemm(const QuantAct& a, int m, const DevWeights& w, const float* bias, void* out, int64_t ldc, int act,
                   float scale, int acc, cudaStream_t s, int out_kind) {
    if (m <= 0) return TELMO_OK;
    GemmArgs g;
    g.m = m;
    g.a = a;
    g.w = &w;
    g.bias = bias;
    g.act = act;
    g.scale = scale;
    g.accumulate = acc;
    g.out = out;
    g.ldc = ldc;
    g.out_kind = out_kind;
    g.error = ctx->error_word;
    ++launches;
    if (prof.on) {
        prof.gemm_ops += 2.0 * m * w.n * static_cast<double>(w.k);
        prof.gemm_bytes += 2.0 * m * w.k + static_cast<double>(w.n) * w.k + (acc ? 8.0 : 4.0) * m * w.n + 4.0 * m +
                           8.0 * w.n;
        prof.begin(kProfGemm, s);
    }
    const int rc = ctx->cuda(gemm_i8x2(g, s), "parakeet gemm");
    if (prof.on) prof.end(kProfGemm, s);
    return rc;
}

int Parakeet::quant(const float* x, int64_t ldx, int m, int k, const QuantAct& q, cudaStream_t s) {
    if (m <= 0) return TELMO_OK;
    ++launches;
    return ctx->cuda(quantize_x2(x, ldx, m, k, q, s), "parakeet quant");
}

int Parakeet::encode(const float* feats, const int* rows, int n_utt, float* out, int* frames_out, int tap,
                     cudaStream_t s) {
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "parakeet: the model is not finalized");
    if (n_utt <= 0 || !feats || !rows || !out || !frames_out)
        return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_encode: bad arguments");
    if (tap < -2 || tap >= c.layers) return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_encode: no layer %d", tap);
    const int d = c.d_model, ch = c.sub_channels, hd = d / c.heads, f0 = c.n_mels;
    const int f1 = out_len(f0), f2 = out_len(f1), f3 = out_len(f2);
    // Per-utterance lengths through the subsampling; task lists.
    std::vector<SubTask> front, dw2t;
    std::vector<TxlTask> att;
    std::vector<ConvTask> conv;
    int64_t feat_at = 0, r1 = 0, r2 = 0, m = 0;
    int tmax = 0;
    for (int u = 0; u < n_utt; ++u) {
        const int t0 = rows[u];
        if (t0 < 1) return ctx->fail(TELMO_ERR_MODEL, "parakeet_encode: utterance %d has no feature frames", u);
        const int t1 = out_len(t0), t2 = out_len(t1), t3 = out_len(t2);
        for (int a = 0; a < t2; a += kSubRows)
            front.push_back({static_cast<int>(feat_at), t0, a, std::min(kSubRows, t2 - a),
                             static_cast<int>(r1 + static_cast<int64_t>(a) * f2)});
        for (int a = 0; a < t3; a += kSubSpan)
            dw2t.push_back({static_cast<int>(r1), t2, a, std::min(kSubSpan, t3 - a),
                            static_cast<int>(r2 + static_cast<int64_t>(a) * f3)});
        frames_out[u] = t3;
        tmax = std::max(tmax, t3);
        feat_at += t0;
        r1 += static_cast<int64_t>(t2) * f2;
        r2 += static_cast<int64_t>(t3) * f3;
        m += t3;
    }
    if (r1 * std::max(ch, 1) > (int64_t(1) << 31) || feat_at * f0 > (int64_t(1) << 31))
        return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_encode: batch too large");
    // The tcgen05 attention takes 128 query rows per task, the mma.sync one 64, the other 32.
    const bool mma = txl_attention_mma_supported(hd);
    const bool tc = txl_attention_tc_supported(hd);
    const int q_rows = tc ? 128 : mma ? 64 : 32;
    if (!mma && txl_attention_smem(hd, tmax) > 227 * 1024)
        return ctx->fail(TELMO_ERR_UNSUPPORTED, "parakeet_encode: an utterance of %d frames is too long", tmax);
    int at = 0;
    for (int u = 0; u < n_utt; ++u) {
        const int t = frames_out[u];
        for (int q0 = 0; q0 < t; q0 += q_rows) att.push_back({at, t, q0, tmax - t});
        for (int r = 0; r < t; r += 32) conv.push_back({at, t, at, r, std::min(32, t - r), 1, 0});
        at += t;
    }
    const int M = static_cast<int>(m), P = 2 * tmax - 1;
    const int64_t ld_ch = static_cast<int64_t>(round_up(ch, 16)), ld_lin = static_cast<int64_t>(round_up(ch * f3, 16));
    const int64_t ld_main = static_cast<int64_t>(round_up(std::max(d, c.ff), 16));
    const int64_t big_ld = std::max<int64_t>(c.ff, 3 * d);
    const size_t task_bytes = piece<SubTask>(front.size()) + piece<SubTask>(dw2t.size()) +
                              piece<TxlTask>(att.size()) + piece<ConvTask>(conv.size());
    const size_t bytes = 2 * piece<float>(static_cast<size_t>(r1) * ch) + quant_bytes(r1, ld_ch) +
                         quant_bytes(M, std::max(ld_lin, ld_main)) + 3 * piece<float>(static_cast<size_t>(M) * d) +
                         piece<float>(static_cast<size_t>(M) * big_ld) + 2 * piece<float>(static_cast<size_t>(P) * d) +
                         quant_bytes(P, static_cast<int64_t>(round_up(d, 16))) + piece<float>(static_cast<size_t>(P) * c.heads) +
                         piece<float>(static_cast<size_t>(M) * c.heads) + task_bytes;
    if (int rc = enc_arena.reserve(ctx, bytes)) return rc;
    Arena& A = enc_arena;
    float* sub_a = A.take<float>(static_cast<size_t>(r1) * ch);
    float* sub_b = A.take<float>(static_cast<size_t>(r1) * ch);
    const QuantAct q_sub = quant_piece(A, r1, ld_ch);
    QuantAct q = quant_piece(A, M, std::max(ld_lin, ld_main));
    QuantAct q_lin = q;
    q_lin.ld = ld_lin;
    q.ld = ld_main;
    float* x = A.take<float>(static_cast<size_t>(M) * d);
    float* attn = A.take<float>(static_cast<size_t>(M) * d);
    float* convo = A.take<float>(static_cast<size_t>(M) * d);
    float* big = A.take<float>(static_cast<size_t>(M) * big_ld);
    float* pos = A.take<float>(static_cast<size_t>(P) * d);
    float* pp = A.take<float>(static_cast<size_t>(P) * d);
    const QuantAct q_pos = quant_piece(A, P, static_cast<int64_t>(round_up(d, 16)));
    float* cpos = A.take<float>(static_cast<size_t>(P) * c.heads);
    float* ukey = A.take<float>(static_cast<size_t>(M) * c.heads);
    SubTask* front_dev = A.take<SubTask>(front.size());
    SubTask* dw2_dev = A.take<SubTask>(dw2t.size());
    TxlTask* att_dev = A.take<TxlTask>(att.size());
    ConvTask* conv_dev = A.take<ConvTask>(conv.size());
    auto upload = [&](void* dst, const void* src, size_t n) {
        return ctx->cuda(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, s), "parakeet tasks");
    };
    if (int rc = upload(front_dev, front.data(), sizeof(SubTask) * front.size())) return rc;
    if (int rc = upload(dw2_dev, dw2t.data(), sizeof(SubTask) * dw2t.size())) return rc;
    if (int rc = upload(att_dev, att.data(), sizeof(TxlTask) * att.size())) return rc;
    if (int rc = upload(conv_dev, conv.data(), sizeof(ConvTask) * conv.size())) return rc;

    // ---- subsampling (src/parakeet.rs:904-993) ----------------------------------------------
    if (prof.on) prof.begin(kProfRows, s);
    ++launches;
    if (int rc = ctx->cuda(sub_front(feats, f0, front_dev, static_cast<int>(front.size()), ch, conv0_w.p, conv0_b.p,
                                     dw1_w.p, dw1_b.p, sub_a, s),
                           "parakeet conv0+dw1"))
        return rc;
    if (prof.on) prof.end(kProfRows, s);
    if (int rc = quant(sub_a, ch, static_cast<int>(r1), ch, q_sub, s)) return rc;
    if (int rc = gemm(q_sub, static_cast<int>(r1), pw1, pw1_b.p, sub_b, ch, kActRelu, 1.0f, 0, s)) return rc;
    if (prof.on) prof.begin(kProfRows, s);
    ++launches;
    if (int rc = ctx->cuda(dw3x3s2(sub_b, f2, dw2_dev, static_cast<int>(dw2t.size()), ch, dw2_w.p, dw2_b.p, sub_a, s),
                           "parakeet dw2"))
        return rc;
    if (prof.on) prof.end(kProfRows, s);
    if (int rc = quant(sub_a, ch, static_cast<int>(r2), ch, q_sub, s)) return rc;
    if (int rc = gemm(q_sub, static_cast<int>(r2), pw2, pw2_b.p, sub_b, ch, kActRelu, 1.0f, 0, s)) return rc;
    // sub_b is [M, f3 * ch] row by row: the permuted linear reads it in place.
    if (int rc = quant(sub_b, static_cast<int64_t>(f3) * ch, M, f3 * ch, q_lin, s)) return rc;
    if (int rc = gemm(q_lin, M, linear, linear_b.p, x, d, kActNone, 1.0f, 0, s)) return rc;
    if (tap == -2)
        return ctx->cuda(cudaMemcpyAsync(out, x, sizeof(float) * M * d, cudaMemcpyDeviceToDevice, s), "copy");

    // ---- positions, once for the batch -----------------------------------------------------------
    ++launches;
    if (int rc = ctx->cuda(positions(tmax, d, pos, s), "parakeet positions")) return rc;
    if (int rc = quant(pos, d, P, d, q_pos, s)) return rc;

    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    bool normed = false;  // q holds LN_ff1(x) of the next layer
    for (int i = 0; i < c.layers; ++i) {
        const PLayer& L = layers[i];
        // Feed-forward 1 (src/parakeet.rs:1020-1042): x += 0.5 ff1_out(silu(ff1_in(LN(x)))).
        if (!normed) {
            ++launches;
            if (int rc = ctx->cuda(ln_chain(x, M, d, L.norm_ff1.g.p, L.norm_ff1.b.p, nullptr, nullptr, nullptr, &q, s),
                                   "ln"))
                return rc;
        }
        if (int rc = gemm(q, M, L.ff1_in, nullptr, big, c.ff, kActSilu, 1.0f, 0, s)) return rc;
        if (int rc = quant(big, c.ff, M, c.ff, q, s)) return rc;
        if (int rc = gemm(q, M, L.ff1_out, nullptr, x, d, kActNone, 0.5f, 1, s)) return rc;
        // Attention (src/parakeet.rs:1044-1090).
        ++launches;
        if (int rc = ctx->cuda(ln_chain(x, M, d, L.norm_att.g.p, L.norm_att.b.p, nullptr, nullptr, nullptr, &q, s), "ln"))
            return rc;
        // The tensor-core attention reads Q, K, V and the projected positions as fp16 high/low
        // planes straight from the products' epilogues; the other kernel reads f32.
        const int kind = mma ? kOutF16Split : kOutF32;
        if (int rc = gemm(q, M, L.qkv, nullptr, big, 3 * d, kActNone, 1.0f, 0, s, kind)) return rc;
        if (int rc = gemm(q_pos, P, L.pos, nullptr, pp, d, kActNone, 1.0f, 0, s, kind)) return rc;
        const __half* qkv16 = reinterpret_cast<const __half*>(big);
        const __half* pp16 = reinterpret_cast<const __half*>(pp);
        if (tc) {
            ++launches;
            if (int rc = ctx->cuda(txl_bias_terms(pp16, P, qkv16, M, c.heads, L.bias_u.p, L.bias_v.p, cpos, ukey, s),
                                   "parakeet bias terms"))
                return rc;
        } else if (mma) {
            ++launches;
            if (int rc = ctx->cuda(txl_pos_bias(pp16, static_cast<int64_t>(P) * d, P, c.heads, hd, L.bias_u.p,
                                                L.bias_v.p, cpos, s),
                                   "parakeet position bias"))
                return rc;
        }
        if (prof.on) prof.begin(kProfAttention, s);
        ++launches;
        const cudaError_t ae =
            tc    ? txl_attention_tc(qkv16, M, pp16, P, cpos, ukey, att_dev, static_cast<int>(att.size()), c.heads, hd,
                                     scale, attn, ctx->error_word, s)
            : mma ? txl_attention_mma(qkv16, static_cast<int64_t>(M) * 3 * d, pp16, static_cast<int64_t>(P) * d, cpos,
                                      P, att_dev, static_cast<int>(att.size()), c.heads, hd, L.bias_u.p, scale, attn, s)
                  : txl_attention(big, pp, att_dev, static_cast<int>(att.size()), c.heads, hd, tmax, L.bias_u.p,
                                  L.bias_v.p, scale, attn, s);
        if (int rc = ctx->cuda(ae, "parakeet attention")) return rc;
        if (prof.on) prof.end(kProfAttention, s);
        if (int rc = quant(attn, d, M, d, q, s)) return rc;
        if (int rc = gemm(q, M, L.out, nullptr, x, d, kActNone, 1.0f, 1, s)) return rc;
        // Convolution module (src/parakeet.rs:1092-1140).
        ++launches;
        if (int rc = ctx->cuda(ln_chain(x, M, d, L.norm_conv.g.p, L.norm_conv.b.p, nullptr, nullptr, nullptr, &q, s),
                               "ln"))
            return rc;
        if (int rc = gemm(q, M, L.pw1, nullptr, big, 2 * d, kActNone, 1.0f, 0, s)) return rc;
        if (prof.on) prof.begin(kProfRows, s);
        ++launches;
        if (int rc = ctx->cuda(glu_dwconv_silu(big, d, c.conv_kernel, 1, conv_dev, static_cast<int>(conv.size()), L.dw_w.p,
                                               L.dw_b.p, convo, s),
                               "parakeet dwconv"))
            return rc;
        if (prof.on) prof.end(kProfRows, s);
        if (int rc = quant(convo, d, M, d, q, s)) return rc;
        if (int rc = gemm(q, M, L.pw2, nullptr, x, d, kActNone, 1.0f, 1, s)) return rc;
        // Feed-forward 2 (src/parakeet.rs:1142-1164).
        ++launches;
        if (int rc = ctx->cuda(ln_chain(x, M, d, L.norm_ff2.g.p, L.norm_ff2.b.p, nullptr, nullptr, nullptr, &q, s), "ln"))
            return rc;
        if (int rc = gemm(q, M, L.ff2_in, nullptr, big, c.ff, kActSilu, 1.0f, 0, s)) return rc;
        if (int rc = quant(big, c.ff, M, c.ff, q, s)) return rc;
        if (int rc = gemm(q, M, L.ff2_out, nullptr, x, d, kActNone, 0.5f, 1, s)) return rc;
        // The closing norm (src/parakeet.rs:1166-1171), fused with the next layer's first norm.
        const bool chain = i + 1 < c.layers && i != tap;
        const PLayer* next = chain ? &layers[i + 1] : nullptr;
        ++launches;
        if (int rc = ctx->cuda(ln_chain(x, M, d, L.norm_out.g.p, L.norm_out.b.p, x, chain ? next->norm_ff1.g.p : nullptr,
                                        chain ? next->norm_ff1.b.p : nullptr, chain ? &q : nullptr, s),
                               "ln"))
            return rc;
        normed = chain;
        if (i == tap) break;
    }
    return ctx->cuda(cudaMemcpyAsync(out, x, sizeof(float) * M * d, cudaMemcpyDeviceToDevice, s), "copy");
}

int Parakeet::decode(const float* encoded, const int* frames, int n_utt, uint32_t* tokens, int* counts, long* total,
                     cudaStream_t s) {
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "parakeet: the model is not finalized");
    if (n_utt <= 0 || !encoded || !frames || !tokens || !counts)
        return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_decode: bad arguments");
    const int d = c.d_model, h = c.pred_hidden, L = c.pred_layers, U = n_utt;
    const int outputs = c.vocab + c.n_durations;
    const int64_t ld_logits = static_cast<int64_t>(round_up(outputs, 4));
    std::vector<TdtState> st(U);
    int64_t m = 0, slots = 0;
    for (int u = 0; u < U; ++u) {
        if (frames[u] < 0) return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_decode: negative frame count");
        st[u] = {static_cast<int>(m), frames[u], 0, 0, static_cast<int>(slots), 0};
        m += frames[u];
        slots += static_cast<int64_t>(frames[u]) * c.max_symbols;
    }
    if (m > (1 << 28) || slots > (1 << 28)) return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_decode: batch too large");
    const int M = static_cast<int>(m);
    const int64_t ld_d = static_cast<int64_t>(round_up(d, 16)), ld_2h = static_cast<int64_t>(round_up(2 * h, 16));
    const size_t bytes = quant_bytes(M, ld_d) + piece<float>(static_cast<size_t>(M) * h) + quant_bytes(U, ld_2h) +
                         piece<float>(static_cast<size_t>(U) * ld_logits) + piece<float>(static_cast<size_t>(U) * L * 2 * h) +
                         2 * piece<float>(static_cast<size_t>(U) * h) + piece<float>(static_cast<size_t>(U) * 4 * h) +
                         piece<TdtState>(U) + 2 * piece<int>(U) + piece<int>(4) +
                         piece<uint32_t>(3 * static_cast<size_t>(slots) + 3) + piece<int>(4 * static_cast<size_t>(U)) +
                         piece<unsigned long long>(2 * static_cast<size_t>(U) + kTdtClocks) + piece<unsigned>(8);
    if (int rc = dec_arena.reserve(ctx, bytes)) return rc;
    Arena& A = dec_arena;
    const QuantAct q_enc = quant_piece(A, M, ld_d);
    float* enc_proj_out = A.take<float>(static_cast<size_t>(M) * h);
    const QuantAct qd = quant_piece(A, U, ld_2h);
    float* logits = A.take<float>(static_cast<size_t>(U) * ld_logits);
    float* state = A.take<float>(static_cast<size_t>(U) * L * 2 * h);
    float* pred = A.take<float>(static_cast<size_t>(U) * h);
    float* fresh = A.take<float>(static_cast<size_t>(U) * h);
    float* gates = A.take<float>(static_cast<size_t>(U) * 4 * h);
    TdtState* st_dev = A.take<TdtState>(U);
    int* predict_token = A.take<int>(U);
    int* offsets = A.take<int>(U);
    int* words = A.take<int>(4);
    uint32_t* raw = A.take<uint32_t>(3 * static_cast<size_t>(slots) + 3);
    int* lists = A.take<int>(4 * static_cast<size_t>(U));
    unsigned long long* keys = A.take<unsigned long long>(2 * static_cast<size_t>(U) + kTdtClocks);
    unsigned* pwords = A.take<unsigned>(8);

    if (int rc = ctx->cuda(cudaMemcpyAsync(st_dev, st.data(), sizeof(TdtState) * U, cudaMemcpyHostToDevice, s), "tdt"))
        return rc;
    if (int rc = ctx->cuda(cudaMemsetAsync(state, 0, sizeof(float) * U * L * 2 * h, s), "tdt")) return rc;
    // The joint's projection of every frame (src/parakeet.rs:1438-1449).
    if (int rc = quant(encoded, d, M, d, q_enc, s)) return rc;
    if (int rc = gemm(q_enc, M, enc_proj, enc_proj_b.p, enc_proj_out, h, kActNone, 1.0f, 0, s)) return rc;

    auto rows_kernel = [&](cudaError_t e, const char* what) {
        ++launches;
        return ctx->cuda(e, what);
    };
    int64_t max_frames = 0;
    for (int u = 0; u < U; ++u) max_frames = std::max<int64_t>(max_frames, frames[u]);
    // Each pass advances every unfinished utterance by a frame or emits one of its at most
    // max_symbols tokens on a frame, so frames * (max_symbols + 1) passes bound the loop.
    const int64_t bound = max_frames * (c.max_symbols + 1) + 1;

    // The persistent decoder: the whole loop in one cooperative launch (tdt_persistent.cu), for
    // one-level (Int8) prediction and joint weights.
    bool one_level = joint.lo_values == nullptr && pred_proj.lo_values == nullptr;
    for (const DevWeights& w : lstm) one_level = one_level && w.lo_values == nullptr;
    if (decoder == 1 && max_frames > 0 && one_level) {
        TdtPersistentArgs pa;
        auto mat = [](const DevWeights& w, const float* bias) {
            TdtMatrix m;
            m.w = w.values;
            m.ld = w.ld;
            m.ws = w.scales;
            m.bias = bias;
            m.n = w.n;
            m.k = w.k;
            return m;
        };
        pa.mats[0] = mat(joint, joint_b.p);
        for (int l = 0; l < L; ++l) pa.mats[1 + l] = mat(lstm[l], lstm_b[l].p);
        pa.mats[L + 1] = mat(pred_proj, pred_proj_b.p);
        pa.n_mats = L + 2;
        pa.layers = L;
        pa.h = h;
        pa.n_utt = U;
        pa.vocab = c.vocab;
        pa.blank = c.blank;
        pa.n_dur = c.n_durations;
        pa.max_symbols = c.max_symbols;
        for (int i = 0; i < c.n_durations; ++i) pa.durations[i] = c.durations[i];
        pa.enc_proj = enc_proj_out;
        pa.embedding = embedding.p;
        pa.state = state;
        pa.pred = pred;
        pa.fresh = fresh;
        pa.gates = gates;
        pa.q_hi = qd.hi;
        pa.q_lo = qd.lo;
        pa.q_scale = qd.scale;
        pa.q_ld = qd.ld;
        pa.st = st_dev;
        pa.tokens = raw;
        pa.lists = lists;
        pa.plist = lists + 2 * U;
        pa.ps_of = lists + 3 * U;
        pa.tok_key = keys;
        pa.dur_key = keys + U;
        pa.words = pwords;
        pa.max_passes = bound;
        pa.phase_ns = prof.on ? keys + 2 * U : nullptr;
        pa.withhold_cta = withhold_cta;
        withhold_cta = -1;
        size_t smem = 0;
        if (L + 2 <= kTdtMaxMats && tdt_persistent_plan(pa, ctx->sms, &smem)) {
            if (int rc = ctx->cuda(cudaMemsetAsync(keys, 0, sizeof(unsigned long long) * (2 * U + kTdtClocks), s), "tdt"))
                return rc;
            if (int rc = ctx->cuda(cudaMemsetAsync(pwords, 0, sizeof(unsigned) * 8, s), "tdt")) return rc;
            if (prof.on) prof.begin(kProfRows, s);
            if (int rc = rows_kernel(tdt_persistent(pa, ctx->sms, smem, s), "tdt persistent")) return rc;
            if (prof.on) prof.end(kProfRows, s);
            if (int rc = rows_kernel(tdt_compact(raw, st_dev, U, offsets, tokens, counts, words + 1, s), "tdt compact"))
                return rc;
            if (int rc = ctx->cuda(cudaMemcpyAsync(host_words + 1, words + 1, sizeof(int), cudaMemcpyDeviceToHost, s),
                                   "tdt"))
                return rc;
            if (int rc = ctx->cuda(cudaMemcpyAsync(host_words + 2, pwords, 2 * sizeof(unsigned), cudaMemcpyDeviceToHost,
                                                   s),
                                   "tdt"))
                return rc;
            if (int rc = ctx->cuda(cudaStreamSynchronize(s), "tdt")) return rc;
            if (host_words[2] == kTdtErrBarrier)
                return ctx->fail(TELMO_ERR_DEVICE_TIMEOUT,
                                 "parakeet_decode: a grid barrier of the decoder timed out; its tokens are invalid");
            if (host_words[2] != 0) return ctx->fail(TELMO_ERR_CUDA, "parakeet_decode: decoding did not finish");
            last_decoder = 1;
            if (total) *total = host_words[1];
            if (pa.phase_ns) {
                unsigned long long ns[kTdtClocks];
                if (int rc = ctx->cuda(cudaMemcpy(ns, pa.phase_ns, sizeof ns, cudaMemcpyDeviceToHost), "tdt")) return rc;
                for (int i = 0; i < kTdtClocks; ++i) phase_ms[i] = ns[i] * 1e-6;
                phase_passes = host_words[3];
            }
            return TELMO_OK;
        }
    }
    last_decoder = 0;

    // Parakeet::predict_rows (src/parakeet.rs:1523-1577) for the utterances with a token, from
    // the layer-0 input rows already quantized in qd; the new projections land in `fresh`.
    auto predict = [&](cudaStream_t st) -> int {
        for (int l = 0; l < L; ++l) {
            if (int rc = gemm(qd, U, lstm[l], lstm_b[l].p, gates, 4 * h, kActNone, 1.0f, 0, st)) return rc;
            if (int rc = rows_kernel(lstm_cell_prep(predict_token, U, h, l, L, gates, state, qd, st), "lstm cell"))
                return rc;
        }
        return gemm(qd, U, pred_proj, pred_proj_b.p, fresh, h, kActNone, 1.0f, 0, st);
    };
    // One joint step for every utterance (src/parakeet.rs:1455-1510).
    auto step = [&](cudaStream_t st) -> int {
        if (int rc = rows_kernel(tdt_joint_prep(enc_proj_out, st_dev, U, h, predict_token, fresh, pred, qd, words, st),
                                 "joint input"))
            return rc;
        if (int rc = gemm(qd, U, joint, joint_b.p, logits, ld_logits, kActNone, 1.0f, 0, st)) return rc;
        if (int rc = rows_kernel(tdt_decide_prep(logits, ld_logits, c.vocab, c.blank, durations_dev, c.n_durations,
                                                 c.max_symbols, st_dev, U, raw, predict_token, words, embedding.p,
                                                 state, h, L, qd, st),
                                 "tdt decide"))
            return rc;
        return predict(st);
    };
    if (int rc = rows_kernel(tdt_start(U, c.blank, h, embedding.p, predict_token, qd, s), "tdt start")) return rc;
    if (int rc = predict(s)) return rc;
    // The kPollSteps passes between two completion checks are recorded once as a CUDA graph on a
    // private stream and replayed on the caller's stream (one launch instead of 8 per pass); if
    // recording fails the passes are launched one by one.
    GraphExec graph;
    long graph_launches = 0;
    if (max_frames > 0) {
        if (!capture_stream && cudaStreamCreateWithFlags(&capture_stream, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            capture_stream = nullptr;
        }
        if (capture_stream) {
            const long before = launches;
            const bool prof_on = prof.on;
            prof.on = false;  // no event records inside the graph
            cudaGraph_t g = nullptr;
            int rc = ctx->cuda(cudaStreamBeginCapture(capture_stream, cudaStreamCaptureModeThreadLocal), "tdt capture");
            if (!rc) {
                for (int i = 0; i < kPollSteps && !rc; ++i) rc = step(capture_stream);
                const cudaError_t e = cudaStreamEndCapture(capture_stream, &g);
                if (!rc && e == cudaSuccess && g) rc = ctx->cuda(cudaGraphInstantiate(&graph.exec, g, 0), "tdt graph");
                if (g) cudaGraphDestroy(g);
            }
            prof.on = prof_on;
            graph_launches = launches - before;
            launches = before;
            if (rc || !graph.exec) {
                cudaGetLastError();
                graph.reset();
            }
        }
    }
    int64_t passes = 0;
    while (max_frames > 0) {
        if (graph.exec) {
            if (int rc = ctx->cuda(cudaGraphLaunch(graph.exec, s), "tdt graph")) return rc;
            launches += graph_launches;
        } else {
            for (int i = 0; i < kPollSteps; ++i)
                if (int rc = step(s)) return rc;
        }
        passes += kPollSteps;
        if (int rc = ctx->cuda(cudaMemcpyAsync(host_words, words, sizeof(int), cudaMemcpyDeviceToHost, s), "tdt"))
            return rc;
        if (int rc = ctx->cuda(cudaStreamSynchronize(s), "tdt")) return rc;
        if (host_words[0] == 0) break;
        if (passes > bound) return ctx->fail(TELMO_ERR_CUDA, "parakeet_decode: decoding did not finish");
    }
    if (int rc = rows_kernel(tdt_compact(raw, st_dev, U, offsets, tokens, counts, words + 1, s), "tdt compact"))
        return rc;
    if (int rc = ctx->cuda(cudaMemcpyAsync(host_words + 1, words + 1, sizeof(int), cudaMemcpyDeviceToHost, s), "tdt"))
        return rc;
    if (int rc = ctx->cuda(cudaStreamSynchronize(s), "tdt")) return rc;
    if (total) *total = host_words[1];
    return TELMO_OK;
}

// ---- the networks the biased beam search reads (Networks, src/parakeet.rs:1641-1676) -----------

int Parakeet::enc_proj_rows(const float* encoded, int64_t frames, float* out, cudaStream_t s) {
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "parakeet: the model is not finalized");
    if (frames <= 0 || frames > (1 << 28) || !encoded || !out)
        return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_enc_proj: bad arguments");
    const int d = c.d_model, h = c.pred_hidden, M = static_cast<int>(frames);
    const int64_t ld = static_cast<int64_t>(round_up(d, 16));
    if (int rc = net_arena.reserve(ctx, quant_bytes(M, ld))) return rc;
    const QuantAct q = quant_piece(net_arena, M, ld);
    if (int rc = quant(encoded, d, M, d, q, s)) return rc;
    return gemm(q, M, enc_proj, enc_proj_b.p, out, h, kActNone, 1.0f, 0, s);
}

int Parakeet::joint_rows(const float* enc_row, const float* preds, int rows, float* out, int64_t ld_out,
                         cudaStream_t s) {
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "parakeet: the model is not finalized");
    const int h = c.pred_hidden, outputs = c.vocab + c.n_durations;
    if (rows <= 0 || rows > (1 << 24) || !enc_row || !preds || !out || ld_out < outputs)
        return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_joint: bad arguments");
    const int64_t ld = static_cast<int64_t>(round_up(h, 16));
    if (int rc = net_arena.reserve(ctx, quant_bytes(rows, ld))) return rc;
    const QuantAct q = quant_piece(net_arena, rows, ld);
    ++launches;
    if (int rc = ctx->cuda(tdt_joint_rows(enc_row, preds, rows, h, q, s), "parakeet joint")) return rc;
    return gemm(q, rows, joint, joint_b.p, out, ld_out, kActNone, 1.0f, 0, s);
}

int Parakeet::predict_rows(const int* tokens, int rows, float* states, float* preds, cudaStream_t s) {
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "parakeet: the model is not finalized");
    const int h = c.pred_hidden, L = c.pred_layers;
    if (rows <= 0 || rows > (1 << 24) || !tokens || !states || !preds)
        return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_predict: bad arguments");
    for (int r = 0; r < rows; ++r)
        if (tokens[r] < 0 || tokens[r] >= c.vocab)
            return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_predict: token %d of row %d is not in the vocabulary",
                              tokens[r], r);
    const int64_t ld = static_cast<int64_t>(round_up(2 * h, 16));
    if (int rc = net_arena.reserve(ctx, quant_bytes(rows, ld) + piece<float>(static_cast<size_t>(rows) * 4 * h) +
                                            piece<int>(rows)))
        return rc;
    const QuantAct q = quant_piece(net_arena, rows, ld);
    float* gates = net_arena.take<float>(static_cast<size_t>(rows) * 4 * h);
    int* tok = net_arena.take<int>(rows);
    if (int rc = ctx->cuda(cudaMemcpyAsync(tok, tokens, sizeof(int) * rows, cudaMemcpyHostToDevice, s), "predict"))
        return rc;
    // Parakeet::predict_rows (src/parakeet.rs:1524-1577): layer l's input [x | h_l] quantized,
    // the gate product, the cell update (which quantizes the next layer's input), pred_proj.
    ++launches;
    if (int rc = ctx->cuda(tdt_predict_input(tok, rows, h, L, embedding.p, states, q, s), "predict")) return rc;
    for (int l = 0; l < L; ++l) {
        if (int rc = gemm(q, rows, lstm[l], lstm_b[l].p, gates, 4 * h, kActNone, 1.0f, 0, s)) return rc;
        ++launches;
        if (int rc = ctx->cuda(lstm_cell_prep(tok, rows, h, l, L, gates, states, q, s), "predict")) return rc;
    }
    return gemm(q, rows, pred_proj, pred_proj_b.p, preds, h, kActNone, 1.0f, 0, s);
}

int Parakeet::transcribe_device(const float* samples, const int64_t* lengths, int n_utt, uint32_t* tokens, int* counts,
                                int* frames_out, long* total, cudaStream_t s) {
    // Parakeet::transcribe (src/parakeet.rs:842-867) without biasing or detokenising.
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "parakeet: the model is not finalized");
    if (n_utt <= 0 || !samples || !lengths || !tokens || !counts || !frames_out)
        return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet transcribe: bad arguments");
    std::vector<int> rows(n_utt);
    int64_t total_rows = 0, total_frames = 0;
    for (int u = 0; u < n_utt; ++u) {
        const size_t r = telmo_logmel_rows(TELMO_FRONTEND_PARAKEET, lengths[u]);
        rows[u] = static_cast<int>(r);
        total_rows += static_cast<int64_t>(r);
        total_frames += r ? static_cast<int64_t>(telmo_parakeet_frames_for(r)) : 0;
    }
    if (total_rows > (1 << 28)) return ctx->fail(TELMO_ERR_ARGUMENT, "parakeet transcribe: batch too large");
    const size_t bytes = piece<float>(static_cast<size_t>(total_rows) * c.n_mels + 1) +
                         piece<float>(static_cast<size_t>(total_frames) * c.d_model + 1);
    if (int rc = e2e_arena.reserve(ctx, bytes)) return rc;
    float* feats = e2e_arena.take<float>(static_cast<size_t>(total_rows) * c.n_mels + 1);
    float* enc = e2e_arena.take<float>(static_cast<size_t>(total_frames) * c.d_model + 1);
    if (prof.on) prof.begin(kProfFrontEnd, s);
    if (int rc = telmo_logmel(reinterpret_cast<telmo_ctx*>(ctx), TELMO_FRONTEND_PARAKEET, samples, lengths, n_utt, feats,
                              rows.data(), s))
        return rc;
    if (prof.on) prof.end(kProfFrontEnd, s);
    if (int rc = encode(feats, rows.data(), n_utt, enc, frames_out, -1, s)) return rc;
    return decode(enc, frames_out, n_utt, tokens, counts, total, s);
}

}  // namespace telmo

using namespace telmo;

static Parakeet* as_parakeet(telmo_parakeet* p) { return reinterpret_cast<Parakeet*>(p); }

extern "C" int telmo_parakeet_create(telmo_ctx* cp, const telmo_parakeet_config* config, telmo_parakeet** out) {
    Ctx* ctx = as_ctx(cp);
    if (!ctx || !config || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    std::string why;
    if (int rc = Parakeet::validate(*config, why))
        return ctx->fail(rc, "config doesn't describe a supported Parakeet TDT model. %s", why.c_str());
    if (int rc = ctx->use_device()) return rc;
    auto* p = new Parakeet();
    p->ctx = ctx;
    p->c = *config;
    p->layers.resize(config->layers);
    p->lstm.resize(config->pred_layers);
    p->lstm_b.resize(config->pred_layers);
    int rc = ctx->cuda(cudaMalloc(&p->durations_dev, sizeof(int) * 8), "parakeet");
    if (!rc)
        rc = ctx->cuda(cudaMemcpy(p->durations_dev, config->durations, sizeof(int) * config->n_durations,
                                  cudaMemcpyHostToDevice),
                       "parakeet");
    if (!rc) rc = ctx->cuda(cudaMallocHost(&p->host_words, sizeof(int) * 4), "parakeet");
    if (rc) {
        delete p;
        return rc;
    }
    *out = reinterpret_cast<telmo_parakeet*>(p);
    return TELMO_OK;
}

extern "C" void telmo_parakeet_free(telmo_parakeet* p) { delete as_parakeet(p); }

namespace telmo {

std::vector<int> parakeet_linear_perm(int sub_channels, int n_mels) {
    // Column f * ch + c of the device matrix is the pack's column c * freqs + f.
    const int ch = sub_channels, freqs = n_mels / 8;
    std::vector<int> perm(static_cast<size_t>(ch) * freqs);
    for (int f = 0; f < freqs; ++f)
        for (int cc = 0; cc < ch; ++cc) perm[static_cast<size_t>(f) * ch + cc] = cc * freqs + f;
    return perm;
}

}  // namespace telmo

namespace {

int parakeet_prepare_matrix(Parakeet* p, const char* name, size_t n, size_t k, Parakeet::Entry* out) {
    if (!p || !name) return TELMO_ERR_ARGUMENT;
    Parakeet::Entry e = p->find(name);
    if (!e.mat) return p->ctx->fail(TELMO_ERR_MODEL, "parakeet: no matrix named %s", name);
    if (static_cast<size_t>(e.n) != n || static_cast<size_t>(e.k) != k)
        return p->ctx->fail(TELMO_ERR_MODEL, "parakeet: %s is [%zu, %zu], expected [%d, %d]", name, n, k, e.n, e.k);
    if (int rc = p->ctx->use_device()) return rc;
    free_weights(e.mat);
    p->finalized = false;
    *out = e;
    return TELMO_OK;
}

}  // namespace

extern "C" int telmo_parakeet_set_matrix(telmo_parakeet* pp, const char* name, int precision, size_t n, size_t k,
                                         const void* panel_values, const float* scales) {
    Parakeet* p = as_parakeet(pp);
    Parakeet::Entry e;
    if (int rc = parakeet_prepare_matrix(p, name, n, k, &e)) return rc;
    if (e.mat == &p->linear) {
        // The subsampling output takes its inputs frequency-major on the device (a Q8_0 row is
        // re-encoded with one row scale, which no column order changes).
        const std::vector<int> perm = parakeet_linear_perm(p->c.sub_channels, p->c.n_mels);
        return upload_weights(p->ctx, precision, n, k, panel_values, scales, e.mat, perm.data());
    }
    return upload_weights(p->ctx, precision, n, k, panel_values, scales, e.mat);
}

namespace telmo {

int parakeet_set_device_matrix(telmo_parakeet* pp, const char* name, int precision, size_t n, size_t k,
                               const int8_t* rows, const int8_t* lo, const float* scales) {
    // Device rows are stored with the columns already in the device's order.
    Parakeet* p = as_parakeet(pp);
    Parakeet::Entry e;
    if (int rc = parakeet_prepare_matrix(p, name, n, k, &e)) return rc;
    if (int rc = check_weight_shape(p->ctx, precision, n, k)) return rc;
    return upload_device_rows(p->ctx, precision, n, k, rows, lo, scales, e.mat);
}

}  // namespace telmo

extern "C" int telmo_parakeet_set_vector(telmo_parakeet* pp, const char* name, size_t len, const float* data) {
    Parakeet* p = as_parakeet(pp);
    if (!p || !name || !data) return TELMO_ERR_ARGUMENT;
    Parakeet::Entry e = p->find(name);
    if (!e.vec) return p->ctx->fail(TELMO_ERR_MODEL, "parakeet: no vector named %s", name);
    if (static_cast<size_t>(e.len) != len)
        return p->ctx->fail(TELMO_ERR_MODEL, "parakeet: %s has %zu values, expected %d", name, len, e.len);
    if (int rc = p->ctx->use_device()) return rc;
    free_vec(*e.vec);
    if (int rc = p->ctx->cuda(cudaMalloc(&e.vec->p, sizeof(float) * len), "parakeet vector")) return rc;
    p->finalized = false;
    return p->ctx->cuda(cudaMemcpy(e.vec->p, data, sizeof(float) * len, cudaMemcpyHostToDevice), "parakeet vector");
}

extern "C" int telmo_parakeet_finalize(telmo_parakeet* pp) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    const std::string m = p->missing();
    if (!m.empty()) return p->ctx->fail(TELMO_ERR_MODEL, "parakeet: the pack has no entry %s", m.c_str());
    p->finalized = true;
    return TELMO_OK;
}

extern "C" size_t telmo_parakeet_frames_for(size_t feature_frames) {
    if (feature_frames == 0) return 0;
    size_t t = feature_frames;
    for (int i = 0; i < 3; ++i) t = (t - 1) / 2 + 1;
    return t;
}

extern "C" size_t telmo_parakeet_frames_for_samples(int64_t samples) {
    return telmo_parakeet_frames_for(telmo_logmel_rows(TELMO_FRONTEND_PARAKEET, samples));
}

extern "C" int telmo_parakeet_encode(telmo_parakeet* pp, const float* features, const int* rows, int n_utt, float* out,
                                     int* frames, int tap_layer, void* stream) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (int rc = p->ctx->use_device()) return rc;
    return p->encode(features, rows, n_utt, out, frames, tap_layer, static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_parakeet_decode(telmo_parakeet* pp, const float* encoded, const int* frames, int n_utt,
                                     uint32_t* tokens, int* counts, long* total, void* stream) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (int rc = p->ctx->use_device()) return rc;
    return p->decode(encoded, frames, n_utt, tokens, counts, total, static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_parakeet_transcribe_device(telmo_parakeet* pp, const float* samples, const int64_t* lengths,
                                                int n_utt, uint32_t* tokens, int* counts, int* frames, void* stream) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (int rc = p->ctx->use_device()) return rc;
    return p->transcribe_device(samples, lengths, n_utt, tokens, counts, frames, nullptr,
                                static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_parakeet_transcribe(telmo_parakeet* pp, const float* samples, const int64_t* lengths, int n_utt,
                                         uint32_t* tokens, int* counts, int* frames, void* stream) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    Ctx* ctx = p->ctx;
    if (n_utt <= 0 || !samples || !lengths || !tokens || !counts || !frames)
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_parakeet_transcribe: bad arguments");
    if (int rc = ctx->use_device()) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int64_t total_samples = 0, slots = 0;
    for (int u = 0; u < n_utt; ++u) {
        if (lengths[u] < 0) return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_parakeet_transcribe: negative length");
        total_samples += lengths[u];
        slots += static_cast<int64_t>(telmo_parakeet_frames_for_samples(lengths[u])) * p->c.max_symbols;
    }
    // Device room for the samples, the packed tokens and the counts.
    const size_t need = sizeof(float) * (total_samples + 1) + 256 + sizeof(uint32_t) * (3 * slots + 3) + 256 +
                        sizeof(int) * n_utt;
    if (need > p->audio_cap) {
        cudaStreamSynchronize(s);
        if (p->audio_dev) cudaFree(p->audio_dev);
        p->audio_dev = nullptr;
        p->audio_cap = 0;
        if (int rc = ctx->cuda(cudaMalloc(&p->audio_dev, need + need / 8), "transcribe")) return rc;
        p->audio_cap = need + need / 8;
    }
    char* base = reinterpret_cast<char*>(p->audio_dev);
    float* audio = p->audio_dev;
    uint32_t* tok_dev = reinterpret_cast<uint32_t*>(base + round_up(sizeof(float) * (total_samples + 1), 256));
    int* cnt_dev = reinterpret_cast<int*>(reinterpret_cast<char*>(tok_dev) +
                                          round_up(sizeof(uint32_t) * (3 * slots + 3), 256));
    if (int rc = ctx->cuda(cudaMemcpyAsync(audio, samples, sizeof(float) * total_samples, cudaMemcpyHostToDevice, s),
                           "transcribe"))
        return rc;
    long total = 0;
    if (int rc = p->transcribe_device(audio, lengths, n_utt, tok_dev, cnt_dev, frames, &total, s)) return rc;
    if (int rc = ctx->cuda(cudaMemcpyAsync(tokens, tok_dev, sizeof(uint32_t) * 3 * total, cudaMemcpyDeviceToHost, s),
                           "transcribe"))
        return rc;
    if (int rc = ctx->cuda(cudaMemcpyAsync(counts, cnt_dev, sizeof(int) * n_utt, cudaMemcpyDeviceToHost, s), "transcribe"))
        return rc;
    return ctx->cuda(cudaStreamSynchronize(s), "transcribe");
}

extern "C" int telmo_parakeet_load_pack(telmo_ctx* ctx, const telmo_pack* pk, telmo_parakeet** out) {
    // Parakeet::from_pack (src/parakeet.rs:691-795) onto the device.
    if (!ctx || !pk || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    Ctx* c = as_ctx(ctx);
    const char* model = telmo_pack_model(pk);
    if (strcmp(model, "parakeet-tdt")) return c->fail(TELMO_ERR_MODEL, "The pack holds %s, not Parakeet TDT.", model);
    const void* cj = nullptr;
    size_t cj_len = 0;
    if (telmo_pack_bytes(pk, "config.json", &cj, &cj_len)) return c->fail(TELMO_ERR_MODEL, "Entry config.json is missing.");
    telmo_parakeet_config cfg;
    if (telmo_parakeet_config_from_json(static_cast<const char*>(cj), cj_len, &cfg))
        return c->fail(TELMO_ERR_MODEL, "%s", telmo_pack_last_error());
    telmo_parakeet* pp = nullptr;
    if (int rc = telmo_parakeet_create(ctx, &cfg, &pp)) return rc;
    Parakeet* p = as_parakeet(pp);
    int rc = pack_load_entries(
        pk,
        [&](const char* name, int precision, size_t n, size_t k, const void* v, const float* s) {
            return telmo_parakeet_set_matrix(pp, name, precision, n, k, v, s);
        },
        [&](const char* name, int precision, size_t n, size_t k, const int8_t* v, const int8_t* lo, const float* s) {
            return parakeet_set_device_matrix(pp, name, precision, n, k, v, lo, s);
        },
        [&](const char* name, size_t len, const float* data) { return telmo_parakeet_set_vector(pp, name, len, data); },
        [&](const std::string& name) {
            Parakeet::Entry e = p->find(name);
            return e.mat != nullptr || e.vec != nullptr;
        });
    if (!rc) rc = telmo_parakeet_finalize(pp);
    if (rc) {
        telmo_parakeet_free(pp);
        return rc;
    }
    *out = pp;
    return TELMO_OK;
}

extern "C" int telmo_parakeet_enc_proj(telmo_parakeet* pp, const float* encoded, size_t frames, float* out,
                                       void* stream) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (int rc = p->ctx->use_device()) return rc;
    return p->enc_proj_rows(encoded, static_cast<int64_t>(frames), out, static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_parakeet_joint(telmo_parakeet* pp, const float* enc_row, const float* preds, int rows,
                                    float* out, size_t ld_out, void* stream) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (int rc = p->ctx->use_device()) return rc;
    return p->joint_rows(enc_row, preds, rows, out, static_cast<int64_t>(ld_out), static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_parakeet_predict(telmo_parakeet* pp, const int* tokens, int rows, float* states, float* preds,
                                      void* stream) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (int rc = p->ctx->use_device()) return rc;
    return p->predict_rows(tokens, rows, states, preds, static_cast<cudaStream_t>(stream));
}

namespace {

// Parakeet's joint and prediction networks as the biased beam search reads them (Networks,
// src/parakeet.rs:1634-1676), on the device: the encoder frames from `first` on are projected for
// the joint once; each call stages the hypotheses' rows to the device, runs the batched product
// and brings the outputs back (the search itself is host logic).
class DeviceTdtNetwork : public biasing::TdtNetwork {
public:
    DeviceTdtNetwork(Parakeet* p, const float* enc_proj, size_t first, float* stage, cudaStream_t s)
        : p_(p), enc_proj_(enc_proj), first_(first), stage_(stage), s_(s) {}
    size_t state_width() const override { return static_cast<size_t>(p_->c.pred_layers) * 2 * p_->c.pred_hidden; }
    size_t pred_width() const override { return static_cast<size_t>(p_->c.pred_hidden); }
    // Rows at most biasing::kMaxBeam, so the staging buffers hold any group.
    int joint(size_t frame, const float* preds, size_t rows, float* out) override {
        const size_t h = pred_width(), outputs = static_cast<size_t>(p_->c.vocab + p_->c.n_durations);
        float* preds_dev = stage_;
        float* out_dev = stage_ + biasing::kMaxBeam * h;
        Ctx* ctx = p_->ctx;
        if (int rc = ctx->cuda(cudaMemcpyAsync(preds_dev, preds, rows * h * 4, cudaMemcpyHostToDevice, s_), "beam joint"))
            return rc;
        if (int rc = p_->joint_rows(enc_proj_ + (frame - first_) * h, preds_dev, static_cast<int>(rows), out_dev,
                                    static_cast<int64_t>(outputs), s_))
            return rc;
        if (int rc = ctx->cuda(cudaMemcpyAsync(out, out_dev, rows * outputs * 4, cudaMemcpyDeviceToHost, s_), "beam joint"))
            return rc;
        return ctx->cuda(cudaStreamSynchronize(s_), "beam joint");
    }
    int predict(const int* tokens, size_t rows, float* states, float* preds) override {
        const size_t h = pred_width(), sw = state_width();
        const size_t outputs = static_cast<size_t>(p_->c.vocab + p_->c.n_durations);
        float* states_dev = stage_ + biasing::kMaxBeam * (h + outputs);
        float* preds_dev = states_dev + biasing::kMaxBeam * sw;
        Ctx* ctx = p_->ctx;
        if (int rc = ctx->cuda(cudaMemcpyAsync(states_dev, states, rows * sw * 4, cudaMemcpyHostToDevice, s_), "beam predict"))
            return rc;
        if (int rc = p_->predict_rows(tokens, static_cast<int>(rows), states_dev, preds_dev, s_)) return rc;
        if (int rc = ctx->cuda(cudaMemcpyAsync(states, states_dev, rows * sw * 4, cudaMemcpyDeviceToHost, s_), "beam predict"))
            return rc;
        if (int rc = ctx->cuda(cudaMemcpyAsync(preds, preds_dev, rows * h * 4, cudaMemcpyDeviceToHost, s_), "beam predict"))
            return rc;
        return ctx->cuda(cudaStreamSynchronize(s_), "beam predict");
    }
    // Floats of staging: preds and joint outputs, states and predictions, for kMaxBeam rows.
    static size_t stage_floats(const Parakeet* p) {
        const size_t h = static_cast<size_t>(p->c.pred_hidden);
        const size_t outputs = static_cast<size_t>(p->c.vocab + p->c.n_durations);
        const size_t sw = static_cast<size_t>(p->c.pred_layers) * 2 * h;
        return biasing::kMaxBeam * (h + outputs + sw + h);
    }

private:
    Parakeet* p_;
    const float* enc_proj_;
    size_t first_;
    float* stage_;
    cudaStream_t s_;
};

}  // namespace

extern "C" int telmo_parakeet_beam_search(telmo_parakeet* pp, const float* encoded, size_t frames, size_t offset,
                                          const float* state, const float* pred, size_t frame, size_t on_frame,
                                          const telmo_words* w, uint32_t* tokens, size_t cap, size_t* n_tokens,
                                          void* stream) {
    // Parakeet::beam_search (src/parakeet.rs:1360-1410), from initial_decoder_state (:1321-1335)
    // when no state is given.
    Parakeet* p = as_parakeet(pp);
    if (!p || !w || !n_tokens || (cap && !tokens) || (frames && !encoded) || (!state) != (!pred))
        return TELMO_ERR_ARGUMENT;
    *n_tokens = 0;
    if (int rc = p->ctx->use_device()) return rc;
    if (!p->finalized) return p->ctx->fail(TELMO_ERR_MODEL, "parakeet: the model is not finalized");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto& c = p->c;
    const size_t h = static_cast<size_t>(c.pred_hidden), sw = static_cast<size_t>(c.pred_layers) * 2 * h;
    biasing::TdtShape shape;
    if (int rc = words_tdt_shape(c.vocab, c.blank, c.durations, c.n_durations, c.max_symbols, &shape)) return rc;
    biasing::TdtStart start;
    if (state) {
        start.state.assign(state, state + sw);
        start.pred.assign(pred, pred + h);
        start.frame = frame;
        start.on_frame = on_frame;
    }
    const size_t first = start.frame > offset ? start.frame - offset : 0;
    const biasing::Words& words = words_of(w);
    if (first >= frames || words.forms.empty()) return TELMO_OK;
    const size_t rows = frames - first;
    float* enc_proj = nullptr;
    float* stage = nullptr;
    int rc = p->ctx->cuda(cudaMalloc(&enc_proj, rows * h * sizeof(float)), "beam search");
    if (!rc) rc = p->ctx->cuda(cudaMalloc(&stage, DeviceTdtNetwork::stage_floats(p) * sizeof(float)), "beam search");
    if (!rc) rc = p->enc_proj_rows(encoded + first * static_cast<size_t>(c.d_model), static_cast<int64_t>(rows), enc_proj, s);
    DeviceTdtNetwork net(p, enc_proj, first, stage, s);
    if (!rc && !state) {
        // The decoder's state before any token: the blank's prediction from zero LSTM states.
        start.state.assign(sw, 0.0f);
        start.pred.assign(h, 0.0f);
        const int blank = c.blank;
        rc = net.predict(&blank, 1, start.state.data(), start.pred.data());
    }
    std::vector<biasing::Token> out;
    if (!rc) {
        // Frames are counted from `first` inside the search, as the projected rows are.
        start.frame = first;
        rc = biasing::beam_search(net, shape, frames, std::move(start), words, &out);
    }
    if (enc_proj) cudaFree(enc_proj);
    if (stage) cudaFree(stage);
    if (rc) return rc;
    for (auto& t : out) t.frame += static_cast<uint32_t>(offset);
    return words_tokens_out(out, tokens, cap, n_tokens);
}

extern "C" int telmo_parakeet_set_decoder(telmo_parakeet* pp, int persistent) {
    auto* p = reinterpret_cast<Parakeet*>(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (persistent != 0 && persistent != 1) return p->ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_set_decoder: 0 or 1");
    p->decoder = persistent;
    return TELMO_OK;
}

extern "C" int telmo_parakeet_test_barrier_timeout(telmo_parakeet* pp, int cta) {
    auto* p = reinterpret_cast<Parakeet*>(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (cta < 0 || cta >= p->ctx->sms)
        return p->ctx->fail(TELMO_ERR_ARGUMENT, "parakeet_test_barrier_timeout: no CTA %d", cta);
    p->withhold_cta = cta;
    return TELMO_OK;
}

extern "C" int telmo_parakeet_last_decoder(const telmo_parakeet* pp) {
    const auto* p = reinterpret_cast<const Parakeet*>(pp);
    return p ? p->last_decoder : -1;
}

extern "C" int telmo_parakeet_decoder_profile(const telmo_parakeet* pp, double* ms, long* passes) {
    const auto* p = reinterpret_cast<const Parakeet*>(pp);
    if (!p || !ms) return TELMO_ERR_ARGUMENT;
    for (int i = 0; i < kTdtClocks; ++i) ms[i] = p->phase_ms[i];
    if (passes) *passes = p->phase_passes;
    return TELMO_OK;
}

extern "C" long telmo_parakeet_launches(const telmo_parakeet* pp) {
    const Parakeet* p = reinterpret_cast<const Parakeet*>(pp);
    if (!p) return -1;
    long n = p->launches;
    if (p->ctx->parakeet_fe) n += p->ctx->parakeet_fe->launches;
    return n;
}

extern "C" int telmo_parakeet_profile(telmo_parakeet* pp, int enable) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    p->prof.on = enable != 0;
    return TELMO_OK;
}

extern "C" int telmo_parakeet_profile_read(telmo_parakeet* pp, double* ms, long* launches, double* gemm_ops,
                                           double* gemm_bytes) {
    Parakeet* p = as_parakeet(pp);
    if (!p) return TELMO_ERR_ARGUMENT;
    if (int rc = p->ctx->use_device()) return rc;
    p->prof.read(ms, launches, gemm_ops, gemm_bytes);
    return TELMO_OK;
}
