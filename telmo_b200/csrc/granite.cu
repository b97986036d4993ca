// granite.cu -- the Granite Speech CTC encoder on the GPU, behind the C ABI.
//
// Host orchestration of Granite::encode (src/granite.rs:609-654) and Granite::block_span
// (:802-952) for a batch of utterances whose frames are packed along the rows of every
// activation matrix: each matrix product runs once over all utterances' rows, and only
// attention (128-frame blocks), the depthwise convolution (zero padding at each utterance's
// edges) and the stride-2 pooling see utterance boundaries, through task lists built here.
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "biasing.h"
#include "frontend.h"
#include "granite_internal.h"
#include "kernels.h"
#include "rowops.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace telmo {

static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int Granite::fail(int code, const char* msg) { return ctx->fail(code, "%s", msg); }

static void free_vec(DevVec& v) {
    if (v.p) cudaFree(v.p);
    v.p = nullptr;
}

Granite::~Granite() {
    cudaSetDevice(ctx->device);
    auto lin = [](Lin& l) { free_weights(&l.w); free_vec(l.b); };
    auto nrm = [](Norm& n) { free_vec(n.g); free_vec(n.b); };
    lin(input); lin(head); lin(mid);
    for (auto& b : blocks) {
        lin(b.ff1.up); lin(b.ff1.down); nrm(b.ff1.norm);
        lin(b.ff2.up); lin(b.ff2.down); nrm(b.ff2.norm);
        nrm(b.norm_att); nrm(b.norm_conv); nrm(b.norm_out);
        free_weights(&b.qkv); free_weights(&b.rel);
        if (b.rel16) cudaFree(b.rel16);
        lin(b.out); lin(b.pw1); lin(b.pw2);
        free_vec(b.dw_w); free_vec(b.dw_b);
    }
    release_buffers();
    release_e2e();
    release_pipeline();
    if (audio_dev) cudaFree(audio_dev);
}

void Granite::release_pipeline() {
    if (copy_stream) cudaStreamSynchronize(copy_stream);
    for (int b = 0; b < 2; ++b) {
        if (group_audio[b]) cudaFree(group_audio[b]);
        if (group_pinned[b]) cudaFreeHost(group_pinned[b]);
        if (group_copied[b]) cudaEventDestroy(group_copied[b]);
        if (group_read[b]) cudaEventDestroy(group_read[b]);
        group_audio[b] = group_pinned[b] = nullptr;
        group_copied[b] = group_read[b] = nullptr;
    }
    group_audio_cap = group_pinned_cap = 0;
    if (tokens_pinned) cudaFreeHost(tokens_pinned);
    if (counts_pinned) cudaFreeHost(counts_pinned);
    tokens_pinned = nullptr;
    counts_pinned = nullptr;
    tokens_pinned_cap = counts_pinned_cap = 0;
    if (call_tokens_dev) cudaFree(call_tokens_dev);
    if (call_counts_dev) cudaFree(call_counts_dev);
    call_tokens_dev = nullptr;
    call_counts_dev = nullptr;
    call_tokens_cap = call_counts_cap = 0;
    if (copy_stream) cudaStreamDestroy(copy_stream);
    copy_stream = nullptr;
}

namespace {

bool host_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// Splits utterances 0..n-1, in order, into ceil(total / limit) groups of about equal samples (an
// utterance longer than the limit alone in its group). Returns the first utterance of each group
// and, last, n.
std::vector<int> balanced_groups(const int64_t* lengths, int n, int64_t limit) {
    int64_t total = 0;
    for (int u = 0; u < n; ++u) total += lengths[u];
    const int64_t groups = std::max<int64_t>(1, (total + limit - 1) / limit);
    std::vector<int> first{0};
    int64_t acc = 0, in_group = 0, g = 1;
    for (int u = 0; u < n; ++u) {
        if (u > first.back() && (in_group + lengths[u] > limit || acc >= g * total / groups)) {
            first.push_back(u);
            ++g;
            in_group = 0;
        }
        acc += lengths[u];
        in_group += lengths[u];
    }
    first.push_back(n);
    return first;
}

}  // namespace

int Granite::transcribe_host(const float* samples, const int64_t* lengths, int n_utt, uint32_t* tokens, int* counts,
                             int* frames, cudaStream_t s) {
    const std::vector<int> first = balanced_groups(lengths, n_utt, group_samples);
    const int groups = static_cast<int>(first.size()) - 1;
    std::vector<int64_t> at(groups + 1, 0);  // first sample of each group
    int64_t biggest = 0, total_frames = 0, most_rows = 0, most_frames = 0;
    int most_utts = 0;
    for (int g = 0; g < groups; ++g) {
        int64_t n = 0, rows = 0, frames_g = 0;
        for (int u = first[g]; u < first[g + 1]; ++u) {
            n += lengths[u];
            const size_t r = telmo_logmel_rows(TELMO_FRONTEND_GRANITE, lengths[u]);
            rows += static_cast<int64_t>(r);
            frames_g += static_cast<int64_t>(telmo_granite_frames_for(reinterpret_cast<telmo_granite*>(this), r));
        }
        at[g + 1] = at[g] + n;
        biggest = std::max(biggest, n);
        most_rows = std::max(most_rows, rows);
        most_frames = std::max(most_frames, frames_g);
        most_utts = std::max(most_utts, first[g + 1] - first[g]);
        total_frames += frames_g;
    }
    if (most_rows > (1 << 30)) return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_granite_transcribe: group too large");
    // The device token buffers every group writes must exist before the first group is queued.
    if (int rc = ensure_e2e(static_cast<int>(most_rows) + 1, static_cast<int>(most_frames) + 1, most_utts)) return rc;
    const bool pinned_in = host_pinned(samples);
    const bool pinned_tokens = host_pinned(tokens), pinned_counts = host_pinned(counts);
    if (!copy_stream && cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking) != cudaSuccess)
        return ctx->fail(TELMO_ERR_CUDA, "transcribe: cannot create the copy stream");
    for (int b = 0; b < 2; ++b) {
        if (!group_copied[b] && cudaEventCreateWithFlags(&group_copied[b], cudaEventDisableTiming) != cudaSuccess)
            return ctx->fail(TELMO_ERR_CUDA, "transcribe: cannot create events");
        if (!group_read[b] && cudaEventCreateWithFlags(&group_read[b], cudaEventDisableTiming) != cudaSuccess)
            return ctx->fail(TELMO_ERR_CUDA, "transcribe: cannot create events");
    }
    const size_t need = static_cast<size_t>(biggest) + 1;
    if (need > group_audio_cap) {
        cudaDeviceSynchronize();
        for (float*& p : group_audio) {
            if (p) cudaFree(p);
            p = nullptr;
        }
        group_audio_cap = 0;
        for (float*& p : group_audio)
            if (int rc = ctx->cuda(cudaMalloc(&p, sizeof(float) * (need + need / 8)), "transcribe")) return rc;
        group_audio_cap = need + need / 8;
    }
    if (!pinned_in && need > group_pinned_cap) {
        cudaDeviceSynchronize();
        for (float*& p : group_pinned) {
            if (p) cudaFreeHost(p);
            p = nullptr;
        }
        group_pinned_cap = 0;
        for (float*& p : group_pinned)
            if (int rc = ctx->cuda(cudaHostAlloc(&p, sizeof(float) * (need + need / 8), cudaHostAllocDefault),
                                   "transcribe"))
                return rc;
        group_pinned_cap = need + need / 8;
    }
    const size_t tok_need = 3 * static_cast<size_t>(total_frames) + 3;
    if (!pinned_tokens && tok_need > tokens_pinned_cap) {
        if (tokens_pinned) cudaFreeHost(tokens_pinned);
        tokens_pinned = nullptr;
        tokens_pinned_cap = 0;
        if (int rc = ctx->cuda(cudaHostAlloc(&tokens_pinned, sizeof(uint32_t) * tok_need, cudaHostAllocDefault),
                               "transcribe"))
            return rc;
        tokens_pinned_cap = tok_need;
    }
    if (!pinned_counts && static_cast<size_t>(n_utt) > counts_pinned_cap) {
        if (counts_pinned) cudaFreeHost(counts_pinned);
        counts_pinned = nullptr;
        counts_pinned_cap = 0;
        if (int rc = ctx->cuda(cudaHostAlloc(&counts_pinned, sizeof(int) * n_utt, cudaHostAllocDefault), "transcribe"))
            return rc;
        counts_pinned_cap = static_cast<size_t>(n_utt);
    }
    if (tok_need > call_tokens_cap || static_cast<size_t>(n_utt) > call_counts_cap) {
        cudaDeviceSynchronize();
        if (call_tokens_dev) cudaFree(call_tokens_dev);
        if (call_counts_dev) cudaFree(call_counts_dev);
        call_tokens_dev = nullptr;
        call_counts_dev = nullptr;
        call_tokens_cap = call_counts_cap = 0;
        const size_t tc = std::max(tok_need, call_tokens_cap), uc = std::max<size_t>(n_utt, call_counts_cap);
        if (int rc = ctx->cuda(cudaMalloc(&call_tokens_dev, sizeof(uint32_t) * tc), "transcribe")) return rc;
        if (int rc = ctx->cuda(cudaMalloc(&call_counts_dev, sizeof(int) * uc), "transcribe")) return rc;
        call_tokens_cap = tc;
        call_counts_cap = uc;
    }
    uint32_t* tok_out = pinned_tokens ? tokens : tokens_pinned;
    int* cnt_out = pinned_counts ? counts : counts_pinned;

    // Group j's audio up into buffer j % 2, once group j - 2 no longer reads it (and, through
    // pinned memory, once the copy of group j - 2 has left the pinned buffer).
    auto put = [&](int j) -> int {
        const int b = j % 2;
        const size_t bytes = sizeof(float) * static_cast<size_t>(at[j + 1] - at[j]);
        const float* src = samples + at[j];
        if (!pinned_in) {
            if (j >= 2)
                if (int rc = ctx->cuda(cudaEventSynchronize(group_copied[b]), "transcribe")) return rc;
            std::memcpy(group_pinned[b], src, bytes);
            src = group_pinned[b];
        }
        if (j >= 2)
            if (int rc = ctx->cuda(cudaStreamWaitEvent(copy_stream, group_read[b], 0), "transcribe")) return rc;
        if (int rc = ctx->cuda(cudaMemcpyAsync(group_audio[b], src, bytes, cudaMemcpyHostToDevice, copy_stream),
                               "transcribe"))
            return rc;
        return ctx->cuda(cudaEventRecord(group_copied[b], copy_stream), "transcribe");
    };

    if (int rc = put(0)) return rc;
    int64_t tok_at = 0;
    for (int g = 0; g < groups; ++g) {
        const int b = g % 2, u0 = first[g], n = first[g + 1] - first[g];
        if (int rc = ctx->cuda(cudaStreamWaitEvent(s, group_copied[b], 0), "transcribe")) return rc;
        if (int rc = transcribe_device(group_audio[b], lengths + u0, n, call_tokens_dev + 3 * tok_at,
                                       call_counts_dev + u0, frames + u0, s))
            return rc;
        if (int rc = ctx->cuda(cudaEventRecord(group_read[b], s), "transcribe")) return rc;
        for (int u = u0; u < u0 + n; ++u) tok_at += frames[u];
        // The next group's audio goes up while this one is transcribed.
        if (g + 1 < groups)
            if (int rc = put(g + 1)) return rc;
    }
    if (int rc = ctx->cuda(cudaMemcpyAsync(tok_out, call_tokens_dev, sizeof(uint32_t) * 3 * tok_at,
                                           cudaMemcpyDeviceToHost, s),
                           "transcribe"))
        return rc;
    if (int rc = ctx->cuda(cudaMemcpyAsync(cnt_out, call_counts_dev, sizeof(int) * n_utt, cudaMemcpyDeviceToHost, s),
                           "transcribe"))
        return rc;
    if (int rc = ctx->cuda(cudaStreamSynchronize(s), "transcribe")) return rc;
    if (!pinned_tokens) std::memcpy(tokens, tokens_pinned, sizeof(uint32_t) * 3 * tok_at);
    if (!pinned_counts) std::memcpy(counts, counts_pinned, sizeof(int) * n_utt);
    return TELMO_OK;
}

void Granite::release_e2e() {
    for (void* p : {static_cast<void*>(feats_dev), static_cast<void*>(enc_dev), static_cast<void*>(ids_dev),
                    static_cast<void*>(tokens_dev), static_cast<void*>(counts_dev), static_cast<void*>(first_dev)})
        if (p) cudaFree(p);
    feats_dev = enc_dev = nullptr;
    ids_dev = tokens_dev = nullptr;
    counts_dev = first_dev = nullptr;
    e2e_rows_cap = e2e_frames_cap = e2e_utt_cap = 0;
}

int Granite::ensure_e2e(int rows, int frames, int n_utt) {
    if (rows <= e2e_rows_cap && frames <= e2e_frames_cap && n_utt <= e2e_utt_cap) return TELMO_OK;
    cudaDeviceSynchronize();
    const int R = std::max(rows, e2e_rows_cap), F = std::max(frames, e2e_frames_cap), U = std::max(n_utt, e2e_utt_cap);
    release_e2e();
    auto alloc = [&](void** p, size_t bytes) { return cudaMalloc(p, bytes) == cudaSuccess; };
    const bool ok = alloc(reinterpret_cast<void**>(&feats_dev), sizeof(float) * R * 4 * c.n_mels) &&
                    alloc(reinterpret_cast<void**>(&enc_dev), sizeof(float) * static_cast<size_t>(F) * c.d_model) &&
                    alloc(reinterpret_cast<void**>(&ids_dev), sizeof(uint32_t) * F) &&
                    alloc(reinterpret_cast<void**>(&tokens_dev), sizeof(uint32_t) * 3 * F) &&
                    alloc(reinterpret_cast<void**>(&counts_dev), sizeof(int) * U) &&
                    alloc(reinterpret_cast<void**>(&first_dev), sizeof(int) * 2 * U);
    if (!ok) {
        release_e2e();
        return ctx->fail(TELMO_ERR_CUDA, "granite: cannot allocate end-to-end buffers");
    }
    e2e_rows_cap = R;
    e2e_frames_cap = F;
    e2e_utt_cap = U;
    return TELMO_OK;
}

int Granite::transcribe_device(const float* samples, const int64_t* lengths, int n_utt, uint32_t* tokens, int* counts,
                               int* frames_out, cudaStream_t s) {
    // Granite::transcribe (src/granite.rs:553-582) without biasing or detokenising: features,
    // encoder, CTC head argmax, collapse.
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "granite: the model is not finalized");
    if (n_utt <= 0 || !samples || !lengths || !tokens || !counts || !frames_out)
        return ctx->fail(TELMO_ERR_ARGUMENT, "granite transcribe: bad arguments");
    std::vector<int> rows(n_utt);
    int64_t total_rows = 0, total_frames = 0;
    for (int u = 0; u < n_utt; ++u) {
        const size_t r = telmo_logmel_rows(TELMO_FRONTEND_GRANITE, lengths[u]);
        rows[u] = static_cast<int>(r);
        total_rows += static_cast<int64_t>(r);
        size_t f = r;
        for (int k = 0; k < c.n_subsample; ++k) f /= 2;
        total_frames += static_cast<int64_t>(f);
    }
    if (total_rows > (1 << 30)) return ctx->fail(TELMO_ERR_ARGUMENT, "granite transcribe: batch too large");
    if (int rc = ensure_e2e(static_cast<int>(total_rows) + 1, static_cast<int>(total_frames) + 1, n_utt)) return rc;
    if (prof.on) prof.begin(kProfFrontEnd, s);
    if (int rc = telmo_logmel(reinterpret_cast<telmo_ctx*>(ctx), TELMO_FRONTEND_GRANITE, samples, lengths, n_utt,
                              feats_dev, rows.data(), s))
        return rc;
    if (prof.on) prof.end(kProfFrontEnd, s);
    if (int rc = encode(feats_dev, rows.data(), n_utt, enc_dev, frames_out, -1, s)) return rc;
    if (int rc = frame_ids(enc_dev, static_cast<int>(total_frames), ids_dev, nullptr, s)) return rc;
    std::vector<int> first(2 * static_cast<size_t>(n_utt));
    int at = 0;
    for (int u = 0; u < n_utt; ++u) {
        first[u] = at;
        first[n_utt + u] = frames_out[u];
        at += frames_out[u];
    }
    if (int rc = ctx->cuda(ctx->uploads.upload(first_dev, first.data(), sizeof(int) * first.size(), s), "transcribe"))
        return rc;
    ++launches;
    return ctx->cuda(ctc_collapse(ids_dev, first_dev, first_dev + n_utt, n_utt, static_cast<uint32_t>(c.blank),
                                  tokens, counts, s),
                     "ctc");
}

void Granite::release_buffers() {
    for (void* p : {static_cast<void*>(x), static_cast<void*>(y), static_cast<void*>(big), static_cast<void*>(att),
                    static_cast<void*>(conv), static_cast<void*>(q.hi), static_cast<void*>(q.lo),
                    static_cast<void*>(q.scale), static_cast<void*>(tasks_dev)})
        if (p) cudaFree(p);
    x = y = big = att = conv = nullptr;
    q = QuantAct();
    tasks_dev = nullptr;
    cap_rows = 0;
    tasks_cap = 0;
}

// Config::from_json's checks (src/granite.rs:132-146), plus the limits of these kernels.
int Granite::validate(const telmo_granite_config& c, std::string& why) {
    char buf[256];
    auto bad = [&](const char* m) { why = m; return TELMO_ERR_MODEL; };
    if (c.heads <= 0 || c.head_dim <= 0 || c.heads * c.head_dim != c.d_model) return bad("heads * head_dim != d_model");
    if (c.head_dim % 16) return bad("head_dim is not a multiple of 16");
    if (c.conv_kernel % 2 == 0 || c.conv_kernel <= 0) return bad("conv_kernel is not odd");
    if (c.context <= 0 || c.context > c.max_relative) return bad("context is 0 or above max_relative");
    if (c.layers < 2) return bad("fewer than 2 layers");
    if (c.blank < 0 || c.blank >= c.vocab) return bad("blank is outside the vocabulary");
    if (c.n_subsample < 0 || c.n_subsample > 8) return bad("too many subsample layers");
    for (int i = 0; i < c.n_subsample; ++i) {
        if (c.subsample_layers[i] < 0 || c.subsample_layers[i] >= c.layers) return bad("a subsample layer is out of range");
        if (i && c.subsample_layers[i] <= c.subsample_layers[i - 1]) return bad("subsample layers are not increasing");
    }
    if (c.d_model % 128 || c.d_model > 2048) {
        snprintf(buf, sizeof buf, "d_model %d: this build needs a multiple of 128 up to 2048", c.d_model);
        why = buf;
        return TELMO_ERR_UNSUPPORTED;
    }
    if (c.context > 128) return TELMO_ERR_UNSUPPORTED;
    if (c.head_dim != 16 && c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128) {
        why = "head_dim must be 16, 32, 64 or 128";
        return TELMO_ERR_UNSUPPORTED;
    }
    if (c.ff <= 0 || c.conv_channels <= 0 || c.n_mels <= 0 || c.vocab <= 0) return bad("a size is not positive");
    return TELMO_OK;
}

Granite::Entry Granite::find(const std::string& name) {
    const int d = c.d_model, cc = c.conv_channels;
    Entry e;
    auto mat = [&](DevWeights* w, int n, int k) { e.mat = w; e.n = n; e.k = k; };
    auto vec = [&](DevVec* v, int len) { e.vec = v; e.len = len; };
    if (name == "input") { mat(&input.w, d, 4 * c.n_mels); return e; }
    if (name == "input.b") { vec(&input.b, d); return e; }
    if (name == "head") { mat(&head.w, c.vocab, d); return e; }
    if (name == "head.b") { vec(&head.b, c.vocab); return e; }
    if (name == "mid") { mat(&mid.w, d, c.vocab); return e; }
    if (name == "mid.b") { vec(&mid.b, d); return e; }
    int i = -1;
    char rest[64] = {0};
    if (sscanf(name.c_str(), "blocks.%d.%63s", &i, rest) != 2 || i < 0 || i >= c.layers) return e;
    Block& b = blocks[i];
    const std::string r(rest);
    if (r == "ff1.up") mat(&b.ff1.up.w, c.ff, d);
    else if (r == "ff1.down") mat(&b.ff1.down.w, d, c.ff);
    else if (r == "ff2.up") mat(&b.ff2.up.w, c.ff, d);
    else if (r == "ff2.down") mat(&b.ff2.down.w, d, c.ff);
    else if (r == "qkv") mat(&b.qkv, 3 * d, d);
    else if (r == "rel") mat(&b.rel, 2 * c.context - 1, c.head_dim);
    else if (r == "out") mat(&b.out.w, d, d);
    else if (r == "pw1") mat(&b.pw1.w, 2 * cc, d);
    else if (r == "pw2") mat(&b.pw2.w, d, cc);
    else if (r == "ff1.norm.w") vec(&b.ff1.norm.g, d);
    else if (r == "ff1.norm.b") vec(&b.ff1.norm.b, d);
    else if (r == "ff1.up.b") vec(&b.ff1.up.b, c.ff);
    else if (r == "ff1.down.b") vec(&b.ff1.down.b, d);
    else if (r == "ff2.norm.w") vec(&b.ff2.norm.g, d);
    else if (r == "ff2.norm.b") vec(&b.ff2.norm.b, d);
    else if (r == "ff2.up.b") vec(&b.ff2.up.b, c.ff);
    else if (r == "ff2.down.b") vec(&b.ff2.down.b, d);
    else if (r == "norm_att.w") vec(&b.norm_att.g, d);
    else if (r == "norm_att.b") vec(&b.norm_att.b, d);
    else if (r == "out.b") vec(&b.out.b, d);
    else if (r == "norm_conv.w") vec(&b.norm_conv.g, d);
    else if (r == "norm_conv.b") vec(&b.norm_conv.b, d);
    else if (r == "pw1.b") vec(&b.pw1.b, 2 * cc);
    else if (r == "dw.w") vec(&b.dw_w, c.conv_kernel * cc);
    else if (r == "dw.b") vec(&b.dw_b, cc);
    else if (r == "pw2.b") vec(&b.pw2.b, d);
    else if (r == "norm_out.w") vec(&b.norm_out.g, d);
    else if (r == "norm_out.b") vec(&b.norm_out.b, d);
    return e;
}

std::string Granite::missing() const {
    auto* self = const_cast<Granite*>(this);
    std::vector<std::string> names = {"input", "input.b", "head", "head.b", "mid", "mid.b"};
    static const char* mats[] = {"ff1.up", "ff1.down", "ff2.up", "ff2.down", "qkv", "rel", "out", "pw1", "pw2"};
    static const char* vecs[] = {"ff1.norm.w", "ff1.norm.b", "ff1.up.b", "ff1.down.b", "ff2.norm.w", "ff2.norm.b",
                                 "ff2.up.b", "ff2.down.b", "norm_att.w", "norm_att.b", "out.b", "norm_conv.w",
                                 "norm_conv.b", "pw1.b", "dw.w", "dw.b", "pw2.b", "norm_out.w", "norm_out.b"};
    for (int i = 0; i < c.layers; ++i) {
        for (auto m : mats) names.push_back("blocks." + std::to_string(i) + "." + m);
        for (auto v : vecs) names.push_back("blocks." + std::to_string(i) + "." + v);
    }
    for (auto& n : names) {
        Entry e = self->find(n);
        if ((e.mat && !e.mat->values) || (e.vec && !e.vec->p)) return n;
    }
    return "";
}

int Granite::ensure(int rows, int tasks) {
    if (rows <= cap_rows && tasks <= tasks_cap) return TELMO_OK;
    cudaDeviceSynchronize();
    const int d = c.d_model, cc = c.conv_channels;
    const int R = rows > cap_rows ? static_cast<int>(rows * 1.1) + 64 : cap_rows;
    const int TK = tasks > tasks_cap ? static_cast<int>(tasks * 1.1) + 64 : tasks_cap;
    release_buffers();
    vocab_ld = static_cast<int64_t>(round_up(c.vocab, 4));
    big_ld = std::max(std::max<int64_t>(c.ff, 3 * d), std::max<int64_t>(2 * cc, vocab_ld));
    const int64_t kmax = std::max(std::max<int64_t>(4 * c.n_mels, d), std::max<int64_t>(std::max(c.ff, cc), c.vocab));
    q.ld = static_cast<int64_t>(round_up(kmax, 16));
    auto alloc = [&](void** p, size_t bytes) { return cudaMalloc(p, bytes) == cudaSuccess; };
    bool ok = alloc(reinterpret_cast<void**>(&x), sizeof(float) * R * d) &&
              alloc(reinterpret_cast<void**>(&y), sizeof(float) * R * d) &&
              alloc(reinterpret_cast<void**>(&att), sizeof(float) * R * d) &&
              alloc(reinterpret_cast<void**>(&big), sizeof(float) * R * big_ld) &&
              alloc(reinterpret_cast<void**>(&conv), sizeof(float) * R * cc) &&
              alloc(reinterpret_cast<void**>(&q.hi), static_cast<size_t>(R) * q.ld) &&
              alloc(reinterpret_cast<void**>(&q.lo), static_cast<size_t>(R) * q.ld) &&
              alloc(reinterpret_cast<void**>(&q.scale), sizeof(float) * R) &&
              alloc(reinterpret_cast<void**>(&tasks_dev), sizeof(int) * 8 * static_cast<size_t>(TK));
    if (!ok) {
        release_buffers();
        return ctx->fail(TELMO_ERR_CUDA, "granite: cannot allocate buffers for %d rows", rows);
    }
    cap_rows = R;
    tasks_cap = TK;
    return TELMO_OK;
}

int Granite::gemm(const QuantAct& a, int m, const Lin& l, float* out, int64_t ldc, int act, float scale, int acc,
                  cudaStream_t s) {
    return gemm_w(a, m, l.w, l.b.p, out, ldc, act, scale, acc, s);
}

int Granite::gemm_w(const QuantAct& a, int m, const DevWeights& w, const float* bias, void* out, int64_t ldc,
                    int act, float scale, int acc, cudaStream_t s, int out_kind) {
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
        // Algorithmic work of this product: 2 m n k operations; bytes: both int8 levels of A,
        // the int8 weights, the f32 output (read too when accumulating), scales and bias.
        prof.gemm_ops += 2.0 * m * w.n * static_cast<double>(w.k);
        prof.gemm_bytes += 2.0 * m * w.k + static_cast<double>(w.n) * w.k + (acc ? 8.0 : 4.0) * m * w.n +
                           4.0 * m + 8.0 * w.n;
        prof.begin(kProfGemm, s);
    }
    const int rc = ctx->cuda(gemm_i8x2(g, s), "granite gemm");
    if (prof.on) prof.end(kProfGemm, s);
    return rc;
}

cudaEvent_t Profiler::take() {
    if (pool.empty()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        return e;
    }
    cudaEvent_t e = pool.back();
    pool.pop_back();
    return e;
}

void Profiler::begin(int kind, cudaStream_t s) {
    cudaEvent_t e = take();
    cudaEventRecord(e, s);
    start[kind].push_back(e);
}

void Profiler::end(int kind, cudaStream_t s) {
    cudaEvent_t e = take();
    cudaEventRecord(e, s);
    stop[kind].push_back(e);
    ++count[kind];
}

void Profiler::read(double* ms, long* launches, double* ops, double* bytes) {
    for (int k = 0; k < kProfKinds; ++k) {
        double total = 0.0;
        for (size_t i = 0; i < start[k].size() && i < stop[k].size(); ++i) {
            cudaEventSynchronize(stop[k][i]);
            float t = 0.0f;
            cudaEventElapsedTime(&t, start[k][i], stop[k][i]);
            total += t;
        }
        if (ms) ms[k] = total;
        if (launches) launches[k] = count[k];
        for (auto e : start[k]) pool.push_back(e);
        for (auto e : stop[k]) pool.push_back(e);
        start[k].clear();
        stop[k].clear();
        count[k] = 0;
    }
    if (ops) *ops = gemm_ops;
    if (bytes) *bytes = gemm_bytes;
    gemm_ops = gemm_bytes = 0.0;
}

Profiler::~Profiler() {
    for (int k = 0; k < kProfKinds; ++k) {
        for (auto e : start[k]) cudaEventDestroy(e);
        for (auto e : stop[k]) cudaEventDestroy(e);
    }
    for (auto e : pool) cudaEventDestroy(e);
}

int Granite::feed_forward(const FF& f, float* xb, int m, cudaStream_t s, bool normed) {
    // Granite::feed_forward (src/granite.rs:752-793). With `normed`, q already holds the
    // quantized LN(x) (the previous block's closing norm computed it).
    const int d = c.d_model;
    if (!normed) {
        if (int rc = ctx->cuda(ln_chain(xb, m, d, f.norm.g.p, f.norm.b.p, nullptr, nullptr, nullptr, &q, s), "ln"))
            return rc;
        ++launches;
    }
    if (int rc = gemm(q, m, f.up, big, big_ld, kActSilu, 1.0f, 0, s)) return rc;
    if (int rc = ctx->cuda(quantize_x2(big, big_ld, m, c.ff, q, s), "quant")) return rc;
    ++launches;
    return gemm(q, m, f.down, xb, d, kActNone, 0.5f, 1, s);
}

int Granite::self_condition(float* xs, int n, cudaStream_t s) {
    const int d = c.d_model;
    if (int rc = ctx->cuda(quantize_x2(xs, d, n, d, q, s), "quant")) return rc;
    ++launches;
    if (int rc = gemm(q, n, head, big, vocab_ld, kActNone, 1.0f, 0, s)) return rc;
    if (int rc = ctx->cuda(softmax_quant(big, n, c.vocab, vocab_ld, q, s), "softmax")) return rc;
    ++launches;
    return gemm(q, n, mid, xs, d, kActNone, 1.0f, 1, s);
}

int Granite::span(const Block& b, float* xs, int t, const float* window, int m, int lo, int out_start, int n,
                  float* out, cudaStream_t s) {
    const int d = c.d_model, cc = c.conv_channels, ctxn = c.context;
    const int stride = b.strided ? 2 : 1;
    // Task words: attention blocks of the span from its first frame (start begins a block), the
    // convolution's output spans centred on stride * o - lo of the window, the pooled pairs.
    std::vector<int> host;
    const int nb = (t + ctxn - 1) / ctxn;
    for (int k = 0; k < nb; ++k) {
        host.push_back(k * ctxn);
        host.push_back(std::min(ctxn, t - k * ctxn));
    }
    const int conv_off = static_cast<int>(host.size());
    int nc = 0;
    for (int r = 0; r < n; r += 32, ++nc)
        host.insert(host.end(), {0, m, -out_start, out_start + r, std::min(32, n - r), stride, -lo});
    const int pool_off = static_cast<int>(host.size());
    if (b.strided)
        for (int r = 0; r < n; ++r) host.push_back(2 * (out_start + r) - lo);
    const int words = static_cast<int>(host.size());
    if (int rc = ensure(std::max(t, m), (words + 7) / 8 + 1)) return rc;
    if (int rc = ctx->cuda(ctx->uploads.upload(tasks_dev, host.data(), sizeof(int) * words, s), "granite tasks"))
        return rc;

    if (int rc = feed_forward(b.ff1, xs, t, s)) return rc;
    // Attention (src/granite.rs:820-851).
    if (int rc = ctx->cuda(ln_chain(xs, t, d, b.norm_att.g.p, b.norm_att.b.p, nullptr, nullptr, nullptr, &q, s), "ln"))
        return rc;
    ++launches;
    const bool mma = granite_attention_mma_supported(c.head_dim, ctxn) && b.rel16;
    if (int rc = gemm_w(q, t, b.qkv, nullptr, big, 3 * d, kActNone, 1.0f, 0, s, mma ? kOutF16Split : kOutF32))
        return rc;
    const float scale = static_cast<float>(std::pow(static_cast<double>(c.head_dim), -0.5));
    const AttnTask* att_tasks = reinterpret_cast<const AttnTask*>(tasks_dev);
    const cudaError_t ae =
        mma && granite_attention_tc_supported(c.head_dim, ctxn)
            ? granite_attention_tc(reinterpret_cast<const __half*>(big), t, c.heads, c.head_dim, ctxn, att_tasks, nb,
                                   static_cast<const __half*>(b.rel16), b.rel.scales, scale, att, ctx->error_word, s)
        : mma ? granite_attention_mma(reinterpret_cast<const __half*>(big), static_cast<int64_t>(t) * 3 * d, c.heads,
                                      c.head_dim, ctxn, att_tasks, nb, static_cast<const __half*>(b.rel16),
                                      b.rel.scales, scale, att, s)
              : granite_attention(big, c.heads, c.head_dim, ctxn, att_tasks, nb, b.rel.values, b.rel.ld, b.rel.scales,
                                  scale, att, s);
    if (int rc = ctx->cuda(ae, "attention")) return rc;
    ++launches;
    if (int rc = ctx->cuda(quantize_x2(att, d, t, d, q, s), "quant")) return rc;
    ++launches;
    if (int rc = gemm(q, t, b.out, xs, d, kActNone, 1.0f, 1, s)) return rc;
    // Convolution module over the window's m frames (src/granite.rs:853-944).
    if (int rc = ctx->cuda(ln_chain(window, m, d, b.norm_conv.g.p, b.norm_conv.b.p, nullptr, nullptr, nullptr, &q, s),
                           "ln"))
        return rc;
    ++launches;
    if (int rc = gemm(q, m, b.pw1, big, 2 * cc, kActNone, 1.0f, 0, s)) return rc;
    if (int rc = ctx->cuda(glu_dwconv_silu(big, cc, c.conv_kernel, stride,
                                           reinterpret_cast<const ConvTask*>(tasks_dev + conv_off), nc, b.dw_w.p,
                                           b.dw_b.p, conv, s),
                           "dwconv"))
        return rc;
    ++launches;
    if (b.strided) {
        if (int rc = ctx->cuda(pool_pairs(window, d, tasks_dev + pool_off, n, out, s), "pool")) return rc;
        ++launches;
    } else {
        if (int rc = ctx->cuda(cudaMemcpyAsync(out, window + static_cast<int64_t>(out_start - lo) * d,
                                               sizeof(float) * static_cast<size_t>(n) * d, cudaMemcpyDeviceToDevice, s),
                               "span"))
            return rc;
    }
    if (int rc = ctx->cuda(quantize_x2(conv, cc, n, cc, q, s), "quant")) return rc;
    ++launches;
    if (int rc = gemm(q, n, b.pw2, out, d, kActNone, 1.0f, 1, s)) return rc;
    if (int rc = feed_forward(b.ff2, out, n, s)) return rc;
    ++launches;
    return ctx->cuda(ln_chain(out, n, d, b.norm_out.g.p, b.norm_out.b.p, out, nullptr, nullptr, nullptr, s), "ln");
}

int Granite::encode(const float* feats, const int* rows, int n_utt, float* out, int* frames_out, int tap,
                    cudaStream_t s) {
    if (!finalized) return ctx->fail(TELMO_ERR_MODEL, "granite: the model is not finalized");
    if (n_utt <= 0 || !feats || !rows || !out) return ctx->fail(TELMO_ERR_ARGUMENT, "granite_encode: bad arguments");
    const int d = c.d_model, cc = c.conv_channels, ctxn = c.context;
    // Per-utterance frame counts at every stage.
    std::vector<int> t(rows, rows + n_utt);
    int64_t total = 0;
    for (int u = 0; u < n_utt; ++u) {
        if (t[u] < 0) return ctx->fail(TELMO_ERR_ARGUMENT, "granite_encode: negative row count");
        int f = t[u];
        for (int k = 0; k < c.n_subsample; ++k) f /= 2;
        if (f == 0) {
            char buf[160];
            snprintf(buf, sizeof buf, "The audio is too short (%d feature rows). The model needs at least %d.", t[u],
                     1 << c.n_subsample);
            return fail(TELMO_ERR_MODEL, buf);
        }
        total += t[u];
    }
    if (total > (1 << 30)) return ctx->fail(TELMO_ERR_ARGUMENT, "granite_encode: too many rows");
    const int M0 = static_cast<int>(total);

    // Task lists for every block: attention blocks, convolution spans, pooling sources.
    struct Plan { int att_off, att_n, conv_off, conv_n, pool_off, pool_n, m, m_out; };
    std::vector<Plan> plans(c.layers);
    std::vector<int> host;  // packed task words
    {
        std::vector<int> len = t;
        for (int i = 0; i < c.layers; ++i) {
            const bool strided = blocks[i].strided;
            Plan& p = plans[i];
            int off = 0, off_out = 0;
            p.att_off = static_cast<int>(host.size());
            for (int u = 0; u < n_utt; ++u) {
                for (int b0 = 0; b0 < len[u]; b0 += ctxn) {
                    host.push_back(off + b0);
                    host.push_back(std::min(ctxn, len[u] - b0));
                }
                off += len[u];
            }
            p.m = off;
            p.att_n = (static_cast<int>(host.size()) - p.att_off) / 2;
            p.conv_off = static_cast<int>(host.size());
            off = 0;
            for (int u = 0; u < n_utt; ++u) {
                const int n_out = strided ? len[u] / 2 : len[u];
                for (int r = 0; r < n_out; r += 32) {
                    host.insert(host.end(), {off, len[u], off_out, r, std::min(32, n_out - r), strided ? 2 : 1, 0});
                }
                off += len[u];
                off_out += n_out;
            }
            p.conv_n = (static_cast<int>(host.size()) - p.conv_off) / 7;
            p.m_out = off_out;
            p.pool_off = static_cast<int>(host.size());
            p.pool_n = 0;
            if (strided) {
                off = 0;
                for (int u = 0; u < n_utt; ++u) {
                    for (int r = 0; r < len[u] / 2; ++r) host.push_back(off + 2 * r);
                    off += len[u];
                }
                p.pool_n = static_cast<int>(host.size()) - p.pool_off;
            }
            for (int u = 0; u < n_utt; ++u)
                if (strided) len[u] /= 2;
            if (i == tap)
                for (int u = 0; u < n_utt; ++u) frames_out[u] = len[u];
        }
        if (tap < 0 || tap >= c.layers)
            for (int u = 0; u < n_utt; ++u) frames_out[u] = len[u];
    }
    const int words = static_cast<int>(host.size());
    if (int rc = ensure(M0, (words + 7) / 8 + 1)) return rc;
    // Through pinned staging: the copy is asynchronous and `host` may go out of scope.
    if (int rc = ctx->cuda(ctx->uploads.upload(tasks_dev, host.data(), sizeof(int) * words, s), "granite tasks"))
        return rc;

    // Input projection (src/granite.rs:724-733).
    const int kin = 4 * c.n_mels;
    if (int rc = ctx->cuda(quantize_x2(feats, kin, M0, kin, q, s), "quant")) return rc;
    ++launches;
    if (int rc = gemm(q, M0, input, x, d, kActNone, 1.0f, 0, s)) return rc;

    const float scale = static_cast<float>(std::pow(static_cast<double>(c.head_dim), -0.5));
    const int sc_layer = c.layers / 2 - 1;
    bool normed = false;  // q holds the next block's quantized first norm
    float* cur = x;
    float* other = y;
    for (int i = 0; i < c.layers; ++i) {
        const Block& b = blocks[i];
        const Plan& p = plans[i];
        const int m = p.m;
        if (int rc = feed_forward(b.ff1, cur, m, s, normed)) return rc;
        normed = false;
        // Attention (src/granite.rs:820-851).
        if (int rc = ctx->cuda(ln_chain(cur, m, d, b.norm_att.g.p, b.norm_att.b.p, nullptr, nullptr, nullptr, &q, s), "ln"))
            return rc;
        ++launches;
        // The tensor-core attention takes Q, K and V as fp16 high/low planes straight from the
        // product's epilogue; the other path takes f32.
        const bool mma = granite_attention_mma_supported(c.head_dim, ctxn) && b.rel16;
        if (int rc = gemm_w(q, m, b.qkv, nullptr, big, 3 * d, kActNone, 1.0f, 0, s, mma ? kOutF16Split : kOutF32))
            return rc;
        if (prof.on) prof.begin(kProfAttention, s);
        const AttnTask* att_tasks = reinterpret_cast<const AttnTask*>(tasks_dev + p.att_off);
        const cudaError_t ae =
            mma && granite_attention_tc_supported(c.head_dim, ctxn)
                ? granite_attention_tc(reinterpret_cast<const __half*>(big), m, c.heads, c.head_dim, ctxn, att_tasks,
                                       p.att_n, static_cast<const __half*>(b.rel16), b.rel.scales, scale, att,
                                       ctx->error_word, s)
            : mma ? granite_attention_mma(reinterpret_cast<const __half*>(big), static_cast<int64_t>(m) * 3 * d, c.heads,
                                          c.head_dim, ctxn, att_tasks, p.att_n, static_cast<const __half*>(b.rel16),
                                          b.rel.scales, scale, att, s)
                  : granite_attention(big, c.heads, c.head_dim, ctxn, att_tasks, p.att_n, b.rel.values, b.rel.ld,
                                    b.rel.scales, scale, att, s);
        if (int rc = ctx->cuda(ae, "attention")) return rc;
        if (prof.on) prof.end(kProfAttention, s);
        ++launches;
        if (int rc = ctx->cuda(quantize_x2(att, d, m, d, q, s), "quant")) return rc;
        ++launches;
        if (int rc = gemm(q, m, b.out, cur, d, kActNone, 1.0f, 1, s)) return rc;
        // Convolution module (src/granite.rs:853-944).
        if (int rc = ctx->cuda(ln_chain(cur, m, d, b.norm_conv.g.p, b.norm_conv.b.p, nullptr, nullptr, nullptr, &q, s), "ln"))
            return rc;
        ++launches;
        if (int rc = gemm(q, m, b.pw1, big, 2 * cc, kActNone, 1.0f, 0, s)) return rc;
        if (int rc = ctx->cuda(glu_dwconv_silu(big, cc, c.conv_kernel, b.strided ? 2 : 1,
                                               reinterpret_cast<const ConvTask*>(tasks_dev + p.conv_off),
                                               p.conv_n, b.dw_w.p, b.dw_b.p, conv, s),
                               "dwconv"))
            return rc;
        ++launches;
        float* target = cur;
        if (b.strided) {
            if (int rc = ctx->cuda(pool_pairs(cur, d, tasks_dev + p.pool_off, p.pool_n, other, s), "pool")) return rc;
            ++launches;
            target = other;
        }
        const int n = p.m_out;
        if (int rc = ctx->cuda(quantize_x2(conv, cc, n, cc, q, s), "quant")) return rc;
        ++launches;
        if (int rc = gemm(q, n, b.pw2, target, d, kActNone, 1.0f, 1, s)) return rc;
        if (int rc = feed_forward(b.ff2, target, n, s)) return rc;
        // The closing norm; unless self-conditioning or a tap comes between, fused with the next
        // block's first norm and its quantization (one pass over the residual stream).
        const bool chain = i + 1 < c.layers && i != sc_layer && i != tap;
        const FF* next_ff1 = chain ? &blocks[i + 1].ff1 : nullptr;
        if (int rc = ctx->cuda(ln_chain(target, n, d, b.norm_out.g.p, b.norm_out.b.p, target,
                                        chain ? next_ff1->norm.g.p : nullptr, chain ? next_ff1->norm.b.p : nullptr,
                                        chain ? &q : nullptr, s),
                               "ln"))
            return rc;
        normed = chain;
        ++launches;
        if (b.strided) std::swap(cur, other);
        if (i == sc_layer) {
            // Self-conditioning (src/granite.rs:1040-1069): x += mid(softmax(head(x))).
            if (int rc = ctx->cuda(quantize_x2(cur, d, n, d, q, s), "quant")) return rc;
            ++launches;
            if (int rc = gemm(q, n, head, big, vocab_ld, kActNone, 1.0f, 0, s)) return rc;
            if (int rc = ctx->cuda(softmax_quant(big, n, c.vocab, vocab_ld, q, s), "softmax")) return rc;
            ++launches;
            if (int rc = gemm(q, n, mid, cur, d, kActNone, 1.0f, 1, s)) return rc;
        }
        if (i == tap) {
            return ctx->cuda(cudaMemcpyAsync(out, cur, sizeof(float) * n * d, cudaMemcpyDeviceToDevice, s), "copy");
        }
    }
    return ctx->cuda(cudaMemcpyAsync(out, cur, sizeof(float) * plans.back().m_out * d, cudaMemcpyDeviceToDevice, s),
                     "copy");
}

int Granite::logits(const float* encoded, int frames, float* out, int64_t ld, cudaStream_t s) {
    const int d = c.d_model;
    if (int rc = ensure(frames, 1)) return rc;
    if (int rc = ctx->cuda(quantize_x2(encoded, d, frames, d, q, s), "quant")) return rc;
    ++launches;
    return gemm(q, frames, head, out, ld, kActNone, 1.0f, 0, s);
}

int Granite::frame_ids(const float* encoded, int frames, uint32_t* ids, float* margin, cudaStream_t s) {
    // frame_scores + argmax (src/granite.rs:690-716, :1139-1147).
    if (frames <= 0) return TELMO_OK;
    if (int rc = ensure(frames, 1)) return rc;
    if (int rc = logits(encoded, frames, big, vocab_ld, s)) return rc;
    ++launches;
    return ctx->cuda(argmax_rows(big, frames, c.vocab, vocab_ld, ids, margin, s), "argmax");
}

}  // namespace telmo

using namespace telmo;

static Granite* as_granite(telmo_granite* g) { return reinterpret_cast<Granite*>(g); }

extern "C" int telmo_granite_create(telmo_ctx* cp, const telmo_granite_config* config, telmo_granite** out) {
    Ctx* ctx = as_ctx(cp);
    if (!ctx || !config || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    std::string why;
    if (int rc = Granite::validate(*config, why))
        return ctx->fail(rc, "config doesn't describe a supported Granite Speech CTC model. %s", why.c_str());
    if (int rc = ctx->use_device()) return rc;
    auto* g = new Granite();
    g->ctx = ctx;
    g->c = *config;
    g->blocks.resize(config->layers);
    for (int i = 0; i < config->layers; ++i)
        for (int k = 0; k < config->n_subsample; ++k)
            if (config->subsample_layers[k] == i) g->blocks[i].strided = true;
    *out = reinterpret_cast<telmo_granite*>(g);
    return TELMO_OK;
}

extern "C" void telmo_granite_free(telmo_granite* g) { delete as_granite(g); }

namespace {

// The checks both matrix setters share: the name, the shape, and exact integers for the relative
// tables (they feed the attention kernels). On success the old matrix is freed.
int granite_prepare_matrix(Granite* g, const char* name, int precision, size_t n, size_t k, Granite::Entry* out) {
    if (!g || !name) return TELMO_ERR_ARGUMENT;
    Granite::Entry e = g->find(name);
    if (!e.mat) return g->ctx->fail(TELMO_ERR_MODEL, "granite: no matrix named %s", name);
    if (static_cast<size_t>(e.n) != n || static_cast<size_t>(e.k) != k)
        return g->ctx->fail(TELMO_ERR_MODEL, "granite: %s is [%zu, %zu], expected [%d, %d]", name, n, k, e.n, e.k);
    if (int rc = g->ctx->use_device()) return rc;
    for (auto& b : g->blocks)
        if (e.mat == &b.rel && precision != TELMO_PRECISION_INT8)
            return g->ctx->fail(TELMO_ERR_UNSUPPORTED,
                                "granite: %s feeds the attention kernel as exact integers; it needs "
                                "TELMO_PRECISION_INT8",
                                name);
    free_weights(e.mat);
    g->finalized = false;
    *out = e;
    return TELMO_OK;
}

// The relative tables also get an fp16 copy for the tensor-core attention (int8 values are exact
// in fp16); the per-position scales stay in the weights' scale vector. value(o, i) is the table's
// int8 value at position o, dimension i.
template <class Value>
int granite_upload_rel16(Granite* g, const DevWeights* mat, size_t n, size_t k, Value value) {
    for (auto& b : g->blocks) {
        if (mat != &b.rel) continue;
        if (b.rel16) cudaFree(b.rel16);
        b.rel16 = nullptr;
        std::vector<__half> rel16(n * k);
        for (size_t o = 0; o < n; ++o)
            for (size_t i = 0; i < k; ++i) rel16[o * k + i] = __float2half(static_cast<float>(value(o, i)));
        if (int rc = g->ctx->cuda(cudaMalloc(&b.rel16, sizeof(__half) * n * k), "granite rel")) return rc;
        return g->ctx->cuda(cudaMemcpy(b.rel16, rel16.data(), sizeof(__half) * n * k, cudaMemcpyHostToDevice),
                            "granite rel");
    }
    return TELMO_OK;
}

}  // namespace

extern "C" int telmo_granite_set_matrix(telmo_granite* gp, const char* name, int precision, size_t n, size_t k,
                                        const void* panel_values, const float* scales) {
    Granite* g = as_granite(gp);
    Granite::Entry e;
    if (int rc = granite_prepare_matrix(g, name, precision, n, k, &e)) return rc;
    if (int rc = upload_weights(g->ctx, precision, n, k, panel_values, scales, e.mat)) return rc;
    const int8_t* v = static_cast<const int8_t*>(panel_values);
    return granite_upload_rel16(g, e.mat, n, k, [&](size_t o, size_t i) { return v[((o / 16) * k + i) * 16 + o % 16]; });
}

namespace telmo {

int granite_set_device_matrix(telmo_granite* gp, const char* name, int precision, size_t n, size_t k,
                              const int8_t* rows, const int8_t* lo, const float* scales) {
    Granite* g = as_granite(gp);
    Granite::Entry e;
    if (int rc = granite_prepare_matrix(g, name, precision, n, k, &e)) return rc;
    if (int rc = check_weight_shape(g->ctx, precision, n, k)) return rc;
    if (int rc = upload_device_rows(g->ctx, precision, n, k, rows, lo, scales, e.mat)) return rc;
    const size_t ld = round_up(k, 16);
    return granite_upload_rel16(g, e.mat, n, k, [&](size_t o, size_t i) { return rows[o * ld + i]; });
}

}  // namespace telmo

extern "C" int telmo_granite_set_vector(telmo_granite* gp, const char* name, size_t len, const float* data) {
    Granite* g = as_granite(gp);
    if (!g || !name || !data) return TELMO_ERR_ARGUMENT;
    Granite::Entry e = g->find(name);
    if (!e.vec) return g->ctx->fail(TELMO_ERR_MODEL, "granite: no vector named %s", name);
    if (static_cast<size_t>(e.len) != len)
        return g->ctx->fail(TELMO_ERR_MODEL, "granite: %s has %zu values, expected %d", name, len, e.len);
    if (int rc = g->ctx->use_device()) return rc;
    if (e.vec->p) cudaFree(e.vec->p);
    e.vec->p = nullptr;
    if (int rc = g->ctx->cuda(cudaMalloc(&e.vec->p, sizeof(float) * len), "granite vector")) return rc;
    g->finalized = false;
    return g->ctx->cuda(cudaMemcpy(e.vec->p, data, sizeof(float) * len, cudaMemcpyHostToDevice), "granite vector");
}

extern "C" int telmo_granite_finalize(telmo_granite* gp) {
    Granite* g = as_granite(gp);
    if (!g) return TELMO_ERR_ARGUMENT;
    const std::string m = g->missing();
    if (!m.empty()) return g->ctx->fail(TELMO_ERR_MODEL, "granite: the pack has no entry %s", m.c_str());
    g->finalized = true;
    return TELMO_OK;
}

extern "C" size_t telmo_granite_frames_for(const telmo_granite* gp, size_t rows) {
    const Granite* g = reinterpret_cast<const Granite*>(gp);
    if (!g) return 0;
    for (int k = 0; k < g->c.n_subsample; ++k) rows /= 2;
    return rows;
}

extern "C" int telmo_granite_encode(telmo_granite* gp, const float* features, const int* rows, int n_utt, float* out,
                                    int* frames, int tap_layer, void* stream) {
    Granite* g = as_granite(gp);
    if (!g || !frames) return TELMO_ERR_ARGUMENT;
    if (int rc = g->ctx->use_device()) return rc;
    return g->encode(features, rows, n_utt, out, frames, tap_layer, static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_granite_logits(telmo_granite* gp, const float* encoded, size_t frames, float* logits, size_t ld,
                                    void* stream) {
    Granite* g = as_granite(gp);
    if (!g || !encoded || !logits) return TELMO_ERR_ARGUMENT;
    if (ld < static_cast<size_t>(g->c.vocab)) return g->ctx->fail(TELMO_ERR_ARGUMENT, "logits: ld below vocab");
    if (frames == 0) return TELMO_OK;
    if (int rc = g->ctx->use_device()) return rc;
    return g->logits(encoded, static_cast<int>(frames), logits, static_cast<int64_t>(ld),
                     static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_granite_frame_ids(telmo_granite* gp, const float* encoded, size_t frames, uint32_t* ids,
                                       float* margin, void* stream) {
    Granite* g = as_granite(gp);
    if (!g || !encoded || !ids) return TELMO_ERR_ARGUMENT;
    if (int rc = g->ctx->use_device()) return rc;
    return g->frame_ids(encoded, static_cast<int>(frames), ids, margin, static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_granite_decode_biased(telmo_granite* gp, const float* encoded, size_t frames, const telmo_words* w,
                                           uint32_t* tokens, size_t cap, size_t* n_tokens, void* stream) {
    // Granite::decode_biased (src/granite.rs:584-604) up to the text rewrites: frame_scores with
    // the words' columns (:690-716) on the device, then ctc_tokens and spot on the host.
    Granite* g = as_granite(gp);
    if (!g || !w || !n_tokens || (cap && !tokens) || (frames && !encoded)) return TELMO_ERR_ARGUMENT;
    *n_tokens = 0;
    if (frames == 0) return TELMO_OK;
    if (frames > (1u << 24)) return g->ctx->fail(TELMO_ERR_ARGUMENT, "decode_biased: too many frames");
    if (int rc = g->ctx->use_device()) return rc;
    if (!g->finalized) return g->ctx->fail(TELMO_ERR_MODEL, "granite: the model is not finalized");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const biasing::Words& words = words_of(w);
    const size_t width = 2 + words.tokens.size();
    uint32_t* ids_dev = nullptr;
    float* scores_dev = nullptr;
    std::vector<uint32_t> ids(frames);
    std::vector<float> scores(words.forms.empty() ? 0 : frames * width);
    int rc = g->ctx->cuda(cudaMalloc(&ids_dev, frames * sizeof(uint32_t)), "decode_biased");
    if (!rc && !scores.empty()) rc = g->ctx->cuda(cudaMalloc(&scores_dev, scores.size() * sizeof(float)), "decode_biased");
    // The logits stay in the model's scratch after the ids; the score rows are gathered from them.
    if (!rc) rc = g->frame_ids(encoded, static_cast<int>(frames), ids_dev, nullptr, s);
    if (!rc && scores_dev)
        rc = words_score_rows(w, g->big, static_cast<int64_t>(frames), g->c.vocab, g->vocab_ld, g->c.blank, scores_dev, s);
    if (!rc)
        rc = g->ctx->cuda(cudaMemcpyAsync(ids.data(), ids_dev, frames * sizeof(uint32_t), cudaMemcpyDeviceToHost, s),
                          "decode_biased");
    if (!rc && scores_dev)
        rc = g->ctx->cuda(cudaMemcpyAsync(scores.data(), scores_dev, scores.size() * sizeof(float), cudaMemcpyDeviceToHost, s),
                          "decode_biased");
    if (!rc) rc = g->ctx->cuda(cudaStreamSynchronize(s), "decode_biased");
    if (ids_dev) cudaFree(ids_dev);
    if (scores_dev) cudaFree(scores_dev);
    if (rc) return rc;
    const std::vector<biasing::Token> greedy = biasing::ctc_tokens(ids.data(), frames, static_cast<uint32_t>(g->c.blank));
    std::vector<biasing::Token> out;
    std::vector<std::pair<size_t, size_t>> ranges;
    biasing::spot(words, greedy, scores.data(), frames, 0, &out, &ranges);
    return words_tokens_out(out, tokens, cap, n_tokens);
}

extern "C" size_t telmo_granite_frames_for_samples(const telmo_granite* g, int64_t samples) {
    return telmo_granite_frames_for(g, telmo_logmel_rows(TELMO_FRONTEND_GRANITE, samples));
}

extern "C" int telmo_granite_transcribe_device(telmo_granite* gp, const float* samples, const int64_t* lengths,
                                               int n_utt, uint32_t* tokens, int* counts, int* frames, void* stream) {
    Granite* g = as_granite(gp);
    if (!g) return TELMO_ERR_ARGUMENT;
    if (int rc = g->ctx->use_device()) return rc;
    return g->transcribe_device(samples, lengths, n_utt, tokens, counts, frames, static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_granite_transcribe(telmo_granite* gp, const float* samples, const int64_t* lengths, int n_utt,
                                        uint32_t* tokens, int* counts, int* frames, void* stream) {
    Granite* g = as_granite(gp);
    if (!g) return TELMO_ERR_ARGUMENT;
    if (n_utt <= 0 || !samples || !lengths || !tokens || !counts || !frames)
        return g->ctx->fail(TELMO_ERR_ARGUMENT, "telmo_granite_transcribe: bad arguments");
    if (!g->finalized) return g->ctx->fail(TELMO_ERR_MODEL, "granite: the model is not finalized");
    for (int u = 0; u < n_utt; ++u)
        if (lengths[u] < 0) return g->ctx->fail(TELMO_ERR_ARGUMENT, "telmo_granite_transcribe: negative length");
    if (int rc = g->ctx->use_device()) return rc;
    return g->transcribe_host(samples, lengths, n_utt, tokens, counts, frames, static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_granite_set_transcribe_group(telmo_granite* gp, double seconds) {
    Granite* g = as_granite(gp);
    if (!g) return TELMO_ERR_ARGUMENT;
    if (!(seconds >= 0.02) || seconds > 1e6)
        return g->ctx->fail(TELMO_ERR_ARGUMENT, "telmo_granite_set_transcribe_group: %g seconds is out of range",
                            seconds);
    g->group_samples = static_cast<int64_t>(seconds * 16000.0);
    return TELMO_OK;
}

extern "C" int telmo_granite_profile(telmo_granite* gp, int enable) {
    Granite* g = as_granite(gp);
    if (!g) return TELMO_ERR_ARGUMENT;
    g->prof.on = enable != 0;
    return TELMO_OK;
}

extern "C" int telmo_granite_profile_read(telmo_granite* gp, double* ms, long* launches, double* gemm_ops,
                                          double* gemm_bytes) {
    Granite* g = as_granite(gp);
    if (!g) return TELMO_ERR_ARGUMENT;
    if (int rc = g->ctx->use_device()) return rc;
    g->prof.read(ms, launches, gemm_ops, gemm_bytes);
    return TELMO_OK;
}

extern "C" long telmo_granite_launches(const telmo_granite* gp) {
    const Granite* g = reinterpret_cast<const Granite*>(gp);
    if (!g) return -1;
    long n = g->launches;
    if (g->ctx->granite_fe) n += g->ctx->granite_fe->launches;
    return n;
}

extern "C" int telmo_ctc_tokens(telmo_ctx* cp, const uint32_t* ids, const int* first, const int* frames, int n_utt,
                                uint32_t blank, uint32_t* tokens, int* counts, void* stream) {
    Ctx* ctx = as_ctx(cp);
    if (!ctx) return TELMO_ERR_ARGUMENT;
    if (n_utt == 0) return TELMO_OK;
    if (!ids || !first || !frames || !tokens || !counts || n_utt < 0)
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_ctc_tokens: bad arguments");
    if (int rc = ctx->use_device()) return rc;
    return ctx->cuda(ctc_collapse(ids, first, frames, n_utt, blank, tokens, counts, static_cast<cudaStream_t>(stream)),
                     "telmo_ctc_tokens");
}
