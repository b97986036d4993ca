// granite_stream.cu -- GraniteStream (src/granite_stream.rs) on the GPU: one utterance encoded
// while it is spoken, each update running only what new audio can change.
//
// Granite's attention stays inside blocks of `context` frames, so an update runs the strided
// blocks over their attention blocks that hold new or changed frames (with the edge frames before
// them read from cached post-attention states by the convolution), and the other blocks from the
// first frame of their current block, the `frozen` frame; earlier outputs are kept as they were.
// The host keeps the reference's bookkeeping (rows, frozen frame, first changed frame, the
// running peak that floors the features); every layer's post-attention states and outputs, the
// samples, the log-mel frames and the features live on the device, and each span runs the
// offline encoder's kernels (Granite::span). A single finished update over a whole utterance is
// the offline encode.
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "frontend.h"
#include "granite_internal.h"

#include <algorithm>
#include <cmath>
#include <vector>

namespace telmo {

namespace {

// A device buffer that grows, keeping its first `keep` bytes.
struct Grow {
    void* p = nullptr;
    size_t cap = 0;
    int ensure(Ctx* ctx, size_t bytes, size_t keep, cudaStream_t s) {
        if (bytes <= cap) return TELMO_OK;
        void* q = nullptr;
        const size_t want = std::max<size_t>(2 * bytes, 1 << 20);  // doubling: few reallocations
        if (int rc = ctx->cuda(cudaMalloc(&q, want), "stream buffer")) return rc;
        if (p && keep) {
            if (int rc = ctx->cuda(cudaMemcpyAsync(q, p, std::min(keep, cap), cudaMemcpyDeviceToDevice, s), "stream"))
                return rc;
            if (int rc = ctx->cuda(cudaStreamSynchronize(s), "stream")) return rc;
        }
        if (p) cudaFree(p);
        p = q;
        cap = want;
        return TELMO_OK;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
    ~Grow() {
        if (p) cudaFree(p);
    }
};

constexpr int HOP = 160, N_FFT = 512;

}  // namespace

struct GraniteStream {
    Granite* g = nullptr;
    Ctx* ctx = nullptr;
    FrontEnd* fe = nullptr;
    Grow samples, logs, features, input, meta, peak, ids_dev;
    std::vector<Grow> states, outs;
    int64_t n = 0;
    int log_frames = 0, rows = 0, frozen = 0, lag = 16, first_changed = 0;
    float peak_v = -INFINITY, floor_peak = -INFINITY;
    bool finished = false;
    std::vector<int> state_rows, out_rows;
    std::vector<uint32_t> ids;

    int update(bool fin, cudaStream_t s);
};

int GraniteStream::update(bool fin, cudaStream_t s) {
    // GraniteStream::update (src/granite_stream.rs:209-361).
    if (finished) return ctx->fail(TELMO_ERR_ARGUMENT, "granite_stream_update: the stream already finished");
    const telmo_granite_config& c = g->c;
    const int d = c.d_model, ctxn = c.context, n_mels = c.n_mels, half = c.conv_kernel / 2, width = 4 * n_mels;
    first_changed = static_cast<int>(ids.size());
    int64_t frames, len;
    if (!fin) {
        // complete_frames (src/granite_features.rs:84-92): windows inside the samples so far.
        frames = n <= N_FFT / 2 ? 0 : (n - N_FFT / 2) / HOP + 1;
        len = n;
    } else if (n >= 2 * HOP) {
        frames = 2 * ((n / HOP + 1) / 2);
        len = std::max<int64_t>(n, (frames - 1) * HOP + 1);
    } else {
        frames = log_frames;
        len = n;
    }
    finished = fin;
    if (frames > (1 << 26)) return ctx->fail(TELMO_ERR_ARGUMENT, "granite_stream_update: stream too long");
    if (frames > log_frames) {
        if (int rc = logs.ensure(ctx, sizeof(float) * frames * n_mels, sizeof(float) * log_frames * n_mels, s))
            return rc;
        if (int rc = fe->granite_stream_frames(samples.as<float>(), n, len, log_frames, static_cast<int>(frames),
                                               logs.as<float>(), peak.as<float>() + 1, meta.p, s))
            return rc;
        float newest = -INFINITY;
        if (int rc = ctx->cuda(cudaMemcpyAsync(&newest, peak.as<float>() + 1, sizeof(float), cudaMemcpyDeviceToHost, s),
                               "stream peak"))
            return rc;
        if (int rc = ctx->cuda(cudaStreamSynchronize(s), "stream peak")) return rc;
        peak_v = std::max(peak_v, newest);
        log_frames = static_cast<int>(frames);
    }
    // A row needs the frame after it for its last delta, until the end repeats the last frame.
    const int new_rows = static_cast<int>(fin ? frames / 2 : (frames > 0 ? (frames - 1) / 2 : 0));
    if (new_rows <= rows) return TELMO_OK;

    // Rows of the first block's current attention block are stacked again with the floor of the
    // loudest frame so far; when it got louder, so are the rows the unfrozen frames read.
    int first_row = rows / ctxn * ctxn;
    if (peak_v > floor_peak) {
        int row = frozen;
        for (int k = 0; k < c.n_subsample; ++k) row = std::max(2 * row - half, 0) / ctxn * ctxn;
        first_row = std::min(first_row, row);
        floor_peak = peak_v;
    }
    if (int rc = features.ensure(ctx, sizeof(float) * new_rows * width, sizeof(float) * rows * width, s)) return rc;
    if (int rc = ctx->cuda(cudaMemcpyAsync(peak.as<float>(), &peak_v, sizeof(float), cudaMemcpyHostToDevice, s), "peak"))
        return rc;
    if (int rc = fe->granite_stream_rows(logs.as<float>(), log_frames, peak.as<float>(), first_row, new_rows,
                                         features.as<float>(), meta.p, s))
        return rc;
    // Input projection of the restacked rows (src/granite.rs:724-733).
    if (int rc = input.ensure(ctx, sizeof(float) * new_rows * d, sizeof(float) * rows * d, s)) return rc;
    // The model's work buffers in power-of-two steps of rows, so a growing utterance reallocates
    // them (a device-wide sync) a few times rather than at every update.
    int reserve = 512;
    while (reserve < new_rows) reserve *= 2;
    if (int rc = g->ensure(reserve, reserve / 4 + 64)) return rc;  // task words of a span: < rows / 6
    const int m_in = new_rows - first_row;
    if (int rc = ctx->cuda(quantize_x2(features.as<float>() + static_cast<int64_t>(first_row) * width, width, m_in,
                                       width, g->q, s),
                           "quant"))
        return rc;
    ++g->launches;
    if (int rc = g->gemm(g->q, m_in, g->input, input.as<float>() + static_cast<int64_t>(first_row) * d, d, kActNone,
                         1.0f, 0, s))
        return rc;
    rows = new_rows;
    // Cached features past the restacked rows are current: keep the stream's rows.
    int changed = first_row, frames_in = rows;
    const int sc_layer = c.layers / 2 - 1;
    for (int i = 0; i < c.layers; ++i) {
        const Block& b = g->blocks[i];
        int start, out_start, frames_out;
        if (b.strided) {
            start = changed / ctxn * ctxn;
            // Outputs before start / 2 whose convolution reaches the changed block.
            out_start = (std::max(start - half, 0) + 1) / 2;
            frames_out = frames_in / 2;
        } else {
            start = out_start = frozen;
            frames_out = frames_in;
        }
        if (start >= frames_in || out_start >= frames_out) return ctx->cuda(cudaStreamSynchronize(s), "stream");
        const int lo = std::max((b.strided ? 2 * out_start : out_start) - half, 0);  // conv_context
        Grow& st = states[i];
        Grow& out = outs[i];
        if (int rc = st.ensure(ctx, sizeof(float) * static_cast<size_t>(frames_in) * d,
                               sizeof(float) * static_cast<size_t>(state_rows[i]) * d, s))
            return rc;
        if (int rc = out.ensure(ctx, sizeof(float) * static_cast<size_t>(frames_out) * d,
                                sizeof(float) * static_cast<size_t>(out_rows[i]) * d, s))
            return rc;
        const float* src = i == 0 ? input.as<float>() : outs[i - 1].as<float>();
        float* x = st.as<float>() + static_cast<int64_t>(start) * d;
        if (int rc = ctx->cuda(cudaMemcpyAsync(x, src + static_cast<int64_t>(start) * d,
                                               sizeof(float) * static_cast<size_t>(frames_in - start) * d,
                                               cudaMemcpyDeviceToDevice, s),
                               "stream"))
            return rc;
        float* o = out.as<float>() + static_cast<int64_t>(out_start) * d;
        if (int rc = g->span(b, x, frames_in - start, st.as<float>() + static_cast<int64_t>(lo) * d, frames_in - lo, lo,
                             out_start, frames_out - out_start, o, s))
            return rc;
        if (i == sc_layer)
            if (int rc = g->self_condition(o, frames_out - out_start, s)) return rc;
        state_rows[i] = frames_in;
        out_rows[i] = frames_out;
        changed = out_start;
        frames_in = frames_out;
    }
    // Frame scores of the changed frames (src/granite_stream.rs:335-345).
    const int first = changed;
    if (int rc = ids_dev.ensure(ctx, sizeof(uint32_t) * frames_in, 0, s)) return rc;
    if (int rc = g->frame_ids(outs.back().as<float>() + static_cast<int64_t>(first) * d, frames_in - first,
                              ids_dev.as<uint32_t>(), nullptr, s))
        return rc;
    ids.resize(frames_in);
    if (int rc = ctx->cuda(cudaMemcpyAsync(ids.data() + first, ids_dev.as<uint32_t>(),
                                           sizeof(uint32_t) * (frames_in - first), cudaMemcpyDeviceToHost, s),
                           "stream ids"))
        return rc;
    if (int rc = ctx->cuda(cudaStreamSynchronize(s), "stream ids")) return rc;
    first_changed = first;
    if (frames_in > lag) frozen = std::max(frozen, (frames_in - 1 - lag) / ctxn * ctxn);
    return TELMO_OK;
}

}  // namespace telmo

using namespace telmo;

struct telmo_granite_stream {
    GraniteStream s;
};

extern "C" int telmo_granite_stream_create(telmo_granite* gp, telmo_granite_stream** out) {
    Granite* g = reinterpret_cast<Granite*>(gp);
    if (!g || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    Ctx* ctx = g->ctx;
    if (int rc = ctx->use_device()) return rc;
    if (!g->finalized) return ctx->fail(TELMO_ERR_MODEL, "granite: the model is not finalized");
    // The reference asserts its strided blocks come first (src/granite_stream.rs:76-84).
    for (int i = 0; i < g->c.n_subsample; ++i)
        if (!g->blocks[i].strided)
            return ctx->fail(TELMO_ERR_MODEL, "granite_stream: streaming needs the strided blocks first");
    if (!ctx->granite_fe) {
        auto* fe = new FrontEnd();
        fe->n_mels = 80;  // Granite Speech's front end (as telmo_logmel builds it)
        if (int rc = fe->init(ctx, FrontEnd::kGranite)) {
            delete fe;
            return rc;
        }
        ctx->granite_fe = fe;
    }
    if (ctx->granite_fe->n_mels != g->c.n_mels)
        return ctx->fail(TELMO_ERR_UNSUPPORTED, "granite_stream: the GPU front end computes %d mels, the model reads %d",
                         ctx->granite_fe->n_mels, g->c.n_mels);
    auto* h = new telmo_granite_stream();
    GraniteStream& st = h->s;
    st.g = g;
    st.ctx = ctx;
    st.fe = ctx->granite_fe;
    st.states.resize(g->c.layers);
    st.outs.resize(g->c.layers);
    st.state_rows.assign(g->c.layers, 0);
    st.out_rows.assign(g->c.layers, 0);
    if (int rc = st.meta.ensure(ctx, 256, 0, nullptr)) {
        delete h;
        return rc;
    }
    if (int rc = st.peak.ensure(ctx, 2 * sizeof(float), 0, nullptr)) {
        delete h;
        return rc;
    }
    *out = h;
    return TELMO_OK;
}

extern "C" void telmo_granite_stream_free(telmo_granite_stream* h) {
    if (!h) return;
    cudaSetDevice(h->s.ctx->device);
    delete h;
}

extern "C" int telmo_granite_stream_set_freeze_lag(telmo_granite_stream* h, int frames) {
    if (!h || frames < 0) return TELMO_ERR_ARGUMENT;
    h->s.lag = frames;
    return TELMO_OK;
}

extern "C" int telmo_granite_stream_push(telmo_granite_stream* h, const float* samples, size_t n) {
    if (!h || (!samples && n)) return TELMO_ERR_ARGUMENT;
    GraniteStream& st = h->s;
    if (st.finished) return st.ctx->fail(TELMO_ERR_ARGUMENT, "granite_stream_push: audio pushed after the stream finished");
    if (n == 0) return TELMO_OK;
    if (int rc = st.ctx->use_device()) return rc;
    const size_t have = static_cast<size_t>(st.n);
    if (int rc = st.samples.ensure(st.ctx, sizeof(float) * (have + n), sizeof(float) * have, nullptr)) return rc;
    if (int rc = st.ctx->cuda(cudaMemcpy(st.samples.as<float>() + have, samples, sizeof(float) * n, cudaMemcpyHostToDevice),
                              "stream push"))
        return rc;
    st.n += static_cast<int64_t>(n);
    return TELMO_OK;
}

extern "C" int telmo_granite_stream_update(telmo_granite_stream* h, int finished, void* stream) {
    if (!h) return TELMO_ERR_ARGUMENT;
    if (int rc = h->s.ctx->use_device()) return rc;
    return h->s.update(finished != 0, static_cast<cudaStream_t>(stream));
}

extern "C" size_t telmo_granite_stream_frames(const telmo_granite_stream* h) { return h ? h->s.ids.size() : 0; }

extern "C" size_t telmo_granite_stream_first_changed(const telmo_granite_stream* h) {
    return h ? static_cast<size_t>(h->s.first_changed) : 0;
}

extern "C" size_t telmo_granite_stream_frozen(const telmo_granite_stream* h) {
    return h ? static_cast<size_t>(h->s.frozen) : 0;
}

extern "C" int telmo_granite_stream_frame_ids(const telmo_granite_stream* h, uint32_t* ids, size_t cap) {
    if (!h || (!ids && cap)) return TELMO_ERR_ARGUMENT;
    const size_t n = std::min(cap, h->s.ids.size());
    std::copy(h->s.ids.begin(), h->s.ids.begin() + n, ids);
    return TELMO_OK;
}

extern "C" int telmo_granite_stream_layer_output(const telmo_granite_stream* h, int layer, float* out, size_t cap_rows,
                                                 size_t* rows) {
    if (!h || layer < 0 || layer >= h->s.g->c.layers) return TELMO_ERR_ARGUMENT;
    const GraniteStream& st = h->s;
    const size_t r = static_cast<size_t>(st.out_rows[layer]);
    if (rows) *rows = r;
    if (!out || cap_rows == 0 || r == 0) return TELMO_OK;
    if (int rc = st.ctx->use_device()) return rc;
    return st.ctx->cuda(cudaMemcpy(out, st.outs[layer].p, sizeof(float) * std::min(r, cap_rows) * st.g->c.d_model,
                                   cudaMemcpyDeviceToHost),
                        "stream output");
}

extern "C" int telmo_granite_stream_features(const telmo_granite_stream* h, float* out, size_t cap_rows, size_t* rows) {
    if (!h) return TELMO_ERR_ARGUMENT;
    const GraniteStream& st = h->s;
    if (rows) *rows = static_cast<size_t>(st.rows);
    if (!out || cap_rows == 0 || st.rows == 0) return TELMO_OK;
    if (int rc = st.ctx->use_device()) return rc;
    return st.ctx->cuda(cudaMemcpy(out, st.features.p,
                                   sizeof(float) * std::min(static_cast<size_t>(st.rows), cap_rows) * 4 * st.g->c.n_mels,
                                   cudaMemcpyDeviceToHost),
                        "stream features");
}
