// api.cu -- the C ABI of libtelmo_b200: contexts, weights and the matrix product.
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "frontend.h"
#include "kernels.h"
#include "rowops.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

using namespace telmo;

namespace {
thread_local std::string g_create_error;
}  // namespace

namespace telmo {

int Ctx::fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    last_error = buf;
    return code;
}

int Ctx::cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return TELMO_OK;
    return fail(TELMO_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int Ctx::use_device() {
    cudaError_t e = cudaSetDevice(device);
    return cuda(e, "cudaSetDevice");
}

void* Ctx::workspace(size_t bytes, cudaStream_t stream) {
    if (bytes <= ws_bytes) return ws;
    // Growing: wait for work that may still read the old buffer, then replace it.
    cudaStreamSynchronize(stream);
    if (ws) cudaFree(ws);
    ws = nullptr;
    ws_bytes = 0;
    size_t want = bytes + bytes / 4 + (1 << 20);
    if (cudaMalloc(&ws, want) != cudaSuccess) return nullptr;
    ws_bytes = want;
    return ws;
}

cudaError_t PinnedRing::upload(void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return cudaSuccess;
    Slot& sl = slot[next];
    next = (next + 1) % kSlots;
    cudaError_t e = cudaSuccess;
    if (sl.done) {
        e = cudaEventSynchronize(sl.done);  // the slot's previous copy has read it
    } else {
        e = cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return e;
    if (bytes > sl.cap) {
        if (sl.buf) cudaFreeHost(sl.buf);
        sl.buf = nullptr;
        sl.cap = 0;
        const size_t want = std::max<size_t>(bytes + bytes / 4, 64 << 10);
        if ((e = cudaHostAlloc(&sl.buf, want, cudaHostAllocDefault)) != cudaSuccess) return e;
        sl.cap = want;
    }
    std::memcpy(sl.buf, src, bytes);
    if ((e = cudaMemcpyAsync(dst, sl.buf, bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess) return e;
    return cudaEventRecord(sl.done, s);
}

PinnedRing::~PinnedRing() {
    for (Slot& sl : slot) {
        if (sl.done) {
            cudaEventSynchronize(sl.done);
            cudaEventDestroy(sl.done);
        }
        if (sl.buf) cudaFreeHost(sl.buf);
    }
}

}  // namespace telmo

static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

extern "C" int telmo_ctx_create(int device, telmo_ctx** out) {
    if (!out) {
        g_create_error = "telmo_ctx_create: out is NULL";
        return TELMO_ERR_ARGUMENT;
    }
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || device < 0 || device >= count) {
        g_create_error = "telmo_ctx_create: no CUDA device " + std::to_string(device) +
                         (e != cudaSuccess ? std::string(" (") + cudaGetErrorString(e) + ")" : "");
        return e != cudaSuccess ? TELMO_ERR_CUDA : TELMO_ERR_ARGUMENT;
    }
    cudaDeviceProp prop;
    if ((e = cudaSetDevice(device)) != cudaSuccess || (e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
        g_create_error = std::string("telmo_ctx_create: ") + cudaGetErrorString(e);
        return TELMO_ERR_CUDA;
    }
    if (prop.major != 10 || prop.minor != 0) {
        g_create_error = "telmo_ctx_create: device " + std::to_string(device) + " is sm_" +
                         std::to_string(prop.major) + std::to_string(prop.minor) +
                         "; this build runs on sm_100a (B200) only";
        return TELMO_ERR_UNSUPPORTED;
    }
    Ctx* ctx = new Ctx();
    ctx->device = device;
    ctx->sms = prop.multiProcessorCount;
    if ((e = cudaMalloc(&ctx->error_word, sizeof(uint32_t))) != cudaSuccess ||
        (e = cudaMemset(ctx->error_word, 0, sizeof(uint32_t))) != cudaSuccess) {
        g_create_error = std::string("telmo_ctx_create: ") + cudaGetErrorString(e);
        delete ctx;
        return TELMO_ERR_CUDA;
    }
    *out = reinterpret_cast<telmo_ctx*>(ctx);
    return TELMO_OK;
}

extern "C" void telmo_ctx_destroy(telmo_ctx* c) {
    Ctx* ctx = as_ctx(c);
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    delete ctx->granite_fe;
    delete ctx->parakeet_fe;
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->error_word) cudaFree(ctx->error_word);
    delete ctx;
}

extern "C" const char* telmo_last_error(const telmo_ctx* c) {
    const Ctx* ctx = reinterpret_cast<const Ctx*>(c);
    return ctx ? ctx->last_error.c_str() : g_create_error.c_str();
}

extern "C" int telmo_ctx_device(const telmo_ctx* c) {
    const Ctx* ctx = reinterpret_cast<const Ctx*>(c);
    return ctx ? ctx->device : -1;
}

extern "C" int telmo_ctx_check(telmo_ctx* c, void* stream) {
    Ctx* ctx = as_ctx(c);
    if (!ctx) return TELMO_ERR_ARGUMENT;
    if (int rc = ctx->use_device()) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = ctx->cuda(cudaStreamSynchronize(s), "telmo_ctx_check")) return rc;
    uint32_t word = 0;
    if (int rc = ctx->cuda(cudaMemcpy(&word, ctx->error_word, sizeof word, cudaMemcpyDeviceToHost),
                           "telmo_ctx_check"))
        return rc;
    if (word != 0) {
        cudaMemset(ctx->error_word, 0, sizeof(uint32_t));
        return ctx->fail(TELMO_ERR_DEVICE_TIMEOUT,
                         "a kernel gave up on a bounded wait (device error %u); its results are invalid",
                         word);
    }
    return TELMO_OK;
}

extern "C" int telmo_encode_int8(const float* rows, size_t n, size_t k, int8_t* values, float* scales) {
    if (!rows || !values || !scales) return TELMO_ERR_ARGUMENT;
    encode_int8_panels(rows, n, k, values, scales);
    return TELMO_OK;
}

extern "C" int telmo_encode_q8_0(const float* rows, size_t n, size_t k, int8_t* values, float* scales) {
    if (!rows || !values || !scales || k % 32) return TELMO_ERR_ARGUMENT;
    encode_q8_0_panels(rows, n, k, values, scales);
    return TELMO_OK;
}

namespace telmo {

void encode_int8_panels(const float* rows, size_t n, size_t k, int8_t* values, float* scales) {
    // quant::encode, Precision::Int8 (src/quant.rs:202-269): quantize_row_int8 per output row,
    // then panel p = o / 16 holds k runs of 16 outputs.
    const size_t panels = (n + 15) / 16;
    memset(values, 0, panels * 16 * k);
    memset(scales, 0, panels * 16 * sizeof(float));
    for (size_t o = 0; o < n; ++o) {
        const float* x = rows + o * k;
        float amax = 0.0f;
        for (size_t i = 0; i < k; ++i) amax = std::fmax(amax, std::fabs(x[i]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const size_t p = o / 16, j = o % 16;
        for (size_t i = 0; i < k; ++i) {
            float q = std::round(x[i] * id);
            q = std::fmin(std::fmax(q, -127.0f), 127.0f);
            values[(p * k + i) * 16 + j] = static_cast<int8_t>(q);
        }
        scales[p * 16 + j] = d;
    }
}

void encode_q8_0_panels(const float* rows, size_t n, size_t k, int8_t* values, float* scales) {
    // quant::encode, Precision::Q8_0 (src/quant.rs:202-269) with quantize_q8_0_block
    // (:172-183): per block of 32 inputs d = amax / 127, q = round(x / d) with the unrounded
    // reciprocal, the scale kept as its f16 value; scales run panel, then block, then output.
    const size_t panels = (n + 15) / 16, blocks = k / 32;
    memset(values, 0, panels * 16 * k);
    memset(scales, 0, panels * blocks * 16 * sizeof(float));
    for (size_t o = 0; o < n; ++o) {
        const float* x = rows + o * k;
        const size_t p = o / 16, j = o % 16;
        for (size_t b = 0; b < blocks; ++b) {
            float amax = 0.0f;
            for (size_t i = 32 * b; i < 32 * b + 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            for (size_t i = 32 * b; i < 32 * b + 32; ++i) {
                const float q = std::fmin(std::fmax(std::round(x[i] * id), -128.0f), 127.0f);
                values[(p * k + i) * 16 + j] = static_cast<int8_t>(q);
            }
            scales[(p * blocks + b) * 16 + j] = __half2float(__float2half_rn(d));
        }
    }
}

namespace {

// Round to the nearest integer, halves to even, for |x| < 2^22: adding 1.5 * 2^23 leaves no
// fraction bits, so the sum is rounded by the addition itself (IEEE round-to-nearest-even).
inline float round_even(float x) { return (x + 12582912.0f) - 12582912.0f; }
inline float clamp127(float x) { return x < -127.0f ? -127.0f : (x > 127.0f ? 127.0f : x); }

void encode_device_row_range(bool q8, size_t o0, size_t o1, size_t k, const int8_t* v, const float* scales,
                             const int* col_perm, int8_t* rows, int8_t* lo, float* sc) {
    const size_t ld = round_up(k, 16), blocks = k / 32;
    std::vector<float> w(q8 ? k : 0);
    for (size_t o = o0; o < o1; ++o) {
        const size_t p = o / 16, j = o % 16;
        const int8_t* src = v + p * k * 16 + j;
        int8_t* dst = rows + o * ld;
        std::fill(dst, dst + ld, int8_t(0));
        if (!q8) {
            for (size_t i = 0; i < k; ++i) dst[i] = src[(col_perm ? col_perm[i] : i) * 16];
            sc[o] = scales[p * 16 + j];
            continue;
        }
        // Q8_0 (src/quant.rs:8-13): w = q * d[block], exact in f32 (d is an f16 value). The row
        // is re-encoded as s * (hi + lo / 254) with one scale per row, by the rule the
        // activations use (quant.cu): s = amax / 127, hi = w / s and lo = (w - hi s) * 254 / s,
        // each rounded to the nearest integer (halves to even) and clamped to [-127, 127]; the
        // representation is within s / 508 (1/64516 of the row's largest weight) of w. The GEMM
        // adds hi_a . lo_w to the low-level sum.
        float amax = 0.0f;
        for (size_t i = 0; i < k; ++i) {
            const size_t c = col_perm ? static_cast<size_t>(col_perm[i]) : i;
            w[i] = static_cast<float>(src[c * 16]) * scales[(p * blocks + c / 32) * 16 + j];
            const float a = std::fabs(w[i]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const float id_lo = id * 254.0f;
        int8_t* dlo = lo + o * ld;
        std::fill(dlo, dlo + ld, int8_t(0));
        for (size_t i = 0; i < k; ++i) {
            const float h = clamp127(round_even(w[i] * id));
            // w - h s with one rounding: h s (7 by 24 significant bits) and the difference, which
            // is near 0 against w, are exact in f64.
            const float e = static_cast<float>(static_cast<double>(w[i]) - static_cast<double>(h) * d);
            const float l = clamp127(round_even(e * id_lo));
            dst[i] = static_cast<int8_t>(h);
            dlo[i] = static_cast<int8_t>(l);
        }
        sc[o] = d;
    }
}

}  // namespace

void encode_device_rows(int precision, size_t n, size_t k, const void* panel_values, const float* scales,
                        const int* col_perm, int8_t* rows, int8_t* lo, float* sc) {
    // Rows are independent: up to 16 host threads take contiguous ranges of them.
    const bool q8 = precision == TELMO_PRECISION_Q8_0;
    const int8_t* v = static_cast<const int8_t*>(panel_values);
    const size_t work = n * k * (q8 ? 8 : 1);
    const size_t hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t threads = std::min<size_t>({hw, 16, std::max<size_t>(1, work >> 21), n});
    if (threads <= 1) {
        encode_device_row_range(q8, 0, n, k, v, scales, col_perm, rows, lo, sc);
        return;
    }
    std::vector<std::thread> pool;
    const size_t per = (n + threads - 1) / threads;
    for (size_t t = 0; t < threads; ++t) {
        const size_t o0 = t * per, o1 = std::min(n, o0 + per);
        if (o0 >= o1) break;
        pool.emplace_back(encode_device_row_range, q8, o0, o1, k, v, scales, col_perm, rows, lo, sc);
    }
    for (auto& th : pool) th.join();
}

int upload_device_rows(Ctx* ctx, int precision, size_t n, size_t k, const int8_t* rows, const int8_t* lo,
                       const float* sc, DevWeights* out) {
    const bool q8 = precision == TELMO_PRECISION_Q8_0;
    const size_t ld = round_up(k, 16);
    out->n = static_cast<int>(n);
    out->k = static_cast<int>(k);
    out->ld = static_cast<int64_t>(ld);
    if (int rc = ctx->cuda(cudaMalloc(&out->values, n * ld), "weights")) return rc;
    if (int rc = ctx->cuda(cudaMalloc(&out->scales, n * sizeof(float)), "weights")) return rc;
    if (int rc = ctx->cuda(cudaMemcpy(out->values, rows, n * ld, cudaMemcpyHostToDevice), "weights")) return rc;
    if (q8) {
        if (int rc = ctx->cuda(cudaMalloc(&out->lo_values, n * ld), "weights")) return rc;
        if (int rc = ctx->cuda(cudaMemcpy(out->lo_values, lo, n * ld, cudaMemcpyHostToDevice), "weights")) return rc;
    }
    return ctx->cuda(cudaMemcpy(out->scales, sc, n * sizeof(float), cudaMemcpyHostToDevice), "weights");
}

int check_weight_shape(Ctx* ctx, int precision, size_t n, size_t k) {
    if (precision != TELMO_PRECISION_INT8 && precision != TELMO_PRECISION_Q8_0)
        return ctx->fail(TELMO_ERR_UNSUPPORTED,
                         "precision %d: this build runs int8 weights (TELMO_PRECISION_INT8, "
                         "TELMO_PRECISION_Q8_0) only",
                         precision);
    if (n == 0 || k == 0 || n > (1u << 30) || k > (1u << 30))
        return ctx->fail(TELMO_ERR_ARGUMENT, "weights: bad sizes n=%zu k=%zu", n, k);
    if (precision == TELMO_PRECISION_Q8_0 && k % 32)
        return ctx->fail(TELMO_ERR_ARGUMENT, "weights: Q8_0 needs inputs in multiples of 32 (k=%zu)", k);
    return TELMO_OK;
}

int upload_weights(Ctx* ctx, int precision, size_t n, size_t k, const void* panel_values,
                   const float* scales, DevWeights* out, const int* col_perm) {
    if (int rc = check_weight_shape(ctx, precision, n, k)) return rc;
    if (!panel_values || !scales) return ctx->fail(TELMO_ERR_ARGUMENT, "weights: null data");
    const bool q8 = precision == TELMO_PRECISION_Q8_0;
    const size_t ld = round_up(k, 16);
    std::vector<int8_t> rows(n * ld), lo(q8 ? n * ld : 0);
    std::vector<float> sc(n);
    encode_device_rows(precision, n, k, panel_values, scales, col_perm, rows.data(), lo.data(), sc.data());
    return upload_device_rows(ctx, precision, n, k, rows.data(), q8 ? lo.data() : nullptr, sc.data(), out);
}

void free_weights(DevWeights* w) {
    if (w->values) cudaFree(w->values);
    if (w->lo_values) cudaFree(w->lo_values);
    if (w->scales) cudaFree(w->scales);
    w->values = nullptr;
    w->lo_values = nullptr;
    w->scales = nullptr;
}

}  // namespace telmo

extern "C" int telmo_weights_upload(telmo_ctx* c, int precision, size_t n, size_t k,
                                    const void* panel_values, const float* scales, telmo_weights** out) {
    Ctx* ctx = as_ctx(c);
    if (!ctx || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    if (int rc = ctx->use_device()) return rc;
    auto* w = new Weights();
    w->ctx = ctx;
    if (int rc = upload_weights(ctx, precision, n, k, panel_values, scales, &w->dev)) {
        free_weights(&w->dev);
        delete w;
        return rc;
    }
    *out = reinterpret_cast<telmo_weights*>(w);
    return TELMO_OK;
}

extern "C" void telmo_weights_free(telmo_weights* wp) {
    auto* w = reinterpret_cast<Weights*>(wp);
    if (!w) return;
    cudaSetDevice(w->ctx->device);
    free_weights(&w->dev);
    delete w;
}

extern "C" int telmo_weights_shape(const telmo_weights* wp, size_t* n, size_t* k) {
    auto* w = reinterpret_cast<const Weights*>(wp);
    if (!w) return TELMO_ERR_ARGUMENT;
    if (n) *n = static_cast<size_t>(w->dev.n);
    if (k) *k = static_cast<size_t>(w->dev.k);
    return TELMO_OK;
}

static int check_out(Ctx* ctx, int c_dtype, size_t ldc, size_t n, const void* c) {
    if (!c) return ctx->fail(TELMO_ERR_ARGUMENT, "c is NULL");
    if (c_dtype != TELMO_DTYPE_F32 && c_dtype != TELMO_DTYPE_BF16 && c_dtype != TELMO_DTYPE_I32_PAIR)
        return ctx->fail(TELMO_ERR_ARGUMENT, "unknown output dtype %d", c_dtype);
    if (ldc < n) return ctx->fail(TELMO_ERR_ARGUMENT, "ldc %zu is below n %zu", ldc, n);
    return TELMO_OK;
}

extern "C" int telmo_quantize_x2(telmo_ctx* c, const float* a, size_t lda, size_t m, size_t k,
                                 int8_t* hi, int8_t* lo, size_t ldq, float* scale, void* stream) {
    Ctx* ctx = as_ctx(c);
    if (!ctx) return TELMO_ERR_ARGUMENT;
    if (m == 0) return TELMO_OK;
    if (!a || !hi || !lo || !scale || k == 0 || lda < k || ldq < k || ldq % 16 || m > (1u << 30))
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_quantize_x2: bad arguments (m=%zu k=%zu lda=%zu ldq=%zu)",
                         m, k, lda, ldq);
    // The kernels store the levels four bytes at a time and the product reads them through
    // tensor maps, which need 16-byte aligned rows.
    const auto misaligned = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) != 0; };
    if (misaligned(hi, 16) || misaligned(lo, 16) || misaligned(scale, 4) || misaligned(a, 4))
        return ctx->fail(TELMO_ERR_ARGUMENT,
                         "telmo_quantize_x2: hi and lo must be 16-byte aligned, a and scale 4-byte aligned");
    if (int rc = ctx->use_device()) return rc;
    QuantAct q;
    q.hi = hi;
    q.lo = lo;
    q.scale = scale;
    q.ld = static_cast<int64_t>(ldq);
    return ctx->cuda(quantize_x2(a, static_cast<int64_t>(lda), static_cast<int>(m), static_cast<int>(k), q,
                                 static_cast<cudaStream_t>(stream)),
                     "telmo_quantize_x2");
}

extern "C" int telmo_conv_module_rows(telmo_ctx* c, const float* in, size_t frames, size_t channels, size_t kernel,
                                      size_t stride, const float* w, const float* bias, float* out, void* stream) {
    Ctx* ctx = as_ctx(c);
    if (!ctx) return TELMO_ERR_ARGUMENT;
    if (!in || !w || !bias || !out || frames == 0 || frames > (1u << 30) || channels == 0 ||
        channels > (1u << 20) || kernel == 0 || kernel % 2 == 0 || kernel > 63 || (stride != 1 && stride != 2))
        return ctx->fail(TELMO_ERR_ARGUMENT,
                         "telmo_conv_module_rows: bad arguments (frames=%zu channels=%zu kernel=%zu stride=%zu)",
                         frames, channels, kernel, stride);
    if (int rc = ctx->use_device()) return rc;
    const int len = static_cast<int>(frames), st = static_cast<int>(stride);
    const int n_out = st == 2 ? len / 2 : len;
    if (n_out == 0) return TELMO_OK;
    std::vector<ConvTask> tasks;
    for (int r = 0; r < n_out; r += 32) tasks.push_back({0, len, 0, r, std::min(32, n_out - r), st, 0});
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t bytes = sizeof(ConvTask) * tasks.size();
    void* dev = ctx->workspace(bytes, s);
    if (!dev) return ctx->fail(TELMO_ERR_CUDA, "telmo_conv_module_rows: workspace of %zu bytes", bytes);
    // A pageable source is staged before cudaMemcpyAsync returns, so `tasks` may be freed after.
    if (int rc = ctx->cuda(cudaMemcpyAsync(dev, tasks.data(), bytes, cudaMemcpyHostToDevice, s), "conv tasks"))
        return rc;
    return ctx->cuda(glu_dwconv_silu(in, static_cast<int>(channels), static_cast<int>(kernel), st,
                                     static_cast<const ConvTask*>(dev), static_cast<int>(tasks.size()), w, bias, out, s),
                     "telmo_conv_module_rows");
}

static int run_gemm(Ctx* ctx, const QuantAct& q, size_t m, const Weights* w, const float* bias, int act,
                    float scale, int accumulate, void* c, int c_dtype, size_t ldc, cudaStream_t stream) {
    GemmArgs g;
    g.m = static_cast<int>(m);
    g.a = q;
    g.w = &w->dev;
    g.bias = bias;
    g.act = act;
    g.scale = scale;
    g.accumulate = accumulate;
    g.out = c;
    g.ldc = static_cast<int64_t>(ldc);
    g.out_kind = c_dtype == TELMO_DTYPE_F32 ? kOutF32 : c_dtype == TELMO_DTYPE_BF16 ? kOutBF16 : kOutI32Pair;
    g.error = ctx->error_word;
    return ctx->cuda(gemm_i8x2(g, stream), "telmo_linear");
}

extern "C" int telmo_linear_q(telmo_ctx* c, const int8_t* hi, const int8_t* lo, size_t ldq,
                              const float* row_scale, size_t m, const telmo_weights* wp, const float* bias,
                              int act, float scale, int accumulate, void* out, int c_dtype, size_t ldc,
                              void* stream) {
    Ctx* ctx = as_ctx(c);
    auto* w = reinterpret_cast<const Weights*>(wp);
    if (!ctx || !w) return TELMO_ERR_ARGUMENT;
    if (w->ctx != ctx) return ctx->fail(TELMO_ERR_ARGUMENT, "the weights belong to another context");
    if (m == 0) return TELMO_OK;
    if (int rc = check_out(ctx, c_dtype, ldc, static_cast<size_t>(w->dev.n), out)) return rc;
    if (!hi || !lo || !row_scale || ldq < static_cast<size_t>(w->dev.k) || ldq % 16 || m > (1u << 30))
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_linear_q: bad activations (ldq=%zu, k=%d)", ldq, w->dev.k);
    if (act < TELMO_ACT_NONE || act > TELMO_ACT_SILU) return ctx->fail(TELMO_ERR_ARGUMENT, "unknown act %d", act);
    if (int rc = ctx->use_device()) return rc;
    QuantAct q;
    q.hi = const_cast<int8_t*>(hi);
    q.lo = const_cast<int8_t*>(lo);
    q.scale = const_cast<float*>(row_scale);
    q.ld = static_cast<int64_t>(ldq);
    return run_gemm(ctx, q, m, w, bias, act, scale, accumulate, out, c_dtype, ldc,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int telmo_linear(telmo_ctx* c, const float* a, size_t lda, size_t m, const telmo_weights* wp,
                            const float* bias, int act, float scale, int accumulate, void* out, int c_dtype,
                            size_t ldc, void* stream) {
    Ctx* ctx = as_ctx(c);
    auto* w = reinterpret_cast<const Weights*>(wp);
    if (!ctx || !w) return TELMO_ERR_ARGUMENT;
    if (w->ctx != ctx) return ctx->fail(TELMO_ERR_ARGUMENT, "the weights belong to another context");
    if (m == 0) return TELMO_OK;
    const size_t k = static_cast<size_t>(w->dev.k), n = static_cast<size_t>(w->dev.n);
    if (!a || lda < k || m > (1u << 30))
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_linear: a is NULL or lda %zu < k %zu", lda, k);
    if (int rc = check_out(ctx, c_dtype, ldc, n, out)) return rc;
    if (act < TELMO_ACT_NONE || act > TELMO_ACT_SILU) return ctx->fail(TELMO_ERR_ARGUMENT, "unknown act %d", act);
    if (int rc = ctx->use_device()) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t ldq = round_up(k, 16);
    const size_t plane = round_up(m * ldq, 256);
    auto* base = static_cast<uint8_t*>(ctx->workspace(2 * plane + round_up(m * sizeof(float), 256), s));
    if (!base) return ctx->fail(TELMO_ERR_CUDA, "telmo_linear: workspace allocation failed");
    QuantAct q;
    q.hi = reinterpret_cast<int8_t*>(base);
    q.lo = reinterpret_cast<int8_t*>(base + plane);
    q.scale = reinterpret_cast<float*>(base + 2 * plane);
    q.ld = static_cast<int64_t>(ldq);
    if (int rc = ctx->cuda(quantize_x2(a, static_cast<int64_t>(lda), static_cast<int>(m), static_cast<int>(k), q, s),
                           "telmo_linear"))
        return rc;
    return run_gemm(ctx, q, m, w, bias, act, scale, accumulate, out, c_dtype, ldc, s);
}
