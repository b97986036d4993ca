// noalloc.cu -- telmo_linear_noalloc: the matrix product without any device allocation.
//
// telmo_linear quantizes its f32 activations into a workspace the context grows with cudaMalloc.
// Some callers cannot let a library allocate: a service that hands all device memory to its own
// pool or fixed budget up front, or a latency-critical stream that cannot afford the implicit
// device synchronisation cudaMalloc and cudaFree bring. This entry point keeps that scratch in a
// fixed-size array in the library's device image instead, so the call itself allocates nothing.
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "kernels.h"

#include <mutex>

namespace telmo {

namespace {

// The scratch: both int8 levels of the quantized activations and one f32 scale per row. Every
// GPU that loads the library holds this much device memory until the process exits.
constexpr size_t kScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_linear_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The device address of the scratch on the current device. In host code g_linear_scratch names
// a host-side stand-in, not device memory, so the address comes from cudaGetSymbolAddress, once
// per device, with that device current. The cached address belongs to the device's context as
// it was at that first call: a host program that calls cudaDeviceReset and goes on using the
// device gets a new context, in which the library's module and its scratch are loaded anew, so
// it must not call telmo_linear_noalloc again in that process.
int scratch_address(Ctx* ctx, void** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (ctx->device < 0 || ctx->device >= kMaxDevices)
        return ctx->fail(TELMO_ERR_UNSUPPORTED, "telmo_linear_noalloc: device %d is out of range", ctx->device);
    if (!g_scratch_ptr[ctx->device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
        if (e != cudaSuccess || !p)
            return ctx->fail(TELMO_ERR_CUDA, "telmo_linear_noalloc: cudaGetSymbolAddress failed: %s",
                             cudaGetErrorString(e));
        g_scratch_ptr[ctx->device] = p;
    }
    *out = g_scratch_ptr[ctx->device];
    return TELMO_OK;
}

}  // namespace

}  // namespace telmo

using namespace telmo;

extern "C" int telmo_linear_noalloc(telmo_ctx* c, const float* a, size_t lda, size_t m, const telmo_weights* wp,
                                    const float* bias, int act, float scale, int accumulate, void* out, int c_dtype,
                                    size_t ldc, void* stream) {
    Ctx* ctx = as_ctx(c);
    auto* w = reinterpret_cast<const Weights*>(wp);
    if (!ctx || !w) return TELMO_ERR_ARGUMENT;
    if (w->ctx != ctx) return ctx->fail(TELMO_ERR_ARGUMENT, "the weights belong to another context");
    if (m == 0) return TELMO_OK;
    const size_t k = static_cast<size_t>(w->dev.k), n = static_cast<size_t>(w->dev.n);
    if (!a || lda < k) return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_linear_noalloc: a is NULL or lda %zu < k %zu", lda, k);
    if (!out) return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_linear_noalloc: c is NULL");
    if (c_dtype != TELMO_DTYPE_F32 && c_dtype != TELMO_DTYPE_BF16 && c_dtype != TELMO_DTYPE_I32_PAIR)
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_linear_noalloc: unknown output dtype %d", c_dtype);
    if (ldc < n) return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_linear_noalloc: ldc %zu is below n %zu", ldc, n);
    if (act < TELMO_ACT_NONE || act > TELMO_ACT_SILU)
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_linear_noalloc: unknown act %d", act);
    // Layout in the scratch: hi [m, ldq], lo [m, ldq], scales [m], each 256-byte aligned.
    const size_t ldq = round_up(k, 16);
    if (m > (size_t(1) << 30) || m > kScratchBytes / ldq)
        return ctx->fail(TELMO_ERR_ARGUMENT,
                         "telmo_linear_noalloc: %zu rows of k=%zu do not fit the fixed %zu-byte scratch", m, k,
                         kScratchBytes);
    const size_t plane = round_up(m * ldq, 256);
    const size_t need = 2 * plane + round_up(m * sizeof(float), 256);
    if (need > kScratchBytes)
        return ctx->fail(TELMO_ERR_ARGUMENT,
                         "telmo_linear_noalloc: %zu rows of k=%zu need %zu bytes of scratch, above the fixed %zu "
                         "(use telmo_linear for larger products)",
                         m, k, need, kScratchBytes);
    if (int rc = ctx->use_device()) return rc;
    void* scratch = nullptr;
    if (int rc = scratch_address(ctx, &scratch)) return rc;
    uint8_t* base = static_cast<uint8_t*>(scratch);
    QuantAct q;
    q.hi = reinterpret_cast<int8_t*>(base);
    q.lo = reinterpret_cast<int8_t*>(base + plane);
    q.scale = reinterpret_cast<float*>(base + 2 * plane);
    q.ld = static_cast<int64_t>(ldq);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The quantization writes every byte the product reads (both levels including the zero
    // columns up to ldq, and the scales), so nothing left by an earlier call needs clearing.
    if (int rc = ctx->cuda(quantize_x2(a, static_cast<int64_t>(lda), static_cast<int>(m), static_cast<int>(k), q, s),
                           "telmo_linear_noalloc"))
        return rc;
    GemmArgs g;
    g.m = static_cast<int>(m);
    g.a = q;
    g.w = &w->dev;
    g.bias = bias;
    g.act = act;
    g.scale = scale;
    g.accumulate = accumulate;
    g.out = out;
    g.ldc = static_cast<int64_t>(ldc);
    g.out_kind = c_dtype == TELMO_DTYPE_F32 ? kOutF32 : c_dtype == TELMO_DTYPE_BF16 ? kOutBF16 : kOutI32Pair;
    g.error = ctx->error_word;
    return ctx->cuda(gemm_i8x2(g, s), "telmo_linear_noalloc");
}
