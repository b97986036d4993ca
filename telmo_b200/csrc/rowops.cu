// rowops.cu -- the memory-bound kernels of the conformer encoder: layer norm fused with the
// split-int8 quantization of the next matrix product, softmax fused with the same, GLU +
// depthwise convolution + SiLU, the stride-2 average pool, the CTC argmax and the CTC collapse.
//
// Arithmetic follows the reference's scalar kernels (src/kernels/scalar.rs): layer-norm
// statistics in f64 and the output rounded to f32 before the affine step (:126-134), softmax
// exponentials in f32 with an f64 sum (:136-147), GLU a / (1 + e^-b) (:149-153), the depthwise
// sum starting from the bias and adding taps in order (:164-187). Explicit __fmul_rn/__fadd_rn
// keep nvcc from contracting steps the reference rounds separately.
#include "kernels.h"
#include "rowops.h"

#include <cfloat>
#include <cstdint>

namespace telmo {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

struct Scales {
    float d, id, id_lo;
};

__device__ __forceinline__ Scales row_scales(float amax) {
    Scales s;
    s.d = __fdiv_rn(amax, 127.0f);
    s.id = s.d != 0.0f ? __fdiv_rn(1.0f, s.d) : 0.0f;
    s.id_lo = __fmul_rn(s.id, 254.0f);
    return s;
}

// Sums and maxima over a row held by P warps: a warp reduction, then (P = 2) an exchange through
// shared memory under a named barrier for the row's two warps. Every reduction of a row has its
// own slot, so one barrier per reduction suffices; both warps add the two halves in the same
// order and so agree on every result.
template <int P>
struct RowReduce {
    double* xch;  // [kSlots][P] of this row's group
    int part, bar, slot;
    static constexpr int kSlots = 6;
    __device__ __forceinline__ void sync() const {
        if (P > 1) asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(32 * P) : "memory");
    }
    __device__ __forceinline__ double sum(double v, int lane) {
        v = warp_sum(v);
        if (P == 1) return v;
        if (lane == 0) xch[slot * P + part] = v;
        sync();
        const double r = xch[slot * P] + xch[slot * P + 1];
        ++slot;
        return r;
    }
    // Two sums reduced together (one exchange, one barrier).
    __device__ __forceinline__ void sum2(double& a, double& b, int lane) {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            a += __shfl_xor_sync(kFull, a, o);
            b += __shfl_xor_sync(kFull, b, o);
        }
        if (P == 1) return;
        if (lane == 0) {
            xch[slot * P + part] = a;
            xch[(slot + 1) * P + part] = b;
        }
        sync();
        a = xch[slot * P] + xch[slot * P + 1];
        b = xch[(slot + 1) * P] + xch[(slot + 1) * P + 1];
        slot += 2;
    }
    __device__ __forceinline__ float max(float v, int lane) {
        v = warp_max(v);
        if (P == 1) return v;
        if (lane == 0) xch[slot * P + part] = static_cast<double>(v);
        sync();
        const float r = fmaxf(static_cast<float>(xch[slot * P]), static_cast<float>(xch[slot * P + 1]));
        ++slot;
        return r;
    }
};

// Layer norm of one row, this warp holding the float4 chunks v[c] = elements off + (c * 32 +
// lane) * 4 .. + 3 of a row of d values.
template <int C, int P>
__device__ __forceinline__ void layer_norm_regs(float4 (&v)[C], int d, int off, const float* __restrict__ gamma,
                                                const float* __restrict__ beta, float eps, int lane,
                                                RowReduce<P>& red) {
    // Both moments in one pass, reduced in f64 over f32 partial sums of each lane's values (the
    // reference sums in f64 throughout; the f32 partials of at most 16 values and the one-pass
    // variance E[x^2] - mean^2 move mean and rstd by about 1e-7 relative for the encoder's rows,
    // |mean| within a few standard deviations). The normalised value is formed in f32 from the
    // rounded mean and rstd, within a few ulp of the reference's f64 (x - mean) * rstd rounded to
    // f32. This keeps the conversion unit, which f64 per-value arithmetic saturates, almost idle.
    float s32 = 0.0f, q32 = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        s32 = __fadd_rn(s32, __fadd_rn(__fadd_rn(v[c].x, v[c].y), __fadd_rn(v[c].z, v[c].w)));
        q32 = __fmaf_rn(v[c].x, v[c].x, __fmaf_rn(v[c].y, v[c].y, __fmaf_rn(v[c].z, v[c].z, __fmaf_rn(v[c].w, v[c].w, q32))));
    }
    double s = s32, q = q32;
    red.sum2(s, q, lane);
    const double mean = s / d;
    const double var = fmax(q / d - mean * mean, 0.0);
    const float mf = static_cast<float>(mean);
    const float rf = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int i = off + (c * 32 + lane) * 4;
        const float4 g = *reinterpret_cast<const float4*>(gamma + i);
        const float4 b = *reinterpret_cast<const float4*>(beta + i);
        v[c].x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].x, mf), rf), g.x), b.x);
        v[c].y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].y, mf), rf), g.y), b.y);
        v[c].z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].z, mf), rf), g.z), b.z);
        v[c].w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].w, mf), rf), g.w), b.w);
    }
}

template <int C, int P>
__device__ __forceinline__ void quantize_regs(const float4 (&v)[C], int off, int lane, int8_t* hi, int8_t* lo,
                                              float* scale_out, bool write_scale, RowReduce<P>& red) {
    float amax = 0.0f;
#pragma unroll
    for (int c = 0; c < C; ++c)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c].x), fabsf(v[c].y)), fmaxf(fabsf(v[c].z), fabsf(v[c].w))));
    const Scales s = row_scales(red.max(amax, lane));
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int i = off + (c * 32 + lane) * 4;
        char4 h, l;
        quant_split_one(v[c].x, s.d, s.id, s.id_lo, h.x, l.x);
        quant_split_one(v[c].y, s.d, s.id, s.id_lo, h.y, l.y);
        quant_split_one(v[c].z, s.d, s.id, s.id_lo, h.z, l.z);
        quant_split_one(v[c].w, s.d, s.id, s.id_lo, h.w, l.w);
        *reinterpret_cast<char4*>(hi + i) = h;
        *reinterpret_cast<char4*>(lo + i) = l;
    }
    if (write_scale && lane == 0) *scale_out = s.d;
}

// y = LN_a(x) [written to y_out if given]; z = LN_b(y) if gamma_b given, else z = y;
// z quantized into q if q.hi given. P warps per row of d = 128 * C values (each holding C / P
// float4 per lane), 8 warps per block.
template <int C, int P>
__global__ void __launch_bounds__(256, 4) ln_chain_kernel(const float* __restrict__ x, int m, int d,
                                                       const float* __restrict__ ga, const float* __restrict__ ba,
                                                       float* __restrict__ y_out, const float* __restrict__ gb,
                                                       const float* __restrict__ bb, QuantAct q, float eps) {
    constexpr int CW = C / P;
    constexpr int kRows = 8 / P;
    __shared__ double xch[kRows][RowReduce<P>::kSlots * P];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int grp = warp / P;
    const int row = blockIdx.x * kRows + grp;
    RowReduce<P> red{xch[grp], warp % P, 1 + grp, 0};
    // A group past the last row still takes part in its own barriers: both of its warps skip
    // together, so nothing waits on them.
    if (row >= m) return;
    const int off = (warp % P) * CW * 128;
    const float* xr = x + static_cast<int64_t>(row) * d + off;
    float4 v[CW];
#pragma unroll
    for (int c = 0; c < CW; ++c) v[c] = *reinterpret_cast<const float4*>(xr + (c * 32 + lane) * 4);
    if (ga) layer_norm_regs<CW, P>(v, d, off, ga, ba, eps, lane, red);
    if (y_out) {
        float* yr = y_out + static_cast<int64_t>(row) * d + off;
#pragma unroll
        for (int c = 0; c < CW; ++c) *reinterpret_cast<float4*>(yr + (c * 32 + lane) * 4) = v[c];
    }
    if (gb) layer_norm_regs<CW, P>(v, d, off, gb, bb, eps, lane, red);
    if (q.hi)
        quantize_regs<CW, P>(v, off, lane, q.hi + static_cast<int64_t>(row) * q.ld,
                             q.lo + static_cast<int64_t>(row) * q.ld, q.scale + row, warp % P == 0, red);
}

// Softmax of each row (n values, rows ld apart) in place, then its split-int8 quantization.
// One warp per row; the exponentials are kept in the row.
__global__ void softmax_quant_kernel(float* __restrict__ x, int m, int n, int64_t ld, QuantAct q) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (row >= m) return;
    float* xr = x + row * ld;
    float mx = -INFINITY;
    for (int i = lane; i < n; i += 32) mx = fmaxf(mx, xr[i]);
    mx = warp_max(mx);
    double sum = 0.0;
    for (int i = lane; i < n; i += 32) {
        const float e = expf(__fsub_rn(xr[i], mx));
        xr[i] = e;
        sum += static_cast<double>(e);
    }
    sum = warp_sum(sum);
    const float inv = static_cast<float>(1.0 / sum);
    float amax = 0.0f;
    for (int i = lane; i < n; i += 32) {
        const float p = __fmul_rn(xr[i], inv);
        xr[i] = p;
        amax = fmaxf(amax, p);
    }
    const Scales s = row_scales(warp_max(amax));
    int8_t* hr = q.hi + static_cast<int64_t>(row) * q.ld;
    int8_t* lr = q.lo + static_cast<int64_t>(row) * q.ld;
    for (int i = lane; i < n; i += 32) {
        signed char h, l;
        quant_split_one(xr[i], s.d, s.id, s.id_lo, h, l);
        hr[i] = h;
        lr[i] = l;
    }
    for (int i = n + lane; i < q.ld; i += 32) hr[i] = lr[i] = 0;
    if (lane == 0) q.scale[row] = s.d;
}

__device__ __forceinline__ float glu_at(const float* __restrict__ big, int64_t row, int cc, int c) {
    const float a = big[row * 2 * cc + c];
    const float b = big[row * 2 * cc + cc + c];
    return mul_sigmoid(a, b);
}

// GLU + depthwise convolution (taps in order from the bias, skipping frames outside the
// utterance) + SiLU, the GLU gate and the SiLU with the approximate exponential and reciprocal
// (mul_sigmoid; a few ulp from a / (1 + expf(-b)); the conversion unit would otherwise bound the
// kernel). Task t
// covers output frames [out_first, out_first + count <= 32) of one utterance; each thread owns
// one channel. The GLU values of every input frame the task reads are staged first -- eight
// frames' loads in flight at a time -- in a shared column per thread, frames outside the
// utterance as zeros: adding w * 0 leaves the sum bit for bit as skipping the tap does (the
// weights are finite), so the taps need no bounds checks. S is the stride of every task.
// The kernel is bound by instruction issue, not by memory: outputs are made kConvGroup at a
// time from a register window of the S * (kConvGroup - 1) + K staged values they read, so each
// staged value is loaded from shared memory once per group rather than once per tap.
constexpr int kConvSpan = 32;  // output frames per task (set by the host's task list)
constexpr int kConvGroup = 4;  // outputs per register window (divides kConvSpan)

template <int K, int S>
__global__ void __launch_bounds__(128) glu_dwconv_silu_kernel(const float* __restrict__ big, int cc,
                                                              const ConvTask* __restrict__ tasks,
                                                              const float* __restrict__ w,
                                                              const float* __restrict__ bias,
                                                              float* __restrict__ out) {
    constexpr int half = K / 2;
    constexpr int kFrames = S * (kConvSpan - 1) + K;  // input frames of a span
    __shared__ float glu[kFrames][128];
    constexpr int kWindow = S * (kConvGroup - 1) + K;
    const ConvTask t = tasks[blockIdx.y];
    const int c = blockIdx.x * 128 + threadIdx.x;
    const bool live = c < cc;
    const int f_lo = S * t.out_first + t.shift - half;
    const int nf = S * (t.count - 1) + K;
    const int64_t two_cc = 2 * static_cast<int64_t>(cc);
    const float* col = big + (live ? c : 0);
    for (int i0 = 0; i0 < nf; i0 += 8) {
        float a[8], b[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int f = f_lo + i0 + u;
            const bool ok = live && i0 + u < nf && static_cast<unsigned>(f) < static_cast<unsigned>(t.in_len);
            const float* p = col + static_cast<int64_t>(t.in_row + (ok ? f : 0)) * two_cc;
            a[u] = ok ? __ldg(p) : 0.0f;
            b[u] = ok ? __ldg(p + cc) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (i0 + u < nf) glu[i0 + u][threadIdx.x] = mul_sigmoid(a[u], b[u]);
    }
    if (!live) return;
    float wk[K];
#pragma unroll
    for (int j = 0; j < K; ++j) wk[j] = __ldg(w + j * cc + c);
    const float bc = __ldg(bias + c);
    float* orow = out + static_cast<int64_t>(t.out_row + t.out_first) * cc + c;
    // The last group may run past the task's count: its window still ends inside the array
    // (S * 31 + K - 1 < kFrames), and the outputs past count, made from unstaged rows, are not
    // stored.
#pragma unroll 1
    for (int r0 = 0; r0 < t.count; r0 += kConvGroup) {
        float win[kWindow];
#pragma unroll
        for (int i = 0; i < kWindow; ++i) win[i] = glu[S * r0 + i][threadIdx.x];
#pragma unroll
        for (int g = 0; g < kConvGroup; ++g) {
            float acc = bc;
#pragma unroll
            for (int j = 0; j < K; ++j) acc = __fadd_rn(acc, __fmul_rn(wk[j], win[S * g + j]));
            acc = mul_sigmoid(acc, acc);
            if (r0 + g < t.count) orow[static_cast<int64_t>(r0 + g) * cc] = acc;
        }
    }
}

// The same at stride 1 with each thread on two adjacent channels (even channel counts, 8-byte
// aligned rows): 8-byte loads, stores and shared-memory words, GLU and SiLU as packed two-wide
// f32 multiplies and adds, and each tap as two scalar multiplies and one packed add. Each packed
// instruction rounds its lanes as the scalar one does, so the bits are the scalar kernel's (the
// same output bits over 60,000 frames of 2048 and 1024 channels on B200); the multiplies stay
// scalar because the compiler fuses a packed multiply feeding a packed add into a packed fused
// multiply-add, with or without -fmad=false (one rounding where the reference has two). 64
// threads cover the same 128 channels and the same shared-memory bytes as one CTA of the scalar
// kernel; 11% faster at kernel 15 (402 us against 454 us, 60,000 frames x 2048 channels).
template <int K, int S = 1>
__global__ void __launch_bounds__(64) glu_dwconv_silu_x2_kernel(const float* __restrict__ big, int cc,
                                                                 const ConvTask* __restrict__ tasks,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ bias,
                                                                 float* __restrict__ out) {
    constexpr int half = K / 2;
    constexpr int kFrames = S * (kConvSpan - 1) + K;
    __shared__ float2 glu[kFrames][64];
    constexpr int kWindow = S * (kConvGroup - 1) + K;
    const ConvTask t = tasks[blockIdx.y];
    const int c = 2 * (blockIdx.x * 64 + threadIdx.x);
    if (c >= cc) return;  // cc is even: c + 1 < cc too
    const int f_lo = S * t.out_first + t.shift - half;
    const int nf = S * (t.count - 1) + K;
    const int64_t two_cc = 2 * static_cast<int64_t>(cc);
    const float* col = big + c;
    for (int i0 = 0; i0 < nf; i0 += 8) {
        float2 a[8], b[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int f = f_lo + i0 + u;
            const bool ok = i0 + u < nf && static_cast<unsigned>(f) < static_cast<unsigned>(t.in_len);
            const float* p = col + static_cast<int64_t>(t.in_row + (ok ? f : 0)) * two_cc;
            a[u] = ok ? __ldg(reinterpret_cast<const float2*>(p)) : make_float2(0.0f, 0.0f);
            b[u] = ok ? __ldg(reinterpret_cast<const float2*>(p + cc)) : make_float2(0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (i0 + u < nf) glu[i0 + u][threadIdx.x] = mul_sigmoid2(a[u], b[u]);
    }
    float2 wk[K];
#pragma unroll
    for (int j = 0; j < K; ++j) wk[j] = __ldg(reinterpret_cast<const float2*>(w + j * cc + c));
    const float2 bc = __ldg(reinterpret_cast<const float2*>(bias + c));
    float* orow = out + static_cast<int64_t>(t.out_row + t.out_first) * cc + c;
    // As the scalar kernel: the last group's window ends inside the array, and its outputs past
    // count, made from rows this task did not fill, are not stored.
#pragma unroll 1
    for (int r0 = 0; r0 < t.count; r0 += kConvGroup) {
        float2 win[kWindow];
#pragma unroll
        for (int i = 0; i < kWindow; ++i) win[i] = glu[S * r0 + i][threadIdx.x];
#pragma unroll
        for (int g = 0; g < kConvGroup; ++g) {
            float2 acc = bc;
#pragma unroll
            for (int j = 0; j < K; ++j) {
                const float2 x = win[S * g + j];
                acc = fadd2_rn(acc, make_float2(__fmul_rn(wk[j].x, x.x), __fmul_rn(wk[j].y, x.y)));
            }
            acc = mul_sigmoid2(acc, acc);
            if (r0 + g < t.count) *reinterpret_cast<float2*>(orow + static_cast<int64_t>(r0 + g) * cc) = acc;
        }
    }
}

// The same without a window, for other kernel sizes (the same GLU and SiLU arithmetic).
__global__ void glu_dwconv_silu_any_kernel(const float* __restrict__ big, int cc, int k,
                                           const ConvTask* __restrict__ tasks, const float* __restrict__ w,
                                           const float* __restrict__ bias, float* __restrict__ out) {
    const ConvTask t = tasks[blockIdx.y];
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cc) return;
    const int half = k / 2;
    for (int r = t.out_first; r < t.out_first + t.count; ++r) {
        float acc = __ldg(bias + c);
        for (int j = 0; j < k; ++j) {
            const int f = t.stride * r + t.shift + j - half;
            if (f >= 0 && f < t.in_len)
                acc = __fadd_rn(acc, __fmul_rn(__ldg(w + j * cc + c), glu_at(big, t.in_row + f, cc, c)));
        }
        acc = mul_sigmoid(acc, acc);
        out[static_cast<int64_t>(t.out_row + r) * cc + c] = acc;
    }
}

// out[r] = (x[2r] + x[2r + 1]) / 2 over each utterance's pairs (src/granite.rs:919-930).
__global__ void pool_pairs_kernel(const float* __restrict__ x, int d, const int* __restrict__ src_row,
                                  int rows, float* __restrict__ out) {
    const int r = blockIdx.x;
    if (r >= rows) return;
    const float* a = x + static_cast<int64_t>(src_row[r]) * d;
    const float* b = a + d;
    float* o = out + static_cast<int64_t>(r) * d;
    for (int i = threadIdx.x * 4; i < d; i += blockDim.x * 4) {
        const float4 p = *reinterpret_cast<const float4*>(a + i);
        const float4 q = *reinterpret_cast<const float4*>(b + i);
        float4 v;
        v.x = __fdiv_rn(__fadd_rn(p.x, q.x), 2.0f);
        v.y = __fdiv_rn(__fadd_rn(p.y, q.y), 2.0f);
        v.z = __fdiv_rn(__fadd_rn(p.z, q.z), 2.0f);
        v.w = __fdiv_rn(__fadd_rn(p.w, q.w), 2.0f);
        *reinterpret_cast<float4*>(o + i) = v;
    }
}

// The first largest value of each row and the gap to the runner-up (src/granite.rs:1139-1147).
__global__ void argmax_kernel(const float* __restrict__ x, int m, int n, int64_t ld, uint32_t* __restrict__ ids,
                              float* __restrict__ margin) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (row >= m) return;
    const float* xr = x + row * ld;
    float b1 = -INFINITY, b2 = -INFINITY;
    int i1 = 0x7fffffff;
    for (int i = lane; i < n; i += 32) {
        const float v = xr[i];
        if (v > b1) { b2 = b1; b1 = v; i1 = i; }
        else if (v > b2) b2 = v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ob1 = __shfl_xor_sync(kFull, b1, o), ob2 = __shfl_xor_sync(kFull, b2, o);
        const int oi1 = __shfl_xor_sync(kFull, i1, o);
        const bool other = ob1 > b1 || (ob1 == b1 && oi1 < i1);
        const float lose = other ? b1 : ob1;
        if (other) { b1 = ob1; i1 = oi1; }
        b2 = fmaxf(fmaxf(b2, ob2), lose);
    }
    if (lane == 0) {
        ids[row] = static_cast<uint32_t>(i1);
        if (margin) margin[row] = __fsub_rn(b1, b2);
    }
}

// ctc_tokens (src/granite.rs:1074-1094), one warp per utterance: a token starts where a
// non-blank id differs from the previous frame's id; its duration is the run of equal ids.
__global__ void ctc_collapse_kernel(const uint32_t* __restrict__ ids, const int* __restrict__ first,
                                    const int* __restrict__ frames, int n_utt, uint32_t blank,
                                    uint32_t* __restrict__ tokens, int* __restrict__ counts) {
    const int u = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (u >= n_utt) return;
    const uint32_t* id = ids + first[u];
    uint32_t* out = tokens + 3 * static_cast<int64_t>(first[u]);
    const int n = frames[u];
    int count = 0;
    for (int base = 0; base < n; base += 32) {
        const int f = base + lane;
        const bool valid = f < n;
        const uint32_t v = valid ? id[f] : blank;
        const bool start = valid && v != blank && (f == 0 || id[f - 1] != v);
        const unsigned mask = __ballot_sync(kFull, start);
        if (start) {
            const int slot = count + __popc(mask & ((1u << lane) - 1));
            int g = f + 1;
            while (g < n && id[g] == v) ++g;
            out[3 * slot] = v;
            out[3 * slot + 1] = static_cast<uint32_t>(f);
            out[3 * slot + 2] = static_cast<uint32_t>(g - f);
        }
        count += __popc(mask);
    }
    if (lane == 0) counts[u] = count;
}

}  // namespace

cudaError_t ln_chain(const float* x, int m, int d, const float* ga, const float* ba, float* y_out,
                     const float* gb, const float* bb, const QuantAct* q, cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    QuantAct qa = q ? *q : QuantAct();
    const float eps = 1e-5f;
#define TELMO_LN_CASE(C, P)                                                                               \
    case C:                                                                                               \
        ln_chain_kernel<C, P><<<(m + 8 / P - 1) / (8 / P), 256, 0, stream>>>(x, m, d, ga, ba, y_out, gb, bb, qa, eps); \
        break;
    switch (d / 128) {
        TELMO_LN_CASE(1, 1)
        TELMO_LN_CASE(2, 1)
        TELMO_LN_CASE(4, 1)
        TELMO_LN_CASE(8, 1)
        TELMO_LN_CASE(12, 2)
        TELMO_LN_CASE(16, 2)
        default: return cudaErrorInvalidValue;
    }
#undef TELMO_LN_CASE
    if (d % 128) return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t softmax_quant(float* x, int m, int n, int64_t ld, const QuantAct& q, cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    constexpr int kWarps = 8;
    softmax_quant_kernel<<<(m + kWarps - 1) / kWarps, kWarps * 32, 0, stream>>>(x, m, n, ld, q);
    return cudaGetLastError();
}

cudaError_t glu_dwconv_silu(const float* big, int cc, int k, int stride, const ConvTask* tasks, int n_tasks,
                            const float* w, const float* bias, float* out, cudaStream_t stream) {
    if (n_tasks <= 0) return cudaSuccess;
    if (stride != 1 && stride != 2) return cudaErrorInvalidValue;
    const int threads = 128;
    constexpr int kMaxTasks = 65535;  // tasks run along gridDim.y
    const auto aligned8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
    // Stride 1 with even channels takes the two-channel kernel; stride 2 stays on the scalar one,
    // whose 77-frame staging at twice the warps per shared-memory byte ran faster (B200, 2048
    // channels, kernel 15: 351 us against 375 us over 60,000 frames).
    const bool pairs = cc % 2 == 0 && aligned8(big) && aligned8(w) && aligned8(bias) && aligned8(out);
    for (int t0 = 0; t0 < n_tasks; t0 += kMaxTasks) {
        const ConvTask* tk = tasks + t0;
        const dim3 grid((cc + threads - 1) / threads, n_tasks - t0 < kMaxTasks ? n_tasks - t0 : kMaxTasks);
#define TELMO_CONV_CASE(K)                                                                                       \
    case K:                                                                                                      \
        if (pairs && stride == 1) glu_dwconv_silu_x2_kernel<K><<<grid, 64, 0, stream>>>(big, cc, tk, w, bias, out); \
        else if (stride == 1) glu_dwconv_silu_kernel<K, 1><<<grid, threads, 0, stream>>>(big, cc, tk, w, bias, out); \
        else glu_dwconv_silu_kernel<K, 2><<<grid, threads, 0, stream>>>(big, cc, tk, w, bias, out);             \
        break;
        switch (k) {
            TELMO_CONV_CASE(3)
            TELMO_CONV_CASE(5)
            TELMO_CONV_CASE(7)
            TELMO_CONV_CASE(9)
            TELMO_CONV_CASE(15)
            default: glu_dwconv_silu_any_kernel<<<grid, threads, 0, stream>>>(big, cc, k, tk, w, bias, out);
        }
#undef TELMO_CONV_CASE
        if (cudaError_t e = cudaGetLastError()) return e;
    }
    return cudaSuccess;
}

cudaError_t pool_pairs(const float* x, int d, const int* src_row, int rows, float* out, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    pool_pairs_kernel<<<rows, 128, 0, stream>>>(x, d, src_row, rows, out);
    return cudaGetLastError();
}

cudaError_t argmax_rows(const float* x, int m, int n, int64_t ld, uint32_t* ids, float* margin, cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    constexpr int kWarps = 8;
    argmax_kernel<<<(m + kWarps - 1) / kWarps, kWarps * 32, 0, stream>>>(x, m, n, ld, ids, margin);
    return cudaGetLastError();
}

cudaError_t ctc_collapse(const uint32_t* ids, const int* first, const int* frames, int n_utt, uint32_t blank,
                         uint32_t* tokens, int* counts, cudaStream_t stream) {
    if (n_utt <= 0) return cudaSuccess;
    constexpr int kWarps = 4;
    ctc_collapse_kernel<<<(n_utt + kWarps - 1) / kWarps, kWarps * 32, 0, stream>>>(ids, first, frames, n_utt, blank,
                                                                                   tokens, counts);
    return cudaGetLastError();
}

}  // namespace telmo
