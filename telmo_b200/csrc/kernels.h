// kernels.h -- host-side launchers of the CUDA kernels (internal to libtelmo_b200).
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace telmo {

// One bit per device for set-up done once per device (kernel attributes): safe to test and set
// from several host threads at once.
struct DeviceOnce {
    std::atomic<uint64_t> bits{0};
    bool done(int dev) const { return dev < 64 && ((bits.load(std::memory_order_acquire) >> dev) & 1); }
    void mark(int dev) {
        if (dev < 64) bits.fetch_or(uint64_t(1) << dev, std::memory_order_release);
    }
};

// kOutF16Split writes each value v as two fp16 planes, hi = fp16(v) at rows 0..m-1 and
// lo = fp16(v - hi) at rows m..2m-1 (ldc apart): the operands of the tensor-core attention.
enum OutKind : int { kOutF32 = 0, kOutBF16 = 1, kOutI32Pair = 2, kOutF16Split = 3 };
enum Act : int { kActNone = 0, kActRelu = 1, kActSilu = 2 };

// Quantized activations for the split-int8 GEMM: two int8 levels and one scale per row, rows
// `ld` bytes apart (ld a multiple of 16, at least K).
struct QuantAct {
    int8_t* hi = nullptr;
    int8_t* lo = nullptr;
    float* scale = nullptr;
    int64_t ld = 0;
};

// Device weights of one linear layer: int8 row-major [n, ld] (ld = k rounded up to 16 bytes,
// zero padded), per-output f32 scales. Q8_0 packs carry a second int8 level: the row stands for
// scale * (values + lo_values / 254), the split the activations use.
struct DevWeights {
    int n = 0, k = 0;
    int64_t ld = 0;
    int8_t* values = nullptr;
    int8_t* lo_values = nullptr;  // null for Int8 packs
    float* scales = nullptr;
};

struct GemmArgs {
    int m = 0;
    QuantAct a;
    const DevWeights* w = nullptr;
    const float* bias = nullptr;  // [n] or null
    int act = kActNone;
    float scale = 1.0f;
    int accumulate = 0;
    void* out = nullptr;          // [m, ldc] of out_kind; kOutI32Pair writes acc_hi then acc_lo
    int64_t ldc = 0;              // planes, each [m, ldc] int32
    int out_kind = kOutF32;
    uint32_t* error = nullptr;    // device error word
};

int num_sms();
cudaError_t gemm_i8x2(const GemmArgs& g, cudaStream_t stream);

// x f32 [m, k] (rows ldx floats apart) -> hi, lo, scale (the oracle's quantize_x2 rule).
#ifdef __CUDACC__
// One value's split-int8 pair: hi = x / d rounded to the nearest integer (halves to even), lo =
// (x - hi d) * 254 / d rounded the same way; id = 1 / d and id_lo = 254 / d as the row's quantizer
// computes them. |x id| and |e id_lo| stay below 127.5 for finite rows (|x| <= 127 d to within
// a few ulp, |e| <= d / 2 likewise), so both levels land in [-127, 127] without a clamp. Adding
// 1.5 * 2^23 rounds to the nearest integer exactly and leaves it in the low byte of the sum's
// bits (two's complement), all on the FMA and integer pipes.
__device__ __forceinline__ void quant_split_one(float x, float d, float id, float id_lo, int8_t& h8, int8_t& l8) {
    const float uh = __fadd_rn(__fmul_rn(x, id), 12582912.0f);
    const float h = __fsub_rn(uh, 12582912.0f);
    const float e = __fmaf_rn(-h, d, x);
    const float ul = __fadd_rn(__fmul_rn(e, id_lo), 12582912.0f);
    h8 = static_cast<int8_t>(__float_as_int(uh) & 0xff);
    l8 = static_cast<int8_t>(__float_as_int(ul) & 0xff);
}


// 2^x and 1/x as the PTX ISA's single approximate instructions (ex2.approx.ftz.f32, relative
// error about 2^-22; rcp.approx.ftz.f32, within 1 ulp).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// a / (1 + e^-b) with e^-b = 2^(-b log2 e): the GLU gate, and (a = b) SiLU. Over the 123M values
// of a 60,000-frame, 2048-channel depthwise conv it gave the bits __fdividef(a, 1 + __expf(-b))
// gives, in fewer instructions (the conv kernel, bound by issue, ran 16% faster).
__device__ __forceinline__ float mul_sigmoid(float a, float b) {
    return __fmul_rn(a, rcp_approx(__fadd_rn(1.0f, ex2_approx(__fmul_rn(b, -1.44269504f)))));
}

// sm_100's packed two-wide f32 multiply and add, each lane rounded to nearest even as the scalar
// mul.rn / add.rn. Unlike the scalar forms they are not kept out of contraction: the compiler
// turns a packed multiply whose result feeds a packed add into one packed fused multiply-add,
// even under -fmad=false (measured on B200: every lane of such a chain gave the fma chain's
// bits; a packed add fed by scalar __fmul_rn products, or a packed multiply whose products a
// scalar __fadd_rn adds, gave the scalar chain's), so callers that must round the product keep
// one side of each multiply-add scalar.
__device__ __forceinline__ uint64_t pack_f2(float2 v) {
    return (static_cast<uint64_t>(__float_as_uint(v.y)) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 unpack_f2(uint64_t v) {
    return make_float2(__uint_as_float(static_cast<uint32_t>(v)), __uint_as_float(static_cast<uint32_t>(v >> 32)));
}
__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack_f2(a)), "l"(pack_f2(b)));
    return unpack_f2(d);
}
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack_f2(a)), "l"(pack_f2(b)));
    return unpack_f2(d);
}

// mul_sigmoid on two lanes: the same bits per lane.
__device__ __forceinline__ float2 mul_sigmoid2(float2 a, float2 b) {
    const float2 t = fmul2_rn(b, make_float2(-1.44269504f, -1.44269504f));
    const float2 s = fadd2_rn(make_float2(1.0f, 1.0f), make_float2(ex2_approx(t.x), ex2_approx(t.y)));
    return fmul2_rn(a, make_float2(rcp_approx(s.x), rcp_approx(s.y)));
}
#endif

cudaError_t quantize_x2(const float* x, int64_t ldx, int m, int k, const QuantAct& q,
                        cudaStream_t stream);

}  // namespace telmo
