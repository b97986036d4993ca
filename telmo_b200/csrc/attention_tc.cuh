// attention_tc.cuh -- device helpers shared by the tcgen05 attention kernels (attention_tc.cu,
// txl_attention_tc.cu): operand staging from the QKV product's fp16 planes, the fp16 split of
// probabilities, the softmax warps' barrier and the register shift of their position spans.
#pragma once

#include "ptx.cuh"

#include <cuda_fp16.h>

namespace telmo {
namespace tc_attention {

constexpr int kBox = 128 * 128;     // one 128-row x 64-fp16 box, 128-byte swizzle (16 KB)
constexpr int kOperand = 4 * kBox;  // hi and lo planes, two 64-column halves each
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void record_error(uint32_t* error, uint32_t code) {
    if (error) atomicCAS(error, 0u, code);
}

// The four boxes of one operand (hi, lo planes; two 64-column halves) at column x, into the
// operand's 64 KB: hi half 0, hi half 1, lo half 0, lo half 1.
__device__ __forceinline__ void load_operand(const CUtensorMap* map, uint64_t* bar, uint8_t* dst, int x, int y_hi,
                                             int y_lo) {
    tma_load_2d(map, bar, dst, x, y_hi);
    tma_load_2d(map, bar, dst + kBox, x + 64, y_hi);
    tma_load_2d(map, bar, dst + 2 * kBox, x, y_lo);
    tma_load_2d(map, bar, dst + 3 * kBox, x + 64, y_lo);
}

// A probability p (0 <= p <= 1) rounded to fp16's 11 significant bits, to nearest even, on the
// integer pipe -- the value fp16(p) stands for, for p >= 2^-14; below that 0, so the low part
// carries p. p - f16_high(p) is exact in f32.
__device__ __forceinline__ float f16_high(float p) {
    const uint32_t u = __float_as_uint(p);
    const uint32_t r = (u + 0x0FFFu + ((u >> 13) & 1u)) & ~0x1FFFu;
    return p >= 6.103515625e-05f ? __uint_as_float(r) : 0.0f;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);  // a in the low half
    return *reinterpret_cast<const uint32_t*>(&h);
}

// The softmax warps' named barrier (barrier 0 is __syncthreads).
template <int kThreadsInBarrier>
__device__ __forceinline__ void epi_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kThreadsInBarrier) : "memory");
}

// v[k] = v[k + D] for k < N when `on` (N + D <= 64), else v unchanged: one stage of a shift by a
// per-lane amount, done on values already in registers (ascending k reads each v[k + D] before
// this stage overwrites it).
template <int N, int D>
__device__ __forceinline__ void shift_down(uint32_t (&v)[64], bool on) {
    static_assert(N + D <= 64, "the stage reads inside the array");
#pragma unroll
    for (int k = 0; k < N; ++k) v[k] = on ? v[k + D] : v[k];
}

}  // namespace tc_attention
}  // namespace telmo
