// mma.cuh -- warp-level tensor-core helpers shared by the attention kernels: cp.async staging,
// ldmatrix fragment loads and mma.sync m16n8k16 (fp16 in, f32 accumulate), plus the fp16
// high/low split that keeps about 21 bits of an f32 operand.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace telmo {
namespace mma {

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    const int n = valid ? 16 : 0;  // 0: fill the 16 bytes with zeros
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

// 4-byte cp.async (through L1), zero-filled when !valid.
__device__ __forceinline__ void cp4(void* dst, const void* src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    const int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Waits until at most N of this thread's committed groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void cp_commit_wait() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void split_half(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
}

// Two f32 values as (hi, lo) fp16x2 registers, the first value in the low half.
__device__ __forceinline__ void split_pack(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    __half h0, l0, h1, l1;
    split_half(x0, h0, l0);
    split_half(x1, h1, l1);
    const __half2 h = __halves2half2(h0, h1), l = __halves2half2(l0, l1);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

__device__ __forceinline__ void ldsm_x4(const __half* p, uint32_t (&r)[4]) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

__device__ __forceinline__ void ldsm_x4_t(const __half* p, uint32_t (&r)[4]) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16 x 16 at row r0, column k0) of a row-major fp16 tile with pitch hp.
__device__ __forceinline__ void load_a(const __half* base, int hp, int r0, int k0, int lane, uint32_t (&a)[4]) {
    ldsm_x4(base + (r0 + (lane % 8) + ((lane / 8) % 2) * 8) * hp + k0 + (lane / 16) * 8, a);
}

// B fragments of two n-tiles: rows n0 .. n0 + 15 of an [n][k] tile, k0 .. k0 + 15.
__device__ __forceinline__ void load_b_nk(const __half* base, int hp, int n0, int k0, int lane, uint32_t (&b)[4]) {
    ldsm_x4(base + (n0 + (lane % 8) + (lane / 16) * 8) * hp + k0 + ((lane / 8) % 2) * 8, b);
}

// B fragments of two n-tiles: columns n0 .. n0 + 15 of a [k][n] tile, rows k0 .. k0 + 15.
__device__ __forceinline__ void load_b_kn(const __half* base, int hp, int k0, int n0, int lane, uint32_t (&b)[4]) {
    ldsm_x4_t(base + (k0 + (lane % 8) + ((lane / 8) % 2) * 8) * hp + n0 + (lane / 16) * 8, b);
}

}  // namespace mma
}  // namespace telmo
