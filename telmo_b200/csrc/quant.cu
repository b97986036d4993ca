// quant.cu -- split-int8 quantization of activation rows, the A operand of the int8 GEMM.
//
// Each row x of k values becomes s * (hi + lo / 254): s = amax / 127 as quantize_row_int8 sets a
// weight row's (src/quant.rs:190-198), hi = x / s rounded to the nearest integer (halves to
// even), then lo = (x - hi * s) * 254 / s rounded the same way, the residual at 254 times finer
// steps. One warp per row; the f32 steps match oracle_quantize_x2 bit for bit.
#include "kernels.h"

namespace telmo {

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__global__ void quantize_x2_kernel(const float* __restrict__ x, int64_t ldx, int m, int k,
                                   int8_t* __restrict__ hi, int8_t* __restrict__ lo, int64_t ldq,
                                   float* __restrict__ scale) {
    const int warps = blockDim.x / 32;
    const int row = blockIdx.x * warps + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (row >= m) return;
    const float* xr = x + row * ldx;
    const bool vec = (k % 4 == 0) && (ldx % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    float amax = 0.0f;
    if (vec) {
        for (int i = lane * 4; i < k; i += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        for (int i = lane; i < k; i += 32) amax = fmaxf(amax, fabsf(xr[i]));
    }
    amax = warp_max(amax);
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float id_lo = __fmul_rn(id, 254.0f);
    int8_t* hr = hi + row * ldq;
    int8_t* lr = lo + row * ldq;
    if (vec && (ldq % 4 == 0)) {
        for (int i = lane * 4; i < k; i += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            char4 h, l;
            quant_split_one(v.x, d, id, id_lo, reinterpret_cast<int8_t&>(h.x), reinterpret_cast<int8_t&>(l.x));
            quant_split_one(v.y, d, id, id_lo, reinterpret_cast<int8_t&>(h.y), reinterpret_cast<int8_t&>(l.y));
            quant_split_one(v.z, d, id, id_lo, reinterpret_cast<int8_t&>(h.z), reinterpret_cast<int8_t&>(l.z));
            quant_split_one(v.w, d, id, id_lo, reinterpret_cast<int8_t&>(h.w), reinterpret_cast<int8_t&>(l.w));
            *reinterpret_cast<char4*>(hr + i) = h;
            *reinterpret_cast<char4*>(lr + i) = l;
        }
    } else {
        for (int i = lane; i < k; i += 32) quant_split_one(xr[i], d, id, id_lo, hr[i], lr[i]);
    }
    for (int i = k + lane; i < ldq; i += 32) hr[i] = lr[i] = 0;
    if (lane == 0) scale[row] = d;
}

// The same for rows of k = 128 * C values (16-byte aligned): the row stays in registers, so it
// is read from memory once. W warps share a row (C / W float4 per lane each), exchanging their
// maxima through shared memory, which keeps long rows at a register count that leaves room for
// several blocks per SM.
template <int C, int W>
__global__ void __launch_bounds__(256) quantize_x2_regs_kernel(const float* __restrict__ x, int64_t ldx, int m,
                                                               int8_t* __restrict__ hi, int8_t* __restrict__ lo,
                                                               int64_t ldq, float* __restrict__ scale) {
    constexpr int CW = C / W;  // float4 per lane
    __shared__ float part[8];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int row = blockIdx.x * (8 / W) + warp / W;
    const int piece = warp % W;
    const bool live = row < m;
    const float* xr = x + static_cast<int64_t>(live ? row : 0) * ldx + piece * CW * 128;
    float4 v[CW];
#pragma unroll
    for (int c = 0; c < CW; ++c)
        v[c] = live ? *reinterpret_cast<const float4*>(xr + (c * 32 + lane) * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    float amax = 0.0f;
#pragma unroll
    for (int c = 0; c < CW; ++c)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c].x), fabsf(v[c].y)), fmaxf(fabsf(v[c].z), fabsf(v[c].w))));
    amax = warp_max(amax);
    if (W > 1) {
        if (lane == 0) part[warp] = amax;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < W; ++i) amax = fmaxf(amax, part[(warp / W) * W + i]);
    }
    if (!live) return;
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float id_lo = __fmul_rn(id, 254.0f);
    int8_t* hr = hi + static_cast<int64_t>(row) * ldq + piece * CW * 128;
    int8_t* lr = lo + static_cast<int64_t>(row) * ldq + piece * CW * 128;
#pragma unroll
    for (int c = 0; c < CW; ++c) {
        char4 h, l;
        quant_split_one(v[c].x, d, id, id_lo, reinterpret_cast<int8_t&>(h.x), reinterpret_cast<int8_t&>(l.x));
        quant_split_one(v[c].y, d, id, id_lo, reinterpret_cast<int8_t&>(h.y), reinterpret_cast<int8_t&>(l.y));
        quant_split_one(v[c].z, d, id, id_lo, reinterpret_cast<int8_t&>(h.z), reinterpret_cast<int8_t&>(l.z));
        quant_split_one(v[c].w, d, id, id_lo, reinterpret_cast<int8_t&>(h.w), reinterpret_cast<int8_t&>(l.w));
        *reinterpret_cast<char4*>(hr + (c * 32 + lane) * 4) = h;
        *reinterpret_cast<char4*>(lr + (c * 32 + lane) * 4) = l;
    }
    if (piece == W - 1) {
        int8_t* hz = hi + static_cast<int64_t>(row) * ldq;
        int8_t* lz = lo + static_cast<int64_t>(row) * ldq;
        for (int i = C * 128 + lane; i < ldq; i += 32) hz[i] = lz[i] = 0;
        if (lane == 0) scale[row] = d;
    }
}

}  // namespace

cudaError_t quantize_x2(const float* x, int64_t ldx, int m, int k, const QuantAct& q,
                        cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    constexpr int kWarps = 8;
    const int grid = (m + kWarps - 1) / kWarps;
    const bool regs = k % 128 == 0 && ldx % 4 == 0 && q.ld % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (regs) {
        switch (k / 128) {
            case 8: quantize_x2_regs_kernel<8, 1><<<grid, 256, 0, stream>>>(x, ldx, m, q.hi, q.lo, q.ld, q.scale);
                return cudaGetLastError();
            case 16: quantize_x2_regs_kernel<16, 1><<<grid, 256, 0, stream>>>(x, ldx, m, q.hi, q.lo, q.ld, q.scale);
                return cudaGetLastError();
            case 32:
                quantize_x2_regs_kernel<32, 2><<<(m + 3) / 4, 256, 0, stream>>>(x, ldx, m, q.hi, q.lo, q.ld, q.scale);
                return cudaGetLastError();
            default: break;
        }
    }
    quantize_x2_kernel<<<grid, kWarps * 32, 0, stream>>>(x, ldx, m, k, q.hi, q.lo, q.ld, q.scale);
    return cudaGetLastError();
}

}  // namespace telmo
