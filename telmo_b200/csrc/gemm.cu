// gemm.cu -- the split-int8 linear on tcgen05 tensor cores.
//
// C[m, n] = epilogue(A[m, k] . W[n, k]^T) where A arrives as two int8 levels per element
// (A = s_row * (hi + lo / 254)) and W is int8 with one scale per output row, the reference's
// Precision::Int8 (src/quant.rs:1-13). Each level is an exact int8 x int8 -> s32 product
// accumulated in TMEM, so both i32 sums are bit-exact; the epilogue combines them, applies the
// row and weight scales and the reference's Epilogue (bias, act, scale, accumulate;
// src/kernels/mod.rs:366-398) and stores f32 or bf16.
//
// Structure: a persistent, warp-specialised kernel, one CTA per SM.
//   warp 0      TMA producer: 128x128-byte boxes of A_hi, A_lo and W per stage, 128-byte swizzle
//   warp 1      MMA issuer: tcgen05.mma kind::i8, M=128, N=BN, K=32, two accumulators per tile
//   warps 2-5   epilogue: tcgen05.ld from TMEM, fused scale/bias/act/residual, global stores
// TMEM holds two tiles' accumulators (2 x 2 x BN columns), so the epilogue of one tile overlaps
// the main loop of the next. Every mbarrier wait is bounded; on timeout the kernel records
// kErrWaitTimeout in the error word and returns.
#include "kernels.h"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <mutex>

namespace telmo {

namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes = int8 elements per stage along K (one 128-byte swizzle row)
constexpr int UMMA_K = 32;
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
    static constexpr int kStages = BN == 128 ? 4 : 3;
    static constexpr int kABytes = BM * BK;         // one level of A
    static constexpr int kBBytes = BN * BK;
    static constexpr int kStageBytes = 2 * kABytes + kBBytes;
    static constexpr int kTmemCols = 4 * BN;        // 2 buffers x 2 levels x BN
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
};

struct Params {
    int m, n, k;
    const float* row_scale;
    const float* w_scale;
    const float* bias;
    int act;
    float scale;
    int accumulate;
    void* out;
    int64_t ldc;
    int out_kind;
    uint32_t* error;
};

__device__ __forceinline__ void record_error(uint32_t* error, uint32_t code) {
    if (error) atomicCAS(error, 0u, code);
}

__device__ __forceinline__ float epilogue_value(int32_t acc_hi, int32_t acc_lo, float rs, float ws,
                                                bool has_bias, float bias, int act, float scale) {
    // Step for step what oracle_epilogue_x2 computes, with no contraction into FMA.
    const float inv254 = 1.0f / 254.0f;
    float v = __fadd_rn(__int2float_rn(acc_hi), __fmul_rn(__int2float_rn(acc_lo), inv254));
    v = __fmul_rn(v, rs);
    v = __fmul_rn(v, ws);
    if (has_bias) v = __fadd_rn(v, bias);
    if (act == kActRelu) v = fmaxf(v, 0.0f);
    else if (act == kActSilu) v = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    return __fmul_rn(v, scale);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_i8x2_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                 const __grid_constant__ CUtensorMap map_w, const Params p) {
    using C = Cfg<BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
    uint64_t* empty = full + C::kStages;
    uint64_t* tmem_full = empty + C::kStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_m = (p.m + BM - 1) / BM, num_n = (p.n + BN - 1) / BN;
    const int tiles = num_m * num_n;
    const int kblocks = (p.k + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 4 * 32);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&map_hi);
        prefetch_tensormap(&map_lo);
        prefetch_tensormap(&map_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_base_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_base_slot;

    if (warp == 0) {
        // ---- TMA producer ------------------------------------------------------------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
                const int m0 = (t % num_m) * BM, n0 = (t / num_m) * BN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) {
                        record_error(p.error, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t* st = smem + stage * C::kStageBytes;
                    mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
                    tma_load_2d(&map_hi, &full[stage], st, kb * BK, m0);
                    tma_load_2d(&map_lo, &full[stage], st + C::kABytes, kb * BK, m0);
                    tma_load_2d(&map_w, &full[stage], st + 2 * C::kABytes, kb * BK, n0);
                    if (++stage == C::kStages) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----------------------------------------------------------------------
        constexpr uint32_t idesc = idesc_i8(BM, BN);
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = static_cast<uint32_t>(it >> 1);
            if (!mbar_wait(&tmem_empty[buf], (use & 1) ^ 1)) {
                record_error(p.error, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t d_hi = tmem_base + static_cast<uint32_t>(buf * 2 * BN);
            const uint32_t d_lo = d_hi + BN;
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_hi = smem_u32(smem + stage * C::kStageBytes);
                    const uint32_t a_lo = a_hi + C::kABytes;
                    const uint32_t b = a_hi + 2 * C::kABytes;
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        const uint64_t db = sw128_desc(b + kk * UMMA_K);
                        mma_i8(d_hi, sw128_desc(a_hi + kk * UMMA_K), db, idesc, acc);
                        mma_i8(d_lo, sw128_desc(a_lo + kk * UMMA_K), db, idesc, acc);
                    }
                    mma_commit(&empty[stage]);
                }
                __syncwarp();
                if (++stage == C::kStages) { stage = 0; phase ^= 1; }
            }
            if (!ok) {
                record_error(p.error, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            if (lane == 0) mma_commit(&tmem_full[buf]);
            __syncwarp();
        }
    } else {
        // ---- epilogue (warps 2..5) -------------------------------------------------------------
        const int quad = warp & 3;  // TMEM lanes this warp may access: 32 * quad ..
        const int r_in_tile = quad * 32 + lane;
        int it = 0;
        for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = static_cast<uint32_t>(it >> 1);
            const int m0 = (t % num_m) * BM, n0 = (t / num_m) * BN;
            if (!mbar_wait(&tmem_full[buf], use & 1)) {
                record_error(p.error, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int row = m0 + r_in_tile;
            const bool row_ok = row < p.m;
            const float rs = row_ok ? p.row_scale[row] : 0.0f;
            const uint32_t t_hi = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                  static_cast<uint32_t>(buf * 2 * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t hi[32], lo[32];
                tmem_ld32(t_hi + c * 32, hi);
                tmem_ld32(t_hi + BN + c * 32, lo);
                tmem_ld_wait();
                const int col0 = n0 + c * 32;
                if (!row_ok || col0 >= p.n) continue;
                const int cols = min(32, p.n - col0);
                if (p.out_kind == kOutI32Pair) {
                    int32_t* o_hi = static_cast<int32_t*>(p.out) + row * p.ldc + col0;
                    int32_t* o_lo = o_hi + static_cast<int64_t>(p.m) * p.ldc;
                    for (int j = 0; j < cols; ++j) {
                        o_hi[j] = static_cast<int32_t>(hi[j]);
                        o_lo[j] = static_cast<int32_t>(lo[j]);
                    }
                    continue;
                }
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int col = min(col0 + j, p.n - 1);
                    const float ws = __ldg(p.w_scale + col);
                    const float bs = p.bias ? __ldg(p.bias + col) : 0.0f;
                    v[j] = epilogue_value(static_cast<int32_t>(hi[j]), static_cast<int32_t>(lo[j]),
                                          rs, ws, p.bias != nullptr, bs, p.act, p.scale);
                }
                if (p.out_kind == kOutF32) {
                    float* o = static_cast<float*>(p.out) + row * p.ldc + col0;
                    const bool vec = cols == 32 && (reinterpret_cast<uintptr_t>(o) & 15) == 0;
                    if (vec) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            float4 x = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                            if (p.accumulate) {
                                const float4 y = *reinterpret_cast<const float4*>(o + j);
                                x.x = __fadd_rn(y.x, x.x); x.y = __fadd_rn(y.y, x.y);
                                x.z = __fadd_rn(y.z, x.z); x.w = __fadd_rn(y.w, x.w);
                            }
                            *reinterpret_cast<float4*>(o + j) = x;
                        }
                    } else {
                        for (int j = 0; j < cols; ++j)
                            o[j] = p.accumulate ? __fadd_rn(o[j], v[j]) : v[j];
                    }
                } else {
                    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + row * p.ldc + col0;
                    for (int j = 0; j < cols; ++j) {
                        const float x = p.accumulate ? __fadd_rn(__bfloat162float(o[j]), v[j]) : v[j];
                        o[j] = __float2bfloat16_rn(x);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[buf]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// A 2-D int8 tensor map over rows of `cols` bytes, `ld` bytes apart, boxes of 128 bytes x
// box_rows rows with the 128-byte swizzle. Reads past `cols` or `rows` fill zeros.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
              uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN>
cudaError_t launch(const GemmArgs& g, cudaStream_t stream) {
    using C = Cfg<BN>;
    const DevWeights& w = *g.w;
    CUtensorMap mh, ml, mw;
    if (!make_map(&mh, g.a.hi, g.m, w.k, g.a.ld, BM) || !make_map(&ml, g.a.lo, g.m, w.k, g.a.ld, BM) ||
        !make_map(&mw, w.values, w.n, w.k, w.ld, BN))
        return cudaErrorInvalidValue;
    static uint64_t configured = 0;  // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(configured >> dev & 1)) {
        cudaError_t e = cudaFuncSetAttribute(gemm_i8x2_kernel<BN>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= uint64_t(1) << dev;
    }
    Params p{g.m, w.n, w.k, g.a.scale, w.scales, g.bias, g.act, g.scale, g.accumulate,
             g.out, g.ldc, g.out_kind, g.error};
    const int tiles = ((g.m + BM - 1) / BM) * ((w.n + BN - 1) / BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    gemm_i8x2_kernel<BN><<<grid, kThreads, C::kSmemBytes, stream>>>(mh, ml, mw, p);
    return cudaGetLastError();
}

}  // namespace

int num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

cudaError_t gemm_i8x2(const GemmArgs& g, cudaStream_t stream) {
    if (g.m <= 0 || !g.w || g.w->n <= 0) return cudaSuccess;
    if ((g.a.ld % 16) || (g.w->ld % 16)) return cudaErrorInvalidValue;
    return launch<128>(g, stream);
}

}  // namespace telmo
