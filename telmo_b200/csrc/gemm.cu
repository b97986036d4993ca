// gemm.cu -- the split-int8 linear on tcgen05 tensor cores.
//
// C[m, n] = epilogue(A[m, k] . W[n, k]^T) where A arrives as two int8 levels per element
// (A = s_row * (hi + lo / 254)) and W is int8 with one scale per output row, the reference's
// Precision::Int8 (src/quant.rs:1-13), or -- for Q8_0 packs, re-encoded at upload -- two int8
// levels under one row scale, W = s_w * (W_hi + W_lo / 254), whose W_lo . A_hi product joins the
// low-level sums. Each level is an exact int8 x int8 -> s32 product
// accumulated in TMEM, so both i32 sums are bit-exact; the epilogue combines them, applies the
// row and weight scales and the reference's Epilogue (bias, act, scale, accumulate;
// src/kernels/mod.rs:366-398) and stores f32 or bf16.
//
// The MMA computes the transposed tile: its A operand is 128 weight rows (output features) and
// its B operand is 128 activation rows of the high level followed by the same 128 rows of the low
// level (N = 256), so one tcgen05.mma (M=128, N=256, K=32) produces both levels' sums and the
// weight tile is read once per K step. TMEM lane i holds feature n0 + i; columns 0..127 hold the
// high sums of rows m0.., columns 128..255 the low sums.
//
// Structure: a persistent, warp-specialised kernel, one CTA per SM.
//   warp 0      TMA producer: 128 x 128-byte boxes of W, A_hi and A_lo per stage (128B swizzle)
//   warp 1      MMA issuer: 4 x tcgen05.mma kind::i8 per 128-byte K step
//   warps 2-17  epilogue: tcgen05.ld of 16 columns at a time, fused scale/bias/act/residual, TMA
//               stores (four warps per TMEM lane quarter, each on a quarter of the tile's
//               activation rows, so four warps per scheduler overlap one another's TMEM loads,
//               scale loads and stores)
// TMEM holds two tiles (2 x 256 columns), so the epilogue of one tile overlaps the main loop of
// the next. Every mbarrier wait is bounded; on timeout the kernel records kErrWaitTimeout in the
// error word and returns.
#include "kernels.h"
#include "ptx.cuh"
#include "tma.h"

#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <cstring>
#include <mutex>

namespace telmo {

namespace {

constexpr int BN = 128;  // output features per tile (MMA M)
constexpr int BM = 128;  // activation rows per tile (MMA N = 2 * BM)
constexpr int BK = 128;  // bytes = int8 elements per stage along K (one 128-byte swizzle row)
constexpr int UMMA_K = 32;
constexpr int kEpiWarps = 16;                // four per TMEM lane quarter, each on a quarter of the columns
constexpr int kRows = 16;                    // activation rows (TMEM columns) per epilogue chunk
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kTileBytes = 128 * BK;  // one 128-row operand box
constexpr int kTmemCols = 2 * 2 * BM;  // 2 buffers x (hi, lo) x BM columns
constexpr int kStageOutBytes = kRows * 32 * 4;  // one 16-row x 32-feature f32 output chunk
constexpr int kOutStaging = kEpiWarps * kStageOutBytes;  // one buffer per epilogue warp

// Pipeline shape per variant: CG = 1, one CTA per 128-feature tile, stages of W + A_hi + A_lo
// (48 KB); CG = 2, a CTA pair per 256-feature tile, each CTA staging its 128 weight rows and
// one activation level (32 KB), so the same shared memory holds six stages. WL (two-level
// weights, from Q8_0 packs; single CTAs only): W + A_hi + A_lo + W_lo (64 KB), three stages.
template <int CG, bool WL = false>
struct Shape {
    static constexpr int kStageBytes = (CG == 1 ? (WL ? 4 : 3) : 2) * kTileBytes;
    static constexpr int kStages = CG == 1 ? (WL ? 3 : 4) : 6;
    static constexpr int kSmemBytes = kStages * kStageBytes + kOutStaging + 1024 + 256;
};

// How the epilogue writes: TMA store of staged chunks, TMA reduce-add (accumulate), or direct
// global stores when the output's alignment rules out TMA.
enum OutPath : int { kDirect = 0, kTmaStore = 1, kTmaReduce = 2 };

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
    int out_path;
    uint32_t* error;
};

__device__ __forceinline__ void record_error(uint32_t* error, uint32_t code) {
    if (error) atomicCAS(error, 0u, code);
}

// The correctly rounded float of an int32 without the conversion unit (which the epilogue would
// otherwise saturate at two conversions per output): x = h * 65536 + l with l in [0, 65536);
// h and l convert exactly through the float bit pattern of 2^23 + n, h * 65536 is exact, and
// the one rounded add yields round-to-nearest-even of x, as __int2float_rn does.
// The biased patterns are built with one add (h + 32768 < 2^16, so adding 0x4b008000 sets the
// same bits as the OR) and one byte permute (the low two bytes under 0x4b00), and the product by
// 65536 being exact, one fused multiply-add rounds the sum exactly once.
__device__ __forceinline__ float exact_i2f(uint32_t bits) {
    const int32_t h = static_cast<int32_t>(bits) >> 16;  // -32768 .. 32767
    const float fh = __fsub_rn(__int_as_float(h + 0x4b008000), 8421376.0f);
    const float fl = __fsub_rn(__uint_as_float(__byte_perm(bits, 0x4b000000u, 0x7610)), 8388608.0f);
    return __fmaf_rn(fh, 65536.0f, fl);
}

// The SiLU epilogue (both output paths): its values already sit a few ulp from the oracle's
// (approximate exponential and reciprocal), so the combination contracts:
// v = (fh + fl / 254) * (rs * ws) + bias, then v / (1 + e^-v).
__device__ __forceinline__ float silu_value(float fh, float fl, float rs, float ws, float bias) {
    const float x = __fmaf_rn(__fmaf_rn(fl, 1.0f / 254.0f, fh), __fmul_rn(rs, ws), bias);
    return mul_sigmoid(x, x);
}

// Step for step what oracle_epilogue_x2 computes, with no contraction into FMA, except under
// SiLU (silu_value above). A missing bias is passed as 0, which leaves every value unchanged (the
// sums are never -0). The conversion unit does the two int-to-float conversions, except under
// SiLU, whose exponential and reciprocal already take two of its slots per value; there the
// integer path above converts the low sum.
template <int ACT>
__device__ __forceinline__ float epilogue_value(uint32_t acc_hi, uint32_t acc_lo, float rs, float ws,
                                                float bias, float scale) {
    const float inv254 = 1.0f / 254.0f;
    const float fh = __int2float_rn(static_cast<int32_t>(acc_hi));
    if (ACT == kActSilu) return __fmul_rn(silu_value(fh, exact_i2f(acc_lo), rs, ws, bias), scale);
    const float fl = __int2float_rn(static_cast<int32_t>(acc_lo));
    float v = __fadd_rn(fh, __fmul_rn(fl, inv254));
    v = __fmul_rn(v, rs);
    v = __fmul_rn(v, ws);
    v = __fadd_rn(v, bias);
    if (ACT == kActRelu) v = fmaxf(v, 0.0f);
    return __fmul_rn(v, scale);
}

// One chunk of one thread's output column (kRows rows): the values computed branch-free, then
// stored (rows_valid of them, each warp store covering 32 consecutive features of one row).
template <int ACT, bool ACC, typename OutT>
__device__ __forceinline__ void store_chunk(const uint32_t (&hi)[kRows], const uint32_t (&lo)[kRows], float my_rs,
                                            float ws, float bs, float scale, OutT* o, int64_t ldc,
                                            int rows_valid, bool n_ok) {
    float v[kRows];
#pragma unroll
    for (int j = 0; j < kRows; ++j)
        v[j] = epilogue_value<ACT>(hi[j], lo[j], __shfl_sync(0xffffffffu, my_rs, j), ws, bs, scale);
    if (!n_ok) return;
    if (rows_valid == kRows) {
        if (ACC) {
            float old[kRows];
#pragma unroll
            for (int j = 0; j < kRows; ++j) old[j] = static_cast<float>(o[j * ldc]);
#pragma unroll
            for (int j = 0; j < kRows; ++j) v[j] = __fadd_rn(old[j], v[j]);
        }
#pragma unroll
        for (int j = 0; j < kRows; ++j) o[j * ldc] = static_cast<OutT>(v[j]);
    } else {
#pragma unroll
        for (int j = 0; j < kRows; ++j)
            if (j < rows_valid) {
                float x = v[j];
                if (ACC) x = __fadd_rn(static_cast<float>(o[j * ldc]), x);
                o[j * ldc] = static_cast<OutT>(x);
            }
    }
}

// The epilogue of a staged chunk, step for step as epilogue_value (except under SiLU, below):
// v = ((float)hi + (float)lo * (1/254)) * rs * ws [+ bias] [act] [* scale], the chunk's kRows
// row scales in registers. A bias of 0 and a scale of 1 change no value and are skipped.
template <int ACT, bool BIAS, bool SCALE>
__device__ __forceinline__ void compute_chunk2(const uint32_t (&hi)[kRows], const uint32_t (&lo)[kRows],
                                               const float (&rs)[kRows], float ws, float bs, float scale,
                                               float (&v)[kRows]) {
    const float inv254 = 1.0f / 254.0f;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        const float fh = __int2float_rn(static_cast<int32_t>(hi[j]));
        float x;
        if (ACT == kActSilu) {
            x = silu_value(fh, exact_i2f(lo[j]), rs[j], ws, BIAS ? bs : 0.0f);
        } else {
            const float fl = __int2float_rn(static_cast<int32_t>(lo[j]));
            x = __fadd_rn(fh, __fmul_rn(fl, inv254));
            x = __fmul_rn(__fmul_rn(x, rs[j]), ws);
            if (BIAS) x = __fadd_rn(x, bs);
        }
        if (ACT == kActRelu) x = fmaxf(x, 0.0f);
        if (SCALE) x = __fmul_rn(x, scale);
        v[j] = x;
    }
}

template <int ACT>
__device__ __forceinline__ void compute_chunk_act(bool bias, bool scale_on, const uint32_t (&hi)[kRows],
                                                  const uint32_t (&lo)[kRows], const float (&rs)[kRows], float ws,
                                                  float bs, float scale, float (&v)[kRows]) {
    if (bias) {
        if (scale_on) compute_chunk2<ACT, true, true>(hi, lo, rs, ws, bs, scale, v);
        else compute_chunk2<ACT, true, false>(hi, lo, rs, ws, bs, scale, v);
    } else {
        if (scale_on) compute_chunk2<ACT, false, true>(hi, lo, rs, ws, bs, scale, v);
        else compute_chunk2<ACT, false, false>(hi, lo, rs, ws, bs, scale, v);
    }
}

__device__ __forceinline__ void compute_chunk_any(int act, bool bias, bool scale_on, const uint32_t (&hi)[kRows],
                                                  const uint32_t (&lo)[kRows], const float (&rs)[kRows], float ws,
                                                  float bs, float scale, float (&v)[kRows]) {
    if (act == kActNone) compute_chunk_act<kActNone>(bias, scale_on, hi, lo, rs, ws, bs, scale, v);
    else if (act == kActRelu) compute_chunk_act<kActRelu>(bias, scale_on, hi, lo, rs, ws, bs, scale, v);
    else compute_chunk_act<kActSilu>(bias, scale_on, hi, lo, rs, ws, bs, scale, v);
}

template <typename OutT>
__device__ __forceinline__ void store_chunk_any(int act, bool acc, const uint32_t (&hi)[kRows],
                                                const uint32_t (&lo)[kRows], float my_rs, float ws, float bs,
                                                float scale, OutT* o, int64_t ldc, int rows_valid, bool n_ok) {
    if (act == kActNone) {
        if (acc) store_chunk<kActNone, true>(hi, lo, my_rs, ws, bs, scale, o, ldc, rows_valid, n_ok);
        else store_chunk<kActNone, false>(hi, lo, my_rs, ws, bs, scale, o, ldc, rows_valid, n_ok);
    } else if (act == kActRelu) {
        if (acc) store_chunk<kActRelu, true>(hi, lo, my_rs, ws, bs, scale, o, ldc, rows_valid, n_ok);
        else store_chunk<kActRelu, false>(hi, lo, my_rs, ws, bs, scale, o, ldc, rows_valid, n_ok);
    } else {
        if (acc) store_chunk<kActSilu, true>(hi, lo, my_rs, ws, bs, scale, o, ldc, rows_valid, n_ok);
        else store_chunk<kActSilu, false>(hi, lo, my_rs, ws, bs, scale, o, ldc, rows_valid, n_ok);
    }
}

template <int CG, bool WL>
__global__ void __launch_bounds__(kThreads, 1)
gemm_i8x2_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_hi,
                 const __grid_constant__ CUtensorMap map_lo, const __grid_constant__ CUtensorMap map_out,
                 const __grid_constant__ CUtensorMap map_out_lo, const __grid_constant__ CUtensorMap map_wl,
                 const Params p) {
    static_assert(!WL || CG == 1, "two-level weights run on single CTAs");
    constexpr int kStages = Shape<CG, WL>::kStages;
    constexpr int kStageBytes = Shape<CG, WL>::kStageBytes;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + kStages * kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + kOutStaging);
    uint64_t* empty = full + kStages;
    uint64_t* tmem_full = empty + kStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // A tile is BM activation rows x CG * BN features; CTA rank r of a pair owns features
    // n0 + r * BN ...; tiles run over "units" (single CTAs or pairs).
    const uint32_t rank = CG == 2 ? cluster_rank() : 0;
    const bool leader = rank == 0;
    const int unit = blockIdx.x / CG, units = gridDim.x / CG;
    const int num_m = (p.m + BM - 1) / BM, num_n = (p.n + CG * BN - 1) / (CG * BN);
    const int tiles = num_m * num_n;
    const int kblocks = (p.k + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            // CG = 1: every epilogue thread arrives; CG = 2: one lane per epilogue warp of both
            // CTAs arrives on the pair's first CTA's barrier.
            mbar_init(&tmem_empty[b], CG == 1 ? kEpiWarps * 32 : 2 * kEpiWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&map_w);
        prefetch_tensormap(&map_hi);
        prefetch_tensormap(&map_lo);
        if (WL) prefetch_tensormap(&map_wl);
        if (p.out_path != kDirect) prefetch_tensormap(&map_out);
        if (p.out_path != kDirect && p.out_kind == kOutF16Split) prefetch_tensormap(&map_out_lo);
    }
    if (warp == 1) {
        if (CG == 1) {
            tmem_alloc(tmem_base_slot, kTmemCols);
            tmem_relinquish();
        } else {
            tmem_alloc_pair(tmem_base_slot, kTmemCols);
            tmem_relinquish_pair();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (CG == 2) cluster_sync();  // both CTAs' barriers exist before either signals the other's
    tc_fence_after();
    const uint32_t tmem_base = *tmem_base_slot;

    // Tiles run activation-block-major: the CTAs working at the same time share a block of
    // activation rows (read from DRAM once, then served by L2) and sweep the features, whose
    // weights (at most a few MB) stay in L2 for the whole product.
    if (warp == 0) {
        // ---- TMA producer ------------------------------------------------------------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int t = unit; t < tiles && !*abort_flag; t += units) {
                const int m0 = (t / num_n) * BM, n0 = (t % num_n) * CG * BN + static_cast<int>(rank) * BN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) {
                        record_error(p.error, kErrWaitTimeout);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t* st = smem + stage * kStageBytes;
                    if (CG == 1) {
                        mbar_arrive_expect_tx(&full[stage], kStageBytes);
                        tma_load_2d(&map_w, &full[stage], st, kb * BK, n0);
                        tma_load_2d(&map_hi, &full[stage], st + kTileBytes, kb * BK, m0);
                        tma_load_2d(&map_lo, &full[stage], st + 2 * kTileBytes, kb * BK, m0);
                        if (WL) tma_load_2d(&map_wl, &full[stage], st + 3 * kTileBytes, kb * BK, n0);
                    } else {
                        // Both CTAs' loads count on the first CTA's barrier, which expects them all.
                        // The first CTA stages the high level (B columns 0..127), the second the low.
                        const uint32_t bar = cluster_addr(&full[stage], 0);
                        if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kStageBytes);
                        tma_load_2d_pair(&map_w, bar, st, kb * BK, n0);
                        tma_load_2d_pair(leader ? &map_hi : &map_lo, bar, st + kTileBytes, kb * BK, m0);
                    }
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer (the pair's first CTA issues for both) -----------------------------
        constexpr uint32_t idesc = idesc_i8(CG * 128, 2 * BM);
        constexpr uint32_t idesc_wl = idesc_i8(128, BM);  // W_lo x the high level only
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        const uint32_t peer_empty0 = CG == 2 ? cluster_addr(&empty[0], 1) : 0;
        const uint32_t peer_tfull0 = CG == 2 ? cluster_addr(&tmem_full[0], 1) : 0;
        for (int t = unit; leader && t < tiles && !*abort_flag; t += units, ++it) {
            const int buf = it & 1;
            const uint32_t use = static_cast<uint32_t>(it >> 1);
            if (!mbar_wait(&tmem_empty[buf], (use & 1) ^ 1)) {
                record_error(p.error, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + static_cast<uint32_t>(buf * 2 * BM);
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t w = smem_u32(smem + stage * kStageBytes);
                    const uint32_t x = w + kTileBytes;  // hi rows, then lo rows: N = 256
                    const uint32_t wl = w + 3 * kTileBytes;
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        if (CG == 1) mma_i8(d, sw128_desc(w + kk * UMMA_K), sw128_desc(x + kk * UMMA_K), idesc, acc);
                        else mma_i8_pair(d, sw128_desc(w + kk * UMMA_K), sw128_desc(x + kk * UMMA_K), idesc, acc);
                        // Two-level weights: W_lo . A_hi joins A_lo . W into the low sums (both
                        // carry the 1/254 step); A_lo . W_lo (1/254^2) is left out.
                        if (WL)
                            mma_i8(d + BM, sw128_desc(wl + kk * UMMA_K), sw128_desc(x + kk * UMMA_K), idesc_wl, 1u);
                    }
                    if (CG == 1) {
                        mma_commit(&empty[stage]);
                    } else {
                        mma_commit_pair(smem_u32(&empty[stage]));
                        mma_commit_pair(peer_empty0 + static_cast<uint32_t>(stage * sizeof(uint64_t)));
                    }
                }
                __syncwarp();
                if (++stage == kStages) { stage = 0; phase ^= 1; }
            }
            if (!ok) {
                record_error(p.error, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            if (lane == 0) {
                if (CG == 1) {
                    mma_commit(&tmem_full[buf]);
                } else {
                    mma_commit_pair(smem_u32(&tmem_full[buf]));
                    mma_commit_pair(peer_tfull0 + static_cast<uint32_t>(buf * sizeof(uint64_t)));
                }
            }
            __syncwarp();
        }
    } else {
        // ---- epilogue (warps 2..17): thread = one output feature, kRows rows per TMEM load; the
        // four warps of a TMEM lane quarter take a quarter of the tile's activation rows each ----
        constexpr int kChunks = BM / (4 * kRows);  // chunks per warp per tile
        const int quad = warp & 3;  // TMEM lanes this warp may access: 32 * quad ..
        const int part = (warp - 2) / 4;
        const bool has_bias = p.bias != nullptr;
        const bool scale_on = p.scale != 1.0f;
        const bool rs_vec = (reinterpret_cast<uintptr_t>(p.row_scale) & 15) == 0;
        uint8_t* sbuf = staging + (warp - 2) * kStageOutBytes;
        int it = 0;
        const uint32_t tempty0 = CG == 2 ? cluster_addr(&tmem_empty[0], 0) : 0;
        for (int t = unit; t < tiles && !*abort_flag; t += units, ++it) {
            const int buf = it & 1;
            const uint32_t use = static_cast<uint32_t>(it >> 1);
            const int m0 = (t / num_n) * BM, n0 = (t % num_n) * CG * BN + static_cast<int>(rank) * BN;
            const int n = n0 + quad * 32 + lane;
            const bool n_ok = n < p.n;
            const float ws = n_ok ? __ldg(p.w_scale + n) : 0.0f;
            const float bs = (has_bias && n_ok) ? __ldg(p.bias + n) : 0.0f;
            // The row scales of this warp's rows into L1 while the tile's products finish (the
            // first and last row of each chunk, in case the scales are not 128-byte aligned), so
            // the loads below hit L1 instead of waiting on L2 after the TMEM load.
            if (lane < 2 * kChunks) {
                const int mc = m0 + (part * kChunks + lane / 2) * kRows + (lane & 1) * (kRows - 1);
                if (mc < p.m) prefetch_l1(p.row_scale + mc);
            }
            if (!mbar_wait(&tmem_full[buf], use & 1)) {
                record_error(p.error, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                   static_cast<uint32_t>(buf * 2 * BM);
#pragma unroll 1
            for (int c = part * kChunks; c < (part + 1) * kChunks; ++c) {
                uint32_t hi[kRows], lo[kRows];
                tmem_ld16(taddr + c * kRows, hi);
                tmem_ld16(taddr + BM + c * kRows, lo);
                tmem_ld_wait();
                const int mc = m0 + c * kRows;
                if (mc >= p.m) continue;
                const float my_rs = (lane < kRows && mc + lane < p.m) ? __ldg(p.row_scale + mc + lane) : 0.0f;
                const int rows_valid = p.m - mc < kRows ? p.m - mc : kRows;
                // The chunk's row scales in registers: broadcast 16-byte loads for a full, aligned
                // chunk, else shuffles of the lanes' own loads.
                float rs[kRows];
                if (rows_valid == kRows && rs_vec) {
                    const float4* r4 = reinterpret_cast<const float4*>(p.row_scale + mc);
#pragma unroll
                    for (int q4 = 0; q4 < kRows / 4; ++q4) {
                        const float4 t4 = __ldg(r4 + q4);
                        rs[4 * q4] = t4.x;
                        rs[4 * q4 + 1] = t4.y;
                        rs[4 * q4 + 2] = t4.z;
                        rs[4 * q4 + 3] = t4.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < kRows; ++j) rs[j] = __shfl_sync(0xffffffffu, my_rs, j);
                }
                const int64_t off = static_cast<int64_t>(mc) * p.ldc + n;
                if (p.out_path != kDirect) {
                    // Stage the kRows x 32 chunk (row = activation row, column = feature) and let
                    // one lane hand it to TMA; the previous chunk's store has read the buffer by
                    // the time this chunk's values are computed, almost always.
                    float v[kRows];
                    compute_chunk_any(p.act, has_bias, scale_on, hi, lo, rs, ws, bs, p.scale, v);
                    if (lane == 0) bulk_wait_read<0>();
                    __syncwarp();
                    if (p.out_kind == kOutF32) {
                        float* sf = reinterpret_cast<float*>(sbuf);
#pragma unroll
                        for (int j = 0; j < kRows; ++j) sf[j * 32 + lane] = v[j];
                    } else if (p.out_kind == kOutF16Split) {
                        __half* sh = reinterpret_cast<__half*>(sbuf);
                        __half* sl = sh + kRows * 32;
#pragma unroll
                        for (int j = 0; j < kRows; ++j) {
                            const __half h = __float2half_rn(v[j]);
                            sh[j * 32 + lane] = h;
                            sl[j * 32 + lane] = __float2half_rn(__fsub_rn(v[j], __half2float(h)));
                        }
                    } else {
                        __nv_bfloat16* sb = reinterpret_cast<__nv_bfloat16*>(sbuf);
#pragma unroll
                        for (int j = 0; j < kRows; ++j) sb[j * 32 + lane] = __float2bfloat16_rn(v[j]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    const int x0 = n0 + quad * 32;
                    if (lane == 0 && x0 < p.n) {
                        if (p.out_path == kTmaReduce) tma_reduce_add_2d(&map_out, sbuf, x0, mc);
                        else tma_store_2d(&map_out, sbuf, x0, mc);
                        if (p.out_kind == kOutF16Split) tma_store_2d(&map_out_lo, sbuf + kRows * 32 * 2, x0, mc);
                        bulk_commit();
                    }
                } else if (p.out_kind == kOutF16Split) {
                    float v[kRows];
                    compute_chunk_any(p.act, has_bias, scale_on, hi, lo, rs, ws, bs, p.scale, v);
                    __half* oh = static_cast<__half*>(p.out) + off;
                    __half* ol = oh + static_cast<int64_t>(p.m) * p.ldc;
#pragma unroll
                    for (int j = 0; j < kRows; ++j)
                        if (j < rows_valid && n_ok) {
                            const __half h = __float2half_rn(v[j]);
                            oh[j * p.ldc] = h;
                            ol[j * p.ldc] = __float2half_rn(__fsub_rn(v[j], __half2float(h)));
                        }
                } else if (p.out_kind == kOutF32) {
                    store_chunk_any(p.act, p.accumulate != 0, hi, lo, my_rs, ws, bs, p.scale,
                                    static_cast<float*>(p.out) + off, p.ldc, rows_valid, n_ok);
                } else if (p.out_kind == kOutBF16) {
                    store_chunk_any(p.act, p.accumulate != 0, hi, lo, my_rs, ws, bs, p.scale,
                                    static_cast<__nv_bfloat16*>(p.out) + off, p.ldc, rows_valid, n_ok);
                } else {
                    int32_t* o_hi = static_cast<int32_t*>(p.out) + static_cast<int64_t>(mc) * p.ldc + n;
                    int32_t* o_lo = o_hi + static_cast<int64_t>(p.m) * p.ldc;
#pragma unroll
                    for (int j = 0; j < kRows; ++j) {
                        if (mc + j < p.m && n_ok) {
                            o_hi[j * p.ldc] = static_cast<int32_t>(hi[j]);
                            o_lo[j * p.ldc] = static_cast<int32_t>(lo[j]);
                        }
                    }
                }
            }
            tc_fence_before();
            if (CG == 1) {
                mbar_arrive(&tmem_empty[buf]);
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(tempty0 + static_cast<uint32_t>(buf * sizeof(uint64_t)));
            }
        }
        if (lane == 0) bulk_wait<0>();
    }

    tc_fence_before();
    __syncthreads();
    // A pair's CTAs leave together: the first CTA's MMAs read the second's shared memory and
    // write its TMEM, and the second's loads signal the first's barriers.
    if (CG == 2) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if (CG == 1) tmem_dealloc(tmem_base, kTmemCols);
        else tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

}  // namespace

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

bool encode_map_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

// A 2-D int8 tensor map over rows of `cols` bytes, `ld` bytes apart, boxes of 128 bytes x 128
// rows with the 128-byte swizzle. Reads past `cols` or `rows` fill zeros.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), 128};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// The output tensor map: m rows of n elements, ldc apart, boxes of 32 elements x kRows rows
// without swizzle. Each
// plane of the split output gets its own map, so TMA drops the rows of a partial chunk past m
// instead of writing them into the other plane.
bool make_out_map(CUtensorMap* map, void* base, int kind, int m, int n, int64_t ldc) {
    auto fn = encode_fn();
    if (!fn) return false;
    const bool two = kind == kOutBF16 || kind == kOutF16Split;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldc) * (two ? 2 : 4)};
    cuuint32_t box[2] = {32, static_cast<cuuint32_t>(kRows)};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType type = kind == kOutBF16        ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : kind == kOutF16Split ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    CUresult r = fn(map, type, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

int num_sms() {
    static std::atomic<int> sms{0};
    int n = sms.load(std::memory_order_relaxed);
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
        sms.store(n, std::memory_order_relaxed);
    }
    return n;
}

cudaError_t gemm_i8x2(const GemmArgs& g, cudaStream_t stream) {
    if (g.m <= 0 || !g.w || g.w->n <= 0) return cudaSuccess;
    if ((g.a.ld % 16) || (g.w->ld % 16)) return cudaErrorInvalidValue;
    const DevWeights& w = *g.w;
    CUtensorMap mw, mh, ml, mwl;
    if (!make_map(&mw, w.values, w.n, w.k, w.ld) || !make_map(&mh, g.a.hi, g.m, w.k, g.a.ld) ||
        !make_map(&ml, g.a.lo, g.m, w.k, g.a.ld))
        return cudaErrorInvalidValue;
    const bool two_level = w.lo_values != nullptr;
    if (two_level ? !make_map(&mwl, w.lo_values, w.n, w.k, w.ld) : false) return cudaErrorInvalidValue;
    if (!two_level) mwl = mw;  // not read
    static DeviceOnce configured;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured.done(dev)) {
        cudaError_t e = cudaFuncSetAttribute(gemm_i8x2_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Shape<1>::kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_i8x2_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Shape<2>::kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_i8x2_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Shape<1, true>::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured.mark(dev);
    }
    // The output goes through TMA when its rows are 16-byte aligned.
    CUtensorMap mo, mo_lo;
    memset(&mo, 0, sizeof mo);
    memset(&mo_lo, 0, sizeof mo_lo);
    int path = kDirect;
    const size_t esize = (g.out_kind == kOutBF16 || g.out_kind == kOutF16Split) ? 2 : 4;
    const bool aligned = (reinterpret_cast<uintptr_t>(g.out) % 16 == 0) && ((g.ldc * esize) % 16 == 0);
    if (aligned && g.out_kind == kOutF32) path = g.accumulate ? kTmaReduce : kTmaStore;
    if (aligned && (g.out_kind == kOutBF16 || g.out_kind == kOutF16Split) && !g.accumulate) path = kTmaStore;
    if (g.out_kind == kOutF16Split && g.accumulate) return cudaErrorInvalidValue;
    if (path != kDirect && !make_out_map(&mo, g.out, g.out_kind, g.m, w.n, g.ldc)) path = kDirect;
    if (path != kDirect && g.out_kind == kOutF16Split &&
        !make_out_map(&mo_lo, static_cast<__half*>(g.out) + static_cast<int64_t>(g.m) * g.ldc, g.out_kind, g.m, w.n,
                      g.ldc))
        path = kDirect;
    Params p{g.m, w.n, w.k, g.a.scale, w.scales, g.bias, g.act, g.scale, g.accumulate,
             g.out, g.ldc, g.out_kind, path, g.error};
    // Products of at least 256 features run on CTA pairs (each MMA spans both SMs' tensor
    // cores; each CTA stages a third less per multiply-add), narrower ones on single CTAs.
    if (w.n >= 2 * BN && !two_level) {
        const int tiles = ((g.m + BM - 1) / BM) * ((w.n + 2 * BN - 1) / (2 * BN));
        const int pairs = std::min(tiles, num_sms() / 2);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * pairs);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = Shape<2>::kSmemBytes;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_i8x2_kernel<2, false>, mw, mh, ml, mo, mo_lo, mwl, p);
        if (e != cudaSuccess) return e;
        return cudaGetLastError();
    }
    const int tiles = ((g.m + BM - 1) / BM) * ((w.n + BN - 1) / BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    if (two_level)
        gemm_i8x2_kernel<1, true><<<grid, kThreads, Shape<1, true>::kSmemBytes, stream>>>(mw, mh, ml, mo, mo_lo, mwl, p);
    else
        gemm_i8x2_kernel<1, false><<<grid, kThreads, Shape<1>::kSmemBytes, stream>>>(mw, mh, ml, mo, mo_lo, mwl, p);
    return cudaGetLastError();
}

}  // namespace telmo
