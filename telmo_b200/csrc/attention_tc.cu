// attention_tc.cu -- Granite's block-local attention with Shaw relative positions
// (Granite::attention, src/granite.rs:965-1036) on the tcgen05 tensor cores.
//
// Per (attention block, head), with the block's len <= 128 query rows and keys:
//   pos = Q . Rel^T over the 255 relative positions, times each position's scale
//   S   = Q . K^T,   S[i][j] = scale * S[i][j] + scale * pos[i][ctx - 1 - i + j]
//   P   = softmax(S) per row over the len keys (f32 exponentials, f64 sum, as the reference)
//   O   = P . V
// Q, K and V arrive as fp16 high/low planes (x = hi + lo, the QKV product's split epilogue), the
// relative table as fp16 (its int8 values are exact) with one f32 scale per position. Every
// product is a kind::f16 tcgen05.mma (M = 128 query rows) accumulating in TMEM: pos as
// Q_hi.Rel + Q_lo.Rel (N = 256 positions), S and O as hi.hi + hi.lo + lo.hi, which keeps about 21
// bits of each operand, so the sums match the reference's f32 sums to about 1e-6 relative.
//
// Structure: a persistent, warp-specialised kernel, one CTA per SM, one (block, head) at a time.
//   warp 0      TMA producer: Q and K as soon as the previous S and position products no longer
//               read their buffers (so they load during the previous softmax), the relative
//               table once the previous O product is done with V, V once the position product is
//               done with the table (V takes the table's buffer)
//   warp 1      MMA issuer: S, then pos (which waits for the previous O product: P lives in pos's
//               columns), then O once P is in TMEM
//   warps 2-9   softmax and output, two warps per TMEM lane quarter (warp w reads lanes
//               32 (w % 4) ..), each on half of a query row's keys: S and a 64-column span of
//               the positions from TMEM, the row's own 32 positions brought to the front of the
//               registers by a five-stage shift on the bits of 31 - lane (a row's positions start
//               at a column that differs per lane, which one TMEM load cannot address), the row
//               maximum and sum across the pair through shared memory,
//               P split to fp16 planes into TMEM (the O product's A operand), then O to global
//               memory.
// TMEM: S in columns 0..127, pos in 128..383 (then P: hi 128..191, lo 192..255), O in 384..511;
// the next task's S product runs while this task's O is read out. Partial blocks (len < 128)
// issue only the key and position columns they use, and blocks of at most 64 rows load only
// those rows. Every wait is bounded; on timeout the
// kernel records kErrWaitTimeout in the error word and returns.
#include "attention_tc.cuh"
#include "kernels.h"
#include "ptx.cuh"
#include "rowops.h"
#include "tma.h"

#include <cuda_fp16.h>

#include <algorithm>

namespace telmo {

namespace {

constexpr int T = 128;    // query rows and keys per block (Granite's context)
constexpr int HD = 128;   // head size
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
using namespace tc_attention;
constexpr int kRelHalf = 2 * kBox;           // 256 positions x 64 fp16
constexpr uint32_t kColS = 0, kColPos = 128, kColP = 128, kColO = 384, kTmemCols = 512;
constexpr int kSmemBytes = 3 * kOperand + 256 * 4 + 2 * 2 * 128 * 8 + 128 + 1024;

struct Bars {
    uint64_t q_full, k_full, r_full, v_full, s_done, p_full, o_done, o_free;
};

__global__ void __launch_bounds__(kThreads, 1)
granite_attention_tc_kernel(const __grid_constant__ CUtensorMap map_qkv, const __grid_constant__ CUtensorMap map_qkv64,
                            const __grid_constant__ CUtensorMap map_rel,
                            int rows, int heads, const AttnTask* __restrict__ tasks, int n_tasks,
                            const float* __restrict__ rel_scale, int positions, float scale, float* __restrict__ att,
                            uint32_t* error) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* buf_q = smem;                 // Q
    uint8_t* buf_k = smem + kOperand;      // K
    uint8_t* buf_r = smem + 2 * kOperand;  // the relative table, then V
    float* rs = reinterpret_cast<float*>(smem + 3 * kOperand);
    float* red_max = rs + 256;                                   // [2 halves][128 rows]
    double* red_sum = reinterpret_cast<double*>(red_max + 256);  // [2 halves][128 rows]
    Bars* bars = reinterpret_cast<Bars*>(red_sum + 256);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int D = heads * HD;
    const int total = n_tasks * heads;

    // Each position's scale times the score scale: the position term of a score is pos * rs[p].
    for (int p = threadIdx.x; p < 256; p += kThreads) rs[p] = p < positions ? __fmul_rn(__ldg(rel_scale + p), scale) : 0.0f;
    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        mbar_init(&bars->k_full, 1);
        mbar_init(&bars->r_full, 1);
        mbar_init(&bars->v_full, 1);
        mbar_init(&bars->s_done, 1);
        mbar_init(&bars->p_full, 32 * kEpiWarps);
        mbar_init(&bars->o_done, 1);
        mbar_init(&bars->o_free, 32 * kEpiWarps);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&map_qkv);
        prefetch_tensormap(&map_qkv64);
        prefetch_tensormap(&map_rel);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&]() {
        record_error(error, kErrWaitTimeout);
        *abort_flag = 1;
    };

    if (warp == 0) {
        // ---- TMA producer ------------------------------------------------------------------
        if (lane == 0) {
            int it = 0;
            for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x, ++it) {
                const AttnTask tk = tasks[w / heads];
                const int h = w % heads;
                const int y_hi = tk.row, y_lo = rows + tk.row;
                const uint32_t prev = (it - 1) & 1;
                // A block of at most 64 rows loads 64-row boxes (the first half of each slot): the
                // products never read its rows past 64 (S and O stop at 16 * ceil(len / 16) keys;
                // query rows past len are not stored).
                const bool short_block = tk.len <= 64;
                const CUtensorMap* mq = short_block ? &map_qkv64 : &map_qkv;
                const uint32_t bytes = short_block ? kOperand / 2 : kOperand;
                // Q and K: the previous S and position products (one commit) are done with their
                // buffers, so both load while the previous softmax runs.
                if (it > 0 && !mbar_wait(&bars->s_done, prev)) { fail(); break; }
                mbar_arrive_expect_tx(&bars->q_full, bytes);
                load_operand(mq, &bars->q_full, buf_q, h * HD, y_hi, y_lo);
                mbar_arrive_expect_tx(&bars->k_full, bytes);
                load_operand(mq, &bars->k_full, buf_k, D + h * HD, y_hi, y_lo);
                // The relative table: the previous O product is done with V in the table's buffer.
                if (it > 0 && !mbar_wait(&bars->o_done, prev)) { fail(); break; }
                mbar_arrive_expect_tx(&bars->r_full, 2 * kRelHalf);
                tma_load_2d(&map_rel, &bars->r_full, buf_r, 0, 0);
                tma_load_2d(&map_rel, &bars->r_full, buf_r + kRelHalf, 64, 0);
                // V: this task's position product is done with the table.
                if (!mbar_wait(&bars->s_done, it & 1)) { fail(); break; }
                mbar_arrive_expect_tx(&bars->v_full, bytes);
                load_operand(mq, &bars->v_full, buf_r, 2 * D + h * HD, y_hi, y_lo);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----------------------------------------------------------------------
        const uint32_t q = smem_u32(buf_q), k = smem_u32(buf_k), r = smem_u32(buf_r);
        int it = 0;
        for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x, ++it) {
            const int len = tasks[w / heads].len;
            const int n16 = (len + 15) & ~15;                       // key columns in use
            const int npos = min(256, (T - 1 + len + 15) & ~15);    // positions 0 .. 126 + len
            const uint32_t prev = (it - 1) & 1;
            // S: Q and K are in, and the previous softmax has read S.
            bool ok = mbar_wait(&bars->q_full, it & 1) && mbar_wait(&bars->k_full, it & 1) &&
                      (it == 0 || mbar_wait(&bars->p_full, prev));
            if (!ok) { fail(); break; }
            tc_fence_after();
            if (lane == 0) {
                const uint32_t id_s = idesc_f16(128, n16, false);
#pragma unroll
                for (int ks = 0; ks < HD / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * kBox + (ks & 3) * 32;
                    mma_f16(tmem + kColS, sw128_desc(q + off), sw128_desc(k + off), id_s, ks > 0);
                    mma_f16(tmem + kColS, sw128_desc(q + off), sw128_desc(k + 2 * kBox + off), id_s, 1u);
                    mma_f16(tmem + kColS, sw128_desc(q + 2 * kBox + off), sw128_desc(k + off), id_s, 1u);
                }
            }
            __syncwarp();
            // pos: the table is in, and the previous O product is done with P in pos's columns.
            ok = mbar_wait(&bars->r_full, it & 1) && (it == 0 || mbar_wait(&bars->o_done, prev));
            if (!ok) { fail(); break; }
            tc_fence_after();
            if (lane == 0) {
                const uint32_t id_pos = idesc_f16(128, npos, false);
#pragma unroll
                for (int ks = 0; ks < HD / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * kBox + (ks & 3) * 32;
                    const uint32_t roff = (ks >> 2) * kRelHalf + (ks & 3) * 32;
                    mma_f16(tmem + kColPos, sw128_desc(q + off), sw128_desc(r + roff), id_pos, ks > 0);
                    mma_f16(tmem + kColPos, sw128_desc(q + 2 * kBox + off), sw128_desc(r + roff), id_pos, 1u);
                }
                mma_commit(&bars->s_done);
            }
            __syncwarp();
            // O: P is in TMEM, V is in, and the previous O has been read out.
            ok = mbar_wait(&bars->p_full, it & 1) && mbar_wait(&bars->v_full, it & 1) &&
                 (it == 0 || mbar_wait(&bars->o_free, prev));
            if (!ok) { fail(); break; }
            tc_fence_after();
            if (lane == 0) {
                constexpr uint32_t id_o = idesc_f16(128, HD, true);
                for (int ks = 0; ks < n16 / 16; ++ks) {
                    const uint32_t voff = ks * 2048;  // 16 keys = two 8-row groups of 128 bytes
                    const uint32_t ph = tmem + kColP + ks * 8, pl = ph + 64;  // 16 keys = 8 columns
                    mma_f16_ts(tmem + kColO, ph, sw128_desc_mn(r + voff, kBox), id_o, ks > 0);
                    mma_f16_ts(tmem + kColO, ph, sw128_desc_mn(r + 2 * kBox + voff, kBox), id_o, 1u);
                    mma_f16_ts(tmem + kColO, pl, sw128_desc_mn(r + voff, kBox), id_o, 1u);
                }
                mma_commit(&bars->o_done);
            }
            __syncwarp();
        }
    } else {
        // ---- softmax and output (warps 2..9): thread = query row 32 (warp % 4) + lane, keys
        // 64 half .. 64 half + 63 -----------------------------------------------------------------
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lanes = tmem + (static_cast<uint32_t>(quad * 32) << 16);
        const int sh = 31 - lane;  // where this lane's positions start in its warp's span
        int it = 0;
        for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x, ++it) {
            const AttnTask tk = tasks[w / heads];
            const int h = w % heads;
            const int len = tk.len;
            if (!mbar_wait(&bars->s_done, it & 1)) { fail(); break; }
            tc_fence_after();
            float lg[64];
            float mx = -INFINITY;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c = 2 * half + cc;
                // Keys 32c .. 32c + 31 of row i read positions 127 - i + 32c + j: for this warp's rows
                // the columns 96 - 32 quad + 32c .. + 63 hold them all; lane l's 32 start at element
                // 31 - l of that span, brought to the front of the lane's registers by shifts of
                // 16, 8, 4, 2 and 1 on the bits of 31 - l (each stage keeps what the later ones
                // can still reach).
                uint32_t p0[32], p1[32], pw[64];
                tmem_ld32(lanes + kColPos + 96 - 32 * quad + 32 * c, p0);
                tmem_ld32(lanes + kColPos + 128 - 32 * quad + 32 * c, p1);
                tmem_ld_wait();
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    pw[k] = p0[k];
                    pw[32 + k] = p1[k];
                }
                shift_down<47, 16>(pw, (sh & 16) != 0);
                shift_down<39, 8>(pw, (sh & 8) != 0);
                shift_down<35, 4>(pw, (sh & 4) != 0);
                shift_down<33, 2>(pw, (sh & 2) != 0);
                shift_down<32, 1>(pw, (sh & 1) != 0);
                uint32_t sv[32];
                tmem_ld32(lanes + kColS + 32 * c, sv);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int key = 32 * c + j;
                    const float pos = __uint_as_float(pw[j]);
                    const float ps = rs[T - 1 - row + key];
                    float v = __fadd_rn(__fmul_rn(__uint_as_float(sv[j]), scale), __fmul_rn(pos, ps));
                    if (key >= len) v = -INFINITY;
                    lg[32 * cc + j] = v;
                    mx = fmaxf(mx, v);
                }
            }
            red_max[half * T + row] = mx;
            epi_sync<32 * kEpiWarps>();
            mx = fmaxf(red_max[row], red_max[T + row]);
            const float mxl = __fmul_rn(mx, kLog2e);
            // The row sum in f64 (as the reference) over f32 partial sums of 8 exponentials.
            double s0 = 0.0, s1 = 0.0;
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                float part = 0.0f;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    lg[8 * g + k] = ex2_approx(__fmaf_rn(lg[8 * g + k], kLog2e, -mxl));
                    part = __fadd_rn(part, lg[8 * g + k]);
                }
                if (g & 1) s1 += static_cast<double>(part);
                else s0 += static_cast<double>(part);
            }
            red_sum[half * T + row] = s0 + s1;
            epi_sync<32 * kEpiWarps>();
            const float inv = static_cast<float>(1.0 / (red_sum[row] + red_sum[T + row]));
            // P into TMEM (pos's first 128 columns) as the O product's A operand: fp16 pairs of
            // consecutive keys per column, hi plane in columns 0..63, lo plane in 64..127.
            uint32_t hv[32], lv[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const float p0 = __fmul_rn(lg[2 * e], inv), p1 = __fmul_rn(lg[2 * e + 1], inv);
                const float h0 = f16_high(p0), h1 = f16_high(p1);
                hv[e] = pack2(h0, h1);
                lv[e] = pack2(__fsub_rn(p0, h0), __fsub_rn(p1, h1));
            }
            tmem_st32(lanes + kColP + 32 * half, hv);
            tmem_st32(lanes + kColP + 64 + 32 * half, lv);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&bars->p_full);
            if (!mbar_wait(&bars->o_done, it & 1)) { fail(); break; }
            tc_fence_after();
            float* orow = att + static_cast<int64_t>(tk.row + row) * D + h * HD;
#pragma unroll
            for (int c = 2 * half; c < 2 * half + 2; ++c) {
                uint32_t ov[32];
                tmem_ld32(lanes + kColO + 32 * c, ov);
                tmem_ld_wait();
                if (row < len) {
#pragma unroll
                    for (int m = 0; m < 8; ++m)
                        *reinterpret_cast<float4*>(orow + 32 * c + 4 * m) =
                            make_float4(__uint_as_float(ov[4 * m]), __uint_as_float(ov[4 * m + 1]),
                                        __uint_as_float(ov[4 * m + 2]), __uint_as_float(ov[4 * m + 3]));
                }
            }
            tc_fence_before();
            mbar_arrive(&bars->o_free);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

DeviceOnce configured;

}  // namespace

bool granite_attention_tc_supported(int hd, int ctx) { return hd == HD && ctx == T; }

cudaError_t granite_attention_tc(const __half* qkv, int rows, int heads, int hd, int ctx, const AttnTask* tasks,
                                 int n_tasks, const __half* rel16, const float* rel_scale, float scale, float* att,
                                 uint32_t* error, cudaStream_t stream) {
    if (n_tasks <= 0) return cudaSuccess;
    if (!granite_attention_tc_supported(hd, ctx) || rows <= 0) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured.done(dev)) {
        const cudaError_t e =
            cudaFuncSetAttribute(granite_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        configured.mark(dev);
    }
    const int D = heads * HD;
    // The QKV product's two fp16 planes as one [2 rows, 3 D] tensor: hi rows 0.., lo rows rows...
    CUtensorMap mq, mq64, mr;
    if (!encode_map_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qkv, static_cast<uint64_t>(3 * D),
                       2 * static_cast<uint64_t>(rows), static_cast<uint64_t>(3 * D) * 2, 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_map_2d(&mq64, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qkv, static_cast<uint64_t>(3 * D),
                       2 * static_cast<uint64_t>(rows), static_cast<uint64_t>(3 * D) * 2, 64, 64,
                       CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_map_2d(&mr, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rel16, HD, static_cast<uint64_t>(2 * ctx - 1), HD * 2, 64,
                       256, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const int total = n_tasks * heads;
    const int grid = std::min(total, num_sms());
    granite_attention_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mq64, mr, rows, heads, tasks, n_tasks, rel_scale,
                                                                       2 * ctx - 1, scale, att, error);
    return cudaGetLastError();
}

}  // namespace telmo
