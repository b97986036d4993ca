// txl_attention_tc.cu -- Parakeet's Transformer-XL relative attention over whole utterances
// (Parakeet::attention, src/parakeet.rs:1176-1282) on the tcgen05 tensor cores.
//
// The reference scores query i against key j of an utterance of t frames as
//   ((q_i + u) . k_j + (q_i + v) . Pos[t - 1 - i + j]) * scale
// with u, v the layer's biases and Pos the projected sinusoid table, then takes the softmax over
// the t keys and P . V. Here the bias parts are per-key and per-position vectors computed once per
// layer (uk[j] = u . k_j, cv[p] = v . Pos[p]; txl_bias_terms), so the products read Q, K, V and
// Pos exactly as the QKV and position products' split epilogues wrote them (fp16 high/low planes).
//
// A task is 128 query rows of one utterance and one head; it walks the keys in chunks of 128.
// Per chunk, all kind::f16 tcgen05.mma with the accumulators in TMEM (M = 128 query rows):
//   BD = Q . Pos^T over the 256-row position window the chunk's (row, key) pairs reach, as two
//        N = 128 halves (the window row of query r and key j is 127 - r + j), hi.hi + hi.lo + lo.hi
//   S  = Q . K^T, N = the chunk's keys rounded up to 16, hi.hi + hi.lo + lo.hi
// then, one query row per thread pair (each thread half of the chunk's keys), the scores, an
// online softmax (running row maximum and sum in f32), the chunk's probabilities relative to the
// running maximum into TMEM as fp16 hi/lo planes, and O_chunk = P . V (A from TMEM, V MN-major
// from shared memory) accumulating in TMEM over the task's chunks; when a row's maximum grows,
// its thread rescales the row's output in TMEM before the next chunk's product adds to it. After
// the last chunk the output is read out and divided by the sum.
//
// Structure: persistent and warp-specialised, one CTA per SM.
//   warp 0      TMA producer: Q once per task; per chunk the first position half (once the
//               previous chunk's position products are done with the position buffer, so it
//               loads during the previous softmax), K (once the previous O
//               product is done with V, which shares K's buffer), the second position half
//               (once the first half's product is done), V (once the S product is done with K)
//   warp 1      MMA issuer: BD first half, S, BD second half, then O once P is in TMEM
//   warps 2-9   softmax and output: warp w reads TMEM lanes 32 (w % 4) ..; warps 2-5 take keys
//               0..63 of a chunk and output columns 0..63, warps 6-9 the rest; a row's own
//               positions come out of a 64-column span of BD by a five-stage register shift on
//               the bits of 31 - lane (one TMEM load cannot start at a per-lane column)
// TMEM: S in columns 0..127, BD in 128..383 (then P: hi 128..191, lo 192..255), O in 384..511.
// Shared memory: Q, K then V, and the two position halves in turn, 64 KB each. Every wait is bounded; on timeout the kernel records kErrWaitTimeout in the
// error word and returns.
#include "attention_tc.cuh"
#include "kernels.h"
#include "parakeet_kernels.h"
#include "ptx.cuh"
#include "tma.h"

#include <cuda_fp16.h>

#include <algorithm>

namespace telmo {

namespace {

using namespace tc_attention;

constexpr int T = 128;    // query rows per task, keys per chunk
constexpr int HD = 128;   // head size
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr uint32_t kColS = 0, kColBD = 128, kColP = 128, kColO = 384, kTmemCols = 512;
constexpr int kSmemBytes = 3 * kOperand + (256 + 128 + 2 * 128 + 2 * 128) * 4 + 256 + 1024;

struct Bars {
    uint64_t q_full, k_full, pa_full, pb_full, v_full, k_free, pa_free, s_done, p_full, o_done, o_free;
};

__global__ void __launch_bounds__(kThreads, 1)
txl_attention_tc_kernel(const __grid_constant__ CUtensorMap map_qkv, const __grid_constant__ CUtensorMap map_pos,
                        int rows, int npos, int heads, const TxlTask* __restrict__ tasks, int n_tasks,
                        const float* __restrict__ cv, const float* __restrict__ uk, float scale,
                        float* __restrict__ att, uint32_t* error) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* buf_q = smem;                  // Q of the task
    uint8_t* buf_kv = smem + kOperand;      // K, then V of the chunk
    uint8_t* buf_pos = smem + 2 * kOperand; // a position half, then the other
    float* cvw = reinterpret_cast<float*>(smem + 3 * kOperand);  // cv over the chunk's window [256]
    float* ukw = cvw + 256;                                       // uk over the chunk's keys [128]
    float* red_max = ukw + 128;                                   // [2 halves][128 rows]
    float* red_sum = red_max + 256;                               // [2 halves][128 rows]
    Bars* bars = reinterpret_cast<Bars*>(red_sum + 256);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int D = heads * HD;
    const int total = n_tasks * heads;

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        mbar_init(&bars->k_full, 1);
        mbar_init(&bars->pa_full, 1);
        mbar_init(&bars->pb_full, 1);
        mbar_init(&bars->v_full, 1);
        mbar_init(&bars->k_free, 1);
        mbar_init(&bars->pa_free, 1);
        mbar_init(&bars->s_done, 1);
        mbar_init(&bars->p_full, kEpiThreads);
        mbar_init(&bars->o_done, 1);
        mbar_init(&bars->o_free, kEpiThreads);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&map_qkv);
        prefetch_tensormap(&map_pos);
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
            int it = 0;  // chunks so far (every per-chunk barrier completes once per chunk)
            bool ok = true;
            for (int w = blockIdx.x; ok && w < total && !*abort_flag; w += gridDim.x) {
                const TxlTask tk = tasks[w / heads];
                const int h = w % heads, t = tk.len, i0 = tk.q_first;
                const int nch = (t + T - 1) / T;
                // Q: the previous task's last products are done with Q's buffer.
                if (it > 0 && !mbar_wait(&bars->s_done, (it - 1) & 1)) { fail(); break; }
                mbar_arrive_expect_tx(&bars->q_full, kOperand);
                load_operand(&map_qkv, &bars->q_full, buf_q, h * HD, tk.row + i0, rows + tk.row + i0);
                for (int c = 0; c < nch; ++c, ++it) {
                    const int j0 = c * T;
                    const int pw = tk.pos_row + t - 1 - i0 - (T - 1) + j0;  // the window's first row
                    const uint32_t prev = (it - 1) & 1;
                    // The first position half: the previous chunk's second position product (the
                    // s_done commit) is done with the position buffer.
                    if (it > 0 && !mbar_wait(&bars->s_done, prev)) { fail(); ok = false; break; }
                    mbar_arrive_expect_tx(&bars->pa_full, kOperand);
                    load_operand(&map_pos, &bars->pa_full, buf_pos, h * HD, pw, npos + pw);
                    if (it > 0 && !mbar_wait(&bars->o_done, prev)) { fail(); ok = false; break; }
                    mbar_arrive_expect_tx(&bars->k_full, kOperand);
                    load_operand(&map_qkv, &bars->k_full, buf_kv, D + h * HD, tk.row + j0, rows + tk.row + j0);
                    if (!mbar_wait(&bars->pa_free, it & 1)) { fail(); ok = false; break; }
                    mbar_arrive_expect_tx(&bars->pb_full, kOperand);
                    load_operand(&map_pos, &bars->pb_full, buf_pos, h * HD, pw + T, npos + pw + T);
                    if (!mbar_wait(&bars->k_free, it & 1)) { fail(); ok = false; break; }
                    mbar_arrive_expect_tx(&bars->v_full, kOperand);
                    load_operand(&map_qkv, &bars->v_full, buf_kv, 2 * D + h * HD, tk.row + j0, rows + tk.row + j0);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----------------------------------------------------------------------
        const uint32_t q = smem_u32(buf_q), kv = smem_u32(buf_kv), pb = smem_u32(buf_pos);
        constexpr uint32_t id_bd = idesc_f16(128, T, false);
        constexpr uint32_t id_o = idesc_f16(128, HD, true);
        // The three hi/lo products of one 128 x 128 (K = 128) block of A . B^T into d.
        auto split_product = [&](uint32_t d, uint32_t b, uint32_t idesc) {
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                const uint32_t off = (ks >> 2) * kBox + (ks & 3) * 32;
                mma_f16(d, sw128_desc(q + off), sw128_desc(b + off), idesc, ks > 0);
                mma_f16(d, sw128_desc(q + off), sw128_desc(b + 2 * kBox + off), idesc, 1u);
                mma_f16(d, sw128_desc(q + 2 * kBox + off), sw128_desc(b + off), idesc, 1u);
            }
        };
        int it = 0, tt = 0;
        bool ok = true;
        for (int w = blockIdx.x; ok && w < total && !*abort_flag; w += gridDim.x, ++tt) {
            const int t = tasks[w / heads].len;
            const int nch = (t + T - 1) / T;
            if (!mbar_wait(&bars->q_full, tt & 1)) { fail(); break; }
            for (int c = 0; c < nch; ++c, ++it) {
                const int n16 = (min(T, t - c * T) + 15) & ~15;
                const uint32_t prev = (it - 1) & 1;
                // First position half: its rows are in, the previous softmax has read S and BD,
                // and the previous O product is done with P in BD's columns.
                ok = mbar_wait(&bars->pa_full, it & 1) &&
                     (it == 0 || (mbar_wait(&bars->p_full, prev) && mbar_wait(&bars->o_done, prev)));
                if (!ok) { fail(); break; }
                tc_fence_after();
                if (lane == 0) {
                    split_product(tmem + kColBD, pb, id_bd);
                    mma_commit(&bars->pa_free);
                }
                __syncwarp();
                if (!mbar_wait(&bars->k_full, it & 1)) { fail(); ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    split_product(tmem + kColS, kv, idesc_f16(128, n16, false));
                    mma_commit(&bars->k_free);
                }
                __syncwarp();
                if (!mbar_wait(&bars->pb_full, it & 1)) { fail(); ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    split_product(tmem + kColBD + T, pb, id_bd);
                    mma_commit(&bars->s_done);
                }
                __syncwarp();
                // O: P is in TMEM (and the output so far rescaled), V is in, and -- at a task's
                // first chunk, whose product starts the output afresh -- the softmax warps have
                // read out the previous task's output. (o_free completes once per task: arriving
                // per chunk would let it run two phases ahead of this wait.)
                ok = mbar_wait(&bars->p_full, it & 1) && mbar_wait(&bars->v_full, it & 1) &&
                     (c > 0 || tt == 0 || mbar_wait(&bars->o_free, (tt - 1) & 1));
                if (!ok) { fail(); break; }
                tc_fence_after();
                if (lane == 0) {
                    for (int ks = 0; ks < n16 / 16; ++ks) {
                        const uint32_t voff = ks * 2048;  // 16 keys = two 8-row groups of 128 bytes
                        const uint32_t ph = tmem + kColP + ks * 8, pl = ph + 64;
                        mma_f16_ts(tmem + kColO, ph, sw128_desc_mn(kv + voff, kBox), id_o, (c > 0 || ks > 0) ? 1u : 0u);
                        mma_f16_ts(tmem + kColO, ph, sw128_desc_mn(kv + 2 * kBox + voff, kBox), id_o, 1u);
                        mma_f16_ts(tmem + kColO, pl, sw128_desc_mn(kv + voff, kBox), id_o, 1u);
                    }
                    mma_commit(&bars->o_done);
                }
                __syncwarp();
            }
        }
    } else {
        // ---- softmax and output (warps 2..9): thread = query row 32 (warp % 4) + lane, keys and
        // output columns 64 half .. 64 half + 63 -----------------------------------------------
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int row = quad * 32 + lane;
        const int et = threadIdx.x - 64;  // 0 .. 255
        const uint32_t lanes = tmem + (static_cast<uint32_t>(quad * 32) << 16);
        const int sh = 31 - lane;  // where this lane's positions start in its warp's span
        int it = 0;
        bool ok = true;
        for (int w = blockIdx.x; ok && w < total && !*abort_flag; w += gridDim.x) {
            const TxlTask tk = tasks[w / heads];
            const int h = w % heads, t = tk.len, i0 = tk.q_first;
            const int nch = (t + T - 1) / T;
            float m_run = -INFINITY, l_run = 0.0f;
            for (int c = 0; c < nch; ++c, ++it) {
                const int j0 = c * T;
                const int pw = tk.pos_row + t - 1 - i0 - (T - 1) + j0;
                // The chunk's bias terms into shared memory (the previous chunk's readers passed
                // two barriers since).
                {
                    const int p = pw + et;
                    cvw[et] = (p >= 0 && p < npos) ? __ldg(cv + static_cast<int64_t>(h) * npos + p) : 0.0f;
                    if (et < T) {
                        const int r = tk.row + j0 + et;
                        ukw[et] = (j0 + et < t) ? __ldg(uk + static_cast<int64_t>(h) * rows + r) : 0.0f;
                    }
                }
                epi_sync<kEpiThreads>();
                if (!mbar_wait(&bars->s_done, it & 1)) { fail(); ok = false; break; }
                tc_fence_after();
                float lg[64];
                float mx = -INFINITY;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int kc = 2 * half + cc;  // 32-key group of the chunk
                    // Keys 32 kc .. + 31 of row r read window rows 127 - r + 32 kc + j: for this warp's
                    // rows the columns 96 - 32 quad + 32 kc .. + 63 of BD hold them all; lane l's 32
                    // start at element 31 - l of that span, brought to the front of the lane's
                    // registers by shifts of 16, 8, 4, 2 and 1 on the bits of 31 - l.
                    uint32_t p0[32], p1[32], pv[64];
                    tmem_ld32(lanes + kColBD + 96 - 32 * quad + 32 * kc, p0);
                    tmem_ld32(lanes + kColBD + 128 - 32 * quad + 32 * kc, p1);
                    tmem_ld_wait();
#pragma unroll
                    for (int k = 0; k < 32; ++k) {
                        pv[k] = p0[k];
                        pv[32 + k] = p1[k];
                    }
                    shift_down<47, 16>(pv, (sh & 16) != 0);
                    shift_down<39, 8>(pv, (sh & 8) != 0);
                    shift_down<35, 4>(pv, (sh & 4) != 0);
                    shift_down<33, 2>(pv, (sh & 2) != 0);
                    shift_down<32, 1>(pv, (sh & 1) != 0);
                    uint32_t sv[32];
                    tmem_ld32(lanes + kColS + 32 * kc, sv);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int key = 32 * kc + j;
                        const int wcol = T - 1 - row + key;
                        const float ac = __fadd_rn(__uint_as_float(sv[j]), ukw[key]);
                        const float bd = __fadd_rn(__uint_as_float(pv[j]), cvw[wcol]);
                        float v = __fmul_rn(__fadd_rn(ac, bd), scale);
                        if (j0 + key >= t) v = -INFINITY;
                        lg[32 * cc + j] = v;
                        mx = fmaxf(mx, v);
                    }
                }
                red_max[half * T + row] = mx;
                epi_sync<kEpiThreads>();
                const float m_new = fmaxf(m_run, fmaxf(red_max[row], red_max[T + row]));
                const float corr = ex2_approx(__fmul_rn(__fsub_rn(m_run, m_new), kLog2e));  // 0 at the first chunk
                const float mxl = __fmul_rn(m_new, kLog2e);
                float part = 0.0f;
#pragma unroll
                for (int k = 0; k < 64; ++k) {
                    lg[k] = ex2_approx(__fmaf_rn(lg[k], kLog2e, -mxl));
                    part = __fadd_rn(part, lg[k]);
                }
                red_sum[half * T + row] = part;
                epi_sync<kEpiThreads>();
                l_run = __fmaf_rn(l_run, corr, __fadd_rn(red_sum[row], red_sum[T + row]));
                m_run = m_new;
                // The chunk's probabilities relative to the running maximum (at most 1) into TMEM
                // as the O product's A operand: fp16 pairs of consecutive keys per column, hi plane
                // in BD's columns 0..63, lo plane in 64..127.
                uint32_t hv[32], lv[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float h0 = f16_high(lg[2 * e]), h1 = f16_high(lg[2 * e + 1]);
                    hv[e] = pack2(h0, h1);
                    lv[e] = pack2(__fsub_rn(lg[2 * e], h0), __fsub_rn(lg[2 * e + 1], h1));
                }
                tmem_st32(lanes + kColP + 32 * half, hv);
                tmem_st32(lanes + kColP + 64 + 32 * half, lv);
                // The output so far (this task's earlier chunks, accumulated in TMEM) is rescaled to
                // the new maximum before this chunk's product adds to it; warps whose rows all kept
                // their maximum skip it.
                if (c > 0) {
                    if (!mbar_wait(&bars->o_done, (it - 1) & 1)) { fail(); ok = false; break; }
                    tc_fence_after();
                    if (__any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll
                        for (int g = 0; g < 2; ++g) {
                            uint32_t ov[32];
                            tmem_ld32(lanes + kColO + 64 * half + 32 * g, ov);
                            tmem_ld_wait();
#pragma unroll
                            for (int k = 0; k < 32; ++k) ov[k] = __float_as_uint(__fmul_rn(__uint_as_float(ov[k]), corr));
                            tmem_st32(lanes + kColO + 64 * half + 32 * g, ov);
                        }
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&bars->p_full);
                if (c + 1 == nch) {
                    // The last chunk: O / sum for this task's rows.
                    if (!mbar_wait(&bars->o_done, it & 1)) { fail(); ok = false; break; }
                    tc_fence_after();
                    const float inv = __fdiv_rn(1.0f, l_run);
                    float* orow = att + static_cast<int64_t>(tk.row + i0 + row) * D + h * HD + 64 * half;
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        uint32_t ov[32];
                        tmem_ld32(lanes + kColO + 64 * half + 32 * g, ov);
                        tmem_ld_wait();
                        if (i0 + row < t) {
#pragma unroll
                            for (int m = 0; m < 8; ++m)
                                *reinterpret_cast<float4*>(orow + 32 * g + 4 * m) =
                                    make_float4(__fmul_rn(__uint_as_float(ov[4 * m]), inv),
                                                __fmul_rn(__uint_as_float(ov[4 * m + 1]), inv),
                                                __fmul_rn(__uint_as_float(ov[4 * m + 2]), inv),
                                                __fmul_rn(__uint_as_float(ov[4 * m + 3]), inv));
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&bars->o_free);
                }
            }
            if (!ok) break;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// cv[h][p] = v_h . Pos[p]_h for the table's positions and uk[h][r] = u_h . K[r]_h for the batch's
// rows (Pos and K as their fp16 hi + lo planes); one warp per head and item.
__global__ void txl_bias_terms_kernel(const __half* __restrict__ pos, int npos, const __half* __restrict__ qkv,
                                      int rows, int heads, const float* __restrict__ bias_u,
                                      const float* __restrict__ bias_v, float* __restrict__ cv, float* __restrict__ uk) {
    const int item = blockIdx.x;
    const int h = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (h >= heads) return;
    const int D = heads * HD;
    const bool is_pos = item < npos;
    const int r = is_pos ? item : item - npos;
    const __half* hi = is_pos ? pos + static_cast<int64_t>(r) * D + h * HD
                              : qkv + static_cast<int64_t>(r) * 3 * D + D + h * HD;
    const int64_t plane = is_pos ? static_cast<int64_t>(npos) * D : static_cast<int64_t>(rows) * 3 * D;
    const float* b = (is_pos ? bias_v : bias_u) + h * HD;
    float acc = 0.0f;
    for (int k = lane; k < HD; k += 32)
        acc = __fmaf_rn(b[k], __fadd_rn(__half2float(hi[k]), __half2float(hi[plane + k])), acc);
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) (is_pos ? cv : uk)[static_cast<int64_t>(h) * (is_pos ? npos : rows) + r] = acc;
}

DeviceOnce configured;

}  // namespace

bool txl_attention_tc_supported(int hd) { return hd == HD; }

cudaError_t txl_bias_terms(const __half* pos, int npos, const __half* qkv, int rows, int heads, const float* bias_u,
                           const float* bias_v, float* cv, float* uk, cudaStream_t s) {
    if (npos + rows <= 0) return cudaSuccess;
    if (heads > 32) return cudaErrorInvalidValue;
    txl_bias_terms_kernel<<<npos + rows, 32 * heads, 0, s>>>(pos, npos, qkv, rows, heads, bias_u, bias_v, cv, uk);
    return cudaGetLastError();
}

cudaError_t txl_attention_tc(const __half* qkv, int rows, const __half* pos, int npos, const float* cv, const float* uk,
                             const TxlTask* tasks, int n_tasks, int heads, int hd, float scale, float* att,
                             uint32_t* error, cudaStream_t s) {
    if (n_tasks <= 0) return cudaSuccess;
    if (!txl_attention_tc_supported(hd) || rows <= 0 || npos <= 0) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured.done(dev)) {
        const cudaError_t e =
            cudaFuncSetAttribute(txl_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        configured.mark(dev);
    }
    const int D = heads * HD;
    // The products' two fp16 planes as one tensor each: QKV [2 rows, 3 D], positions [2 npos, D].
    CUtensorMap mq, mp;
    if (!encode_map_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qkv, static_cast<uint64_t>(3 * D),
                       2 * static_cast<uint64_t>(rows), static_cast<uint64_t>(3 * D) * 2, 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_map_2d(&mp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pos, static_cast<uint64_t>(D),
                       2 * static_cast<uint64_t>(npos), static_cast<uint64_t>(D) * 2, 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const int grid = std::min(n_tasks * heads, num_sms());
    txl_attention_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(mq, mp, rows, npos, heads, tasks, n_tasks, cv, uk, scale,
                                                               att, error);
    return cudaGetLastError();
}

}  // namespace telmo
