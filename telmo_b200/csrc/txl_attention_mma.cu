// txl_attention_mma.cu -- Parakeet's Transformer-XL relative attention over whole utterances
// (Parakeet::attention, src/parakeet.rs:1176-1282) on the tensor cores.
//
// One CTA per (64 query rows of one utterance, head), walking the keys in chunks of CK. Eight
// warps: warp w takes query rows 16 (w % 4) .. + 15 and the half w / 4 of every chunk's keys, with
// its own running softmax state; the two halves are merged at the end. Q, K, V and the projected
// positions arrive as fp16 high/low planes (x = hi + lo, written by the products' epilogues). Per
// chunk and warp:
//   BD = Qu . Pos^T over the 16 + CK - 1 positions its rows reach, plus c[p] = (v - u) . Pos[p],
//        which makes it (q + v) . Pos (u, v the biases; c is computed once per layer)
//   AC = Qu . K^T
//   S[i][j] = (AC[i][j] + BD[i][t - 1 - i + j]) * scale, keys past the utterance masked
//   then an online softmax (running row maximum and sum, f32) and O += exp(S - max) . V.
// Products run on mma.sync m16n8k16 (fp16 in, f32 accumulate) as hi.hi + hi.lo + lo.hi, which keeps
// about 21 bits of every operand. The probabilities go from the S accumulators straight into A
// fragments. Shared memory holds no score row, so an utterance may be of any length.
//
// Against the reference's arithmetic: sums run over ascending d in f32 as there but in the
// tensor cores' order; the maximum and the sum of exponentials are kept online instead of over
// the whole row (each rescale is one f32 exponential); O is divided by the sum at the end instead
// of each probability before the product. Each differs from the reference by f32 rounding.
#include "mma.cuh"
#include "parakeet_kernels.h"

#include <cuda_fp16.h>

namespace telmo {

namespace {

constexpr int R = 64;  // query rows per CTA
constexpr unsigned kFull = 0xffffffffu;

template <int HD, int CK>
struct TxlSmem {
    static constexpr int HP = HD + 8;    // fp16 pitch: rows start 16 bytes apart in banks
    static constexpr int PRW = R + CK;   // staged positions per chunk (R + CK - 1 used)
    static constexpr int KH = CK / 2;    // keys per warp per chunk
    static constexpr int PW = 16 + KH;   // positions one warp's rows reach (15 + KH used)
    static constexpr int SPW = PW + 4;   // f32 pitch of a warp's position scratch
    __half qh[R * HP], ql[R * HP];
    __half kh[CK * HP], kl[CK * HP];
    __half vh[CK * HP], vl[CK * HP];
    union {
        struct {
            __half ph[PRW * HP], pl[PRW * HP];
        } pos;
        float merge[R / 16][HD / 8][32][4];  // the second key half's O, after the loop
    } u;
    float cp[PRW];
    float mlm[R / 16][32][4];                // its (m0, m1, l0, l1) per lane
    float scr[2 * R / 16][16 * SPW];
};

using mma::cp16;
using mma::cp4;
using mma::cp_commit;
using mma::cp_wait;
using mma::load_a;
using mma::load_b_kn;
using mma::load_b_nk;
using mma::mma16816;
using mma::split_half;
using mma::split_pack;

constexpr int kThreads = 2 * R / 16 * 32;  // 256

// Rows [r0, r0 + n) of a plane pair (hi at src, lo at src + plane; rows ld apart) into hi/lo
// tiles; rows whose index r0 + r is outside [lo_ok, hi_ok) are zero.
template <int HD>
__device__ __forceinline__ void stage_rows(__half* hi, __half* lo, const __half* src, int64_t ld, int64_t plane,
                                           int r0, int n, int lo_ok, int hi_ok, int tid) {
    constexpr int HP = HD + 8, CH = HD / 8;
    for (int e = tid; e < 2 * n * CH; e += kThreads) {
        const int pl = e / (n * CH), r = (e / CH) % n, c = e % CH;
        const int row = r0 + r;
        const bool ok = row >= lo_ok && row < hi_ok;
        const __half* s = src + pl * plane + (ok ? static_cast<int64_t>(row) * ld : 0) + c * 8;
        cp16((pl ? lo : hi) + r * HP + c * 8, s, ok);
    }
}

template <int HD, int CK>
__global__ void __launch_bounds__(kThreads, 1)
txl_attention_mma_kernel(const __half* __restrict__ qkv, int64_t plane, const __half* __restrict__ pos,
                         int64_t pplane, const float* __restrict__ cpos, int npos, const TxlTask* __restrict__ tasks,
                         int heads, const float* __restrict__ bias_u, float scale, float* __restrict__ att) {
    using S = TxlSmem<HD, CK>;
    constexpr int HP = S::HP, PW = S::PW, SPW = S::SPW, KH = S::KH, PRW = S::PRW;
    constexpr int KT = HD / 16;  // k-steps over d
    constexpr int NT = KH / 8;   // key n-tiles per warp and chunk
    constexpr int PT = PW / 8;   // position n-tiles per warp
    constexpr int OT = HD / 8;   // output n-tiles
    static_assert(NT % 2 == 0 && PT % 2 == 0, "n-tiles come in pairs");
    extern __shared__ __align__(16) uint8_t smem_raw[];
    S& sm = *reinterpret_cast<S*>(smem_raw);

    const TxlTask task = tasks[blockIdx.x];
    const int h = blockIdx.y;
    const int t = task.len, i0 = task.q_first;
    const int D = heads * HD;
    const int64_t ld = 3 * static_cast<int64_t>(D);
    const __half* qbase = qkv + static_cast<int64_t>(task.row) * ld + h * HD;
    const __half* pbase = pos + static_cast<int64_t>(task.pos_row) * D + h * HD;
    const float* cbase = cpos + static_cast<int64_t>(h) * npos + task.pos_row;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int g = lane / 4, tq = lane % 4;
    const int rb = warp % (R / 16), half = warp / (R / 16);
    const int rw = rb * 16;                     // the warp's first row in the CTA
    const int off_w = R - 16 - rw + half * KH;  // its first staged position
    const int nchunks = (t + CK - 1) / CK;

    auto stage_kp = [&](int c) {
        const int j0 = c * CK;
        stage_rows<HD>(sm.kh, sm.kl, qbase + D, ld, plane, j0, CK, 0, t, tid);
        // Positions t - 1 - (i0 + R - 1) + j0 onwards; valid ones are 0 .. 2t - 2.
        const int p0 = t - i0 - R + j0;
        stage_rows<HD>(sm.u.pos.ph, sm.u.pos.pl, pbase, D, pplane, p0, PRW, 0, 2 * t - 1, tid);
        for (int r = tid; r < PRW; r += kThreads) {
            const int pi = p0 + r;
            const bool ok = pi >= 0 && pi < 2 * t - 1;
            cp4(&sm.cp[r], cbase + (ok ? pi : 0), ok);
        }
        cp_commit();
    };
    auto stage_v = [&](int c) {
        stage_rows<HD>(sm.vh, sm.vl, qbase + 2 * D, ld, plane, c * CK, CK, 0, t, tid);
        cp_commit();
    };
    // Q (its fp16 parts) arrives through cp.async with the first chunk's operands; rows past the
    // utterance are zero.
    stage_rows<HD>(sm.qh, sm.ql, qbase, ld, plane, i0, R, 0, t, tid);
    cp_commit();
    stage_kp(0);
    stage_v(0);
    cp_wait<2>();
    __syncthreads();
    // Q + u, split again into fp16 parts, in place (each element by the thread that reads it).
    for (int e = tid; e < R * HD / 2; e += kThreads) {
        const int r = e / (HD / 2), c = (e % (HD / 2)) * 2;
        float x0 = 0.0f, x1 = 0.0f;
        if (i0 + r < t) {
            const __half2 hi = *reinterpret_cast<const __half2*>(sm.qh + r * HP + c);
            const __half2 lo = *reinterpret_cast<const __half2*>(sm.ql + r * HP + c);
            x0 = __fadd_rn(__fadd_rn(__low2float(hi), __low2float(lo)), __ldg(bias_u + h * HD + c));
            x1 = __fadd_rn(__fadd_rn(__high2float(hi), __high2float(lo)), __ldg(bias_u + h * HD + c + 1));
        }
        split_half(x0, sm.qh[r * HP + c], sm.ql[r * HP + c]);
        split_half(x1, sm.qh[r * HP + c + 1], sm.ql[r * HP + c + 1]);
    }

    float o[OT][4];
#pragma unroll
    for (int n = 0; n < OT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY;  // running maxima of rows g and g + 8
    float l0 = 0.0f, l1 = 0.0f;            // this thread's share of the running sums
    float* scr = sm.scr[warp];

    for (int c = 0; c < nchunks; ++c) {
        const int j0 = c * CK + half * KH;  // this warp's first key
        cp_wait<1>();  // K and positions of this chunk
        __syncthreads();
        // ---- BD over the warp's positions, plus c[p], into its scratch ----------------------------
        {
            // The high product and the two cross products go to separate accumulators (two
            // independent MMA chains instead of one), summed after the loop.
            float bd[PT][4], bx[PT][4];
#pragma unroll
            for (int n = 0; n < PT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) bd[n][e] = bx[n][e] = 0.0f;
#pragma unroll
            for (int k = 0; k < KT; ++k) {
                uint32_t ah[4], al[4];
                load_a(sm.qh, HP, rw, k * 16, lane, ah);
                load_a(sm.ql, HP, rw, k * 16, lane, al);
#pragma unroll
                for (int n = 0; n < PT; n += 2) {
                    uint32_t bh[4], bl[4];
                    load_b_nk(sm.u.pos.ph, HP, off_w + n * 8, k * 16, lane, bh);
                    load_b_nk(sm.u.pos.pl, HP, off_w + n * 8, k * 16, lane, bl);
                    mma16816(bd[n], ah, bh[0], bh[1]);
                    mma16816(bx[n], ah, bl[0], bl[1]);
                    mma16816(bx[n], al, bh[0], bh[1]);
                    mma16816(bd[n + 1], ah, bh[2], bh[3]);
                    mma16816(bx[n + 1], ah, bl[2], bl[3]);
                    mma16816(bx[n + 1], al, bh[2], bh[3]);
                }
            }
#pragma unroll
            for (int n = 0; n < PT; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) bd[n][e] = __fadd_rn(bd[n][e], bx[n][e]);
#pragma unroll
            for (int n = 0; n < PT; ++n) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int p = n * 8 + 2 * tq + e;
                    const float cv = sm.cp[off_w + p];
                    scr[g * SPW + p] = __fadd_rn(bd[n][e], cv);
                    scr[(g + 8) * SPW + p] = __fadd_rn(bd[n][2 + e], cv);
                }
            }
        }
        // ---- AC = Qu . K^T over the warp's keys -------------------------------------------------------
        float s[NT][4], sx[NT][4], sy[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[n][e] = sx[n][e] = sy[n][e] = 0.0f;
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            uint32_t ah[4], al[4];
            load_a(sm.qh, HP, rw, k * 16, lane, ah);
            load_a(sm.ql, HP, rw, k * 16, lane, al);
#pragma unroll
            for (int n = 0; n < NT; n += 2) {
                uint32_t bh[4], bl[4];
                load_b_nk(sm.kh, HP, half * KH + n * 8, k * 16, lane, bh);
                load_b_nk(sm.kl, HP, half * KH + n * 8, k * 16, lane, bl);
                mma16816(s[n], ah, bh[0], bh[1]);
                mma16816(sx[n], ah, bl[0], bl[1]);
                mma16816(sy[n], al, bh[0], bh[1]);
                mma16816(s[n + 1], ah, bh[2], bh[3]);
                mma16816(sx[n + 1], ah, bl[2], bl[3]);
                mma16816(sy[n + 1], al, bh[2], bh[3]);
            }
        }
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[n][e] = __fadd_rn(s[n][e], __fadd_rn(sx[n][e], sy[n][e]));
        __syncwarp();
        // ---- scores, online softmax --------------------------------------------------------------
        // Row r (0..15 of the warp) and key jj (0..KH-1 of the warp) read scratch column jj + 15 - r.
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = g + (e / 2) * 8;
                const int jj = n * 8 + 2 * tq + (e % 2);
                float v = __fmul_rn(__fadd_rn(s[n][e], scr[r * SPW + jj + 15 - r]), scale);
                if (j0 + jj >= t) v = -INFINITY;
                s[n][e] = v;
                if (e < 2) mx0 = fmaxf(mx0, v);
                else mx1 = fmaxf(mx1, v);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 2));
        // A half whose keys all lie past the utterance keeps its state (its maximum stays -inf
        // until a valid key arrives, and exp(-inf - m) is 0).
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        const bool grew = n0 != m0 || n1 != m1;
        if (__any_sync(kFull, grew)) {
            const float c0 = n0 == -INFINITY ? 1.0f : expf(__fsub_rn(m0, n0));
            const float c1 = n1 == -INFINITY ? 1.0f : expf(__fsub_rn(m1, n1));
            l0 = __fmul_rn(l0, c0);
            l1 = __fmul_rn(l1, c1);
#pragma unroll
            for (int n = 0; n < OT; ++n) {
                o[n][0] = __fmul_rn(o[n][0], c0);
                o[n][1] = __fmul_rn(o[n][1], c0);
                o[n][2] = __fmul_rn(o[n][2], c1);
                o[n][3] = __fmul_rn(o[n][3], c1);
            }
            m0 = n0;
            m1 = n1;
        }
        float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mm = e < 2 ? m0 : m1;
                const float ex = mm == -INFINITY ? 0.0f : expf(__fsub_rn(s[n][e], mm));
                s[n][e] = ex;
                if (e < 2) sum0 = __fadd_rn(sum0, ex);
                else sum1 = __fadd_rn(sum1, ex);
            }
        }
        l0 = __fadd_rn(l0, sum0);
        l1 = __fadd_rn(l1, sum1);
        // The exponentials as A fragments (keys as k), high and low fp16 parts.
        uint32_t ph[NT / 2][4], pl[NT / 2][4];
#pragma unroll
        for (int ks = 0; ks < NT / 2; ++ks) {
            split_pack(s[2 * ks][0], s[2 * ks][1], ph[ks][0], pl[ks][0]);
            split_pack(s[2 * ks][2], s[2 * ks][3], ph[ks][1], pl[ks][1]);
            split_pack(s[2 * ks + 1][0], s[2 * ks + 1][1], ph[ks][2], pl[ks][2]);
            split_pack(s[2 * ks + 1][2], s[2 * ks + 1][3], ph[ks][3], pl[ks][3]);
        }
        __syncthreads();  // every warp is done with this chunk's K and positions
        if (c + 1 < nchunks) stage_kp(c + 1);
        else cp_commit();
        cp_wait<1>();     // V of this chunk
        __syncthreads();
        // ---- O += P . V over the warp's keys ------------------------------------------------------
#pragma unroll
        for (int ks = 0; ks < NT / 2; ++ks) {
#pragma unroll
            for (int n = 0; n < OT; n += 2) {
                uint32_t bh[4], bl[4];
                load_b_kn(sm.vh, HP, half * KH + ks * 16, n * 8, lane, bh);
                load_b_kn(sm.vl, HP, half * KH + ks * 16, n * 8, lane, bl);
                mma16816(o[n], ph[ks], bh[0], bh[1]);
                mma16816(o[n], ph[ks], bl[0], bl[1]);
                mma16816(o[n], pl[ks], bh[0], bh[1]);
                mma16816(o[n + 1], ph[ks], bh[2], bh[3]);
                mma16816(o[n + 1], ph[ks], bl[2], bl[3]);
                mma16816(o[n + 1], pl[ks], bh[2], bh[3]);
            }
        }
        __syncthreads();  // every warp is done with this chunk's V
        if (c + 1 < nchunks) stage_v(c + 1);
        else cp_commit();
    }
    cp_wait<0>();
    l0 = __fadd_rn(l0, __shfl_xor_sync(kFull, l0, 1));
    l0 = __fadd_rn(l0, __shfl_xor_sync(kFull, l0, 2));
    l1 = __fadd_rn(l1, __shfl_xor_sync(kFull, l1, 1));
    l1 = __fadd_rn(l1, __shfl_xor_sync(kFull, l1, 2));
    __syncthreads();  // the position buffers become the merge buffer
    if (half == 1) {
#pragma unroll
        for (int n = 0; n < OT; ++n)
            *reinterpret_cast<float4*>(sm.u.merge[rb][n][lane]) = make_float4(o[n][0], o[n][1], o[n][2], o[n][3]);
        *reinterpret_cast<float4*>(sm.mlm[rb][lane]) = make_float4(m0, m1, l0, l1);
    }
    __syncthreads();
    if (half == 1) return;
    // Merge the two key halves: O = (Oa e^(ma - m) + Ob e^(mb - m)) / (la e^(ma - m) + lb e^(mb - m)).
    const float4 other = *reinterpret_cast<const float4*>(sm.mlm[rb][lane]);
    const float M0 = fmaxf(m0, other.x), M1 = fmaxf(m1, other.y);
    const float a0 = m0 == -INFINITY ? 0.0f : expf(__fsub_rn(m0, M0));
    const float b0 = other.x == -INFINITY ? 0.0f : expf(__fsub_rn(other.x, M0));
    const float a1 = m1 == -INFINITY ? 0.0f : expf(__fsub_rn(m1, M1));
    const float b1 = other.y == -INFINITY ? 0.0f : expf(__fsub_rn(other.y, M1));
    const float inv0 = __fdiv_rn(1.0f, __fadd_rn(__fmul_rn(l0, a0), __fmul_rn(other.z, b0)));
    const float inv1 = __fdiv_rn(1.0f, __fadd_rn(__fmul_rn(l1, a1), __fmul_rn(other.w, b1)));
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int i = i0 + rw + g + hh * 8;
        if (i >= t) continue;
        const float a = hh ? a1 : a0, b = hh ? b1 : b0, inv = hh ? inv1 : inv0;
        float* orow = att + (static_cast<int64_t>(task.row) + i) * D + h * HD;
#pragma unroll
        for (int n = 0; n < OT; ++n) {
            const float4 ob = *reinterpret_cast<const float4*>(sm.u.merge[rb][n][lane]);
            const float x0 = __fadd_rn(__fmul_rn(o[n][hh * 2], a), __fmul_rn(hh ? ob.z : ob.x, b));
            const float x1 = __fadd_rn(__fmul_rn(o[n][hh * 2 + 1], a), __fmul_rn(hh ? ob.w : ob.y, b));
            *reinterpret_cast<float2*>(orow + n * 8 + 2 * tq) = make_float2(__fmul_rn(x0, inv), __fmul_rn(x1, inv));
        }
    }
}

// c[h][p] = (bias_v - bias_u)_h . Pos[p]_h for every head and position; one warp per head.
__global__ void txl_pos_bias_kernel(const __half* __restrict__ pos, int64_t pplane, int npos, int heads, int hd,
                                    const float* __restrict__ bias_u, const float* __restrict__ bias_v,
                                    float* __restrict__ cpos) {
    const int p = blockIdx.x;
    const int h = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (p >= npos || h >= heads) return;
    const int64_t row = static_cast<int64_t>(p) * heads * hd + h * hd;
    float acc = 0.0f;
    for (int d = lane; d < hd; d += 32) {
        const float x = __fadd_rn(__half2float(pos[row + d]), __half2float(pos[pplane + row + d]));
        acc = __fmaf_rn(__fsub_rn(bias_v[h * hd + d], bias_u[h * hd + d]), x, acc);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
    if (lane == 0) cpos[static_cast<int64_t>(h) * npos + p] = acc;
}

template <int HD, int CK>
cudaError_t launch(const __half* qkv, int64_t plane, const __half* pos, int64_t pplane, const float* cpos, int npos,
                   const TxlTask* tasks, int n_tasks, int heads, const float* bias_u, float scale, float* att,
                   cudaStream_t s) {
    const int smem = static_cast<int>(sizeof(TxlSmem<HD, CK>));
    const cudaError_t e =
        cudaFuncSetAttribute(txl_attention_mma_kernel<HD, CK>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(n_tasks, heads);
    txl_attention_mma_kernel<HD, CK><<<grid, kThreads, smem, s>>>(qkv, plane, pos, pplane, cpos, npos, tasks, heads, bias_u,
                                                             scale, att);
    return cudaGetLastError();
}

}  // namespace

bool txl_attention_mma_supported(int hd) { return hd == 64 || hd == 128; }

cudaError_t txl_pos_bias(const __half* pos, int64_t pplane, int npos, int heads, int hd, const float* bias_u,
                         const float* bias_v, float* cpos, cudaStream_t s) {
    if (npos <= 0) return cudaSuccess;
    if (heads > 32) return cudaErrorInvalidValue;
    txl_pos_bias_kernel<<<npos, 32 * heads, 0, s>>>(pos, pplane, npos, heads, hd, bias_u, bias_v, cpos);
    return cudaGetLastError();
}

cudaError_t txl_attention_mma(const __half* qkv, int64_t plane, const __half* pos, int64_t pplane, const float* cpos,
                              int npos, const TxlTask* tasks, int n_tasks, int heads, int hd, const float* bias_u,
                              float scale, float* att, cudaStream_t s) {
    if (n_tasks <= 0) return cudaSuccess;
    if (hd == 128) return launch<128, 64>(qkv, plane, pos, pplane, cpos, npos, tasks, n_tasks, heads, bias_u, scale, att, s);
    if (hd == 64) return launch<64, 64>(qkv, plane, pos, pplane, cpos, npos, tasks, n_tasks, heads, bias_u, scale, att, s);
    return cudaErrorInvalidValue;
}

}  // namespace telmo
