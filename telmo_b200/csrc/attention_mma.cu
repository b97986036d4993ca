// attention_mma.cu -- Granite's block-local attention with Shaw relative positions
// (Granite::attention, src/granite.rs:965-1036) on the tensor cores.
//
// One CTA per (attention block, head): the block's len <= 128 query rows, eight warps of 16 rows.
// Q, K and V arrive as fp16 high/low planes (x = hi + lo, written by the QKV product's
// epilogue), the relative-position table as fp16 (its int8 values are exact) with one f32 scale
// per position. For each warp:
//   pos = Q . Rel^T over the 144 positions its rows reach, times each position's scale
//   S   = Q . K^T,  S[i][j] = scale * S[i][j] + scale * pos[i][ctx - 1 - i + j]
//   P   = softmax(S) per row over the len keys (f32 exponentials, f64 sum, as the reference)
//   O   = P . V
// Products run on mma.sync m16n8k16 (fp16 in, f32 accumulate) as hi.hi + hi.lo + lo.hi, which
// keeps about 21 bits of every operand, so they match the reference's f32 sums to about 1e-6
// relative; Q.Rel^T needs only Q's two parts. Operands are staged with cp.async; shared memory
// is reused from phase to phase (Rel -> position scratch, Q -> P, K -> V).
#include "mma.cuh"
#include "rowops.h"

#include <cuda_fp16.h>

namespace telmo {

namespace {

constexpr int T = 128;    // query rows and keys per block (Granite's context)
constexpr int PR = 256;   // staged relative positions (255 used)
constexpr int PW = 144;   // positions one warp's 16 rows reach (143), 18 n-tiles of 8
constexpr int SP = 148;   // f32 pitch of a warp's position scratch

template <int HD>
struct MmaSmem {
    static constexpr int HP = HD + 8;  // fp16 pitch: consecutive rows start 16 bytes apart in banks
    __half qh[T * HP], ql[T * HP];     // Q, then P
    __half kh[T * HP], kl[T * HP];     // K, then V
    union {
        __half rel[PR * HP];
        float scratch[8][16 * SP];
    } u;
    float rscale[PR];
};

using mma::cp16;
using mma::cp_commit_wait;
using mma::load_a;
using mma::load_b_kn;
using mma::load_b_nk;
using mma::mma16816;
using mma::split_half;

// Stages rows [0, T) of a [rows][ld] fp16 plane pair (hi at src, lo at src + plane) into hi/lo
// tiles; rows >= len are zero.
template <int HD>
__device__ __forceinline__ void stage_pair(__half* hi, __half* lo, const __half* src, int64_t ld, int64_t plane,
                                           int len, int tid) {
    constexpr int HP = HD + 8, CH = HD / 8;  // 16-byte chunks per row
    for (int e = tid; e < 2 * T * CH; e += 256) {
        const int pl = e / (T * CH), r = (e / CH) % T, c = e % CH;
        const __half* s = src + pl * plane + r * ld + c * 8;
        __half* d = (pl ? lo : hi) + r * HP + c * 8;
        cp16(d, r < len ? s : src, r < len);
    }
}

template <int HD>
__global__ void __launch_bounds__(256, 1)
granite_attention_mma_kernel(const __half* __restrict__ qkv, int64_t plane, int heads, int ctx,
                             const AttnTask* __restrict__ tasks, const __half* __restrict__ rel16,
                             const float* __restrict__ rel_scale, float scale, float* __restrict__ att) {
    using S = MmaSmem<HD>;
    constexpr int HP = S::HP;
    constexpr int NT = T / 8;    // key n-tiles
    constexpr int KT = HD / 16;  // k-steps over d
    constexpr int PT = PW / 8;   // position n-tiles per warp (18)
    extern __shared__ __align__(16) uint8_t smem_raw[];
    S& sm = *reinterpret_cast<S*>(smem_raw);

    const AttnTask task = tasks[blockIdx.x];
    const int len = task.len;
    const int h = blockIdx.y;
    const int D = heads * HD;
    const int64_t ld = 3 * static_cast<int64_t>(D);
    const __half* base = qkv + task.row * ld + h * HD;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int positions = 2 * ctx - 1;

    // ---- stage Q, K (fp16 parts) and the relative table -------------------------------------------
    stage_pair<HD>(sm.qh, sm.ql, base, ld, plane, len, tid);
    stage_pair<HD>(sm.kh, sm.kl, base + D, ld, plane, len, tid);
    for (int e = tid; e < PR * (HD / 8); e += 256) {
        const int p = e / (HD / 8), c = e % (HD / 8);
        cp16(sm.u.rel + p * HP + c * 8, p < positions ? rel16 + p * HD + c * 8 : rel16, p < positions);
    }
    for (int p = tid; p < PR; p += 256) sm.rscale[p] = p < positions ? __ldg(rel_scale + p) : 0.0f;
    cp_commit_wait();
    __syncthreads();

    const int g = lane / 4, t = lane % 4;
    const int rw = warp * 16;             // this warp's first row
    const bool active = rw < len;
    // Row i reaches positions ctx - 1 - i .. ctx - 1 - i + 127; the warp's rows need p_w0 onwards.
    const int p_w0 = ctx - 1 - (rw + 15);

    // ---- pos = Q . Rel^T for positions p_w0 .. p_w0 + 143 (kept in registers) ----------------------
    float pacc[PT][4];
#pragma unroll
    for (int n = 0; n < PT; ++n) pacc[n][0] = pacc[n][1] = pacc[n][2] = pacc[n][3] = 0.0f;
    if (active) {
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            uint32_t ah[4], al[4];
            load_a(sm.qh, HP, rw, k * 16, lane, ah);
            load_a(sm.ql, HP, rw, k * 16, lane, al);
#pragma unroll
            for (int n = 0; n < PT; n += 2) {
                uint32_t b[4];
                load_b_nk(sm.u.rel, HP, p_w0 + n * 8, k * 16, lane, b);
                mma16816(pacc[n], ah, b[0], b[1]);
                mma16816(pacc[n], al, b[0], b[1]);
                mma16816(pacc[n + 1], ah, b[2], b[3]);
                mma16816(pacc[n + 1], al, b[2], b[3]);
            }
        }
    }
    __syncthreads();  // the table is no longer read: its space becomes the position scratch
    float* scr = sm.u.scratch[warp];
#pragma unroll
    for (int n = 0; n < PT; ++n) {
        const int c = n * 8 + 2 * t;
        const float s0 = sm.rscale[p_w0 + c], s1 = sm.rscale[p_w0 + c + 1];
        scr[g * SP + c] = __fmul_rn(pacc[n][0], s0);
        scr[g * SP + c + 1] = __fmul_rn(pacc[n][1], s1);
        scr[(g + 8) * SP + c] = __fmul_rn(pacc[n][2], s0);
        scr[(g + 8) * SP + c + 1] = __fmul_rn(pacc[n][3], s1);
    }
    __syncwarp();

    // ---- S = Q . K^T, plus the shifted positions; row softmax; P replaces the warp's Q rows --------
    if (active) {
        float s[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            uint32_t ah[4], al[4];
            load_a(sm.qh, HP, rw, k * 16, lane, ah);
            load_a(sm.ql, HP, rw, k * 16, lane, al);
#pragma unroll
            for (int n = 0; n < NT; n += 2) {
                uint32_t bh[4], bl[4];
                load_b_nk(sm.kh, HP, n * 8, k * 16, lane, bh);
                load_b_nk(sm.kl, HP, n * 8, k * 16, lane, bl);
                mma16816(s[n], ah, bh[0], bh[1]);
                mma16816(s[n], ah, bl[0], bl[1]);
                mma16816(s[n], al, bh[0], bh[1]);
                mma16816(s[n + 1], ah, bh[2], bh[3]);
                mma16816(s[n + 1], ah, bl[2], bl[3]);
                mma16816(s[n + 1], al, bh[2], bh[3]);
            }
        }
        // Row r (0..15 of the warp) and key j read scratch column j + 15 - r.
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = g + (e / 2) * 8;
                const int j = n * 8 + 2 * t + (e % 2);
                float v = __fadd_rn(__fmul_rn(s[n][e], scale), __fmul_rn(scr[r * SP + j + 15 - r], scale));
                if (j >= len) v = -INFINITY;
                s[n][e] = v;
                if (e < 2) mx0 = fmaxf(mx0, v);
                else mx1 = fmaxf(mx1, v);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        double sum0 = 0.0, sum1 = 0.0;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float ex = expf(__fsub_rn(s[n][e], e < 2 ? mx0 : mx1));
                s[n][e] = ex;
                if (e < 2) sum0 += static_cast<double>(ex);
                else sum1 += static_cast<double>(ex);
            }
        }
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
        const float inv0 = static_cast<float>(1.0 / sum0), inv1 = static_cast<float>(1.0 / sum1);
        __syncwarp();
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = rw + g + (e / 2) * 8;
                const int j = n * 8 + 2 * t + (e % 2);
                split_half(__fmul_rn(s[n][e], e < 2 ? inv0 : inv1), sm.qh[r * HP + j], sm.ql[r * HP + j]);
            }
        }
    }
    __syncthreads();  // every warp is done with K

    // ---- V replaces K --------------------------------------------------------------------------------
    stage_pair<HD>(sm.kh, sm.kl, base + 2 * D, ld, plane, len, tid);
    cp_commit_wait();
    __syncthreads();

    // ---- O = P . V --------------------------------------------------------------------------------
    if (!active) return;
    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
#pragma unroll
    for (int k = 0; k < T / 16; ++k) {
        uint32_t ah[4], al[4];
        load_a(sm.qh, HP, rw, k * 16, lane, ah);
        load_a(sm.ql, HP, rw, k * 16, lane, al);
#pragma unroll
        for (int n = 0; n < HD / 8; n += 2) {
            uint32_t bh[4], bl[4];
            load_b_kn(sm.kh, HP, k * 16, n * 8, lane, bh);
            load_b_kn(sm.kl, HP, k * 16, n * 8, lane, bl);
            mma16816(o[n], ah, bh[0], bh[1]);
            mma16816(o[n], ah, bl[0], bl[1]);
            mma16816(o[n], al, bh[0], bh[1]);
            mma16816(o[n + 1], ah, bh[2], bh[3]);
            mma16816(o[n + 1], ah, bl[2], bl[3]);
            mma16816(o[n + 1], al, bh[2], bh[3]);
        }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int i = rw + g + hh * 8;
        if (i >= len) continue;
        float* orow = att + (task.row + i) * static_cast<int64_t>(D) + h * HD;
#pragma unroll
        for (int n = 0; n < HD / 8; ++n)
            *reinterpret_cast<float2*>(orow + n * 8 + 2 * t) = make_float2(o[n][hh * 2], o[n][hh * 2 + 1]);
    }
}

template <int HD>
cudaError_t launch(const __half* qkv, int64_t plane, int heads, int ctx, const AttnTask* tasks, int n_tasks,
                   const __half* rel16, const float* rel_scale, float scale, float* att, cudaStream_t stream) {
    const int smem = static_cast<int>(sizeof(MmaSmem<HD>));
    static DeviceOnce configured;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured.done(dev)) {
        cudaError_t e = cudaFuncSetAttribute(granite_attention_mma_kernel<HD>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured.mark(dev);
    }
    dim3 grid(n_tasks, heads);
    granite_attention_mma_kernel<HD><<<grid, 256, smem, stream>>>(qkv, plane, heads, ctx, tasks, rel16, rel_scale,
                                                                  scale, att);
    return cudaGetLastError();
}

}  // namespace

bool granite_attention_mma_supported(int hd, int ctx) { return ctx == T && (hd == 64 || hd == 128); }

cudaError_t granite_attention_mma(const __half* qkv, int64_t plane, int heads, int hd, int ctx, const AttnTask* tasks,
                                  int n_tasks, const __half* rel16, const float* rel_scale, float scale, float* att,
                                  cudaStream_t stream) {
    if (n_tasks <= 0) return cudaSuccess;
    if (!granite_attention_mma_supported(hd, ctx)) return cudaErrorInvalidValue;
    if (hd == 128) return launch<128>(qkv, plane, heads, ctx, tasks, n_tasks, rel16, rel_scale, scale, att, stream);
    return launch<64>(qkv, plane, heads, ctx, tasks, n_tasks, rel16, rel_scale, scale, att, stream);
}

}  // namespace telmo
