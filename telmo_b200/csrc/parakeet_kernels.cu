// parakeet_kernels.cu -- the Parakeet-specific kernels: the subsampling convolutions, the
// relative position table, Transformer-XL attention over a whole utterance and the steps of
// batched greedy TDT decoding.
//
// Arithmetic follows the reference: conv3x3s2_row (src/kernels/scalar.rs:194-232) starts from
// the bias and adds taps dt-major with separate rounding; positions (src/parakeet.rs:1618-1630)
// in f64; attention (src/parakeet.rs:1176-1282) sums every dot product over ascending d (or j)
// with fused multiply-adds, adds the shifted position score before scaling, and takes the
// softmax with f32 exponentials and an f64 sum; the LSTM (src/parakeet.rs:1524-1577) uses
// sigmoid = 1 / (1 + e^-x) and tanh in f32.
#include "parakeet_kernels.h"

#include <cmath>

namespace telmo {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float madd(float acc, float w, float v) { return __fadd_rn(acc, __fmul_rn(w, v)); }

}  // namespace

// Fused conv0 + ReLU + depthwise conv1 (Parakeet::subsample's first two convolutions,
// src/parakeet.rs:937-941). One CTA per span of kSubRows output time steps t2: it stages the
// feature rows the span reads once, then for each block of kSubCh channels computes conv0 + ReLU
// for the t1 rows the span needs into shared memory (2 x kSubRows + 1 rows, so about 1/8 of conv0
// is computed twice across neighbouring spans) and the depthwise conv from there. Thread =
// (channel, group of positions); each thread keeps its channel's 9 taps in registers.
__global__ void __launch_bounds__(256) sub_front_kernel(const float* __restrict__ feats, int f0,
                                                        const SubTask* __restrict__ tasks, int ch,
                                                        const float* __restrict__ w0, const float* __restrict__ b0,
                                                        const float* __restrict__ w1, const float* __restrict__ b1,
                                                        float* __restrict__ out) {
    extern __shared__ float smf[];
    const SubTask t = tasks[blockIdx.x];
    const int c = threadIdx.x % kSubCh, grp = threadIdx.x / kSubCh;
    constexpr int kGroups = 256 / kSubCh;
    const int f1n = (f0 - 1) / 2 + 1, f2n = (f1n - 1) / 2 + 1;
    const int t1n = (t.t0 - 1) / 2 + 1;
    const int t1_base = max(0, 2 * t.t2_first - 1);
    const int t1_last = min(t1n - 1, 2 * (t.t2_first + t.t2_count - 1) + 1);
    const int t1_rows = t1_last - t1_base + 1;
    const int t0_base = max(0, 2 * t1_base - 1);
    const int t0_last = min(t.t0 - 1, 2 * t1_last + 1);
    const int t0_rows = t0_last - t0_base + 1;
    float* stage = smf;                                  // [t0_rows][f0]
    float* h1 = smf + (4 * kSubRows + 3) * f0;           // [t1_rows][f1n][kSubCh]
    for (int i = threadIdx.x; i < t0_rows * f0; i += 256)
        stage[i] = feats[static_cast<int64_t>(t.feat_row + t0_base) * f0 + i];
    for (int c0 = 0; c0 < ch; c0 += kSubCh) {
        const bool live = c0 + c < ch;
        float w[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = live ? w0[k * ch + c0 + c] : 0.0f;
        const float bias0 = live ? b0[c0 + c] : 0.0f;
        __syncthreads();
        // conv0 + ReLU: h1[t1][f1][c], row by row (no index division), frequencies strided by group.
        for (int r = 0; r < t1_rows; ++r) {
            const int t1 = t1_base + r;
            const float* rows[3];
            bool ok[3];
#pragma unroll
            for (int dt = 0; dt < 3; ++dt) {
                const int t0 = 2 * t1 + dt - 1;
                ok[dt] = t0 >= 0 && t0 < t.t0;
                rows[dt] = stage + (ok[dt] ? t0 - t0_base : 0) * f0;
            }
            float* hrow = h1 + r * f1n * kSubCh + c;
            for (int f1 = grp; f1 < f1n; f1 += kGroups) {
                float o = bias0;
#pragma unroll
                for (int dt = 0; dt < 3; ++dt) {
                    if (!ok[dt]) continue;
#pragma unroll
                    for (int df = 0; df < 3; ++df) {
                        const int ff = 2 * f1 + df - 1;
                        if (ff < 0 || ff >= f0) continue;
                        o = madd(o, w[dt * 3 + df], rows[dt][ff]);
                    }
                }
                hrow[f1 * kSubCh] = fmaxf(o, 0.0f);
            }
        }
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = live ? w1[k * ch + c0 + c] : 0.0f;
        const float bias1 = live ? b1[c0 + c] : 0.0f;
        __syncthreads();
        // Depthwise conv1: out[t2][f2][c]
        for (int r = 0; r < t.t2_count; ++r) {
            const int t2 = t.t2_first + r;
            const float* rows[3];
            bool ok[3];
#pragma unroll
            for (int dt = 0; dt < 3; ++dt) {
                const int t1 = 2 * t2 + dt - 1;
                ok[dt] = t1 >= 0 && t1 < t1n;
                rows[dt] = h1 + (ok[dt] ? t1 - t1_base : 0) * f1n * kSubCh + c;
            }
            float* orow = out + (static_cast<int64_t>(t.out_row) + static_cast<int64_t>(r) * f2n) * ch + c0 + c;
            for (int f2 = grp; f2 < f2n; f2 += kGroups) {
                float acc = bias1;
#pragma unroll
                for (int dt = 0; dt < 3; ++dt) {
                    if (!ok[dt]) continue;
#pragma unroll
                    for (int df = 0; df < 3; ++df) {
                        const int f1 = 2 * f2 + df - 1;
                        if (f1 < 0 || f1 >= f1n) continue;
                        acc = madd(acc, w[dt * 3 + df], rows[dt][f1 * kSubCh]);
                    }
                }
                if (live) orow[static_cast<int64_t>(f2) * ch] = acc;
            }
        }
        __syncthreads();  // the next channel block's conv0 overwrites h1
    }
}

// Depthwise 3x3 stride-2 convolution over [t_in, f_in, ch] rows of one utterance (conv3x3s2_row
// with depthwise, src/kernels/scalar.rs:194-232). One CTA per (task, block of kSubCh channels);
// thread = (channel, group of output positions) with the channel's 9 taps in registers, so each
// warp reads 32 consecutive channels of one input position per tap.
__global__ void __launch_bounds__(256) dw3x3s2_kernel(const float* __restrict__ in, int f_in, const SubTask* __restrict__ tasks,
                                                      int ch, const float* __restrict__ w, const float* __restrict__ b,
                                                      float* __restrict__ out) {
    const SubTask t = tasks[blockIdx.x];
    const int c = blockIdx.y * kSubCh + threadIdx.x % kSubCh, grp = threadIdx.x / kSubCh;
    constexpr int kGroups = 256 / kSubCh;
    if (c >= ch) return;
    const int f_out = (f_in - 1) / 2 + 1;
    const int t_in = t.t0;
    float wr[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) wr[k] = w[k * ch + c];
    const float bias = b[c];
    const float* src = in + static_cast<int64_t>(t.feat_row) * ch + c;
    for (int r = 0; r < t.t2_count; ++r) {
        const int to = t.t2_first + r;
        const float* rows[3];
        bool ok[3];
#pragma unroll
        for (int dt = 0; dt < 3; ++dt) {
            const int ti = 2 * to + dt - 1;
            ok[dt] = ti >= 0 && ti < t_in;
            rows[dt] = src + static_cast<int64_t>(ok[dt] ? ti : 0) * f_in * ch;
        }
        float* orow = out + (static_cast<int64_t>(t.out_row) + static_cast<int64_t>(r) * f_out) * ch + c;
        for (int fo = grp; fo < f_out; fo += kGroups) {
            float acc = bias;
#pragma unroll
            for (int dt = 0; dt < 3; ++dt) {
                if (!ok[dt]) continue;
#pragma unroll
                for (int df = 0; df < 3; ++df) {
                    const int fi = 2 * fo + df - 1;
                    if (fi < 0 || fi >= f_in) continue;
                    acc = madd(acc, wr[dt * 3 + df], __ldg(rows[dt] + static_cast<int64_t>(fi) * ch));
                }
            }
            orow[static_cast<int64_t>(fo) * ch] = acc;
        }
    }
}

// positions (src/parakeet.rs:1618-1630): row r of [2t - 1, d] is position t - 1 - r, sine and
// cosine interleaved. A row depends only on its position, so the table of a shorter utterance
// of t' frames is rows t - t' .. t + t' - 2 of this one.
__global__ void positions_kernel(int t, int d, float* __restrict__ out) {
    const int r = blockIdx.x;
    if (r >= 2 * t - 1) return;
    const double p = static_cast<double>(t) - 1.0 - static_cast<double>(r);
    float* row = out + static_cast<int64_t>(r) * d;
    const double lg = log(10000.0) / static_cast<double>(d);
    for (int i = threadIdx.x; i < d / 2; i += blockDim.x) {
        const double freq = exp(-static_cast<double>(2 * i) * lg);
        const double angle = p * freq;
        row[2 * i] = static_cast<float>(sin(angle));
        row[2 * i + 1] = static_cast<float>(cos(angle));
    }
}

// Transformer-XL attention of one head over one utterance, for 32 query rows per CTA:
//   S[i][j] = ((q_i + u) . k_j + (q_i + v) . p_{t-1-i+j}) * scale,  P = softmax_j(S),  O = P . V
// with p the projected position rows of the utterance (2t - 1 of them). 256 threads; S lives in
// shared memory ([32][t]); K, positions and V pass through in chunks of 32 rows.
template <int HD>
__global__ void __launch_bounds__(256) txl_attention_kernel(const float* __restrict__ qkv, const float* __restrict__ pp,
                                                            const TxlTask* __restrict__ tasks, int heads,
                                                            const float* __restrict__ bias_u,
                                                            const float* __restrict__ bias_v, float scale,
                                                            float* __restrict__ att) {
    constexpr int R = 32, CH = 32;
    extern __shared__ float sm[];
    const TxlTask task = tasks[blockIdx.x];
    const int h = blockIdx.y;
    const int t = task.len, i0 = task.q_first;
    const int rows = min(R, t - i0);
    const int D = heads * HD;
    const int64_t ld = 3 * static_cast<int64_t>(D);
    const float* base = qkv + static_cast<int64_t>(task.row) * ld + h * HD;
    const float* pbase = pp + static_cast<int64_t>(task.pos_row) * D + h * HD;
    const int tp = (t + 3) / 4 * 4;  // pitch of S
    float* qu = sm;                  // [R][HD + 1]
    float* qv = qu + R * (HD + 1);   // [R][HD + 1]
    float* chunk = qv + R * (HD + 1);  // [CH][HD + 1]
    float* S = chunk + CH * (HD + 1);  // [R][tp]
    const int tid = threadIdx.x;

    for (int e = tid; e < R * HD; e += 256) {
        const int r = e / HD, dd = e % HD;
        float q = r < rows ? base[static_cast<int64_t>(i0 + r) * ld + dd] : 0.0f;
        qu[r * (HD + 1) + dd] = __fadd_rn(q, bias_u[h * HD + dd]);
        qv[r * (HD + 1) + dd] = __fadd_rn(q, bias_v[h * HD + dd]);
    }
    // Each thread computes 4 (row, column) pairs of a 32 x 32 output chunk.
    const int cr = tid / 8;         // row 0..31
    const int cc = (tid % 8) * 4;   // columns cc .. cc + 3

    // ---- content scores against every key ----------------------------------------------------
    for (int j0 = 0; j0 < t; j0 += CH) {
        __syncthreads();
        for (int e = tid; e < CH * HD; e += 256) {
            const int j = e / HD, dd = e % HD;
            chunk[j * (HD + 1) + dd] = j0 + j < t ? base[static_cast<int64_t>(j0 + j) * ld + D + dd] : 0.0f;
        }
        __syncthreads();
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        const float* q = qu + cr * (HD + 1);
        for (int dd = 0; dd < HD; ++dd) {
            const float qd = q[dd];
            a0 = __fmaf_rn(qd, chunk[(cc + 0) * (HD + 1) + dd], a0);
            a1 = __fmaf_rn(qd, chunk[(cc + 1) * (HD + 1) + dd], a1);
            a2 = __fmaf_rn(qd, chunk[(cc + 2) * (HD + 1) + dd], a2);
            a3 = __fmaf_rn(qd, chunk[(cc + 3) * (HD + 1) + dd], a3);
        }
        const float a[4] = {a0, a1, a2, a3};
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (j0 + cc + e < t) S[cr * tp + j0 + cc + e] = a[e];
    }
    // ---- position scores: row i reads position index t - 1 - i + j ------------------------------
    // The block's rows need indices from t - 1 - (i0 + rows - 1) to t - 1 - i0 + t - 1.
    const int p_lo = t - 1 - (i0 + rows - 1), p_hi = 2 * t - 2 - i0;
    for (int p0 = p_lo; p0 <= p_hi; p0 += CH) {
        __syncthreads();
        for (int e = tid; e < CH * HD; e += 256) {
            const int j = e / HD, dd = e % HD;
            chunk[j * (HD + 1) + dd] = p0 + j <= p_hi ? pbase[static_cast<int64_t>(p0 + j) * D + dd] : 0.0f;
        }
        __syncthreads();
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        const float* q = qv + cr * (HD + 1);
        for (int dd = 0; dd < HD; ++dd) {
            const float qd = q[dd];
            a0 = __fmaf_rn(qd, chunk[(cc + 0) * (HD + 1) + dd], a0);
            a1 = __fmaf_rn(qd, chunk[(cc + 1) * (HD + 1) + dd], a1);
            a2 = __fmaf_rn(qd, chunk[(cc + 2) * (HD + 1) + dd], a2);
            a3 = __fmaf_rn(qd, chunk[(cc + 3) * (HD + 1) + dd], a3);
        }
        const float a[4] = {a0, a1, a2, a3};
        const int i = i0 + cr;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int pidx = p0 + cc + e;
            const int j = pidx - (t - 1 - i);
            if (cr < rows && pidx <= p_hi && j >= 0 && j < t)
                S[cr * tp + j] = __fmul_rn(__fadd_rn(S[cr * tp + j], a[e]), scale);
        }
    }
    __syncthreads();
    // ---- softmax per row (8 warps x 4 rows) ------------------------------------------------------
    const int warp = tid / 32, lane = tid % 32;
    for (int r = warp; r < R; r += 8) {
        if (r >= rows) continue;
        float* row = S + r * tp;
        float mx = -INFINITY;
        for (int j = lane; j < t; j += 32) mx = fmaxf(mx, row[j]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        double sum = 0.0;
        for (int j = lane; j < t; j += 32) {
            const float e = expf(__fsub_rn(row[j], mx));
            row[j] = e;
            sum += static_cast<double>(e);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
        const float inv = static_cast<float>(1.0 / sum);
        for (int j = lane; j < t; j += 32) row[j] = __fmul_rn(row[j], inv);
    }
    // ---- O = P . V over ascending keys: each thread owns (row cr, 4 columns per 32-column group) --
    constexpr int G = HD / 32;
    float o[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.0f;
    for (int j0 = 0; j0 < t; j0 += CH) {
        __syncthreads();
        for (int e = tid; e < CH * HD; e += 256) {
            const int j = e / HD, dd = e % HD;
            chunk[j * (HD + 1) + dd] = j0 + j < t ? base[static_cast<int64_t>(j0 + j) * ld + 2 * D + dd] : 0.0f;
        }
        __syncthreads();
        const int jn = min(CH, t - j0);
        for (int j = 0; j < jn; ++j) {
            const float pj = S[cr * tp + j0 + j];
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[g][e] = __fmaf_rn(pj, chunk[j * (HD + 1) + g * 32 + cc + e], o[g][e]);
        }
    }
    if (cr < rows) {
        float* orow = att + static_cast<int64_t>(task.row + i0 + cr) * D + h * HD;
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < 4; ++e) orow[g * 32 + cc + e] = o[g][e];
    }
}

// ---- greedy TDT steps (decode_inner, src/parakeet.rs:1412-1513) --------------------------------
//
// One decoding pass is four of these per-utterance kernels around four matrix products:
// joint_prep (commit the last prediction, z = relu(enc_proj[t] + pred), quantize z) -> joint
// product -> decide_prep (token and duration, the state step, the LSTM input [emb(token) | h0]
// quantized) -> LSTM product -> cell_prep (cell update, the next layer's input or the top
// hidden state quantized) -> ... -> pred_proj product. Every row is quantized by the rule of
// quantize_x2 (quant.cu), so the products see the same operands as before the fusion.

// Split-int8 quantization (the rule of quantize_x2) of a row of k values staged in shared memory,
// by a CTA of 128 threads; the row's padding up to ld is zeroed.
__device__ void quantize_row_cta(const float* row, int k, int64_t ld, int8_t* hi, int8_t* lo, float* scale,
                                 float* red) {
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    float amax = 0.0f;
    for (int i = tid; i < k; i += 128) amax = fmaxf(amax, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float id_lo = __fmul_rn(id, 254.0f);
    for (int i = tid; i < k; i += 128) quant_split_one(row[i], d, id, id_lo, hi[i], lo[i]);
    for (int i = k + tid; i < ld; i += 128) hi[i] = lo[i] = 0;
    if (tid == 0) *scale = d;
    __syncthreads();
}

__device__ __forceinline__ float sigmoid_ref(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// The start of decoding (initial_decoder_state, src/parakeet.rs:1321-1336): every utterance
// feeds the blank token to a zero LSTM state, so its layer-0 input is [emb(blank) | 0].
__global__ void __launch_bounds__(128) tdt_start_kernel(int n_utt, int blank, int h, const float* __restrict__ embedding,
                                                        int* __restrict__ predict_token, QuantAct q) {
    extern __shared__ float row[];
    __shared__ float red[4];
    const int u = blockIdx.x;
    if (u >= n_utt) return;
    if (threadIdx.x == 0) predict_token[u] = blank;
    for (int j = threadIdx.x; j < h; j += 128) {
        row[j] = embedding[static_cast<int64_t>(blank) * h + j];
        row[h + j] = 0.0f;
    }
    __syncthreads();
    quantize_row_cta(row, 2 * h, q.ld, q.hi + static_cast<int64_t>(u) * q.ld, q.lo + static_cast<int64_t>(u) * q.ld,
                     q.scale + u, red);
}

// pred = fresh for the utterances that predicted last pass; then z = relu(enc_proj[t] + pred)
// for the utterances still decoding (zeros for the others), quantized.
__global__ void __launch_bounds__(128) tdt_joint_prep_kernel(const float* __restrict__ enc_proj,
                                                             const TdtState* __restrict__ st, int n_utt, int h,
                                                             const int* __restrict__ predict_token,
                                                             const float* __restrict__ fresh, float* __restrict__ pred,
                                                             QuantAct q, int* __restrict__ active) {
    extern __shared__ float row[];
    __shared__ float red[4];
    const int u = blockIdx.x;
    if (u >= n_utt) return;
    if (u == 0 && threadIdx.x == 0) *active = 0;
    const TdtState s = st[u];
    const bool commit = predict_token[u] >= 0;
    const bool live = s.t < s.frames;
    float* pu = pred + static_cast<int64_t>(u) * h;
    const float* fu = fresh + static_cast<int64_t>(u) * h;
    if (live) {
        const float* e = enc_proj + (static_cast<int64_t>(s.enc_first) + s.t) * h;
        for (int j = threadIdx.x; j < h; j += 128) {
            float p = pu[j];
            if (commit) {
                p = fu[j];
                pu[j] = p;
            }
            row[j] = fmaxf(__fadd_rn(e[j], p), 0.0f);
        }
    } else {
        for (int j = threadIdx.x; j < h; j += 128) {
            if (commit) pu[j] = fu[j];
            row[j] = 0.0f;
        }
    }
    __syncthreads();
    quantize_row_cta(row, h, q.ld, q.hi + static_cast<int64_t>(u) * q.ld, q.lo + static_cast<int64_t>(u) * q.ld,
                     q.scale + u, red);
}

// The token and duration choices of one joint step and the state machine after them: blank ->
// advance by max(duration, 1); a token -> emit it, predict next, advance by its duration or,
// for duration 0, count symbols on this frame up to max_symbols. A predicting utterance's LSTM
// layer-0 input [emb(token) | h0] is quantized for the next product.
__global__ void __launch_bounds__(128) tdt_decide_prep_kernel(
    const float* __restrict__ logits, int64_t ld, int vocab, int blank, const int* __restrict__ durations, int n_dur,
    int max_symbols, TdtState* __restrict__ st, int n_utt, uint32_t* __restrict__ tokens,
    int* __restrict__ predict_token, int* __restrict__ active, const float* __restrict__ embedding,
    const float* __restrict__ state, int h, int layers, QuantAct q) {
    extern __shared__ float row[];
    __shared__ float red[4];
    __shared__ float bv[4];
    __shared__ int bi_sh[4];
    __shared__ int tok_sh;
    const int u = blockIdx.x;
    if (u >= n_utt) return;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    TdtState s = st[u];
    if (s.t >= s.frames) {
        if (tid == 0) predict_token[u] = -1;
        return;
    }
    const float* r = logits + static_cast<int64_t>(u) * ld;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < vocab; i += 128) {
        const float v = r[i];
        if (v > best) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, best, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
        bv[warp] = best;
        bi_sh[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        // The first maximum over the four warps' winners: lowest index on ties.
        float bb = bv[0];
        int ii = bi_sh[0];
        for (int w = 1; w < 4; ++w)
            if (bv[w] > bb || (bv[w] == bb && bi_sh[w] < ii)) { bb = bv[w]; ii = bi_sh[w]; }
        int di = 0;
        for (int i = 1; i < n_dur; ++i)
            if (r[vocab + i] > r[vocab + di]) di = i;
        const int duration = durations[di];
        int tok = -1;
        if (ii == blank) {
            s.t += duration > 1 ? duration : 1;
            s.on_frame = 0;
        } else {
            uint32_t* out = tokens + 3 * static_cast<int64_t>(s.tok_first + s.count);
            out[0] = static_cast<uint32_t>(ii);
            out[1] = static_cast<uint32_t>(s.t);
            out[2] = static_cast<uint32_t>(duration);
            s.count += 1;
            tok = ii;
            if (duration > 0) {
                s.t += duration;
                s.on_frame = 0;
            } else {
                s.on_frame += 1;
                if (s.on_frame >= max_symbols) {
                    s.t += 1;
                    s.on_frame = 0;
                }
            }
        }
        st[u] = s;
        predict_token[u] = tok;
        tok_sh = tok;
        if (s.t < s.frames) atomicAdd(active, 1);
    }
    __syncthreads();
    const int tok = tok_sh;
    if (tok < 0) return;
    const float* h0 = state + static_cast<int64_t>(u) * layers * 2 * h;
    for (int j = tid; j < h; j += 128) {
        row[j] = embedding[static_cast<int64_t>(tok) * h + j];
        row[h + j] = h0[j];
    }
    __syncthreads();
    quantize_row_cta(row, 2 * h, q.ld, q.hi + static_cast<int64_t>(u) * q.ld, q.lo + static_cast<int64_t>(u) * q.ld,
                     q.scale + u, red);
}

// c = f c + i g, h = o tanh(c) for layer `layer` of the predicting utterances; then the next
// layer's input [h_layer | h_(layer+1)] or, after the top layer, h_top, quantized.
__global__ void __launch_bounds__(128) lstm_cell_prep_kernel(const int* __restrict__ predict_token, int n_utt, int h,
                                                             int layer, int layers, const float* __restrict__ gates,
                                                             float* __restrict__ state, QuantAct q) {
    extern __shared__ float row[];
    __shared__ float red[4];
    const int u = blockIdx.x;
    if (u >= n_utt || predict_token[u] < 0) return;
    const float* g = gates + static_cast<int64_t>(u) * 4 * h;
    float* base = state + static_cast<int64_t>(u) * layers * 2 * h;
    float* hs = base + layer * 2 * h;
    float* cs = hs + h;
    const bool top = layer + 1 == layers;
    for (int j = threadIdx.x; j < h; j += 128) {
        const float i = sigmoid_ref(g[j]);
        const float f = sigmoid_ref(g[h + j]);
        const float gg = tanhf(g[2 * h + j]);
        const float o = sigmoid_ref(g[3 * h + j]);
        const float c = __fadd_rn(__fmul_rn(f, cs[j]), __fmul_rn(i, gg));
        const float hn = __fmul_rn(o, tanhf(c));
        cs[j] = c;
        hs[j] = hn;
        row[j] = hn;
        if (!top) row[h + j] = base[(layer + 1) * 2 * h + j];
    }
    __syncthreads();
    quantize_row_cta(row, top ? h : 2 * h, q.ld, q.hi + static_cast<int64_t>(u) * q.ld,
                     q.lo + static_cast<int64_t>(u) * q.ld, q.scale + u, red);
}

// ---- the networks the biased beam search reads (src/parakeet.rs:1641-1676) --------------------

// q row r = relu(enc_row + preds[r]), one CTA per prediction row (TdtNetwork::joint, :1653-1670).
__global__ void __launch_bounds__(128) tdt_joint_rows_kernel(const float* __restrict__ enc_row,
                                                             const float* __restrict__ preds, int rows, int h,
                                                             QuantAct q) {
    extern __shared__ float row[];
    __shared__ float red[4];
    const int r = blockIdx.x;
    if (r >= rows) return;
    const float* p = preds + static_cast<int64_t>(r) * h;
    for (int j = threadIdx.x; j < h; j += 128) row[j] = fmaxf(__fadd_rn(enc_row[j], p[j]), 0.0f);
    __syncthreads();
    quantize_row_cta(row, h, q.ld, q.hi + static_cast<int64_t>(r) * q.ld, q.lo + static_cast<int64_t>(r) * q.ld,
                     q.scale + r, red);
}

// q row r = [emb(tokens[r]) | h_0 of state row r], the first LSTM layer's input (predict_rows).
__global__ void __launch_bounds__(128) tdt_predict_input_kernel(const int* __restrict__ tokens, int rows, int h,
                                                                int layers, const float* __restrict__ embedding,
                                                                const float* __restrict__ states, QuantAct q) {
    extern __shared__ float row[];
    __shared__ float red[4];
    const int r = blockIdx.x;
    if (r >= rows) return;
    const float* e = embedding + static_cast<int64_t>(tokens[r]) * h;
    const float* h0 = states + static_cast<int64_t>(r) * layers * 2 * h;
    for (int j = threadIdx.x; j < h; j += 128) {
        row[j] = e[j];
        row[h + j] = h0[j];
    }
    __syncthreads();
    quantize_row_cta(row, 2 * h, q.ld, q.hi + static_cast<int64_t>(r) * q.ld, q.lo + static_cast<int64_t>(r) * q.ld,
                     q.scale + r, red);
}

// Moves each utterance's tokens from its worst-case slot (3 * tok_first words in) to the prefix
// sum of the counts before it; counts[u] gets its count and *total the sum. One CTA: thread 0
// forms the prefix sums in `offsets`, then every warp copies whole utterances.
__global__ void __launch_bounds__(1024) tdt_compact_kernel(const uint32_t* __restrict__ raw,
                                                           const TdtState* __restrict__ st, int n_utt,
                                                           int* __restrict__ offsets, uint32_t* __restrict__ out,
                                                           int* __restrict__ counts, int* __restrict__ total) {
    if (threadIdx.x == 0) {
        int at = 0;
        for (int u = 0; u < n_utt; ++u) {
            offsets[u] = at;
            at += st[u].count;
        }
        *total = at;
    }
    __syncthreads();
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    for (int u = warp; u < n_utt; u += blockDim.x / 32) {
        const TdtState s = st[u];
        const uint32_t* src = raw + 3 * static_cast<int64_t>(s.tok_first);
        uint32_t* dst = out + 3 * static_cast<int64_t>(offsets[u]);
        for (int i = lane; i < 3 * s.count; i += 32) dst[i] = src[i];
        if (lane == 0) counts[u] = s.count;
    }
}

// ---- launchers ---------------------------------------------------------------------------------

size_t sub_front_smem(int f0) {
    const int f1 = (f0 - 1) / 2 + 1;
    return sizeof(float) * ((4 * kSubRows + 3) * f0 + (2 * kSubRows + 1) * f1 * kSubCh);
}

cudaError_t sub_front(const float* feats, int f0, const SubTask* tasks, int n_tasks, int ch, const float* w0,
                      const float* b0, const float* w1, const float* b1, float* out, cudaStream_t s) {
    if (n_tasks <= 0) return cudaSuccess;
    const size_t smem = sub_front_smem(f0);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    const cudaError_t e =
        cudaFuncSetAttribute(sub_front_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    sub_front_kernel<<<n_tasks, 256, smem, s>>>(feats, f0, tasks, ch, w0, b0, w1, b1, out);
    return cudaGetLastError();
}

cudaError_t dw3x3s2(const float* in, int f_in, const SubTask* tasks, int n_tasks, int ch, const float* w,
                    const float* b, float* out, cudaStream_t s) {
    if (n_tasks <= 0) return cudaSuccess;
    dim3 grid(n_tasks, (ch + kSubCh - 1) / kSubCh);
    dw3x3s2_kernel<<<grid, 256, 0, s>>>(in, f_in, tasks, ch, w, b, out);
    return cudaGetLastError();
}

cudaError_t positions(int t, int d, float* out, cudaStream_t s) {
    if (t <= 0) return cudaSuccess;
    positions_kernel<<<2 * t - 1, 128, 0, s>>>(t, d, out);
    return cudaGetLastError();
}

size_t txl_attention_smem(int hd, int max_t) {
    return sizeof(float) * (2 * 32 * (hd + 1) + 32 * (hd + 1) + 32 * ((max_t + 3) / 4 * 4));
}

cudaError_t txl_attention(const float* qkv, const float* pp, const TxlTask* tasks, int n_tasks, int heads, int hd,
                          int max_t, const float* bias_u, const float* bias_v, float scale, float* att,
                          cudaStream_t s) {
    if (n_tasks <= 0) return cudaSuccess;
    const size_t smem = txl_attention_smem(hd, max_t);
    dim3 grid(n_tasks, heads);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    auto launch = [&](auto kernel) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        kernel<<<grid, 256, smem, s>>>(qkv, pp, tasks, heads, bias_u, bias_v, scale, att);
        return cudaGetLastError();
    };
    switch (hd) {
        case 32: return launch(txl_attention_kernel<32>);
        case 64: return launch(txl_attention_kernel<64>);
        case 128: return launch(txl_attention_kernel<128>);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t tdt_start(int n_utt, int blank, int h, const float* embedding, int* predict_token, const QuantAct& q,
                      cudaStream_t s) {
    if (n_utt <= 0) return cudaSuccess;
    tdt_start_kernel<<<n_utt, 128, sizeof(float) * 2 * h, s>>>(n_utt, blank, h, embedding, predict_token, q);
    return cudaGetLastError();
}

cudaError_t tdt_joint_prep(const float* enc_proj, const TdtState* st, int n_utt, int h, const int* predict_token,
                           const float* fresh, float* pred, const QuantAct& q, int* active, cudaStream_t s) {
    if (n_utt <= 0) return cudaSuccess;
    tdt_joint_prep_kernel<<<n_utt, 128, sizeof(float) * h, s>>>(enc_proj, st, n_utt, h, predict_token, fresh, pred, q,
                                                                 active);
    return cudaGetLastError();
}

cudaError_t tdt_decide_prep(const float* logits, int64_t ld, int vocab, int blank, const int* durations, int n_dur,
                            int max_symbols, TdtState* st, int n_utt, uint32_t* tokens, int* predict_token, int* active,
                            const float* embedding, const float* state, int h, int layers, const QuantAct& q,
                            cudaStream_t s) {
    if (n_utt <= 0) return cudaSuccess;
    tdt_decide_prep_kernel<<<n_utt, 128, sizeof(float) * 2 * h, s>>>(logits, ld, vocab, blank, durations, n_dur,
                                                                      max_symbols, st, n_utt, tokens, predict_token,
                                                                      active, embedding, state, h, layers, q);
    return cudaGetLastError();
}

cudaError_t lstm_cell_prep(const int* predict_token, int n_utt, int h, int layer, int layers, const float* gates,
                           float* state, const QuantAct& q, cudaStream_t s) {
    if (n_utt <= 0) return cudaSuccess;
    lstm_cell_prep_kernel<<<n_utt, 128, sizeof(float) * 2 * h, s>>>(predict_token, n_utt, h, layer, layers, gates,
                                                                     state, q);
    return cudaGetLastError();
}

cudaError_t tdt_joint_rows(const float* enc_row, const float* preds, int rows, int h, const QuantAct& q,
                           cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    tdt_joint_rows_kernel<<<rows, 128, sizeof(float) * h, s>>>(enc_row, preds, rows, h, q);
    return cudaGetLastError();
}

cudaError_t tdt_predict_input(const int* tokens, int rows, int h, int layers, const float* embedding,
                              const float* states, const QuantAct& q, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    tdt_predict_input_kernel<<<rows, 128, sizeof(float) * 2 * h, s>>>(tokens, rows, h, layers, embedding, states, q);
    return cudaGetLastError();
}

cudaError_t tdt_compact(const uint32_t* raw, const TdtState* st, int n_utt, int* offsets, uint32_t* out, int* counts,
                        int* total, cudaStream_t s) {
    tdt_compact_kernel<<<1, 1024, 0, s>>>(raw, st, n_utt, offsets, out, counts, total);
    return cudaGetLastError();
}


}  // namespace telmo
