// tdt_persistent.cu -- greedy TDT decoding of a batch of utterances as one persistent kernel.
//
// The whole of decode_inner (src/parakeet.rs:1412-1513) with predict_rows (:1523-1577) for every
// utterance of the batch runs inside one cooperative launch of one CTA per SM. The prediction
// and joint networks' int8 weights (joint, every LSTM layer, pred_proj: about 12 MB at the
// benchmark's shape) are spread over the CTAs in units of 8 output rows and stay in shared
// memory for the whole decode, so a pass streams only the activations. Each pass is
//
//   joint    logits of every live utterance; the token and duration argmax folded into the
//            product's epilogue (a packed (value, index) maximum per row, atomically combined)
//   decide   the TDT state step per live utterance; a predicting one quantizes [emb(token) | h_0]
//   lstm l   gates of the predicting utterances            } for every layer l
//   cell l   c, h update; the next layer's input quantized  }
//   pred     pred_proj of the top hidden state
//   prepare  commit the new projections; z = relu(enc_proj[t] + pred) of every utterance still
//            decoding, quantized for the next pass's joint product
//
// with a grid barrier between the phases. The products are exact int8 x int8 -> s32 mma.sync
// sums of the split activations (x = s (hi + lo / 254), the rule of quantize_x2) and use the
// tcgen05 GEMM's epilogue arithmetic, so every logit, gate and projection, and with them every
// token, is bit-identical to the launch-per-phase decoder (parakeet_kernels.cu). Rows are
// compacted to the live (or predicting) utterances, so finished utterances cost nothing.
//
// Every wait is bounded: a grid barrier that has not completed within about a second records
// kTdtErrBarrier and every CTA returns; more passes than the host's bound record kTdtErrPasses.
#include "parakeet_kernels.h"

#include <cmath>
#include <cstdint>

namespace telmo {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 64;  // k granularity of the products (and of the smem row padding)
// A warp's ring: `stages` stages of 16 rows x CH k bytes in both planes (CH = 128 where every
// k is a multiple of 128, else 64); the CTA's ring is kWarps of them.
constexpr int kWarpRing = 16 * 1024;  // bytes per warp: 8 stages of 64 or 4 of 128
constexpr uint64_t kBarrierNs = 1000000000ull;      // one second

constexpr unsigned kFull = 0xffffffffu;

// words[]: the error code, passes run, the grid barrier's arrivals, (unused), the number of
// predicting rows, and the two live counts (by pass parity).
enum { kWErr = 0, kWPasses = 1, kWBarCount = 2, kWPred = 4, kWLive = 5 };

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void cp16_cg(void* dst, const void* src) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint4 lds128(const int8_t* p) {
    uint4 v;
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

// d += a . b over k = 32 (exact s32 sums).
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The tcgen05 GEMM's epilogue for act none and scale 1: ((float)hi + (float)lo / 254) * rs * ws
// + bias, each step rounded on its own.
__device__ __forceinline__ float epilogue(int hi, int lo, float rs, float ws, float bias) {
    const float inv254 = 1.0f / 254.0f;
    float v = __fadd_rn(__int2float_rn(hi), __fmul_rn(__int2float_rn(lo), inv254));
    v = __fmul_rn(v, rs);
    v = __fmul_rn(v, ws);
    return __fadd_rn(v, bias);
}

// A (value, index) pair ordered so that the unsigned maximum is the first maximum of the values
// (the largest value, the lowest index among equal ones). NaN never wins; -0 ties +0.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    if (v != v) v = -INFINITY;
    if (v == 0.0f) v = 0.0f;
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(u) << 32) | (0xffffffffu - static_cast<unsigned>(idx));
}
__device__ __forceinline__ int key_index(unsigned long long k) {
    return static_cast<int>(0xffffffffu - static_cast<unsigned>(k & 0xffffffffu));
}

__device__ __forceinline__ float sigmoid_ref(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

struct Smem {
    int8_t* w[kTdtMaxMats];  // this CTA's weight units per matrix
    int first[kTdtMaxMats];  // its first unit index per matrix (units first, first + G, ...)
    int units[kTdtMaxMats];
    int8_t* ring;
};

constexpr int kVals = 8;  // values per thread in the per-row phases: rows of up to 2048 values

// The CTA quantizes the k values it holds (thread t holds v[i] = value t + 256 i) into row `row`
// of the activation buffer, by the rule of quantize_x2: d = amax / 127, hi = round(x / d),
// lo = round((x - hi d) * 254 / d), clamped.
__device__ __forceinline__ void cta_quantize(const TdtPersistentArgs& a, int row, int k, const float (&v)[kVals],
                                             float* red) {
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kVals; ++i)
        if (tid + kThreads * i < k) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) amax = fmaxf(amax, red[w]);
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float id_lo = __fmul_rn(id, 254.0f);
    int8_t* hi = a.q_hi + static_cast<int64_t>(row) * a.q_ld;
    int8_t* lo = a.q_lo + static_cast<int64_t>(row) * a.q_ld;
#pragma unroll
    for (int i = 0; i < kVals; ++i) {
        const int j = tid + kThreads * i;
        if (j < k) quant_split_one(v[i], d, id, id_lo, hi[j], lo[j]);
    }
    if (tid == 0) a.q_scale[row] = d;
    __syncthreads();  // red[] is free again
}

// Grid barrier over all CTAs (a cooperative launch keeps them resident): every CTA adds one to
// a counter that only grows and waits until it reaches G times the barrier's number. A wait that
// runs past a second records kTdtErrBarrier and returns false; the CTA then leaves, and the
// others leave at their next barrier, whose waits are bounded the same way.
__device__ bool grid_sync(const TdtPersistentArgs& a, unsigned& gen) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned target = (gen + 1) * gridDim.x;
        unsigned* count = a.words + kWBarCount;
        __threadfence();
        if (gen != 0 || static_cast<int>(blockIdx.x) != a.withhold_cta) atomicAdd(count, 1u);
        const uint64_t t0 = global_ns();
        uint32_t polls = 0;
        int good = 1;
        while (static_cast<int>(ld_acquire(count) - target) < 0) {
            if (++polls > 1024) __nanosleep(64);
            if ((polls & 255) == 0 && global_ns() - t0 > kBarrierNs) {
                atomicCAS(a.words + kWErr, 0u, static_cast<unsigned>(kTdtErrBarrier));
                good = 0;
                break;
            }
        }
        ok = good;
    }
    __syncthreads();
    ++gen;
    return ok != 0;
}

// One product over `rows` activation rows of the buffer (k = mats[m].k) against this CTA's
// NU units of matrix m. Warp w takes the 16-row tiles w, w + 8, ... and streams each tile's rows
// (both planes, CH k bytes a chunk) through its own 16 KB ring with cp.async, so the warps never
// wait for one another. JOINT: no output; the token and duration maxima of each
// row go to the key arrays.
template <int NU, int CH, bool JOINT>
__device__ void product(const TdtPersistentArgs& a, const Smem& sm, int m, int rows, float* out, int64_t ldo) {
    constexpr int STAGES = kWarpRing / (2 * 16 * CH);
    constexpr int kStage = 2 * 16 * CH;  // one warp's stage
    constexpr int STEPS = CH / 32;       // k32 products per chunk
    const TdtMatrix& M = a.mats[m];
    if (rows == 0) return;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32, g = lane / 4, q = lane % 4;
    // CTA 0's warp 0 clocks the products: the whole (global timer), and in SM cycles the shares
    // spent waiting for staged rows and in epilogues.
    const bool clock = a.phase_ns && blockIdx.x == 0 && tid == 0;
    const uint64_t t_start = clock ? global_ns() : 0;
    const long long c_start = clock ? clock64() : 0;
    long long waited = 0, in_epilogue = 0;
    const int KC = M.k / CH;
    const int tiles = (rows + 15) / 16;
    const int my_tiles = tiles > warp ? (tiles - warp + kWarps - 1) / kWarps : 0;
    const int total = my_tiles * KC;
    const int stride = M.smem_stride;
    int8_t* ring = sm.ring + warp * kWarpRing;
    // Each CTA walks k from its own starting chunk, so the CTAs (which all read the same rows)
    // spread their requests over the rows' lines; the integer sums do not depend on the order.
    const int rot = blockIdx.x % KC;
    // Lane l copies the 16-byte pieces l % (CH / 16) + i (CH / 16) of the tile's rows in both
    // planes: consecutive lanes cover consecutive bytes of a row.
    constexpr int kSegs = CH / 16;            // 16-byte pieces per row and chunk
    constexpr int kRowsPerPass = 32 / kSegs;  // rows one warp-wide copy covers
    // With 128-byte rows the two 64-byte halves of odd rows trade places, so the fragment reads
    // of rows g and g + 1 fall on different banks.
    const int crow = lane / kSegs, cseg = (lane % kSegs) * 16;
    const int cswz = CH == 128 ? (((cseg >> 6) ^ (crow & 1)) << 6) | (cseg & 63) : cseg;
    int is_tile = warp, is_k = rot, is_n = 0;  // the next chunk to stage
    auto issue = [&]() {
        if (is_n < total) {
            int8_t* dst = ring + (is_n % STAGES) * kStage + crow * CH + cswz;
            const int8_t* src_h = a.q_hi + static_cast<int64_t>(is_tile * 16 + crow) * a.q_ld + is_k * CH + cseg;
            const int8_t* src_l = a.q_lo + (src_h - a.q_hi);
            const int lim = rows - is_tile * 16 - crow;
#pragma unroll
            for (int i = 0; i < 16 / kRowsPerPass; ++i) {
                if (i * kRowsPerPass < lim) {
                    cp16_cg(dst + i * kRowsPerPass * CH, src_h + static_cast<int64_t>(i * kRowsPerPass) * a.q_ld);
                    cp16_cg(dst + 16 * CH + i * kRowsPerPass * CH, src_l + static_cast<int64_t>(i * kRowsPerPass) * a.q_ld);
                }
            }
            if (++is_k == KC) is_k = 0;
            if (is_k == rot) is_tile += kWarps;
            ++is_n;
        }
        cp_commit();
    };

    // This thread's output columns (two per 8-row unit) with their scales and biases.
    float wsv[NU][2], bsv[NU][2];
#pragma unroll
    for (int j = 0; j < NU; ++j) {
        const int col0 = (sm.first[m] + j * static_cast<int>(gridDim.x)) * 8 + 2 * q;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const bool ok = col0 + e < M.n;
            wsv[j][e] = ok ? __ldg(M.ws + col0 + e) : 0.0f;
            bsv[j][e] = ok && M.bias ? __ldg(M.bias + col0 + e) : 0.0f;
        }
    }

    int acc_h[NU][4], acc_l[NU][4];
#pragma unroll
    for (int j = 0; j < NU; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc_h[j][e] = acc_l[j][e] = 0;

    for (int c = 0; c < STAGES - 1; ++c) issue();
    int tile = warp, kk = 0, kc = rot;  // the chunk to multiply: tile, position in its walk, k chunk
    // Weight rows hold their 16-byte segments XOR-swizzled (seg ^ xr): rows g and g + 1 of a
    // fragment read land in different halves of a 128-byte line.
    const int xr = stride % 128 == 0 ? (g & 1) << 2 : 0;
    const int8_t* wrow = sm.w[m] + g * stride;
    for (int c = 0; c < total; ++c) {
        const long long tw = clock ? clock64() : 0;
        cp_wait<STAGES - 2>();
        __syncwarp();
        if (clock) waited += clock64() - tw;
        issue();
        const int8_t* st = ring + (c % STAGES) * kStage + 16 * q;
#pragma unroll
        for (int p = 0; p < STEPS / 2; ++p) {  // 64 k bytes: two k32 products per plane
            const int8_t* wk = wrow + ((((kc * CH + 64 * p) >> 4) + q) ^ xr) * 16;
            uint4 b[NU];
#pragma unroll
            for (int j = 0; j < NU; ++j) b[j] = lds128(wk + j * 8 * stride);
            const int pa = CH == 128 ? 64 * (p ^ (g & 1)) : 64 * p;  // rows g and g + 8: same parity
            const uint4 h0 = lds128(st + g * CH + pa);
            const uint4 h1 = lds128(st + (g + 8) * CH + pa);
            const uint4 l0 = lds128(st + 16 * CH + g * CH + pa);
            const uint4 l1 = lds128(st + 16 * CH + (g + 8) * CH + pa);
#pragma unroll
            for (int j = 0; j < NU; ++j) {
                mma_s8(acc_h[j], h0.x, h1.x, h0.y, h1.y, b[j].x, b[j].y);
                mma_s8(acc_l[j], l0.x, l1.x, l0.y, l1.y, b[j].x, b[j].y);
            }
#pragma unroll
            for (int j = 0; j < NU; ++j) {
                mma_s8(acc_h[j], h0.z, h1.z, h0.w, h1.w, b[j].z, b[j].w);
                mma_s8(acc_l[j], l0.z, l1.z, l0.w, l1.w, b[j].z, b[j].w);
            }
        }
        if (++kc == KC) kc = 0;
        if (++kk == KC) {
            const long long te = clock ? clock64() : 0;
            const int r0 = tile * 16 + g;
            const float rs[2] = {__ldcg(a.q_scale + min(r0, rows - 1)), __ldcg(a.q_scale + min(r0 + 8, rows - 1))};
            unsigned long long tok[2] = {0ull, 0ull}, dur[2] = {0ull, 0ull};
#pragma unroll
            for (int j = 0; j < NU; ++j) {
                const int col0 = (sm.first[m] + j * static_cast<int>(gridDim.x)) * 8 + 2 * q;
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int row = r0 + 8 * rr;
                    float v[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e)
                        v[e] = epilogue(acc_h[j][2 * rr + e], acc_l[j][2 * rr + e], rs[rr], wsv[j][e], bsv[j][e]);
                    if (row >= rows) continue;
                    if (JOINT) {
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int n = col0 + e;
                            if (n < a.vocab) {
                                const unsigned long long k = argmax_key(v[e], n);
                                tok[rr] = k > tok[rr] ? k : tok[rr];
                            } else if (n < a.vocab + a.n_dur) {
                                const unsigned long long k = argmax_key(v[e], n - a.vocab);
                                dur[rr] = k > dur[rr] ? k : dur[rr];
                            }
                        }
                    } else {
                        float* o = out + static_cast<int64_t>(row) * ldo + col0;
                        if (col0 + 1 < M.n)
                            *reinterpret_cast<float2*>(o) = make_float2(v[0], v[1]);
                        else if (col0 < M.n)
                            o[0] = v[0];
                    }
                }
            }
            if (JOINT) {
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
                    for (int o = 1; o <= 2; o <<= 1) {
                        const unsigned long long t = __shfl_xor_sync(kFull, tok[rr], o);
                        const unsigned long long d = __shfl_xor_sync(kFull, dur[rr], o);
                        tok[rr] = t > tok[rr] ? t : tok[rr];
                        dur[rr] = d > dur[rr] ? d : dur[rr];
                    }
                    const int row = r0 + 8 * rr;
                    if (q == 0 && row < rows) {
                        if (tok[rr]) atomicMax(a.tok_key + row, tok[rr]);
                        if (dur[rr]) atomicMax(a.dur_key + row, dur[rr]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < NU; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc_h[j][e] = acc_l[j][e] = 0;
            kk = 0;
            tile += kWarps;
            if (clock) in_epilogue += clock64() - te;
        }
    }
    cp_wait<0>();
    __syncwarp();
    if (clock) {
        const uint64_t ns = global_ns() - t_start;
        const double cycles = static_cast<double>(clock64() - c_start);
        a.phase_ns[kTdtPhases] += ns;
        a.phase_ns[kTdtPhases + 1] += static_cast<uint64_t>(ns * (waited / cycles));
        a.phase_ns[kTdtPhases + 2] += static_cast<uint64_t>(ns * (in_epilogue / cycles));
    }
}

template <int CH, bool JOINT>
__device__ void product_units(const TdtPersistentArgs& a, const Smem& sm, int m, int rows, float* out, int64_t ldo) {
    switch (sm.units[m]) {
    case 0: break;
    case 1: product<1, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    case 2: product<2, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    case 3: product<3, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    case 4: product<4, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    case 5: product<5, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    case 6: product<6, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    case 7: product<7, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    default: product<8, CH, JOINT>(a, sm, m, rows, out, ldo); break;
    }
}

template <bool JOINT>
__device__ void product_any(const TdtPersistentArgs& a, const Smem& sm, int m, int rows, float* out, int64_t ldo) {
    if (a.chunk == 128)
        product_units<128, JOINT>(a, sm, m, rows, out, ldo);
    else
        product_units<64, JOINT>(a, sm, m, rows, out, ldo);
}

// The cell update of layer l for predicting row s, then that row's next operand: [h_l | h_(l+1)]
// below the top layer, h_top after it. One CTA per row.
__device__ void cell(const TdtPersistentArgs& a, int s, int l, float* red) {
    const int tid = threadIdx.x, h = a.h;
    const int u = __ldcg(a.plist + s);
    const float* gt = a.gates + static_cast<int64_t>(s) * 4 * h;
    float* base = a.state + static_cast<int64_t>(u) * a.layers * 2 * h;
    float* hs = base + l * 2 * h;
    float* cs = hs + h;
    const bool top = l + 1 == a.layers;
    const float* nx = base + (l + 1) * 2 * h;
    float v[kVals];
#pragma unroll
    for (int i = 0; i < kVals; ++i) {
        const int j = tid + kThreads * i;
        v[i] = 0.0f;
        if (j < h) {
            const float ig = sigmoid_ref(__ldcg(gt + j));
            const float fg = sigmoid_ref(__ldcg(gt + h + j));
            const float gg = tanhf(__ldcg(gt + 2 * h + j));
            const float og = sigmoid_ref(__ldcg(gt + 3 * h + j));
            const float c = __fadd_rn(__fmul_rn(fg, __ldcg(cs + j)), __fmul_rn(ig, gg));
            const float hn = __fmul_rn(og, tanhf(c));
            cs[j] = c;
            hs[j] = hn;
            v[i] = hn;
        } else if (!top && j < 2 * h) {
            v[i] = __ldcg(nx + j - h);
        }
    }
    cta_quantize(a, s, top ? h : 2 * h, v, red);
}

__global__ void __launch_bounds__(kThreads, 1) tdt_persistent_kernel(const __grid_constant__ TdtPersistentArgs a) {
    extern __shared__ __align__(128) int8_t smem[];
    const int tid = threadIdx.x;
    const int G = gridDim.x, cta = blockIdx.x;
    const int h = a.h, U = a.n_utt;
    // Phase clock (CTA 0, thread 0, when a.phase_ns is given): time from one barrier to the
    // next, barrier included, summed per phase kind.
    const bool clock = a.phase_ns && cta == 0 && tid == 0;
    uint64_t t_prev = clock ? global_ns() : 0, acc[kTdtPhases] = {};
    auto mark = [&](int phase) {
        if (clock) {
            const uint64_t t = global_ns();
            acc[phase] += t - t_prev;
            t_prev = t;
        }
    };
    unsigned gen = 0;
    __shared__ float red[kWarps];
    __shared__ int bcast[4];

    // This CTA's units of every matrix, staged once (rows past n are zero).
    Smem sm;
    {
        int at = 0;
        for (int m = 0; m < a.n_mats; ++m) {
            const TdtMatrix& M = a.mats[m];
            const int first = (cta - M.offset + G) % G;
            const int units = first < M.units ? (M.units - first + G - 1) / G : 0;
            sm.first[m] = first;
            sm.units[m] = units;
            sm.w[m] = smem + at;
            at += units * 8 * M.smem_stride;
        }
        sm.ring = smem + a.ring_offset;
        for (int m = 0; m < a.n_mats; ++m) {
            const TdtMatrix& M = a.mats[m];
            const int segs = M.k / 16, per_unit = 8 * segs;
            for (int i = tid; i < sm.units[m] * per_unit; i += kThreads) {
                const int unit = i / per_unit, r = (i % per_unit) / segs, seg = i % segs;
                const int row = (sm.first[m] + unit * G) * 8 + r;
                const int xr = M.smem_stride % 128 == 0 ? (r & 1) << 2 : 0;
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (row < M.n) v = __ldg(reinterpret_cast<const uint4*>(M.w + static_cast<int64_t>(row) * M.ld) + seg);
                *reinterpret_cast<uint4*>(sm.w[m] + (unit * 8 + r) * M.smem_stride + (seg ^ xr) * 16) = v;
            }
        }
    }

    int* live[2] = {a.lists, a.lists + U};
    int* plist = a.plist;
    int* ps_of = a.ps_of;
    unsigned* words = a.words;
    const int m_joint = 0, m_pred = a.layers + 1;

    // Start (initial_decoder_state, src/parakeet.rs:1321-1336): every utterance feeds the blank
    // token to a zero state; all of them are live and predicting.
    for (int s = cta; s < U; s += G) {
        if (tid == 0) {
            plist[s] = s;
            ps_of[s] = s;
            live[0][s] = s;
        }
        const float* emb = a.embedding + static_cast<int64_t>(a.blank) * h;
        float v[kVals];
#pragma unroll
        for (int i = 0; i < kVals; ++i) {
            const int j = tid + kThreads * i;
            v[i] = j < h ? __ldg(emb + j) : 0.0f;
        }
        cta_quantize(a, s, 2 * h, v, red);
    }
    if (cta == 0 && tid == 0) {
        words[kWPred] = U;
        words[kWLive] = U;
        words[kWLive + 1] = 0;
    }
    if (!grid_sync(a, gen)) return;
    mark(0);

    int cur = 0;
    int n_live = U;
    long long passes = 0;
    bool first_pass = true;
    for (;;) {
        int n_pred = U;
        if (!first_pass) {
            // Joint product with the argmax in its epilogue (src/parakeet.rs:1455-1470).
            if (cta == 0 && tid == 0) {
                words[kWPred] = 0;
                words[kWLive + (cur ^ 1)] = 0;
            }
            product_any<true>(a, sm, m_joint, n_live, nullptr, 0);
            if (!grid_sync(a, gen)) return;
            mark(1);
            // The TDT step per live utterance (src/parakeet.rs:1471-1510).
            for (int s = cta; s < n_live; s += G) {
                if (tid == 0) {
                    int tok = -1, pslot = -1;
                    const int u = __ldcg(live[cur] + s);
                    const unsigned long long tk = __ldcg(a.tok_key + s), dk = __ldcg(a.dur_key + s);
                    a.tok_key[s] = 0ull;
                    a.dur_key[s] = 0ull;
                    TdtState st;
                    st.enc_first = __ldcg(&a.st[u].enc_first);
                    st.frames = __ldcg(&a.st[u].frames);
                    st.t = __ldcg(&a.st[u].t);
                    st.on_frame = __ldcg(&a.st[u].on_frame);
                    st.tok_first = __ldcg(&a.st[u].tok_first);
                    st.count = __ldcg(&a.st[u].count);
                    // Every row's keys are set (each column has a CTA); the guards only keep
                    // the indices in range.
                    const int id = tk ? key_index(tk) : a.blank;
                    const int di = dk ? key_index(dk) : 0;
                    const int duration = a.durations[di >= 0 && di < a.n_dur ? di : 0];
                    if (id == a.blank) {
                        st.t += duration > 1 ? duration : 1;
                        st.on_frame = 0;
                    } else {
                        uint32_t* o = a.tokens + 3 * static_cast<int64_t>(st.tok_first + st.count);
                        o[0] = static_cast<uint32_t>(id);
                        o[1] = static_cast<uint32_t>(st.t);
                        o[2] = static_cast<uint32_t>(duration);
                        st.count += 1;
                        tok = id;
                        if (duration > 0) {
                            st.t += duration;
                            st.on_frame = 0;
                        } else {
                            st.on_frame += 1;
                            if (st.on_frame >= a.max_symbols) {
                                st.t += 1;
                                st.on_frame = 0;
                            }
                        }
                        pslot = static_cast<int>(atomicAdd(words + kWPred, 1u));
                        plist[pslot] = u;
                    }
                    a.st[u].t = st.t;
                    a.st[u].on_frame = st.on_frame;
                    a.st[u].count = st.count;
                    ps_of[u] = pslot;
                    bcast[0] = u;
                    bcast[1] = tok;
                    bcast[2] = pslot;
                }
                __syncthreads();
                const int u = bcast[0], tok = bcast[1], pslot = bcast[2];
                __syncthreads();
                if (tok >= 0) {
                    const float* emb = a.embedding + static_cast<int64_t>(tok) * h;
                    const float* h0 = a.state + static_cast<int64_t>(u) * a.layers * 2 * h;
                    float v[kVals];
#pragma unroll
                    for (int i = 0; i < kVals; ++i) {
                        const int j = tid + kThreads * i;
                        v[i] = j < h ? __ldg(emb + j) : (j < 2 * h ? __ldcg(h0 + j - h) : 0.0f);
                    }
                    cta_quantize(a, pslot, 2 * h, v, red);
                }
            }
            if (!grid_sync(a, gen)) return;
            mark(2);
            n_pred = static_cast<int>(__ldcg(words + kWPred));
        }
        if (n_pred > 0) {
            // The prediction network for the predicting rows (src/parakeet.rs:1523-1577).
            for (int l = 0; l < a.layers; ++l) {
                product_any<false>(a, sm, 1 + l, n_pred, a.gates, 4 * h);
                if (!grid_sync(a, gen)) return;
                mark(3);
                for (int s = cta; s < n_pred; s += G) cell(a, s, l, red);
                if (!grid_sync(a, gen)) return;
                mark(4);
            }
            product_any<false>(a, sm, m_pred, n_pred, a.fresh, h);
            if (!grid_sync(a, gen)) return;
            mark(5);
        }
        // Commit the new projections; the next pass's joint operand for every utterance with
        // frames left (src/parakeet.rs:1455-1459).
        const int nxt = cur ^ 1;
        for (int s = cta; s < n_live; s += G) {
            if (tid == 0) {
                const int u = __ldcg(live[cur] + s);
                int slot = -1;
                if (__ldcg(&a.st[u].t) < __ldcg(&a.st[u].frames)) {
                    slot = static_cast<int>(atomicAdd(words + kWLive + nxt, 1u));
                    live[nxt][slot] = u;
                }
                bcast[0] = u;
                bcast[1] = slot;
                bcast[2] = __ldcg(ps_of + u);
                bcast[3] = __ldcg(&a.st[u].enc_first) + __ldcg(&a.st[u].t);
            }
            __syncthreads();
            const int u = bcast[0], slot = bcast[1], pslot = bcast[2], erow = bcast[3];
            __syncthreads();
            float* pu = a.pred + static_cast<int64_t>(u) * h;
            const float* fr = a.fresh + static_cast<int64_t>(pslot) * h;
            const float* e = a.enc_proj + static_cast<int64_t>(erow) * h;
            float v[kVals];
#pragma unroll
            for (int i = 0; i < kVals; ++i) {
                const int j = tid + kThreads * i;
                v[i] = 0.0f;
                if (j < h) {
                    float p;
                    if (pslot >= 0) {
                        p = __ldcg(fr + j);
                        pu[j] = p;
                    } else {
                        p = __ldcg(pu + j);
                    }
                    if (slot >= 0) v[i] = fmaxf(__fadd_rn(__ldg(e + j), p), 0.0f);
                }
            }
            if (slot >= 0) cta_quantize(a, slot, h, v, red);
        }
        if (!grid_sync(a, gen)) return;
        mark(6);
        cur = nxt;
        n_live = static_cast<int>(__ldcg(words + kWLive + cur));
        first_pass = false;
        ++passes;
        if (cta == 0 && tid == 0) words[kWPasses] = static_cast<unsigned>(passes);
        if (n_live == 0) break;
        // Every CTA counts the same passes, so all of them stop together.
        if (passes > a.max_passes) {
            if (cta == 0 && tid == 0) atomicCAS(words + kWErr, 0u, static_cast<unsigned>(kTdtErrPasses));
            return;
        }
    }
    if (clock)
        for (int i = 0; i < kTdtPhases; ++i) a.phase_ns[i] = acc[i];
}

}  // namespace

bool tdt_persistent_plan(TdtPersistentArgs& a, int sms, size_t* smem_bytes) {
    if (sms <= 0 || a.n_mats < 3 || a.n_mats > kTdtMaxMats || a.h % kChunk || 2 * a.h > kVals * kThreads ||
        a.n_dur < 1 || a.n_dur > 8)
        return false;
    long max_total = 0;
    for (int m = 0; m < a.n_mats; ++m) {
        TdtMatrix& M = a.mats[m];
        if (M.k % kChunk || M.ld % 16 || M.n <= 0) return false;
        M.units = (M.n + 7) / 8;
        M.max_units = (M.units + sms - 1) / sms;
        if (M.max_units > 8) return false;
        M.smem_stride = M.k;  // rows unpadded; their segments are swizzled instead
    }
    int off = 0;
    for (int m = 0; m < a.n_mats; ++m) {
        a.mats[m].offset = off;
        off = (off + a.mats[m].units) % sms;
    }
    for (int c = 0; c < sms; ++c) {
        long total = 0;
        for (int m = 0; m < a.n_mats; ++m) {
            const TdtMatrix& M = a.mats[m];
            const int first = (c - M.offset + sms) % sms;
            const int units = first < M.units ? (M.units - first + sms - 1) / sms : 0;
            total += static_cast<long>(units) * 8 * M.smem_stride;
        }
        max_total = total > max_total ? total : max_total;
    }
    a.ring_offset = static_cast<int>((max_total + 127) / 128 * 128);
    a.chunk = 128;
    for (int m = 0; m < a.n_mats; ++m)
        if (a.mats[m].k % 128) a.chunk = 64;
    *smem_bytes = static_cast<size_t>(a.ring_offset) + static_cast<size_t>(kWarps) * kWarpRing;
    return *smem_bytes <= 227 * 1024 - 256;  // the static shared memory stays within the SM's share
}

cudaError_t tdt_persistent(const TdtPersistentArgs& a, int grid, size_t smem_bytes, cudaStream_t s) {
    if (cudaError_t e = cudaFuncSetAttribute(tdt_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem_bytes)))
        return e;
    int per_sm = 0;
    if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tdt_persistent_kernel, kThreads,
                                                                      smem_bytes))
        return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    void* params[] = {const_cast<TdtPersistentArgs*>(&a)};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(tdt_persistent_kernel), dim3(grid), dim3(kThreads),
                                       params, smem_bytes, s);
}

}  // namespace telmo
