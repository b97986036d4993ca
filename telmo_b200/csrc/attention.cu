// attention.cu -- Granite's block-local attention with Shaw relative positions
// (Granite::attention, src/granite.rs:965-1036).
//
// One CTA per (attention block, head). For the block's len <= ctx frames:
//   S = scale * (Q . K^T) + scale * shift(Q . Rel^T),  S[i][j] += pos[i][ctx - 1 - i + j]
//   P = softmax(S) per row (f32 exponentials, f64 sum), O = P . V
// Rel is the int8 table of 2 * ctx - 1 positions widened as q * scale (src/granite.rs:315-327).
// Every dot product runs over ascending d (or j) with fused multiply-adds, the order the
// reference's matmul_serial tiles use, so Q.K^T, Q.Rel^T and P.V match its sums.
//
// Thread (ty, tx) of a 16 x 16 grid owns an 8 x 8 block of each 128 x 128 tile.
#include "rowops.h"

namespace telmo {

namespace {

constexpr int T = 128;   // tile rows / cols
constexpr int SP = 132;  // padded row pitch (floats) of the shared tiles, keeps float4 alignment
constexpr int DC = 32;   // d values per staged chunk

template <int HD>
struct AttnSmem {
    float s[T * SP];        // scores / probabilities [i][j]
    float q[HD * SP];       // Q transposed [d][i]
    float b[DC * SP];       // a staged chunk: K^T [d][j], Rel^T [d][p] or V [j][c]
};

__device__ __forceinline__ void load8(const float* p, float (&r)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w; r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
}

template <int HD>
__global__ void __launch_bounds__(256, 1)
granite_attention_kernel(const float* __restrict__ qkv, int heads, int ctx, const AttnTask* __restrict__ tasks,
                         const int8_t* __restrict__ rel_w, int64_t ld_rel, const float* __restrict__ rel_scale,
                         float scale, float* __restrict__ att) {
    extern __shared__ __align__(16) float smem_f[];
    AttnSmem<HD>& sm = *reinterpret_cast<AttnSmem<HD>*>(smem_f);
    const AttnTask task = tasks[blockIdx.x];
    const int h = blockIdx.y;
    const int len = task.len;
    const int D = heads * HD;
    const int64_t ld = 3 * static_cast<int64_t>(D);
    const float* base = qkv + task.row * ld + h * HD;
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int positions = 2 * ctx - 1;

    // Q^T into shared memory, zero past len.
    for (int e = tid; e < HD * T; e += 256) {
        const int i = e / HD, d = e % HD;
        sm.q[d * SP + i] = i < len ? base[i * ld + d] : 0.0f;
    }

    // ---- S = scale * Q.K^T ---------------------------------------------------------------
    float acc[8][8];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = 0.0f;
    for (int d0 = 0; d0 < HD; d0 += DC) {
        __syncthreads();
        for (int e = tid; e < DC * T; e += 256) {
            const int j = e / DC, dd = e % DC;
            sm.b[dd * SP + j] = (j < len && d0 + dd < HD) ? base[j * ld + D + d0 + dd] : 0.0f;
        }
        __syncthreads();
        const int dmax = HD - d0 < DC ? HD - d0 : DC;
        for (int dd = 0; dd < dmax; ++dd) {
            float qa[8], kb[8];
            load8(&sm.q[(d0 + dd) * SP + ty * 8], qa);
            load8(&sm.b[dd * SP + tx * 8], kb);
#pragma unroll
            for (int a = 0; a < 8; ++a)
#pragma unroll
                for (int b = 0; b < 8; ++b) acc[a][b] = __fmaf_rn(qa[a], kb[b], acc[a][b]);
        }
    }
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) sm.s[(ty * 8 + a) * SP + tx * 8 + b] = __fmul_rn(acc[a][b], scale);

    // ---- S[i][j] += scale * (Q . Rel^T)[i][ctx - 1 - i + j], positions in two halves ----------
    for (int p0 = 0; p0 < positions; p0 += T) {
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = 0; b < 8; ++b) acc[a][b] = 0.0f;
        for (int d0 = 0; d0 < HD; d0 += DC) {
            __syncthreads();
            for (int e = tid; e < DC * T; e += 256) {
                const int p = e / DC, dd = e % DC;
                const int pp = p0 + p;
                float v = 0.0f;
                if (pp < positions && d0 + dd < HD)
                    v = __fmul_rn(static_cast<float>(rel_w[pp * ld_rel + d0 + dd]), __ldg(rel_scale + pp));
                sm.b[dd * SP + p] = v;
            }
            __syncthreads();
            const int dmax = HD - d0 < DC ? HD - d0 : DC;
            for (int dd = 0; dd < dmax; ++dd) {
                float qa[8], rb[8];
                load8(&sm.q[(d0 + dd) * SP + ty * 8], qa);
                load8(&sm.b[dd * SP + tx * 8], rb);
#pragma unroll
                for (int a = 0; a < 8; ++a)
#pragma unroll
                    for (int b = 0; b < 8; ++b) acc[a][b] = __fmaf_rn(qa[a], rb[b], acc[a][b]);
            }
        }
        // Scatter: position p of row i is key j = p - (ctx - 1) + i; each (i, j) gets one term.
#pragma unroll
        for (int a = 0; a < 8; ++a) {
            const int i = ty * 8 + a;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const int p = p0 + tx * 8 + b;
                const int j = p - (ctx - 1) + i;
                if (i < len && p < positions && j >= 0 && j < len)
                    sm.s[i * SP + j] = __fadd_rn(sm.s[i * SP + j], __fmul_rn(acc[a][b], scale));
            }
        }
    }
    __syncthreads();

    // ---- softmax of each row over its len keys; zero the padding -----------------------------
    const int warp = tid / 32, lane = tid % 32;
    for (int i = warp; i < T; i += 8) {
        float* row = &sm.s[i * SP];
        if (i >= len) {
            for (int j = lane; j < T; j += 32) row[j] = 0.0f;
            continue;
        }
        float mx = -INFINITY;
        for (int j = lane; j < len; j += 32) mx = fmaxf(mx, row[j]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        double sum = 0.0;
        for (int j = lane; j < len; j += 32) {
            const float e = expf(__fsub_rn(row[j], mx));
            row[j] = e;
            sum += static_cast<double>(e);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float inv = static_cast<float>(1.0 / sum);
        for (int j = lane; j < T; j += 32) row[j] = j < len ? __fmul_rn(row[j], inv) : 0.0f;
    }

    // ---- O = P . V over ascending keys ------------------------------------------------------
    for (int c0 = 0; c0 < HD; c0 += T) {
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = 0; b < 8; ++b) acc[a][b] = 0.0f;
        for (int j0 = 0; j0 < len; j0 += DC) {
            __syncthreads();
            for (int e = tid; e < DC * T; e += 256) {
                const int jj = e / T, c = e % T;
                sm.b[jj * SP + c] = (j0 + jj < len && c0 + c < HD) ? base[(j0 + jj) * ld + 2 * D + c0 + c] : 0.0f;
            }
            __syncthreads();
            const int jmax = len - j0 < DC ? len - j0 : DC;
            for (int jj = 0; jj < jmax; ++jj) {
                float pa[8], vb[8];
#pragma unroll
                for (int a = 0; a < 8; ++a) pa[a] = sm.s[(ty * 8 + a) * SP + j0 + jj];
                load8(&sm.b[jj * SP + tx * 8], vb);
#pragma unroll
                for (int a = 0; a < 8; ++a)
#pragma unroll
                    for (int b = 0; b < 8; ++b) acc[a][b] = __fmaf_rn(pa[a], vb[b], acc[a][b]);
            }
        }
#pragma unroll
        for (int a = 0; a < 8; ++a) {
            const int i = ty * 8 + a;
            if (i >= len) continue;
            float* o = att + (task.row + i) * static_cast<int64_t>(D) + h * HD + c0;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const int c = tx * 8 + b;
                if (c0 + c < HD) o[c] = acc[a][b];
            }
        }
    }
}

template <int HD>
cudaError_t launch_attention(const float* qkv, int heads, int ctx, const AttnTask* tasks, int n_tasks,
                             const int8_t* rel_w, int64_t ld_rel, const float* rel_scale, float scale,
                             float* att, cudaStream_t stream) {
    const int smem = static_cast<int>(sizeof(AttnSmem<HD>));
    static DeviceOnce configured;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured.done(dev)) {
        cudaError_t e = cudaFuncSetAttribute(granite_attention_kernel<HD>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured.mark(dev);
    }
    dim3 grid(n_tasks, heads);
    granite_attention_kernel<HD><<<grid, 256, smem, stream>>>(qkv, heads, ctx, tasks, rel_w, ld_rel, rel_scale,
                                                              scale, att);
    return cudaGetLastError();
}

}  // namespace

cudaError_t granite_attention(const float* qkv, int heads, int hd, int ctx, const AttnTask* tasks, int n_tasks,
                              const int8_t* rel_w, int64_t ld_rel, const float* rel_scale, float scale,
                              float* att, cudaStream_t stream) {
    if (n_tasks <= 0) return cudaSuccess;
    if (ctx > T || ctx <= 0) return cudaErrorInvalidValue;
    switch (hd) {
        case 16: return launch_attention<16>(qkv, heads, ctx, tasks, n_tasks, rel_w, ld_rel, rel_scale, scale, att, stream);
        case 32: return launch_attention<32>(qkv, heads, ctx, tasks, n_tasks, rel_w, ld_rel, rel_scale, scale, att, stream);
        case 64: return launch_attention<64>(qkv, heads, ctx, tasks, n_tasks, rel_w, ld_rel, rel_scale, scale, att, stream);
        case 128: return launch_attention<128>(qkv, heads, ctx, tasks, n_tasks, rel_w, ld_rel, rel_scale, scale, att, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace telmo
