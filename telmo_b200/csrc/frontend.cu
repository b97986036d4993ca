// frontend.cu -- the two log-mel front ends on the GPU, for batches of utterances.
//
// Granite (GraniteFrontEnd, src/granite_features.rs): reflect-padded centred STFT (FFT 512, a
// 400-sample periodic Hann window centred in it, hop 160), power, 80 HTK mel filters summed in
// f64, log10(max(x, 1e-10)), a floor 8 below the utterance's peak, / 4 + 1, deltas over three
// frames, two frames to a row of 320.
// Parakeet (FrontEnd, src/features.rs): pre-emphasis 0.97 in f32, zero-padded centred STFT with
// a symmetric Hann window, power, 128 Slaney mels in f64, ln(x + 2^-24), and each mel bin
// normalised over the utterance (std with n - 1, plus 1e-5).
//
// The 512-point real FFT is the reference's algorithm (RealFft::forward, src/fft.rs:97-134):
// a 256-point complex radix-2 DIT over packed even/odd samples, then the split into 257 bins.
// Twiddles come from host tables computed with the reference's expressions, and every f64 step
// is an explicit round-to-nearest operation in the reference's order (no FMA contraction), so
// spectra match the CPU's.
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "frontend.h"

#include <cmath>
#include <vector>

namespace telmo {

namespace {

constexpr int N_FFT = 512, HALF = 256, BINS = 257, HOP = 160, WIN = 400;

struct FftTables {
    double half_re[HALF / 2], half_im[HALF / 2];  // e^(-2 pi i j / 256), j < 128
    double split_re[BINS], split_im[BINS];        // e^(-2 pi i k / 512), k <= 256
    double window[N_FFT];                          // the front end's window, centred
    int rev[HALF];                                 // 8-bit reversal
};

__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }

// One frame per warp, kFrameWarps frames per CTA: a frame's FFT is 128 butterflies per stage, so
// a warp (four butterflies per lane, __syncwarp between stages) keeps every lane busy with no
// block-wide barrier; each warp owns 512 doubles of shared memory.
constexpr int kFrameWarps = 8;

// One frame's power spectrum, in a warp. On entry z = zr + i zi (zr = buf, zi = buf + 256) holds
// the packed samples at their bit-reversed positions; on exit power[k] = buf[k], k <= 256. Each
// butterfly and bin is the reference's arithmetic step for step, whichever lane computes it.
__device__ void warp_power_spectrum(const FftTables* __restrict__ T, double* buf, int lane) {
    double* zr = buf;
    double* zi = buf + HALF;
#pragma unroll
    for (int lg = 0; lg < 8; ++lg) {  // sizes 2 .. 256
        const int half = 1 << lg, step = HALF >> (lg + 1);
        __syncwarp();
#pragma unroll
        for (int q = 0; q < HALF / 2 / 32; ++q) {
            const int t = lane + 32 * q;
            const int grp = t >> lg, j = t & (half - 1);
            const int a = grp * 2 * half + j, b = a + half;
            const double wr = T->half_re[j * step], wi = T->half_im[j * step];
            const double xr = zr[b], xi = zi[b];
            const double br = dsub(dmul(xr, wr), dmul(xi, wi));
            const double bi = dadd(dmul(xr, wi), dmul(xi, wr));
            const double ar = zr[a], ai = zi[a];
            zr[a] = dadd(ar, br);
            zi[a] = dadd(ai, bi);
            zr[b] = dsub(ar, br);
            zi[b] = dsub(ai, bi);
        }
    }
    __syncwarp();
    double pw[(BINS + 31) / 32];
#pragma unroll
    for (int i = 0; i < (BINS + 31) / 32; ++i) {
        const int k = lane + 32 * i;
        if (k >= BINS) break;
        const double r = zr[k % HALF], im = zi[k % HALF];
        const double cr = zr[(HALF - k) % HALF], ci = -zi[(HALF - k) % HALF];
        const double er = dmul(dadd(r, cr), 0.5), ei = dmul(dadd(im, ci), 0.5);
        const double dr = dsub(r, cr), di = dsub(im, ci);
        const double orr = dmul(di, 0.5), oi = dmul(-dr, 0.5);
        const double wr = T->split_re[k], wi = T->split_im[k];
        const double xr = dadd(er, dsub(dmul(wr, orr), dmul(wi, oi)));
        const double xi = dadd(ei, dadd(dmul(wr, oi), dmul(wi, orr)));
        pw[i] = dadd(dmul(xr, xr), dmul(xi, xi));
    }
    __syncwarp();  // every lane has read z
#pragma unroll
    for (int i = 0; i < (BINS + 31) / 32; ++i) {
        const int k = lane + 32 * i;
        if (k >= BINS) break;
        buf[k] = pw[i];
    }
    __syncwarp();
}

// Which utterance a global frame index belongs to (frame_first is increasing, n entries).
__device__ __forceinline__ int find_utt(const int* __restrict__ frame_first, int n, int f) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (frame_first[mid] <= f) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Granite log_frame (src/granite_features.rs:95-133) for frames 0 .. frames - 1 of the batch.
__global__ void __launch_bounds__(32 * kFrameWarps) granite_logmel_kernel(const float* __restrict__ samples,
                                                                          const FrontMeta meta, int frames,
                                                                          const FftTables* __restrict__ T,
                                                                          const MelTable mel, float* __restrict__ logs) {
    __shared__ double bufs[kFrameWarps][N_FFT];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int f = blockIdx.x * kFrameWarps + warp;
    if (f >= frames) return;  // no block-wide barrier follows
    double* buf = bufs[warp];
    const int u = find_utt(meta.frame_first, meta.n_utt, f);
    const int local = f - meta.frame_first[u];
    const float* x = samples + meta.sample_first[u];
    const long n = meta.sample_count[u];
    const long len = meta.padded_len[u];
    const long start = static_cast<long>(local) * HOP - N_FFT / 2;
    // The reflect-padded, windowed samples, packed two to a complex value at its bit-reversed slot.
#pragma unroll
    for (int q = 0; q < HALF / 32; ++q) {
        const int m = lane + 32 * q;
        double v[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int i = 2 * m + e;
            const long j = start + i;
            const long jj = j < 0 ? -j : (j >= len ? 2 * (len - 1) - j : j);
            const double smp = jj < n ? static_cast<double>(x[jj]) : 0.0;
            v[e] = dmul(smp, T->window[i]);
        }
        buf[T->rev[m]] = v[0];
        buf[HALF + T->rev[m]] = v[1];
    }
    warp_power_spectrum(T, buf, lane);
    for (int m = lane; m < mel.n_mels; m += 32) {
        double acc = 0.0;
        const int first = mel.first[m], cnt = mel.count[m];
        const float* w = mel.weights + mel.offset[m];
        for (int k = 0; k < cnt; ++k) acc = dadd(acc, dmul(static_cast<double>(w[k]), buf[first + k]));
        const float energy = fmaxf(static_cast<float>(acc), 1e-10f);
        logs[static_cast<long>(f) * mel.n_mels + m] = static_cast<float>(log10(static_cast<double>(energy)));
    }
}

// Each utterance's largest log10 value (one CTA per utterance).
__global__ void utt_max_kernel(const float* __restrict__ logs, const FrontMeta meta, int n_mels, float* __restrict__ peak) {
    const int u = blockIdx.x;
    const long a = static_cast<long>(meta.frame_first[u]) * n_mels;
    const long b = a + static_cast<long>(meta.frame_count[u]) * n_mels;
    float mx = -INFINITY;
    for (long i = a + threadIdx.x; i < b; i += blockDim.x) mx = fmaxf(mx, logs[i]);
    __shared__ float red[32];
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        mx = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (threadIdx.x == 0) peak[u] = mx;
    }
}

// stack_rows (src/granite_features.rs:138-158): one CTA per feature row (two frames).
__global__ void granite_stack_kernel(const float* __restrict__ logs, const FrontMeta meta, int n_mels,
                                     const float* __restrict__ peak, const int* __restrict__ row_first,
                                     float* __restrict__ out) {
    const int r = blockIdx.x;  // global row
    // rows of utterance u start at row_first[u]; frames at frame_first[u] (2 per row)
    int lo = 0, hi = meta.n_utt - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (row_first[mid] <= r) lo = mid;
        else hi = mid - 1;
    }
    const int u = lo;
    const int frames = meta.frame_count[u];
    const float floor_v = __fsub_rn(peak[u], 8.0f);
    const float* L = logs + static_cast<long>(meta.frame_first[u]) * n_mels;
    const int local_row = r - row_first[u];
    float* o = out + static_cast<long>(r) * 4 * n_mels;
    for (int i = threadIdx.x; i < 2 * n_mels; i += blockDim.x) {
        const int f = 2 * local_row + i / n_mels, m = i % n_mels;
        const int before = f > 0 ? f - 1 : 0, after = f + 1 < frames ? f + 1 : frames - 1;
        const float v = __fadd_rn(__fdiv_rn(fmaxf(L[f * n_mels + m], floor_v), 4.0f), 1.0f);
        const float va = __fadd_rn(__fdiv_rn(fmaxf(L[after * n_mels + m], floor_v), 4.0f), 1.0f);
        const float vb = __fadd_rn(__fdiv_rn(fmaxf(L[before * n_mels + m], floor_v), 4.0f), 1.0f);
        float* row = o + (i / n_mels) * 2 * n_mels;
        row[m] = v;
        row[n_mels + m] = __fdiv_rn(__fsub_rn(va, vb), 2.0f);
    }
}

// Parakeet log_mel_frame (src/features.rs:156-173) for frames 0 .. frames - 1: pre-emphasised
// samples under the 400-sample window (zero outside the utterance), ln(acc + 2^-24) in f64.
__global__ void __launch_bounds__(32 * kFrameWarps) parakeet_logmel_kernel(const float* __restrict__ samples,
                                                                           const FrontMeta meta, int frames,
                                                                           const FftTables* __restrict__ T,
                                                                           const MelTable mel,
                                                                           double* __restrict__ logs) {
    __shared__ double bufs[kFrameWarps][N_FFT];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int f = blockIdx.x * kFrameWarps + warp;
    if (f >= frames) return;  // no block-wide barrier follows
    double* buf = bufs[warp];
    const int u = find_utt(meta.frame_first, meta.n_utt, f);
    const int local = f - meta.frame_first[u];
    const float* x = samples + meta.sample_first[u];
    const long n = meta.sample_count[u];
    constexpr int offset = (N_FFT - WIN) / 2;
#pragma unroll
    for (int q = 0; q < HALF / 32; ++q) {
        const int m = lane + 32 * q;
        double v[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int i = 2 * m + e;
            v[e] = 0.0;
            if (i >= offset && i < offset + WIN) {
                // Sample index of window position i: f * hop + i - n_fft / 2.
                const long j = static_cast<long>(local) * HOP + i - N_FFT / 2;
                if (j >= 0 && j < n) {
                    const float pe = j == 0 ? x[0] : __fsub_rn(x[j], __fmul_rn(0.97f, x[j - 1]));
                    v[e] = dmul(static_cast<double>(pe), T->window[i]);
                }
            }
        }
        buf[T->rev[m]] = v[0];
        buf[HALF + T->rev[m]] = v[1];
    }
    warp_power_spectrum(T, buf, lane);
    const double guard = 1.0 / 16777216.0;
    for (int m = lane; m < mel.n_mels; m += 32) {
        double acc = 0.0;
        const int first = mel.first[m], cnt = mel.count[m];
        const float* w = mel.weights + mel.offset[m];
        for (int k = 0; k < cnt; ++k) acc = dadd(acc, dmul(static_cast<double>(w[k]), buf[first + k]));
        logs[static_cast<long>(f) * mel.n_mels + m] = log(dadd(acc, guard));
    }
}

// normalize (src/features.rs:199-216): one CTA per (utterance, bin block of 32): mean and
// variance over the utterance's frames in f64, then (x - mean) / (std + 1e-5).
__global__ void parakeet_normalize_kernel(const double* __restrict__ logs, const FrontMeta meta, int n_mels,
                                          float* __restrict__ out) {
    const int u = blockIdx.x;
    const int m = blockIdx.y * 32 + threadIdx.x % 32;
    const int part = threadIdx.x / 32, parts = blockDim.x / 32;
    const int frames = meta.frame_count[u];
    const long base = static_cast<long>(meta.frame_first[u]) * n_mels;
    __shared__ double red[32][33];
    __shared__ double mean_s[32], scale_s[32];
    double s = 0.0;
    if (m < n_mels)
        for (int f = part; f < frames; f += parts) s = dadd(s, logs[base + static_cast<long>(f) * n_mels + m]);
    red[part][threadIdx.x % 32] = s;
    __syncthreads();
    if (part == 0) {
        double t = 0.0;
        for (int p = 0; p < parts; ++p) t = dadd(t, red[p][threadIdx.x % 32]);
        mean_s[threadIdx.x % 32] = t / frames;
    }
    __syncthreads();
    const double mean = mean_s[threadIdx.x % 32];
    double q = 0.0;
    if (m < n_mels)
        for (int f = part; f < frames; f += parts) {
            const double dlt = dsub(logs[base + static_cast<long>(f) * n_mels + m], mean);
            q = dadd(q, dmul(dlt, dlt));
        }
    __syncthreads();
    red[part][threadIdx.x % 32] = q;
    __syncthreads();
    if (part == 0) {
        double t = 0.0;
        for (int p = 0; p < parts; ++p) t = dadd(t, red[p][threadIdx.x % 32]);
        const double var = t / (frames - 1);
        scale_s[threadIdx.x % 32] = 1.0 / dadd(sqrt(var), 1e-5);
    }
    __syncthreads();
    const double scale = scale_s[threadIdx.x % 32];
    if (m < n_mels)
        for (int f = part; f < frames; f += parts) {
            const long at = base + static_cast<long>(f) * n_mels + m;
            out[at] = static_cast<float>(dmul(dsub(logs[at], mean), scale));
        }
}

// ---- host tables ------------------------------------------------------------------------------

void linspace_f32(float start, float end, int steps, float* out) {
    // torch.linspace in f32 (src/granite_features.rs:221-233).
    const float step = (end - start) / static_cast<float>(steps - 1);
    for (int i = 0; i < steps; ++i)
        out[i] = i < steps / 2 ? start + step * static_cast<float>(i) : end - step * static_cast<float>(steps - 1 - i);
}

void sparse_filters(const std::vector<std::vector<float>>& dense, HostMel& mel) {
    mel.first.clear();
    mel.count.clear();
    mel.offset.clear();
    mel.weights.clear();
    for (const auto& w : dense) {
        int first = 0, last = 0;
        bool found = false;
        for (int b = 0; b < BINS; ++b)
            if (w[b] != 0.0f) { first = b; found = true; break; }
        last = first;
        if (found)
            for (int b = BINS - 1; b >= 0; --b)
                if (w[b] != 0.0f) { last = b + 1; break; }
        mel.first.push_back(first);
        mel.count.push_back(last - first);
        mel.offset.push_back(static_cast<int>(mel.weights.size()));
        for (int b = first; b < last; ++b) mel.weights.push_back(w[b]);
    }
}

}  // namespace

// htk_mel_filters (src/granite_features.rs:236-271), in its f32 rounding.
void htk_mel_filters(int n_mels, HostMel& mel) {
    const double nyquist = 8000.0;
    float all_freqs[BINS];
    linspace_f32(0.0f, static_cast<float>(nyquist), BINS, all_freqs);
    const double m_max = 2595.0 * std::log10(1.0 + nyquist / 700.0);
    std::vector<float> mels(n_mels + 2), f_pts(n_mels + 2);
    linspace_f32(0.0f, static_cast<float>(m_max), n_mels + 2, mels.data());
    for (int i = 0; i < n_mels + 2; ++i) {
        const float p = static_cast<float>(std::pow(10.0, static_cast<double>(mels[i] / 2595.0f)));
        f_pts[i] = 700.0f * (p - 1.0f);
    }
    std::vector<std::vector<float>> dense(n_mels, std::vector<float>(BINS));
    for (int m = 0; m < n_mels; ++m) {
        const float d0 = f_pts[m + 1] - f_pts[m], d1 = f_pts[m + 2] - f_pts[m + 1];
        for (int b = 0; b < BINS; ++b) {
            const float f = all_freqs[b];
            const float down = -(f_pts[m] - f) / d0;
            const float up = (f_pts[m + 2] - f) / d1;
            dense[m][b] = std::fmax(std::fmin(down, up), 0.0f);
        }
    }
    sparse_filters(dense, mel);
}

static double hz_to_mel_slaney(double hz) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    return hz >= min_log_hz ? min_log_mel + std::log(hz / min_log_hz) / logstep : hz / f_sp;
}

static double mel_to_hz_slaney(double mel) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    return mel >= min_log_mel ? min_log_hz * std::exp(logstep * (mel - min_log_mel)) : f_sp * mel;
}

// slaney_mel_filters (src/features.rs:379-412), in its f32 rounding.
void slaney_mel_filters(int n_mels, HostMel& mel) {
    double fft_freqs[BINS];
    for (int k = 0; k < BINS; ++k) fft_freqs[k] = static_cast<double>(k) * 16000.0 / N_FFT;
    const double max_mel = hz_to_mel_slaney(8000.0);
    std::vector<double> pts(n_mels + 2);
    for (int i = 0; i < n_mels + 2; ++i) pts[i] = mel_to_hz_slaney(max_mel * i / (n_mels + 1));
    std::vector<std::vector<float>> dense(n_mels, std::vector<float>(BINS));
    for (int m = 0; m < n_mels; ++m) {
        const double lo = pts[m], center = pts[m + 1], hi = pts[m + 2];
        const double enorm = 2.0 / (hi - lo);
        for (int b = 0; b < BINS; ++b) {
            const double f = fft_freqs[b];
            const double w = std::fmin((f - lo) / (center - lo), (hi - f) / (hi - center));
            const float wf = static_cast<float>(w > 0.0 ? w : 0.0);
            dense[m][b] = static_cast<float>(static_cast<double>(wf) * enorm);
        }
    }
    sparse_filters(dense, mel);
}

int FrontEnd::init(Ctx* c, Kind k) {
    ctx = c;
    kind = k;
    FftTables t;
    const double pi = 3.14159265358979323846;
    for (int j = 0; j < HALF / 2; ++j) {
        const double a = -2.0 * pi * j / HALF;
        t.half_re[j] = std::cos(a);
        t.half_im[j] = std::sin(a);
    }
    for (int k2 = 0; k2 < BINS; ++k2) {
        const double a = -2.0 * pi * k2 / N_FFT;
        t.split_re[k2] = std::cos(a);
        t.split_im[k2] = std::sin(a);
    }
    for (int i = 0; i < HALF; ++i) {
        int r = 0;
        for (int b = 0; b < 8; ++b)
            if (i & (1 << b)) r |= 1 << (7 - b);
        t.rev[i] = r;
    }
    for (int i = 0; i < N_FFT; ++i) t.window[i] = 0.0;
    HostMel hm;
    if (kind == kGranite) {
        // periodic Hann in f32, centred (src/granite_features.rs:47-52, :209-217).
        const float step = static_cast<float>(2.0 * pi / WIN);
        for (int i = 0; i < WIN; ++i) {
            const float xx = static_cast<float>(i) * step;
            t.window[(N_FFT - WIN) / 2 + i] = static_cast<double>(0.5f + -0.5f * static_cast<float>(std::cos(static_cast<double>(xx))));
        }
        htk_mel_filters(n_mels, hm);
    } else {
        // symmetric Hann rounded to f32 (src/features.rs:75-82).
        for (int i = 0; i < WIN; ++i) {
            const double w = 0.5 - 0.5 * std::cos(2.0 * pi * i / (WIN - 1));
            t.window[(N_FFT - WIN) / 2 + i] = static_cast<double>(static_cast<float>(w));
        }
        slaney_mel_filters(n_mels, hm);
    }
    if (int rc = ctx->cuda(cudaMalloc(&tables, sizeof(FftTables)), "front end")) return rc;
    if (int rc = ctx->cuda(cudaMemcpy(tables, &t, sizeof(FftTables), cudaMemcpyHostToDevice), "front end")) return rc;
    const int nm = n_mels;
    if (int rc = ctx->cuda(cudaMalloc(&mel_dev, sizeof(int) * 3 * nm + sizeof(float) * hm.weights.size()), "front end"))
        return rc;
    std::vector<int> ints(3 * nm);
    for (int m = 0; m < nm; ++m) {
        ints[m] = hm.first[m];
        ints[nm + m] = hm.count[m];
        ints[2 * nm + m] = hm.offset[m];
    }
    uint8_t* p = static_cast<uint8_t*>(mel_dev);
    if (int rc = ctx->cuda(cudaMemcpy(p, ints.data(), sizeof(int) * 3 * nm, cudaMemcpyHostToDevice), "front end")) return rc;
    if (int rc = ctx->cuda(cudaMemcpy(p + sizeof(int) * 3 * nm, hm.weights.data(), sizeof(float) * hm.weights.size(),
                                      cudaMemcpyHostToDevice),
                           "front end"))
        return rc;
    mel.n_mels = nm;
    mel.first = reinterpret_cast<int*>(p);
    mel.count = mel.first + nm;
    mel.offset = mel.first + 2 * nm;
    mel.weights = reinterpret_cast<float*>(p + sizeof(int) * 3 * nm);
    return TELMO_OK;
}

FrontEnd::~FrontEnd() {
    if (tables) cudaFree(tables);
    if (mel_dev) cudaFree(mel_dev);
    if (meta_dev) cudaFree(meta_dev);
    if (scratch) cudaFree(scratch);
}

// Per-utterance layout: samples packed one after another; frames and rows likewise.
int FrontEnd::plan(const int64_t* lengths, int n_utt, std::vector<int>& out_rows) {
    out_rows.assign(n_utt, 0);
    std::vector<int64_t> words(5 * static_cast<size_t>(n_utt) + 1);
    int64_t samples = 0, frames = 0;
    for (int u = 0; u < n_utt; ++u) {
        const int64_t n = lengths[u];
        int64_t f;
        if (kind == kGranite) {
            if (n < 2 * HOP) return ctx->fail(TELMO_ERR_MODEL, "The audio is too short (%lld samples). It needs at least %d.",
                                              static_cast<long long>(n), 2 * HOP);
            const int64_t rows = (n / HOP + 1) / 2;
            f = 2 * rows;
            out_rows[u] = static_cast<int>(rows);
        } else {
            f = n / HOP;
            if (f < 2) return ctx->fail(TELMO_ERR_MODEL, "The audio is too short (%lld samples). It needs at least %d.",
                                        static_cast<long long>(n), 2 * HOP);
            out_rows[u] = static_cast<int>(f);
        }
        samples += n;
        frames += f;
    }
    if (frames > (1 << 30) || samples > (int64_t(1) << 40)) return ctx->fail(TELMO_ERR_ARGUMENT, "front end: batch too large");
    total_frames = static_cast<int>(frames);
    total_samples = samples;
    return TELMO_OK;
}

int FrontEnd::run(const float* samples_dev, const int64_t* lengths, int n_utt, float* features, int* rows_out,
                  cudaStream_t s) {
    std::vector<int> rows;
    if (int rc = plan(lengths, n_utt, rows)) return rc;
    // Device metadata: frame_first, frame_count, row_first (int) and sample_first, sample_count,
    // padded_len (int64).
    std::vector<int> ints(3 * static_cast<size_t>(n_utt));
    std::vector<int64_t> longs(3 * static_cast<size_t>(n_utt));
    int64_t sf = 0;
    int ff = 0, rf = 0;
    for (int u = 0; u < n_utt; ++u) {
        const int frames = kind == kGranite ? 2 * rows[u] : rows[u];
        ints[u] = ff;
        ints[n_utt + u] = frames;
        ints[2 * n_utt + u] = rf;
        longs[u] = sf;
        longs[n_utt + u] = lengths[u];
        const int64_t padded = std::max<int64_t>(lengths[u], static_cast<int64_t>(frames - 1) * HOP + 1);
        longs[2 * n_utt + u] = padded;
        ff += frames;
        rf += rows[u];
        sf += lengths[u];
        rows_out[u] = rows[u];
    }
    const size_t meta_bytes = sizeof(int64_t) * longs.size() + sizeof(int) * ints.size() + sizeof(float) * n_utt;
    if (meta_bytes > meta_cap) {
        cudaDeviceSynchronize();  // queued batches may still read the old buffers
        if (meta_dev) cudaFree(meta_dev);
        meta_dev = nullptr;
        meta_cap = 0;
        if (int rc = ctx->cuda(cudaMalloc(&meta_dev, meta_bytes * 2), "front end")) return rc;
        meta_cap = meta_bytes * 2;
    }
    const size_t log_bytes = static_cast<size_t>(total_frames) * n_mels * (kind == kGranite ? sizeof(float) : sizeof(double));
    if (log_bytes > scratch_cap) {
        cudaDeviceSynchronize();
        if (scratch) cudaFree(scratch);
        scratch = nullptr;
        scratch_cap = 0;
        if (int rc = ctx->cuda(cudaMalloc(&scratch, log_bytes + log_bytes / 4), "front end")) return rc;
        scratch_cap = log_bytes + log_bytes / 4;
    }
    uint8_t* m = static_cast<uint8_t*>(meta_dev);
    int64_t* dl = reinterpret_cast<int64_t*>(m);
    int* di = reinterpret_cast<int*>(m + sizeof(int64_t) * longs.size());
    float* peak = reinterpret_cast<float*>(di + ints.size());
    // Through pinned staging: the copies are asynchronous and the host vectors may go out of scope.
    if (int rc = ctx->cuda(ctx->uploads.upload(dl, longs.data(), sizeof(int64_t) * longs.size(), s), "meta")) return rc;
    if (int rc = ctx->cuda(ctx->uploads.upload(di, ints.data(), sizeof(int) * ints.size(), s), "meta")) return rc;
    FrontMeta meta;
    meta.n_utt = n_utt;
    meta.frame_first = di;
    meta.frame_count = di + n_utt;
    meta.sample_first = dl;
    meta.sample_count = dl + n_utt;
    meta.padded_len = dl + 2 * n_utt;
    const int* row_first = di + 2 * n_utt;
    if (kind == kGranite) {
        float* logs = static_cast<float*>(scratch);
        granite_logmel_kernel<<<(total_frames + kFrameWarps - 1) / kFrameWarps, 32 * kFrameWarps, 0, s>>>(
            samples_dev, meta, total_frames, static_cast<const FftTables*>(tables), mel, logs);
        utt_max_kernel<<<n_utt, 256, 0, s>>>(logs, meta, n_mels, peak);
        granite_stack_kernel<<<rf, 160, 0, s>>>(logs, meta, n_mels, peak, row_first, features);
        launches += 3;
    } else {
        double* logs = static_cast<double*>(scratch);
        parakeet_logmel_kernel<<<(total_frames + kFrameWarps - 1) / kFrameWarps, 32 * kFrameWarps, 0, s>>>(
            samples_dev, meta, total_frames, static_cast<const FftTables*>(tables), mel, logs);
        dim3 grid(n_utt, (n_mels + 31) / 32);
        parakeet_normalize_kernel<<<grid, 256, 0, s>>>(logs, meta, n_mels, features);
        launches += 2;
    }
    return ctx->cuda(cudaGetLastError(), "front end");
}

// ---- the Granite front end over part of one utterance (GraniteStream) ------------------------

namespace {
struct StreamMetaHost {
    int64_t sample_first, sample_count, padded_len;
    int frame_first, frame_count, row_first;
};
}  // namespace

int FrontEnd::stream_meta(const void* host_meta, void* meta_dev, FrontMeta& meta, const int*& row_first,
                          cudaStream_t s) {
    const StreamMetaHost& h = *static_cast<const StreamMetaHost*>(host_meta);
    int64_t longs[3] = {h.sample_first, h.sample_count, h.padded_len};
    int ints[3] = {h.frame_first, h.frame_count, h.row_first};
    uint8_t* m = static_cast<uint8_t*>(meta_dev);
    int64_t* dl = reinterpret_cast<int64_t*>(m);
    int* di = reinterpret_cast<int*>(m + sizeof longs);
    if (int rc = ctx->cuda(cudaMemcpyAsync(dl, longs, sizeof longs, cudaMemcpyHostToDevice, s), "stream meta")) return rc;
    if (int rc = ctx->cuda(cudaMemcpyAsync(di, ints, sizeof ints, cudaMemcpyHostToDevice, s), "stream meta")) return rc;
    meta.n_utt = 1;
    meta.frame_first = di;
    meta.frame_count = di + 1;
    meta.sample_first = dl;
    meta.sample_count = dl + 1;
    meta.padded_len = dl + 2;
    row_first = di + 2;
    return TELMO_OK;
}

int FrontEnd::granite_stream_frames(const float* samples, int64_t n, int64_t len, int f0, int f1, float* logs,
                                    float* new_peak, void* meta_dev, cudaStream_t s) {
    // log_frame (src/granite_features.rs:95-133) of frames f0..f1: the kernel's frame f of the
    // one utterance is local frame f - frame_first = f + f0, written to logs + f * n_mels.
    if (f1 <= f0) return TELMO_OK;
    StreamMetaHost h{0, n, len, -f0, f1 - f0, 0};
    FrontMeta meta;
    const int* row_first = nullptr;
    if (int rc = stream_meta(&h, meta_dev, meta, row_first, s)) return rc;
    float* out = logs + static_cast<int64_t>(f0) * n_mels;
    granite_logmel_kernel<<<(f1 - f0 + kFrameWarps - 1) / kFrameWarps, 32 * kFrameWarps, 0, s>>>(
        samples, meta, f1 - f0, static_cast<const FftTables*>(tables), mel, out);
    // Their largest value: the same kernel over frames 0..f1 - f0 of the block just written.
    StreamMetaHost hm{0, n, len, 0, f1 - f0, 0};
    FrontMeta mm;
    if (int rc = stream_meta(&hm, static_cast<uint8_t*>(meta_dev) + 64, mm, row_first, s)) return rc;
    utt_max_kernel<<<1, 256, 0, s>>>(out, mm, n_mels, new_peak);
    launches += 2;
    return ctx->cuda(cudaGetLastError(), "stream front end");
}

int FrontEnd::granite_stream_rows(const float* logs, int frames, const float* peak, int first, int last,
                                  float* features, void* meta_dev, cudaStream_t s) {
    // stack_rows (src/granite_features.rs:138-158) of rows first..last over `frames` frames: the
    // kernel's row r is local row r - row_first = r + first.
    if (last <= first) return TELMO_OK;
    StreamMetaHost h{0, 0, 0, 0, frames, -first};
    FrontMeta meta;
    const int* row_first = nullptr;
    if (int rc = stream_meta(&h, static_cast<uint8_t*>(meta_dev) + 128, meta, row_first, s)) return rc;
    granite_stack_kernel<<<last - first, 160, 0, s>>>(logs, meta, n_mels, peak, row_first,
                                                      features + static_cast<int64_t>(first) * 4 * n_mels);
    ++launches;
    return ctx->cuda(cudaGetLastError(), "stream front end");
}

}  // namespace telmo

using namespace telmo;

namespace {
struct FrontHandle {
    Ctx* ctx;
    FrontEnd fe;
};
}  // namespace

extern "C" int telmo_logmel(telmo_ctx* cp, int kind, const float* samples, const int64_t* lengths, int n_utt,
                            float* features, int* rows, void* stream) {
    Ctx* ctx = as_ctx(cp);
    if (!ctx) return TELMO_ERR_ARGUMENT;
    if (n_utt <= 0 || !samples || !lengths || !features || !rows)
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_logmel: bad arguments");
    if (kind != TELMO_FRONTEND_GRANITE && kind != TELMO_FRONTEND_PARAKEET)
        return ctx->fail(TELMO_ERR_ARGUMENT, "telmo_logmel: unknown front end %d", kind);
    if (int rc = ctx->use_device()) return rc;
    FrontEnd*& fe = kind == TELMO_FRONTEND_GRANITE ? ctx->granite_fe : ctx->parakeet_fe;
    if (!fe) {
        fe = new FrontEnd();
        fe->n_mels = kind == TELMO_FRONTEND_GRANITE ? 80 : 128;
        if (int rc = fe->init(ctx, kind == TELMO_FRONTEND_GRANITE ? FrontEnd::kGranite : FrontEnd::kParakeet)) {
            delete fe;
            fe = nullptr;
            return rc;
        }
    }
    return fe->run(samples, lengths, n_utt, features, rows, static_cast<cudaStream_t>(stream));
}

extern "C" size_t telmo_logmel_rows(int kind, int64_t samples) {
    if (kind == TELMO_FRONTEND_GRANITE) return samples < 2 * HOP ? 0 : static_cast<size_t>((samples / HOP + 1) / 2);
    if (kind == TELMO_FRONTEND_PARAKEET) return samples / HOP < 2 ? 0 : static_cast<size_t>(samples / HOP);
    return 0;
}
