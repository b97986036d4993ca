/*
 * frontend.c -- oracle restatement of telmo's two log-mel front ends.
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Compiled with -ffp-contract=off: every f32 step
 * rounds where the reference's does.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define N_FFT 512
#define WIN 400
#define HOP 160
#define BINS (N_FFT / 2 + 1)

typedef struct {
    size_t first_bin, count;
    float w[BINS];
} mel_filter;

/* torch.linspace in f32 (src/granite_features.rs:221-233). */
static void linspace_f32(float start, float end, size_t steps, float *out)
{
    float step = (end - start) / (float)(steps - 1);
    for (size_t i = 0; i < steps; i++)
        out[i] = i < steps / 2 ? start + step * (float)i : end - step * (float)(steps - 1 - i);
}

static void sparse_filter(const float *weights, mel_filter *f)
{
    size_t first = 0, last;
    int found = 0;
    for (size_t b = 0; b < BINS; b++)
        if (weights[b] != 0.0f) {
            first = b;
            found = 1;
            break;
        }
    last = first;
    if (found)
        for (size_t b = BINS; b-- > 0;)
            if (weights[b] != 0.0f) {
                last = b + 1;
                break;
            }
    f->first_bin = first;
    f->count = last - first;
    for (size_t b = 0; b < f->count; b++) f->w[b] = weights[first + b];
}

/* htk_mel_filters (src/granite_features.rs:236-271). */
static void htk_mel_filters(size_t n_mels, mel_filter *filters)
{
    double nyquist = 8000.0;
    float all_freqs[BINS];
    linspace_f32(0.0f, (float)nyquist, BINS, all_freqs);
    double m_max = 2595.0 * log10(1.0 + nyquist / 700.0);
    float *mels = (float *)malloc((n_mels + 2) * sizeof(float));
    float *f_pts = (float *)malloc((n_mels + 2) * sizeof(float));
    linspace_f32(0.0f, (float)m_max, n_mels + 2, mels);
    for (size_t i = 0; i < n_mels + 2; i++) {
        float p = (float)pow(10.0, (double)(mels[i] / 2595.0f));
        f_pts[i] = 700.0f * (p - 1.0f);
    }
    float weights[BINS];
    for (size_t m = 0; m < n_mels; m++) {
        float d0 = f_pts[m + 1] - f_pts[m], d1 = f_pts[m + 2] - f_pts[m + 1];
        for (size_t b = 0; b < BINS; b++) {
            float f = all_freqs[b];
            float down = -(f_pts[m] - f) / d0;
            float up = (f_pts[m + 2] - f) / d1;
            weights[b] = fmaxf(fminf(down, up), 0.0f);
        }
        sparse_filter(weights, &filters[m]);
    }
    free(mels);
    free(f_pts);
}

static double hz_to_mel_slaney(double hz)
{
    /* src/features.rs:354-365 */
    double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    double logstep = log(6.4) / 27.0;
    return hz >= min_log_hz ? min_log_mel + log(hz / min_log_hz) / logstep : hz / f_sp;
}

static double mel_to_hz_slaney(double mel)
{
    double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    double logstep = log(6.4) / 27.0;
    return mel >= min_log_mel ? min_log_hz * exp(logstep * (mel - min_log_mel)) : f_sp * mel;
}

/* slaney_mel_filters (src/features.rs:379-412). */
static void slaney_mel_filters(size_t n_mels, mel_filter *filters)
{
    double fft_freqs[BINS];
    for (size_t k = 0; k < BINS; k++) fft_freqs[k] = (double)k * 16000.0 / (double)N_FFT;
    double max_mel = hz_to_mel_slaney(8000.0);
    double *pts = (double *)malloc((n_mels + 2) * sizeof(double));
    for (size_t i = 0; i < n_mels + 2; i++)
        pts[i] = mel_to_hz_slaney(max_mel * (double)i / (double)(n_mels + 1));
    float weights[BINS];
    for (size_t m = 0; m < n_mels; m++) {
        double lo = pts[m], center = pts[m + 1], hi = pts[m + 2];
        double enorm = 2.0 / (hi - lo);
        for (size_t b = 0; b < BINS; b++) {
            double f = fft_freqs[b];
            double lower = (f - lo) / (center - lo), upper = (hi - f) / (hi - center);
            double w = fmin(lower, upper);
            float wf = (float)(w > 0.0 ? w : 0.0);
            weights[b] = (float)((double)wf * enorm);
        }
        sparse_filter(weights, &filters[m]);
    }
    free(pts);
}

size_t oracle_granite_rows_for(size_t samples)
{
    return (samples / HOP + 1) / 2; /* (samples / HOP).div_ceil(2) */
}

void oracle_granite_log_frames(const float *samples, size_t n, size_t len, size_t f0, size_t f1,
                               size_t n_mels, float *logs)
{
    /* log_frame (src/granite_features.rs:95-133) for frames f0..f1 into logs[(f - f0) * n_mels]:
     * the n samples zero-padded to len, reflected at both ends. */
    double window[N_FFT];
    memset(window, 0, sizeof window);
    /* periodic Hann 400 centered in 512 (src/granite_features.rs:47-52, :209-217). */
    float step = (float)(2.0 * M_PI / (double)WIN);
    for (size_t i = 0; i < WIN; i++) {
        float x = (float)i * step;
        window[(N_FFT - WIN) / 2 + i] = (double)(0.5f + -0.5f * (float)cos((double)x));
    }
    mel_filter *filters = (mel_filter *)malloc(n_mels * sizeof(mel_filter));
    htk_mel_filters(n_mels, filters);
    double seg[N_FFT], spec[2 * BINS], power[BINS];
    for (size_t f = f0; f < f1; f++) {
        long start = (long)(f * HOP) - N_FFT / 2;
        for (long i = 0; i < N_FFT; i++) {
            long j = start + i;
            size_t jj = j < 0 ? (size_t)(-j) : ((size_t)j >= len ? 2 * (len - 1) - (size_t)j : (size_t)j);
            double s = jj < n ? (double)samples[jj] : 0.0;
            seg[i] = s * window[i];
        }
        oracle_real_fft(seg, N_FFT, spec);
        for (size_t b = 0; b < BINS; b++)
            power[b] = spec[2 * b] * spec[2 * b] + spec[2 * b + 1] * spec[2 * b + 1];
        for (size_t m = 0; m < n_mels; m++) {
            double acc = 0.0;
            for (size_t k = 0; k < filters[m].count; k++)
                acc += (double)filters[m].w[k] * power[filters[m].first_bin + k];
            float energy = fmaxf((float)acc, 1e-10f);
            logs[(f - f0) * n_mels + m] = (float)log10((double)energy);
        }
    }
    free(filters);
}

void oracle_granite_stack_rows(const float *logs, size_t frames, size_t n_mels, float peak,
                               size_t first, size_t last, float *out)
{
    /* stack_rows (src/granite_features.rs:138-158): rows first..last into out[(row - first)]. */
    float floor_v = peak - 8.0f;
    for (size_t f = 2 * first; f < 2 * last; f++) {
        float *row = out + (f - 2 * first) * 2 * n_mels;
        size_t before = f ? f - 1 : 0, after = f + 1 < frames ? f + 1 : frames - 1;
        for (size_t m = 0; m < n_mels; m++) {
            float v = fmaxf(logs[f * n_mels + m], floor_v) / 4.0f + 1.0f;
            float va = fmaxf(logs[after * n_mels + m], floor_v) / 4.0f + 1.0f;
            float vb = fmaxf(logs[before * n_mels + m], floor_v) / 4.0f + 1.0f;
            row[m] = v;
            row[n_mels + m] = (va - vb) / 2.0f;
        }
    }
}

int oracle_granite_features(const float *samples, size_t n, size_t n_mels, float *out)
{
    /* GraniteFrontEnd::compute (src/granite_features.rs:161-186). */
    if (n < 2 * HOP) return -1;
    size_t rows = oracle_granite_rows_for(n), frames = 2 * rows;
    size_t len = (frames - 1) * HOP + 1;
    if (len < n) len = n;
    float *logs = (float *)malloc(frames * n_mels * sizeof(float));
    oracle_granite_log_frames(samples, n, len, 0, frames, n_mels, logs);
    float peak = -INFINITY;
    for (size_t i = 0; i < frames * n_mels; i++) peak = fmaxf(peak, logs[i]);
    oracle_granite_stack_rows(logs, frames, n_mels, peak, 0, rows, out);
    free(logs);
    return 0;
}

int oracle_parakeet_features(const float *samples, size_t n, float *out)
{
    /* FrontEnd::compute with FrontEndConfig::parakeet (src/features.rs:101-216). */
    const size_t n_mels = 128;
    size_t frames = n / HOP;
    if (frames < 2) return -1;
    const size_t pad = N_FFT / 2, offset = (N_FFT - WIN) / 2;
    double window[WIN];
    for (size_t i = 0; i < WIN; i++) {
        double w = 0.5 - 0.5 * cos(2.0 * M_PI * (double)i / (double)(WIN - 1));
        window[i] = (double)(float)w;
    }
    mel_filter *filters = (mel_filter *)malloc(n_mels * sizeof(mel_filter));
    slaney_mel_filters(n_mels, filters);
    /* pre-emphasis in f32, then centered zero padding (src/features.rs:120-134). */
    double *padded = (double *)calloc(n + 2 * pad, sizeof(double));
    padded[pad] = (double)samples[0];
    for (size_t i = 1; i < n; i++) {
        float e = 0.97f * samples[i - 1];
        padded[pad + i] = (double)(samples[i] - e);
    }
    double *logs = (double *)malloc(frames * n_mels * sizeof(double));
    double seg[N_FFT], spec[2 * BINS], power[BINS];
    memset(seg, 0, sizeof seg);
    const double guard = 1.0 / 16777216.0;
    for (size_t f = 0; f < frames; f++) {
        /* the window covers padded[f * hop + offset .. + 400] (window_span, :147-153). */
        const double *x = padded + f * HOP + offset;
        for (size_t i = 0; i < WIN; i++) seg[offset + i] = x[i] * window[i];
        oracle_real_fft(seg, N_FFT, spec);
        for (size_t b = 0; b < BINS; b++)
            power[b] = spec[2 * b] * spec[2 * b] + spec[2 * b + 1] * spec[2 * b + 1];
        for (size_t m = 0; m < n_mels; m++) {
            double acc = 0.0;
            for (size_t k = 0; k < filters[m].count; k++)
                acc += (double)filters[m].w[k] * power[filters[m].first_bin + k];
            logs[f * n_mels + m] = log(acc + guard);
        }
    }
    (void)pad;
    /* normalize (src/features.rs:199-216): per bin, std with n - 1, plus 1e-5. */
    for (size_t m = 0; m < n_mels; m++) {
        double sum = 0.0;
        for (size_t f = 0; f < frames; f++) sum += logs[f * n_mels + m];
        double mean = sum / (double)frames, var = 0.0;
        for (size_t f = 0; f < frames; f++) {
            double d = logs[f * n_mels + m] - mean;
            var += d * d;
        }
        var /= (double)(frames - 1);
        double scale = 1.0 / (sqrt(var) + 1e-5);
        for (size_t f = 0; f < frames; f++)
            out[f * n_mels + m] = (float)((logs[f * n_mels + m] - mean) * scale);
    }
    free(padded);
    free(logs);
    free(filters);
    return 0;
}
