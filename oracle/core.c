/*
 * core.c -- oracle restatement of telmo's quantization, matrix product and row kernels.
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Compiled with -ffp-contract=off so that every fused
 * multiply-add here is an explicit fmaf, as in the reference's SIMD tiles.
 */
#include "oracle.h"
#include "pool.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define PANEL 16 /* src/kernels/mod.rs:30 */
#define KC 256   /* src/kernels/mod.rs:34 */

/* ---- quant.rs ---------------------------------------------------------------------------- */

float oracle_quantize_row_int8(const float *x, size_t k, int8_t *q)
{
    /* src/quant.rs:190-198: amax / 127, values rounded half away from zero and clamped. */
    float amax = 0.0f;
    for (size_t i = 0; i < k; i++) amax = fmaxf(amax, fabsf(x[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (size_t i = 0; i < k; i++) {
        float v = roundf(x[i] * id);
        if (v < -127.0f) v = -127.0f;
        if (v > 127.0f) v = 127.0f;
        q[i] = (int8_t)v;
    }
    return d;
}

void oracle_encode_int8(const float *w, size_t n, size_t k, int8_t *values, float *scales)
{
    /* src/quant.rs:202-269, Precision::Int8: panel p holds k runs of 16 outputs. */
    size_t panels = (n + PANEL - 1) / PANEL;
    memset(values, 0, panels * k * PANEL);
    memset(scales, 0, panels * PANEL * sizeof(float));
    int8_t *q = (int8_t *)malloc(k ? k : 1);
    for (size_t o = 0; o < n; o++) {
        size_t p = o / PANEL, j = o % PANEL;
        scales[p * PANEL + j] = oracle_quantize_row_int8(w + o * k, k, q);
        for (size_t i = 0; i < k; i++) values[(p * k + i) * PANEL + j] = q[i];
    }
    free(q);
}

void oracle_decode_int8(const int8_t *values, const float *scales, size_t n, size_t k, float *out)
{
    /* src/quant.rs:281-303: w = (q as f32) * scale, one rounding. */
    for (size_t o = 0; o < n; o++) {
        size_t p = o / PANEL, j = o % PANEL;
        for (size_t i = 0; i < k; i++)
            out[o * k + i] = (float)values[(p * k + i) * PANEL + j] * scales[p * PANEL + j];
    }
}

/* quantize_q8_0_block (src/quant.rs:172-183): d = amax / 127, q = round(x * (1 / d)) with the
 * unrounded d, saturating to i8 as Rust's `as i8` does; returns d as its f16 value. */
static float quantize_q8_0_block(const float *x, int8_t *q)
{
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int i = 0; i < 32; i++) {
        float v = roundf(x[i] * id);
        if (v < -128.0f) v = -128.0f;
        if (v > 127.0f) v = 127.0f;
        q[i] = (int8_t)v;
    }
    return oracle_f16_to_f32(oracle_f32_to_f16(d));
}

void oracle_encode_q8_0(const float *w, size_t n, size_t k, int8_t *values, float *scales)
{
    /* src/quant.rs:202-269, Precision::Q8_0: the int8 panels as Int8's; scales per block of 32
     * inputs, in panel order, then block order, then output. k is a multiple of 32. */
    size_t panels = (n + PANEL - 1) / PANEL, blocks = k / 32;
    memset(values, 0, panels * k * PANEL);
    memset(scales, 0, panels * blocks * PANEL * sizeof(float));
    int8_t q[32];
    for (size_t o = 0; o < n; o++) {
        size_t p = o / PANEL, j = o % PANEL;
        for (size_t b = 0; b < blocks; b++) {
            scales[(p * blocks + b) * PANEL + j] = quantize_q8_0_block(w + o * k + 32 * b, q);
            for (int i = 0; i < 32; i++) values[(p * k + 32 * b + i) * PANEL + j] = q[i];
        }
    }
}

void oracle_decode_q8_0(const int8_t *values, const float *scales, size_t n, size_t k, float *out)
{
    /* src/quant.rs:281-303: w = (q as f32) * d[block], exact (d is an f16 value). */
    size_t blocks = k / 32;
    for (size_t o = 0; o < n; o++) {
        size_t p = o / PANEL, j = o % PANEL;
        for (size_t i = 0; i < k; i++)
            out[o * k + i] =
                (float)values[(p * k + i) * PANEL + j] * scales[(p * blocks + i / 32) * PANEL + j];
    }
}

uint16_t oracle_f32_to_bf16(float x)
{
    /* src/quant.rs:149-156 */
    uint32_t bits;
    memcpy(&bits, &x, 4);
    if (isnan(x)) return (uint16_t)((bits >> 16) | 0x40);
    return (uint16_t)((bits + 0x7fff + ((bits >> 16) & 1)) >> 16);
}

float oracle_bf16_to_f32(uint16_t h)
{
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t oracle_f32_to_f16(float x)
{
    /* src/quant.rs:92-126, round to nearest even. */
    uint32_t bits;
    memcpy(&bits, &x, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    int32_t exp = (int32_t)((bits >> 23) & 0xff);
    uint32_t man = bits & 0x7fffff;
    if (exp == 0xff) {
        uint16_t nan = man ? (uint16_t)(0x200 | (man >> 13)) : 0;
        return sign | 0x7c00 | nan;
    }
    int32_t e = exp - 127 + 15;
    if (e >= 0x1f) return sign | 0x7c00;
    if (e <= 0) {
        uint32_t shift = (uint32_t)(126 - exp);
        if (shift > 24) return sign;
        uint32_t full = man | 0x800000;
        uint32_t m = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (m & 1))) m++;
        return sign | (uint16_t)m;
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return sign | (uint16_t)h;
}

float oracle_f16_to_f32(uint16_t h)
{
    /* src/quant.rs:128-146 */
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0 && man == 0) bits = sign;
    else if (exp == 0) {
        float v = (float)man * (1.0f / 16777216.0f);
        return sign ? -v : v;
    } else if (exp == 0x1f && man) bits = sign | 0x7fc00000 | (man << 13);
    else if (exp == 0x1f) bits = sign | 0x7f800000;
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ---- kernels/mod.rs: the matrix product --------------------------------------------------- */

static inline float activate(float v, int act)
{
    /* src/kernels/scalar.rs:110-116 */
    switch (act) {
    case ORACLE_ACT_RELU: return fmaxf(v, 0.0f);
    case ORACLE_ACT_SILU: return v / (1.0f + expf(-v));
    default: return v;
    }
}

static inline void store_row(const float *acc, float *c, size_t cols, const float *bias, int act,
                             float scale, int accumulate)
{
    /* src/kernels/scalar.rs:118-124 */
    for (size_t j = 0; j < cols; j++) {
        float v = acc[j] + (bias ? bias[j] : 0.0f);
        v = activate(v, act) * scale;
        c[j] = accumulate ? c[j] + v : v;
    }
}

/* A rows x 16 tile of a . b over kc inputs, b holding kc runs of 16 values k_stride apart:
 * out[r][j] = fma(a[r][i], b[i][j], out[r][j]) for ascending i (src/kernels/mod.rs:885-931,
 * the fused form the AVX2/AVX-512 tiles compute). */
static void tile_generic(size_t kc, const float *a, size_t lda, size_t rows, const float *b,
                         size_t k_stride, float *out, int load)
{
    for (size_t r = 0; r < rows; r++) {
        float acc[PANEL];
        for (int j = 0; j < PANEL; j++) acc[j] = load ? out[r * PANEL + j] : 0.0f;
        for (size_t i = 0; i < kc; i++) {
            float av = a[r * lda + i];
            const float *bp = b + i * k_stride;
            for (int j = 0; j < PANEL; j++) acc[j] = fmaf(av, bp[j], acc[j]);
        }
        memcpy(out + r * PANEL, acc, sizeof acc);
    }
}

#if defined(__x86_64__)
/* R x 16 register tiles, the AVX-512 shape (8 rows, src/kernels/avx512.rs:15, :43-106) and the
 * AVX2 shape (6 rows, src/kernels/mod.rs:31), one function per row count so the accumulators
 * stay in registers; every row sums in the same fused order as tile_generic. */
#define TELMO_TILE512(R)                                                                        \
    __attribute__((target("avx512f,fma"))) static void tile512_##R(                             \
        size_t kc, const float *a, size_t lda, const float *b, size_t k_stride, float *out,     \
        int load)                                                                               \
    {                                                                                           \
        __m512 c[R];                                                                            \
        for (int r = 0; r < R; r++)                                                             \
            c[r] = load ? _mm512_loadu_ps(out + r * PANEL) : _mm512_setzero_ps();               \
        for (size_t i = 0; i < kc; i++) {                                                       \
            __m512 bv = _mm512_loadu_ps(b + i * k_stride);                                      \
            for (int r = 0; r < R; r++)                                                         \
                c[r] = _mm512_fmadd_ps(_mm512_set1_ps(a[r * lda + i]), bv, c[r]);               \
        }                                                                                       \
        for (int r = 0; r < R; r++) _mm512_storeu_ps(out + r * PANEL, c[r]);                    \
    }
TELMO_TILE512(1) TELMO_TILE512(2) TELMO_TILE512(3) TELMO_TILE512(4)
TELMO_TILE512(5) TELMO_TILE512(6) TELMO_TILE512(7) TELMO_TILE512(8)

__attribute__((target("avx512f,fma"))) static void
tile_avx512(size_t kc, const float *a, size_t lda, size_t rows, const float *b, size_t k_stride,
            float *out, int load)
{
    switch (rows) {
    case 1: tile512_1(kc, a, lda, b, k_stride, out, load); break;
    case 2: tile512_2(kc, a, lda, b, k_stride, out, load); break;
    case 3: tile512_3(kc, a, lda, b, k_stride, out, load); break;
    case 4: tile512_4(kc, a, lda, b, k_stride, out, load); break;
    case 5: tile512_5(kc, a, lda, b, k_stride, out, load); break;
    case 6: tile512_6(kc, a, lda, b, k_stride, out, load); break;
    case 7: tile512_7(kc, a, lda, b, k_stride, out, load); break;
    default: tile512_8(kc, a, lda, b, k_stride, out, load); break;
    }
}

#define TELMO_TILE256(R)                                                                        \
    __attribute__((target("avx2,fma"))) static void tile256_##R(                                \
        size_t kc, const float *a, size_t lda, const float *b, size_t k_stride, float *out,     \
        int load)                                                                               \
    {                                                                                           \
        __m256 c[2 * R];                                                                        \
        for (int r = 0; r < R; r++) {                                                           \
            c[2 * r] = load ? _mm256_loadu_ps(out + r * PANEL) : _mm256_setzero_ps();           \
            c[2 * r + 1] = load ? _mm256_loadu_ps(out + r * PANEL + 8) : _mm256_setzero_ps();   \
        }                                                                                       \
        for (size_t i = 0; i < kc; i++) {                                                       \
            __m256 b0 = _mm256_loadu_ps(b + i * k_stride);                                      \
            __m256 b1 = _mm256_loadu_ps(b + i * k_stride + 8);                                  \
            for (int r = 0; r < R; r++) {                                                       \
                __m256 av = _mm256_set1_ps(a[r * lda + i]);                                     \
                c[2 * r] = _mm256_fmadd_ps(av, b0, c[2 * r]);                                   \
                c[2 * r + 1] = _mm256_fmadd_ps(av, b1, c[2 * r + 1]);                           \
            }                                                                                   \
        }                                                                                       \
        for (int r = 0; r < R; r++) {                                                           \
            _mm256_storeu_ps(out + r * PANEL, c[2 * r]);                                        \
            _mm256_storeu_ps(out + r * PANEL + 8, c[2 * r + 1]);                                \
        }                                                                                       \
    }
TELMO_TILE256(1) TELMO_TILE256(2) TELMO_TILE256(3) TELMO_TILE256(4) TELMO_TILE256(5)
TELMO_TILE256(6)

__attribute__((target("avx2,fma"))) static void
tile_avx2(size_t kc, const float *a, size_t lda, size_t rows, const float *b, size_t k_stride,
          float *out, int load)
{
    switch (rows) {
    case 1: tile256_1(kc, a, lda, b, k_stride, out, load); break;
    case 2: tile256_2(kc, a, lda, b, k_stride, out, load); break;
    case 3: tile256_3(kc, a, lda, b, k_stride, out, load); break;
    case 4: tile256_4(kc, a, lda, b, k_stride, out, load); break;
    case 5: tile256_5(kc, a, lda, b, k_stride, out, load); break;
    default: tile256_6(kc, a, lda, b, k_stride, out, load); break;
    }
}

/* widen (src/kernels/avx512.rs:221): 16 int8 values to f32, times the panel's scales. */
__attribute__((target("avx512f"))) static void
widen_avx512(size_t kc, const int8_t *src, const float *scales, float *out)
{
    __m512 s = _mm512_loadu_ps(scales);
    for (size_t i = 0; i < kc; i++) {
        __m128i q = _mm_loadu_si128((const __m128i *)(src + i * PANEL));
        __m512 v = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(q));
        _mm512_storeu_ps(out + i * PANEL, _mm512_mul_ps(v, s));
    }
}
#endif

static int have_avx512(void)
{
#if defined(__x86_64__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("fma");
#else
    return 0;
#endif
}

typedef void (*tile_fn)(size_t, const float *, size_t, size_t, const float *, size_t, float *, int);

static tile_fn pick_tile(size_t *tile_rows)
{
#if defined(__x86_64__)
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("fma")) {
        *tile_rows = 8;
        return tile_avx512;
    }
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) {
        *tile_rows = 6;
        return tile_avx2;
    }
#endif
    *tile_rows = 6;
    return tile_generic;
}

typedef struct {
    const float *a;
    size_t lda, m;
    const int8_t *values; /* int8 panels, or NULL for a row-major f32 b */
    const float *scales;
    int q8;               /* values are Q8_0: one scale per 32 inputs */
    const float *b;       /* row-major f32 [k, ldb] */
    size_t ldb, n, k;
    float *c;
    size_t ldc;
    const float *bias;
    int act;
    float scale;
    int accumulate;
    size_t per_task, panels;
} gemm_job;

/* gemm_panels (src/kernels/mod.rs:530-653) for the panels of one task. */
static void gemm_panels(const gemm_job *J, size_t p0, size_t p1)
{
    size_t tile_rows;
    tile_fn tile = pick_tile(&tile_rows);
    const int avx512 = have_avx512();
    (void)avx512;
    size_t k = J->k;
    float *wide = (float *)malloc(KC * PANEL * sizeof(float));
    float *partial = (float *)malloc((J->m ? J->m : 1) * PANEL * sizeof(float));
    for (size_t p = p0; p < p1; p++) {
        size_t col = p * PANEL;
        size_t cols = J->n - col < PANEL ? J->n - col : PANEL;
        for (size_t k0 = 0; k0 < k; k0 += KC) {
            size_t kc = k - k0 < KC ? k - k0 : KC;
            const float *bp;
            size_t k_stride;
            if (J->values) {
                /* widen (src/kernels/scalar.rs:82-106): q as f32 * scale, the scale of the
                 * input's block of 32 for Q8_0 (src/kernels/mod.rs:577). */
                const int8_t *src = J->values + (p * k + k0) * PANEL;
                if (J->q8) {
                    const float *s = J->scales + (p * (k / 32) + k0 / 32) * PANEL;
                    for (size_t i = 0; i < kc; i++)
                        for (int j = 0; j < PANEL; j++)
                            wide[i * PANEL + j] = (float)src[i * PANEL + j] * s[(i / 32) * PANEL + j];
                } else {
                const float *s = J->scales + p * PANEL;
#if defined(__x86_64__)
                if (avx512)
                    widen_avx512(kc, src, s, wide);
                else
#endif
                    for (size_t i = 0; i < kc; i++)
                        for (int j = 0; j < PANEL; j++)
                            wide[i * PANEL + j] = (float)src[i * PANEL + j] * s[j];
                }
                bp = wide;
                k_stride = PANEL;
            } else {
                /* BView::row_major reads 16 columns of each row; columns past n are padding. */
                if (cols == PANEL) {
                    bp = J->b + k0 * J->ldb + col;
                    k_stride = J->ldb;
                } else {
                    for (size_t i = 0; i < kc; i++)
                        for (int j = 0; j < PANEL; j++)
                            wide[i * PANEL + j] =
                                (size_t)j < cols ? J->b[(k0 + i) * J->ldb + col + j] : 0.0f;
                    bp = wide;
                    k_stride = PANEL;
                }
            }
            for (size_t row = 0; row < J->m; row += tile_rows) {
                size_t rows = J->m - row < tile_rows ? J->m - row : tile_rows;
                tile(kc, J->a + row * J->lda + k0, J->lda, rows, bp, k_stride,
                     partial + row * PANEL, k0 > 0);
            }
        }
        if (k == 0) memset(partial, 0, J->m * PANEL * sizeof(float));
        for (size_t r = 0; r < J->m; r++)
            store_row(partial + r * PANEL, J->c + r * J->ldc + col, cols,
                      J->bias ? J->bias + col : NULL, J->act, J->scale, J->accumulate);
    }
    free(wide);
    free(partial);
}

static void gemm_task(void *ctx, size_t t)
{
    const gemm_job *J = (const gemm_job *)ctx;
    size_t p0 = t * J->per_task, p1 = p0 + J->per_task;
    if (p1 > J->panels) p1 = J->panels;
    gemm_panels(J, p0, p1);
}

static void run_gemm(gemm_job *J, int threads)
{
    if (J->m == 0 || J->n == 0) return;
    J->panels = (J->n + PANEL - 1) / PANEL;
    if (threads < 1) threads = 1;
    /* A few tasks per thread (src/kernels/mod.rs:678-687). */
    size_t per = (J->panels + (size_t)threads * 4 - 1) / ((size_t)threads * 4);
    J->per_task = per ? per : 1;
    size_t tasks = (J->panels + J->per_task - 1) / J->per_task;
    oracle_parallel_for(tasks, threads, gemm_task, J);
}

void oracle_linear_int8(const float *a, size_t lda, size_t m, const int8_t *values,
                        const float *scales, size_t n, size_t k, float *c, size_t ldc,
                        const float *bias, int act, float scale, int accumulate, int threads)
{
    gemm_job J = {a, lda, m, values, scales, 0, NULL, 0, n, k, c, ldc, bias, act, scale, accumulate,
                  0, 0};
    run_gemm(&J, threads);
}

void oracle_linear_q8_0(const float *a, size_t lda, size_t m, const int8_t *values,
                        const float *scales, size_t n, size_t k, float *c, size_t ldc,
                        const float *bias, int act, float scale, int accumulate, int threads)
{
    gemm_job J = {a, lda, m, values, scales, 1, NULL, 0, n, k, c, ldc, bias, act, scale, accumulate,
                  0, 0};
    run_gemm(&J, threads);
}

void oracle_matmul_rowmajor(const float *a, size_t lda, size_t m, const float *b, size_t k,
                            size_t n, size_t ldb, float *c, size_t ldc, const float *bias, int act,
                            float scale, int accumulate)
{
    gemm_job J = {a, lda, m, NULL, NULL, 0, b, ldb, n, k, c, ldc, bias, act, scale, accumulate, 0, 0};
    run_gemm(&J, 1);
}

/* ---- the split int8 activation rule ------------------------------------------------------- */

void oracle_quantize_x2(const float *x, size_t m, size_t k, size_t ldx, int8_t *hi, int8_t *lo,
                        size_t ldq, float *row_scale)
{
    for (size_t r = 0; r < m; r++) {
        const float *row = x + r * ldx;
        float amax = 0.0f;
        for (size_t i = 0; i < k; i++) amax = fmaxf(amax, fabsf(row[i]));
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        float id_lo = id * 254.0f;
        for (size_t i = 0; i < k; i++) {
            /* Each level rounded to the nearest integer, halves to even (the default mode). */
            float h = nearbyintf(row[i] * id);
            h = fminf(fmaxf(h, -127.0f), 127.0f);
            float e = fmaf(-h, d, row[i]);
            float l = nearbyintf(e * id_lo);
            l = fminf(fmaxf(l, -127.0f), 127.0f);
            hi[r * ldq + i] = (int8_t)h;
            lo[r * ldq + i] = (int8_t)l;
        }
        for (size_t i = k; i < ldq; i++) hi[r * ldq + i] = lo[r * ldq + i] = 0;
        row_scale[r] = d;
    }
}

void oracle_gemm_i8_x2_acc(const int8_t *hi, const int8_t *lo, size_t ldq, size_t m,
                           const int8_t *values, size_t n, size_t k, int32_t *acc_hi,
                           int32_t *acc_lo)
{
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            const int8_t *w = values + (j / PANEL) * k * PANEL + (j % PANEL);
            int32_t sh = 0, sl = 0;
            for (size_t t = 0; t < k; t++) {
                int32_t wv = w[t * PANEL];
                sh += (int32_t)hi[i * ldq + t] * wv;
                sl += (int32_t)lo[i * ldq + t] * wv;
            }
            acc_hi[i * n + j] = sh;
            acc_lo[i * n + j] = sl;
        }
}

void oracle_q8_0_two_level(const int8_t *values, const float *scales, size_t n, size_t k,
                           int8_t *w_hi, int8_t *w_lo, float *w_scale)
{
    /* The CUDA upload's re-encoding of a Q8_0 row (test restatement): w = q * d[block] exact,
     * then the split rule of oracle_quantize_x2 with one scale per row. */
    float *w = (float *)malloc((k ? k : 1) * sizeof(float));
    for (size_t o = 0; o < n; o++) {
        size_t p = o / PANEL, j = o % PANEL, blocks = k / 32;
        for (size_t i = 0; i < k; i++)
            w[i] = (float)values[(p * k + i) * PANEL + j] * scales[(p * blocks + i / 32) * PANEL + j];
        oracle_quantize_x2(w, 1, k, k, w_hi + o * k, w_lo + o * k, k, w_scale + o);
    }
    free(w);
}

void oracle_gemm_i8_x2w_acc(const int8_t *hi, const int8_t *lo, size_t ldq, size_t m,
                            const int8_t *w_hi, const int8_t *w_lo, size_t n, size_t k,
                            int32_t *acc_hi, int32_t *acc_lo)
{
    /* Two-level weights (row-major [n, k]): acc_hi = hi . W_hi, acc_lo = lo . W_hi + hi . W_lo. */
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            int32_t sh = 0, sl = 0;
            for (size_t t = 0; t < k; t++) {
                int32_t a = hi[i * ldq + t], b = lo[i * ldq + t];
                sh += a * w_hi[j * k + t];
                sl += b * w_hi[j * k + t] + a * w_lo[j * k + t];
            }
            acc_hi[i * n + j] = sh;
            acc_lo[i * n + j] = sl;
        }
}

void oracle_epilogue_x2(const int32_t *acc_hi, const int32_t *acc_lo, size_t m, size_t n,
                        const float *row_scale, const float *w_scales, const float *bias, int act,
                        float scale, int accumulate, float *c, size_t ldc)
{
    const float inv254 = 1.0f / 254.0f;
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            float lo = (float)acc_lo[i * n + j] * inv254;
            float v = (float)acc_hi[i * n + j] + lo;
            v = v * row_scale[i];
            v = v * w_scales[j];
            if (bias) v = v + bias[j];
            v = activate(v, act) * scale;
            c[i * ldc + j] = accumulate ? c[i * ldc + j] + v : v;
        }
}

/* ---- kernels/scalar.rs: row kernels -------------------------------------------------------- */

void oracle_layer_norm(const float *x, float *out, const float *gamma, const float *beta,
                       size_t n, float eps)
{
    /* src/kernels/scalar.rs:126-134: mean and variance in f64. */
    double sum = 0.0;
    for (size_t i = 0; i < n; i++) sum += (double)x[i];
    double mean = sum / (double)n, var = 0.0;
    for (size_t i = 0; i < n; i++) {
        double d = (double)x[i] - mean;
        var += d * d;
    }
    var /= (double)n;
    double rstd = 1.0 / sqrt(var + (double)eps);
    for (size_t i = 0; i < n; i++) {
        float y = (float)(((double)x[i] - mean) * rstd);
        out[i] = y * gamma[i] + beta[i];
    }
}

void oracle_softmax(float *x, size_t n)
{
    /* src/kernels/scalar.rs:136-147: f32 exponentials, f64 sum, one f32 reciprocal. */
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
    double sum = 0.0;
    for (size_t i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += (double)x[i];
    }
    float inv = (float)(1.0 / sum);
    for (size_t i = 0; i < n; i++) x[i] *= inv;
}

void oracle_glu(const float *a, const float *b, float *out, size_t n)
{
    for (size_t i = 0; i < n; i++) out[i] = a[i] / (1.0f + expf(-b[i])); /* scalar.rs:149 */
}

void oracle_silu(float *x, size_t n)
{
    for (size_t i = 0; i < n; i++) x[i] = activate(x[i], ORACLE_ACT_SILU); /* scalar.rs:155 */
}

void oracle_dwconv1d_frame(const float *input, size_t channels, size_t frames, size_t t,
                           const float *w, size_t kernel, const float *bias, float *out)
{
    /* src/kernels/scalar.rs:164-187: "same" zero padding, weights [kernel, channels]. */
    memcpy(out, bias, channels * sizeof(float));
    size_t half = kernel / 2;
    for (size_t j = 0; j < kernel; j++) {
        if (t + j < half) continue;
        size_t src = t + j - half;
        if (src >= frames) continue;
        const float *row = input + src * channels, *wj = w + j * channels;
        for (size_t c = 0; c < channels; c++) out[c] += wj[c] * row[c];
    }
}

void oracle_conv3x3s2_row(const float *input, size_t in_t, size_t in_f, size_t channels,
                          int depthwise, const float *w, const float *bias, size_t t, float *out)
{
    /* src/kernels/scalar.rs:194-232 */
    size_t out_f = (in_f - 1) / 2 + 1;
    for (size_t f = 0; f < out_f; f++) {
        float *o = out + f * channels;
        memcpy(o, bias, channels * sizeof(float));
        for (size_t dt = 0; dt < 3; dt++) {
            if (2 * t + dt < 1) continue;
            size_t st = 2 * t + dt - 1;
            if (st >= in_t) continue;
            for (size_t df = 0; df < 3; df++) {
                if (2 * f + df < 1) continue;
                size_t sf = 2 * f + df - 1;
                if (sf >= in_f) continue;
                const float *wk = w + (dt * 3 + df) * channels;
                if (depthwise) {
                    const float *src = input + (st * in_f + sf) * channels;
                    for (size_t c = 0; c < channels; c++) o[c] += wk[c] * src[c];
                } else {
                    float v = input[st * in_f + sf];
                    for (size_t c = 0; c < channels; c++) o[c] += wk[c] * v;
                }
            }
        }
    }
}

/* ---- fft.rs -------------------------------------------------------------------------------- */

int oracle_real_fft(const double *input, size_t n, double *out)
{
    /* RealFft::new + forward (src/fft.rs:57-134): n/2-point complex radix-2 DIT on packed
     * even/odd samples, then the split into n/2 + 1 real-transform bins. */
    if (n < 4 || (n & (n - 1))) return -1;
    size_t m = n / 2, bits = 0;
    while (((size_t)1 << bits) < m) bits++;
    double *sr = (double *)malloc(m * sizeof(double)), *si = (double *)malloc(m * sizeof(double));
    for (size_t i = 0; i < m; i++) {
        size_t r = 0;
        for (size_t b = 0; b < bits; b++)
            if (i & ((size_t)1 << b)) r |= (size_t)1 << (bits - 1 - b);
        sr[r] = input[2 * i];
        si[r] = input[2 * i + 1];
    }
    for (size_t size = 2; size <= m; size *= 2) {
        size_t half = size / 2, step = m / size;
        for (size_t start = 0; start < m; start += size)
            for (size_t j = 0; j < half; j++) {
                double ang = -2.0 * M_PI * (double)(j * step) / (double)m;
                double wr = cos(ang), wi = sin(ang);
                double ar = sr[start + j], ai = si[start + j];
                double xr = sr[start + j + half], xi = si[start + j + half];
                double br = xr * wr - xi * wi, bi = xr * wi + xi * wr;
                sr[start + j] = ar + br;
                si[start + j] = ai + bi;
                sr[start + j + half] = ar - br;
                si[start + j + half] = ai - bi;
            }
    }
    for (size_t k = 0; k <= m; k++) {
        double zr = sr[k % m], zi = si[k % m];
        double cr = sr[(m - k) % m], ci = -si[(m - k) % m];
        double er = (zr + cr) * 0.5, ei = (zi + ci) * 0.5;
        double dr = zr - cr, di = zi - ci;
        double orr = di * 0.5, oi = -dr * 0.5;
        double ang = -2.0 * M_PI * (double)k / (double)n;
        double wr = cos(ang), wi = sin(ang);
        out[2 * k] = er + (wr * orr - wi * oi);
        out[2 * k + 1] = ei + (wr * oi + wi * orr);
    }
    free(sr);
    free(si);
    return 0;
}

size_t oracle_ctc_tokens(const uint32_t *ids, size_t frames, uint32_t blank, uint32_t *out)
{
    /* ctc_tokens (src/granite.rs:1074-1094): repeats merge, blanks drop, a blank between two
     * equal ids separates them. */
    size_t count = 0;
    int have_prev = 0;
    uint32_t prev = 0;
    for (size_t f = 0; f < frames; f++) {
        uint32_t id = ids[f];
        if (id != blank) {
            if (have_prev && prev == id) {
                if (count) out[3 * (count - 1) + 2] += 1;
            } else {
                out[3 * count] = id;
                out[3 * count + 1] = (uint32_t)f;
                out[3 * count + 2] = 1;
                count++;
            }
        }
        prev = id;
        have_prev = 1;
    }
    return count;
}
