/*
 * granite.c -- oracle restatement of telmo's Granite Speech CTC encoder and greedy CTC decode.
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 */
#include "oracle.h"
#include "pool.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int8_t *v;
    float *s;
    size_t n, k;
    int q8; /* Precision::Q8_0: one scale per 32 inputs */
} mat;

/* Kernels::linear over a matrix in either 8-bit precision. */
static void mat_linear(const float *a, size_t lda, size_t m, const mat *w, float *c, size_t ldc,
                       const float *bias, int act, float scale, int accumulate, int threads)
{
    if (w->q8)
        oracle_linear_q8_0(a, lda, m, w->v, w->s, w->n, w->k, c, ldc, bias, act, scale, accumulate,
                           threads);
    else
        oracle_linear_int8(a, lda, m, w->v, w->s, w->n, w->k, c, ldc, bias, act, scale, accumulate,
                           threads);
}
typedef struct {
    float *p;
    size_t len;
} vec;
typedef struct {
    mat w;
    vec b;
} lin;
typedef struct {
    vec g, b;
} norm;
typedef struct {
    norm norm;
    lin up, down;
} ffm;
typedef struct {
    int strided;
    ffm ff1, ff2;
    norm norm_att, norm_conv, norm_out;
    mat qkv, rel;
    lin out, pw1, pw2;
    vec dw_w, dw_b;
} block;

struct oracle_granite {
    oracle_granite_config c;
    lin input, head, mid;
    block *blocks;
};

oracle_granite *oracle_granite_new(const oracle_granite_config *config)
{
    if (config->layers < 2 || config->layers > 256 || config->heads <= 0 ||
        config->heads * config->head_dim != config->d_model || config->conv_kernel % 2 == 0 ||
        config->context <= 0 || config->n_subsample < 0 || config->n_subsample > 8)
        return NULL;
    oracle_granite *g = (oracle_granite *)calloc(1, sizeof *g);
    g->c = *config;
    g->blocks = (block *)calloc((size_t)config->layers, sizeof(block));
    for (int i = 0; i < config->layers; i++)
        for (int s = 0; s < config->n_subsample; s++)
            if (config->subsample_layers[s] == i) g->blocks[i].strided = 1;
    return g;
}

static void free_mat(mat *m) { free(m->v); free(m->s); }
static void free_lin(lin *l) { free_mat(&l->w); free(l->b.p); }
static void free_norm(norm *n) { free(n->g.p); free(n->b.p); }
static void free_ff(ffm *f) { free_norm(&f->norm); free_lin(&f->up); free_lin(&f->down); }

void oracle_granite_free(oracle_granite *g)
{
    if (!g) return;
    free_lin(&g->input);
    free_lin(&g->head);
    free_lin(&g->mid);
    for (int i = 0; i < g->c.layers; i++) {
        block *b = &g->blocks[i];
        free_ff(&b->ff1);
        free_ff(&b->ff2);
        free_norm(&b->norm_att);
        free_norm(&b->norm_conv);
        free_norm(&b->norm_out);
        free_mat(&b->qkv);
        free_mat(&b->rel);
        free_lin(&b->out);
        free_lin(&b->pw1);
        free_lin(&b->pw2);
        free(b->dw_w.p);
        free(b->dw_b.p);
    }
    free(g->blocks);
    free(g);
}

/* Expected shapes of every entry, as Granite::from_pack asks for them (src/granite.rs:443-500). */
static mat *find_mat(oracle_granite *g, const char *name, size_t *n, size_t *k)
{
    const oracle_granite_config *c = &g->c;
    size_t d = (size_t)c->d_model, cc = (size_t)c->conv_channels;
    if (!strcmp(name, "input")) { *n = d; *k = 4 * (size_t)c->n_mels; return &g->input.w; }
    if (!strcmp(name, "head")) { *n = (size_t)c->vocab; *k = d; return &g->head.w; }
    if (!strcmp(name, "mid")) { *n = d; *k = (size_t)c->vocab; return &g->mid.w; }
    int i, used = 0;
    char rest[64];
    if (sscanf(name, "blocks.%d.%63s%n", &i, rest, &used) != 2 || i < 0 || i >= c->layers)
        return NULL;
    block *b = &g->blocks[i];
    if (!strcmp(rest, "ff1.up")) { *n = (size_t)c->ff; *k = d; return &b->ff1.up.w; }
    if (!strcmp(rest, "ff1.down")) { *n = d; *k = (size_t)c->ff; return &b->ff1.down.w; }
    if (!strcmp(rest, "ff2.up")) { *n = (size_t)c->ff; *k = d; return &b->ff2.up.w; }
    if (!strcmp(rest, "ff2.down")) { *n = d; *k = (size_t)c->ff; return &b->ff2.down.w; }
    if (!strcmp(rest, "qkv")) { *n = 3 * d; *k = d; return &b->qkv; }
    if (!strcmp(rest, "rel")) {
        *n = 2 * (size_t)c->context - 1;
        *k = (size_t)c->head_dim;
        return &b->rel;
    }
    if (!strcmp(rest, "out")) { *n = d; *k = d; return &b->out.w; }
    if (!strcmp(rest, "pw1")) { *n = 2 * cc; *k = d; return &b->pw1.w; }
    if (!strcmp(rest, "pw2")) { *n = d; *k = cc; return &b->pw2.w; }
    return NULL;
}

static vec *find_vec(oracle_granite *g, const char *name, size_t *len)
{
    const oracle_granite_config *c = &g->c;
    size_t d = (size_t)c->d_model, cc = (size_t)c->conv_channels;
    if (!strcmp(name, "input.b")) { *len = d; return &g->input.b; }
    if (!strcmp(name, "head.b")) { *len = (size_t)c->vocab; return &g->head.b; }
    if (!strcmp(name, "mid.b")) { *len = d; return &g->mid.b; }
    int i;
    char rest[64];
    if (sscanf(name, "blocks.%d.%63s", &i, rest) != 2 || i < 0 || i >= c->layers) return NULL;
    block *b = &g->blocks[i];
    struct { const char *n; vec *v; size_t len; } table[] = {
        {"ff1.norm.w", &b->ff1.norm.g, d}, {"ff1.norm.b", &b->ff1.norm.b, d},
        {"ff1.up.b", &b->ff1.up.b, (size_t)c->ff}, {"ff1.down.b", &b->ff1.down.b, d},
        {"ff2.norm.w", &b->ff2.norm.g, d}, {"ff2.norm.b", &b->ff2.norm.b, d},
        {"ff2.up.b", &b->ff2.up.b, (size_t)c->ff}, {"ff2.down.b", &b->ff2.down.b, d},
        {"norm_att.w", &b->norm_att.g, d}, {"norm_att.b", &b->norm_att.b, d},
        {"out.b", &b->out.b, d},
        {"norm_conv.w", &b->norm_conv.g, d}, {"norm_conv.b", &b->norm_conv.b, d},
        {"pw1.b", &b->pw1.b, 2 * cc},
        {"dw.w", &b->dw_w, (size_t)c->conv_kernel * cc}, {"dw.b", &b->dw_b, cc},
        {"pw2.b", &b->pw2.b, d},
        {"norm_out.w", &b->norm_out.g, d}, {"norm_out.b", &b->norm_out.b, d},
    };
    for (size_t t = 0; t < sizeof table / sizeof table[0]; t++)
        if (!strcmp(rest, table[t].n)) {
            *len = table[t].len;
            return table[t].v;
        }
    return NULL;
}

static int set_matrix(oracle_granite *g, const char *name, size_t n, size_t k, const int8_t *values,
                      const float *scales, int q8)
{
    size_t en, ek;
    mat *m = find_mat(g, name, &en, &ek);
    if (!m || en != n || ek != k || (q8 && k % 32)) return -1;
    size_t panels = (n + 15) / 16, nscales = panels * 16 * (q8 ? k / 32 : 1);
    free_mat(m);
    m->v = (int8_t *)malloc(panels * 16 * k);
    m->s = (float *)malloc(nscales * sizeof(float));
    memcpy(m->v, values, panels * 16 * k);
    memcpy(m->s, scales, nscales * sizeof(float));
    m->n = n;
    m->k = k;
    m->q8 = q8;
    return 0;
}

int oracle_granite_set_matrix(oracle_granite *g, const char *name, size_t n, size_t k,
                              const int8_t *values, const float *scales)
{
    return set_matrix(g, name, n, k, values, scales, 0);
}

int oracle_granite_set_matrix_q8_0(oracle_granite *g, const char *name, size_t n, size_t k,
                                   const int8_t *values, const float *scales)
{
    return set_matrix(g, name, n, k, values, scales, 1);
}

int oracle_granite_set_vector(oracle_granite *g, const char *name, size_t len, const float *data)
{
    size_t elen;
    vec *v = find_vec(g, name, &elen);
    if (!v || elen != len) return -1;
    free(v->p);
    v->p = (float *)malloc(len * sizeof(float));
    memcpy(v->p, data, len * sizeof(float));
    v->len = len;
    return 0;
}

int oracle_granite_missing(const oracle_granite *g, char *first, size_t cap)
{
    int missing = 0;
#define CHECK(ptr, label)                                                                       \
    do {                                                                                        \
        if (!(ptr)) {                                                                           \
            if (!missing && first && cap) snprintf(first, cap, "%s", label);                    \
            missing++;                                                                          \
        }                                                                                       \
    } while (0)
    CHECK(g->input.w.v, "input"); CHECK(g->input.b.p, "input.b");
    CHECK(g->head.w.v, "head"); CHECK(g->head.b.p, "head.b");
    CHECK(g->mid.w.v, "mid"); CHECK(g->mid.b.p, "mid.b");
    for (int i = 0; i < g->c.layers; i++) {
        const block *b = &g->blocks[i];
        char label[64];
        snprintf(label, sizeof label, "blocks.%d", i);
        CHECK(b->ff1.norm.g.p && b->ff1.norm.b.p && b->ff1.up.w.v && b->ff1.up.b.p &&
                  b->ff1.down.w.v && b->ff1.down.b.p, label);
        CHECK(b->ff2.norm.g.p && b->ff2.norm.b.p && b->ff2.up.w.v && b->ff2.up.b.p &&
                  b->ff2.down.w.v && b->ff2.down.b.p, label);
        CHECK(b->norm_att.g.p && b->norm_att.b.p && b->qkv.v && b->rel.v && b->out.w.v &&
                  b->out.b.p, label);
        CHECK(b->norm_conv.g.p && b->norm_conv.b.p && b->pw1.w.v && b->pw1.b.p && b->dw_w.p &&
                  b->dw_b.p && b->pw2.w.v && b->pw2.b.p && b->norm_out.g.p && b->norm_out.b.p,
              label);
    }
#undef CHECK
    return missing;
}

size_t oracle_granite_frames_for(const oracle_granite *g, size_t rows)
{
    /* Config::frames_for (src/granite.rs:155-158). */
    for (int s = 0; s < g->c.n_subsample; s++) rows /= 2;
    return rows;
}

/* ---- the encoder ---------------------------------------------------------------------------- */

static void linear(const float *a, size_t m, const lin *l, float *c, int act, float scale,
                   int accumulate, int threads)
{
    mat_linear(a, l->w.k, m, &l->w, c, l->w.n, l->b.p, act, scale, accumulate, threads);
}

/* Row-wise work split into chunks of rows across threads, as for_rows does
 * (src/kernels/mod.rs:770-789); rows are independent, so results do not depend on threads. */
typedef struct {
    void (*row)(void *ctx, size_t r);
    void *ctx;
    size_t rows, chunk;
} rows_job;

static void rows_task(void *p, size_t t)
{
    const rows_job *J = (const rows_job *)p;
    size_t end = (t + 1) * J->chunk < J->rows ? (t + 1) * J->chunk : J->rows;
    for (size_t r = t * J->chunk; r < end; r++) J->row(J->ctx, r);
}

static void for_rows(size_t rows, size_t chunk, int threads, void (*row)(void *, size_t),
                     void *ctx)
{
    rows_job J = {row, ctx, rows, chunk};
    oracle_parallel_for((rows + chunk - 1) / chunk, threads, rows_task, &J);
}

typedef struct {
    const norm *nm;
    const float *x;
    float *out;
    size_t d;
} ln_ctx;

static void ln_row(void *p, size_t r)
{
    const ln_ctx *C = (const ln_ctx *)p;
    oracle_layer_norm(C->x + r * C->d, C->out + r * C->d, C->nm->g.p, C->nm->b.p, C->d, 1e-5f);
}

static int g_threads = 1; /* row-kernel threads of the current encode call */

static void layer_norm_rows(const norm *nm, const float *x, float *out, size_t t, size_t d)
{
    /* Granite::norm (src/granite.rs:735-749), eps 1e-5. */
    ln_ctx C = {nm, x, out, d};
    for_rows(t, 16, g_threads, ln_row, &C);
}

typedef struct {
    const float *big;
    float *glu, *dst;
    size_t cc, m, stride, kernel;
    const float *w, *bias;
    size_t vocab;
} conv_ctx;

static void glu_row(void *p, size_t r)
{
    const conv_ctx *C = (const conv_ctx *)p;
    oracle_glu(C->big + r * 2 * C->cc, C->big + r * 2 * C->cc + C->cc, C->glu + r * C->cc, C->cc);
}

static void softmax_row(void *p, size_t r)
{
    const conv_ctx *C = (const conv_ctx *)p;
    oracle_softmax(C->dst + r * C->vocab, C->vocab);
}

typedef struct {
    float *h, *big, *att, *glu;
} scratch;

/* Granite::feed_forward (src/granite.rs:752-793): x += 0.5 * down(SiLU(up(LN(x)) + b)) + ... */
static void feed_forward(const oracle_granite *g, const ffm *f, float *x, size_t t, scratch *s,
                         int threads)
{
    size_t d = (size_t)g->c.d_model;
    layer_norm_rows(&f->norm, x, s->h, t, d);
    linear(s->h, t, &f->up, s->big, ORACLE_ACT_SILU, 1.0f, 0, threads);
    linear(s->big, t, &f->down, x, ORACLE_ACT_NONE, 0.5f, 1, threads);
}

typedef struct {
    const oracle_granite *g;
    const block *b;
    const float *qkv;
    size_t t, blocks;
    float *att;
} att_job;

/* One (head, block) task of Granite::attention (src/granite.rs:965-1036). */
static void attention_task(void *ctx, size_t task)
{
    const att_job *J = (const att_job *)ctx;
    const oracle_granite_config *c = &J->g->c;
    size_t d = (size_t)c->d_model, hd = (size_t)c->head_dim, ctxn = (size_t)c->context;
    size_t positions = 2 * ctxn - 1;
    float scale = (float)pow((double)hd, -0.5);
    size_t h = task / J->blocks, blk = task % J->blocks;
    size_t i0 = blk * ctxn, len = J->t - i0 < ctxn ? J->t - i0 : ctxn;
    const float *q = J->qkv + i0 * 3 * d + h * hd;
    size_t ld = (len + 15) / 16 * 16;
    float *kt = (float *)calloc(hd * ld, sizeof(float));
    for (size_t j = 0; j < len; j++) {
        const float *key = J->qkv + (i0 + j) * 3 * d + d + h * hd;
        for (size_t i = 0; i < hd; i++) kt[i * ld + j] = key[i];
    }
    float *scores = (float *)malloc(len * len * sizeof(float));
    oracle_matmul_rowmajor(q, 3 * d, len, kt, hd, len, ld, scores, len, NULL, ORACLE_ACT_NONE,
                           scale, 0);
    float *pos = (float *)malloc(len * positions * sizeof(float));
    mat_linear(q, 3 * d, len, &J->b->rel, pos, positions, NULL, ORACLE_ACT_NONE, scale, 0, 1);
    for (size_t i = 0; i < len; i++) {
        float *row = scores + i * len;
        const float *p = pos + i * positions + ctxn - 1 - i;
        for (size_t j = 0; j < len; j++) row[j] += p[j];
        oracle_softmax(row, len);
    }
    oracle_matmul_rowmajor(scores, len, len, J->qkv + i0 * 3 * d + 2 * d + h * hd, len, hd,
                           3 * d, J->att + i0 * d + h * hd, d, NULL, ORACLE_ACT_NONE, 1.0f, 0);
    free(kt);
    free(scores);
    free(pos);
}

/* Granite::block_span (src/granite.rs:795-952): one block over input frames start..end, whose
 * input x ([end - start, d]) ends up holding their post-attention states, writing outputs from
 * out_start on (end / 2 of them in all for a strided block, end otherwise) to out. left holds the
 * post-attention states of frames lo..start, lo = conv_context(b, out_start), which the
 * convolution reads at the left edge. start begins an attention block. */
static size_t conv_context(const oracle_granite *g, const block *b, size_t out_start)
{
    /* Granite::conv_context (src/granite.rs:955-960). */
    size_t half = (size_t)g->c.conv_kernel / 2;
    size_t first = b->strided ? 2 * out_start : out_start;
    return first > half ? first - half : 0;
}

typedef struct {
    const float *glu;
    float *dst;
    size_t cc, m, stride, kernel, out_start, lo;
    const float *w, *bias;
} span_conv;

static void span_dwconv_row(void *p, size_t r)
{
    const span_conv *C = (const span_conv *)p;
    oracle_dwconv1d_frame(C->glu, C->cc, C->m, C->stride * (C->out_start + r) - C->lo, C->w, C->kernel,
                          C->bias, C->dst + r * C->cc);
    oracle_silu(C->dst + r * C->cc, C->cc);
}

static void block_span(const oracle_granite *g, const block *b, float *x, size_t start, size_t end,
                       const float *left, size_t out_start, float *out, scratch *s, int threads)
{
    const oracle_granite_config *c = &g->c;
    size_t d = (size_t)c->d_model, cc = (size_t)c->conv_channels, t = end - start;
    feed_forward(g, &b->ff1, x, t, s, threads);
    layer_norm_rows(&b->norm_att, x, s->h, t, d);
    mat_linear(s->h, d, t, &b->qkv, s->big, 3 * d, NULL, ORACLE_ACT_NONE, 1.0f, 0, threads);
    att_job J = {g, b, s->big, t, (t + (size_t)c->context - 1) / (size_t)c->context, s->att};
    oracle_parallel_for((size_t)c->heads * J.blocks, threads, attention_task, &J);
    linear(s->att, t, &b->out, x, ORACLE_ACT_NONE, 1.0f, 1, threads);
    /* The convolution module (src/granite.rs:853-944) over the post-attention states of lo..end:
     * left's rows, then x's. */
    size_t lo = conv_context(g, b, out_start), m = end - lo;
    size_t stride = b->strided ? 2 : 1, out_end = b->strided ? end / 2 : end, n = out_end - out_start;
#define STATE(f) ((f) < start ? left + ((f) - lo) * d : x + ((f) - start) * d)
    float *states = (float *)malloc((m ? m : 1) * d * sizeof(float));
    for (size_t f = lo; f < end; f++) memcpy(states + (f - lo) * d, STATE(f), d * sizeof(float));
    layer_norm_rows(&b->norm_conv, states, s->h, m, d);
    linear(s->h, m, &b->pw1, s->big, ORACLE_ACT_NONE, 1.0f, 0, threads);
    conv_ctx G = {s->big, s->glu, NULL, cc, m, 1, 0, NULL, NULL, 0};
    for_rows(m, 16, threads, glu_row, &G);
    span_conv C = {s->glu, s->big, cc, m, stride, (size_t)c->conv_kernel, out_start, lo, b->dw_w.p, b->dw_b.p};
    for_rows(n, 8, threads, span_dwconv_row, &C);
    for (size_t r = 0; r < n; r++) {
        float *row = out + r * d;
        size_t f = stride * (out_start + r);
        if (b->strided) {
            const float *p = STATE(f), *q = STATE(f + 1);
            for (size_t i = 0; i < d; i++) row[i] = (p[i] + q[i]) / 2.0f;
        } else
            memcpy(row, STATE(f), d * sizeof(float));
    }
#undef STATE
    free(states);
    linear(s->big, n, &b->pw2, out, ORACLE_ACT_NONE, 1.0f, 1, threads);
    feed_forward(g, &b->ff2, out, n, s, threads);
    layer_norm_rows(&b->norm_out, out, s->h, n, d);
    memcpy(out, s->h, n * d * sizeof(float));
}

/* Granite::self_conditioning (src/granite.rs:1040-1069). */
static void self_conditioning(const oracle_granite *g, const float *x, size_t t, float *inj,
                              int threads)
{
    size_t vocab = (size_t)g->c.vocab;
    float *logits = (float *)malloc((t ? t : 1) * vocab * sizeof(float));
    linear(x, t, &g->head, logits, ORACLE_ACT_NONE, 1.0f, 0, threads);
    conv_ctx C = {NULL, NULL, logits, 0, 0, 0, 0, NULL, NULL, vocab};
    for_rows(t, 4, threads, softmax_row, &C);
    linear(logits, t, &g->mid, inj, ORACLE_ACT_NONE, 1.0f, 0, threads);
    free(logits);
}

long oracle_granite_encode(const oracle_granite *g, const float *features, size_t rows,
                           float *out, int tap_layer, int threads)
{
    /* Granite::encode (src/granite.rs:609-654). */
    const oracle_granite_config *c = &g->c;
    if (oracle_granite_missing(g, NULL, 0)) return -1;
    if (oracle_granite_frames_for(g, rows) == 0) return -1;
    g_threads = threads < 1 ? 1 : threads;
    size_t d = (size_t)c->d_model, cc = (size_t)c->conv_channels;
    size_t widest = (size_t)c->ff;
    if (3 * d > widest) widest = 3 * d;
    if (2 * cc > widest) widest = 2 * cc;
    scratch s;
    s.h = (float *)malloc(rows * d * sizeof(float));
    s.big = (float *)malloc(rows * widest * sizeof(float));
    s.att = (float *)malloc(rows * d * sizeof(float));
    s.glu = (float *)malloc(rows * cc * sizeof(float));
    float *x = (float *)malloc(rows * d * sizeof(float));
    float *y = (float *)malloc(rows * d * sizeof(float));
    linear(features, rows, &g->input, x, ORACLE_ACT_NONE, 1.0f, 0, threads);
    size_t t = rows;
    int sc_layer = c->layers / 2 - 1;
    for (int i = 0; i < c->layers; i++) {
        const block *b = &g->blocks[i];
        size_t out_t = b->strided ? t / 2 : t;
        block_span(g, b, x, 0, t, NULL, 0, y, &s, threads);
        float *tmp = x;
        x = y;
        y = tmp;
        t = out_t;
        if (i == sc_layer) {
            self_conditioning(g, x, t, s.att, threads);
            for (size_t e = 0; e < t * d; e++) x[e] += s.att[e];
        }
        if (i == tap_layer) break;
    }
    memcpy(out, x, t * d * sizeof(float));
    free(s.h);
    free(s.big);
    free(s.att);
    free(s.glu);
    free(x);
    free(y);
    return (long)t;
}

void oracle_granite_logits(const oracle_granite *g, const float *encoded, size_t frames,
                           float *logits, int threads)
{
    linear(encoded, frames, &g->head, logits, ORACLE_ACT_NONE, 1.0f, 0, threads);
}

void oracle_granite_frame_ids(const oracle_granite *g, const float *encoded, size_t frames,
                              uint32_t *ids, float *margin, int threads)
{
    /* frame_scores + argmax, the first largest value (src/granite.rs:690-716, :1139-1147). */
    size_t vocab = (size_t)g->c.vocab;
    float *logits = (float *)malloc((frames ? frames : 1) * vocab * sizeof(float));
    oracle_granite_logits(g, encoded, frames, logits, threads);
    for (size_t f = 0; f < frames; f++) {
        const float *row = logits + f * vocab;
        size_t best = 0;
        for (size_t v = 0; v < vocab; v++)
            if (row[v] > row[best]) best = v;
        float second = -INFINITY;
        for (size_t v = 0; v < vocab; v++)
            if (v != best && row[v] > second) second = row[v];
        ids[f] = (uint32_t)best;
        if (margin) margin[f] = row[best] - second;
    }
    free(logits);
}

/* ---- GraniteStream (src/granite_stream.rs) ----------------------------------------------------- */

typedef struct {
    float *states; /* post-attention states at the layer's input rate, [frames, d] */
    size_t states_rows;
    float *out; /* outputs at its output rate, the self-conditioning injection added */
    size_t out_rows;
} layer_cache;

struct oracle_granite_stream {
    const oracle_granite *g;
    float *samples;
    size_t n, cap;
    float *logs; /* log10 mel energies of every frame computed, before the floor */
    size_t log_frames;
    float peak, floor_peak;
    int finished;
    size_t rows;
    float *features, *input;
    layer_cache *layers;
    size_t frozen, lag;
    uint32_t *ids;
    size_t n_ids, first_changed;
};

static void *grow(void *p, size_t bytes) { return realloc(p, bytes ? bytes : 1); }

oracle_granite_stream *oracle_granite_stream_new(const oracle_granite *g)
{
    oracle_granite_stream *st = (oracle_granite_stream *)calloc(1, sizeof *st);
    st->g = g;
    st->peak = -INFINITY;
    st->floor_peak = -INFINITY;
    st->lag = 16; /* DEFAULT_FREEZE_LAG (src/granite_stream.rs:23) */
    st->layers = (layer_cache *)calloc((size_t)g->c.layers, sizeof(layer_cache));
    return st;
}

void oracle_granite_stream_free(oracle_granite_stream *st)
{
    if (!st) return;
    for (int i = 0; i < st->g->c.layers; i++) {
        free(st->layers[i].states);
        free(st->layers[i].out);
    }
    free(st->layers);
    free(st->samples);
    free(st->logs);
    free(st->features);
    free(st->input);
    free(st->ids);
    free(st);
}

void oracle_granite_stream_set_freeze_lag(oracle_granite_stream *st, size_t frames) { st->lag = frames; }

int oracle_granite_stream_push(oracle_granite_stream *st, const float *samples, size_t n)
{
    if (st->finished) return -1;
    if (st->n + n > st->cap) {
        st->cap = (st->n + n) * 2;
        st->samples = (float *)grow(st->samples, st->cap * sizeof(float));
    }
    memcpy(st->samples + st->n, samples, n * sizeof(float));
    st->n += n;
    return 0;
}

/* GraniteStream::update (src/granite_stream.rs:209-361). */
int oracle_granite_stream_update(oracle_granite_stream *st, int finished, int threads)
{
    const oracle_granite *g = st->g;
    const oracle_granite_config *c = &g->c;
    if (st->finished) return -1;
    g_threads = threads < 1 ? 1 : threads;
    size_t d = (size_t)c->d_model, ctx = (size_t)c->context, n_mels = (size_t)c->n_mels;
    size_t half = (size_t)c->conv_kernel / 2, width = 4 * n_mels, n = st->n;
    st->first_changed = st->n_ids;
    size_t frames, len;
    if (!finished) {
        frames = n <= 256 ? 0 : (n - 256) / 160 + 1; /* complete_frames (src/granite_features.rs:84-92) */
        len = n;
    } else if (n >= 2 * 160) {
        frames = 2 * oracle_granite_rows_for(n);
        len = (frames - 1) * 160 + 1;
        if (len < n) len = n;
    } else {
        frames = st->log_frames;
        len = n;
    }
    st->finished = finished;
    if (frames > st->log_frames) {
        st->logs = (float *)grow(st->logs, frames * n_mels * sizeof(float));
        oracle_granite_log_frames(st->samples, n, len, st->log_frames, frames, n_mels,
                                  st->logs + st->log_frames * n_mels);
        for (size_t i = st->log_frames * n_mels; i < frames * n_mels; i++) st->peak = fmaxf(st->peak, st->logs[i]);
        st->log_frames = frames;
    }
    /* A row needs the frame after it for its last delta, until the end repeats the last frame. */
    size_t rows = finished ? frames / 2 : (frames ? (frames - 1) / 2 : 0);
    if (rows <= st->rows) return 0;

    size_t first_row = st->rows / ctx * ctx;
    if (st->peak > st->floor_peak) {
        size_t row = st->frozen;
        for (int k = 0; k < c->n_subsample; k++) row = (2 * row > half ? 2 * row - half : 0) / ctx * ctx;
        if (row < first_row) first_row = row;
        st->floor_peak = st->peak;
    }
    st->features = (float *)grow(st->features, rows * width * sizeof(float));
    oracle_granite_stack_rows(st->logs, st->log_frames, n_mels, st->peak, first_row, rows,
                              st->features + first_row * width);
    st->input = (float *)grow(st->input, rows * d * sizeof(float));
    linear(st->features + first_row * width, rows - first_row, &g->input, st->input + first_row * d,
           ORACLE_ACT_NONE, 1.0f, 0, threads);
    st->rows = rows;

    size_t widest = (size_t)c->ff;
    if (3 * d > widest) widest = 3 * d;
    if (2 * (size_t)c->conv_channels > widest) widest = 2 * (size_t)c->conv_channels;
    scratch s;
    s.h = (float *)malloc(rows * d * sizeof(float));
    s.big = (float *)malloc(rows * widest * sizeof(float));
    s.att = (float *)malloc(rows * d * sizeof(float));
    s.glu = (float *)malloc(rows * (size_t)c->conv_channels * sizeof(float));
    size_t changed = first_row, frames_in = rows;
    int sc_layer = c->layers / 2 - 1, done = 1;
    for (int i = 0; i < c->layers; i++) {
        const block *b = &g->blocks[i];
        layer_cache *L = &st->layers[i];
        size_t start, out_start, frames_out;
        if (b->strided) {
            start = changed / ctx * ctx;
            /* Outputs before start / 2 whose convolution reaches the changed block. */
            out_start = ((start > half ? start - half : 0) + 1) / 2;
            frames_out = frames_in / 2;
        } else {
            start = out_start = st->frozen;
            frames_out = frames_in;
        }
        if (start >= frames_in || out_start >= frames_out) { /* too little audio for an output */
            done = 0;
            break;
        }
        size_t lo = conv_context(g, b, out_start);
        const float *input = i == 0 ? st->input : st->layers[i - 1].out;
        float *x = (float *)malloc((frames_in - start) * d * sizeof(float));
        memcpy(x, input + start * d, (frames_in - start) * d * sizeof(float));
        float *out = (float *)calloc((frames_out - out_start) * d, sizeof(float));
        block_span(g, b, x, start, frames_in, L->states + lo * d, out_start, out, &s, threads);
        if (i == sc_layer) {
            size_t rows_out = frames_out - out_start;
            float *inj = (float *)malloc(rows_out * d * sizeof(float));
            self_conditioning(g, out, rows_out, inj, threads);
            for (size_t e = 0; e < rows_out * d; e++) out[e] += inj[e];
            free(inj);
        }
        L->states = (float *)grow(L->states, frames_in * d * sizeof(float));
        memcpy(L->states + start * d, x, (frames_in - start) * d * sizeof(float));
        L->states_rows = frames_in;
        L->out = (float *)grow(L->out, frames_out * d * sizeof(float));
        memcpy(L->out + out_start * d, out, (frames_out - out_start) * d * sizeof(float));
        L->out_rows = frames_out;
        free(x);
        free(out);
        changed = out_start;
        frames_in = frames_out;
    }
    free(s.h);
    free(s.big);
    free(s.att);
    free(s.glu);
    if (!done) return 0;

    size_t first = changed;
    st->ids = (uint32_t *)grow(st->ids, frames_in * sizeof(uint32_t));
    oracle_granite_frame_ids(g, st->layers[c->layers - 1].out + first * d, frames_in - first, st->ids + first,
                             NULL, threads);
    st->n_ids = frames_in;
    st->first_changed = first;
    if (frames_in > st->lag) {
        size_t fz = (frames_in - 1 - st->lag) / ctx * ctx;
        if (fz > st->frozen) st->frozen = fz;
    }
    return 0;
}

size_t oracle_granite_stream_frames(const oracle_granite_stream *st) { return st->n_ids; }
size_t oracle_granite_stream_first_changed(const oracle_granite_stream *st) { return st->first_changed; }
size_t oracle_granite_stream_frozen(const oracle_granite_stream *st) { return st->frozen; }
size_t oracle_granite_stream_rows(const oracle_granite_stream *st) { return st->rows; }

void oracle_granite_stream_frame_ids(const oracle_granite_stream *st, uint32_t *out)
{
    memcpy(out, st->ids, st->n_ids * sizeof(uint32_t));
}

size_t oracle_granite_stream_layer_output(const oracle_granite_stream *st, int layer, float *out)
{
    const layer_cache *L = &st->layers[layer];
    if (out) memcpy(out, L->out, L->out_rows * (size_t)st->g->c.d_model * sizeof(float));
    return L->out_rows;
}

size_t oracle_granite_stream_features(const oracle_granite_stream *st, float *out)
{
    if (out) memcpy(out, st->features, st->rows * 4 * (size_t)st->g->c.n_mels * sizeof(float));
    return st->rows;
}
