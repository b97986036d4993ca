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

static void dwconv_row(void *p, size_t r)
{
    const conv_ctx *C = (const conv_ctx *)p;
    oracle_dwconv1d_frame(C->glu, C->cc, C->m, C->stride * r, C->w, C->kernel, C->bias,
                          C->dst + r * C->cc);
    oracle_silu(C->dst + r * C->cc, C->cc);
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

/* Granite::block_span over a whole utterance (start 0, no left context, src/granite.rs:802-952).
 * x holds t input frames and ends up holding the post-attention states; out gets the outputs. */
static void block_span(const oracle_granite *g, const block *b, float *x, size_t t, float *out,
                       scratch *s, int threads)
{
    const oracle_granite_config *c = &g->c;
    size_t d = (size_t)c->d_model, cc = (size_t)c->conv_channels;
    feed_forward(g, &b->ff1, x, t, s, threads);
    layer_norm_rows(&b->norm_att, x, s->h, t, d);
    mat_linear(s->h, d, t, &b->qkv, s->big, 3 * d, NULL, ORACLE_ACT_NONE, 1.0f, 0, threads);
    att_job J = {g, b, s->big, t, (t + (size_t)c->context - 1) / (size_t)c->context, s->att};
    oracle_parallel_for((size_t)c->heads * J.blocks, threads, attention_task, &J);
    linear(s->att, t, &b->out, x, ORACLE_ACT_NONE, 1.0f, 1, threads);
    /* The convolution module (src/granite.rs:853-944), lo = 0 and m = t. */
    size_t m = t, stride = b->strided ? 2 : 1, n = b->strided ? t / 2 : t;
    layer_norm_rows(&b->norm_conv, x, s->h, m, d);
    linear(s->h, m, &b->pw1, s->big, ORACLE_ACT_NONE, 1.0f, 0, threads);
    conv_ctx C = {s->big, s->glu, s->big, cc, m, stride, (size_t)c->conv_kernel, b->dw_w.p,
                  b->dw_b.p, 0};
    for_rows(m, 16, threads, glu_row, &C);
    /* Every output row reads only glu, and rows below n of big are free after the GLU. */
    for_rows(n, 8, threads, dwconv_row, &C);
    for (size_t r = 0; r < n; r++) {
        float *row = out + r * d;
        if (b->strided) {
            const float *p = x + 2 * r * d, *q = x + (2 * r + 1) * d;
            for (size_t i = 0; i < d; i++) row[i] = (p[i] + q[i]) / 2.0f;
        } else
            memcpy(row, x + r * d, d * sizeof(float));
    }
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
        block_span(g, b, x, t, y, &s, threads);
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
