/*
 * parakeet.c -- oracle restatement of telmo's Parakeet TDT encoder and greedy TDT decoder.
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
} pmat;
typedef struct {
    float *p;
    size_t len;
} pvec;

typedef struct {
    pvec norm_ff1_w, norm_ff1_b, norm_att_w, norm_att_b, norm_conv_w, norm_conv_b, norm_ff2_w,
        norm_ff2_b, norm_out_w, norm_out_b, bias_u, bias_v, dw_w, dw_b;
    pmat ff1_in, ff1_out, qkv, pos, out, pw1, pw2, ff2_in, ff2_out;
} player;

struct oracle_parakeet {
    oracle_parakeet_config c;
    pvec conv0_w, conv0_b, dw1_w, dw1_b, pw1_b, dw2_w, dw2_b, pw2_b, linear_b;
    pmat pw1, pw2, linear;
    player *layers;
    pmat lstm[8];
    pvec lstm_b[8];
    pvec embedding, pred_proj_b, enc_proj_b, joint_b;
    pmat pred_proj, enc_proj, joint;
};

static size_t pp_d(const oracle_parakeet *p) { return (size_t)p->c.d_model; }

oracle_parakeet *oracle_parakeet_new(const oracle_parakeet_config *c)
{
    if (c->heads <= 0 || c->d_model % c->heads || c->n_mels % 8 || c->conv_kernel % 2 == 0 ||
        c->n_durations <= 0 || c->n_durations > 8 || c->blank + 1 != c->vocab || c->layers <= 0 ||
        c->pred_layers <= 0 || c->pred_layers > 8)
        return NULL;
    oracle_parakeet *p = (oracle_parakeet *)calloc(1, sizeof *p);
    p->c = *c;
    p->layers = (player *)calloc((size_t)c->layers, sizeof(player));
    return p;
}

static void pfree_m(pmat *m) { free(m->v); free(m->s); }

void oracle_parakeet_free(oracle_parakeet *p)
{
    if (!p) return;
    pvec *vs[] = {&p->conv0_w, &p->conv0_b, &p->dw1_w, &p->dw1_b, &p->pw1_b, &p->dw2_w,
                  &p->dw2_b, &p->pw2_b, &p->linear_b, &p->embedding, &p->pred_proj_b,
                  &p->enc_proj_b, &p->joint_b};
    for (size_t i = 0; i < sizeof vs / sizeof vs[0]; i++) free(vs[i]->p);
    pfree_m(&p->pw1); pfree_m(&p->pw2); pfree_m(&p->linear);
    pfree_m(&p->pred_proj); pfree_m(&p->enc_proj); pfree_m(&p->joint);
    for (int l = 0; l < 8; l++) { pfree_m(&p->lstm[l]); free(p->lstm_b[l].p); }
    for (int i = 0; i < p->c.layers; i++) {
        player *L = &p->layers[i];
        pvec *lv[] = {&L->norm_ff1_w, &L->norm_ff1_b, &L->norm_att_w, &L->norm_att_b,
                      &L->norm_conv_w, &L->norm_conv_b, &L->norm_ff2_w, &L->norm_ff2_b,
                      &L->norm_out_w, &L->norm_out_b, &L->bias_u, &L->bias_v, &L->dw_w, &L->dw_b};
        for (size_t j = 0; j < sizeof lv / sizeof lv[0]; j++) free(lv[j]->p);
        pmat *lm[] = {&L->ff1_in, &L->ff1_out, &L->qkv, &L->pos, &L->out, &L->pw1, &L->pw2,
                      &L->ff2_in, &L->ff2_out};
        for (size_t j = 0; j < sizeof lm / sizeof lm[0]; j++) pfree_m(lm[j]);
    }
    free(p->layers);
    free(p);
}

/* Shapes as Parakeet::from_pack asks for them (src/parakeet.rs:691-795). */
static pmat *pfind_m(oracle_parakeet *p, const char *name, size_t *n, size_t *k)
{
    const oracle_parakeet_config *c = &p->c;
    size_t d = pp_d(p), ch = (size_t)c->sub_channels, h = (size_t)c->pred_hidden;
    size_t outputs = (size_t)(c->vocab + c->n_durations);
    if (!strcmp(name, "sub.pw1")) { *n = ch; *k = ch; return &p->pw1; }
    if (!strcmp(name, "sub.pw2")) { *n = ch; *k = ch; return &p->pw2; }
    if (!strcmp(name, "sub.linear")) { *n = d; *k = ch * (size_t)(c->n_mels / 8); return &p->linear; }
    if (!strcmp(name, "dec.pred_proj")) { *n = h; *k = h; return &p->pred_proj; }
    if (!strcmp(name, "dec.enc_proj")) { *n = h; *k = d; return &p->enc_proj; }
    if (!strcmp(name, "dec.joint")) { *n = outputs; *k = h; return &p->joint; }
    int l;
    char rest[64];
    if (sscanf(name, "dec.lstm.%d%63s", &l, rest) == 1 && l >= 0 && l < c->pred_layers) {
        *n = 4 * h; *k = 2 * h; return &p->lstm[l];
    }
    int i;
    if (sscanf(name, "layers.%d.%63s", &i, rest) != 2 || i < 0 || i >= c->layers) return NULL;
    player *L = &p->layers[i];
    size_t ff = (size_t)c->ff;
    if (!strcmp(rest, "ff1_in")) { *n = ff; *k = d; return &L->ff1_in; }
    if (!strcmp(rest, "ff1_out")) { *n = d; *k = ff; return &L->ff1_out; }
    if (!strcmp(rest, "ff2_in")) { *n = ff; *k = d; return &L->ff2_in; }
    if (!strcmp(rest, "ff2_out")) { *n = d; *k = ff; return &L->ff2_out; }
    if (!strcmp(rest, "qkv")) { *n = 3 * d; *k = d; return &L->qkv; }
    if (!strcmp(rest, "pos")) { *n = d; *k = d; return &L->pos; }
    if (!strcmp(rest, "out")) { *n = d; *k = d; return &L->out; }
    if (!strcmp(rest, "pw1")) { *n = 2 * d; *k = d; return &L->pw1; }
    if (!strcmp(rest, "pw2")) { *n = d; *k = d; return &L->pw2; }
    return NULL;
}

static pvec *pfind_v(oracle_parakeet *p, const char *name, size_t *len)
{
    const oracle_parakeet_config *c = &p->c;
    size_t d = pp_d(p), ch = (size_t)c->sub_channels, h = (size_t)c->pred_hidden;
    struct { const char *n; pvec *v; size_t len; } top[] = {
        {"sub.conv0.w", &p->conv0_w, 9 * ch}, {"sub.conv0.b", &p->conv0_b, ch},
        {"sub.dw1.w", &p->dw1_w, 9 * ch}, {"sub.dw1.b", &p->dw1_b, ch},
        {"sub.pw1.b", &p->pw1_b, ch}, {"sub.dw2.w", &p->dw2_w, 9 * ch},
        {"sub.dw2.b", &p->dw2_b, ch}, {"sub.pw2.b", &p->pw2_b, ch},
        {"sub.linear.b", &p->linear_b, d}, {"dec.embedding", &p->embedding, (size_t)c->vocab * h},
        {"dec.pred_proj.b", &p->pred_proj_b, h}, {"dec.enc_proj.b", &p->enc_proj_b, h},
        {"dec.joint.b", &p->joint_b, (size_t)(c->vocab + c->n_durations)},
    };
    for (size_t t = 0; t < sizeof top / sizeof top[0]; t++)
        if (!strcmp(name, top[t].n)) { *len = top[t].len; return top[t].v; }
    int l;
    char rest[64];
    if (sscanf(name, "dec.lstm.%d%63s", &l, rest) == 2 && !strcmp(rest, ".b") && l >= 0 &&
        l < c->pred_layers) {
        *len = 4 * h;
        return &p->lstm_b[l];
    }
    int i;
    if (sscanf(name, "layers.%d.%63s", &i, rest) != 2 || i < 0 || i >= c->layers) return NULL;
    player *L = &p->layers[i];
    struct { const char *n; pvec *v; size_t len; } t2[] = {
        {"norm_ff1.w", &L->norm_ff1_w, d}, {"norm_ff1.b", &L->norm_ff1_b, d},
        {"norm_att.w", &L->norm_att_w, d}, {"norm_att.b", &L->norm_att_b, d},
        {"norm_conv.w", &L->norm_conv_w, d}, {"norm_conv.b", &L->norm_conv_b, d},
        {"norm_ff2.w", &L->norm_ff2_w, d}, {"norm_ff2.b", &L->norm_ff2_b, d},
        {"norm_out.w", &L->norm_out_w, d}, {"norm_out.b", &L->norm_out_b, d},
        {"bias_u", &L->bias_u, d}, {"bias_v", &L->bias_v, d},
        {"dw.w", &L->dw_w, (size_t)c->conv_kernel * d}, {"dw.b", &L->dw_b, d},
    };
    for (size_t t = 0; t < sizeof t2 / sizeof t2[0]; t++)
        if (!strcmp(rest, t2[t].n)) { *len = t2[t].len; return t2[t].v; }
    return NULL;
}

static int pset_matrix(oracle_parakeet *p, const char *name, size_t n, size_t k, const int8_t *values,
                       const float *scales, int q8)
{
    size_t en, ek;
    pmat *m = pfind_m(p, name, &en, &ek);
    if (!m || en != n || ek != k || (q8 && k % 32)) return -1;
    size_t panels = (n + 15) / 16, nscales = panels * 16 * (q8 ? k / 32 : 1);
    pfree_m(m);
    m->v = (int8_t *)malloc(panels * 16 * k);
    m->s = (float *)malloc(nscales * sizeof(float));
    memcpy(m->v, values, panels * 16 * k);
    memcpy(m->s, scales, nscales * sizeof(float));
    m->n = n;
    m->k = k;
    m->q8 = q8;
    return 0;
}

int oracle_parakeet_set_matrix(oracle_parakeet *p, const char *name, size_t n, size_t k,
                               const int8_t *values, const float *scales)
{
    return pset_matrix(p, name, n, k, values, scales, 0);
}

int oracle_parakeet_set_matrix_q8_0(oracle_parakeet *p, const char *name, size_t n, size_t k,
                                    const int8_t *values, const float *scales)
{
    return pset_matrix(p, name, n, k, values, scales, 1);
}

int oracle_parakeet_set_vector(oracle_parakeet *p, const char *name, size_t len, const float *data)
{
    size_t elen;
    pvec *v = pfind_v(p, name, &elen);
    if (!v || elen != len) return -1;
    free(v->p);
    v->p = (float *)malloc(len * sizeof(float));
    memcpy(v->p, data, len * sizeof(float));
    v->len = len;
    return 0;
}

static void plinear(const pmat *w, const float *a, size_t m, float *c, const float *bias, int act,
                    float scale, int accumulate, int threads)
{
    if (w->q8)
        oracle_linear_q8_0(a, w->k, m, w->v, w->s, w->n, w->k, c, w->n, bias, act, scale, accumulate,
                           threads);
    else
        oracle_linear_int8(a, w->k, m, w->v, w->s, w->n, w->k, c, w->n, bias, act, scale, accumulate,
                           threads);
}

static void pnorm(const pvec *g, const pvec *b, const float *x, float *out, size_t t, size_t d)
{
    for (size_t r = 0; r < t; r++) oracle_layer_norm(x + r * d, out + r * d, g->p, b->p, d, 1e-5f);
}

size_t oracle_parakeet_frames_for(size_t feature_frames)
{
    /* Three stride-2 convolutions: n -> (n - 1) / 2 + 1 (src/parakeet.rs:909-913). */
    size_t t = feature_frames;
    for (int i = 0; i < 3; i++) t = (t - 1) / 2 + 1;
    return t;
}

/* Parakeet::subsample (src/parakeet.rs:904-993). Returns x [t3, d]. */
static float *subsample(const oracle_parakeet *p, const float *features, size_t frames,
                        size_t *t_out, int threads)
{
    const oracle_parakeet_config *c = &p->c;
    size_t ch = (size_t)c->sub_channels, d = pp_d(p);
#define OUT(n) (((n) - 1) / 2 + 1)
    size_t t0 = frames, f0 = (size_t)c->n_mels, t1 = OUT(t0), f1 = OUT(f0), t2 = OUT(t1),
           f2 = OUT(f1), t3 = OUT(t2), f3 = OUT(f2);
#undef OUT
    float *h1 = (float *)malloc(t1 * f1 * ch * sizeof(float));
    for (size_t t = 0; t < t1; t++) {
        oracle_conv3x3s2_row(features, t0, f0, ch, 0, p->conv0_w.p, p->conv0_b.p, t,
                             h1 + t * f1 * ch);
        for (size_t i = 0; i < f1 * ch; i++) h1[t * f1 * ch + i] = fmaxf(h1[t * f1 * ch + i], 0.0f);
    }
    float *d1 = (float *)malloc(t2 * f2 * ch * sizeof(float));
    for (size_t t = 0; t < t2; t++)
        oracle_conv3x3s2_row(h1, t1, f1, ch, 1, p->dw1_w.p, p->dw1_b.p, t, d1 + t * f2 * ch);
    float *h2 = (float *)malloc(t2 * f2 * ch * sizeof(float));
    plinear(&p->pw1, d1, t2 * f2, h2, p->pw1_b.p, ORACLE_ACT_RELU, 1.0f, 0, threads);
    float *d2 = (float *)malloc(t3 * f3 * ch * sizeof(float));
    for (size_t t = 0; t < t3; t++)
        oracle_conv3x3s2_row(h2, t2, f2, ch, 1, p->dw2_w.p, p->dw2_b.p, t, d2 + t * f3 * ch);
    float *h3 = (float *)malloc(t3 * f3 * ch * sizeof(float));
    plinear(&p->pw2, d2, t3 * f3, h3, p->pw2_b.p, ORACLE_ACT_RELU, 1.0f, 0, threads);
    /* PyTorch flattens channel by channel: flat[t][c * f3 + f] = h3[t][f][c]. */
    float *flat = (float *)malloc(t3 * f3 * ch * sizeof(float));
    for (size_t t = 0; t < t3; t++)
        for (size_t f = 0; f < f3; f++)
            for (size_t cc = 0; cc < ch; cc++)
                flat[t * f3 * ch + cc * f3 + f] = h3[t * f3 * ch + f * ch + cc];
    float *x = (float *)malloc(t3 * d * sizeof(float));
    plinear(&p->linear, flat, t3, x, p->linear_b.p, ORACLE_ACT_NONE, 1.0f, 0, threads);
    free(h1); free(d1); free(h2); free(d2); free(h3); free(flat);
    *t_out = t3;
    return x;
}

/* positions (src/parakeet.rs:1618-1630): [2t - 1, d], positions t - 1 down to 1 - t. */
void oracle_parakeet_positions(size_t t, size_t d, float *out)
{
    for (size_t r = 0; r < 2 * t - 1; r++) {
        double pos = (double)t - 1.0 - (double)r;
        for (size_t i = 0; i < d / 2; i++) {
            double freq = exp(-((double)(2 * i)) * (log(10000.0) / (double)d));
            double angle = pos * freq;
            out[r * d + 2 * i] = (float)sin(angle);
            out[r * d + 2 * i + 1] = (float)cos(angle);
        }
    }
}

typedef struct {
    const oracle_parakeet *p;
    const player *L;
    const float *qkv, *pp;
    size_t t;
    float *att;
} patt_job;

/* One head of Parakeet::attention (src/parakeet.rs:1176-1282), all query rows at once (the
 * reference's 48-row blocks only split the work; every sum is per row). */
static void pattention_head(void *ctx, size_t h)
{
    const patt_job *J = (const patt_job *)ctx;
    const oracle_parakeet_config *c = &J->p->c;
    size_t d = pp_d(J->p), hd = d / (size_t)c->heads, t = J->t, npos = 2 * t - 1;
    float scale = 1.0f / sqrtf((float)hd);
    size_t ldk = (t + 15) / 16 * 16, ldp = (npos + 15) / 16 * 16;
    float *kt = (float *)calloc(hd * ldk, sizeof(float));
    float *pt = (float *)calloc(hd * ldp, sizeof(float));
    for (size_t j = 0; j < t; j++)
        for (size_t i = 0; i < hd; i++) kt[i * ldk + j] = J->qkv[j * 3 * d + d + h * hd + i];
    for (size_t j = 0; j < npos; j++)
        for (size_t i = 0; i < hd; i++) pt[i * ldp + j] = J->pp[j * d + h * hd + i];
    float *qu = (float *)malloc(t * hd * sizeof(float)), *qv = (float *)malloc(t * hd * sizeof(float));
    for (size_t r = 0; r < t; r++)
        for (size_t i = 0; i < hd; i++) {
            float q = J->qkv[r * 3 * d + h * hd + i];
            qu[r * hd + i] = q + J->L->bias_u.p[h * hd + i];
            qv[r * hd + i] = q + J->L->bias_v.p[h * hd + i];
        }
    float *scores = (float *)malloc(t * t * sizeof(float));
    oracle_matmul_rowmajor(qu, hd, t, kt, hd, t, ldk, scores, t, NULL, ORACLE_ACT_NONE, 1.0f, 0);
    float *bd = (float *)malloc(t * npos * sizeof(float));
    oracle_matmul_rowmajor(qv, hd, t, pt, hd, npos, ldp, bd, npos, NULL, ORACLE_ACT_NONE, 1.0f, 0);
    for (size_t i = 0; i < t; i++) {
        float *row = scores + i * t;
        const float *pos = bd + i * npos + (t - 1 - i);
        for (size_t j = 0; j < t; j++) row[j] = (row[j] + pos[j]) * scale;
        oracle_softmax(row, t);
    }
    oracle_matmul_rowmajor(scores, t, t, J->qkv + 2 * d + h * hd, t, hd, 3 * d, J->att + h * hd, d,
                           NULL, ORACLE_ACT_NONE, 1.0f, 0);
    free(kt); free(pt); free(qu); free(qv); free(scores); free(bd);
}

/* Parakeet::layer (src/parakeet.rs:1011-1172). */
static void player_run(const oracle_parakeet *p, const player *L, float *x, size_t t,
                       const float *pos, int threads)
{
    const oracle_parakeet_config *c = &p->c;
    size_t d = pp_d(p), ff = (size_t)c->ff, npos = 2 * t - 1;
    float *h = (float *)malloc(t * d * sizeof(float));
    size_t big_w = ff > 3 * d ? ff : 3 * d;
    float *big = (float *)malloc(t * big_w * sizeof(float));
    float *att = (float *)malloc(t * d * sizeof(float));
    float *pp = (float *)malloc(npos * d * sizeof(float));
    pnorm(&L->norm_ff1_w, &L->norm_ff1_b, x, h, t, d);
    plinear(&L->ff1_in, h, t, big, NULL, ORACLE_ACT_SILU, 1.0f, 0, threads);
    plinear(&L->ff1_out, big, t, x, NULL, ORACLE_ACT_NONE, 0.5f, 1, threads);
    pnorm(&L->norm_att_w, &L->norm_att_b, x, h, t, d);
    plinear(&L->qkv, h, t, big, NULL, ORACLE_ACT_NONE, 1.0f, 0, threads);
    plinear(&L->pos, pos, npos, pp, NULL, ORACLE_ACT_NONE, 1.0f, 0, threads);
    patt_job J = {p, L, big, pp, t, att};
    oracle_parallel_for((size_t)c->heads, threads, pattention_head, &J);
    plinear(&L->out, att, t, x, NULL, ORACLE_ACT_NONE, 1.0f, 1, threads);
    pnorm(&L->norm_conv_w, &L->norm_conv_b, x, h, t, d);
    plinear(&L->pw1, h, t, big, NULL, ORACLE_ACT_NONE, 1.0f, 0, threads);
    for (size_t r = 0; r < t; r++) oracle_glu(big + r * 2 * d, big + r * 2 * d + d, h + r * d, d);
    for (size_t r = 0; r < t; r++) {
        oracle_dwconv1d_frame(h, d, t, r, L->dw_w.p, (size_t)c->conv_kernel, L->dw_b.p, att + r * d);
        oracle_silu(att + r * d, d);
    }
    plinear(&L->pw2, att, t, x, NULL, ORACLE_ACT_NONE, 1.0f, 1, threads);
    pnorm(&L->norm_ff2_w, &L->norm_ff2_b, x, h, t, d);
    plinear(&L->ff2_in, h, t, big, NULL, ORACLE_ACT_SILU, 1.0f, 0, threads);
    plinear(&L->ff2_out, big, t, x, NULL, ORACLE_ACT_NONE, 0.5f, 1, threads);
    pnorm(&L->norm_out_w, &L->norm_out_b, x, h, t, d);
    memcpy(x, h, t * d * sizeof(float));
    free(h); free(big); free(att); free(pp);
}

long oracle_parakeet_encode(const oracle_parakeet *p, const float *features, size_t frames,
                            float *out, int tap_layer, int threads)
{
    /* Parakeet::encode (src/parakeet.rs:880-902). tap_layer -2 stops after the subsampling. */
    if (frames < 1) return -1;
    size_t t, d = pp_d(p);
    float *x = subsample(p, features, frames, &t, threads);
    if (tap_layer != -2) {
        float *pos = (float *)malloc((2 * t - 1) * d * sizeof(float));
        oracle_parakeet_positions(t, d, pos);
        for (int i = 0; i < p->c.layers; i++) {
            player_run(p, &p->layers[i], x, t, pos, threads);
            if (i == tap_layer) break;
        }
        free(pos);
    }
    memcpy(out, x, t * d * sizeof(float));
    free(x);
    return (long)t;
}

static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); } /* src/parakeet.rs:1678 */

/* Parakeet::predict_rows for one token (src/parakeet.rs:1524-1577): state [layers][2][h]
 * (hidden, cell), pred [h]. */
static void predict(const oracle_parakeet *p, size_t token, float *state, float *pred, int threads)
{
    size_t h = (size_t)p->c.pred_hidden;
    float *input = (float *)malloc(2 * h * sizeof(float));
    float *gates = (float *)malloc(4 * h * sizeof(float));
    memcpy(input, p->embedding.p + token * h, h * sizeof(float));
    for (int l = 0; l < p->c.pred_layers; l++) {
        float *hs = state + (size_t)l * 2 * h, *cs = hs + h;
        memcpy(input + h, hs, h * sizeof(float));
        plinear(&p->lstm[l], input, 1, gates, p->lstm_b[l].p, ORACLE_ACT_NONE, 1.0f, 0, threads);
        for (size_t j = 0; j < h; j++) {
            float i = sigmoidf_(gates[j]), f = sigmoidf_(gates[h + j]);
            float g = tanhf(gates[2 * h + j]), o = sigmoidf_(gates[3 * h + j]);
            cs[j] = f * cs[j] + i * g;
            hs[j] = o * tanhf(cs[j]);
        }
        memcpy(input, hs, h * sizeof(float));
    }
    plinear(&p->pred_proj, input, 1, pred, p->pred_proj_b.p, ORACLE_ACT_NONE, 1.0f, 0, threads);
    free(input);
    free(gates);
}

/* ---- the networks the biased beam search reads (src/parakeet.rs:1641-1676) ------------------ */

void oracle_parakeet_enc_proj(const oracle_parakeet *p, const float *encoded, size_t frames,
                              float *out, int threads)
{
    plinear(&p->enc_proj, encoded, frames, out, p->enc_proj_b.p, ORACLE_ACT_NONE, 1.0f, 0, threads);
}

void oracle_parakeet_joint(const oracle_parakeet *p, const float *enc_row, const float *preds,
                           size_t rows, float *out)
{
    /* TdtNetwork::joint (:1653-1670): z = relu(e + p) per row, then one product over the rows. */
    size_t h = (size_t)p->c.pred_hidden;
    float *z = (float *)malloc((rows ? rows : 1) * h * sizeof(float));
    for (size_t r = 0; r < rows; r++)
        for (size_t j = 0; j < h; j++) z[r * h + j] = fmaxf(enc_row[j] + preds[r * h + j], 0.0f);
    plinear(&p->joint, z, rows, out, p->joint_b.p, ORACLE_ACT_NONE, 1.0f, 0, 1);
    free(z);
}

void oracle_parakeet_predict(const oracle_parakeet *p, const int *tokens, size_t rows, float *states,
                             float *preds)
{
    /* TdtNetwork::predict (:1672-1675) -> predict_rows: each row's state and prediction. */
    size_t h = (size_t)p->c.pred_hidden, sw = (size_t)p->c.pred_layers * 2 * h;
    for (size_t r = 0; r < rows; r++) predict(p, (size_t)tokens[r], states + r * sw, preds + r * h, 1);
}

static size_t argmax_first(const float *v, size_t n)
{
    size_t best = 0;
    for (size_t i = 0; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

int oracle_tdt_step(const float *logits, int vocab, int blank, const int *durations, int n_durations,
                    int max_symbols, size_t *t, int *on_frame, uint32_t *token)
{
    /* One pass of decode_inner's loop after the joint (src/parakeet.rs:1482-1510). */
    size_t id = argmax_first(logits, (size_t)vocab);
    size_t duration = (size_t)durations[argmax_first(logits + vocab, (size_t)n_durations)];
    if (id == (size_t)blank) {
        *t += duration > 1 ? duration : 1;
        *on_frame = 0;
        return 0;
    }
    token[0] = (uint32_t)id;
    token[1] = (uint32_t)*t;
    token[2] = (uint32_t)duration;
    if (duration > 0) {
        *t += duration;
        *on_frame = 0;
    } else if (++*on_frame >= max_symbols) {
        *t += 1;
        *on_frame = 0;
    }
    return 1;
}

size_t oracle_parakeet_decode_sure(const oracle_parakeet *p, const float *encoded, size_t frames,
                                   uint32_t *tokens, float *min_margin, float threshold,
                                   size_t *sure, int threads)
{
    /* Parakeet::decode / decode_inner greedy TDT (src/parakeet.rs:1285-1296, :1412-1513).
     * min_margin (may be NULL) receives the smallest top-2 logit gap of any joint step's token
     * or duration choice; sure (may be NULL) the number of tokens emitted before the first step
     * whose gap is at or below threshold (every token when no step is), the prefix that any
     * decoder whose logits differ by less than the threshold must reproduce; returns the number
     * of tokens. */
    const oracle_parakeet_config *c = &p->c;
    size_t h = (size_t)c->pred_hidden, d = pp_d(p);
    size_t vocab = (size_t)c->vocab, outputs = vocab + (size_t)c->n_durations;
    float *state = (float *)calloc((size_t)c->pred_layers * 2 * h, sizeof(float));
    float *pred = (float *)calloc(h, sizeof(float));
    predict(p, (size_t)c->blank, state, pred, threads);
    float *enc_proj = (float *)malloc((frames ? frames : 1) * h * sizeof(float));
    plinear(&p->enc_proj, encoded, frames, enc_proj, p->enc_proj_b.p, ORACLE_ACT_NONE, 1.0f, 0,
            threads);
    (void)d;
    float *z = (float *)malloc(h * sizeof(float));
    float *logits = (float *)malloc(outputs * sizeof(float));
    size_t t = 0, count = 0;
    int on_frame = 0;
    float worst = INFINITY;
    int unsure = 0;
    size_t sure_count = 0;
    while (t < frames) {
        for (size_t j = 0; j < h; j++) z[j] = fmaxf(enc_proj[t * h + j] + pred[j], 0.0f);
        plinear(&p->joint, z, 1, logits, p->joint_b.p, ORACLE_ACT_NONE, 1.0f, 0, threads);
        size_t token = argmax_first(logits, vocab);
        size_t di = argmax_first(logits + vocab, (size_t)c->n_durations);
        for (size_t v = 0; v < vocab; v++)
            if (v != token) worst = fminf(worst, logits[token] - logits[v]);
        for (size_t v = 0; v < (size_t)c->n_durations; v++)
            if (v != di) worst = fminf(worst, logits[vocab + di] - logits[vocab + v]);
        if (!unsure && worst <= threshold) {
            unsure = 1;
            sure_count = count;
        }
        if (oracle_tdt_step(logits, c->vocab, c->blank, c->durations, c->n_durations,
                            c->max_symbols, &t, &on_frame, tokens + 3 * count)) {
            count++;
            predict(p, token, state, pred, threads);
        }
    }
    if (min_margin) *min_margin = worst;
    if (sure) *sure = unsure ? sure_count : count;
    free(state); free(pred); free(enc_proj); free(z); free(logits);
    return count;
}

size_t oracle_parakeet_decode(const oracle_parakeet *p, const float *encoded, size_t frames,
                              uint32_t *tokens, float *min_margin, int threads)
{
    return oracle_parakeet_decode_sure(p, encoded, frames, tokens, min_margin, 0.0f, NULL, threads);
}
