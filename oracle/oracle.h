/*
 * oracle.h -- CPU restatement of telmo's CPU path for the int8 encoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the parity tests, the smoke check and
 * the CPU-baseline leg of bench.py compare the CUDA path against. The product (telmo_b200) never
 * links, loads or calls it.
 *
 * Every function names the reference function it restates (paths relative to the telmo 0.5.1
 * source tree). The restatement keeps the reference's arithmetic where it matters for parity:
 * f32 sums in ascending input order with fused multiply-add (the AVX-512/AVX2 tile,
 * src/kernels/mod.rs:885-931), int8 weights widened as the correctly rounded q * scale
 * (src/kernels/scalar.rs:82-90), f64 statistics in layer norm and f64 sums in softmax
 * (src/kernels/scalar.rs:126-147), f64 FFT and mel sums in the front ends.
 *
 * Parity pins: the front ends are checked against the reference's golden feature tensors and the
 * small known-answer tests of the reference's unit tests (see tests/test_oracle_pins.py). The
 * encoder restatement has no golden tensors of its own here (they need the real checkpoints),
 * so it is pinned through its parts.
 */
#ifndef TELMO_ORACLE_H
#define TELMO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_ACT_NONE = 0, ORACLE_ACT_RELU = 1, ORACLE_ACT_SILU = 2 };

/* ---- quant.rs ---------------------------------------------------------------------------- */
/* quantize_row_int8 (src/quant.rs:190-198). Returns the scale. */
float oracle_quantize_row_int8(const float *x, size_t k, int8_t *q);
/* encode for Precision::Int8 from Rows::F32 (src/quant.rs:202-269): 16-output panels. */
void oracle_encode_int8(const float *w, size_t n, size_t k, int8_t *values, float *scales);
/* decode (src/quant.rs:272-303) for Precision::Int8. out is row-major [n, k]. */
void oracle_decode_int8(const int8_t *values, const float *scales, size_t n, size_t k, float *out);
/* encode / decode for Precision::Q8_0 (src/quant.rs:202-303, quantize_q8_0_block :172-183): k a
 * multiple of 32, scales per block of 32 inputs in panel, block, output order. */
void oracle_encode_q8_0(const float *w, size_t n, size_t k, int8_t *values, float *scales);
void oracle_decode_q8_0(const int8_t *values, const float *scales, size_t n, size_t k, float *out);
/* f32_to_bf16 / bf16_to_f32 / f32_to_f16 / f16_to_f32 (src/quant.rs:92-164). */
uint16_t oracle_f32_to_bf16(float x);
float oracle_bf16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float x);
float oracle_f16_to_f32(uint16_t h);

/* ---- kernels/mod.rs: the matrix product --------------------------------------------------- */
/* Kernels::linear / matmul over int8 PackedWeights (src/kernels/mod.rs:530-701):
 * c[m, n] = (accumulate ? c : 0) + scale * act(a . w^T + bias), sums in ascending k with FMA,
 * weights widened per panel. threads > 1 splits panels like Pool::run (mod.rs:678-687); results
 * are bit-identical for every thread count. */
void oracle_linear_int8(const float *a, size_t lda, size_t m, const int8_t *values,
                        const float *scales, size_t n, size_t k, float *c, size_t ldc,
                        const float *bias, int act, float scale, int accumulate, int threads);
/* The same product over Q8_0 panels: widen with each input's block scale
 * (src/kernels/scalar.rs:92-106, src/kernels/mod.rs:577). */
void oracle_linear_q8_0(const float *a, size_t lda, size_t m, const int8_t *values,
                        const float *scales, size_t n, size_t k, float *c, size_t ldc,
                        const float *bias, int act, float scale, int accumulate, int threads);
/* Kernels::matmul_serial with BView::row_major (src/kernels/mod.rs:324-340, :732-765):
 * b is row-major [k, ldb], its first n columns used. */
void oracle_matmul_rowmajor(const float *a, size_t lda, size_t m, const float *b, size_t k,
                            size_t n, size_t ldb, float *c, size_t ldc, const float *bias, int act,
                            float scale, int accumulate);

/* ---- the split int8 activation rule of the CUDA path (no reference counterpart) ------------
 * Each activation row x (length k) becomes s * (hi + lo / 254) with hi, lo in [-127, 127]:
 * s = amax / 127 as quantize_row_int8 (src/quant.rs:190-198) sets a weight row's, hi = x / s
 * and then lo = (x - hi * s) * 254 / s, each rounded to the nearest integer with halves to even
 * (the rounding the CUDA kernels get from one add of 1.5 * 2^23). The CUDA kernels follow the
 * same f32 steps, so hi, lo and s agree bit for bit. */
void oracle_quantize_x2(const float *x, size_t m, size_t k, size_t ldx, int8_t *hi, int8_t *lo,
                        size_t ldq, float *row_scale);
/* Exact i32 sums of the two levels against int8 weights in panels: acc_hi[m, n], acc_lo[m, n]. */
void oracle_gemm_i8_x2_acc(const int8_t *hi, const int8_t *lo, size_t ldq, size_t m,
                           const int8_t *values, size_t n, size_t k, int32_t *acc_hi,
                           int32_t *acc_lo);
/* The CUDA epilogue over those sums, step for step:
 * v = ((float)acc_hi + (float)acc_lo * (1/254)) * row_scale[i] * w_scale[j]; then bias, act,
 * scale and accumulate as Epilogue (src/kernels/mod.rs:366-398, scalar.rs:110-124). */
/* The CUDA build's re-encoding of Q8_0 panels into two int8 levels under one scale per row
 * (row-major [n, k] outputs), and its integer sums with them: acc_lo = lo . W_hi + hi . W_lo. */
void oracle_q8_0_two_level(const int8_t *values, const float *scales, size_t n, size_t k,
                           int8_t *w_hi, int8_t *w_lo, float *w_scale);
void oracle_gemm_i8_x2w_acc(const int8_t *hi, const int8_t *lo, size_t ldq, size_t m,
                            const int8_t *w_hi, const int8_t *w_lo, size_t n, size_t k,
                            int32_t *acc_hi, int32_t *acc_lo);
void oracle_epilogue_x2(const int32_t *acc_hi, const int32_t *acc_lo, size_t m, size_t n,
                        const float *row_scale, const float *w_scales, const float *bias, int act,
                        float scale, int accumulate, float *c, size_t ldc);

/* ---- kernels/scalar.rs: row kernels -------------------------------------------------------- */
void oracle_layer_norm(const float *x, float *out, const float *gamma, const float *beta,
                       size_t n, float eps);                                  /* scalar.rs:126 */
void oracle_softmax(float *x, size_t n);                                      /* scalar.rs:136 */
void oracle_glu(const float *a, const float *b, float *out, size_t n);        /* scalar.rs:149 */
void oracle_silu(float *x, size_t n);                                         /* scalar.rs:155 */
void oracle_dwconv1d_frame(const float *input, size_t channels, size_t frames, size_t t,
                           const float *w, size_t kernel, const float *bias, float *out);
void oracle_conv3x3s2_row(const float *input, size_t in_t, size_t in_f, size_t channels,
                          int depthwise, const float *w, const float *bias, size_t t,
                          float *out);                                        /* scalar.rs:194 */

/* ---- fft.rs -------------------------------------------------------------------------------- */
/* RealFft::forward (src/fft.rs:97-134): n real f64 in, n/2+1 complex out (re, im interleaved). */
int oracle_real_fft(const double *input, size_t n, double *out);

/* ---- granite_features.rs / features.rs ----------------------------------------------------- */
/* GraniteFrontEnd::rows_for (src/granite_features.rs:66-69). */
size_t oracle_granite_rows_for(size_t samples);
/* GraniteFrontEnd::compute (src/granite_features.rs:161-186): out [rows, 4 * n_mels].
 * Returns 0, or -1 when the audio is too short (fewer than 320 samples). */
int oracle_granite_features(const float *samples, size_t n, size_t n_mels, float *out);
/* The pieces of it a stream runs: log_frame (src/granite_features.rs:95-133) for frames f0..f1
 * of n samples zero-padded to len (logs[(f - f0) * n_mels]), and stack_rows (:138-158) of rows
 * first..last of frames logs with the given peak (out[(row - first) * 4 * n_mels]). */
void oracle_granite_log_frames(const float *samples, size_t n, size_t len, size_t f0, size_t f1,
                               size_t n_mels, float *logs);
void oracle_granite_stack_rows(const float *logs, size_t frames, size_t n_mels, float peak,
                               size_t first, size_t last, float *out);
/* FrontEnd::compute (src/features.rs:101-216) with FrontEndConfig::parakeet: out [n/160, 128].
 * Returns 0, or -1 when the audio is too short. */
int oracle_parakeet_features(const float *samples, size_t n, float *out);

/* ---- granite.rs ---------------------------------------------------------------------------- */
typedef struct oracle_granite oracle_granite;
typedef struct {
    int d_model, heads, head_dim, layers, ff, conv_kernel, conv_channels, n_mels, context,
        max_relative, n_subsample, subsample_layers[8], vocab, blank;
} oracle_granite_config;

oracle_granite *oracle_granite_new(const oracle_granite_config *config);
void oracle_granite_free(oracle_granite *g);
/* Pack entries by name, as Granite::from_pack reads them (src/granite.rs:424-500): matrices
 * ("input", "blocks.3.ff1.up", "blocks.3.qkv", "blocks.3.rel", "head", ...) as int8 panels
 * with their scales, and vectors ("input.b", "blocks.3.ff1.norm.w", "blocks.3.dw.w", ...).
 * The data is copied. Returns 0, or -1 for an unknown name or a wrong size. */
int oracle_granite_set_matrix(oracle_granite *g, const char *name, size_t n, size_t k,
                              const int8_t *values, const float *scales);
/* The same for a Q8_0 matrix (scales per 32 inputs, as oracle_encode_q8_0 lays them out). */
int oracle_granite_set_matrix_q8_0(oracle_granite *g, const char *name, size_t n, size_t k,
                                   const int8_t *values, const float *scales);
int oracle_granite_set_vector(oracle_granite *g, const char *name, size_t len, const float *data);
/* Names that were never set; 0 when the model is complete. */
int oracle_granite_missing(const oracle_granite *g, char *first_missing, size_t cap);
/* Config::frames_for (src/granite.rs:155-158). */
size_t oracle_granite_frames_for(const oracle_granite *g, size_t rows);
/* Granite::encode (src/granite.rs:609-654): features [rows, 4 * n_mels] -> out [frames, d].
 * tap_layer >= 0 stops after that block (its output goes to out). Returns frames, or -1. */
long oracle_granite_encode(const oracle_granite *g, const float *features, size_t rows,
                           float *out, int tap_layer, int threads);
/* Granite::frame_scores + argmax (src/granite.rs:690-716, :1139-1147): ids [frames], and the
 * top-2 margin of every frame's logits (for the "margin above 1e-2" rule). */
void oracle_granite_frame_ids(const oracle_granite *g, const float *encoded, size_t frames,
                              uint32_t *ids, float *margin, int threads);
/* Granite::ctc_logits (src/granite.rs:657-673). logits [frames, vocab]. */
void oracle_granite_logits(const oracle_granite *g, const float *encoded, size_t frames,
                           float *logits, int threads);

/* ---- parakeet.rs ----------------------------------------------------------------------------- */
typedef struct oracle_parakeet oracle_parakeet;
/* GraniteStream (src/granite_stream.rs): one utterance transcribed while it is spoken. push
 * appends 16 kHz samples; update encodes what is new (finished: the audio is complete). The
 * model's strided blocks must come first. */
typedef struct oracle_granite_stream oracle_granite_stream;
oracle_granite_stream *oracle_granite_stream_new(const oracle_granite *g);
void oracle_granite_stream_free(oracle_granite_stream *st);
void oracle_granite_stream_set_freeze_lag(oracle_granite_stream *st, size_t frames);
int oracle_granite_stream_push(oracle_granite_stream *st, const float *samples, size_t n);
int oracle_granite_stream_update(oracle_granite_stream *st, int finished, int threads);
size_t oracle_granite_stream_frames(const oracle_granite_stream *st);
size_t oracle_granite_stream_first_changed(const oracle_granite_stream *st);
size_t oracle_granite_stream_frozen(const oracle_granite_stream *st);
size_t oracle_granite_stream_rows(const oracle_granite_stream *st);
void oracle_granite_stream_frame_ids(const oracle_granite_stream *st, uint32_t *out);
size_t oracle_granite_stream_layer_output(const oracle_granite_stream *st, int layer, float *out);
size_t oracle_granite_stream_features(const oracle_granite_stream *st, float *out);

typedef struct {
    int d_model, heads, layers, ff, conv_kernel, sub_channels, n_mels, pred_hidden, pred_layers,
        vocab, blank, n_durations, durations[8], max_symbols;
} oracle_parakeet_config;

oracle_parakeet *oracle_parakeet_new(const oracle_parakeet_config *config);
void oracle_parakeet_free(oracle_parakeet *p);
/* Pack entries by name, as Parakeet::from_pack reads them (src/parakeet.rs:691-795). */
int oracle_parakeet_set_matrix(oracle_parakeet *p, const char *name, size_t n, size_t k,
                               const int8_t *values, const float *scales);
/* The same for a Q8_0 matrix (scales per 32 inputs, as oracle_encode_q8_0 lays them out). */
int oracle_parakeet_set_matrix_q8_0(oracle_parakeet *p, const char *name, size_t n, size_t k,
                                    const int8_t *values, const float *scales);
int oracle_parakeet_set_vector(oracle_parakeet *p, const char *name, size_t len, const float *data);
/* Encoder frames for a number of feature frames (three stride-2 convolutions). */
size_t oracle_parakeet_frames_for(size_t feature_frames);
/* positions (src/parakeet.rs:1618-1630): out [2t - 1, d]. */
void oracle_parakeet_positions(size_t t, size_t d, float *out);
/* Parakeet::encode (src/parakeet.rs:880-902): features [frames, n_mels] -> out [t, d].
 * tap_layer >= 0 stops after that layer, -2 after the subsampling. Returns t, or -1. */
long oracle_parakeet_encode(const oracle_parakeet *p, const float *features, size_t frames,
                            float *out, int tap_layer, int threads);
/* Greedy TDT decoding (src/parakeet.rs:1285-1296, :1412-1513): (id, frame, duration) triples,
 * at most frames * max_symbols + frames of them; min_margin gets the smallest top-2 gap of any
 * token or duration choice. Returns the token count. */
size_t oracle_parakeet_decode(const oracle_parakeet *p, const float *encoded, size_t frames,
                              uint32_t *tokens, float *min_margin, int threads);
/* As oracle_parakeet_decode; sure receives the number of tokens emitted before the first step
 * whose top-2 gap is at or below threshold (all of them when no step is). */
size_t oracle_parakeet_decode_sure(const oracle_parakeet *p, const float *encoded, size_t frames,
                                   uint32_t *tokens, float *min_margin, float threshold,
                                   size_t *sure, int threads);
/* The networks the biased beam search reads (src/parakeet.rs:1641-1676): the joint's projection
 * of encoder frames [frames, h]; the joint's outputs [rows, vocab + durations] for prediction
 * rows at one projected frame; predict_rows for one token per row, states [rows][layers][2][h]
 * updated in place, preds [rows, h]. */
void oracle_parakeet_enc_proj(const oracle_parakeet *p, const float *encoded, size_t frames,
                              float *out, int threads);
void oracle_parakeet_joint(const oracle_parakeet *p, const float *enc_row, const float *preds,
                           size_t rows, float *out);
void oracle_parakeet_predict(const oracle_parakeet *p, const int *tokens, size_t rows, float *states,
                             float *preds);
/* One step of the greedy TDT loop after the joint (src/parakeet.rs:1482-1510): the first
 * argmax over logits[0, vocab) is the token, durations[first argmax over the n_durations
 * logits after them] the duration; a blank moves *t on by max(duration, 1); a token is written
 * to token[0..2] as (id, *t, duration) and moves *t on by its duration, or for duration 0 after
 * max_symbols tokens on the frame by 1. Returns 1 when a token was emitted. */
int oracle_tdt_step(const float *logits, int vocab, int blank, const int *durations, int n_durations,
                    int max_symbols, size_t *t, int *on_frame, uint32_t *token);

/* ctc_tokens (src/granite.rs:1074-1094): writes (id, frame, duration) triples, returns count. */
size_t oracle_ctc_tokens(const uint32_t *ids, size_t frames, uint32_t blank, uint32_t *out);

#ifdef __cplusplus
}
#endif
#endif
