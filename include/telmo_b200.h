/*
 * telmo_b200.h -- C ABI of the B200-native telmo hot path (libtelmo_b200.so).
 *
 * Plain C types only: device buffers are passed as pointers to device memory (any allocator),
 * host buffers as pointers to host memory, streams as the cudaStream_t value cast to void*
 * (NULL = the legacy default stream). Every entry point returns TELMO_OK (0) or a negative
 * status; telmo_last_error() gives the message. Argument errors are the checks the reference
 * makes with assert!/panics (e.g. src/kernels/mod.rs:672-677) and its Error::Model returns
 * (src/error.rs:5-24); nothing here aborts the process.
 *
 * One telmo_ctx per GPU. Calls on one context must not run concurrently (the caller serialises
 * them; streams are per call). Weights and models are bound to the context that made them.
 */
#ifndef TELMO_B200_H
#define TELMO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define TELMO_OK 0
#define TELMO_ERR_ARGUMENT (-1)       /* a contract violation: bad shape, null pointer, size */
#define TELMO_ERR_CUDA (-2)           /* a CUDA runtime error */
#define TELMO_ERR_DEVICE_TIMEOUT (-3) /* a kernel's bounded wait gave up (see telmo_ctx_check) */
#define TELMO_ERR_UNSUPPORTED (-4)    /* a precision or mode this build does not run */
#define TELMO_ERR_MODEL (-5)          /* model problems: too-short audio, incomplete weights */

/* Weight precisions, as telmo's Precision (src/quant.rs:22-30). */
#define TELMO_PRECISION_F32 0
#define TELMO_PRECISION_F16 1
#define TELMO_PRECISION_BF16 2
#define TELMO_PRECISION_INT8 3
#define TELMO_PRECISION_Q8_0 4

/* Epilogue activations, as telmo's Act (src/kernels/mod.rs:366-373). */
#define TELMO_ACT_NONE 0
#define TELMO_ACT_RELU 1
#define TELMO_ACT_SILU 2

/* Output element types of telmo_linear. TELMO_DTYPE_I32_PAIR writes the two exact int32 sums of
 * the split-int8 product instead of the scaled result: plane 0 (rows 0..m-1, ldc apart) holds
 * the high level's sums and plane 1 (starting m * ldc elements later) the low level's. */
#define TELMO_DTYPE_F32 0
#define TELMO_DTYPE_BF16 1
#define TELMO_DTYPE_I32_PAIR 2

typedef struct telmo_ctx telmo_ctx;
typedef struct telmo_weights telmo_weights;

/* ---- context ------------------------------------------------------------------------------- */

/* Creates a context on CUDA device `device`. Replaces the reference's Kernels::new(Isa)
 * (src/kernels/mod.rs:493) and its thread Pool (src/threads.rs:103): work runs on CUDA streams. */
int telmo_ctx_create(int device, telmo_ctx **out);
void telmo_ctx_destroy(telmo_ctx *ctx);
/* The message of the last failed call on this context (or of the last failed telmo_ctx_create
 * on this thread when ctx is NULL). Valid until the next call on the context. */
const char *telmo_last_error(const telmo_ctx *ctx);
/* Waits for `stream`, then reads and clears the context's device error word. Returns
 * TELMO_ERR_DEVICE_TIMEOUT when a kernel gave up on a bounded wait since the last check. */
int telmo_ctx_check(telmo_ctx *ctx, void *stream);
/* The device the context runs on. */
int telmo_ctx_device(const telmo_ctx *ctx);

/* ---- weights ------------------------------------------------------------------------------- */

/* quant::encode for Precision::Int8 (src/quant.rs:202-269), on the host: a row-major f32
 * [n, k] matrix becomes 16-output panels (ceil(n/16) * 16 * k int8 values) and
 * ceil(n/16) * 16 f32 scales, one per output row, amax / 127 (src/quant.rs:190-198). */
int telmo_encode_int8(const float *rows, size_t n, size_t k, int8_t *panel_values, float *scales);
/* quant::encode for Precision::Q8_0 (src/quant.rs:202-269, quantize_q8_0_block :172-183): k a
 * multiple of 32; the same panels of int8 values and ceil(n/16) * (k/32) * 16 f32 scales (f16
 * values), panel, then block, then output. */
int telmo_encode_q8_0(const float *rows, size_t n, size_t k, int8_t *panel_values, float *scales);

/* Uploads a weight matrix in the reference's panel layout -- PackedWeights::from_parts
 * (src/kernels/mod.rs:214-237) over a pack's bytes (src/pack.rs:280-304) -- and lays it out for
 * the tensor cores. TELMO_PRECISION_INT8 (one scale per output) and TELMO_PRECISION_Q8_0 (one
 * scale per 32 inputs of each output, k a multiple of 32) run in this build; a Q8_0 row is
 * re-encoded as two int8 levels under one row scale, within 1/64516 of the row's largest
 * weight of the pack's exact values. */
int telmo_weights_upload(telmo_ctx *ctx, int precision, size_t n, size_t k,
                         const void *panel_values, const float *scales, telmo_weights **out);
void telmo_weights_free(telmo_weights *w);
int telmo_weights_shape(const telmo_weights *w, size_t *n, size_t *k);

/* ---- the matrix product -------------------------------------------------------------------- */

/* Kernels::linear / Kernels::matmul with packed int8 weights (src/kernels/mod.rs:657-701):
 * c[m, n] = (accumulate ? c : 0) + scale * act(a[m, k] . w^T + bias), with the Epilogue of
 * src/kernels/mod.rs:375-398. a is f32 [m, lda] and c [m, ldc] of c_dtype, both device memory;
 * bias is a device f32 [n] or NULL. Activations are quantized to two int8 levels per element
 * (see telmo_quantize_x2) into the context's workspace, then multiplied on the tensor cores. */
int telmo_linear(telmo_ctx *ctx, const float *a, size_t lda, size_t m, const telmo_weights *w,
                 const float *bias, int act, float scale, int accumulate, void *c, int c_dtype,
                 size_t ldc, void *stream);

/* The activation quantization telmo_linear applies, exposed for checking: row r of a (k
 * values) becomes scale[r] * (hi + lo / 254): scale = amax / 127 as quantize_row_int8
 * (src/quant.rs:190-198) sets a weight row's, hi = a / scale and lo = (a - hi * scale) * 254 /
 * scale, each rounded to the nearest integer (halves to even).
 * hi and lo are device int8 [m, ldq], ldq >= k and a multiple of 16; columns k..ldq are zeroed. */
int telmo_quantize_x2(telmo_ctx *ctx, const float *a, size_t lda, size_t m, size_t k, int8_t *hi,
                      int8_t *lo, size_t ldq, float *scale, void *stream);

/* telmo_linear without any device allocation. It has no counterpart in the reference: telmo's
 * CPU matmul never allocates device memory, but telmo_linear grows a workspace with cudaMalloc,
 * which some callers cannot allow -- a service that gives all device memory to its own pool or
 * fixed budget up front, or a latency-critical stream that cannot take the device-wide
 * synchronisation that cudaMalloc and cudaFree imply. Here the quantized activations go to a
 * fixed 8 MiB scratch array compiled into the library (every GPU that loads the library holds
 * it until the process exits): both levels (m * round_up(k, 16) bytes each) and m f32 scales,
 * each rounded up to 256 bytes, must fit -- up to 4088 rows at k = 1024, 1023 at k = 4096;
 * larger products are TELMO_ERR_ARGUMENT (use telmo_linear). Arguments,
 * results and errors are otherwise those of telmo_linear. The first call on each device looks
 * up the array's device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture. All calls in the process share the one array: calls whose work may overlap
 * on the GPU (different streams, or different host threads) race and must be serialised by the
 * caller. */
int telmo_linear_noalloc(telmo_ctx *ctx, const float *a, size_t lda, size_t m,
                         const telmo_weights *w, const float *bias, int act, float scale,
                         int accumulate, void *c, int c_dtype, size_t ldc, void *stream);

/* The conformer convolution module's row kernels over one utterance, the reference's Kernels
 * entries glu, dwconv1d_frame and silu (src/kernels/mod.rs:462-470; scalar arithmetic at
 * src/kernels/scalar.rs:149-187): row f of `in` (device f32 [frames, 2 * channels], the
 * pointwise product's output) gives g_f = a / (1 + e^-b) over its halves a | b; output frame r
 * is SiLU(bias + sum_j w[j] * g_{stride * r + j - kernel / 2}) (taps w device f32
 * [kernel, channels], frames outside the utterance skipped), written to out (device f32
 * [out frames, channels]) for r < frames (stride 1) or frames / 2 (stride 2). The tap sum is
 * the reference's (from the bias, taps in order, each product rounded); the exponentials and
 * divisions are the fast ones, a few ulp from expf and IEEE division. The task list goes
 * through the context's workspace, as telmo_linear's operand does. */
int telmo_conv_module_rows(telmo_ctx *ctx, const float *in, size_t frames, size_t channels,
                           size_t kernel, size_t stride, const float *w, const float *bias,
                           float *out, void *stream);

/* telmo_linear on activations that telmo_quantize_x2 already split. */
int telmo_linear_q(telmo_ctx *ctx, const int8_t *hi, const int8_t *lo, size_t ldq,
                   const float *row_scale, size_t m, const telmo_weights *w, const float *bias,
                   int act, float scale, int accumulate, void *c, int c_dtype, size_t ldc,
                   void *stream);

/* ---- log-mel front ends ---------------------------------------------------------------------- */

#define TELMO_FRONTEND_GRANITE 0  /* GraniteFrontEnd (src/granite_features.rs): 320-wide rows */
#define TELMO_FRONTEND_PARAKEET 1 /* FrontEnd with FrontEndConfig::parakeet (src/features.rs) */

/* Rows of features for an utterance of `samples` samples at 16 kHz: Granite's rows_for
 * (src/granite_features.rs:66-69), Parakeet's frames_for (src/features.rs:94-98); 0 when the
 * audio is too short. */
size_t telmo_logmel_rows(int kind, int64_t samples);

/* GraniteFrontEnd::compute (src/granite_features.rs:161-186) or FrontEnd::compute
 * (src/features.rs:101-117) for a batch: samples holds every utterance's 16 kHz samples one
 * after another (device f32), lengths (host) their counts; features (device f32) receives every
 * utterance's rows one after another ([rows, 320] for Granite, [rows, 128] for Parakeet), rows
 * (host) their counts. Too-short audio is TELMO_ERR_MODEL, as in the reference. */
int telmo_logmel(telmo_ctx *ctx, int kind, const float *samples, const int64_t *lengths, int n_utt,
                 float *features, int *rows, void *stream);

/* ---- the Granite Speech CTC encoder --------------------------------------------------------- */

/* The architecture, as Granite's Config (src/granite.rs:37-164): config.json's sizes. */
typedef struct telmo_granite_config {
    int d_model, heads, head_dim, layers, ff, conv_kernel, conv_channels, n_mels, context,
        max_relative;
    int n_subsample;          /* entries used in subsample_layers */
    int subsample_layers[8];  /* the blocks that halve the frame rate, increasing */
    int vocab, blank;
} telmo_granite_config;

typedef struct telmo_granite telmo_granite;

/* A model shell on the context, checked as Config::from_json checks a config
 * (src/granite.rs:132-146). Its weights come next, entry by entry. */
int telmo_granite_create(telmo_ctx *ctx, const telmo_granite_config *config, telmo_granite **out);
void telmo_granite_free(telmo_granite *g);
/* Pack entries by their names in a telmo pack (src/granite.rs:224-371, read back by
 * Granite::from_pack, :424-500): matrices "input", "head", "mid", "blocks.<i>.{ff1.up, ff1.down,
 * ff2.up, ff2.down, qkv, rel, out, pw1, pw2}" in the panel layout of telmo_weights_upload, and
 * f32 vectors "input.b", "head.b", "mid.b", "blocks.<i>.{ff1.norm.w, ff1.norm.b, ff1.up.b,
 * ff1.down.b, ff2..., norm_att.w/.b, out.b, norm_conv.w/.b, pw1.b, dw.w, dw.b, pw2.b,
 * norm_out.w/.b}". A wrong name or size is TELMO_ERR_MODEL. */
int telmo_granite_set_matrix(telmo_granite *g, const char *name, int precision, size_t n, size_t k,
                             const void *panel_values, const float *scales);
int telmo_granite_set_vector(telmo_granite *g, const char *name, size_t len, const float *data);
/* Checks that every entry is present (Granite::from_pack's lookups). */
int telmo_granite_finalize(telmo_granite *g);
/* Config::frames_for (src/granite.rs:155-158): encoder frames for `rows` feature rows. */
size_t telmo_granite_frames_for(const telmo_granite *g, size_t rows);

/* Granite::encode (src/granite.rs:609-654) over a batch: features holds every utterance's rows
 * [rows[u], 4 * n_mels] one after the other (device f32); out receives every utterance's
 * frames [frames[u], d_model] one after the other (device f32, sized for the sum of
 * telmo_granite_frames_for(rows[u])). rows is a host array; frames (host) receives the counts.
 * tap_layer >= 0 stops after that block and returns its output (the reference's `tap`); -1 runs
 * the whole encoder. An utterance with too few rows is TELMO_ERR_MODEL, as in the reference. */
int telmo_granite_encode(telmo_granite *g, const float *features, const int *rows, int n_utt,
                         float *out, int *frames, int tap_layer, void *stream);
/* Granite::ctc_logits (src/granite.rs:657-673): logits [frames, ld] of encoder output. */
int telmo_granite_logits(telmo_granite *g, const float *encoded, size_t frames, float *logits,
                         size_t ld, void *stream);
/* Granite::frame_ids (src/granite.rs:677-716): each frame's most likely token, the first where
 * several tie (argmax, :1139-1147), into device ids; margin (device, may be NULL) receives the
 * gap between the best and the second-best logit. */
int telmo_granite_frame_ids(telmo_granite *g, const float *encoded, size_t frames, uint32_t *ids,
                            float *margin, void *stream);

/* Encoder frames for an utterance of `samples` 16 kHz samples (front end rows, then
 * frames_for). */
size_t telmo_granite_frames_for_samples(const telmo_granite *g, int64_t samples);

/* Model::transcribe / Granite::transcribe (src/model.rs:154-159, src/granite.rs:553-582) for a
 * batch, up to the token ids (no biasing, no detokenising): front end, encoder, CTC head argmax
 * and collapse. samples: every utterance's 16 kHz samples one after another, HOST memory
 * (pinned memory copies fastest); lengths (host) their counts. frames (host, n_utt) receives
 * each utterance's encoder frame count F[u]; tokens (host) receives utterance u's tokens as
 * (id, frame, duration) triples starting at element 3 * (F[0] + ... + F[u-1]) -- size it for
 * 3 * sum of telmo_granite_frames_for_samples(lengths[u]) -- and counts (host, n_utt) their
 * numbers. The utterances run in groups of consecutive utterances with at most the transcribe
 * group's audio (2048 s unless set below; ceil(total / group) groups of about equal audio, an
 * utterance longer than a group alone in its own): while one group is transcribed on `stream`,
 * the next group's samples go up on the model's own copy stream (staged through pinned memory
 * when `samples` is pageable); the tokens and counts of all groups stay on the device and come
 * back in one copy after the last group. Returns once the tokens, counts and frames are in host
 * memory. */
int telmo_granite_transcribe(telmo_granite *g, const float *samples, const int64_t *lengths,
                             int n_utt, uint32_t *tokens, int *counts, int *frames, void *stream);
/* The audio per group of telmo_granite_transcribe, in seconds (at least 0.02). */
int telmo_granite_set_transcribe_group(telmo_granite *g, double seconds);
/* The same with samples, tokens and counts in device memory (lengths and frames on the host);
 * returns once the work is queued on `stream` (frames is filled on the host right away). */
int telmo_granite_transcribe_device(telmo_granite *g, const float *samples,
                                    const int64_t *lengths, int n_utt, uint32_t *tokens,
                                    int *counts, int *frames, void *stream);
/* CUDA kernels this model has launched so far (front end included). */
long telmo_granite_launches(const telmo_granite *g);

/* Per-kernel timing, the reference's Timings (src/parakeet.rs:151-200) for the GPU: while
 * enabled, every matrix product, attention launch and front-end pass is bracketed by CUDA events
 * on its stream. telmo_granite_profile_read waits for them and returns, per class (0 matrix
 * products, 1 attention, 2 row kernels, 3 front end), the summed milliseconds and launch counts,
 * and the matrix products' algorithmic operations (2 m n k) and bytes; then it starts over. */
int telmo_granite_profile(telmo_granite *g, int enable);
int telmo_granite_profile_read(telmo_granite *g, double *ms, long *launches, double *gemm_ops,
                               double *gemm_bytes);

/* ---- streaming (GraniteStream, src/granite_stream.rs) ----------------------------------------- */

/* One utterance transcribed while it is spoken: push appends 16 kHz samples (host), update
 * encodes what the new audio can change -- the strided blocks over their attention blocks with
 * new or changed frames, the others from the first frame of their current attention block (the
 * frozen frame; earlier outputs stay as they were once the next block has freeze_lag frames) --
 * and refreshes the frame ids from the first frame it may have changed. With finished the audio
 * is complete and its end is padded as the offline front end pads it; a single finished update
 * over a whole utterance gives exactly what telmo_granite_encode and telmo_granite_frame_ids
 * give. The model's strided blocks must come first and it must read 80 mels. A stream uses its
 * model's work buffers: one stream or batch call of a model at a time. */
typedef struct telmo_granite_stream telmo_granite_stream;
int telmo_granite_stream_create(telmo_granite *g, telmo_granite_stream **out);
void telmo_granite_stream_free(telmo_granite_stream *st);
/* Encoder frames (80 ms) the next block must have before the one before it freezes (16). */
int telmo_granite_stream_set_freeze_lag(telmo_granite_stream *st, int frames);
int telmo_granite_stream_push(telmo_granite_stream *st, const float *samples, size_t n);
int telmo_granite_stream_update(telmo_granite_stream *st, int finished, void *stream);
/* Encoder frames so far, the first frame the last update may have changed, the frozen frame. */
size_t telmo_granite_stream_frames(const telmo_granite_stream *st);
size_t telmo_granite_stream_first_changed(const telmo_granite_stream *st);
size_t telmo_granite_stream_frozen(const telmo_granite_stream *st);
/* The frame ids so far (host, up to cap), the CTC blank included. */
int telmo_granite_stream_frame_ids(const telmo_granite_stream *st, uint32_t *ids, size_t cap);
/* Block `layer`'s outputs so far ([rows, d_model], host, up to cap_rows) and the feature rows so
 * far ([rows, 320], host), for comparing with an offline pass. */
int telmo_granite_stream_layer_output(const telmo_granite_stream *st, int layer, float *out,
                                      size_t cap_rows, size_t *rows);
int telmo_granite_stream_features(const telmo_granite_stream *st, float *out, size_t cap_rows,
                                  size_t *rows);

/* ctc_tokens (src/granite.rs:1074-1094) on the device for n_utt utterances: utterance u's ids
 * are ids[first[u] .. first[u] + frames[u]) (first, frames: device int arrays); its tokens go to
 * tokens + 3 * first[u] as (id, frame, duration) triples and their number to counts[u]. */
int telmo_ctc_tokens(telmo_ctx *ctx, const uint32_t *ids, const int *first, const int *frames,
                     int n_utt, uint32_t blank, uint32_t *tokens, int *counts, void *stream);

/* ---- Parakeet TDT (src/parakeet.rs) ------------------------------------------------------------ */

/* Config (src/parakeet.rs:52-68): the encoder, the prediction network and the joint. */
typedef struct {
    int d_model, heads, layers, ff, conv_kernel;
    int sub_channels;          /* channels of the subsampling convolutions */
    int n_mels;                /* feature width (128 for the Parakeet front end) */
    int pred_hidden, pred_layers;
    int vocab, blank;          /* tokens plus the blank, which is the last */
    int n_durations;           /* entries used in durations */
    int durations[8];
    int max_symbols;           /* tokens one frame may emit before decoding moves on */
} telmo_parakeet_config;

typedef struct telmo_parakeet telmo_parakeet;

/* A model shell, checked as Config::from_json checks a config (src/parakeet.rs:70-145). */
int telmo_parakeet_create(telmo_ctx *ctx, const telmo_parakeet_config *config,
                          telmo_parakeet **out);
void telmo_parakeet_free(telmo_parakeet *p);
/* Pack entries by name as Parakeet::from_pack reads them (src/parakeet.rs:691-795): matrices
 * "sub.pw1", "sub.pw2", "sub.linear" (whose columns read the last convolution channel-major,
 * c * freqs + f, as the pack stores it), "layers.<i>.{ff1_in, ff1_out, qkv, pos, out, pw1, pw2,
 * ff2_in, ff2_out}", "dec.lstm.<l>", "dec.pred_proj", "dec.enc_proj", "dec.joint"; vectors
 * "sub.{conv0,dw1,dw2}.{w,b}" (weights [9, channels], tap first), "sub.{pw1,pw2,linear}.b",
 * "layers.<i>.{norm_ff1,norm_att,norm_conv,norm_ff2,norm_out}.{w,b}", "layers.<i>.{bias_u,
 * bias_v, dw.w, dw.b}", "dec.lstm.<l>.b", "dec.embedding", "dec.{pred_proj,enc_proj,joint}.b". */
int telmo_parakeet_set_matrix(telmo_parakeet *p, const char *name, int precision, size_t n,
                              size_t k, const void *panel_values, const float *scales);
int telmo_parakeet_set_vector(telmo_parakeet *p, const char *name, size_t len, const float *data);
int telmo_parakeet_finalize(telmo_parakeet *p);
/* Encoder frames for `feature_frames` feature frames: three stride-2 convolutions,
 * n -> (n - 1) / 2 + 1 (src/parakeet.rs:909-913). */
size_t telmo_parakeet_frames_for(size_t feature_frames);
/* The same for an utterance of `samples` 16 kHz samples (Parakeet front end frames first). */
size_t telmo_parakeet_frames_for_samples(int64_t samples);

/* Parakeet::encode (src/parakeet.rs:880-902) over a batch: features holds every utterance's
 * feature frames [rows[u], n_mels] one after another (device f32); out receives every
 * utterance's encoder frames [frames[u], d_model] one after another (device). rows is a host
 * array; frames (host) receives the counts. tap_layer -2 returns the subsampling output, i >= 0
 * layer i's output, -1 the encoder's output. */
int telmo_parakeet_encode(telmo_parakeet *p, const float *features, const int *rows, int n_utt,
                          float *out, int *frames, int tap_layer, void *stream);
/* Parakeet::decode (src/parakeet.rs:1285-1296, greedy TDT decode_inner :1412-1513) for a batch
 * of encoder outputs (device, packed as telmo_parakeet_encode writes them; frames a host array).
 * tokens (device) receives (id, frame, duration) triples, utterance u's starting at element
 * 3 * (counts[0] + ... + counts[u-1]); size it for 3 * max_symbols * (sum of frames). counts
 * (device, n_utt) receives each utterance's number of tokens, *total (host) their sum. */
int telmo_parakeet_decode(telmo_parakeet *p, const float *encoded, const int *frames, int n_utt,
                          uint32_t *tokens, int *counts, long *total, void *stream);
/* Parakeet::transcribe (src/parakeet.rs:842-867) without biasing or detokenising, for a batch:
 * front end, encoder, greedy TDT decoding. samples, lengths and frames as
 * telmo_granite_transcribe takes them; tokens (host) receives the triples packed as
 * telmo_parakeet_decode packs them (size it for 3 * max_symbols * the sum of
 * telmo_parakeet_frames_for_samples(lengths[u])), counts (host) their numbers. */
int telmo_parakeet_transcribe(telmo_parakeet *p, const float *samples, const int64_t *lengths,
                              int n_utt, uint32_t *tokens, int *counts, int *frames,
                              void *stream);
/* The same with samples, tokens and counts in device memory (lengths and frames on the host). */
int telmo_parakeet_transcribe_device(telmo_parakeet *p, const float *samples,
                                     const int64_t *lengths, int n_utt, uint32_t *tokens,
                                     int *counts, int *frames, void *stream);
/* The networks the reference's biased TDT beam search reads (Networks, src/parakeet.rs:1641-1676;
 * tdt_beam::TdtNetwork, src/biasing/tdt_beam.rs:15-26), batched on the device:
 *  - telmo_parakeet_enc_proj: the joint's projection of encoder frames (device [frames, d_model]
 *    -> device out [frames, pred_hidden]), as decode_inner computes it once (:1438-1449);
 *  - telmo_parakeet_joint: TdtNetwork::joint at one frame -- out row r (device, ld_out >= vocab +
 *    n_durations floats apart) = joint(relu(enc_row + preds[r])) + b for device enc_row
 *    [pred_hidden] (a row of telmo_parakeet_enc_proj's output) and preds [rows, pred_hidden];
 *  - telmo_parakeet_predict: TdtNetwork::predict / predict_rows (:1524-1577) -- host tokens
 *    [rows], each row's device state [rows][pred_layers][2][pred_hidden] (hidden, cell) updated
 *    in place, device preds [rows, pred_hidden] written.
 * Calls on one model run in stream order; a token outside the vocabulary is TELMO_ERR_ARGUMENT. */
int telmo_parakeet_enc_proj(telmo_parakeet *p, const float *encoded, size_t frames, float *out,
                            void *stream);
int telmo_parakeet_joint(telmo_parakeet *p, const float *enc_row, const float *preds, int rows,
                         float *out, size_t ld_out, void *stream);
int telmo_parakeet_predict(telmo_parakeet *p, const int *tokens, int rows, float *states,
                           float *preds, void *stream);
/* Selects the greedy TDT decoder: 1 (the default) runs the whole loop as one persistent
 * cooperative kernel with the prediction and joint weights held in shared memory, where the
 * model fits (pred_hidden a multiple of 64, the weights within the SMs' shared memory); 0 runs
 * it as a replayed CUDA graph of per-phase launches. Both give the same tokens bit for bit.
 * Replaces the decoder choice the reference makes implicitly (it has one CPU decoder). */
int telmo_parakeet_set_decoder(telmo_parakeet *p, int persistent);
/* Which decoder the last decode ran: 1 persistent, 0 per-phase launches, -1 none yet. */
int telmo_parakeet_last_decoder(const telmo_parakeet *p);
/* A test of the persistent decoder's failure path, which has no counterpart in the reference (its
 * decoder runs on one CPU thread): in the next persistent decode, CTA `cta` does not arrive at
 * the first grid barrier, so every CTA's bounded wait there runs out after about a second, the
 * kernel returns without touching the tokens, and the decode returns TELMO_ERR_DEVICE_TIMEOUT.
 * No copy or tensor-core operation is in flight at that barrier; the context stays usable and
 * the decode after it runs normally. */
int telmo_parakeet_test_barrier_timeout(telmo_parakeet *p, int cta);
/* The persistent decoder's own clock for the last decode run with profiling on: ms[10], per
 * phase kind (start, joint, decide, LSTM products, cells, pred_proj product, prepare; each from
 * one grid barrier to the next), then CTA 0's time inside the products and, of that, waiting
 * for staged activation rows and in epilogues; and the passes it ran. */
int telmo_parakeet_decoder_profile(const telmo_parakeet *p, double *ms, long *passes);
/* CUDA kernels this model has launched so far (front end included). */
long telmo_parakeet_launches(const telmo_parakeet *p);
/* Per-class timing as telmo_granite_profile / telmo_granite_profile_read give it. */
int telmo_parakeet_profile(telmo_parakeet *p, int enable);
int telmo_parakeet_profile_read(telmo_parakeet *p, double *ms, long *launches, double *gemm_ops,
                                double *gemm_bytes);

/* ---- decoding that favours special words (src/biasing.rs, src/biasing/) -------------------- */

/* Boost (src/biasing.rs:40-150): Parakeet's bonus per token of a special word and its beam;
 * Granite's spotting bonus per token, the margin a spotted word must beat the greedy words by,
 * and the extra margin per letter a word has below five. Bonuses 0-10, margins 0-50, beam 1-16. */
typedef struct {
    float bonus;
    int beam;
    float spotting_bonus;
    float spotting_margin;
    float short_word_margin;
} telmo_boost;
/* The reference's defaults: 1.5, 4, 4.0, 2.0, 3.0. */
void telmo_boost_default(telmo_boost *b);

/* Special words ready for decoding (Compiled, src/biasing.rs:740-870), built on the host from
 * their spellings already split into the model's tokens -- this library has no tokenizer. Form i
 * is form_lengths[i] (1-32) tokens of form_tokens, in order, and form_letters[i] letters and
 * digits in its spelling (a word of fewer than five needs a larger spotting margin). A caller
 * passes each spelling Compiled::new favours (the word and its capitalized form, a spoken form's
 * capitalizations); repeated token sequences count once. boundary[t] says whether a word may end
 * just before vocabulary token t (Tokenizer::is_word_boundary: it starts a word or holds no letter
 * or digit), wordlike[t] whether it holds a letter or digit. Failures are TELMO_ERR_ARGUMENT with
 * the reason in telmo_words_last_error() (per thread). Host only. */
typedef struct telmo_words telmo_words;
int telmo_words_create(size_t vocab, const uint8_t *boundary, const uint8_t *wordlike,
                       const uint32_t *form_tokens, const size_t *form_lengths,
                       const size_t *form_letters, size_t n_forms, const telmo_boost *boost,
                       telmo_words **out);
void telmo_words_free(telmo_words *w);
const char *telmo_words_last_error(void);
/* Distinct forms, and the sorted distinct tokens of all forms (Compiled::tokens: columns 2.. of
 * the score rows); returns their number, writing up to cap. */
size_t telmo_words_forms(const telmo_words *w);
size_t telmo_words_columns(const telmo_words *w, uint32_t *tokens, size_t cap);
/* The matcher (src/biasing.rs:653-679) on a state of three words (node, covered, half; all zero
 * at the start): the state after a token and the change in bonus, and the change when the audio
 * ends. For tests and for callers that run their own search. */
int telmo_words_step(const telmo_words *w, const uint64_t *state, uint32_t token, uint64_t *next,
                     float *delta);
int telmo_words_finish(const telmo_words *w, const uint64_t *state, float *delta);

/* spot (src/biasing/spotting.rs:95-245): replaces greedy CTC tokens by special words where an
 * alignment of the word plus its bonus beats the greedy path over the same frames by the margin.
 * greedy: n_greedy (id, frame, duration) triples of frames first..; scores: score rows of every
 * frame from 0, [frames, 2 + columns] (a frame's best logit, the blank's, then the columns'). Writes
 * the tokens (triples, up to cap; *n_tokens is the number, TELMO_ERR_ARGUMENT when it exceeds cap)
 * and for each spotted word the [begin, end) pair of output tokens it holds (ranges may be NULL).
 * Host only. */
int telmo_spot(const telmo_words *w, const uint32_t *greedy, size_t n_greedy, const float *scores,
               size_t frames, size_t first, uint32_t *tokens, size_t cap, size_t *n_tokens,
               size_t *ranges, size_t ranges_cap, size_t *n_ranges);
/* Granite::decode_biased (src/granite.rs:584-604) up to the text rewrites: the CTC head and
 * greedy ids on the device, the score rows gathered there (score_row, src/biasing/spotting.rs:
 * 10-15) so only [frames, 2 + columns] floats come back, then ctc_tokens and spot on the host.
 * encoded: device [frames, d_model]; tokens: host triples, up to cap. Spoken forms, symbols and
 * fillers (text rewrites) are outside this library. Synchronizes the stream. */
int telmo_granite_decode_biased(telmo_granite *g, const float *encoded, size_t frames,
                                const telmo_words *w, uint32_t *tokens, size_t cap,
                                size_t *n_tokens, void *stream);

/* tdt_beam::beam_search (src/biasing/tdt_beam.rs:141-401) over a caller's networks
 * (tdt_beam::TdtNetwork): joint(user, frame, preds [rows, pred_width], rows, out [rows, vocab +
 * n_durations]) and predict(user, tokens [rows], rows, states [rows, state_width] updated,
 * preds [rows, pred_width] written), each returning 0 or a status that ends the search. The search
 * decodes frames start_frame..frames from the given decoder state and writes the best hypothesis's
 * tokens as triples (up to cap). Host only. */
typedef int (*telmo_tdt_joint_fn)(void *user, size_t frame, const float *preds, size_t rows, float *out);
typedef int (*telmo_tdt_predict_fn)(void *user, const int *tokens, size_t rows, float *states,
                                    float *preds);
int telmo_tdt_beam_search(int vocab, int blank, const int *durations, int n_durations, int max_symbols,
                          size_t state_width, size_t pred_width, telmo_tdt_joint_fn joint,
                          telmo_tdt_predict_fn predict, void *user, size_t frames, size_t start_frame,
                          size_t start_on_frame, const float *start_state, const float *start_pred,
                          const telmo_words *w, uint32_t *tokens, size_t cap, size_t *n_tokens);
/* Parakeet::beam_search (src/parakeet.rs:1360-1410) over this model's device networks: the
 * joint's projection of encoded frames offset.. once (device), then per search step one batched
 * joint over the hypotheses at the step's frame and one batched prediction over those that
 * emitted. encoded: device [frames, d_model], the utterance's frames from `offset`; state and pred
 * (host, pred_layers * 2 * pred_hidden and pred_hidden floats) with frame and on_frame give the
 * decoder state to continue from, or NULL for the state before any token (initial_decoder_state,
 * :1321-1335, frame 0). Token frames count from the utterance's start. With no special words the
 * search returns no tokens, as the reference's does (decode greedily instead). Synchronizes the
 * stream. */
int telmo_parakeet_beam_search(telmo_parakeet *p, const float *encoded, size_t frames, size_t offset,
                               const float *state, const float *pred, size_t frame, size_t on_frame,
                               const telmo_words *w, uint32_t *tokens, size_t cap, size_t *n_tokens,
                               void *stream);

/* ---- packs (src/pack.rs) ------------------------------------------------------------------- */

/* The reference's weight file: "TELMOPAK", format version 1, 64-byte aligned entry data, a JSON
 * index and a "TELMOIDX" trailer, checked as Pack::parse (src/pack.rs:98-259) checks it. Packs
 * are read on the host (the whole file); the error text of a failed pack call is
 * telmo_pack_last_error() (per thread). */
typedef struct telmo_pack telmo_pack;
#define TELMO_PACK_MATRIX 0
#define TELMO_PACK_F32 1
#define TELMO_PACK_BYTES 2
#define TELMO_PACK_DEVICE 3 /* this build's extension: an 8-bit matrix in the device layout */
int telmo_pack_open(const char *path, telmo_pack **out);
int telmo_pack_from_bytes(const void *data, size_t len, telmo_pack **out);
void telmo_pack_free(telmo_pack *p);
const char *telmo_pack_last_error(void);
/* The model the pack holds ("granite-speech-ctc", "parakeet-tdt"), a metadata value (or null). */
const char *telmo_pack_model(const telmo_pack *p);
const char *telmo_pack_meta(const telmo_pack *p, const char *key);
/* Entry i: its name, kind (TELMO_PACK_*), precision (matrices), n and k (matrices; for f32
 * tensors the first dimension and the rest's product) and data bytes. */
size_t telmo_pack_entry_count(const telmo_pack *p);
int telmo_pack_entry_info(const telmo_pack *p, size_t i, const char **name, int *kind, int *precision,
                          size_t *n, size_t *k, size_t *bytes);
/* A bytes entry's data (config.json, tokenizer.json), valid while the pack lives. */
int telmo_pack_bytes(const telmo_pack *p, const char *name, const void **data, size_t *len);
/* A pack whose Int8 and Q8_0 matrices are stored in the device layout (TELMO_PACK_DEVICE; no
 * counterpart in the reference, which reads its panels on the CPU): n rows of round_up(k, 16) int8
 * values with one f32 scale per row, and for Q8_0 a second level of rows (w = s (hi + lo / 254)),
 * the columns in the order the model's kernels read them. Loading such a pack copies each matrix
 * to the device as it is instead of repacking panels on the host, and gives the same model bit
 * for bit. Runs on the host (no GPU); the other entries are kept as they are. A device entry is
 * {"type": "device", "precision", "n", "k", "offset", "bytes", "scales_offset", "scales_bytes"}
 * plus "lo_offset" and "lo_bytes" for Q8_0. The reference's reader refuses these packs. */
int telmo_pack_to_device(const telmo_pack *src, telmo_pack **out);
/* Writes the pack's file to path. */
int telmo_pack_save(const telmo_pack *p, const char *path);
/* Config::from_json (src/granite.rs:60-146, src/parakeet.rs:70-141) of a model's config.json. */
int telmo_granite_config_from_json(const char *json, size_t len, telmo_granite_config *out);
int telmo_parakeet_config_from_json(const char *json, size_t len, telmo_parakeet_config *out);
/* Granite::from_pack / Parakeet::from_pack (src/granite.rs:225-231, src/parakeet.rs:691-795) onto
 * the device: the config from config.json, every entry the model knows uploaded as it is stored
 * (Int8 or Q8_0 matrices, in panels or in the device layout), the model finalized; entries it
 * does not know are ignored. */
int telmo_granite_load_pack(telmo_ctx *ctx, const telmo_pack *p, telmo_granite **out);
int telmo_parakeet_load_pack(telmo_ctx *ctx, const telmo_pack *p, telmo_parakeet **out);

#ifdef __cplusplus
}
#endif
#endif
