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

/* Uploads a weight matrix in the reference's panel layout -- PackedWeights::from_parts
 * (src/kernels/mod.rs:214-237) over a pack's bytes (src/pack.rs:280-304) -- and lays it out for
 * the tensor cores. Only TELMO_PRECISION_INT8 runs in this build. */
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
 * values) becomes scale[r] * (hi + lo / 254), hi = round(a / scale) as quantize_row_int8
 * (src/quant.rs:190-198) with scale = amax / 127, lo = round((a - hi * scale) * 254 / scale).
 * hi and lo are device int8 [m, ldq], ldq >= k and a multiple of 16; columns k..ldq are zeroed. */
int telmo_quantize_x2(telmo_ctx *ctx, const float *a, size_t lda, size_t m, size_t k, int8_t *hi,
                      int8_t *lo, size_t ldq, float *scale, void *stream);

/* telmo_linear on activations that telmo_quantize_x2 already split. */
int telmo_linear_q(telmo_ctx *ctx, const int8_t *hi, const int8_t *lo, size_t ldq,
                   const float *row_scale, size_t m, const telmo_weights *w, const float *bias,
                   int act, float scale, int accumulate, void *c, int c_dtype, size_t ldc,
                   void *stream);

#ifdef __cplusplus
}
#endif
#endif
