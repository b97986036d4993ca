// rowops.h -- launchers of the encoder's memory-bound kernels and the attention kernel.
#pragma once

#include "kernels.h"

#include <cuda_fp16.h>

namespace telmo {

// One span of a depthwise convolution: output frames [out_first, out_first + count) of one
// utterance whose input frames are rows in_row .. in_row + in_len - 1 (zero outside) and whose
// output frame r goes to row out_row + r. Output frame r is centred on input frame
// stride * r + shift: shift is 0 for a whole utterance and -lo for a window that starts at input
// frame lo of a stream. stride is 1, or 2 for the blocks that halve the frame rate.
struct ConvTask {
    int in_row, in_len, out_row, out_first, count, stride, shift;
};

// One attention block: rows [row, row + len) of one utterance, len <= context.
struct AttnTask {
    int row, len;
};

// y = LN_a(x) (written to y_out if not null), then z = LN_b(y) if gb is not null, then z split
// into q if q is not null. x, y_out are [m, d] f32 with d a multiple of 128 (up to 2048).
cudaError_t ln_chain(const float* x, int m, int d, const float* ga, const float* ba, float* y_out,
                     const float* gb, const float* bb, const QuantAct* q, cudaStream_t stream);

// Row softmax of x [m, n] (rows ld apart) in place, then its split-int8 quantization into q.
cudaError_t softmax_quant(float* x, int m, int n, int64_t ld, const QuantAct& q, cudaStream_t stream);

// out[row, cc] = SiLU(dw_b + sum_j dw_w[j] * GLU(big)[frame]) for every task; every task of a
// launch has the given stride (1, or 2 for the blocks that halve the frame rate).
cudaError_t glu_dwconv_silu(const float* big, int cc, int k, int stride, const ConvTask* tasks, int n_tasks,
                            const float* w, const float* bias, float* out, cudaStream_t stream);

// out[r] = (x[src_row[r]] + x[src_row[r] + 1]) / 2.
cudaError_t pool_pairs(const float* x, int d, const int* src_row, int rows, float* out, cudaStream_t stream);

// ids[r] = first argmax of row r of x [m, n]; margin[r] = top1 - top2 (margin may be null).
cudaError_t argmax_rows(const float* x, int m, int n, int64_t ld, uint32_t* ids, float* margin,
                        cudaStream_t stream);

// CTC collapse of each utterance's frame ids (frames[u] ids from ids + first[u]) into
// (id, frame, duration) triples at tokens + 3 * first[u]; counts[u] = number of tokens.
cudaError_t ctc_collapse(const uint32_t* ids, const int* first, const int* frames, int n_utt, uint32_t blank,
                         uint32_t* tokens, int* counts, cudaStream_t stream);

// Block-local attention with Shaw relative positions (src/granite.rs:965-1036) over qkv
// [rows, 3 * heads * hd] for every task and head; rel_w int8 [2 * ctx - 1, ld_rel] with one
// scale per row; att [rows, heads * hd].
cudaError_t granite_attention(const float* qkv, int heads, int hd, int ctx, const AttnTask* tasks, int n_tasks,
                              const int8_t* rel_w, int64_t ld_rel, const float* rel_scale, float scale,
                              float* att, cudaStream_t stream);

// The same on the tensor cores (attention_mma.cu), for context 128 and head sizes 64 or 128:
// qkv as fp16 high/low planes ([rows, 3 * heads * hd] each, the low one `plane` elements after
// the high one), the relative table as fp16 [2 * ctx - 1, hd] with one f32 scale per row.
bool granite_attention_mma_supported(int hd, int ctx);
cudaError_t granite_attention_mma(const __half* qkv, int64_t plane, int heads, int hd, int ctx, const AttnTask* tasks,
                                  int n_tasks, const __half* rel16, const float* rel_scale, float scale, float* att,
                                  cudaStream_t stream);

// The same on the tcgen05 tensor cores (attention_tc.cu), for context 128 and head size 128:
// the QKV product's fp16 planes of `rows` rows each (the low plane right after the high one);
// a wait that times out records kErrWaitTimeout in `error`.
bool granite_attention_tc_supported(int hd, int ctx);
cudaError_t granite_attention_tc(const __half* qkv, int rows, int heads, int hd, int ctx, const AttnTask* tasks,
                                 int n_tasks, const __half* rel16, const float* rel_scale, float scale, float* att,
                                 uint32_t* error, cudaStream_t stream);

}  // namespace telmo
