// parakeet_kernels.h -- launchers of the Parakeet-specific kernels (internal to libtelmo_b200).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace telmo {

// One span of a stride-2 3x3 convolution over one utterance: output rows (time steps)
// [t2_first, t2_first + t2_count) of the utterance whose input starts at row feat_row and has
// t0 time steps; output time step r goes to out_row + (r - t2_first) * out_freqs.
struct SubTask {
    int feat_row, t0, t2_first, t2_count, out_row;
};

// Query rows [q_first, q_first + 32) (64 for the tensor-core kernel) of one utterance of len
// frames whose rows start at row and whose projected positions start at row pos_row of the
// position projection.
struct TxlTask {
    int row, len, q_first, pos_row;
};

// Greedy TDT decoding state of one utterance: encoder rows enc_first .. + frames - 1, the next
// frame t, tokens emitted on t so far, where its tokens go and how many it has emitted.
struct TdtState {
    int enc_first, frames, t, on_frame, tok_first, count;
};

// Output time steps of the first convolutions per sub_front task, and channels per CTA.
constexpr int kSubRows = 4;
constexpr int kSubCh = 16;

// Fused conv0 (1 -> ch, ReLU) + depthwise conv1 over features [rows, f0]; out [t2 * f2, ch]
// per task, every task spanning at most kSubRows output time steps.
size_t sub_front_smem(int f0);
cudaError_t sub_front(const float* feats, int f0, const SubTask* tasks, int n_tasks, int ch, const float* w0,
                      const float* b0, const float* w1, const float* b1, float* out, cudaStream_t s);

// Depthwise 3x3 stride-2 convolution: in [t0 * f_in, ch] per task (task.t0 input time steps)
// -> out [count * f_out, ch].
cudaError_t dw3x3s2(const float* in, int f_in, const SubTask* tasks, int n_tasks, int ch, const float* w,
                    const float* b, float* out, cudaStream_t s);

// The relative position table for t frames, out [2t - 1, d]; an utterance of t' <= t frames
// uses its rows t - t' .. t + t' - 2.
cudaError_t positions(int t, int d, float* out, cudaStream_t s);

// Transformer-XL relative attention (src/parakeet.rs:1176-1282) of every task and head: qkv
// [rows, 3 d] f32, pp the projected positions [*, d], att [rows, d]. hd is 32, 64 or 128.
size_t txl_attention_smem(int hd, int max_t);
cudaError_t txl_attention(const float* qkv, const float* pp, const TxlTask* tasks, int n_tasks, int heads, int hd,
                          int max_t, const float* bias_u, const float* bias_v, float scale, float* att,
                          cudaStream_t s);

// The same on the tensor cores (txl_attention_mma.cu), for head sizes 64 and 128, over tasks of
// 64 query rows: qkv [rows, 3d] and the projected positions pos [npos, d] as fp16 high/low planes
// (low plane `plane` / `pplane` elements after the high one), and cpos [heads, npos] from
// txl_pos_bias.
bool txl_attention_mma_supported(int hd);
cudaError_t txl_attention_mma(const __half* qkv, int64_t plane, const __half* pos, int64_t pplane, const float* cpos,
                              int npos, const TxlTask* tasks, int n_tasks, int heads, int hd, const float* bias_u,
                              float scale, float* att, cudaStream_t s);
// cpos[h][p] = (bias_v - bias_u) . pos[p] over head h's columns, pos as fp16 planes.
cudaError_t txl_pos_bias(const __half* pos, int64_t pplane, int npos, int heads, int hd, const float* bias_u,
                         const float* bias_v, float* cpos, cudaStream_t s);

// One greedy TDT pass is joint_prep -> joint product -> decide_prep -> LSTM product ->
// cell_prep per layer (the last followed by the pred_proj product). Each prep kernel runs one
// CTA per utterance and leaves the next product's split-int8 operand rows in q; state is
// [n_utt, layers, 2, h] (hidden, cell); predict_token[u] is the token that utterance feeds the
// prediction network this pass, or -1.

// Start of decoding: predict_token[u] = blank and q row u = [emb(blank) | 0] for every utterance.
cudaError_t tdt_start(int n_utt, int blank, int h, const float* embedding, int* predict_token, const QuantAct& q,
                      cudaStream_t s);
// pred[u] = fresh[u] where predict_token[u] >= 0; then q row u = relu(enc_proj[u's current frame]
// + pred[u]) (zeros for finished utterances); *active = 0.
cudaError_t tdt_joint_prep(const float* enc_proj, const TdtState* st, int n_utt, int h, const int* predict_token,
                           const float* fresh, float* pred, const QuantAct& q, int* active, cudaStream_t s);
// Token and duration choice from logits [n_utt, ld] and the state step after it; tokens are
// (id, frame, duration) triples; *active counts the utterances with frames left afterwards.
// For an utterance that emitted a token, q row u = [emb(token) | h_0].
cudaError_t tdt_decide_prep(const float* logits, int64_t ld, int vocab, int blank, const int* durations, int n_dur,
                            int max_symbols, TdtState* st, int n_utt, uint32_t* tokens, int* predict_token, int* active,
                            const float* embedding, const float* state, int h, int layers, const QuantAct& q,
                            cudaStream_t s);
// The cell update of `layer` from gates [n_utt, 4h] (i, f, g, o) for the predicting utterances,
// then q row u = [h_layer | h_(layer+1)], or h_top after the top layer.
cudaError_t lstm_cell_prep(const int* predict_token, int n_utt, int h, int layer, int layers, const float* gates,
                           float* state, const QuantAct& q, cudaStream_t s);
// Tokens from each utterance's worst-case slot (3 * tok_first words into raw) to consecutive
// places in out (prefix sums of the counts, kept in offsets [n_utt]); counts[u] and *total.
cudaError_t tdt_compact(const uint32_t* raw, const TdtState* st, int n_utt, int* offsets, uint32_t* out, int* counts,
                        int* total, cudaStream_t s);

}  // namespace telmo
