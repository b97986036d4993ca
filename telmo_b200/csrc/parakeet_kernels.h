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

// The same on the tcgen05 tensor cores (txl_attention_tc.cu), for head size 128, over tasks of
// 128 query rows: qkv [rows, 3d] and pos [npos, d] as fp16 high/low planes (each low plane right
// after its high one), cv [heads, npos] and uk [heads, rows] from txl_bias_terms; a wait that times
// out records kErrWaitTimeout in `error`.
bool txl_attention_tc_supported(int hd);
cudaError_t txl_attention_tc(const __half* qkv, int rows, const __half* pos, int npos, const float* cv, const float* uk,
                             const TxlTask* tasks, int n_tasks, int heads, int hd, float scale, float* att,
                             uint32_t* error, cudaStream_t s);
// cv[h][p] = bias_v . pos[p] and uk[h][r] = bias_u . k[r] over head h's columns (the scores' bias
// parts: (q + u) . k + (q + v) . pos = q . k + uk + q . pos + cv).
cudaError_t txl_bias_terms(const __half* pos, int npos, const __half* qkv, int rows, int heads, const float* bias_u,
                           const float* bias_v, float* cv, float* uk, cudaStream_t s);

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
// ---- the persistent decoder (tdt_persistent.cu) ----

constexpr int kTdtMaxMats = 10;  // joint, up to 8 LSTM layers, pred_proj
// Phase kinds of the persistent decoder's clock: start, joint, decide, LSTM products, cells,
// pred_proj product, prepare; then CTA 0's own time in the products and, of that, the time its
// thread 0 waited for staged activation rows and spent in epilogues.
constexpr int kTdtPhases = 7;
constexpr int kTdtClocks = kTdtPhases + 3;
enum TdtError : unsigned { kTdtErrBarrier = 1, kTdtErrPasses = 2 };

// One matrix of the prediction or joint network: int8 [n, ld] weights, per-row scales, bias
// (or null), k inputs. units (of 8 rows) .. smem_stride are filled in by tdt_persistent_plan.
struct TdtMatrix {
    const int8_t* w = nullptr;
    int64_t ld = 0;
    const float* ws = nullptr;
    const float* bias = nullptr;
    int n = 0, k = 0;
    int units = 0, max_units = 0, offset = 0, smem_stride = 0;
};

// Everything the persistent decoder reads and writes. Rows of q, gates and fresh are compacted
// slots; state is [n_utt, layers, 2, h]; lists holds the two live lists [2][n_utt], plist
// [n_utt] the predicting utterances by slot, ps_of [n_utt] each utterance's predicting slot or
// -1. tok_key, dur_key [n_utt] and words [8] start zeroed.
struct TdtPersistentArgs {
    TdtMatrix mats[kTdtMaxMats];  // 0 joint, 1 .. layers LSTM, layers + 1 pred_proj
    int n_mats = 0, layers = 0, h = 0, n_utt = 0;
    int vocab = 0, blank = 0, n_dur = 0, max_symbols = 0;
    int durations[8] = {};
    const float* enc_proj = nullptr;   // [frames, h]
    const float* embedding = nullptr;  // [vocab, h]
    float* state = nullptr;
    float* pred = nullptr;   // [n_utt, h]
    float* fresh = nullptr;  // [n_utt, h] by slot
    float* gates = nullptr;  // [n_utt, 4h] by slot
    int8_t* q_hi = nullptr;
    int8_t* q_lo = nullptr;
    float* q_scale = nullptr;
    int64_t q_ld = 0;
    TdtState* st = nullptr;
    uint32_t* tokens = nullptr;
    int* lists = nullptr;
    int* plist = nullptr;
    int* ps_of = nullptr;
    unsigned long long* tok_key = nullptr;
    unsigned long long* dur_key = nullptr;
    unsigned* words = nullptr;  // error code, passes, barrier state, counters
    unsigned long long* phase_ns = nullptr;  // [kTdtClocks] or null: time per phase kind
    long long max_passes = 0;
    int ring_offset = 0;  // shared memory: the weight units, then the warps' rings
    int chunk = 0;        // k bytes per ring stage: 128 where every k allows, else 64
    int withhold_cta = -1;  // a test of the timeout path: this CTA never arrives at the first grid barrier
};

// Assigns every matrix's 8-row units to `sms` CTAs and sizes the shared memory; false if the
// model does not fit (h not a multiple of 64, more than 8 units of a matrix per CTA, or more
// than 227 KB), in which case the launch-per-phase decoder is used.
bool tdt_persistent_plan(TdtPersistentArgs& a, int sms, size_t* smem_bytes);
// Runs the whole greedy decode; the error code lands in words[0], the passes in words[1].
cudaError_t tdt_persistent(const TdtPersistentArgs& a, int grid, size_t smem_bytes, cudaStream_t s);

// The networks the biased beam search reads: q row r = relu(enc_row + preds[r]) (the joint's
// operand), and q row r = [emb(tokens[r]) | h_0 of state row r] (the first LSTM layer's).
cudaError_t tdt_joint_rows(const float* enc_row, const float* preds, int rows, int h, const QuantAct& q,
                           cudaStream_t s);
cudaError_t tdt_predict_input(const int* tokens, int rows, int h, int layers, const float* embedding,
                              const float* states, const QuantAct& q, cudaStream_t s);
// Tokens from each utterance's worst-case slot (3 * tok_first words into raw) to consecutive
// places in out (prefix sums of the counts, kept in offsets [n_utt]); counts[u] and *total.
cudaError_t tdt_compact(const uint32_t* raw, const TdtState* st, int n_utt, int* offsets, uint32_t* out, int* counts,
                        int* total, cudaStream_t s);

}  // namespace telmo
