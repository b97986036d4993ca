// granite_internal.h -- the device model behind telmo_granite handles.
#pragma once

#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "kernels.h"

#include <string>
#include <vector>

namespace telmo {

struct DevVec {
    float* p = nullptr;
};
struct Lin {
    DevWeights w;
    DevVec b;
};
struct Norm {
    DevVec g, b;
};
struct FF {
    Norm norm;
    Lin up, down;
};
// One conformer block, as Granite's Block (src/granite.rs:186-206).
struct Block {
    bool strided = false;
    FF ff1, ff2;
    Norm norm_att, norm_conv, norm_out;
    DevWeights qkv, rel;
    Lin out, pw1, pw2;
    DevVec dw_w, dw_b;
};

struct Granite {
    Ctx* ctx = nullptr;
    telmo_granite_config c{};
    Lin input, head, mid;
    std::vector<Block> blocks;
    bool finalized = false;
    long launches = 0;  // kernels launched so far (for benchmark accounting)

    // Activation buffers, sized for cap_rows packed rows.
    int cap_rows = 0, tasks_cap = 0;
    float *x = nullptr, *y = nullptr, *big = nullptr, *att = nullptr, *conv = nullptr;
    QuantAct q;
    int* tasks_dev = nullptr;
    int64_t big_ld = 0, vocab_ld = 0;

    struct Entry {
        DevWeights* mat = nullptr;
        DevVec* vec = nullptr;
        int n = 0, k = 0, len = 0;
    };

    ~Granite();
    static int validate(const telmo_granite_config& c, std::string& why);
    Entry find(const std::string& name);
    std::string missing() const;
    int fail(int code, const char* msg);
    int ensure(int rows, int tasks);
    void release_buffers();
    int gemm(const QuantAct& a, int m, const Lin& l, float* out, int64_t ldc, int act, float scale, int acc,
             cudaStream_t s);
    int gemm_w(const QuantAct& a, int m, const DevWeights& w, const float* bias, float* out, int64_t ldc, int act,
               float scale, int acc, cudaStream_t s);
    int feed_forward(const FF& f, float* x, int m, cudaStream_t s);
    int encode(const float* feats, const int* rows, int n_utt, float* out, int* frames_out, int tap, cudaStream_t s);
    int logits(const float* encoded, int frames, float* out, int64_t ld, cudaStream_t s);
    int frame_ids(const float* encoded, int frames, uint32_t* ids, float* margin, cudaStream_t s);
};

}  // namespace telmo
