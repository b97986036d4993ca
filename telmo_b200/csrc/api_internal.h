// api_internal.h -- the structures behind the C ABI's opaque handles.
#pragma once

#include <functional>
#include <string>

#include "kernels.h"

#include <cstdarg>
#include <string>

struct telmo_ctx;
struct telmo_pack;

namespace telmo {

struct FrontEnd;

// Pinned host staging for the small host-to-device uploads a call makes (task lists, batch
// layouts): the copy runs asynchronously from page-locked memory, so the host need not wait for
// the stream before its source vector goes out of scope. A slot is reused only after the event
// recorded behind its last copy has completed; with several slots the host can run a few
// batches ahead of the device.
struct PinnedRing {
    static constexpr int kSlots = 8;
    struct Slot {
        void* buf = nullptr;
        size_t cap = 0;
        cudaEvent_t done = nullptr;
    } slot[kSlots];
    int next = 0;

    // Copies `bytes` from host `src` to device `dst` in stream order on `s`.
    cudaError_t upload(void* dst, const void* src, size_t bytes, cudaStream_t s);
    ~PinnedRing();
};

struct Ctx {
    FrontEnd* granite_fe = nullptr;   // created on first use
    FrontEnd* parakeet_fe = nullptr;
    int device = 0;
    int sms = 148;
    uint32_t* error_word = nullptr;  // device error word the kernels record into
    void* ws = nullptr;              // growable workspace for telmo_linear's quantized operand
    size_t ws_bytes = 0;
    PinnedRing uploads;              // the calls' small host-to-device uploads
    std::string last_error;

    int fail(int code, const char* fmt, ...);
    int cuda(cudaError_t e, const char* what);
    int use_device();
    void* workspace(size_t bytes, cudaStream_t stream);
};

struct Weights {
    Ctx* ctx = nullptr;
    DevWeights dev;
};

inline Ctx* as_ctx(telmo_ctx* c) { return reinterpret_cast<Ctx*>(c); }

void encode_int8_panels(const float* rows, size_t n, size_t k, int8_t* values, float* scales);
void encode_q8_0_panels(const float* rows, size_t n, size_t k, int8_t* values, float* scales);
// col_perm (or null): column i of the uploaded matrix is the pack's column col_perm[i].
int upload_weights(Ctx* ctx, int precision, size_t n, size_t k, const void* panel_values,
                   const float* scales, DevWeights* out, const int* col_perm = nullptr);
void free_weights(DevWeights* w);

// Uploads a pack's matrix and f32 entries whose names `knows` accepts (pack.cu).
using PackMatrixFn = std::function<int(const char*, int, size_t, size_t, const void*, const float*)>;
using PackVectorFn = std::function<int(const char*, size_t, const float*)>;
using PackKnowsFn = std::function<bool(const std::string&)>;
int pack_load_entries(const telmo_pack* pk, const PackMatrixFn& set_matrix, const PackVectorFn& set_vector,
                      const PackKnowsFn& knows);

}  // namespace telmo
