// api_internal.h -- the structures behind the C ABI's opaque handles.
#pragma once

#include <functional>
#include <string>
#include <vector>

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
// The device layout of a weight matrix: n rows of ld = round_up(k, 16) int8 values (zero past k)
// and one f32 scale per row; Q8_0 weights add a second, low level of rows (w = s (hi + lo / 254)).
// encode_device_rows turns the reference's 16-output panels into it on the host; col_perm (or
// null): column i of the result is the panel's column col_perm[i]. rows and lo hold n * ld values
// (lo only for Q8_0), sc n. check_weight_shape refuses precisions and shapes the GEMM cannot run.
void encode_device_rows(int precision, size_t n, size_t k, const void* panel_values, const float* scales,
                        const int* col_perm, int8_t* rows, int8_t* lo, float* sc);
int check_weight_shape(Ctx* ctx, int precision, size_t n, size_t k);
int upload_device_rows(Ctx* ctx, int precision, size_t n, size_t k, const int8_t* rows, const int8_t* lo,
                       const float* sc, DevWeights* out);
// encode_device_rows followed by upload_device_rows.
int upload_weights(Ctx* ctx, int precision, size_t n, size_t k, const void* panel_values,
                   const float* scales, DevWeights* out, const int* col_perm = nullptr);
void free_weights(DevWeights* w);

// Uploads a pack's matrix and f32 entries whose names `knows` accepts (pack.cu).
using PackMatrixFn = std::function<int(const char*, int, size_t, size_t, const void*, const float*)>;
using PackDeviceFn =
    std::function<int(const char*, int, size_t, size_t, const int8_t*, const int8_t*, const float*)>;
using PackVectorFn = std::function<int(const char*, size_t, const float*)>;
using PackKnowsFn = std::function<bool(const std::string&)>;
int pack_load_entries(const telmo_pack* pk, const PackMatrixFn& set_matrix, const PackDeviceFn& set_device,
                      const PackVectorFn& set_vector, const PackKnowsFn& knows);
// A matrix already in the device layout (a pack's device entry): rows and lo (Q8_0) of
// n * round_up(k, 16) values, scales of n.
int granite_set_device_matrix(telmo_granite* g, const char* name, int precision, size_t n, size_t k,
                              const int8_t* rows, const int8_t* lo, const float* scales);
int parakeet_set_device_matrix(telmo_parakeet* p, const char* name, int precision, size_t n, size_t k,
                               const int8_t* rows, const int8_t* lo, const float* scales);
// Parakeet's subsampling output matrix ("sub.linear") takes its inputs frequency-major on the
// device: column i of the device matrix is the pack's column perm[i].
std::vector<int> parakeet_linear_perm(int sub_channels, int n_mels);

}  // namespace telmo
