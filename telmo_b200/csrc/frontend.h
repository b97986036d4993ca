// frontend.h -- the batched log-mel front ends (see frontend.cu).
#pragma once

#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

namespace telmo {

struct Ctx;

// Per-utterance layout of a batch on the device.
struct FrontMeta {
    int n_utt;
    const int* frame_first;     // first global frame of each utterance
    const int* frame_count;
    const int64_t* sample_first;
    const int64_t* sample_count;
    const int64_t* padded_len;  // Granite: the zero-padded length the reflection uses
};

// Sparse mel filters on the device: filter m covers bins first[m] .. first[m] + count[m].
struct MelTable {
    int n_mels = 0;
    const int* first = nullptr;
    const int* count = nullptr;
    const int* offset = nullptr;
    const float* weights = nullptr;
};

struct HostMel {
    std::vector<int> first, count, offset;
    std::vector<float> weights;
};

void htk_mel_filters(int n_mels, HostMel& mel);
void slaney_mel_filters(int n_mels, HostMel& mel);

struct FrontEnd {
    enum Kind { kGranite, kParakeet };
    Ctx* ctx = nullptr;
    Kind kind = kGranite;
    int n_mels = 80;
    void* tables = nullptr;
    void* mel_dev = nullptr;
    MelTable mel;
    void* meta_dev = nullptr;
    size_t meta_cap = 0;
    void* scratch = nullptr;
    size_t scratch_cap = 0;
    int total_frames = 0;
    int64_t total_samples = 0;
    long launches = 0;

    ~FrontEnd();
    int init(Ctx* c, Kind k);
    int plan(const int64_t* lengths, int n_utt, std::vector<int>& out_rows);
    // samples_dev: every utterance's samples one after another; features: [sum rows, width].
    int run(const float* samples_dev, const int64_t* lengths, int n_utt, float* features, int* rows_out,
            cudaStream_t s);
    // The Granite front end over part of one utterance, as a stream runs it: the log10 frames
    // f0..f1 of its n samples zero-padded to len into logs + f0 * n_mels and their maximum into
    // *new_peak; rows first..last of `frames` frames floored 8 below *peak into features + first
    // * 4 * n_mels. meta_dev: 192 bytes of device memory the calls stage their layout in.
    int granite_stream_frames(const float* samples, int64_t n, int64_t len, int f0, int f1, float* logs,
                              float* new_peak, void* meta_dev, cudaStream_t s);
    int granite_stream_rows(const float* logs, int frames, const float* peak, int first, int last, float* features,
                            void* meta_dev, cudaStream_t s);
    int stream_meta(const void* host_meta, void* meta_dev, FrontMeta& meta, const int*& row_first, cudaStream_t s);
};

}  // namespace telmo
