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
};

}  // namespace telmo
