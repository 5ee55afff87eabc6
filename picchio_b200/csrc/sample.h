// sample.h - sample_logits (picchio.c:1540-1649) on the device.
//
// One draw per single-sequence step from the step's logits row: repetition
// penalty over the history, temperature, top-k, softmax, top-p, then the
// xorshift64 draw (picchio.c:1520-1526).  The generator state and the history
// live in device memory, so CUDA-graph replays and the on-device generation
// loop sample without a host round trip.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace pc {

constexpr int SAMPLE_HIST_CAP = 4096;  // g_history (picchio.c:1516)
constexpr int SAMPLE_SORT_CAP = 4096;  // top-p candidates sorted inside the block
constexpr int SAMPLE_TOPK_SMALL = 2048;  // top-k up to this needs the large sort only on ties
constexpr int SAMPLE_ERR_CANDIDATES = 16;  // device error flag: top-p candidates overflowed the in-block sort

// Settings, written by the host (pc_set_sampling).
struct SampleParams {
    float temperature;
    float top_p;
    float rep;
    float inv_temp;  // 1.0f / temperature, rounded as the reference's fp32 division
    int top_k;
    int pad[3];
};

// Device-resident state: settings, generator, history length, and the
// hand-over between the draw kernel and the large-sort continuation.
struct SampleState {
    SampleParams p;
    unsigned long long rng;
    int hist_len;
    int stage;   // 1: the top-p candidates wait for the large sort
    int n_nz;    // nonzero probabilities (compacted list length)
    int n_cand;  // top-p candidates among them
    int status;  // 0 ok; 1: more top-p candidates than the in-block sort holds
    int pad;
};

struct Sampler {
    bool on = false;
    bool big = false;  // launch the large-sort continuation
    int V = 0;
    SampleState *state = nullptr;
    int *hist = nullptr;
    int *cnt = nullptr;      // [V] occurrence counts of the penalty (zero between draws)
    float *w = nullptr;      // [V] working values
    float *nz_val = nullptr; // [V] nonzero values in index order
    int *nz_idx = nullptr;   // [V] their token ids
    float *ck = nullptr, *sk = nullptr;  // [V] candidate keys in / sorted
    int *cv = nullptr, *sv = nullptr;    // [V] candidate positions in / sorted
    void *tmp = nullptr;
    size_t tmp_bytes = 0;
};

// Allocates the buffers of a vocabulary of V ids (no-op when already done).
cudaError_t sampler_init(Sampler &s, int V);
void sampler_free(Sampler &s);
// One draw from logits[0..V): the id goes to ids[0] (and ids2[0] when not
// null), and is appended to the history.  Without the large sort (s.big
// false), more than SAMPLE_SORT_CAP top-p candidates (only possible when
// more than SAMPLE_TOPK_SMALL values tie at the top-k threshold) set *err to
// SAMPLE_ERR_CANDIDATES.  Adds the kernels it launched to `launches`.
cudaError_t sampler_launch(const Sampler &s, const float *logits, int *ids, int *ids2, int *err, cudaStream_t st,
                           int &launches);

}  // namespace pc
