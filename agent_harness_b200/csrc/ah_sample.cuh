// ah_sample.cuh — temperature + top-k sampling on the device (ah_sample.cu).
#pragma once

#include "ah_common.cuh"

namespace ah {

constexpr int kSampleMaxK = 64;      // largest top_k (the reference's generate uses 40)
constexpr int kSampleMaxRanks = 8;   // tensor-parallel ranks whose candidates k_sample_merge ranks
constexpr int kSampleSlice = 4096;   // logits per slice CTA when a row is split

struct SampleCand {
  float v;  // logit
  int i;    // global vocabulary index (INT_MAX: no candidate)
};

// The uniform draw in [0, 1) (24 random bits) of sequence `seq` at step `step`.
__host__ __device__ float sample_uniform(uint64_t seed, int64_t step, int seq);

// The top-k of logits[b][0 .. n) (row stride ld) for b < batch, with global
// indices local + idx_base.  With `cand` null it samples (the step is
// *step_dev when given, else `step`) and writes tok[b] (and
// tok_log[step * batch + b]); else it writes the k sorted candidates
// cand[b][k] for k_sample_merge.  With a workspace of
// sample_workspace_bytes(batch, n) (16-byte aligned) rows longer than one
// slice are split over kSampleSlice-logit CTAs; without one (ws null) one CTA
// walks each row.
size_t sample_workspace_bytes(int batch, int64_t n);
int sample_launch(const float* logits, int64_t ld, int batch, int64_t n, int k, int64_t idx_base, float temperature,
                  uint64_t seed, int64_t step, const int* step_dev, SampleCand* cand, int* tok, int* tok_log,
                  void* ws, size_t ws_bytes, cudaStream_t st);
// The world ranks' candidates all[world][batch][k] -> the global top-k and the
// sample, written to tok[b] and tok_log[*step_dev * batch + b].
int sample_merge_launch(const SampleCand* all, int world, int batch, int k, float temperature, uint64_t seed,
                        const int* step_dev, int* tok, int* tok_log, cudaStream_t st);

}  // namespace ah
