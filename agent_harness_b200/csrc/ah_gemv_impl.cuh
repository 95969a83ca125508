// ah_gemv_impl.cuh — host-side interface of the fused Q4 GEMV launcher, shared
// by the standalone GEMV entry points and the decoder.
#pragma once

#include "ah_gemv.cuh"

struct AhQ4Weight;

namespace ah {

// k-split workspace: per-chunk partial outputs and per-tile arrival counters
// (the counters start at zero and the last arriving CTA of a tile resets its
// counter, so consecutive launches need no memset).
struct GemvWorkspace {
  float* partial = nullptr;
  size_t partial_floats = 0;
  int* counters = nullptr;
  int64_t n_counters = 0;
};

struct GemvPlan {
  int nt;                   // n8 tensor-core column tiles (4 tokens each)
  int64_t pairs_per_chunk;  // 64-column block pairs per CTA
  int ksplit;               // CTAs along K per 16-row tile
  size_t smem;              // dynamic shared memory bytes
};

GemvPlan gemv_plan(const Q4Tiled& w, int batch);
// Grows `ws` to hold the k-split state of `plan` (cudaMalloc; not capturable).
int gemv_workspace_reserve(GemvWorkspace& ws, const Q4Tiled& w, const GemvPlan& plan, int batch);
void gemv_workspace_free(GemvWorkspace& ws);
// Launches the fused GEMV with the given prologue/epilogue; `pdl` enables
// programmatic dependent launch (weights are prefetched before the kernel waits
// for its predecessor's output).
int gemv_launch(GemvArgs a, int prologue, int epilogue, GemvWorkspace& ws, cudaStream_t st, bool pdl);

const Q4Tiled& q4w_tiled(const AhQ4Weight* w);
int q4w_create_q4_0_multi(const void* const* srcs, const int64_t* src_rows, int nsrc, int mode, int64_t cols,
                          AhQ4Weight** out, cudaStream_t st);

}  // namespace ah
