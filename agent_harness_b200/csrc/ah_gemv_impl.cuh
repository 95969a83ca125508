// ah_gemv_impl.cuh — host-side interface of the fused Q4 GEMV launcher, shared
// by the standalone GEMV entry points and the decoder.
#pragma once

#include "ah_gemv.cuh"

struct AhQ4Weight;

namespace ah {

struct GemvPlan {
  int nt;                   // n8 tensor-core column tiles (4 tokens each)
  int64_t pairs_per_chunk;  // 64-column block pairs per K-chunk (cluster CTA)
  int ksplit;               // always 1: a launch covers the full K
  size_t smem;              // dynamic shared memory bytes
  bool rows_mode;           // persistent full-K CTAs instead of clusters
  size_t smem_base;         // rows mode: shared memory besides the tile stages
  int n_stages;             // rows mode: row tiles in flight (0: rows mode unavailable)
};

GemvPlan gemv_plan(const Q4Tiled& w, int batch);
// kp_window > 0: a cluster-mode launch over a window of that many block pairs
GemvPlan gemv_plan(const Q4Tiled& w, int batch, bool rows_mode, int64_t kp_window = 0);
// Launches the fused GEMV with the given prologue/epilogue; `pdl` enables
// programmatic dependent launch (weights are prefetched before the kernel waits
// for its predecessor's output).
int gemv_launch(GemvArgs a, int prologue, int epilogue, cudaStream_t st, bool pdl);
// Resolves the kernel's shared-memory attribute and occupancy for (w, batch,
// prologue, epilogue) without launching, so a later launch can be captured.
int gemv_prepare(const Q4Tiled& w, int batch, int prologue, int epilogue);

// The tcgen05 GEMM c[m][ldc] = a[m][lda] . W^T (ah_gemm_tc.cu) and the
// workspace it needs for m rows (1024-byte aligned).  Epilogues: store;
// SwiGLU over an interleaved gate/up weight (16-row tiles of 8 gate rows,
// then the 8 up rows of the same outputs; c gets rows/2 columns
// silu(gate) * up); residual add (c += a . W^T).  With norm_w (f16, cols
// entries) each row of a is RMS-normalised first (inference/math.rs:53-63).
enum GemmEpilogue { kGemmEpiStore = 0, kGemmEpiSwiglu = 1, kGemmEpiAdd = 2 };
size_t gemm_workspace_bytes(const Q4Tiled& w, int64_t m);
int gemm_run(const Q4Tiled& w, const float* a, int64_t lda, int64_t m, float* c, int64_t ldc, void* ws,
             size_t ws_bytes, cudaStream_t st, int epi = kGemmEpiStore, const uint16_t* norm_w = nullptr,
             float eps = 0.0f);

// The tcgen05 batched GEMV (ah_bgemv_tc.cu): the same products as
// gemv_launch for 1..16 tokens, weights dequantised into tensor memory, work
// split stream-K over persistent CTAs.  Needs a 1024-byte aligned workspace of
// bgemv_workspace_bytes(w); bgemv_prepare sets kernel attributes ahead of a
// graph capture.  K windows (pair_end) are not supported.
size_t bgemv_workspace_bytes(const Q4Tiled& w);
int bgemv_prepare(const Q4Tiled& w, int epilogue);
int bgemv_launch(const GemvArgs& a, int prologue, int epilogue, void* ws, size_t ws_bytes, cudaStream_t st,
                 bool pdl);

const Q4Tiled& q4w_tiled(const AhQ4Weight* w);
// An uninitialised tiled weight of the given shape (f32 scales when `engine`);
// its planes are filled by the caller's kernel.
int q4w_alloc(int64_t rows, int64_t cols, bool engine, AhQ4Weight** out);
uint4* q4w_nib_mut(AhQ4Weight* w);
void* q4w_scales_mut(AhQ4Weight* w);
int q4w_create_q4_0_multi(const void* const* srcs, const int64_t* src_rows, int nsrc, int mode, int64_t cols,
                          AhQ4Weight** out, cudaStream_t st);
// The same from engine-format sources (quantize() output: f32 scales per
// 32-column group, packed nibbles, low nibble first).
int q4w_create_engine_multi(const float* const* scales, const uint8_t* const* packed, const int64_t* src_rows,
                            int nsrc, int mode, int64_t cols, AhQ4Weight** out, cudaStream_t st);

}  // namespace ah
