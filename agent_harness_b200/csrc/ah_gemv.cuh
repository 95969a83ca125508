// ah_gemv.cuh — the fused Q4 dequant+GEMV kernel (batch 1..16) shared by the
// standalone GEMV entry points and the decoder's fused layer kernels.
//
// Weight layout in HBM ("tiled Q4"): rows are grouped into 16-row tiles and
// columns into 64-column block pairs.  For tile rt and pair kp the 16 rows x 2
// blocks x 16 bytes of nibbles are stored as 32 lane-major 16-byte chunks
// (uint4 nib[rt][kp][lane]); lane l = 4g+t holds four 32-bit words:
//   w0 = block 2kp, row g;  w1 = block 2kp, row g+8;
//   w2 = block 2kp+1, row g; w3 = block 2kp+1, row g+8.
// Nibble p (bits 4p..4p+3) of a word is block element
// 2t + (p>>2) + 16*(p&1) + 8*((p>>1)&1), the m16n8k16 A-fragment order: one AND
// per register turns a nibble pair into two f16 subnormals, q*2^-24 (k-step 0)
// or q*2^-20 (k-step 1), which the tensor core multiplies exactly.  The -8
// offset is applied through the accumulator start value, -8*sum(x) per block.
// Scales sit in their own plane, 8 entries per (rt,kp): entry g holds
// {d(2kp,g), d(2kp,g+8), d(2kp+1,g), d(2kp+1,g+8)} as f16 (Q4_0) or f32 (engine).
//
// The activation x is split in-kernel: per (token, 32-column block) it is
// scaled by 2^s so the block's max |x| lands in [2^14, 2^15) and stored in
// shared memory as two f16 values hi + lo carrying ~22 significant bits
// (k-step-1 columns stored /16 to meet the x16 larger A values), together with
// {2^(24-s), -8*2^-24*sum(hi), -8*2^-24*sum(lo)}.  The tensor core forms
// sum_j (q_j-8) * x_j with f32 accumulation over each block (the -8 enters as
// the accumulator start value) and the block scale d * 2^(24-s) is applied in
// f32.  Dequantised weights never leave registers.
#pragma once

#include "ah_common.cuh"
#include "ah_sm100.cuh"

namespace ah {

// inference/math.rs:83-95 silu (the GEMV and GEMM SwiGLU epilogues, the
// prefill row kernels)
__device__ __forceinline__ float silu_ref(float x) {
  const float sg = x >= 0.0f ? __fdiv_rn(1.0f, 1.0f + expf(-x)) : __fdiv_rn(expf(x), 1.0f + expf(x));
  return x * sg;
}


constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvMaxBatch = 16;
constexpr int kGemvCluster = kGemvWarps;  // CTAs per cluster = K-chunks = warps per CTA
constexpr int kGemvU = 4;                 // block pairs per register batch (two batches in flight)
// Wide batches (3-4 n8 tiles) keep 2 pairs per batch and cap registers so two
// CTAs fit per SM.
template <int NT>
constexpr int kGemvBatchPairs = NT >= 3 ? 2 : kGemvU;
// Minimum resident CTAs per SM for the cluster kernel's __launch_bounds__
// (the rows kernel always asks for 2): 2 for wide batches (a 128-register cap); 0 leaves narrow batches at the compiler's own choice
// (~128 registers for 1 tile, ~138 for 2).  An explicit 1 would let those
// take 150-200 registers, i.e. one CTA per SM, which made batch-1 GEMVs up
// to 1.9x slower.
template <int NT>
constexpr int kGemvMinBlocks = NT >= 3 ? 2 : 0;
constexpr int kGemvSmemLimit = 200 * 1024;
constexpr int kGemvRowsSmem = 96 * 1024;   // rows mode only while x's split takes at most this much
constexpr int kGemvRowsCtaSmem = 112 * 1024;  // rows mode: two CTAs (16 warps) per SM
constexpr int kGemvMaxStages = 4;          // rows mode: row tiles in flight per CTA

struct Q4Tiled {
  const uint4* nib;    // [r16][kp][32]
  const void* scales;  // [r16][kp][8] of uint2 (f16x4) or float4
  int64_t rows, cols;  // logical shape
  int64_t r16, kp;     // tiles, block pairs
  bool f32_scales;
};

// ---- epilogue / prologue selectors --------------------------------------------
enum GemvPrologue : int { kProPlain = 0, kProRmsNorm = 1 };
enum GemvEpilogue : int { kEpiStore = 0, kEpiAdd = 1, kEpiSwiglu = 2 };

struct GemvArgs {
  Q4Tiled w;
  const float* x;          // [batch][x_stride] f32
  int64_t x_stride;
  float* y;                // [batch][y_stride] f32
  int64_t y_stride;
  int batch;
  // RMSNorm prologue (inference/math.rs:53-63): x is normalised as
  // (x * 1/rms) * norm_w while it is split; 1/rms per token comes from the
  // producer's partial sums of squares of x, ss_in [batch][n_ss_in].
  const uint16_t* norm_w;
  float eps;
  const float* ss_in;
  int n_ss_in;
  // epilogue: optional per-16-row-tile partial sums of squares of the values
  // written, [batch][r16] (feeds the next kernel's RMSNorm prologue)
  float* ss_out;
  int64_t pairs_per_chunk; // block pairs per K-chunk (cluster CTA)
  int early_trigger;       // set by the launcher: grid fits in one resident wave
  int n_stages;            // rows mode: row tiles in flight in shared memory
  // cluster mode: the block pairs [pair_begin, pair_end) of K this launch
  // covers (pair_end 0: all of K); a GEMV whose split of x would not fit runs
  // as launches over K windows, the later ones adding into y
  int64_t pair_begin, pair_end;
  int* err;                // device error word (a bounded wait that gave up)
  // Store epilogue scatter (tensor-parallel all-reduce over peer memory): with
  // n_peer > 0 every output element goes to peer_y[p] + row*peer_row + b for
  // p < n_peer (local and peer GPUs' receive buffers) instead of y: rows of
  // `peer_row` floats with the tokens contiguous, so a tile's outputs leave
  // as one contiguous run per destination.
  int n_peer;
  int peer_row;
  float* peer_y[8];
};

// ---- small PTX helpers -------------------------------------------------------
__device__ __forceinline__ uint4 ldg_stream_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_nc_v2(const uint2* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldg_nc_f4(const float4* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

}  // namespace ah
