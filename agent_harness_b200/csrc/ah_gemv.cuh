// ah_gemv.cuh — the fused Q4 dequant+GEMV kernel (batch 1..16) shared by the
// standalone GEMV entry points and the decoder's fused layer kernels.
//
// Weight layout in HBM ("tiled Q4"): rows are grouped into 16-row tiles and
// columns into 64-column block pairs.  For tile rt and pair kp the 16 rows x 2
// blocks x 16 bytes of nibbles are stored as 32 lane-major 16-byte chunks
// (uint4 nib[rt][kp][lane]); lane l = 4g+t holds four 32-bit words:
//   w0 = block 2kp, row g;  w1 = block 2kp, row g+8;
//   w2 = block 2kp+1, row g; w3 = block 2kp+1, row g+8.
// Nibble p (bits 4p..4p+3) of a word is block element 2t + 8*(p&3) + (p>>2),
// which is exactly the m16n8k16 A-fragment order, so two LOP3s plus one packed
// f16 op turn a word's 8 nibbles into 8 exact f16 (q-8) values in registers.
// Scales sit in their own plane, 8 entries per (rt,kp): entry g holds
// {d(2kp,g), d(2kp,g+8), d(2kp+1,g), d(2kp+1,g+8)} as f16 (Q4_0) or f32 (engine).
//
// The activation x is scaled by 2^s per (token, 32-column block) so that the
// block's max |x| lands in [2^14, 2^15), and split into two f16 planes hi + lo
// that together carry ~22 significant bits; the tensor core then forms
// sum_j (q_j-8) * x_j with f32 accumulation over each 32-element block, and
// the block scale d (times 2^-s) is applied in f32.  Dequantised weights never
// leave registers.
#pragma once

#include "ah_common.cuh"
#include "ah_sm100.cuh"

namespace ah {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvMaxBatch = 16;

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
  // prologue: RMSNorm of x with f16 weight, eps (inference/math.rs:53-63);
  // ss_in holds the producer's partial sums of squares of x, [batch][n_ss_in]
  const uint16_t* norm_w;
  float eps;
  const float* ss_in;
  int n_ss_in;
  // epilogue: optional per-16-row-tile partial sums of squares of the values
  // written, [batch][r16] (feeds the next kernel's RMSNorm prologue)
  float* ss_out;
  // k-split: each CTA covers pairs [ky*pairs_per_chunk, ...) of its tile row
  int64_t pairs_per_chunk;
  int ksplit;
  float* partial;          // [ksplit][r16*16][batch] when ksplit > 1
  int* counters;           // [r16] zero-initialised, reset by the last CTA
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

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(magic));  // (a & b) | c
  return r;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                      *reinterpret_cast<__half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}

// 8 nibbles of one word -> four f16x2 (q-8) pairs P0..P3 in A-fragment order.
__device__ __forceinline__ void unpack_word(uint32_t w, uint32_t& p0, uint32_t& p1, uint32_t& p2, uint32_t& p3) {
  const uint32_t kMagic = 0x64006400u;       // f16 1024.0 in both halves
  const uint32_t kSub = 0x64086408u;         // f16 1032.0
  const uint32_t kOne16 = 0x2C002C00u;       // f16 1/16
  const uint32_t kNeg72 = 0xD480D480u;       // f16 -72.0
  const uint32_t w8 = w >> 8;
  p0 = hsub2_u32(lop3_and_or(w, 0x000F000Fu, kMagic), kSub);             // 1024+n - 1032
  p1 = hfma2_u32(lop3_and_or(w, 0x00F000F0u, kMagic), kOne16, kNeg72);   // (1024+16n)/16 - 72
  p2 = hsub2_u32(lop3_and_or(w8, 0x000F000Fu, kMagic), kSub);
  p3 = hfma2_u32(lop3_and_or(w8, 0x00F000F0u, kMagic), kOne16, kNeg72);
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
