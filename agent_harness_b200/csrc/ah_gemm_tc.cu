// ah_gemm_tc.cu — Q4 prefill GEMM on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory).
//
//   C[m][n] = sum_k A[m][k] * W[n][k],  W[n][k] = d(n, k/32) * (q(n,k) - 8)
//
// A (tokens x cols, f32) is converted once per call by k_gemm_prep into a
// row-major f16 copy, each token row scaled by an exact power of two 2^s so
// its max |a| lies in [2^14, 2^15) (f16 keeps 11 significant bits over the
// row's whole range; C rows are multiplied by 2^-s in the epilogue).  A TMA
// tensor map with 128-byte swizzle brings 128-token x 64-column boxes of it
// into shared memory in the tensor core's K-major SWIZZLE_128B image.  W stays in the GEMV's tiled Q4 layout in HBM (see
// ah_gemv.cuh): the kernel bulk-copies the nibble and scale chunks of a
// 208-row x 64-column tile into shared memory, four dequant warps expand them
// to f16 d*(q-8) (one rounding, RNE) straight into the swizzled B image, and
// one thread issues the MMAs:
//
//   warp 0      raw weight producer   (2-D TMA boxes of 13 row tiles -> raw ring)
//   warp 1      activation producer   (cp.async.bulk -> A ring, 3 stages)
//   warp 2      TMEM owner + MMA issuer (tcgen05.mma M=128 N=208 K=16, f16 in,
//               f32 accumulate; tcgen05.commit frees a stage)
//   warps 3..10 dequant (raw ring -> B ring); warps 3..6 then run the
//               epilogue (tcgen05.ld 32x32b -> shared staging -> bulk copy to C)
//
// A CTA owns 256 tokens (two M=128 accumulators, TMEM columns [0,208) and
// [256,464)) x 208 weight rows over the full K.  For the MLP up-projection
// shape (M 512, N 14336, K 4096) that is 2 x 69 = 138 CTAs: one wave on 148
// SMs, one CTA per SM (shared memory ~207 KB).
//
// Every mbarrier wait is bounded; a wait that gives up records AH_ETIMEOUT in
// the device error word, raises a CTA-wide abort flag, and the kernel drains
// its own bulk copies and MMAs before freeing tensor memory and returning.
//
// Reference: the prefill of inference/mod.rs:547-562 runs forward() token by
// token (mod.rs:550), i.e. one gemv_4bit_into (inference/math.rs:255-295) per
// token and projection; this kernel computes the same products for all
// tokens of a prompt at once.

#include <algorithm>
#include <mutex>

#include "ah_common.cuh"
#include "ah_gemv_impl.cuh"
#include "ah_sm100.cuh"
#include "ah_tc.cuh"
#include "ah_tma.cuh"

struct AhQ4Weight;

namespace ah {
namespace {

constexpr int kTokTile = 128;                       // tokens per MMA (TMEM lanes)
constexpr int kRowTiles = 13;                       // 16-row weight tiles per CTA
constexpr int kBN = kRowTiles * 16;                 // 208 = MMA N
constexpr int kBK = 64;                             // columns per k-step (one block pair)
constexpr int kStages = 3;                          // A/B operand ring
constexpr int kRawStages = 4;                       // raw weight ring
constexpr int kATileBytes = kTokTile * kBK * 2;     // 16384
constexpr int kBBytes = kBN * kBK * 2;              // 26624
constexpr int kRawNibBytes = kRowTiles * 512;       // 6656
constexpr int kRawBytes = kRawNibBytes + kRowTiles * 128;  // + f32 scales worst case
constexpr int kTmemCols = 512;
constexpr int kAccColStride = 256;                  // TMEM column offset of token half 1
constexpr int kDequantWarps = 8;  // >= 4: the first four cover the TMEM lane quarters in the epilogue
constexpr int kGemmThreads = (3 + kDequantWarps) * 32;
constexpr uint32_t kWaitLimit = 1u << 24;
constexpr int kStageStride = kBN + 4;  // f32 per staged C row: 848 B, 16-byte stores conflict-free
constexpr int kGluStride = kBN / 2 + 4;  // the same for a SwiGLU row (104 outputs): 432 B

constexpr uint32_t kIdesc = idesc_f16(kTokTile, kBN);

template <int kHalves>
struct GemmSmem {
  static constexpr int kA = 0;
  static constexpr int kB = kA + kStages * kHalves * kATileBytes;
  static constexpr int kRaw = kB + kStages * kBBytes;
  static constexpr int kBars = kRaw + kRawStages * kRawBytes;
  // the epilogue stages 128 rows of C over the (then idle) operand rings (a
  // SwiGLU epilogue: both token halves at once)
  static_assert(kTokTile * kStageStride * 4 <= kBars, "C staging must fit below the barriers");
  static_assert(2 * kTokTile * kGluStride * 4 <= kBars, "SwiGLU staging must fit below the barriers");
  static constexpr int kNumBars = 3 * kStages + 2 * kRawStages + 1;
  static constexpr int kMisc = kBars + kNumBars * 8;
  static constexpr int kTotal = kMisc + 16;
  static constexpr size_t kDynamic = (size_t)kTotal + 1024;  // slack for 1 KB alignment
};

struct GemmArgs {
  CUtensorMap tm_nib;     // nibble plane as uint32 [r16][kp*128], box 128 x kRowTiles
  CUtensorMap tm_scale;   // scale plane as uint32 [r16][kp*16|32], box 16|32 x kRowTiles
  Q4Tiled w;
  CUtensorMap tm_a;       // f16 activations [M_pad][kp*64], box 64 x 128, 128-byte swizzle
  const uint8_t* at;      // the same activations (row-major f16)
  const float* row_inv;   // [M_pad] 2^-s per token row
  float* c;
  int64_t ldc;
  int64_t m;
  int* err;
  int epi;     // GemmEpilogue
  bool c_vec;  // ldc % 4 == 0 and c 16-byte aligned
};

// Waits on `bar`'s phase `parity`; on give-up raises the CTA abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag,
                                              int code) {
  if (mbar_wait_bounded(bar, parity, err, code, kWaitLimit)) return true;
  *abort_flag = 1;
  return false;
}

// ---- activation prep: f32 rows -> scaled row-major f16 -------------------------
// One CTA per (padded) token row of kp*64 f16 (columns past K are zero).  The
// row is read once into registers (kChunks <= kPrepChunks 8-column chunks per
// thread, i.e. up to 16384 columns); longer rows take a second read.
constexpr int kPrepThreads = 256;
constexpr int kPrepChunks = 8;

__device__ __forceinline__ void prep_load8(const float* row, int64_t k0, int64_t k_cols, bool vec, bool live,
                                           float (&v)[8]) {
  if (vec && k0 + 8 <= k_cols) {
    const float4 p0 = __ldg(reinterpret_cast<const float4*>(row + k0));
    const float4 p1 = __ldg(reinterpret_cast<const float4*>(row + k0 + 4));
    v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
    v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (live && k0 + i < k_cols) ? row[k0 + i] : 0.0f;
  }
}

__device__ __forceinline__ void prep_store8(uint8_t* out_row, int64_t c, const float (&v)[8], float scale) {
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 hv = __floats2half2_rn(v[2 * i] * scale, v[2 * i + 1] * scale);
    h[i] = *reinterpret_cast<const uint32_t*>(&hv);
  }
  *reinterpret_cast<uint4*>(out_row + c * 16) = make_uint4(h[0], h[1], h[2], h[3]);
}

// Block-wide sum (kPrepThreads threads) through red[]; every thread gets it.
__device__ __forceinline__ float prep_block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red[] may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int i = 1; i < kPrepThreads / 32; ++i) t += red[i];
  return t;
}

// With norm_w: the row is RMS-normalised first (inference/math.rs:53-63:
// x * 1/sqrt(mean(x^2) + eps) * w, w f16), so a GEMM can take the hidden rows
// directly.
__device__ __forceinline__ void prep_norm8(float (&v)[8], int64_t k0, int64_t k_cols, float inv,
                                           const uint16_t* __restrict__ norm_w) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
    v[i] = k0 + i < k_cols ? (v[i] * inv) * __half2float(__ushort_as_half(norm_w[k0 + i])) : 0.0f;
}

template <int kChunks>
__global__ void __launch_bounds__(kPrepThreads) k_gemm_prep(const float* __restrict__ a, int64_t lda, int64_t m_rows,
                                                            int64_t k_cols, int64_t kp, bool vec_rows,
                                                            const uint16_t* __restrict__ norm_w, float eps,
                                                            uint8_t* __restrict__ at, float* __restrict__ row_inv) {
  // the GEMM may start its prologue and weight loads now; it waits for this
  // grid's completion before reading the tiles
  pdl_launch_dependents();
  const int64_t m = blockIdx.x;
  const int tid = threadIdx.x;
  const bool live = m < m_rows;
  const float* row = a + (live ? m : 0) * lda;
  const bool vec = live && vec_rows;
  const int64_t nchunks = kp * 8;
  const bool in_regs = nchunks <= (int64_t)kPrepThreads * kChunks;
  __shared__ float red[kPrepThreads / 32];
  float v[kChunks][8];
  if (in_regs) {
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int64_t c = tid + (int64_t)j * kPrepThreads;
      if (c < nchunks) prep_load8(row, c * 8, k_cols, vec, live, v[j]);
    }
  }
  // RMSNorm factor of the row
  float inv = 1.0f;
  if (norm_w) {
    float ss = 0.0f;
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
        if (tid + (int64_t)j * kPrepThreads < nchunks)
#pragma unroll
          for (int i = 0; i < 8; ++i) ss = fmaf(v[j][i], v[j][i], ss);
    } else if (live) {
      for (int64_t k = tid; k < k_cols; k += kPrepThreads) ss = fmaf(row[k], row[k], ss);
    }
    ss = prep_block_sum(ss, red);
    inv = __fdiv_rn(1.0f, sqrtf(__fdiv_rn(ss, (float)k_cols) + eps));  // inference/math.rs:59
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < kChunks; ++j) {
        const int64_t c = tid + (int64_t)j * kPrepThreads;
        if (c < nchunks) prep_norm8(v[j], c * 8, k_cols, inv, norm_w);
      }
    }
  }
  // max |a| over the row (NaN ignored here; it still reaches C)
  float amax = 0.0f;
  if (in_regs) {
#pragma unroll
    for (int j = 0; j < kChunks; ++j)
      if (tid + (int64_t)j * kPrepThreads < nchunks)
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[j][i]));
  } else if (live) {
    for (int64_t k = tid; k < k_cols; k += kPrepThreads) {
      const float x = norm_w ? (row[k] * inv) * __half2float(__ushort_as_half(norm_w[k])) : row[k];
      amax = fmaxf(amax, fabsf(x));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __syncthreads();  // red[] may still be read by the RMSNorm reduction
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < kPrepThreads / 32; ++i) amax = fmaxf(amax, red[i]);
  // exponent s with amax * 2^s in [2^14, 2^15), clamped so 2^s and 2^-s are
  // normal floats; zero rows and non-finite maxima keep s = 0
  int s = 0;
  const uint32_t ab = __float_as_uint(amax);
  if (amax > 0.0f && ((ab >> 23) & 0xFF) != 0xFF) {
    const int e = (int)((ab >> 23) & 0xFF) - 126;  // amax in [2^(e-1), 2^e)
    s = min(max(15 - e, -120), 120);
  }
  const float scale = __uint_as_float((uint32_t)(127 + s) << 23);
  if (tid == 0) row_inv[m] = live ? __uint_as_float((uint32_t)(127 - s) << 23) : 0.0f;
  uint8_t* out_row = at + (size_t)m * (size_t)kp * 128;
  if (in_regs) {
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int64_t c = tid + (int64_t)j * kPrepThreads;
      if (c < nchunks) prep_store8(out_row, c, v[j], scale);
    }
  } else {
    for (int64_t c = tid; c < nchunks; c += kPrepThreads) {
      float w[8];
      prep_load8(row, c * 8, k_cols, vec, live, w);
      if (norm_w) prep_norm8(w, c * 8, k_cols, inv, norm_w);
      prep_store8(out_row, c, w, scale);
    }
  }
}

// ---- the GEMM ------------------------------------------------------------------
template <int kHalves, bool kF32>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm_q4_tc(const __grid_constant__ GemmArgs g) {
  using L = GemmSmem<kHalves>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* a_full = bars;
  uint64_t* b_full = bars + kStages;
  uint64_t* ab_empty = bars + 2 * kStages;
  uint64_t* raw_full = bars + 3 * kStages;
  uint64_t* raw_empty = raw_full + kRawStages;
  uint64_t* acc_full = raw_empty + kRawStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t kp = g.w.kp;
  const int64_t rt0 = (int64_t)blockIdx.x * kRowTiles;
  const int nrt = (int)(g.w.r16 - rt0 < kRowTiles ? g.w.r16 - rt0 : kRowTiles);
  const int64_t mt0 = (int64_t)blockIdx.y * kHalves;
  // CTAs sharing a token tile start their K walk at staggered block pairs, so
  // at any moment they fetch different activation tiles from L2
  const int64_t k_rot = (int64_t)blockIdx.x * kp / gridDim.x;
  constexpr int kScaleBytes = kF32 ? 128 : 64;  // per (row tile, pair)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&b_full[i], kDequantWarps);
      mbar_init(&ab_empty[i], 1);
    }
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kDequantWarps);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---- raw weight producer: one nibble box + one scale box per k-step ----
    if (lane == 0) {
      // boxes are full size; rows past the matrix arrive zero-filled
      constexpr uint32_t kStageTx = kRowTiles * (512 + kScaleBytes);
      int64_t issued = 0;
      for (int64_t s = 0; s < kp; ++s) {
        const int r = (int)(s % kRawStages);
        if (*abort_flag) break;
        if (s >= kRawStages &&
            !wait_or_abort(&raw_empty[r], (uint32_t)((s / kRawStages - 1) & 1), g.err, abort_flag, AH_ETIMEOUT))
          break;
        uint8_t* dst = smem + L::kRaw + r * kRawBytes;
        mbar_arrive_expect_tx(&raw_full[r], kStageTx);
        const int64_t kpos = (s + k_rot) % kp;
        tma_load_2d(dst, &g.tm_nib, (int)(kpos * 128), (int)rt0, &raw_full[r]);
        tma_load_2d(dst + kRawNibBytes, &g.tm_scale, (int)(kpos * (kScaleBytes / 4)), (int)rt0, &raw_full[r]);
        ++issued;
      }
      // drain: the copies of the last stages have landed before the CTA can exit
      if (*abort_flag) {
        for (int64_t s = issued > kRawStages ? issued - kRawStages : 0; s < issued; ++s)
          mbar_wait_bounded(&raw_full[s % kRawStages], (uint32_t)((s / kRawStages) & 1), g.err, AH_ETIMEOUT,
                            kWaitLimit);
      }
    }
  } else if (warp == 1) {
    // ---- activation producer ----
    if (lane == 0) {
      pdl_wait();  // the tiles come from the preceding prep grid
      int64_t issued = 0;
      for (int64_t s = 0; s < kp; ++s) {
        const int st = (int)(s % kStages);
        if (*abort_flag) break;
        if (s >= kStages &&
            !wait_or_abort(&ab_empty[st], (uint32_t)((s / kStages - 1) & 1), g.err, abort_flag, AH_ETIMEOUT))
          break;
        mbar_arrive_expect_tx(&a_full[st], (uint32_t)(kHalves * kATileBytes));
        for (int h = 0; h < kHalves; ++h) {
          tma_load_2d(smem + L::kA + (st * kHalves + h) * kATileBytes, &g.tm_a, (int)(((s + k_rot) % kp) * kBK),
                      (int)((mt0 + h) * kTokTile), &a_full[st]);
        }
        ++issued;
      }
      if (*abort_flag) {
        for (int64_t s = issued > kStages ? issued - kStages : 0; s < issued; ++s)
          mbar_wait_bounded(&a_full[s % kStages], (uint32_t)((s / kStages) & 1), g.err, AH_ETIMEOUT, kWaitLimit);
      }
    }
  } else if (warp == 2) {
    // ---- MMA issuer ----
    if (lane == 0) {
      for (int64_t s = 0; s < kp; ++s) {
        const int st = (int)(s % kStages);
        const uint32_t ph = (uint32_t)((s / kStages) & 1);
        if (*abort_flag) break;
        if (!wait_or_abort(&a_full[st], ph, g.err, abort_flag, AH_ETIMEOUT)) break;
        if (!wait_or_abort(&b_full[st], ph, g.err, abort_flag, AH_ETIMEOUT)) break;
        tc_fence_after();
        const uint32_t b_addr = smem_u32(smem + L::kB + st * kBBytes);
#pragma unroll
        for (int h = 0; h < kHalves; ++h) {
          const uint32_t a_addr = smem_u32(smem + L::kA + (st * kHalves + h) * kATileBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_f16(tmem_base + h * kAccColStride, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), kIdesc,
                    (s > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&ab_empty[st]);
      }
      // completes when every MMA above has (also on abort, so TMEM can be freed)
      mma_commit(acc_full);
    }
  } else {
    // ---- dequant warps, then epilogue ----
    const int wd = warp - 3;
    const int gq = lane >> 2, t = lane & 3;
    for (int64_t s = 0; s < kp; ++s) {
      const int r = (int)(s % kRawStages);
      const int st = (int)(s % kStages);
      bool ok = true;
      if (lane == 0) {
        if (*abort_flag) ok = false;
        else {
          ok = wait_or_abort(&raw_full[r], (uint32_t)((s / kRawStages) & 1), g.err, abort_flag, AH_ETIMEOUT);
          if (ok && s >= kStages)
            ok = wait_or_abort(&ab_empty[st], (uint32_t)((s / kStages - 1) & 1), g.err, abort_flag, AH_ETIMEOUT);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const uint8_t* raw = smem + L::kRaw + r * kRawBytes;
      const uint32_t bst = smem_u32(smem + L::kB + st * kBBytes);
      for (int rt = wd; rt < nrt; rt += kDequantWarps) {
        const uint4 nv = *reinterpret_cast<const uint4*>(raw + rt * 512 + lane * 16);
        const uint32_t wv[4] = {nv.x, nv.y, nv.z, nv.w};
        float dsc[4];
        __half dh[4];
        if (kF32) {
          const float4 d4 = *reinterpret_cast<const float4*>(raw + kRawNibBytes + rt * 128 + gq * 16);
          dsc[0] = d4.x; dsc[1] = d4.y; dsc[2] = d4.z; dsc[3] = d4.w;
        } else {
          const uint2 d2 = *reinterpret_cast<const uint2*>(raw + kRawNibBytes + rt * 64 + gq * 8);
          dh[0] = __ushort_as_half((unsigned short)(d2.x & 0xFFFFu));
          dh[1] = __ushort_as_half((unsigned short)(d2.x >> 16));
          dh[2] = __ushort_as_half((unsigned short)(d2.y & 0xFFFFu));
          dh[3] = __ushort_as_half((unsigned short)(d2.y >> 16));
        }
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const int blk = wi >> 1, half = wi & 1;
          const int row = rt * 16 + gq + 8 * half;  // (row & 7) == gq
          const uint32_t row_addr = bst + row * 128 + 4 * t;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // nibbles j and j+4 of the word are block elements 2t+off and
            // 2t+off+1, off = {0,16,8,24}[j]; 1024+q is exact in f16.
            const uint32_t bits = ((wv[wi] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
            __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&bits), __float2half2_rn(1032.0f));
            __half2 v;
            if (kF32) {
              const float2 qf = __half22float2(q);
              v = __floats2half2_rn(qf.x * dsc[wi], qf.y * dsc[wi]);
            } else {
              v = __hmul2(q, __half2half2(dh[wi]));
            }
            const int chunk = 4 * blk + ((j & 1) << 1) + (j >> 1);  // k/8 for off {0,16,8,24}
            sts32(row_addr + ((chunk ^ gq) << 4), *reinterpret_cast<const uint32_t*>(&v));
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&b_full[st]);
        mbar_arrive(&raw_empty[r]);
      }
    }
    // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (its token rows).
    // Each thread stages its row segment (208 columns, scaled by 2^-s) in the
    // now idle operand rings and writes it with one bulk copy, so C leaves the
    // SM as whole 832-byte row runs instead of 16-byte pieces of 32 rows (the
    // residual-add epilogue adds the run into C with one bulk reduce).  Where
    // the bulk copy cannot address C (unaligned, ragged by a non multiple of 4
    // columns), threads store their 16-column pieces directly.  Dequant warps
    // past the first four have no epilogue work, except under the SwiGLU
    // epilogue: there warps 3..6 take token half 0 and warps 7..10 half 1.
    // Its 16-column TMEM chunks are whole weight tiles (8 gate rows, then the
    // 8 up rows of the same outputs), so each yields 8 outputs
    // silu(g * 2^-s) * (u * 2^-s).
    const bool glu = g.epi == kGemmEpiSwiglu;
    const int h_first = glu && wd >= 4 ? 1 : 0;
    const int h_step = glu ? 2 : 1;
    const bool epi_warp = glu ? (wd < 4 || kHalves == 2) : wd < 4;
    const bool have =
        __all_sync(0xffffffffu, epi_warp && mbar_wait_bounded(acc_full, 0, g.err, AH_ETIMEOUT, kWaitLimit));
    tc_fence_after();
    pdl_wait();  // row_inv comes from the preceding prep grid
    if (have && !*abort_flag) {
      const int q = warp & 3;
      const int64_t n0 = rt0 * 16;
      const int64_t n_rows = g.w.rows;
      const int ncols = (int)(n_rows - n0 < kBN ? n_rows - n0 : kBN);
      const int64_t o0 = glu ? n0 / 2 : n0;            // first output column
      const int64_t n_out = glu ? n_rows / 2 : n_rows;  // output columns of C
      const int ocols = glu ? ncols / 2 : ncols;
      const bool bulk = g.c_vec && (ocols % 4) == 0;
      float* stage = glu ? reinterpret_cast<float*>(smem) + (h_first * kTokTile + q * 32 + lane) * kGluStride
                         : reinterpret_cast<float*>(smem) + (q * 32 + lane) * kStageStride;
      for (int h = h_first; h < kHalves; h += h_step) {
        const int64_t m = (mt0 + h) * kTokTile + q * 32 + lane;
        const float inv = m < g.m ? g.row_inv[m] : 0.0f;
        float* crow = g.c + m * g.ldc;
        if (bulk && h > h_first) bulk_wait_read0();  // the previous row's copy has read the stage
#pragma unroll 1
        for (int c0 = 0; c0 < kBN; c0 += 16) {
          float v[16];
          tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * kAccColStride + c0), v);
          if (glu) {
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = silu_ref(v[i] * inv) * (v[i + 8] * inv);
            if (bulk) {
              *reinterpret_cast<float4*>(stage + c0 / 2) = make_float4(o[0], o[1], o[2], o[3]);
              *reinterpret_cast<float4*>(stage + c0 / 2 + 4) = make_float4(o[4], o[5], o[6], o[7]);
              continue;
            }
            if (m >= g.m) continue;
            const int64_t n = o0 + c0 / 2;
            if (g.c_vec && n + 8 <= n_out) {
              st_cs_f4(reinterpret_cast<float4*>(crow + n), make_float4(o[0], o[1], o[2], o[3]));
              st_cs_f4(reinterpret_cast<float4*>(crow + n + 4), make_float4(o[4], o[5], o[6], o[7]));
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i)
                if (n + i < n_out) crow[n + i] = o[i];
            }
            continue;
          }
          if (bulk) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(stage + c0 + i) =
                  make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
            continue;
          }
          if (m >= g.m) continue;
          const int64_t n = n0 + c0;
          if (g.epi == kGemmEpiAdd) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (n + i < n_rows) crow[n + i] += v[i] * inv;  // residual: hidden[i] += out[i]
          } else if (g.c_vec && n + 16 <= n_rows) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              st_cs_f4(reinterpret_cast<float4*>(crow + n + i),
                       make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv));
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (n + i < n_rows) crow[n + i] = v[i] * inv;
          }
        }
        if (bulk && m < g.m) {
          fence_proxy_async_smem();
          if (g.epi == kGemmEpiAdd)
            bulk_s2g_add_f32(crow + o0, smem_u32(stage), (uint32_t)ocols * 4u);
          else
            bulk_s2g(crow + o0, smem_u32(stage), (uint32_t)ocols * 4u);
          bulk_commit();
        }
      }
      if (bulk) bulk_wait_all();  // C written before the CTA retires
    }
  }

  // teardown: every MMA has completed (acc_full) before TMEM is released
  if (warp == 2 && lane == 0 && *abort_flag) mbar_wait_bounded(acc_full, 0, g.err, AH_ETIMEOUT, kWaitLimit);
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int kHalves, bool kF32>
int gemm_launch(const GemmArgs& a, int64_t grid_x, int64_t grid_y, cudaStream_t st) {
  using L = GemmSmem<kHalves>;
  static_assert(L::kDynamic <= 227 * 1024, "shared memory budget");
  auto kern = k_gemm_q4_tc<kHalves, kF32>;
  // the shared-memory cap is set once per device, race-free across host threads
  constexpr int kMaxDevices = 64;
  static std::once_flag once[kMaxDevices];
  static cudaError_t set_rc[kMaxDevices];
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  AH_REQUIRE(dev >= 0 && dev < kMaxDevices, "gemm: device %d out of range", dev);
  std::call_once(once[dev], [&] {
    set_rc[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kDynamic);
  });
  if (set_rc[dev] != cudaSuccess)
    return fail(AH_ECUDA, "gemm: cudaFuncSetAttribute: %s", cudaGetErrorString(set_rc[dev]));
  // programmatic dependent launch: the prologue (barriers, TMEM, the first
  // weight stages) overlaps the activation prep; A is read after pdl_wait()
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid_x, (unsigned)grid_y);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kDynamic;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AH_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return AH_OK;
}

inline int64_t gemm_halves(int64_t m) { return m > kTokTile ? 2 : 1; }
inline int64_t gemm_m_pad(int64_t m) {
  const int64_t tile = kTokTile * gemm_halves(m);
  return (m + tile - 1) / tile * tile;
}
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem, uint64_t inner,
              uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  auto fn = tensor_map_encoder();
  if (!fn) return fail(AH_ECUDA, "tensor map: cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner * elem};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AH_ECUDA, "tensor map: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AH_OK;
}

// Workspace: f16 activation tiles (M_pad x kp*64 x 2 B) + one f32 per padded row.
size_t gemm_workspace_bytes(const Q4Tiled& w, int64_t m) {
  const int64_t mp = gemm_m_pad(m);
  return align_up((size_t)mp * (size_t)w.kp * kBK * 2, 1024) + align_up((size_t)mp * 4, 256);
}

int gemm_run(const Q4Tiled& w, const float* a, int64_t lda, int64_t m, float* c, int64_t ldc, void* ws,
             size_t ws_bytes, cudaStream_t st, int epi, const uint16_t* norm_w, float eps) {
  AH_REQUIRE(m >= 0, "gemm: negative M");
  if (m == 0) return AH_OK;
  AH_REQUIRE(a != nullptr && c != nullptr && ws != nullptr, "gemm: null pointer");
  AH_REQUIRE(epi == kGemmEpiStore || epi == kGemmEpiSwiglu || epi == kGemmEpiAdd, "gemm: unknown epilogue %d", epi);
  AH_REQUIRE(epi != kGemmEpiSwiglu || w.rows % 16 == 0, "gemm: a SwiGLU epilogue needs whole 16-row tiles");
  AH_REQUIRE(lda >= w.cols && ldc >= (epi == kGemmEpiSwiglu ? w.rows / 2 : w.rows),
             "gemm: lda must be >= cols and ldc >= the output columns");
  AH_REQUIRE(ws_bytes >= gemm_workspace_bytes(w, m), "gemm: workspace of %zu bytes is below the %zu needed",
             ws_bytes, gemm_workspace_bytes(w, m));
  AH_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 1023) == 0, "gemm: workspace must be 1024-byte aligned");
  const int64_t mp = gemm_m_pad(m);
  uint8_t* at = static_cast<uint8_t*>(ws);
  float* row_inv = reinterpret_cast<float*>(at + align_up((size_t)mp * (size_t)w.kp * kBK * 2, 1024));
  const bool vec_rows = (lda % 4 == 0) && aligned16(a) && (w.cols % 8 == 0);
  // registers for as many chunks as a row needs (fewer registers: more CTAs
  // per SM hide the load latency of short rows)
  const int64_t per_thread = (w.kp * 8 + kPrepThreads - 1) / kPrepThreads;
  auto prep = per_thread <= 2 ? k_gemm_prep<2> : per_thread <= 4 ? k_gemm_prep<4> : k_gemm_prep<kPrepChunks>;
  prep<<<(unsigned)mp, kPrepThreads, 0, st>>>(a, lda, m, w.cols, w.kp, vec_rows, norm_w, eps, at, row_inv);
  AH_LAUNCH_CHECK();
  alignas(64) GemmArgs g{};
  g.w = w;
  g.at = at;
  g.row_inv = row_inv;
  g.c = c;
  g.ldc = ldc;
  g.m = m;
  g.err = device_error_word();
  g.epi = epi;
  g.c_vec = (ldc % 4 == 0) && aligned16(c);
  // weight planes as uint32 rows of 16-row tiles; activations as f16 rows
  int rc = encode_2d(&g.tm_nib, w.nib, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)w.kp * 128, (uint64_t)w.r16, 128,
                     kRowTiles, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != AH_OK) return rc;
  const uint32_t sc_u32 = w.f32_scales ? 32 : 16;  // per (row tile, pair)
  rc = encode_2d(&g.tm_scale, w.scales, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)w.kp * sc_u32, (uint64_t)w.r16,
                 sc_u32, kRowTiles, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != AH_OK) return rc;
  rc = encode_2d(&g.tm_a, at, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)w.kp * kBK, (uint64_t)mp, kBK, kTokTile,
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != AH_OK) return rc;
  const int64_t gx = (w.r16 + kRowTiles - 1) / kRowTiles;
  const int64_t halves = gemm_halves(m);
  const int64_t gy = mp / (kTokTile * halves);
  AH_REQUIRE(gy <= 65535, "gemm: M too large for one launch");
  if (halves == 2)
    return w.f32_scales ? gemm_launch<2, true>(g, gx, gy, st) : gemm_launch<2, false>(g, gx, gy, st);
  return w.f32_scales ? gemm_launch<1, true>(g, gx, gy, st) : gemm_launch<1, false>(g, gx, gy, st);
}

// ---- allocation-free variant ------------------------------------------------------
// ah_q4w_gemm_noalloc keeps its workspace in this fixed per-device buffer instead
// of a caller allocation.  Every byte the GEMM reads from it is written by the
// k_gemm_prep launch of the same call, so nothing needs clearing between calls;
// calls that overlap in time on one device race on it.
constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) uint8_t g_gemm_static_scratch[kStaticScratchBytes];

// Device address of g_gemm_static_scratch in the current device's context,
// looked up once per device.
int static_scratch(void** out) {
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  constexpr int kMaxDevices = 64;
  AH_REQUIRE(dev >= 0 && dev < kMaxDevices, "static scratch: device %d out of range", dev);
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(AH_ECUDA, "cudaGetSymbolAddress(g_gemm_static_scratch): %s", cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return AH_OK;
}

}  // namespace ah

extern "C" {

AH_API int ah_q4w_gemm_noalloc(const AhQ4Weight* w, const float* a_dev, int64_t lda, int64_t m, float* c_dev,
                               int64_t ldc, void* stream) {
  AH_REQUIRE(w != nullptr, "ah_q4w_gemm_noalloc: null weight");
  AH_REQUIRE(m >= 0, "ah_q4w_gemm_noalloc: negative M");
  if (m == 0) return AH_OK;
  const ah::Q4Tiled& t = ah::q4w_tiled(w);
  void* base = nullptr;
  const int rc = ah::static_scratch(&base);
  if (rc != AH_OK) return rc;
  // the GEMM wants a 1024-byte aligned workspace; the buffer is 256-aligned
  const uintptr_t b = reinterpret_cast<uintptr_t>(base);
  const uintptr_t al = (b + 1023) & ~uintptr_t(1023);
  const size_t usable = ah::kStaticScratchBytes - (size_t)(al - b);
  const size_t need = ah::gemm_workspace_bytes(t, m);
  AH_REQUIRE(need <= usable,
             "ah_q4w_gemm_noalloc: M=%lld x cols=%lld needs %zu scratch bytes; the static buffer holds %zu",
             (long long)m, (long long)t.cols, need, usable);
  return ah::gemm_run(t, a_dev, lda, m, c_dev, ldc, reinterpret_cast<void*>(al), usable, ah::as_stream(stream));
}

AH_API int ah_q4w_gemm_workspace_bytes(const AhQ4Weight* w, int64_t m, size_t* bytes) {
  AH_REQUIRE(w != nullptr && bytes != nullptr, "ah_q4w_gemm_workspace_bytes: null argument");
  AH_REQUIRE(m >= 0, "ah_q4w_gemm_workspace_bytes: negative M");
  *bytes = ah::gemm_workspace_bytes(ah::q4w_tiled(w), m);
  return AH_OK;
}

AH_API int ah_q4w_gemm(const AhQ4Weight* w, const float* a_dev, int64_t lda, int64_t m, float* c_dev, int64_t ldc,
                       void* workspace_dev, size_t workspace_bytes, void* stream) {
  AH_REQUIRE(w != nullptr, "ah_q4w_gemm: null weight");
  return ah::gemm_run(ah::q4w_tiled(w), a_dev, lda, m, c_dev, ldc, workspace_dev, workspace_bytes,
                      ah::as_stream(stream));
}

AH_API int ah_q4w_gemm_ex(const AhQ4Weight* w, const float* a_dev, int64_t lda, int64_t m, float* c_dev, int64_t ldc,
                          int epilogue, const uint16_t* norm_w_dev, float eps, void* workspace_dev,
                          size_t workspace_bytes, void* stream) {
  AH_REQUIRE(w != nullptr, "ah_q4w_gemm_ex: null weight");
  return ah::gemm_run(ah::q4w_tiled(w), a_dev, lda, m, c_dev, ldc, workspace_dev, workspace_bytes,
                      ah::as_stream(stream), epilogue, norm_w_dev, eps);
}

}  // extern "C"
