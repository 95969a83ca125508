// ah_bgemv_tc.cu — the batched decode GEMV (up to 16 tokens) on the 5th-
// generation tensor cores: weight rows are the MMA's M operand, read from
// tensor memory, and the tokens its N operand.
//
//   y[b][r] = sum_k W[r][k] * x[b][k],  W[r][k] = d(r, k/32) * (q(r,k) - 8)
//
// The mma.sync GEMV carries 16 tokens as 32 n8 columns (f16 hi + lo of x)
// and runs latency-bound near 1 TB/s.  Here a work unit is 128 weight rows (8
// row tiles of the tiled Q4 layout, ah_gemv.cuh) x 128 columns (two block
// pairs), a "step":
//
//   warp 0      raw weight producer: 2-D TMA boxes of the 8 tiles' nibbles and
//               scales per step into a 12-stage raw ring (~110 KB in flight)
//   warp 1      token producer: 2-D TMA of the 16 x 128 f16 token tile
//               (128-byte swizzle) into a 16-slot ring
//   warps 2, 15 TMEM owner (warp 2) and two MMA issuers taking alternate
//               steps: tcgen05.mma M=128 N=16 K=16 with A in tensor memory
//               (kind::f16, f32 accumulators, one per issuer)
//   warps 3..10 dequant d*(q-8) (one RNE rounding to f16) from the raw ring
//               into tensor memory with tcgen05.st.16x256b: that store's
//               register layout is the m16n8 fragment layout the tiled Q4
//               nibbles are stored in, so lane l's 16-byte nibble word of a
//               tile lands as-is (warps 3..6 take even steps, 7..10 odd ones)
//   warps 11..14 epilogue: tcgen05.ld 32x32b (thread = weight row, 16 token
//               columns), scale by 2^-s per token, store / add / SwiGLU /
//               peer stores
//
// Writing A to tensor memory instead of a shared-memory image keeps shared-
// memory traffic at ~11 KB per 9 KB of weights (raw ring in and out, tokens):
// a swizzled f16 image of A would add 32 KB per step and cap the kernel near
// 4 TB/s.  The dequant places the 64 values of a row and pair in the order
// the nibbles arrive (column 8*rep + 2t + e holds weight columns
// 32*(rep>>1) + 2t + {0,16,8,24}[2*(rep&1)+e] + {0,1}); the token prep writes
// x in the same order, so the MMA sums matching products.
//
// Work split (stream-K): the launch has G <= #SMs persistent CTAs; the
// T = row_blocks x steps_per_block steps are cut into G equal contiguous
// ranges.  A row block whose steps fall in one CTA's range is finished by
// that CTA's epilogue.  Otherwise each CTA writes its partial sums to a slot in
// global memory and bumps a per-(row block, lane quarter) counter; the warp
// that arrives last adds the partials in CTA order (so results do not depend
// on timing) and runs the epilogue.  The counters are zeroed by the prep
// kernel of every call.
//
// The tokens come from k_bgemv_prep: x (optionally RMSNorm'ed) per token
// scaled by an exact power of two into [2^14, 2^15) and rounded to f16, the
// precision of the prefill GEMM; the epilogue multiplies by 2^-s.
//
// Every mbarrier wait is bounded (AH_ETIMEOUT in the device error word); on
// give-up the kernel raises a CTA abort flag, drains its copies and MMAs,
// frees tensor memory and returns.
//
// Reference: the decode GEMVs of inference/mod.rs:411-538 (gemv_4bit_into,
// inference/math.rs:255-295) for each of the batch's tokens.
#include <algorithm>
#include <mutex>

#include "ah_common.cuh"
#include "ah_gemv_impl.cuh"
#include "ah_sm100.cuh"
#include "ah_tc.cuh"
#include "ah_tma.cuh"

#define AH_TRY_BG(expr)           \
  do {                            \
    int _rc = (expr);             \
    if (_rc != AH_OK) return _rc; \
  } while (0)

namespace ah {
namespace {

constexpr int kBgRowTiles = 8;                        // 16-row tiles per row block
constexpr int kBgM = kBgRowTiles * 16;                // 128 weight rows = MMA M = TMEM lanes
constexpr int kBgN = 16;                              // tokens = MMA N
constexpr int kBgPairs = 2;                           // block pairs (64 columns) per step
constexpr int kBgRawStages = 12;
constexpr int kBgAStages = 6;                         // TMEM A stages
// token ring: slots of 4 steps' tiles (one barrier wait and one commit per 4
// steps for the MMA thread), 16 steps deep -- at least as deep as the raw
// ring, so a step's token tile is requested no later than its weights (the
// TMA queue serves requests in order)
constexpr int kBgBGroup = 4;
constexpr int kBgBSlots = 4;
constexpr int kBgRawNib = kBgRowTiles * kBgPairs * 512;          // 8192
constexpr int kBgRawStride = kBgRawNib + kBgRowTiles * kBgPairs * 128;  // 10240 (f32 scales worst case)
constexpr int kBgBPair = kBgN * 64 * 2;               // 2048: 16 tokens x 64 f16
constexpr int kBgBStep = kBgPairs * kBgBPair;         // 4096: one step's token tile
constexpr int kBgBSlot = kBgBGroup * kBgBStep;        // 16384
constexpr uint32_t kBgTmemCols = 512;
// kBgIssuers MMA issuer threads (in different warps) take the steps in turn,
// each into its own accumulator (columns ((segment & 1) * kBgIssuers + t) * 16):
// an MMA issue blocks while the previous MMA runs (M=128, K=16: ~56 ns
// whatever N up to 128), so one issuer's barrier waits and bookkeeping would
// leave the tensor core idle; the other's MMAs fill those gaps.  The epilogue
// adds the accumulators.  Measured on the 70B gate/up (57344 x 8192, batch
// 16): one issuer 172 us, two 111 us, three 126 us, four 124 us.
constexpr int kBgIssuers = 2;
constexpr int kBgACol0 = 2 * kBgIssuers * kBgN;       // A stage a at columns kBgACol0 + 64a
constexpr int kBgACols = kBgPairs * 32;               // 64 columns per stage
static_assert(kBgACol0 + kBgAStages * kBgACols <= (int)kBgTmemCols, "TMEM budget");
static_assert(kBgRawStages % 2 == 0 && kBgAStages % 2 == 0, "stage parity selects the dequant group");
static_assert(kBgBGroup * kBgBSlots >= kBgRawStages, "token tiles are requested ahead of their weights");
static_assert((kBgBSlots & (kBgBSlots - 1)) == 0, "a power of two");
static_assert(kBgBGroup % kBgIssuers == 0, "every issuer takes the same number of steps of a token slot");
constexpr int kBgDequantWarp0 = 3;
constexpr int kBgEpiWarp0 = 11;
// issuer 0 is warp 2 (the TMEM owner), issuers 1.. are warps 15..
constexpr int kBgIssuerWarp1 = 15;
constexpr int kBgThreads = (kBgIssuerWarp1 + kBgIssuers - 1) * 32;
constexpr uint32_t kBgWait = 1u << 24;
constexpr uint32_t kBgIdesc = idesc_f16(kBgM, kBgN);
constexpr int kBgPrepThreads = 512;
constexpr int64_t kBgPrepStageMaxK = 50176;           // f32 row staging: 196 KB of shared memory

struct BgSmem {
  static constexpr int kRaw = 0;
  static constexpr int kB = kRaw + kBgRawStages * kBgRawStride;
  static constexpr int kBars = kB + kBgBSlots * kBgBSlot;
  // raw_full, raw_empty, a_full, a_empty, b_full, b_empty, acc_full[2], acc_empty[2], mma_done
  static constexpr int kNumBars = 2 * kBgRawStages + 2 * kBgAStages + 2 * kBgBSlots + 5;
  static constexpr int kMisc = kBars + kNumBars * 8;
  static constexpr int kTotal = kMisc + 16;
  static constexpr size_t kDynamic = (size_t)kTotal + 1024;  // slack for the 1 KB alignment
  static_assert(kB % 1024 == 0, "B slots need 1 KB alignment for the 128-byte swizzle");
};

struct BgArgs {
  CUtensorMap tm_nib;    // nibble plane as uint32 [r16][kp*128], box 256 x 8
  CUtensorMap tm_scale;  // scale plane as uint32 [r16][kp*16|32], box 32|64 x 8
  CUtensorMap tm_x;      // tokens f16 [16][kp*64] (pair-permuted), box 64 x 16, 128-byte swizzle
  GemvArgs g;            // weight, y, epilogue operands (x is read by the prep kernel)
  const float* row_inv;  // [16] 2^-s per token
  float* partial;        // [G][2][128][16] stream-K partial sums
  int* counter;          // [row blocks][4] arrivals per (row block, lane quarter)
  int64_t steps;         // steps per row block = ceil(kp / 2)
  int64_t total;         // row blocks x steps
};

// Weight column (within a 64-column block pair) of the MMA's k index km: the
// order in which k_bgemv_tc's dequant places a row's values in tensor memory.
__host__ __device__ __forceinline__ int bg_kperm(int km) {
  const int rep = km >> 4, t = (km >> 2) & 3, e = (km >> 1) & 1, s = km & 1;
  const int j = 2 * (rep & 1) + e;
  return 32 * (rep >> 1) + 2 * t + 16 * (j & 1) + 8 * (j >> 1) + s;
}

// ---- token prep: f32 rows (optionally RMSNorm'ed) -> scaled, pair-permuted f16 ----
// grid 16 (one CTA per token row; rows past the batch are zero).  Also zeroes
// the stream-K counters of the GEMV that follows.  kStage: the row is read once
// (16-byte loads, several in flight per thread), normalised into shared memory
// as f32, and the permuted f16 tiles are written from there; rows longer than
// kBgPrepStageMaxK are read twice from global memory instead.  The GEMV's MMAs
// wait for this grid, so its latency is on every decode GEMV's critical path
// (the first, scalar version took ~12 us per call at K = 8192).
template <int PRO, bool kStage>
__global__ void __launch_bounds__(kBgPrepThreads) k_bgemv_prep(const GemvArgs a, int64_t kp, uint8_t* __restrict__ xt,
                                                                float* __restrict__ row_inv, int* __restrict__ counter,
                                                                int n_counter) {
  // the GEMV may start its prologue and weight loads; it waits for this grid
  pdl_launch_dependents();
  // x, the sums of squares, xt and the counters belong to earlier kernels
  pdl_wait();
  extern __shared__ float stage[];  // kStage: [kp * 64] normalised row
  const int b = blockIdx.x, tid = threadIdx.x;
  for (int i = b * kBgPrepThreads + tid; i < n_counter; i += kBgN * kBgPrepThreads) counter[i] = 0;
  const bool live = b < a.batch;
  const int64_t K = a.w.cols, kpad = kp * 64;
  const float* row = a.x + (live ? b : 0) * a.x_stride;
  __shared__ float red[kBgPrepThreads / 32];
  __shared__ float s_inv;
  float inv = 1.0f;
  if (PRO == kProRmsNorm) {
    // 1/rms from the producer's partial sums of squares (inference/math.rs:53-63)
    float ss = 0.0f;
    if (live)
      for (int i = tid; i < a.n_ss_in; i += kBgPrepThreads) ss += a.ss_in[b * a.n_ss_in + i];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int w = 0; w < kBgPrepThreads / 32; ++w) t += red[w];
      s_inv = __fdiv_rn(1.0f, sqrtf(__fdiv_rn(t, (float)K) + a.eps));  // inference/math.rs:59
    }
    __syncthreads();
    inv = s_inv;
  }
  auto xv = [&](int64_t k) -> float {
    if (!live || k >= K) return 0.0f;
    float v = row[k];
    if (PRO == kProRmsNorm) v = (v * inv) * __half2float(__ushort_as_half(a.norm_w[k]));
    return v;
  };
  float amax = 0.0f;
  if (kStage) {
    const bool vec = live && (reinterpret_cast<uintptr_t>(row) & 15) == 0 && (K & 3) == 0 &&
                     (PRO != kProRmsNorm || (reinterpret_cast<uintptr_t>(a.norm_w) & 7) == 0);
    if (vec) {
      float4* st4 = reinterpret_cast<float4*>(stage);
#pragma unroll 4
      for (int64_t c = tid; c < kpad / 4; c += kBgPrepThreads) {
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c * 4 < K) {
          v = __ldg(reinterpret_cast<const float4*>(row) + c);
          if (PRO == kProRmsNorm) {
            const uint2 nw = __ldg(reinterpret_cast<const uint2*>(a.norm_w) + c);
            v.x = (v.x * inv) * __half2float(__ushort_as_half((unsigned short)(nw.x & 0xFFFFu)));
            v.y = (v.y * inv) * __half2float(__ushort_as_half((unsigned short)(nw.x >> 16)));
            v.z = (v.z * inv) * __half2float(__ushort_as_half((unsigned short)(nw.y & 0xFFFFu)));
            v.w = (v.w * inv) * __half2float(__ushort_as_half((unsigned short)(nw.y >> 16)));
          }
        }
        amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
        st4[c] = v;
      }
    } else {
#pragma unroll 4
      for (int64_t k = tid; k < kpad; k += kBgPrepThreads) {
        const float v = xv(k);
        amax = fmaxf(amax, fabsf(v));
        stage[k] = v;
      }
    }
  } else {
    for (int64_t k = tid; k < K; k += kBgPrepThreads) amax = fmaxf(amax, fabsf(xv(k)));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  __syncthreads();  // red[] is reused; the staged row is complete
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < kBgPrepThreads / 32; ++i) amax = fmaxf(amax, red[i]);
  // exponent s with amax * 2^s in [2^14, 2^15), clamped so 2^s and 2^-s are
  // normal floats; zero rows and non-finite maxima keep s = 0
  int s = 0;
  const uint32_t ab = __float_as_uint(amax);
  if (amax > 0.0f && ((ab >> 23) & 0xFF) != 0xFF) {
    const int e = (int)((ab >> 23) & 0xFF) - 126;  // amax in [2^(e-1), 2^e)
    s = min(max(15 - e, -120), 120);
  }
  const float scale = __uint_as_float((uint32_t)(127 + s) << 23);
  if (tid == 0) row_inv[b] = live ? __uint_as_float((uint32_t)(127 - s) << 23) : 0.0f;
  // 8 MMA-order columns (16 bytes) per chunk; a pair holds 8 chunks
  uint4* out = reinterpret_cast<uint4*>(xt + (size_t)b * (size_t)kp * 128);
  for (int64_t c = tid; c < kp * 8; c += kBgPrepThreads) {
    const int64_t base = (c >> 3) * 64;
    const int km0 = (int)(c & 7) * 8;
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t k0 = base + bg_kperm(km0 + 2 * i), k1 = base + bg_kperm(km0 + 2 * i + 1);
      const float v0 = kStage ? stage[k0] : xv(k0), v1 = kStage ? stage[k1] : xv(k1);
      const __half2 v = __floats2half2_rn(v0 * scale, v1 * scale);
      h[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
    out[c] = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

__device__ __forceinline__ bool bg_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  if (mbar_wait_bounded(bar, parity, err, AH_ETIMEOUT, kBgWait)) return true;
  *abort_flag = 1;
  return false;
}

// Wait with a short sleep after each failed poll, for the producers and the
// dequant warps: their spinning would take issue slots and barrier-unit cycles
// from the MMA issuers sharing their SM sub-partitions.
__device__ __forceinline__ bool bg_wait_nap(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  for (uint32_t it = 0; it < (kBgWait >> 2); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(32);
  }
  if (err) atomicExch(err, AH_ETIMEOUT);
  *abort_flag = 1;
  return false;
}

// The same with a short sleep between polls, for waits that span many steps.
__device__ __forceinline__ bool bg_wait_idle(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  for (uint32_t it = 0; it < (kBgWait >> 4); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(200);
  }
  if (err) atomicExch(err, AH_ETIMEOUT);
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ float silu_bg(float x) {  // inference/math.rs:83-95
  const float sg = x >= 0.0f ? __fdiv_rn(1.0f, 1.0f + expf(-x)) : __fdiv_rn(expf(x), 1.0f + expf(x));
  return x * sg;
}

// CTA whose step range holds global step s (ranges [c*T/G, (c+1)*T/G), G <= T).
__device__ __forceinline__ int64_t bg_owner(int64_t s, int64_t G, int64_t T) { return ((s + 1) * G - 1) / T; }

// Epilogue of one weight row (thread) and its 16 token sums v (unscaled):
// row rb*128 + 32q + lane, 16-row tile rb*8 + 2q + lane/16.
template <int EPI>
__device__ __forceinline__ void bg_epilogue(const GemvArgs& g, int64_t rb, int q, int lane, float (&v)[16],
                                            const float (&inv)[16]) {
  const int64_t R = rb * kBgM + q * 32 + lane;
  const int64_t rt = rb * kBgRowTiles + q * 2 + (lane >> 4);
  const int B = g.batch;
#pragma unroll
  for (int b = 0; b < kBgN; ++b) v[b] *= inv[b];
  if (EPI == kEpiSwiglu) {
    // lanes 0-7 of each 16 carry a tile's gate rows, lanes 8-15 the matching
    // up rows (inference/ffn.rs:155-174)
    const int r = lane & 15;
#pragma unroll
    for (int b = 0; b < kBgN; ++b) {
      const float u = __shfl_down_sync(0xFFFFFFFFu, v[b], 8);
      if (r < 8 && b < B) {
        const int64_t o = rt * 8 + r;
        if (o < g.w.rows / 2) g.y[b * g.y_stride + o] = silu_bg(v[b]) * u;
      }
    }
    return;
  }
  const bool live = R < g.w.rows;
  float h[kBgN];
  if (EPI == kEpiStore && g.n_peer > 0) {
    // tensor-parallel scatter: rows of peer_row floats, tokens contiguous
#pragma unroll
    for (int b = 0; b < kBgN; ++b) h[b] = (live && b < B) ? v[b] : 0.0f;
    if (live)
      for (int pr = 0; pr < g.n_peer; ++pr) {
        float* d = g.peer_y[pr] + R * g.peer_row;
#pragma unroll
        for (int b = 0; b < kBgN; ++b)
          if (b < B) d[b] = h[b];  // NVLink stores
      }
  } else {
#pragma unroll
    for (int b = 0; b < kBgN; ++b) {
      h[b] = 0.0f;
      if (live && b < B) {
        float* d = g.y + b * g.y_stride + R;
        h[b] = (EPI == kEpiAdd) ? *d + v[b] : v[b];  // residual: hidden[i] += out[i]
        *d = h[b];
      }
    }
  }
  if (g.ss_out) {
    // per-tile sums of squares of the values written (the next RMSNorm's input)
#pragma unroll
    for (int b = 0; b < kBgN; ++b) {
      float sq = h[b] * h[b];
#pragma unroll
      for (int o = 8; o; o >>= 1) sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
      if ((lane & 15) == 0 && b < B && rt < g.w.r16) g.ss_out[b * g.w.r16 + rt] = sq;
    }
  }
}

// Stream-K fixup of a row block that several CTAs share: this CTA's partial
// sums go to its slot; the warp that arrives last for (rb, q) adds every
// slot in CTA order and runs the epilogue.
template <int EPI>
__device__ __forceinline__ void bg_fixup(const BgArgs& p, int64_t rb, int q, int lane, const float (&v)[16],
                                      const float (&inv)[16], int64_t c, int64_t G) {
  const int64_t T = p.total, S = p.steps;
  const int slot = (c * T / G) / S == rb ? 0 : 1;  // the CTA's first row block, or its last
  float4* mine = reinterpret_cast<float4*>(p.partial + ((c * 2 + slot) * kBgM + q * 32 + lane) * kBgN);
#pragma unroll
  for (int i = 0; i < 4; ++i) __stcg(mine + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
  __threadfence();
  __syncwarp();
  const int64_t c0 = bg_owner(rb * S, G, T), c1 = bg_owner(rb * S + S - 1, G, T);
  int old = 0;
  if (lane == 0) old = atom_add_acq_rel_gpu(&p.counter[rb * 4 + q], 1);
  old = __shfl_sync(0xFFFFFFFFu, old, 0);
  if (old != (int)(c1 - c0)) return;  // another CTA's segment of this row block is still running
  __threadfence();
  float acc[kBgN];
#pragma unroll
  for (int b = 0; b < kBgN; ++b) acc[b] = 0.0f;
  for (int64_t cc = c0; cc <= c1; ++cc) {
    const int sl = (cc * T / G) / S == rb ? 0 : 1;
    const float4* src = reinterpret_cast<const float4*>(p.partial + ((cc * 2 + sl) * kBgM + q * 32 + lane) * kBgN);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 t = __ldcg(src + i);
      acc[4 * i] += t.x;
      acc[4 * i + 1] += t.y;
      acc[4 * i + 2] += t.z;
      acc[4 * i + 3] += t.w;
    }
  }
  bg_epilogue<EPI>(p.g, rb, q, lane, acc, inv);
}

// ---- the GEMV ------------------------------------------------------------------------
template <int EPI, bool kF32>
__global__ void __launch_bounds__(kBgThreads, 1) k_bgemv_tc(const __grid_constant__ BgArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BgSmem::kBars);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + kBgRawStages;
  uint64_t* a_full = raw_empty + kBgRawStages;
  uint64_t* a_empty = a_full + kBgAStages;
  uint64_t* b_full = a_empty + kBgAStages;
  uint64_t* b_empty = b_full + kBgBSlots;
  uint64_t* acc_full = b_empty + kBgBSlots;  // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BgSmem::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + BgSmem::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const GemvArgs& g = p.g;
  int* err = g.err;
  const int64_t G = gridDim.x, T = p.total, S = p.steps;
  const int64_t c = blockIdx.x;
  const int64_t start = c * T / G;
  const int n = (int)((c + 1) * T / G - start);  // >= 1: the host keeps G <= T
  constexpr int kScBytes = kF32 ? 128 : 64;       // scales per (row tile, pair)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBgRawStages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 4);  // the four dequant warps of the stage's parity
    }
    for (int i = 0; i < kBgAStages; ++i) {
      mbar_init(&a_full[i], 4);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kBgBSlots; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], kBgIssuers);  // each issuer commits after its last step of the slot
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], kBgIssuers);
      mbar_init(&acc_empty[i], 4);  // the four epilogue warps
    }
    mbar_init(mma_done, kBgIssuers);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, kBgTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- raw weight producer: one nibble box + one scale box per step ----
    if (lane == 0) {
      // full boxes; rows and columns past the matrix arrive zero-filled
      constexpr uint32_t kTx = kBgRowTiles * kBgPairs * (512 + kScBytes);
      int issued = 0;
      int64_t rb = start / S, ks = start - rb * S;
      for (int i = 0; i < n; ++i) {
        const int r = i % kBgRawStages;
        if (*abort_flag) break;
        if (i >= kBgRawStages && !bg_wait_nap(&raw_empty[r], (uint32_t)((i / kBgRawStages - 1) & 1), err, abort_flag))
          break;
        uint8_t* dst = smem + BgSmem::kRaw + r * kBgRawStride;
        mbar_arrive_expect_tx(&raw_full[r], kTx);
        tma_load_2d(dst, &p.tm_nib, (int)(ks * kBgPairs * 128), (int)(rb * kBgRowTiles), &raw_full[r]);
        tma_load_2d(dst + kBgRawNib, &p.tm_scale, (int)(ks * kBgPairs * (kScBytes / 4)), (int)(rb * kBgRowTiles),
                    &raw_full[r]);
        ++issued;
        if (++ks == S) {
          ks = 0;
          ++rb;
        }
      }
      // every weight load is issued: the next kernel's CTAs may take SMs as this grid's retire
      pdl_launch_dependents();
      if (*abort_flag)
        for (int i = issued > kBgRawStages ? issued - kBgRawStages : 0; i < issued; ++i)
          mbar_wait_bounded(&raw_full[i % kBgRawStages], (uint32_t)((i / kBgRawStages) & 1), err, AH_ETIMEOUT,
                            kBgWait);
    }
  } else if (warp == 1) {
    // ---- token producer: slot g holds the tiles of steps 4g .. 4g+3 ----
    if (lane == 0) {
      pdl_wait();  // the token tiles come from the preceding prep grid
      const int ng = (n + kBgBGroup - 1) / kBgBGroup;
      int64_t ks = start % S;
      int issued = 0;
      for (int gi = 0; gi < ng; ++gi) {
        const int bs = gi & (kBgBSlots - 1);
        if (*abort_flag) break;
        if (gi >= kBgBSlots && !bg_wait_nap(&b_empty[bs], (uint32_t)((gi / kBgBSlots - 1) & 1), err, abort_flag))
          break;
        const int cnt = n - gi * kBgBGroup < kBgBGroup ? n - gi * kBgBGroup : kBgBGroup;
        uint8_t* dst = smem + BgSmem::kB + bs * kBgBSlot;
        mbar_arrive_expect_tx(&b_full[bs], (uint32_t)(cnt * kBgBStep));
        for (int j = 0; j < cnt; ++j) {
          tma_load_2d(dst + j * kBgBStep, &p.tm_x, (int)(ks * kBgPairs * 64), 0, &b_full[bs]);
          tma_load_2d(dst + j * kBgBStep + kBgBPair, &p.tm_x, (int)(ks * kBgPairs * 64 + 64), 0, &b_full[bs]);
          if (++ks == S) ks = 0;
        }
        ++issued;
      }
      if (*abort_flag)
        for (int gi = issued > kBgBSlots ? issued - kBgBSlots : 0; gi < issued; ++gi)
          mbar_wait_bounded(&b_full[gi & (kBgBSlots - 1)], (uint32_t)((gi / kBgBSlots) & 1), err, AH_ETIMEOUT,
                            kBgWait);
    }
  } else if (warp == 2 || warp >= kBgIssuerWarp1) {
    // ---- MMA issuers: issuer t takes the steps i with i % kBgIssuers == t ----
    if (lane == 0) {
      const int t = warp == 2 ? 0 : warp - kBgIssuerWarp1 + 1;
      const uint64_t bdesc0 = sw128_desc(smem_u32(smem + BgSmem::kB));
      int64_t ks0 = start % S;
      bool ok = true;
      for (int i0 = 0, seg = 0; ok && i0 < n; ++seg) {
        const int len = (int)(S - ks0 < (int64_t)(n - i0) ? S - ks0 : (int64_t)(n - i0));
        // the epilogue has read this accumulator buffer's previous segment
        if (seg >= 2 && !bg_wait(&acc_empty[seg & 1], (uint32_t)(((seg >> 1) - 1) & 1), err, abort_flag)) break;
        const uint32_t acc = tmem + (uint32_t)(((seg & 1) * kBgIssuers + t) * kBgN);
        bool first = true;
        for (int i = i0 + (t - i0 % kBgIssuers + kBgIssuers) % kBgIssuers; i < i0 + len; i += kBgIssuers) {
          const int a = i % kBgAStages;
          const int gi = i / kBgBGroup, bs = gi & (kBgBSlots - 1);
          // another role's give-up also shows as this thread's own bounded wait failing
          if ((i & 15) < kBgIssuers && *abort_flag) {
            ok = false;
            break;
          }
          // the slot's token tiles: waited for at this issuer's first step of the slot
          if (i % kBgBGroup < kBgIssuers && !bg_wait(&b_full[bs], (uint32_t)((gi / kBgBSlots) & 1), err, abort_flag)) {
            ok = false;
            break;
          }
          if (!bg_wait(&a_full[a], (uint32_t)((i / kBgAStages) & 1), err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ta = tmem + (uint32_t)(kBgACol0 + a * kBgACols);
          // descriptor start addresses count 16-byte units
          const uint64_t bd = bdesc0 + (uint64_t)((bs * kBgBSlot + (i % kBgBGroup) * kBgBStep) >> 4);
#pragma unroll
          for (int m = 0; m < kBgPairs * 4; ++m)
            mma_f16_ts(acc, ta + (uint32_t)((m >> 2) * 32 + (m & 3) * 8),
                       bd + (uint64_t)(((m >> 2) * kBgBPair + (m & 3) * 32) >> 4), kBgIdesc,
                       (!first || m > 0) ? 1u : 0u);
          first = false;
          mma_commit(&a_empty[a]);
          // this issuer's last step of the slot (or of the CTA's range)
          if (i % kBgBGroup == kBgBGroup - kBgIssuers + t || i + kBgIssuers >= n) mma_commit(&b_empty[bs]);
        }
        // arrives once this issuer's MMAs of the segment are done (at once if it had none)
        mma_commit(&acc_full[seg & 1]);
        i0 += len;
        ks0 = 0;
      }
      // completes when every MMA above has (also on abort, so TMEM can be freed)
      mma_commit(mma_done);
    }
  } else if (warp < kBgEpiWarp0) {
    // ---- dequant: raw ring -> f16 A stages in tensor memory ----
    // warp w writes TMEM lanes 32*(w%4) .. +31: row tiles 2q and 2q+1 of the block
    const int q = warp & 3;
    const int grp = (warp - kBgDequantWarp0) >> 2;  // 0: even steps, 1: odd steps
    const int gq = lane >> 2;
    for (int i = grp; i < n; i += 2) {
      const int r = i % kBgRawStages, a = i % kBgAStages;
      bool ok = true;
      if (lane == 0) {
        if (*abort_flag) {
          ok = false;
        } else {
          ok = bg_wait_nap(&raw_full[r], (uint32_t)((i / kBgRawStages) & 1), err, abort_flag);
          // the MMAs that read this A stage last time have completed
          if (ok && i >= kBgAStages)
            ok = bg_wait_nap(&a_empty[a], (uint32_t)((i / kBgAStages - 1) & 1), err, abort_flag);
        }
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      const uint8_t* raw = smem + BgSmem::kRaw + r * kBgRawStride;
#pragma unroll
      for (int ti = 0; ti < 2; ++ti) {
        const int tile = 2 * q + ti;
#pragma unroll
        for (int pp = 0; pp < kBgPairs; ++pp) {
          const uint4 nv = *reinterpret_cast<const uint4*>(raw + tile * (kBgPairs * 512) + pp * 512 + lane * 16);
          const uint32_t wv[4] = {nv.x, nv.y, nv.z, nv.w};  // word wi = 2*blk + h: row gq + 8h, block blk
          const uint8_t* sc = raw + kBgRawNib + tile * (kBgPairs * kScBytes) + pp * kScBytes;
          float dsc[4];
          __half dh[4];
          if (kF32) {
            const float4 d4 = *reinterpret_cast<const float4*>(sc + gq * 16);
            dsc[0] = d4.x; dsc[1] = d4.y; dsc[2] = d4.z; dsc[3] = d4.w;
          } else {
            const uint2 d2 = *reinterpret_cast<const uint2*>(sc + gq * 8);
            dh[0] = __ushort_as_half((unsigned short)(d2.x & 0xFFFFu));
            dh[1] = __ushort_as_half((unsigned short)(d2.x >> 16));
            dh[2] = __ushort_as_half((unsigned short)(d2.y & 0xFFFFu));
            dh[3] = __ushort_as_half((unsigned short)(d2.y >> 16));
          }
          uint32_t rg[16];
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const int blk = wi >> 1, h = wi & 1;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // nibbles j and j+4 of the word are block elements 2t+off and
              // 2t+off+1, off = {0,16,8,24}[j]; 1024+q is exact in f16
              const uint32_t bits = ((wv[wi] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
              const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&bits), __float2half2_rn(1032.0f));
              __half2 v;
              if (kF32) {
                const float2 qf = __half22float2(qv);
                v = __floats2half2_rn(qf.x * dsc[wi], qf.y * dsc[wi]);
              } else {
                v = __hmul2(qv, __half2half2(dh[wi]));
              }
              // register 4*rep + 2h + e -> lane gq + 8h, column 8*rep + 2t + e
              rg[4 * (2 * blk + (j >> 1)) + 2 * h + (j & 1)] = *reinterpret_cast<const uint32_t*>(&v);
            }
          }
          tmem_st16x256_x4(tmem + ((uint32_t)(32 * q + 16 * ti) << 16) + (uint32_t)(kBgACol0 + a * kBgACols + pp * 32),
                           rg);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[r]);
        mbar_arrive(&a_full[a]);
      }
    }
  } else if (warp < kBgEpiWarp0 + 4) {
    // ---- epilogue: accumulator -> outputs (or a stream-K partial) ----
    const int q = warp & 3;
    pdl_wait();  // row_inv, the counters and y follow the preceding grids
    float inv[kBgN];
#pragma unroll
    for (int b = 0; b < kBgN; ++b) inv[b] = p.row_inv[b];
    int seg = 0;
    for (int i = 0; i < n; ++seg) {
      const int64_t s = start + i, rb = s / S, ks = s - rb * S;
      const int len = (int)(S - ks < (int64_t)(n - i) ? S - ks : (int64_t)(n - i));
      bool ok = true;
      // a long wait (a whole segment of MMAs): poll with back-off so the
      // MMA thread and the dequant warps keep the issue slots
      if (lane == 0) ok = !*abort_flag && bg_wait_idle(&acc_full[seg & 1], (uint32_t)((seg >> 1) & 1), err, abort_flag);
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      // issuer t has a step in the segment [i, i + len) iff (t - i) mod
      // kBgIssuers < len; the accumulators are added in issuer order
      float v[kBgN];
#pragma unroll
      for (int b = 0; b < kBgN; ++b) v[b] = 0.0f;
      const uint32_t tacc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((seg & 1) * kBgIssuers * kBgN);
#pragma unroll
      for (int t = 0; t < kBgIssuers; ++t) {
        if ((t - i % kBgIssuers + kBgIssuers) % kBgIssuers >= len) continue;  // warp-uniform
        float w[kBgN];
        tmem_ld16(tacc + (uint32_t)(t * kBgN), w);
#pragma unroll
        for (int b = 0; b < kBgN; ++b) v[b] += w[b];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[seg & 1]);
      if (ks == 0 && len == S)
        bg_epilogue<EPI>(g, rb, q, lane, v, inv);
      else
        bg_fixup<EPI>(p, rb, q, lane, v, inv, c, G);
      i += len;
    }
    // peer slots: the stores reach the other GPUs before this grid completes
    if (EPI == kEpiStore && g.n_peer > 0) __threadfence_system();
  }

  // teardown: every MMA has completed before tensor memory is released
  if (warp == 2 && lane == 0) mbar_wait_bounded(mma_done, 0, err, AH_ETIMEOUT, kBgWait);
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kBgTmemCols);
  }
}

inline size_t bg_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace: pair-permuted f16 tokens [16][kp*64], 2^-s per token, the
// stream-K partial slots of up to #SMs CTAs, and the (row block, quarter)
// counters.
struct BgLayout {
  size_t row_inv, partial, counter, total;
  int n_counter;
};
BgLayout bg_layout(const Q4Tiled& w) {
  BgLayout L{};
  const int64_t nb = (w.r16 + kBgRowTiles - 1) / kBgRowTiles;
  L.row_inv = bg_align((size_t)kBgN * (size_t)w.kp * 128, 256);
  L.partial = L.row_inv + 256;
  L.counter = bg_align(L.partial + (size_t)sm_count() * 2 * kBgM * kBgN * 4, 256);
  L.n_counter = (int)(nb * 4);
  L.total = bg_align(L.counter + (size_t)L.n_counter * 4, 1024);
  return L;
}

template <int EPI, bool kF32>
int bg_attr() {
  // the shared-memory cap is set once per device, race-free across host threads
  constexpr int kMaxDevices = 64;
  static std::once_flag once[kMaxDevices];
  static cudaError_t set_rc[kMaxDevices];
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  AH_REQUIRE(dev >= 0 && dev < kMaxDevices, "bgemv: device %d out of range", dev);
  std::call_once(once[dev], [&] {
    set_rc[dev] = cudaFuncSetAttribute(k_bgemv_tc<EPI, kF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)BgSmem::kDynamic);
  });
  if (set_rc[dev] != cudaSuccess)
    return fail(AH_ECUDA, "bgemv: cudaFuncSetAttribute: %s", cudaGetErrorString(set_rc[dev]));
  return AH_OK;
}

template <int EPI>
int bg_attr_epi(bool f32) {
  return f32 ? bg_attr<EPI, true>() : bg_attr<EPI, false>();
}

// The staged prep kernels' shared-memory cap (the row as f32), once per device.
int bg_prep_attr() {
  constexpr int kMaxDevices = 64;
  static std::once_flag once[kMaxDevices];
  static cudaError_t set_rc[kMaxDevices];
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  AH_REQUIRE(dev >= 0 && dev < kMaxDevices, "bgemv: device %d out of range", dev);
  std::call_once(once[dev], [&] {
    const int bytes = (int)(kBgPrepStageMaxK * 4);
    set_rc[dev] = cudaFuncSetAttribute(k_bgemv_prep<kProPlain, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (set_rc[dev] == cudaSuccess)
      set_rc[dev] =
          cudaFuncSetAttribute(k_bgemv_prep<kProRmsNorm, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  if (set_rc[dev] != cudaSuccess)
    return fail(AH_ECUDA, "bgemv: prep cudaFuncSetAttribute: %s", cudaGetErrorString(set_rc[dev]));
  return AH_OK;
}

int bg_attr_any(int epi, bool f32) {
  AH_TRY_BG(bg_prep_attr());
  if (epi == kEpiStore) return bg_attr_epi<kEpiStore>(f32);
  if (epi == kEpiAdd) return bg_attr_epi<kEpiAdd>(f32);
  return bg_attr_epi<kEpiSwiglu>(f32);
}

int launch_ex(const void* kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, void** params) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AH_CUDA_TRY(cudaLaunchKernelExC(&cfg, kern, params));
  return AH_OK;
}

}  // namespace

size_t bgemv_workspace_bytes(const Q4Tiled& w) { return bg_layout(w).total; }

int bgemv_prepare(const Q4Tiled& w, int epi) { return bg_attr_any(epi, w.f32_scales); }

int bgemv_launch(const GemvArgs& a, int pro, int epi, void* ws, size_t ws_bytes, cudaStream_t st, bool pdl) {
  AH_REQUIRE(a.batch >= 1 && a.batch <= kBgN, "bgemv: batch must be 1..16");
  AH_REQUIRE(a.x != nullptr && a.y != nullptr && ws != nullptr, "bgemv: null pointer");
  AH_REQUIRE(pro != kProRmsNorm || (a.norm_w != nullptr && a.ss_in != nullptr && a.n_ss_in > 0),
             "bgemv: RMSNorm prologue needs a norm weight and the producer's partial sums of squares");
  AH_REQUIRE(epi != kEpiSwiglu || a.w.rows % 16 == 0, "bgemv: SwiGLU epilogue needs interleaved rows %% 16 == 0");
  AH_REQUIRE(epi == kEpiStore || a.n_peer == 0, "bgemv: the peer scatter is a store epilogue");
  AH_REQUIRE(a.pair_end == 0, "bgemv: K windows are a mma.sync GEMV plan");
  AH_REQUIRE(a.w.kp * kBgPairs * 128 < (int64_t)INT32_MAX && a.w.r16 < (int64_t)INT32_MAX,
             "bgemv: weight too large for 32-bit TMA coordinates");
  const BgLayout L = bg_layout(a.w);
  AH_REQUIRE(ws_bytes >= L.total, "bgemv: workspace of %zu bytes is below the %zu needed", ws_bytes, L.total);
  AH_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 1023) == 0, "bgemv: workspace must be 1024-byte aligned");
  AH_TRY_BG(bg_attr_any(epi, a.w.f32_scales));
  uint8_t* base = static_cast<uint8_t*>(ws);
  uint8_t* xt = base;
  float* row_inv = reinterpret_cast<float*>(base + L.row_inv);
  int* counter = reinterpret_cast<int*>(base + L.counter);

  GemvArgs g = a;
  g.err = device_error_word();
  AH_REQUIRE(g.err != nullptr, "bgemv: device error word unavailable");
  int64_t kp = a.w.kp;
  int n_counter = L.n_counter;
  void* prep_params[] = {&g, &kp, &xt, &row_inv, &counter, &n_counter};
  const bool stage = kp * 64 <= kBgPrepStageMaxK;
  const void* prep =
      pro == kProRmsNorm
          ? (stage ? reinterpret_cast<const void*>(k_bgemv_prep<kProRmsNorm, true>)
                   : reinterpret_cast<const void*>(k_bgemv_prep<kProRmsNorm, false>))
          : (stage ? reinterpret_cast<const void*>(k_bgemv_prep<kProPlain, true>)
                   : reinterpret_cast<const void*>(k_bgemv_prep<kProPlain, false>));
  const size_t prep_smem = stage ? (size_t)kp * 64 * 4 : 0;
  if (inject_failure(AH_INJECT_LAUNCH)) return fail(AH_ECUDA, "bgemv: kernel launch failed (injected)");
  AH_TRY_BG(launch_ex(prep, dim3(kBgN), dim3(kBgPrepThreads), prep_smem, st, pdl, prep_params));

  alignas(64) BgArgs p{};
  p.g = g;
  p.row_inv = row_inv;
  p.partial = reinterpret_cast<float*>(base + L.partial);
  p.counter = counter;
  const int64_t nb = (a.w.r16 + kBgRowTiles - 1) / kBgRowTiles;
  p.steps = (a.w.kp + kBgPairs - 1) / kBgPairs;
  p.total = nb * p.steps;
  // weight planes as uint32 rows of 16-row tiles; tokens as f16 rows
  AH_TRY_BG(encode_2d(&p.tm_nib, a.w.nib, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)a.w.kp * 128,
                   (uint64_t)a.w.r16, kBgPairs * 128, kBgRowTiles, CU_TENSOR_MAP_SWIZZLE_NONE));
  const uint32_t sc_u32 = a.w.f32_scales ? 32 : 16;  // per (row tile, pair)
  AH_TRY_BG(encode_2d(&p.tm_scale, a.w.scales, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)a.w.kp * sc_u32,
                   (uint64_t)a.w.r16, kBgPairs * sc_u32, kBgRowTiles, CU_TENSOR_MAP_SWIZZLE_NONE));
  AH_TRY_BG(encode_2d(&p.tm_x, xt, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)a.w.kp * 64, kBgN, 64, kBgN,
                   CU_TENSOR_MAP_SWIZZLE_128B));
  const int64_t G = std::min<int64_t>(sm_count(), p.total);
  const void* kern = nullptr;
  const bool f32 = a.w.f32_scales;
  if (epi == kEpiStore)
    kern = f32 ? (const void*)k_bgemv_tc<kEpiStore, true> : (const void*)k_bgemv_tc<kEpiStore, false>;
  else if (epi == kEpiAdd)
    kern = f32 ? (const void*)k_bgemv_tc<kEpiAdd, true> : (const void*)k_bgemv_tc<kEpiAdd, false>;
  else
    kern = f32 ? (const void*)k_bgemv_tc<kEpiSwiglu, true> : (const void*)k_bgemv_tc<kEpiSwiglu, false>;
  void* params[] = {&p};
  return launch_ex(kern, dim3((unsigned)G), dim3(kBgThreads), BgSmem::kDynamic, st, true, params);
}

}  // namespace ah

extern "C" {

AH_API int ah_q4w_gemv_tc_workspace_bytes(const AhQ4Weight* w, size_t* bytes) {
  AH_REQUIRE(w != nullptr && bytes != nullptr, "ah_q4w_gemv_tc_workspace_bytes: null argument");
  *bytes = ah::bgemv_workspace_bytes(ah::q4w_tiled(w));
  return AH_OK;
}

AH_API int ah_q4w_gemv_tc(const AhQ4Weight* w, const float* x_dev, int64_t x_stride, int batch, float* y_dev,
                          int64_t y_stride, int accumulate, void* workspace_dev, size_t workspace_bytes,
                          void* stream) {
  AH_REQUIRE(w != nullptr, "ah_q4w_gemv_tc: null weight");
  const ah::Q4Tiled& t = ah::q4w_tiled(w);
  AH_REQUIRE(x_stride >= t.cols && y_stride >= t.rows, "ah_q4w_gemv_tc: x_stride must be >= cols, y_stride >= rows");
  ah::GemvArgs a{};
  a.w = t;
  a.x = x_dev;
  a.x_stride = x_stride;
  a.y = y_dev;
  a.y_stride = y_stride;
  a.batch = batch;
  return ah::bgemv_launch(a, ah::kProPlain, accumulate ? ah::kEpiAdd : ah::kEpiStore, workspace_dev, workspace_bytes,
                          ah::as_stream(stream), true);
}

}  // extern "C"
