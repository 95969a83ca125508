// ah_decoder.cu — the Llama-shaped decoder step (inference/mod.rs:333-545)
// built from the fused GEMV plus three small kernels, replayed as CUDA graphs.
//
// One step for `batch` sequences at a shared position `pos` (device scalar):
//   embed      hidden = f16->f32(token_embd[token]); partial sums of squares
//   per layer  qkv   = Wqkv . RMSNorm(hidden)        (GEMV, RMSNorm prologue)
//              attn  = GQA attention over the f16 KV cache, RoPE on q/k and
//                      the KV append fused in (k_attention)
//              hidden += Wo . attn                    (GEMV, residual epilogue)
//              act   = silu(Wg . n) * (Wu . n), n = RMSNorm(hidden)
//                                                     (GEMV, SwiGLU epilogue)
//              hidden += Wd . act                     (GEMV, residual epilogue)
//   head       logits = Wlm . RMSNorm(hidden); next = argmax(logits)
//   advance    pos += 1 (and, while prefilling, the next prompt token)
// RMSNorm statistics travel as per-16-row partial sums of squares written by
// the kernel that produced `hidden` (embed or a residual epilogue).
//
// Tensor parallelism over `world` ranks (one process or thread per GPU):
//   * q/k/v and gate/up keep this rank's heads / FFN rows (column split);
//   * o and down keep this rank's K columns (row split), so their GEMVs give
//     partial sums that one NCCL all-reduce per attention / MLP block adds
//     before the residual add (k_residual_add);
//   * the LM head keeps a vocab slice: each rank takes its argmax and an
//     all-gather of (max, index) pairs picks the first global maximum;
//   * embeddings, norms and `hidden` are replicated (identical on all ranks).
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>
#include <vector>

#include <nccl.h>

#include "ah_gemv_impl.cuh"
#include "ah_prefill.cuh"
#include "ah_sample.cuh"
#include "ah_tma.cuh"

using namespace ah;

namespace ah {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kAttnSplits = 64;     // context splits per (sequence, kv head)
constexpr int kAttnMaxChunk = 128;  // positions per split staged in shared memory
constexpr int kArgmaxChunks = 64;

struct AttnArgs {
  const float* qkv;       // [B][dq + 2*dkv]
  uint16_t* kc;           // [B][L][nkv][max_seq][hd]
  uint16_t* vc;
  const float2* rope;     // [max_seq][hd/2] (cos, sin)
  const int* pos;         // device scalar: position of this step's token
  float* part;            // [B][nkv][S][G][hd] partial sums, then [B][nkv][S][G][2] (max, sum)
  int* cnt;               // [B][nkv]
  float* out;             // [B][dq]
  int* err;               // device error word (bounded waits)
  int layer, n_layer, n_head, n_kv, hd, max_seq;
  int batch;              // sequences in this step
  float scale;
};

inline size_t attn_smem_bytes(int G, int hd) {
  return (size_t)2 * kAttnMaxChunk * hd * 2 +                       // K, V rows (f16)
         sizeof(float) * ((size_t)G * hd + 2 * hd + (size_t)G * kAttnMaxChunk + 2 * G) + 16;
}

// grid (n_kv, kAttnSplits, B).  CTA (h, s, b) handles the G = n_head/n_kv query
// heads of kv head h over context split s: its K and V rows arrive in shared
// memory with two bulk (TMA) copies, the scores, softmax pieces and weighted V
// are computed there, and the last CTA of (b, h) combines the splits.  Split 0
// also appends this step's k (after RoPE) and v to the cache.  Follows
// inference/mod.rs:469-502 with per-head RoPE (attention.rs:126-139).
__global__ void __launch_bounds__(kAttnThreads) k_attention(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smraw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const int hd = a.hd, G = a.n_head / a.n_kv, half = hd / 2;
  const int dq = a.n_head * hd, dkv = a.n_kv * hd;
  uint16_t* Ks = reinterpret_cast<uint16_t*>(smraw);     // [chunk][hd]
  uint16_t* Vs = Ks + kAttnMaxChunk * hd;                  // [chunk][hd]
  float* q = reinterpret_cast<float*>(Vs + kAttnMaxChunk * hd);  // [G][hd] rotated queries
  float* knew = q + G * hd;            // [hd] this step's k (rotated, f16-rounded)
  float* vnew = knew + hd;             // [hd]
  float* sc = vnew + hd;               // [G][kAttnMaxChunk] scores, then weights
  float* red = sc + G * kAttnMaxChunk; // [G][2]
  __shared__ __align__(8) uint64_t bar;
  __shared__ int last;
  pdl_launch_dependents();
  pdl_wait();
  const int pos = *a.pos;
  const int n_ctx = pos + 1;
  // splits in use: at least 64 positions each (short contexts need few)
  const int n_split = min(kAttnSplits, (n_ctx + 63) / 64);
  if (s >= n_split) return;
  const int chunk = (n_ctx + n_split - 1) / n_split;
  const int p0 = min(s * chunk, n_ctx), p1 = min(p0 + chunk, n_ctx);
  const int n = p1 - p0;
  const int ncache = max(0, min(p1, pos) - p0);  // rows already in the cache
  const size_t head_off = ((((size_t)b * a.n_layer + a.layer) * a.n_kv + h) * a.max_seq) * hd;
  uint16_t* kh = a.kc + head_off;
  uint16_t* vh = a.vc + head_off;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar, (uint32_t)(2 * ncache * hd * 2));
    if (ncache > 0) {
      bulk_g2s(Ks, kh + (size_t)p0 * hd, (uint32_t)(ncache * hd * 2), &bar);
      bulk_g2s(Vs, vh + (size_t)p0 * hd, (uint32_t)(ncache * hd * 2), &bar);
    }
  }
  const float* row = a.qkv + (size_t)b * (dq + 2 * dkv);
  const float2* cs = a.rope + (size_t)pos * half;
  // RoPE on adjacent pairs (2i, 2i+1), theta_i = pos * base^(-i/half) (math.rs:119-151)
  for (int i = tid; i < G * half; i += kAttnThreads) {
    const int g = i / half, k = i - g * half;
    const float x0 = row[(h * G + g) * hd + 2 * k], x1 = row[(h * G + g) * hd + 2 * k + 1];
    const float2 c = cs[k];
    q[g * hd + 2 * k] = x0 * c.x - x1 * c.y;
    q[g * hd + 2 * k + 1] = x0 * c.y + x1 * c.x;
  }
  for (int k = tid; k < half; k += kAttnThreads) {
    const float x0 = row[dq + h * hd + 2 * k], x1 = row[dq + h * hd + 2 * k + 1];
    const float2 c = cs[k];
    // the cache holds f16 (the decode configs' f16 KV); use the rounded values
    knew[2 * k] = __half2float(__float2half_rn(x0 * c.x - x1 * c.y));
    knew[2 * k + 1] = __half2float(__float2half_rn(x0 * c.y + x1 * c.x));
  }
  for (int d = tid; d < hd; d += kAttnThreads) vnew[d] = __half2float(__float2half_rn(row[dq + dkv + h * hd + d]));
  __syncthreads();  // q/knew/vnew ready, barrier initialised
  if (s == 0)
    for (int d = tid; d < hd; d += kAttnThreads) {
      kh[(size_t)pos * hd + d] = __half_as_ushort(__float2half_rn(knew[d]));
      vh[(size_t)pos * hd + d] = __half_as_ushort(__float2half_rn(vnew[d]));
    }
  const bool ok = mbar_wait_bounded(&bar, 0, a.err, 0x401);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) mbar_wait_bounded(&bar, 0, a.err, 0x402);  // let copies in flight land
    return;
  }
  if (pos >= p0 && pos < p1)  // this step's row comes from registers, not the cache
    for (int d = tid; d < hd; d += kAttnThreads) {
      Ks[(pos - p0) * hd + d] = __half_as_ushort(__float2half_rn(knew[d]));
      Vs[(pos - p0) * hd + d] = __half_as_ushort(__float2half_rn(vnew[d]));
    }
  __syncthreads();
  // scores: one warp per position, lanes over head dims (hd = 32 * per_lane).
  // Loops run to the compile-time maxima (4 dims per lane, 8 heads per group)
  // under uniform predicates, so kv[] and dot[] stay in registers.
  const int per_lane = hd / 32;
  for (int i = warp; i < n; i += kAttnThreads / 32) {
    float kv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const uint16_t* kr = Ks + i * hd + lane * per_lane;
    if (per_lane == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(kr);  // 8-byte aligned: hd = 128
      kv[0] = __half2float(__ushort_as_half((unsigned short)(u.x & 0xFFFFu)));
      kv[1] = __half2float(__ushort_as_half((unsigned short)(u.x >> 16)));
      kv[2] = __half2float(__ushort_as_half((unsigned short)(u.y & 0xFFFFu)));
      kv[3] = __half2float(__ushort_as_half((unsigned short)(u.y >> 16)));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (e < per_lane) kv[e] = __half2float(__ushort_as_half(kr[e]));
    }
    float dot[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      dot[g] = 0.0f;
      if (g < G) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (e < per_lane) dot[g] = fmaf(q[g * hd + lane * per_lane + e], kv[e], dot[g]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int g = 0; g < 8; ++g)
        if (g < G) dot[g] += __shfl_xor_sync(0xFFFFFFFFu, dot[g], o);
    if (lane == 0)
#pragma unroll
      for (int g = 0; g < 8; ++g)
        if (g < G) sc[g * kAttnMaxChunk + i] = dot[g] * a.scale;
  }
  __syncthreads();
  // softmax pieces per head: m = max, weights exp(s - m), l = sum
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[g * kAttnMaxChunk + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    float l = 0.0f;
    for (int i = lane; i < n; i += 32) {
      const float e = expf(sc[g * kAttnMaxChunk + i] - m);
      sc[g * kAttnMaxChunk + i] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    if (lane == 0) {
      red[g * 2] = m;
      red[g * 2 + 1] = l;
    }
  }
  __syncthreads();
  // weighted V: thread per head dim
  const size_t bh = (size_t)b * a.n_kv + h;
  float* pacc = a.part + ((bh * kAttnSplits + s) * G) * hd;                                   // [G][hd]
  float* pml = a.part + (size_t)gridDim.z * a.n_kv * kAttnSplits * G * hd + (bh * kAttnSplits + s) * G * 2;
  for (int d = tid; d < hd; d += kAttnThreads) {
    float acc[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) acc[g] = 0.0f;
    for (int i = 0; i < n; ++i) {
      const float v = __half2float(__ushort_as_half(Vs[i * hd + d]));
#pragma unroll
      for (int g = 0; g < 8; ++g)
        if (g < G) acc[g] = fmaf(sc[g * kAttnMaxChunk + i], v, acc[g]);
    }
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (g < G) pacc[g * hd + d] = acc[g];
  }
  if (tid < G) {
    pml[tid * 2] = n > 0 ? red[tid * 2] : -INFINITY;
    pml[tid * 2 + 1] = n > 0 ? red[tid * 2 + 1] : 0.0f;
  }
  // the last split to finish combines (deterministic split order)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(&a.cnt[bh], 1) == n_split - 1;
    if (last) __threadfence();
  }
  __syncthreads();
  if (!last) return;
  const float* acc_base = a.part + (bh * kAttnSplits * G) * hd;
  const float* ml_base = a.part + (size_t)gridDim.z * a.n_kv * kAttnSplits * G * hd + bh * kAttnSplits * G * 2;
  // reuse sc: [G][S] split weights exp(m_s - M); red[g] = 1/L
  float* fm = sc;
  static_assert(kAttnMaxChunk >= kAttnSplits, "combine weights must fit in the score buffer");
  if (tid < G) {
    float M = -INFINITY;
    for (int t = 0; t < n_split; ++t) M = fmaxf(M, __ldcg(ml_base + (t * G + tid) * 2));
    float L = 0.0f;
    for (int t = 0; t < n_split; ++t) {
      const float mt = __ldcg(ml_base + (t * G + tid) * 2);
      const float f = (mt == -INFINITY) ? 0.0f : expf(mt - M);
      fm[tid * kAttnSplits + t] = f;
      L = fmaf(__ldcg(ml_base + (t * G + tid) * 2 + 1), f, L);
    }
    red[tid] = 1.0f / L;
  }
  __syncthreads();
  for (int i4 = tid; i4 < G * hd / 4; i4 += kAttnThreads) {  // four consecutive head dims per thread
    const int g = (i4 * 4) / hd;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
    for (int t = 0; t < n_split; ++t) {
      const float f = fm[g * kAttnSplits + t];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(acc_base + (size_t)t * G * hd) + i4);
      acc.x = fmaf(v.x, f, acc.x);
      acc.y = fmaf(v.y, f, acc.y);
      acc.z = fmaf(v.z, f, acc.z);
      acc.w = fmaf(v.w, f, acc.w);
    }
    const float inv = red[g];
    float* o = a.out + (size_t)b * dq + (size_t)h * G * hd + i4 * 4;  // mod.rs:492-500
    o[0] = acc.x * inv;
    o[1] = acc.y * inv;
    o[2] = acc.z * inv;
    o[3] = acc.w * inv;
  }
  if (tid == 0) a.cnt[bh] = 0;
}

// ---------------------------------------------------------------------------
// Tensor-core decode attention for head_dim 64 / 128 and GQA groups <= 8.
//
// Work items (sequence b, kv head h, context split s) are spread over a
// persistent grid sized to the resident CTAs, so no wave of idle CTAs is
// launched for short contexts or large batches.  Each CTA takes a contiguous
// run of items, so consecutive items mostly share (b, h) and the q / k / v
// preparation below runs once per (b, h), and the next item's K / V tiles are
// requested as soon as this item's MMAs have read the current ones.  A
// %globaltimer trace of a batch-16, 2048-position layer had put ~8 us on each
// item: 1.5-3.5 us preparing q again for every split, 1.5 us merging with an
// expf per output element, 1.2 us on the split counter.  Per item:
//   * K and V rows [p0, p1) arrive by TMA in 32-row boxes of 128-byte column
//     halves with the 128-byte swizzle, so the fragment loads below are free of
//     bank conflicts; this step's k / v (after RoPE, f16-rounded) replace row
//     `pos` in shared memory and split 0 appends them to the cache.
//   * S = Q K^T on mma.sync m16n8k16: the G query heads are the M rows, q is
//     scaled by a power of two and split into f16 hi + lo parts (two MMAs), so
//     the scores carry f32 accuracy against the f16 keys.
//   * softmax pieces per warp, then O^T = V^T P^T: V^T comes from transposed
//     fragment loads and P^T is the S accumulator itself (its C layout is the
//     B operand layout), again split hi + lo.
//   * the four warps' (max, sum, O) merge in shared memory; one split writes
//     the output, several write partials and the last to finish combines them.
// Same arithmetic as k_attention (inference/mod.rs:469-502, per-head RoPE as in
// attention.rs:126-139), up to f32 rounding order.
// ---------------------------------------------------------------------------
constexpr int kAttnBoxRows = 32;  // rows per TMA box of the cache views

template <int HD>
struct AttnTcSmem {
  static constexpr int kHalves = HD / 64;                 // 128-byte column halves per row
  static constexpr int kHalfBytes = kAttnMaxChunk * 128;  // one column half of the K or V tile
  static constexpr int kQStride = HD + 8;                 // halves per staged q row (conflict-free)
  static constexpr int kK = 0;
  static constexpr int kV = kK + kHalves * kHalfBytes;
  static constexpr int kQ = kV + kHalves * kHalfBytes;    // q hi, q lo: [2][8][kQStride] f16
  static constexpr int kRed = kQ + 2 * 8 * kQStride * 2;  // [4 warps][HD][8] f32 partial O^T
  static constexpr int kMl = kRed + 4 * HD * 8 * 4;       // [4 warps][8][2] (max, sum)
  static constexpr int kNew = kMl + 4 * 8 * 2 * 4;        // k, v of this step: [2][HD] f32
  static constexpr int kWmax = kNew + 2 * HD * 4;         // [4] per-warp max |q|, then merge factors
  static constexpr int kBytes = kWmax + 16 + 48 * 4;      // [8][4] exp(m_w - M), [8] L, [8] M
  static constexpr int kAlloc = kBytes + 1024;            // the tiles need a 1024-byte aligned base
};

struct AttnTcParams {
  CUtensorMap tm_k;  // K cache as [B*L*nkv*max_seq][HD] f16, box 64 x 32, 128-byte swizzle
  CUtensorMap tm_v;  // V cache, same view
  AttnArgs a;
};

// Byte offset of 16-byte chunk `c` of row `r` inside a 128-byte-swizzled half.
__device__ __forceinline__ uint32_t swz128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// x = hi + lo with hi, lo f16 (lo holds the rounding error of hi).
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  hi = pack_h2(h0, h1);
  lo = pack_h2(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1)));
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attention_tc(const __grid_constant__ AttnTcParams p) {
  using S = AttnTcSmem<HD>;
  constexpr int KS = HD / 16;                            // 16-wide k-steps over the head dims
  constexpr int kQPer = 8 * (HD / 2) / kAttnThreads;     // rotated q pairs per thread (8 head slots)
  const AttnArgs& a = p.a;
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint8_t* Ks = sm + S::kK;
  uint8_t* Vs = sm + S::kV;
  __half* Qh = reinterpret_cast<__half*>(sm + S::kQ);
  __half* Ql = Qh + 8 * S::kQStride;
  float* red = reinterpret_cast<float*>(sm + S::kRed);
  float* mls = reinterpret_cast<float*>(sm + S::kMl);
  float* knew = reinterpret_cast<float*>(sm + S::kNew);
  float* vnew = knew + HD;
  float* wmax = reinterpret_cast<float*>(sm + S::kWmax);
  __shared__ __align__(8) uint64_t bar;
  __shared__ int last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int G = a.n_head / a.n_kv, half = HD / 2;
  const int dq = a.n_head * HD, dkv = a.n_kv * HD;
  pdl_launch_dependents();
  pdl_wait();
  const int pos = *a.pos;
  const int n_ctx = pos + 1;
  int n_split = min(kAttnSplits, (n_ctx + 63) / 64);
  // many sequences x kv heads (batched decode): fewer, longer splits (up to
  // the tile's kAttnMaxChunk rows) halve the per-item fixed costs
  if (a.batch * a.n_kv * n_split > 4 * (int)gridDim.x)
    n_split = max(1, min(n_split, (n_ctx + kAttnMaxChunk - 1) / kAttnMaxChunk));
  const int chunk = (n_ctx + n_split - 1) / n_split;  // <= kAttnMaxChunk (max_seq is checked at creation)
  const int kw = (chunk + 63) >> 6;                   // 16-position k-steps per warp (1 or 2)
  const int n_items = a.batch * a.n_kv * n_split;
  // each CTA takes a contiguous run of items: consecutive items mostly share
  // (sequence, kv head), whose q / k / v preparation is then done once
  const int it0 = (int)(((int64_t)blockIdx.x * n_items) / gridDim.x);
  const int it1 = (int)(((int64_t)(blockIdx.x + 1) * n_items) / gridDim.x);
  if (it0 >= it1) return;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const float2* cs = a.rope + (size_t)pos * half;
  // K / V rows [p0, p1) of an item by TMA into the tiles (thread 0)
  auto issue_tiles = [&](int it) {
    const int s_ = it % n_split, bh_ = it / n_split;
    const int h_ = bh_ % a.n_kv, b_ = bh_ / a.n_kv;
    const int q0 = min(s_ * chunk, n_ctx), nn = min(q0 + chunk, n_ctx) - q0;
    const int nb = (nn + kAttnBoxRows - 1) / kAttnBoxRows;
    const size_t hrow = (((size_t)b_ * a.n_layer + a.layer) * a.n_kv + h_) * a.max_seq;
    mbar_arrive_expect_tx(&bar, (uint32_t)(nb * 2 * S::kHalves * kAttnBoxRows * 128));
    for (int j = 0; j < nb; ++j)
#pragma unroll
      for (int hf = 0; hf < S::kHalves; ++hf) {
        const int y = (int)(hrow + q0 + j * kAttnBoxRows);
        tma_load_2d(Ks + hf * S::kHalfBytes + j * kAttnBoxRows * 128, &p.tm_k, hf * 64, y, &bar);
        tma_load_2d(Vs + hf * S::kHalfBytes + j * kAttnBoxRows * 128, &p.tm_v, hf * 64, y, &bar);
      }
  };
  if (tid == 0) issue_tiles(it0);
  uint32_t phase = 0;
  int cur_bh = -1;
  float qs = 1.0f;
  for (int item = it0; item < it1; ++item, phase ^= 1u) {
    const int s = item % n_split, bh = item / n_split;
    const int h = bh % a.n_kv, b = bh / a.n_kv;
    const int p0 = min(s * chunk, n_ctx), p1 = min(p0 + chunk, n_ctx), n = p1 - p0;
    const size_t head_row = (((size_t)b * a.n_layer + a.layer) * a.n_kv + h) * a.max_seq;
    if (bh != cur_bh) {
    cur_bh = bh;
    // RoPE on adjacent pairs (2i, 2i+1), theta_i = pos * base^(-i/half) (math.rs:119-151)
    const float* row = a.qkv + (size_t)b * (dq + 2 * dkv);
    float2 qr[kQPer];
    float mx = 0.0f;
#pragma unroll
    for (int u = 0; u < kQPer; ++u) {
      const int i = tid + u * kAttnThreads;  // pair index over [8 head slots][half]
      const int gg = i / half, k = i - gg * half;
      float2 v = make_float2(0.0f, 0.0f);
      if (gg < G) {
        const float2 x = *reinterpret_cast<const float2*>(row + (h * G + gg) * HD + 2 * k);
        const float2 c = cs[k];
        v = make_float2(x.x * c.x - x.y * c.y, x.x * c.y + x.y * c.x);
      }
      qr[u] = v;
      mx = fmaxf(mx, fmaxf(fabsf(v.x), fabsf(v.y)));
    }
    for (int k = tid; k < half; k += kAttnThreads) {
      const float2 x = *reinterpret_cast<const float2*>(row + dq + h * HD + 2 * k);
      const float2 c = cs[k];
      // the cache holds f16 (the decode configs' f16 KV); use the rounded values
      knew[2 * k] = __half2float(__float2half_rn(x.x * c.x - x.y * c.y));
      knew[2 * k + 1] = __half2float(__float2half_rn(x.x * c.y + x.y * c.x));
    }
    for (int d = tid; d < HD; d += kAttnThreads) vnew[d] = __half2float(__float2half_rn(row[dq + dkv + h * HD + d]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) wmax[warp] = mx;
    __syncthreads();  // wmax, knew, vnew ready
    // q * 2^e with max |q| * 2^e in [2^14, 2^15): f16 hi / lo parts keep f32 accuracy
    const float qm = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
    int ex = 0;
    if (qm > 0.0f) frexpf(qm, &ex);
    const int sh = qm > 0.0f ? min(15 - ex, 100) : 0;
    qs = ldexpf(1.0f, sh);
#pragma unroll
    for (int u = 0; u < kQPer; ++u) {
      const int i = tid + u * kAttnThreads;
      const int gg = i / half, k = i - gg * half;
      uint32_t hi, lo;
      split_h2(qr[u].x * qs, qr[u].y * qs, hi, lo);
      *reinterpret_cast<uint32_t*>(Qh + gg * S::kQStride + 2 * k) = hi;
      *reinterpret_cast<uint32_t*>(Ql + gg * S::kQStride + 2 * k) = lo;
    }
    }  // q / k / v of (b, h) prepared
    if (s == 0) {
      uint16_t* kh = a.kc + (head_row + pos) * HD;
      uint16_t* vh = a.vc + (head_row + pos) * HD;
      for (int d = tid; d < HD; d += kAttnThreads) {
        kh[d] = __half_as_ushort(__float2half_rn(knew[d]));
        vh[d] = __half_as_ushort(__float2half_rn(vnew[d]));
      }
    }
    const bool ok = mbar_wait_bounded(&bar, phase, a.err, 0x403);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) mbar_wait_bounded(&bar, phase, a.err, 0x404);  // let copies in flight land
      return;
    }
    // this step's row replaces the cache row at pos; V rows past n up to the end
    // of the last working warp's range (read with zero weight) are cleared so
    // stale values cannot leak
    if (pos >= p0 && pos < p1) {
      const int r = pos - p0;
      for (int d = tid; d < HD; d += kAttnThreads) {
        const uint32_t off = (d >> 6) * S::kHalfBytes + swz128(r, (d & 63) >> 3) + (d & 7) * 2;
        *reinterpret_cast<uint16_t*>(Ks + off) = __half_as_ushort(__float2half_rn(knew[d]));
        *reinterpret_cast<uint16_t*>(Vs + off) = __half_as_ushort(__float2half_rn(vnew[d]));
      }
    }
    const int nz = (n + 16 * kw - 1) / (16 * kw) * (16 * kw);  // <= 32 * nbox: inside the loaded boxes
    for (int i = tid; i < (nz - n) * (HD / 8); i += kAttnThreads) {
      const int r = n + i / (HD / 8), cc = i % (HD / 8);
      *reinterpret_cast<uint4*>(Vs + (cc >> 3) * S::kHalfBytes + swz128(r, cc & 7)) = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();  // q parts and K / V tiles final

    // ---- this warp's positions [wp0, wp0 + 16 kw) of the tile ----
    const int wp0 = warp * 16 * kw;
    float oacc[KS][4];
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) oacc[mt][0] = oacc[mt][1] = oacc[mt][2] = oacc[mt][3] = 0.0f;
    float mrow = -INFINITY, lrow = 0.0f;  // softmax pieces of head g over this warp's positions
    if (wp0 < n) {
      uint32_t qh[KS][2], ql[KS][2];  // A fragments, rows 0-7 = heads (rows 8-15 are zero)
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        qh[kk][0] = *reinterpret_cast<const uint32_t*>(Qh + g * S::kQStride + kk * 16 + 2 * t);
        qh[kk][1] = *reinterpret_cast<const uint32_t*>(Qh + g * S::kQStride + kk * 16 + 8 + 2 * t);
        ql[kk][0] = *reinterpret_cast<const uint32_t*>(Ql + g * S::kQStride + kk * 16 + 2 * t);
        ql[kk][1] = *reinterpret_cast<const uint32_t*>(Ql + g * S::kQStride + kk * 16 + 8 + 2 * t);
      }
      float sacc[4][4];
      const uint32_t kbase = smem_u32(Ks);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
        if (j < 2 * kw) {
          const int prow = wp0 + 8 * j + (lane & 7);  // the position whose row this lane addresses
#pragma unroll
          for (int k2 = 0; k2 < HD / 32; ++k2) {
            const int d0 = k2 * 32 + (lane >> 3) * 8;  // matrix lane/8: dims d0..d0+7
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kbase + (d0 >> 6) * S::kHalfBytes + swz128(prow, (d0 & 63) >> 3), b0, b1, b2, b3);
            mma16816(sacc[j], qh[2 * k2][0], 0u, qh[2 * k2][1], 0u, b0, b1, sacc[j]);
            mma16816(sacc[j], ql[2 * k2][0], 0u, ql[2 * k2][1], 0u, b0, b1, sacc[j]);
            mma16816(sacc[j], qh[2 * k2 + 1][0], 0u, qh[2 * k2 + 1][1], 0u, b2, b3, sacc[j]);
            mma16816(sacc[j], ql[2 * k2 + 1][0], 0u, ql[2 * k2 + 1][1], 0u, b2, b3, sacc[j]);
          }
        }
      }
      // scores of head g at positions wp0 + 8j + 2t + e; -inf past n
      const float mult = a.scale / qs;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool live = j < 2 * kw && wp0 + 8 * j + 2 * t + e < n;
          sacc[j][e] = live ? sacc[j][e] * mult : -INFINITY;
          mrow = fmaxf(mrow, sacc[j][e]);
        }
      mrow = fmaxf(mrow, __shfl_xor_sync(0xFFFFFFFFu, mrow, 1));
      mrow = fmaxf(mrow, __shfl_xor_sync(0xFFFFFFFFu, mrow, 2));
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float w = sacc[j][e] == -INFINITY ? 0.0f : expf(sacc[j][e] - mrow);
          sacc[j][e] = w;
          lrow += w;
        }
      lrow += __shfl_xor_sync(0xFFFFFFFFu, lrow, 1);
      lrow += __shfl_xor_sync(0xFFFFFFFFu, lrow, 2);
      // O^T[dim][head] += V^T[dim][pos] . P^T[pos][head], 16 positions per k-step
      const uint32_t vbase = smem_u32(Vs);
      const int mi = lane >> 3;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (q < kw) {
          uint32_t ph0, pl0, ph1, pl1;
          split_h2(sacc[2 * q][0], sacc[2 * q][1], ph0, pl0);
          split_h2(sacc[2 * q + 1][0], sacc[2 * q + 1][1], ph1, pl1);
          const int prow = wp0 + 16 * q + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            const int d0 = mt * 16 + ((mi & 1) << 3);
            uint32_t a0, a1, a2, a3;
            ldsm_x4_trans(vbase + (d0 >> 6) * S::kHalfBytes + swz128(prow, (d0 & 63) >> 3), a0, a1, a2, a3);
            mma16816(oacc[mt], a0, a1, a2, a3, ph0, ph1, oacc[mt]);
            mma16816(oacc[mt], a0, a1, a2, a3, pl0, pl1, oacc[mt]);
          }
        }
      }
    }
    // per-warp pieces: O^T[dim][head slot] and (max, sum) per head
    float* rw = red + warp * HD * 8;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      *reinterpret_cast<float2*>(rw + (mt * 16 + g) * 8 + 2 * t) = make_float2(oacc[mt][0], oacc[mt][1]);
      *reinterpret_cast<float2*>(rw + (mt * 16 + g + 8) * 8 + 2 * t) = make_float2(oacc[mt][2], oacc[mt][3]);
    }
    if (t == 0) {
      mls[(warp * 8 + g) * 2] = mrow;
      mls[(warp * 8 + g) * 2 + 1] = lrow;
    }
    // the tiles' generic writes (this step's row, the cleared V tail) are
    // ordered before the next item's TMA overwrites them
    fence_proxy_async_smem();
    __syncthreads();
    // every warp has read the tiles: the next item's rows load during the
    // merge, the partial stores and the split counter below
    if (tid == 0 && item + 1 < it1) issue_tiles(item + 1);
    // per-head merge factors of the four warps: exp(m_w - M), and L
    float* mf = wmax + 4;  // [8][4] factors, then [8] L (inside the misc area)
    if (tid < 8) {
      const int gg = tid;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) M = fmaxf(M, mls[(w * 8 + gg) * 2]);
      float L = 0.0f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float mw = mls[(w * 8 + gg) * 2];
        const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
        mf[gg * 4 + w] = f;
        L = fmaf(f, mls[(w * 8 + gg) * 2 + 1], L);
      }
      mf[32 + gg] = L;
      mf[40 + gg] = M;
    }
    __syncthreads();
    float* pacc = a.part + (((size_t)bh * kAttnSplits + s) * G) * HD;  // [G][hd]
    float* pml = a.part + (size_t)a.batch * a.n_kv * kAttnSplits * G * HD + ((size_t)bh * kAttnSplits + s) * G * 2;
    for (int i = tid; i < 8 * HD; i += kAttnThreads) {
      const int gg = i & 7, d = i >> 3;
      if (gg < G) {
        const float M = mf[40 + gg], L = mf[32 + gg];
        float O = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) O = fmaf(mf[gg * 4 + w], red[w * HD * 8 + i], O);
        if (n_split == 1) {
          a.out[(size_t)b * dq + (size_t)(h * G + gg) * HD + d] = O / L;  // mod.rs:492-500
        } else {
          pacc[gg * HD + d] = O;
          if (d == 0) {
            pml[gg * 2] = M;
            pml[gg * 2 + 1] = L;
          }
        }
      }
    }
    if (n_split > 1) {
      // the last split of (b, h) to finish combines; the counter's acq_rel add
      // publishes this CTA's partials (ordered by the barrier) and, in the last
      // CTA, makes every split's partials visible
      __syncthreads();
      if (tid == 0) last = atom_add_acq_rel_gpu(&a.cnt[bh], 1) == n_split - 1;
      __syncthreads();
      if (last) {
        const float* acc_base = a.part + ((size_t)bh * kAttnSplits * G) * HD;
        const float2* ml_base = reinterpret_cast<const float2*>(
            a.part + (size_t)a.batch * a.n_kv * kAttnSplits * G * HD + (size_t)bh * kAttnSplits * G * 2);
        float* fm = red;                     // [G][kAttnSplits] split weights exp(m_s - M) / L
        static_assert(kAttnSplits <= 64, "two splits per lane");
        for (int gg = warp; gg < G; gg += kAttnThreads / 32) {  // one warp per head, lanes over splits
          const float2 v0 = lane < n_split ? __ldcg(ml_base + lane * G + gg) : make_float2(-INFINITY, 0.0f);
          const float2 v1 =
              lane + 32 < n_split ? __ldcg(ml_base + (lane + 32) * G + gg) : make_float2(-INFINITY, 0.0f);
          float M = fmaxf(v0.x, v1.x);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
          const float f0 = v0.x == -INFINITY ? 0.0f : expf(v0.x - M);
          const float f1 = v1.x == -INFINITY ? 0.0f : expf(v1.x - M);
          float L = fmaf(f1, v1.y, f0 * v0.y);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, o);
          const float inv = 1.0f / L;
          fm[gg * kAttnSplits + lane] = f0 * inv;
          fm[gg * kAttnSplits + lane + 32] = f1 * inv;
        }
        __syncthreads();
        for (int i4 = tid; i4 < G * HD / 4; i4 += kAttnThreads) {  // four consecutive head dims per thread
          const int gg = (i4 * 4) / HD;
          float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          for (int u0 = 0; u0 < n_split; u0 += 16) {  // 16 independent loads in flight
            float4 v[16];
#pragma unroll
            for (int k = 0; k < 16; ++k)
              if (u0 + k < n_split) v[k] = __ldcg(reinterpret_cast<const float4*>(acc_base + (size_t)(u0 + k) * G * HD) + i4);
#pragma unroll
            for (int k = 0; k < 16; ++k)
              if (u0 + k < n_split) {
                const float f = fm[gg * kAttnSplits + u0 + k];
                acc.x = fmaf(v[k].x, f, acc.x);
                acc.y = fmaf(v[k].y, f, acc.y);
                acc.z = fmaf(v[k].z, f, acc.z);
                acc.w = fmaf(v[k].w, f, acc.w);
              }
          }
          *reinterpret_cast<float4*>(a.out + (size_t)b * dq + (size_t)h * G * HD + i4 * 4) = acc;
        }
        if (tid == 0) a.cnt[bh] = 0;
      }
    }
    __syncthreads();  // red / fm / mf are reused by the next item
  }
}

// hidden = f16 -> f32 (token_embd[token]) (mod.rs:392-397); ss partials per 16.
// grid ((d + 255) / 256, B); d is a multiple of 16.
__global__ void __launch_bounds__(256) k_embed(const uint16_t* __restrict__ emb, const int* __restrict__ tok,
                                               float* __restrict__ hidden, float* __restrict__ ss, int d, int vocab) {
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = i < d;
  pdl_launch_dependents();
  pdl_wait();
  const int t = tok[b];
  const int tv = (t >= 0 && t < vocab) ? t : 0;
  const float v = live ? f16_bits_to_f32(emb[(size_t)tv * d + i]) : 0.0f;
  if (live) hidden[(size_t)b * d + i] = v;
  float q = v * v;
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  if (live && (i & 15) == 0) ss[(size_t)b * (d / 16) + i / 16] = q;
}

// Greedy next token per sequence (sampling.rs:4-14: the first strict maximum;
// NaN never wins; all -inf or NaN gives 0).  grid (kArgmaxChunks, B).
// With `pair` set (tensor parallelism) the shard's candidate (value, index +
// idx_base) is written there instead of the token.
struct ArgPair;
__global__ void __launch_bounds__(256) k_argmax(const float* __restrict__ logits, int vocab, float* pv, int* pi,
                                                int* cnt, int* tok, int* tok_log, const int* pos, int batch,
                                                ArgPair* pair, int idx_base) {
  const int b = blockIdx.y, c = blockIdx.x, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const int chunk = (vocab + kArgmaxChunks - 1) / kArgmaxChunks;
  const int i0 = c * chunk, i1 = min(i0 + chunk, vocab);
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int i = i0 + tid; i < i1; i += 256) {
    const float v = logits[(size_t)b * vocab + i];
    if (v > bv) { bv = v; bi = i; }
  }
  __shared__ float sv[256];
  __shared__ int si[256];
  sv[tid] = bv;
  si[tid] = bi;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (tid < o) {
      const float v2 = sv[tid + o];
      const int i2 = si[tid + o];
      if (v2 > sv[tid] || (v2 == sv[tid] && i2 < si[tid])) { sv[tid] = v2; si[tid] = i2; }
    }
    __syncthreads();
  }
  __shared__ int last;
  if (tid == 0) {
    pv[b * kArgmaxChunks + c] = sv[0];
    pi[b * kArgmaxChunks + c] = si[0];
    __threadfence();
    last = atomicAdd(&cnt[b], 1) == kArgmaxChunks - 1;
    if (last) __threadfence();
  }
  __syncthreads();
  if (!last || tid != 0) return;
  float best = -INFINITY;
  int besti = INT_MAX;
  for (int k = 0; k < kArgmaxChunks; ++k) {
    const float v = __ldcg(pv + b * kArgmaxChunks + k);
    const int i = __ldcg(pi + b * kArgmaxChunks + k);
    if (v > best || (v == best && i < besti)) { best = v; besti = i; }
  }
  cnt[b] = 0;
  if (pair) {
    float* pp = reinterpret_cast<float*>(pair) + 2 * b;
    pp[0] = best;
    reinterpret_cast<int*>(pp)[1] = besti == INT_MAX ? INT_MAX : besti + idx_base;
    return;
  }
  const int next = (besti == INT_MAX) ? 0 : besti;
  tok[b] = next;
  tok_log[(size_t)(*pos) * batch + b] = next;
}

// hidden += part (the all-reduced o / down projection) and the per-16-row
// sums of squares of the new hidden.  grid ((d + 255) / 256, B).
__global__ void __launch_bounds__(256) k_residual_add(float* __restrict__ hidden, const float* __restrict__ part,
                                                      float* __restrict__ ss, int d) {
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = i < d;
  pdl_launch_dependents();
  pdl_wait();
  float h = 0.0f;
  if (live) {
    h = hidden[(size_t)b * d + i] + part[(size_t)b * d + i];  // inference/mod.rs:505 residual
    hidden[(size_t)b * d + i] = h;
  }
  float q = h * h;
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  if (live && (i & 15) == 0) ss[(size_t)b * (d / 16) + i / 16] = q;
}

// ---- tensor-parallel all-reduce over NVLink peer memory ------------------------
// Each rank's o / down GEMV stores its partial into slot `rank` of every rank's
// receive buffer (peer stores, [d][max_batch] so a tile's 16 rows x batch
// outputs are one contiguous run); k_peer_signal then publishes the collective's
// sequence number into every rank's flag slot `rank`, and k_residual_add_peer
// waits for all ranks' flags before summing the slots in rank order (so every
// rank computes the identical sum).  Waits are bounded: a rank that never
// signals makes the wait record AH_ETIMEOUT and leave hidden untouched.
struct PeerFlags {
  unsigned* flag[8];  // each rank's flag array, as mapped on this GPU
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void k_peer_signal(unsigned* seq, PeerFlags f, int rank, int world) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  const unsigned s = *seq + 1u;
  *seq = s;
  for (int r = 0; r < world; ++r) st_release_sys(f.flag[r] + rank, s);
}

constexpr uint32_t kPeerWaitLimit = 1u << 22;  // x ~100 ns sleeps: ~0.4 s

// hidden += sum_r slot[r] (rank order), and the per-16-row sums of squares.
// grid ((d + 255) / 256, B).
__global__ void __launch_bounds__(256) k_residual_add_peer(float* __restrict__ hidden, const float* __restrict__ slots,
                                                           int world, int batch, float* __restrict__ ss, int d,
                                                           const unsigned* flag, const unsigned* seq, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const unsigned s = *seq;
    int good = 1;
    for (int r = 0; r < world && good; ++r) {
      uint32_t it = 0;
      while (ld_acquire_sys(flag + r) < s) {
        if (++it > kPeerWaitLimit) {
          atomicExch(err, AH_ETIMEOUT);
          good = 0;
          break;
        }
        __nanosleep(100);
      }
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = i < d;
  float h = 0.0f;
  if (live) {
    float sum = 0.0f;
    for (int r = 0; r < world; ++r) sum += slots[((size_t)r * d + i) * batch + b];  // slot r: [d][batch]
    h = hidden[(size_t)b * d + i] + sum;
    hidden[(size_t)b * d + i] = h;
  }
  float q = h * h;
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  if (live && (i & 15) == 0) ss[(size_t)b * (d / 16) + i / 16] = q;
}

// Candidate of one vocab shard: value and global index (INT_MAX: none).
struct ArgPair {
  float v;
  int i;
};

// The first global maximum over the ranks' shard candidates (shards hold
// increasing vocab ranges, and each candidate is its shard's first maximum).
__global__ void k_argmax_merge(const ArgPair* __restrict__ all, int world, int* tok, int* tok_log, const int* pos,
                               int batch) {
  pdl_wait();
  const int b = threadIdx.x;
  if (b >= batch) return;
  float best = -INFINITY;
  int besti = INT_MAX;
  for (int r = 0; r < world; ++r) {
    const ArgPair p = all[(size_t)r * batch + b];
    if (p.i != INT_MAX && (p.v > best || (p.v == best && p.i < besti))) {
      best = p.v;
      besti = p.i;
    }
  }
  const int next = besti == INT_MAX ? 0 : besti;
  tok[b] = next;
  tok_log[(size_t)(*pos) * batch + b] = next;
}

// pos += 1; while prefilling, also load the next prompt token.
__global__ void k_advance(int* pos, int* tok, const int* prompt, int n_prompt, int batch) {
  pdl_wait();
  const int p = *pos + 1;
  if (threadIdx.x < batch && prompt != nullptr && p < n_prompt) tok[threadIdx.x] = prompt[threadIdx.x * n_prompt + p];
  __syncthreads();
  if (threadIdx.x == 0) *pos = p;
}

// After a prefill of positions 0 .. p-1: position p next, with prompt token p.
__global__ void k_prefill_state(int* pos, int* tok, const int* prompt, int n_prompt, int p, int batch) {
  if (threadIdx.x < batch) tok[threadIdx.x] = prompt[threadIdx.x * n_prompt + p];
  if (threadIdx.x == 0) *pos = p;
}

__global__ void k_rope_table(float2* t, int max_seq, int half, float base) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= max_seq * half) return;
  const int p = i / half, k = i - p * half;
  const float theta = (float)p * powf(base, -((float)k) / ((float)half));  // math.rs:139
  float sn, cs;
  sincosf(theta, &sn, &cs);
  t[i] = make_float2(cs, sn);
}

}  // namespace
}  // namespace ah

// ---------------------------------------------------------------------------
// Model object
// ---------------------------------------------------------------------------
// Smallest batch whose decode GEMVs run on the tcgen05 batched GEMV by default.
constexpr int kBgemvMinBatchDefault = 9;

struct AhModel {
  AhModelConfig c{};  // the full (unsharded) model
  int device = 0;
  int tp_rank = 0, tp_world = 1;
  ncclComm_t comm = nullptr;
  int nh = 0, nkv = 0, nff = 0, nvoc = 0;  // this rank's heads, kv heads, FFN rows, vocab rows
  int dq = 0, dkv = 0;                     // this rank's q and k/v widths
  std::vector<AhQ4Weight*> wqkv, wo, wgu, wd;
  AhQ4Weight* lm = nullptr;
  std::vector<void*> pend[5];  // q, k, v, gate, up awaiting fusion (Q4_0 blocks or scales + packed)
  std::vector<int> pend_fmt[5];  // kProjQ4_0 / kProjEngine per pending buffer
  uint16_t *tok_embd = nullptr, *attn_norm = nullptr, *ffn_norm = nullptr, *out_norm = nullptr;
  uint16_t *kc = nullptr, *vc = nullptr;
  CUtensorMap tm_k{}, tm_v{};  // TMA views of kc / vc for the tensor-core attention
  bool attn_tc = false;        // head_dim 64 or 128: k_attention_tc
  int attn_grid = 0;           // its persistent grid (resident CTAs)
  float2* rope = nullptr;
  float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr, *ss = nullptr;
  float* att_part = nullptr;
  int* att_cnt = nullptr;
  float* part = nullptr;   // [B][d] o / down partial sums (tensor parallelism)
  // peer-memory all-reduce: one block per rank holding the receive slots
  // [2 parities][world][B][d] f32, the flags [world] and the local sequence
  // counter; peer_block[r] is rank r's block as mapped here (IPC)
  void* comm_block = nullptr;
  size_t comm_flags_off = 0;
  void* peer_block[8] = {};
  bool p2p = false;
  void* am_pair = nullptr; // [B] this shard's argmax candidate
  void* am_all = nullptr;  // [world][B] all shards' candidates
  float* am_v = nullptr;
  int* am_i = nullptr;
  int* am_cnt = nullptr;
  int* d_pos = nullptr;
  int* d_tok = nullptr;
  int* d_prompt = nullptr;
  int* tok_log = nullptr;  // [max_seq][max_batch]
  int* err = nullptr;      // device error word
  int batch = 1;
  int pos = 0;
  int n_prompt_dev = 0;
  bool ready_checked = false;
  cudaGraphExec_t g_step[2] = {nullptr, nullptr};  // [0] prefill step, [1] full step
  int g_batch[2] = {0, 0};
  const int* g_prompt[2] = {nullptr, nullptr};
  int g_nprompt[2] = {0, 0};
  std::vector<void*> allocs;
  // prompt prefill through the GEMMs (allocated on first use for kPrefillRows rows)
  int pf_mode = 1;  // 0: token by token, as the reference; 1: GEMM prefill from kPrefillMinTokens
  float *pf_h = nullptr, *pf_qkv = nullptr, *pf_attn = nullptr, *pf_part = nullptr;
  float* pf_act = nullptr;
  void* pf_ws = nullptr;
  size_t pf_ws_bytes = 0;
  // decode steps of at least bg_min_batch sequences run their GEMVs on the
  // tcgen05 batched GEMV (17: never); its workspace is allocated on first use
  int bg_min_batch = kBgemvMinBatchDefault;
  void* bg_ws = nullptr;
  size_t bg_ws_bytes = 0;
  // next-token choice: greedy (temperature 0, the default) or temperature +
  // top-k sampling (inference/sampling.rs:17-64) seeded per (seed, position, sequence)
  float samp_temp = 0.0f;
  int samp_k = 40;
  uint64_t samp_seed = 0;
  SampleCand* samp_cand = nullptr;  // [max_batch][kSampleMaxK] this rank's candidates
  SampleCand* samp_all = nullptr;   // [world][max_batch][kSampleMaxK] all ranks' (tensor parallel)
  void* samp_ws = nullptr;          // the split top-k's slice candidates
  size_t samp_ws_bytes = 0;
};

namespace {

int dalloc(AhModel* m, void** p, size_t bytes) {
  if (ah::dev_malloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return fail(AH_ENOMEM, "model: cudaMalloc of %zu bytes failed", bytes);
  }
  m->allocs.push_back(*p);
  return AH_OK;
}

#define AH_TRY(expr)              \
  do {                            \
    int _rc = (expr);             \
    if (_rc != AH_OK) return _rc; \
  } while (0)

int model_ready(AhModel* m) {
  const int L = m->c.n_layer;
  for (int l = 0; l < L; ++l)
    if (!m->wqkv[l] || !m->wo[l] || !m->wgu[l] || !m->wd[l])
      return fail(AH_EINVAL, "model: layer %d is missing projection weights", l);
  if (!m->lm) return fail(AH_EINVAL, "model: output.weight not loaded");
  return AH_OK;
}

GemvArgs gemv_args(const AhQ4Weight* w, const float* x, int64_t xs, float* y, int64_t ys, int batch) {
  GemvArgs a{};
  a.w = q4w_tiled(w);
  a.x = x;
  a.x_stride = xs;
  a.y = y;
  a.y_stride = ys;
  a.batch = batch;
  return a;
}

// Sums the o / down partials over the tensor-parallel ranks and adds them to
// hidden (with the RMSNorm partial sums of the result).
int reduce_residual(AhModel* m, cudaStream_t st) {
  const int B = m->batch, d = m->c.n_embd;
  if (ncclAllReduce(m->part, m->part, (size_t)B * d, ncclFloat, ncclSum, m->comm, st) != ncclSuccess)
    return fail(AH_ENCCL, "model: all-reduce of the block output failed");
  return launch_pdl(k_residual_add, dim3((d + 255) / 256, B), dim3(256), 0, st, m->hidden, (const float*)m->part,
                    m->ss, d);
}

// Peer-memory variant.  Parity `par` selects the receive slots: a step has 2
// collectives per layer (even), so o-projections always use parity 0 and
// down-projections parity 1, and a rank can only reuse a parity's slots after
// every rank has read them (it has waited for their next collective's flags).
float* peer_slots(const AhModel* m, int r, int par) {
  return static_cast<float*>(m->peer_block[r]) + (size_t)par * m->tp_world * m->c.max_batch * m->c.n_embd +
         (size_t)m->tp_rank * m->c.max_batch * m->c.n_embd;
}
void set_peer_scatter(const AhModel* m, GemvArgs& a, int par) {
  a.n_peer = m->tp_world;
  a.peer_row = m->c.max_batch;  // slots are [d][max_batch]
  for (int r = 0; r < m->tp_world; ++r) a.peer_y[r] = peer_slots(m, r, par);
}
int reduce_residual_peer(AhModel* m, int par, cudaStream_t st) {
  const int B = m->batch, d = m->c.n_embd, W = m->tp_world;
  PeerFlags f{};
  for (int r = 0; r < W; ++r)
    f.flag[r] = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(m->peer_block[r]) + m->comm_flags_off);
  unsigned* local_flags = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(m->comm_block) + m->comm_flags_off);
  unsigned* seq = local_flags + 64;  // the local counter sits after the flag slots
  k_peer_signal<<<1, 32, 0, st>>>(seq, f, m->tp_rank, W);
  AH_LAUNCH_CHECK();
  const float* slots = static_cast<const float*>(m->comm_block) + (size_t)par * W * m->c.max_batch * d;
  k_residual_add_peer<<<dim3((d + 255) / 256, B), 256, 0, st>>>(m->hidden, slots, W, m->c.max_batch, m->ss, d,
                                                                local_flags, seq, m->err);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

// Decode attention of one layer: the tensor-core kernel for head_dim 64 / 128,
// the scalar one otherwise.
int launch_attention(AhModel* m, const AttnArgs& at, size_t attn_smem, cudaStream_t st) {
  if (!m->attn_tc)
    return launch_pdl(k_attention, dim3(m->nkv, kAttnSplits, at.batch), dim3(kAttnThreads), attn_smem, st, at);
  AttnTcParams p;
  p.tm_k = m->tm_k;
  p.tm_v = m->tm_v;
  p.a = at;
  if (m->c.head_dim == 128)
    return launch_pdl(k_attention_tc<128>, dim3(m->attn_grid), dim3(kAttnThreads), (size_t)AttnTcSmem<128>::kAlloc,
                      st, p);
  return launch_pdl(k_attention_tc<64>, dim3(m->attn_grid), dim3(kAttnThreads), (size_t)AttnTcSmem<64>::kAlloc, st,
                    p);
}

int step_gemv(AhModel* m, const GemvArgs& a, int pro, int epi, cudaStream_t st);

// Enqueues one decoder step (all layers; with_head adds LM head + argmax).
int enqueue_step(AhModel* m, bool with_head, const int* prompt, int n_prompt, cudaStream_t st) {
  const AhModelConfig& c = m->c;
  const int B = m->batch, d = c.n_embd;
  const bool tp = m->tp_world > 1;
  AH_TRY(launch_pdl(k_embed, dim3((d + 255) / 256, B), dim3(256), 0, st, (const uint16_t*)m->tok_embd,
                    (const int*)m->d_tok, m->hidden, m->ss, d, c.vocab_size));
  const size_t attn_smem = attn_smem_bytes(m->nh / m->nkv, c.head_dim);
  for (int l = 0; l < c.n_layer; ++l) {
    GemvArgs q = gemv_args(m->wqkv[l], m->hidden, d, m->qkv, m->dq + 2 * m->dkv, B);
    q.norm_w = m->attn_norm + (size_t)l * d;
    q.eps = c.rms_eps;
    q.ss_in = m->ss;
    q.n_ss_in = d / 16;
    AH_TRY(step_gemv(m, q, kProRmsNorm, kEpiStore, st));
    AttnArgs at{};
    at.qkv = m->qkv;
    at.kc = m->kc;
    at.vc = m->vc;
    at.rope = m->rope;
    at.pos = m->d_pos;
    at.part = m->att_part;
    at.cnt = m->att_cnt;
    at.out = m->attn;
    at.layer = l;
    at.n_layer = c.n_layer;
    at.n_head = m->nh;
    at.n_kv = m->nkv;
    at.hd = c.head_dim;
    at.max_seq = c.max_seq;
    at.scale = 1.0f / sqrtf((float)c.head_dim);  // mod.rs:478
    at.err = m->err;
    at.batch = B;
    AH_TRY(launch_attention(m, at, attn_smem, st));
    if (tp && m->p2p) {
      GemvArgs o = gemv_args(m->wo[l], m->attn, m->dq, m->part, d, B);
      set_peer_scatter(m, o, 0);
      AH_TRY(step_gemv(m, o, kProPlain, kEpiStore, st));
      AH_TRY(reduce_residual_peer(m, 0, st));
    } else if (tp) {
      AH_TRY(step_gemv(m, gemv_args(m->wo[l], m->attn, m->dq, m->part, d, B), kProPlain, kEpiStore, st));
      AH_TRY(reduce_residual(m, st));
    } else {
      GemvArgs o = gemv_args(m->wo[l], m->attn, m->dq, m->hidden, d, B);
      o.ss_out = m->ss;
      AH_TRY(step_gemv(m, o, kProPlain, kEpiAdd, st));
    }
    GemvArgs gu = gemv_args(m->wgu[l], m->hidden, d, m->act, m->nff, B);
    gu.norm_w = m->ffn_norm + (size_t)l * d;
    gu.eps = c.rms_eps;
    gu.ss_in = m->ss;
    gu.n_ss_in = d / 16;
    AH_TRY(step_gemv(m, gu, kProRmsNorm, kEpiSwiglu, st));
    if (tp && m->p2p) {
      GemvArgs dn = gemv_args(m->wd[l], m->act, m->nff, m->part, d, B);
      set_peer_scatter(m, dn, 1);
      AH_TRY(step_gemv(m, dn, kProPlain, kEpiStore, st));
      AH_TRY(reduce_residual_peer(m, 1, st));
    } else if (tp) {
      AH_TRY(step_gemv(m, gemv_args(m->wd[l], m->act, m->nff, m->part, d, B), kProPlain, kEpiStore, st));
      AH_TRY(reduce_residual(m, st));
    } else {
      GemvArgs dn = gemv_args(m->wd[l], m->act, m->nff, m->hidden, d, B);
      dn.ss_out = m->ss;
      AH_TRY(step_gemv(m, dn, kProPlain, kEpiAdd, st));
    }
  }
  if (with_head) {
    GemvArgs h = gemv_args(m->lm, m->hidden, d, m->logits, m->nvoc, B);
    h.norm_w = m->out_norm;
    h.eps = c.rms_eps;
    h.ss_in = m->ss;
    h.n_ss_in = d / 16;
    AH_TRY(step_gemv(m, h, kProRmsNorm, kEpiStore, st));
  }
  if (with_head && m->samp_temp > 0.0f) {
    // temperature + top-k sampling (mod.rs:552-553): one kernel on one GPU;
    // under tensor parallelism each rank's top-k of its vocab slice, an
    // all-gather, and the same merge and draw on every rank
    const int K = m->samp_k;
    if (!tp) {
      AH_TRY(sample_launch(m->logits, m->nvoc, B, m->nvoc, K, 0, m->samp_temp, m->samp_seed, 0, m->d_pos, nullptr,
                           m->d_tok, m->tok_log, m->samp_ws, m->samp_ws_bytes, st));
    } else {
      AH_TRY(sample_launch(m->logits, m->nvoc, B, m->nvoc, K, (int64_t)m->tp_rank * m->nvoc, m->samp_temp,
                           m->samp_seed, 0, m->d_pos, m->samp_cand, nullptr, nullptr, m->samp_ws, m->samp_ws_bytes,
                           st));
      if (ncclAllGather(m->samp_cand, m->samp_all, (size_t)B * K * sizeof(SampleCand), ncclUint8, m->comm, st) !=
          ncclSuccess)
        return fail(AH_ENCCL, "model: all-gather of the sampling candidates failed");
      AH_TRY(sample_merge_launch(m->samp_all, m->tp_world, B, K, m->samp_temp, m->samp_seed, m->d_pos, m->d_tok,
                                 m->tok_log, st));
    }
  } else if (with_head) {
    ArgPair* pair = tp ? static_cast<ArgPair*>(m->am_pair) : nullptr;
    AH_TRY(launch_pdl(k_argmax, dim3(kArgmaxChunks, B), dim3(256), 0, st, (const float*)m->logits, m->nvoc, m->am_v,
                      m->am_i, m->am_cnt, m->d_tok, m->tok_log, (const int*)m->d_pos, B, pair,
                      m->tp_rank * m->nvoc));
    if (tp) {
      if (ncclAllGather(m->am_pair, m->am_all, (size_t)B * sizeof(ArgPair), ncclUint8, m->comm, st) != ncclSuccess)
        return fail(AH_ENCCL, "model: all-gather of the argmax candidates failed");
      AH_TRY(launch_pdl(k_argmax_merge, dim3(1), dim3(32), 0, st, (const ArgPair*)m->am_all, m->tp_world, m->d_tok,
                        m->tok_log, (const int*)m->d_pos, B));
    }
  }
  AH_TRY(launch_pdl(k_advance, dim3(1), dim3(32), 0, st, m->d_pos, m->d_tok, prompt, n_prompt, B));
  return AH_OK;
}

// ---- prompt prefill through the GEMMs ---------------------------------------------
// The decoder's only state between steps is the KV cache and the position, so
// the prefill writes the cache for prompt positions 0 .. P-1 of every sequence
// and leaves the position at P with prompt token P next: exactly the state the
// token-by-token prefill (inference/mod.rs:550) leaves.  Positions go in chunks
// of up to kPrefillRows rows (sequences x positions); per chunk and layer the
// projections run as tcgen05 GEMMs and the row kernels of ah_prefill.cu do
// norms, RoPE + KV append, causal attention, SwiGLU and residual adds.  The
// last layer stops after its KV append (its outputs feed nothing cached).
constexpr int kPrefillRows = 2048;
constexpr int kPrefillMinTokens = 8;

int prefill_buffers(AhModel* m) {
  if (m->pf_h) return AH_OK;
  const AhModelConfig& c = m->c;
  const size_t R = kPrefillRows, d = c.n_embd;
  int rc = AH_OK;
  auto A = [&](void** p, size_t bytes) {
    if (rc == AH_OK) rc = dalloc(m, p, bytes);
  };
  A((void**)&m->pf_h, R * d * 4);
  A((void**)&m->pf_qkv, R * (size_t)(m->dq + 2 * m->dkv) * 4);
  A((void**)&m->pf_attn, R * (size_t)m->dq * 4);
  if (m->tp_world > 1) A((void**)&m->pf_part, R * d * 4);
  A((void**)&m->pf_act, R * (size_t)m->nff * 4);
  size_t ws = 0;
  for (const AhQ4Weight* w : {m->wqkv[0], m->wo[0], m->wgu[0], m->wd[0]})
    ws = std::max(ws, gemm_workspace_bytes(q4w_tiled(w), (int64_t)R));
  A(&m->pf_ws, ws + 1024);
  m->pf_ws_bytes = ws;
  return rc;
}

// A block's output projection added into the hidden rows (pf_h += a . W^T).
int block_out(AhModel* m, const AhQ4Weight* w, const float* a, int64_t lda, int64_t rows, void* ws, cudaStream_t st,
              const char* what) {
  const int d = m->c.n_embd;
  if (m->tp_world == 1)
    return gemm_run(q4w_tiled(w), a, lda, rows, m->pf_h, d, ws, m->pf_ws_bytes, st, kGemmEpiAdd);
  AH_TRY(gemm_run(q4w_tiled(w), a, lda, rows, m->pf_part, d, ws, m->pf_ws_bytes, st));
  if (ncclAllReduce(m->pf_part, m->pf_part, (size_t)rows * d, ncclFloat, ncclSum, m->comm, st) != ncclSuccess)
    return fail(AH_ENCCL, "prefill: all-reduce of the %s block output failed", what);
  return prefill_add(m->pf_h, m->pf_part, rows * d, st);
}

int prefill_gemm(AhModel* m, const int* prompt, int n_prompt, int P, cudaStream_t st) {
  const AhModelConfig& c = m->c;
  const int B = m->batch, d = c.n_embd, L = c.n_layer, hd = c.head_dim;
  const int ldq = m->dq + 2 * m->dkv;
  AH_TRY(prefill_buffers(m));
  void* ws = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(m->pf_ws) + 1023) & ~uintptr_t(1023));
  const int C = std::max(1, kPrefillRows / B);
  const float scale = 1.0f / sqrtf((float)hd);  // mod.rs:478
  for (int p0 = 0; p0 < P; p0 += C) {
    const PrefillRows pr{B, std::min(C, P - p0), p0, n_prompt};
    const int64_t rows = (int64_t)B * pr.cnt;
    AH_TRY(prefill_embed(m->tok_embd, prompt, pr, d, c.vocab_size, m->pf_h, st));
    for (int l = 0; l < L; ++l) {
      // RMSNorm inside each GEMM's activation prep
      AH_TRY(gemm_run(q4w_tiled(m->wqkv[l]), m->pf_h, d, rows, m->pf_qkv, ldq, ws, m->pf_ws_bytes, st,
                      kGemmEpiStore, m->attn_norm + (size_t)l * d, c.rms_eps));
      AH_TRY(prefill_rope_append(m->pf_qkv, ldq, m->rope, m->kc, m->vc, l, L, m->nh, m->nkv, hd, c.max_seq, pr, st));
      if (l + 1 == L) break;
      AH_TRY(prefill_attention(m->pf_qkv, ldq, m->kc, m->vc, l, L, m->nh, m->nkv, hd, c.max_seq, scale, pr,
                               m->pf_attn, m->dq, st));
      // one GPU: the o and down GEMMs add into the hidden rows in their
      // epilogue; tensor parallel: partial sums, all-reduce, then the add
      AH_TRY(block_out(m, m->wo[l], m->pf_attn, m->dq, rows, ws, st, "attention"));
      AH_TRY(gemm_run(q4w_tiled(m->wgu[l]), m->pf_h, d, rows, m->pf_act, m->nff, ws, m->pf_ws_bytes, st,
                      kGemmEpiSwiglu, m->ffn_norm + (size_t)l * d, c.rms_eps));
      AH_TRY(block_out(m, m->wd[l], m->pf_act, m->nff, rows, ws, st, "MLP"));
    }
  }
  k_prefill_state<<<1, 32, 0, st>>>(m->d_pos, m->d_tok, prompt, n_prompt, P, B);
  AH_LAUNCH_CHECK();
  m->pos = P;
  return AH_OK;
}

bool use_bgemv(const AhModel* m) { return m->batch >= m->bg_min_batch; }

// Whether a decode GEMV of this weight runs on the tcgen05 batched GEMV.  Its
// time is set by the MMA rate (a 128-row x 16-column tile per ~56 ns per SM,
// whatever the batch), the mma.sync GEMV's grows with the batch: measured on
// the 70B projections and their tensor-parallel slices (bench.py --workload
// bgemv), the tcgen05 kernel wins from 20 MB of Q4 weights at 9-12 sequences
// (K >= 4096) and from 5 MB at 13-16 (K >= 2048; shorter rows leave too few
// steps per row block).  min_batch 1 forces it for every GEMV.
bool bgemv_pays(const AhModel* m, const Q4Tiled& w) {
  if (!use_bgemv(m)) return false;
  if (m->bg_min_batch <= 1) return true;
  const double mb = (double)w.rows * (double)w.cols * 18.0 / 32.0 / 1e6;
  if (m->batch >= 13) return mb >= 5.0 && w.cols >= 2048;
  return mb >= 20.0 && w.cols >= 4096;
}

// One decode-step GEMV: the tcgen05 batched GEMV where it pays, else the
// mma.sync GEMV.
int step_gemv(AhModel* m, const GemvArgs& a, int pro, int epi, cudaStream_t st) {
  if (bgemv_pays(m, a.w)) {
    void* ws = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(m->bg_ws) + 1023) & ~uintptr_t(1023));
    return bgemv_launch(a, pro, epi, ws, m->bg_ws_bytes, st, true);
  }
  return gemv_launch(a, pro, epi, st, true);
}

// Kernel attributes and occupancy are resolved before a capture starts.
int prepare_step(AhModel* m) {
  const AhModelConfig& c = m->c;
  const int B = m->batch;
  if (use_bgemv(m)) {
    if (!m->bg_ws) {
      size_t ws = 0;
      for (const AhQ4Weight* w : {m->lm, m->wqkv[0], m->wo[0], m->wgu[0], m->wd[0]})
        ws = std::max(ws, bgemv_workspace_bytes(q4w_tiled(w)));
      AH_TRY(dalloc(m, &m->bg_ws, ws + 1024));
      m->bg_ws_bytes = ws;
    }
    AH_TRY(bgemv_prepare(q4w_tiled(m->lm), kEpiStore));
    AH_TRY(bgemv_prepare(q4w_tiled(m->lm), kEpiAdd));
    AH_TRY(bgemv_prepare(q4w_tiled(m->lm), kEpiSwiglu));
  }
  AH_TRY(gemv_prepare(q4w_tiled(m->lm), B, kProRmsNorm, kEpiStore));
  AH_TRY(gemv_prepare(q4w_tiled(m->wqkv[0]), B, kProRmsNorm, kEpiStore));
  const int ro = m->tp_world > 1 ? kEpiStore : kEpiAdd;
  AH_TRY(gemv_prepare(q4w_tiled(m->wo[0]), B, kProPlain, ro));
  AH_TRY(gemv_prepare(q4w_tiled(m->wgu[0]), B, kProRmsNorm, kEpiSwiglu));
  AH_TRY(gemv_prepare(q4w_tiled(m->wd[0]), B, kProPlain, ro));
  const size_t attn_smem = attn_smem_bytes(m->nh / m->nkv, c.head_dim);
  AH_CUDA_TRY(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem));
  if (m->attn_tc) {
    // persistent grid: every resident CTA, capped at the largest item count
    const bool w128 = c.head_dim == 128;
    const void* kern = w128 ? (const void*)k_attention_tc<128> : (const void*)k_attention_tc<64>;
    const int smem = w128 ? AttnTcSmem<128>::kAlloc : AttnTcSmem<64>::kAlloc;
    AH_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int per_sm = 0;
    AH_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAttnThreads, smem));
    AH_REQUIRE(per_sm >= 1, "model: the attention kernel does not fit on an SM");
    m->attn_grid = std::min(per_sm * sm_count(), B * m->nkv * kAttnSplits);
  }
  return AH_OK;
}

int run_step_graph(AhModel* m, int which, const int* prompt, int n_prompt, cudaStream_t st) {
  if (!m->g_step[which] || m->g_batch[which] != m->batch || m->g_prompt[which] != prompt ||
      m->g_nprompt[which] != n_prompt) {
    AH_TRY(prepare_step(m));
    if (m->g_step[which]) cudaGraphExecDestroy(m->g_step[which]);
    m->g_step[which] = nullptr;
    cudaStream_t cap;
    AH_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    cudaGraph_t g = nullptr;
    AH_CUDA_TRY(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, which == 1, prompt, n_prompt, cap);
    cudaError_t e = cudaStreamEndCapture(cap, &g);
    cudaStreamDestroy(cap);
    if (rc != AH_OK) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return fail(AH_ECUDA, "model: step capture failed: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(&m->g_step[which], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(AH_ECUDA, "model: step graph instantiate: %s", cudaGetErrorString(e));
    m->g_batch[which] = m->batch;
    m->g_prompt[which] = prompt;
    m->g_nprompt[which] = n_prompt;
  }
  AH_CUDA_TRY(cudaGraphLaunch(m->g_step[which], st));
  m->pos += 1;
  return AH_OK;
}

}  // namespace

extern "C" {

uint64_t ah_model_tensor_seed(uint64_t seed, int kind, int layer) {
  return splitmix64(splitmix64(seed + 0x1000003ull * (uint64_t)(kind + 1)) + (uint64_t)layer);
}

}  // extern "C"

namespace {
// Creates the model (tensor-parallel shard `rank` of `world`, or the whole
// model for world 1) on the current device; takes ownership of `comm`.
int model_create(const AhModelConfig* cfg, int rank, int world, ncclComm_t comm, AhModel** out) {
  AH_REQUIRE(cfg && out, "model_create: null argument");
  *out = nullptr;
  const AhModelConfig& c = *cfg;
  AH_REQUIRE(c.n_layer > 0 && c.n_embd > 0 && c.n_ff > 0 && c.n_head > 0 && c.n_head_kv > 0 && c.head_dim > 0 &&
                 c.vocab_size > 0 && c.max_seq > 0 && c.max_batch >= 1 && c.max_batch <= kGemvMaxBatch,
             "model_create: non-positive dimension or batch outside 1..16");
  AH_REQUIRE(world >= 1 && rank >= 0 && rank < world, "model_create: rank %d of %d", rank, world);
  AH_REQUIRE(c.n_head_kv % world == 0 && c.n_ff % world == 0 && c.vocab_size % world == 0,
             "model_create: %d ranks must divide n_head_kv, n_ff and vocab_size", world);
  const int nh = c.n_head / world, nkv = c.n_head_kv / world, nff = c.n_ff / world, nvoc = c.vocab_size / world;
  AH_REQUIRE(c.n_embd % 64 == 0 && nff % 64 == 0 && (nh * c.head_dim) % 64 == 0,
             "model_create: n_embd, n_ff / ranks and heads per rank * head_dim must be multiples of 64");
  AH_REQUIRE(c.n_head % c.n_head_kv == 0 && c.n_head / c.n_head_kv <= 8, "model_create: GQA group must divide, <= 8");
  AH_REQUIRE(c.head_dim % 32 == 0 && c.head_dim <= 128, "model_create: head_dim must be 32, 64, 96 or 128");
  AH_REQUIRE(c.max_seq <= kAttnSplits * kAttnMaxChunk, "model_create: max_seq above %d", kAttnSplits * kAttnMaxChunk);
  AhModel* m = new (std::nothrow) AhModel();
  if (!m) return fail(AH_ENOMEM, "model_create: host allocation");
  m->c = c;
  m->tp_rank = rank;
  m->tp_world = world;
  m->comm = comm;
  m->nh = nh;
  m->nkv = nkv;
  m->nff = nff;
  m->nvoc = nvoc;
  cudaGetDevice(&m->device);
  m->dq = nh * c.head_dim;
  m->dkv = nkv * c.head_dim;
  const int L = c.n_layer, B = c.max_batch, d = c.n_embd;
  m->wqkv.assign(L, nullptr);
  m->wo.assign(L, nullptr);
  m->wgu.assign(L, nullptr);
  m->wd.assign(L, nullptr);
  for (auto& p : m->pend) p.assign(L, nullptr);
  for (auto& f : m->pend_fmt) f.assign(L, 0);
  int rc = AH_OK;
  auto A = [&](void** p, size_t bytes) {
    if (rc == AH_OK) rc = dalloc(m, p, bytes);
  };
  A((void**)&m->tok_embd, (size_t)c.vocab_size * d * 2);
  A((void**)&m->attn_norm, (size_t)L * d * 2);
  A((void**)&m->ffn_norm, (size_t)L * d * 2);
  A((void**)&m->out_norm, (size_t)d * 2);
  const size_t kv = (size_t)B * L * nkv * c.max_seq * c.head_dim * 2;
  A((void**)&m->kc, kv);
  A((void**)&m->vc, kv);
  A((void**)&m->rope, (size_t)c.max_seq * (c.head_dim / 2) * sizeof(float2));
  A((void**)&m->hidden, (size_t)B * d * 4);
  A((void**)&m->qkv, (size_t)B * (m->dq + 2 * m->dkv) * 4);
  A((void**)&m->attn, (size_t)B * m->dq * 4);
  A((void**)&m->act, (size_t)B * nff * 4);
  A((void**)&m->logits, (size_t)B * nvoc * 4);
  A((void**)&m->ss, (size_t)B * (d / 16) * 4);
  const int G = nh / nkv;
  A((void**)&m->att_part, (size_t)B * nkv * kAttnSplits * G * (c.head_dim + 2) * 4 + 16);
  A((void**)&m->att_cnt, (size_t)B * nkv * 4);
  A((void**)&m->am_v, (size_t)B * kArgmaxChunks * 4);
  A((void**)&m->am_i, (size_t)B * kArgmaxChunks * 4);
  A((void**)&m->am_cnt, (size_t)B * 4);
  A((void**)&m->d_pos, 16);
  A((void**)&m->d_tok, (size_t)B * 4);
  A((void**)&m->tok_log, (size_t)c.max_seq * B * 4);
  if (world > 1) {
    m->comm_flags_off = ((size_t)2 * world * B * d * 4 + 255) / 256 * 256;
    A(&m->comm_block, m->comm_flags_off + 256 + 64);
    A((void**)&m->part, (size_t)B * d * 4);
    A(&m->am_pair, (size_t)B * sizeof(ArgPair));
    A(&m->am_all, (size_t)world * B * sizeof(ArgPair));
  }
  if (rc == AH_OK) {
    m->err = device_error_word();
    if (!m->err) rc = fail(AH_ENOMEM, "model_create: device error word");
  }
  if (rc != AH_OK) {
    ah_model_destroy(m);
    return rc;
  }
  if (m->comm_block) cudaMemset(m->comm_block, 0, m->comm_flags_off + 256 + 64);
  cudaMemset(m->att_cnt, 0, (size_t)B * nkv * 4);
  cudaMemset(m->am_cnt, 0, (size_t)B * 4);
  cudaMemset(m->kc, 0, kv);
  cudaMemset(m->vc, 0, kv);
  cudaMemset(m->d_pos, 0, 16);
  cudaMemset(m->d_tok, 0, (size_t)B * 4);
  if (c.head_dim == 64 || c.head_dim == 128) {
    const uint64_t kv_rows = (uint64_t)B * L * nkv * c.max_seq;
    rc = encode_2d(&m->tm_k, m->kc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)c.head_dim, kv_rows, 64,
                   kAttnBoxRows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == AH_OK)
      rc = encode_2d(&m->tm_v, m->vc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)c.head_dim, kv_rows, 64,
                     kAttnBoxRows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != AH_OK) {
      ah_model_destroy(m);
      return rc;
    }
    m->attn_tc = true;
  }
  const int n = c.max_seq * (c.head_dim / 2);
  k_rope_table<<<(n + 255) / 256, 256>>>(m->rope, c.max_seq, c.head_dim / 2, c.rope_freq_base);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    ah_model_destroy(m);
    return fail(AH_ECUDA, "model_create: %s", cudaGetErrorString(e));
  }
  *out = m;
  return AH_OK;
}
}  // namespace

extern "C" {

int ah_model_create(const AhModelConfig* cfg, AhModel** out) { return model_create(cfg, 0, 1, nullptr, out); }

int ah_nccl_unique_id(void* id_out, size_t bytes) {
  AH_REQUIRE(id_out && bytes >= sizeof(ncclUniqueId), "nccl_unique_id: need a %zu-byte buffer", sizeof(ncclUniqueId));
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return fail(AH_ENCCL, "ncclGetUniqueId failed");
  std::memcpy(id_out, &id, sizeof(id));
  return AH_OK;
}

int ah_model_create_tp(const AhModelConfig* cfg, int rank, int world, const void* nccl_id, AhModel** out) {
  AH_REQUIRE(cfg && out && nccl_id, "model_create_tp: null argument");
  AH_REQUIRE(world >= 1 && rank >= 0 && rank < world, "model_create_tp: rank %d of %d", rank, world);
  ncclComm_t comm = nullptr;
  if (world > 1) {
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    if (inject_failure(AH_INJECT_NCCL))
      return fail(AH_ENCCL, "ncclCommInitRank(rank %d of %d) failed (injected)", rank, world);
    if (ncclCommInitRank(&comm, world, id, rank) != ncclSuccess)
      return fail(AH_ENCCL, "ncclCommInitRank(rank %d of %d) failed", rank, world);
  }
  const int rc = model_create(cfg, rank, world, comm, out);
  if (rc != AH_OK && comm) ncclCommDestroy(comm);
  return rc;
}

int ah_debug_residual_add_peer(float* hidden, const float* slots, int world, int batch, int d, float* ss,
                               const unsigned* flags, const unsigned* seq, void* stream) {
  AH_REQUIRE(hidden && slots && ss && flags && seq, "debug_residual_add_peer: null argument");
  AH_REQUIRE(world >= 1 && world <= 8 && batch >= 1 && batch <= 16 && d > 0 && d % 16 == 0,
             "debug_residual_add_peer: world 1..8, batch 1..16, d a positive multiple of 16");
  int* err = device_error_word();
  AH_REQUIRE(err != nullptr, "debug_residual_add_peer: device error word unavailable");
  k_residual_add_peer<<<dim3((d + 255) / 256, batch), 256, 0, as_stream(stream)>>>(hidden, slots, world, batch, ss, d,
                                                                                   flags, seq, err);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_model_ipc_handle(AhModel* m, void* handle_out, size_t bytes) {
  AH_REQUIRE(m && handle_out && bytes >= sizeof(cudaIpcMemHandle_t), "model_ipc_handle: need a %zu-byte buffer",
             sizeof(cudaIpcMemHandle_t));
  AH_REQUIRE(m->tp_world > 1 && m->comm_block, "model_ipc_handle: not a tensor-parallel model");
  cudaIpcMemHandle_t h;
  AH_CUDA_TRY(cudaIpcGetMemHandle(&h, m->comm_block));
  std::memcpy(handle_out, &h, sizeof(h));
  return AH_OK;
}

int ah_model_ipc_open(AhModel* m, const void* handles, size_t bytes) {
  AH_REQUIRE(m && handles, "model_ipc_open: null argument");
  const int W = m->tp_world;
  AH_REQUIRE(W > 1 && W <= 8 && m->comm_block, "model_ipc_open: not a tensor-parallel model of <= 8 ranks");
  AH_REQUIRE(bytes >= (size_t)W * sizeof(cudaIpcMemHandle_t), "model_ipc_open: need %d handles", W);
  AH_REQUIRE(!m->p2p, "model_ipc_open: already open");
  const auto* hs = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < W; ++r) {
    if (r == m->tp_rank) {
      m->peer_block[r] = m->comm_block;
      continue;
    }
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, hs[r], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != m->tp_rank && m->peer_block[q]) cudaIpcCloseMemHandle(m->peer_block[q]);
      return fail(AH_ECUDA, "model_ipc_open: rank %d's buffer: %s", r, cudaGetErrorString(e));
    }
    m->peer_block[r] = p;
  }
  m->p2p = true;
  for (auto& g : m->g_step)  // graphs captured with the NCCL path are stale
    if (g) {
      cudaGraphExecDestroy(g);
      g = nullptr;
    }
  return AH_OK;
}

int ah_model_shard(const AhModel* m, int* rank, int* world, int* n_head, int* n_head_kv, int* n_ff, int* vocab) {
  AH_REQUIRE(m, "model_shard: null model");
  if (rank) *rank = m->tp_rank;
  if (world) *world = m->tp_world;
  if (n_head) *n_head = m->nh;
  if (n_head_kv) *n_head_kv = m->nkv;
  if (n_ff) *n_ff = m->nff;
  if (vocab) *vocab = m->nvoc;
  return AH_OK;
}

int ah_model_destroy(AhModel* m) {
  if (!m) return AH_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(m->device);
  for (auto& g : m->g_step)
    if (g) cudaGraphExecDestroy(g);
  for (auto* w : m->wqkv) ah_q4w_destroy(w);
  for (auto* w : m->wo) ah_q4w_destroy(w);
  for (auto* w : m->wgu) ah_q4w_destroy(w);
  for (auto* w : m->wd) ah_q4w_destroy(w);
  ah_q4w_destroy(m->lm);
  for (auto& v : m->pend)
    for (void* p : v)
      if (p) cudaFree(p);
  if (m->p2p)
    for (int r = 0; r < m->tp_world; ++r)
      if (r != m->tp_rank && m->peer_block[r]) cudaIpcCloseMemHandle(m->peer_block[r]);
  for (void* p : m->allocs) cudaFree(p);
  if (m->d_prompt) cudaFree(m->d_prompt);
  if (m->comm) ncclCommDestroy(m->comm);
  cudaSetDevice(cur);
  delete m;
  return AH_OK;
}

}  // extern "C"

namespace {
// One projection's source: Q4_0 blocks, or the engine format that quantize()
// returns (quantization.rs:369-404: f32 scale per 32-column group, packed
// nibbles with the even element in the low nibble).
enum ProjFormat : int { kProjQ4_0 = 0, kProjEngine = 1 };
struct ProjSrc {
  int fmt;
  const void* q4;
  const float* scales;
  const uint8_t* packed;
};

size_t proj_scale_bytes(int64_t rows, int64_t cols) { return (size_t)rows * (cols / 32) * 4; }
size_t proj_bytes(int fmt, int64_t rows, int64_t cols) {
  return fmt == kProjQ4_0 ? (size_t)rows * (cols / 32) * 18 : proj_scale_bytes(rows, cols) + (size_t)rows * cols / 2;
}

// Loads (or replaces) one projection.  o, down and the LM head are repacked at
// once; q/k/v and gate/up wait in staging until their group is complete, then
// become one fused weight (q|k|v stacked, gate/up interleaved by 8 rows).  The
// parts of a group must share a format.
int load_projection(AhModel* m, int kind, int layer, const ProjSrc& src, cudaStream_t st) {
  const int d = m->c.n_embd;
  auto direct = [&](AhQ4Weight*& w, int64_t rows, int64_t cols) -> int {
    if (w) ah_q4w_destroy(w);
    w = nullptr;
    if (src.fmt == kProjQ4_0) return ah_q4w_from_q4_0(src.q4, rows, cols, &w, st);
    return ah_q4w_from_engine(src.scales, src.packed, rows, cols, &w, st);
  };
  if (kind == AH_T_WO) return direct(m->wo[layer], d, m->dq);
  if (kind == AH_T_WDOWN) return direct(m->wd[layer], d, m->nff);
  if (kind == AH_T_LM_HEAD) return direct(m->lm, m->nvoc, d);
  const int slot = kind == AH_T_WQ ? 0 : kind == AH_T_WK ? 1 : kind == AH_T_WV ? 2 : kind == AH_T_WGATE ? 3 : 4;
  const int64_t rows = slot == 0 ? m->dq : slot <= 2 ? m->dkv : m->nff;
  void*& p = m->pend[slot][layer];
  if (p && m->pend_fmt[slot][layer] != src.fmt) {
    cudaFree(p);
    p = nullptr;
  }
  if (!p && ah::dev_malloc(&p, proj_bytes(src.fmt, rows, d)) != cudaSuccess) {
    cudaGetLastError();
    p = nullptr;
    return fail(AH_ENOMEM, "model_load_tensor: staging of %zu bytes", proj_bytes(src.fmt, rows, d));
  }
  m->pend_fmt[slot][layer] = src.fmt;
  if (src.fmt == kProjQ4_0) {
    AH_CUDA_TRY(cudaMemcpyAsync(p, src.q4, proj_bytes(src.fmt, rows, d), cudaMemcpyDeviceToDevice, st));
  } else {
    const size_t sb = proj_scale_bytes(rows, d);
    AH_CUDA_TRY(cudaMemcpyAsync(p, src.scales, sb, cudaMemcpyDeviceToDevice, st));
    AH_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(p) + sb, src.packed, (size_t)rows * d / 2,
                                cudaMemcpyDeviceToDevice, st));
  }
  const bool qkv = slot <= 2;
  const int k0 = qkv ? 0 : 3, nsrc = qkv ? 3 : 2;
  for (int k = k0; k < k0 + nsrc; ++k)
    if (!m->pend[k][layer]) return AH_OK;  // the group is not complete yet
  for (int k = k0; k < k0 + nsrc; ++k)
    AH_REQUIRE(m->pend_fmt[k][layer] == src.fmt, "model_load_tensor: %s of layer %d mix Q4_0 and engine formats",
               qkv ? "q, k and v" : "gate and up", layer);
  const int64_t rws[3] = {qkv ? m->dq : m->nff, qkv ? m->dkv : m->nff, m->dkv};
  AhQ4Weight*& w = qkv ? m->wqkv[layer] : m->wgu[layer];
  if (w) ah_q4w_destroy(w);
  w = nullptr;
  if (src.fmt == kProjQ4_0) {
    const void* srcs[3] = {m->pend[k0][layer], m->pend[k0 + 1][layer], qkv ? m->pend[2][layer] : nullptr};
    AH_TRY(q4w_create_q4_0_multi(srcs, rws, nsrc, qkv ? 0 : 1, d, &w, st));
  } else {
    const float* sc[3] = {};
    const uint8_t* pk[3] = {};
    for (int k = 0; k < nsrc; ++k) {
      sc[k] = static_cast<const float*>(m->pend[k0 + k][layer]);
      pk[k] = static_cast<const uint8_t*>(m->pend[k0 + k][layer]) + proj_scale_bytes(rws[k], d);
    }
    AH_TRY(q4w_create_engine_multi(sc, pk, rws, nsrc, qkv ? 0 : 1, d, &w, st));
  }
  AH_CUDA_TRY(cudaStreamSynchronize(st));
  for (int k = k0; k < k0 + nsrc; ++k) {
    cudaFree(m->pend[k][layer]);
    m->pend[k][layer] = nullptr;
  }
  return AH_OK;
}

bool is_projection(int kind) { return kind >= AH_T_WQ && kind <= AH_T_LM_HEAD; }
}  // namespace

extern "C" {

int ah_model_load_tensor(AhModel* m, int kind, int layer, const void* data, void* stream) {
  AH_REQUIRE(m && data, "model_load_tensor: null argument");
  const AhModelConfig& c = m->c;
  const int d = c.n_embd;
  cudaStream_t st = as_stream(stream);
  const bool per_layer = !(kind == AH_T_TOK_EMBD || kind == AH_T_OUT_NORM || kind == AH_T_LM_HEAD);
  AH_REQUIRE(!per_layer || (layer >= 0 && layer < c.n_layer), "model_load_tensor: layer %d out of range", layer);
  switch (kind) {
    case AH_T_TOK_EMBD:
      AH_CUDA_TRY(cudaMemcpyAsync(m->tok_embd, data, (size_t)c.vocab_size * d * 2, cudaMemcpyDeviceToDevice, st));
      return AH_OK;
    case AH_T_ATTN_NORM:
      AH_CUDA_TRY(cudaMemcpyAsync(m->attn_norm + (size_t)layer * d, data, (size_t)d * 2, cudaMemcpyDeviceToDevice, st));
      return AH_OK;
    case AH_T_FFN_NORM:
      AH_CUDA_TRY(cudaMemcpyAsync(m->ffn_norm + (size_t)layer * d, data, (size_t)d * 2, cudaMemcpyDeviceToDevice, st));
      return AH_OK;
    case AH_T_OUT_NORM:
      AH_CUDA_TRY(cudaMemcpyAsync(m->out_norm, data, (size_t)d * 2, cudaMemcpyDeviceToDevice, st));
      return AH_OK;
    case AH_T_WO: case AH_T_WDOWN: case AH_T_LM_HEAD: case AH_T_WQ: case AH_T_WK: case AH_T_WV: case AH_T_WGATE:
    case AH_T_WUP: {
      ProjSrc src{};
      src.fmt = kProjQ4_0;
      src.q4 = data;
      return load_projection(m, kind, layer, src, st);
    }
    default:
      return fail(AH_EINVAL, "model_load_tensor: unknown kind %d", kind);
  }
}

int ah_model_load_tensor_engine(AhModel* m, int kind, int layer, const float* scales, const uint8_t* packed,
                                void* stream) {
  AH_REQUIRE(m && scales && packed, "model_load_tensor_engine: null argument");
  AH_REQUIRE(is_projection(kind), "model_load_tensor_engine: kind %d is not a projection", kind);
  AH_REQUIRE(kind == AH_T_LM_HEAD || (layer >= 0 && layer < m->c.n_layer),
             "model_load_tensor_engine: layer %d out of range", layer);
  ProjSrc src{};
  src.fmt = kProjEngine;
  src.scales = scales;
  src.packed = packed;
  return load_projection(m, kind, layer, src, as_stream(stream));
}

int ah_model_load_tensor_f32(AhModel* m, int kind, int layer, const float* data, void* stream) {
  AH_REQUIRE(m && data, "model_load_tensor_f32: null argument");
  const AhModelConfig& c = m->c;
  const int d = c.n_embd;
  const bool per_layer = !(kind == AH_T_TOK_EMBD || kind == AH_T_OUT_NORM || kind == AH_T_LM_HEAD);
  AH_REQUIRE(!per_layer || (layer >= 0 && layer < c.n_layer), "model_load_tensor_f32: layer %d out of range", layer);
  if (!is_projection(kind)) {  // embeddings and norms are held as f16 (round to nearest even)
    uint16_t* dst = kind == AH_T_TOK_EMBD    ? m->tok_embd
                    : kind == AH_T_ATTN_NORM ? m->attn_norm + (size_t)layer * d
                    : kind == AH_T_FFN_NORM  ? m->ffn_norm + (size_t)layer * d
                    : kind == AH_T_OUT_NORM  ? m->out_norm
                                             : nullptr;
    AH_REQUIRE(dst, "model_load_tensor_f32: unknown kind %d", kind);
    return ah_f32_to_f16(data, dst, kind == AH_T_TOK_EMBD ? (int64_t)c.vocab_size * d : d, stream);
  }
  // quantize() with group 32 (inference/mod.rs:267), then the engine-format load
  const int64_t rows = kind == AH_T_WQ || kind == AH_T_WO ? (kind == AH_T_WQ ? m->dq : d)
                       : kind == AH_T_WK || kind == AH_T_WV ? m->dkv
                       : kind == AH_T_WGATE || kind == AH_T_WUP ? m->nff
                       : kind == AH_T_LM_HEAD ? m->nvoc
                                              : d;
  const int64_t cols = kind == AH_T_WO ? m->dq : kind == AH_T_WDOWN ? m->nff : d;
  const int64_t n = rows * cols;
  float* sc = nullptr;
  uint8_t* pk = nullptr;
  if (ah::dev_malloc(&sc, (size_t)(n / 32) * 4) != cudaSuccess || ah::dev_malloc(&pk, (size_t)n / 2) != cudaSuccess) {
    cudaGetLastError();
    if (sc) cudaFree(sc);
    return fail(AH_ENOMEM, "model_load_tensor_f32: quantization buffers of %lld elements", (long long)n);
  }
  int rc = ah_quantize_q4(data, n, 32, sc, pk, stream);
  if (rc == AH_OK) rc = ah_model_load_tensor_engine(m, kind, layer, sc, pk, stream);
  if (rc == AH_OK && cudaStreamSynchronize(as_stream(stream)) != cudaSuccess)
    rc = fail(AH_ECUDA, "model_load_tensor_f32: %s", cudaGetErrorString(cudaGetLastError()));
  cudaFree(sc);
  cudaFree(pk);
  return rc;
}

int ah_model_init_random(AhModel* m, uint64_t seed, float w_std, float emb_std, float norm_std) {
  AH_REQUIRE(m, "model_init_random: null model");
  const AhModelConfig& c = m->c;
  const int d = c.n_embd;
  cudaStream_t st = nullptr;
  AH_TRY(ah_synth_f16(m->tok_embd, (int64_t)c.vocab_size * d, 0.0f, emb_std, ah_model_tensor_seed(seed, AH_T_TOK_EMBD, 0),
                      0, st));
  AH_TRY(ah_synth_f16(m->out_norm, d, 1.0f, norm_std, ah_model_tensor_seed(seed, AH_T_OUT_NORM, 0), 0, st));
  // each rank draws its slice of the same full logical tensors, so a sharded
  // model computes what the whole one does: row slices of q/k/v/gate/up/LM
  // head, column slices of o/down (synth draws element (r, c) of the full
  // matrix wherever the slice starts)
  const int R = m->tp_rank;
  const int64_t max_rows = std::max<int64_t>({(int64_t)m->dq, (int64_t)m->nff, (int64_t)d});
  const int64_t max_cols = std::max<int64_t>({(int64_t)m->dq, (int64_t)m->nff, (int64_t)d});
  void* tmp = nullptr;
  const size_t tmp_bytes = (size_t)std::max<int64_t>(max_rows * (d / 32), (int64_t)d * (max_cols / 32)) * 18;
  if (ah::dev_malloc(&tmp, tmp_bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(AH_ENOMEM, "model_init_random: staging of %zu bytes", tmp_bytes);
  }
  struct Spec { int kind; int64_t row0, rows, col0, cols, full_cols; };
  const int64_t dq_full = (int64_t)c.n_head * c.head_dim, dkv_full = (int64_t)c.n_head_kv * c.head_dim;
  const Spec specs[7] = {{AH_T_WQ, (int64_t)R * m->dq, m->dq, 0, d, d},
                         {AH_T_WK, (int64_t)R * m->dkv, m->dkv, 0, d, d},
                         {AH_T_WV, (int64_t)R * m->dkv, m->dkv, 0, d, d},
                         {AH_T_WO, 0, d, (int64_t)R * m->dq, m->dq, dq_full},
                         {AH_T_WGATE, (int64_t)R * m->nff, m->nff, 0, d, d},
                         {AH_T_WUP, (int64_t)R * m->nff, m->nff, 0, d, d},
                         {AH_T_WDOWN, 0, d, (int64_t)R * m->nff, m->nff, (int64_t)c.n_ff}};
  (void)dkv_full;
  int rc = AH_OK;
  for (int l = 0; l < c.n_layer && rc == AH_OK; ++l) {
    rc = ah_synth_f16(m->attn_norm + (size_t)l * d, d, 1.0f, norm_std, ah_model_tensor_seed(seed, AH_T_ATTN_NORM, l),
                      0, st);
    if (rc == AH_OK)
      rc = ah_synth_f16(m->ffn_norm + (size_t)l * d, d, 1.0f, norm_std, ah_model_tensor_seed(seed, AH_T_FFN_NORM, l),
                        0, st);
    for (const Spec& sp : specs) {
      if (rc != AH_OK) break;
      rc = ah_synth_q4_0(tmp, sp.row0, sp.rows, sp.col0, sp.cols, sp.full_cols, w_std,
                         ah_model_tensor_seed(seed, sp.kind, l), st);
      if (rc == AH_OK) rc = ah_model_load_tensor(m, sp.kind, l, tmp, st);
    }
  }
  if (rc == AH_OK) {
    // the LM head is the largest tensor: generate this rank's rows in their own buffer
    void* lmb = nullptr;
    if (ah::dev_malloc(&lmb, (size_t)m->nvoc * (d / 32) * 18) != cudaSuccess) {
      cudaGetLastError();
      rc = fail(AH_ENOMEM, "model_init_random: output.weight staging");
    } else {
      rc = ah_synth_q4_0(lmb, (int64_t)R * m->nvoc, m->nvoc, 0, d, d, w_std,
                         ah_model_tensor_seed(seed, AH_T_LM_HEAD, 0), st);
      if (rc == AH_OK) rc = ah_model_load_tensor(m, AH_T_LM_HEAD, 0, lmb, st);
      cudaStreamSynchronize(st);
      cudaFree(lmb);
    }
  }
  cudaStreamSynchronize(st);
  cudaFree(tmp);
  return rc;
}

int ah_model_reset(AhModel* m, int batch, void* stream) {
  AH_REQUIRE(m && batch >= 1 && batch <= m->c.max_batch, "model_reset: batch must be 1..max_batch");
  AH_TRY(model_ready(m));
  cudaStream_t st = as_stream(stream);
  m->batch = batch;
  m->pos = 0;
  AH_CUDA_TRY(cudaMemsetAsync(m->d_pos, 0, 4, st));
  return AH_OK;
}

int ah_model_set_sampling(AhModel* m, float temperature, int top_k, uint64_t seed) {
  AH_REQUIRE(m, "model_set_sampling: null model");
  AH_REQUIRE(!(temperature > 0.0f) || (top_k >= 1 && top_k <= kSampleMaxK),
             "model_set_sampling: top_k must be 1..%d", kSampleMaxK);
  AH_REQUIRE(m->tp_world <= kSampleMaxRanks, "model_set_sampling: more than %d ranks", kSampleMaxRanks);
  if (temperature > 0.0f && !m->samp_cand) {
    const size_t per = (size_t)m->c.max_batch * kSampleMaxK * sizeof(SampleCand);
    AH_TRY(dalloc(m, (void**)&m->samp_cand, per));
    AH_TRY(dalloc(m, (void**)&m->samp_all, per * m->tp_world));
    m->samp_ws_bytes = sample_workspace_bytes(m->c.max_batch, m->nvoc);
    if (m->samp_ws_bytes) AH_TRY(dalloc(m, &m->samp_ws, m->samp_ws_bytes));
  }
  m->samp_temp = temperature > 0.0f ? temperature : 0.0f;
  m->samp_k = top_k;
  m->samp_seed = seed;
  // the captured steps hold the other head: capture again on the next step
  for (int i = 0; i < 2; ++i) {
    if (m->g_step[i]) cudaGraphExecDestroy(m->g_step[i]);
    m->g_step[i] = nullptr;
  }
  return AH_OK;
}

int ah_model_set_batched_gemv(AhModel* m, int min_batch) {
  AH_REQUIRE(m && min_batch >= 1 && min_batch <= kGemvMaxBatch + 1,
             "model_set_batched_gemv: min_batch must be 1..17");
  if (m->bg_min_batch == min_batch) return AH_OK;
  m->bg_min_batch = min_batch;
  // the captured steps hold the other GEMV: capture again on the next step
  for (int i = 0; i < 2; ++i) {
    if (m->g_step[i]) cudaGraphExecDestroy(m->g_step[i]);
    m->g_step[i] = nullptr;
  }
  return AH_OK;
}

int ah_model_set_prefill(AhModel* m, int mode) {
  AH_REQUIRE(m && (mode == 0 || mode == 1), "model_set_prefill: mode must be 0 or 1");
  m->pf_mode = mode;
  return AH_OK;
}

int ah_model_position(const AhModel* m, int* pos) {
  AH_REQUIRE(m && pos, "model_position: null argument");
  *pos = m->pos;
  return AH_OK;
}

int ah_model_forward(AhModel* m, const int32_t* tokens, float* logits, void* stream) {
  AH_REQUIRE(m && tokens, "model_forward: null argument");
  AH_REQUIRE(m->pos < m->c.max_seq, "model_forward: KV cache full (max_seq %d)", m->c.max_seq);
  cudaStream_t st = as_stream(stream);
  AH_CUDA_TRY(cudaMemcpyAsync(m->d_tok, tokens, (size_t)m->batch * 4, cudaMemcpyDeviceToDevice, st));
  AH_TRY(run_step_graph(m, 1, nullptr, 0, st));
  if (logits)
    AH_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, (size_t)m->batch * m->nvoc * 4, cudaMemcpyDeviceToDevice,
                                st));
  return AH_OK;
}

int ah_model_decode(AhModel* m, int n, int32_t* out, void* stream) {
  AH_REQUIRE(m && n >= 0, "model_decode: bad arguments");
  AH_REQUIRE(m->pos >= 1, "model_decode: feed at least one token first");
  AH_REQUIRE(m->pos + n <= m->c.max_seq + 1, "model_decode: would exceed max_seq");
  cudaStream_t st = as_stream(stream);
  // token i of the output is the argmax taken after position pos-1+i
  const int first = m->pos - 1;
  for (int i = 0; i < n; ++i) {
    if (i > 0) AH_TRY(run_step_graph(m, 1, nullptr, 0, st));
  }
  if (out && n > 0)
    AH_CUDA_TRY(cudaMemcpyAsync(out, m->tok_log + (size_t)first * m->batch, (size_t)n * m->batch * 4,
                                cudaMemcpyDeviceToDevice, st));
  return AH_OK;
}

int ah_model_generate(AhModel* m, const int32_t* prompt, int batch, int n_prompt, int n_new, int32_t* out,
                      void* stream) {
  AH_REQUIRE(m && prompt && n_prompt >= 1 && n_new >= 0, "model_generate: bad arguments");
  AH_REQUIRE(n_prompt + n_new - 1 <= m->c.max_seq, "model_generate: prompt + new tokens exceed max_seq");
  cudaStream_t st = as_stream(stream);
  AH_TRY(ah_model_reset(m, batch, stream));
  if (m->d_prompt) cudaFree(m->d_prompt);
  m->d_prompt = nullptr;
  if (ah::dev_malloc(&m->d_prompt, (size_t)batch * n_prompt * 4) != cudaSuccess) {
    cudaGetLastError();
    return fail(AH_ENOMEM, "model_generate: prompt buffer");
  }
  AH_CUDA_TRY(cudaMemcpyAsync(m->d_prompt, prompt, (size_t)batch * n_prompt * 4, cudaMemcpyHostToDevice, st));
  // first prompt token of every sequence
  std::vector<int32_t> first(batch);
  for (int b = 0; b < batch; ++b) first[b] = prompt[(size_t)b * n_prompt];
  AH_CUDA_TRY(cudaMemcpyAsync(m->d_tok, first.data(), (size_t)batch * 4, cudaMemcpyHostToDevice, st));
  AH_CUDA_TRY(cudaStreamSynchronize(st));
  if (m->pf_mode == 1 && n_prompt - 1 >= kPrefillMinTokens)
    AH_TRY(prefill_gemm(m, m->d_prompt, n_prompt, n_prompt - 1, st));  // positions 0 .. n_prompt-2
  else
    for (int p = 0; p + 1 < n_prompt; ++p) AH_TRY(run_step_graph(m, 0, m->d_prompt, n_prompt, st));
  if (n_new == 0) {
    AH_CUDA_TRY(cudaStreamSynchronize(st));
    return AH_OK;
  }
  AH_TRY(run_step_graph(m, 1, nullptr, 0, st));  // last prompt token: logits -> first new token
  for (int i = 1; i < n_new; ++i) AH_TRY(run_step_graph(m, 1, nullptr, 0, st));
  if (out)
    AH_CUDA_TRY(cudaMemcpyAsync(out, m->tok_log + (size_t)(n_prompt - 1) * batch, (size_t)n_new * batch * 4,
                                cudaMemcpyDeviceToHost, st));
  AH_CUDA_TRY(cudaStreamSynchronize(st));
  return AH_OK;
}

}  // extern "C"
