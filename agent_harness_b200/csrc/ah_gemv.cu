// ah_gemv.cu — weight upload/repack into the tiled Q4 layout, the fused
// dequant+GEMV kernel (batch 1..16) with its prologue/epilogue variants, and
// the C-ABI entry points built on it.  Layout and arithmetic: ah_gemv.cuh.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "ah_gemv.cuh"
#include "ah_gemv_impl.cuh"

using namespace ah;

// ---------------------------------------------------------------------------
// Weight handle
// ---------------------------------------------------------------------------
struct AhQ4Weight {
  int device = 0;
  Q4Tiled t{};
  int64_t weight_bytes = 0;
  void* nib_alloc = nullptr;
  void* scale_alloc = nullptr;
  GemvWorkspace ws;  // lazily sized k-split workspace for ah_q4w_gemv
  std::mutex mu;
};

namespace ah {
namespace {

constexpr int kThreads = 256;

// Source of combined row R of a repacked matrix.
struct RowSource {
  int mode;              // 0 = concat of up to 3 sources, 1 = interleave 8 rows of src0 / 8 rows of src1
  int64_t rows[3];
  const uint8_t* q4_0[3];   // Q4_0 blocks, [src_rows][cols/32][18]
  const float* eng_s[3];    // engine scales [src_rows][ceil(cols/32)]
  const uint8_t* eng_p[3];  // engine packed nibbles, linear index src_row*cols + col
};

__device__ __forceinline__ bool map_row(const RowSource& s, int64_t R, int& src, int64_t& sr) {
  if (s.mode == 1) {
    const int64_t T = R >> 4, i = R & 15;
    src = (int)(i >> 3);
    sr = T * 8 + (i & 7);
    return sr < s.rows[src];
  }
  int64_t r = R;
  for (int k = 0; k < 3; ++k) {
    if (r < s.rows[k]) { src = k; sr = r; return true; }
    r -= s.rows[k];
  }
  return false;
}

// One thread per (tile, pair, lane): gathers 4 words of 8 nibbles in fragment
// order (see ah_gemv.cuh) and, for t == 0, the 4 scales of row pair g.
template <bool kEngine>
__global__ void __launch_bounds__(kThreads) k_repack(uint4* __restrict__ nib, void* __restrict__ scales, RowSource src,
                                                     int64_t rows, int64_t cols, int64_t r16, int64_t kp) {
  const int64_t total = r16 * kp * 32;
  const int64_t nb_src = (cols + 31) / 32;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int lane = (int)(idx & 31);
    const int64_t tp = idx >> 5;
    const int64_t rt = tp / kp, p = tp % kp;
    const int g = lane >> 2, t = lane & 3;
    uint32_t words[4];
    float dsc[4];
    uint32_t dh[4];
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      const int blk = wi >> 1, half = wi & 1;
      const int64_t R = rt * 16 + g + 8 * half;
      const int64_t b = 2 * p + blk;
      uint32_t word = 0;
      float d = 0.0f;
      uint32_t dbits = 0;
      int s = 0;
      int64_t sr = 0;
      const bool live_row = R < rows && map_row(src, R, s, sr) && b < nb_src;
      if (live_row) {
        if (kEngine) {
          d = src.eng_s[s][sr * nb_src + b];
        } else {
          const uint8_t* bp = src.q4_0[s] + (sr * nb_src + b) * 18;
          dbits = (uint32_t)bp[0] | ((uint32_t)bp[1] << 8);
        }
      }
#pragma unroll
      for (int pp = 0; pp < 8; ++pp) {
        const int e = 2 * t + 8 * (pp & 3) + (pp >> 2);
        uint32_t q = 8;  // padding: weight (8-8)*d = 0
        if (live_row && b * 32 + e < cols) {
          if (kEngine) {
            const int64_t lin = sr * cols + b * 32 + e;
            const uint32_t byte = src.eng_p[s][lin >> 1];
            q = (lin & 1) ? (byte >> 4) & 0xFu : byte & 0xFu;
          } else {
            const uint32_t byte = src.q4_0[s][(sr * nb_src + b) * 18 + 2 + (e >> 1)];
            q = (e & 1) ? (byte >> 4) & 0xFu : byte & 0xFu;
          }
        }
        word |= q << (4 * pp);
      }
      words[wi] = word;
      dsc[wi] = live_row ? d : 0.0f;
      dh[wi] = live_row ? dbits : 0u;
    }
    nib[idx] = make_uint4(words[0], words[1], words[2], words[3]);
    if (t == 0) {
      const int64_t si = tp * 8 + g;
      if (kEngine) {
        reinterpret_cast<float4*>(scales)[si] = make_float4(dsc[0], dsc[1], dsc[2], dsc[3]);
      } else {
        // f16 scales are copied bit-for-bit from the blocks.
        reinterpret_cast<uint2*>(scales)[si] = make_uint2(dh[0] | (dh[1] << 16), dh[2] | (dh[3] << 16));
      }
    }
  }
}

}  // namespace

int q4w_create(const RowSource& src, bool engine, int64_t rows, int64_t cols, AhQ4Weight** out, cudaStream_t st) {
  AH_REQUIRE(out != nullptr, "q4w_create: null out");
  *out = nullptr;
  AH_REQUIRE(rows > 0 && cols > 0, "q4w_create: rows and cols must be positive");
  AH_REQUIRE(cols % 32 == 0 || engine, "q4w_create: Q4_0 sources need cols %% 32 == 0");
  AhQ4Weight* w = new (std::nothrow) AhQ4Weight();
  if (!w) return fail(AH_ENOMEM, "q4w_create: host allocation failed");
  cudaGetDevice(&w->device);
  const int64_t nb = (cols + 31) / 32;
  w->t.rows = rows;
  w->t.cols = cols;
  w->t.r16 = (rows + 15) / 16;
  w->t.kp = (nb + 1) / 2;
  w->t.f32_scales = engine;
  const size_t nib_bytes = (size_t)w->t.r16 * w->t.kp * 32 * 16;
  const size_t sc_bytes = (size_t)w->t.r16 * w->t.kp * 8 * (engine ? 16 : 8);
  if (cudaMalloc(&w->nib_alloc, nib_bytes) != cudaSuccess || cudaMalloc(&w->scale_alloc, sc_bytes) != cudaSuccess) {
    cudaGetLastError();
    if (w->nib_alloc) cudaFree(w->nib_alloc);
    if (w->scale_alloc) cudaFree(w->scale_alloc);
    delete w;
    return fail(AH_ENOMEM, "q4w_create: cudaMalloc of %zu bytes failed", nib_bytes + sc_bytes);
  }
  w->t.nib = static_cast<const uint4*>(w->nib_alloc);
  w->t.scales = w->scale_alloc;
  w->weight_bytes = engine ? rows * ((cols + 1) / 2) + rows * nb * 4 : rows * nb * 18;
  const int64_t total = w->t.r16 * w->t.kp * 32;
  int64_t grid = (total + kThreads - 1) / kThreads;
  grid = std::min<int64_t>(grid, (int64_t)sm_count() * 16);
  if (engine)
    k_repack<true><<<(int)grid, kThreads, 0, st>>>(static_cast<uint4*>(w->nib_alloc), w->scale_alloc, src, rows, cols,
                                                   w->t.r16, w->t.kp);
  else
    k_repack<false><<<(int)grid, kThreads, 0, st>>>(static_cast<uint4*>(w->nib_alloc), w->scale_alloc, src, rows, cols,
                                                    w->t.r16, w->t.kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFree(w->nib_alloc);
    cudaFree(w->scale_alloc);
    delete w;
    return fail(AH_ECUDA, "q4w_create: repack launch failed: %s", cudaGetErrorString(e));
  }
  *out = w;
  return AH_OK;
}

int q4w_create_q4_0_multi(const void* const* srcs, const int64_t* src_rows, int nsrc, int mode, int64_t cols,
                          AhQ4Weight** out, cudaStream_t st) {
  AH_REQUIRE(nsrc >= 1 && nsrc <= 3, "q4w_create: 1..3 sources");
  RowSource s{};
  s.mode = mode;
  int64_t rows = 0;
  for (int k = 0; k < nsrc; ++k) {
    AH_REQUIRE(srcs[k] != nullptr && src_rows[k] > 0, "q4w_create: null source");
    s.q4_0[k] = static_cast<const uint8_t*>(srcs[k]);
    s.rows[k] = src_rows[k];
    rows += src_rows[k];
  }
  if (mode == 1) {
    AH_REQUIRE(nsrc == 2 && src_rows[0] == src_rows[1] && src_rows[0] % 8 == 0,
               "q4w_create: interleave needs two sources of equal rows, rows %% 8 == 0");
  }
  return q4w_create(s, false, rows, cols, out, st);
}

const Q4Tiled& q4w_tiled(const AhQ4Weight* w) { return w->t; }

// ---------------------------------------------------------------------------
// The fused GEMV kernel
// ---------------------------------------------------------------------------
namespace {

constexpr int kXsBudget = 96 * 1024;  // shared memory for the split-x planes

template <bool kF32>
struct ScaleT;
template <>
struct ScaleT<false> {  // Q4_0: four f16 scales per lane entry
  using V = uint2;
  static __device__ __forceinline__ V load(const V* p) { return ldg_nc_v2(p); }
  static __device__ __forceinline__ void get(const V& v, int blk, float& dg, float& dg8) {
    const uint32_t u = blk ? v.y : v.x;
    dg = __half2float(__ushort_as_half((unsigned short)(u & 0xFFFFu)));
    dg8 = __half2float(__ushort_as_half((unsigned short)(u >> 16)));
  }
};
template <>
struct ScaleT<true> {  // engine format: four f32 scales
  using V = float4;
  static __device__ __forceinline__ V load(const V* p) { return ldg_nc_f4(p); }
  static __device__ __forceinline__ void get(const V& v, int blk, float& dg, float& dg8) {
    dg = blk ? v.z : v.x;
    dg8 = blk ? v.w : v.y;
  }
};

__device__ __forceinline__ float silu_ref(float x) {  // inference/math.rs:83-95
  const float sg = x >= 0.0f ? __fdiv_rn(1.0f, 1.0f + expf(-x)) : __fdiv_rn(expf(x), 1.0f + expf(x));
  return x * sg;
}

// Position of chunk-relative column kk inside an x plane (halves): the 8
// values lane t needs for one 32-column block are contiguous (one LDS.128).
__device__ __forceinline__ int xs_pos(int kk) {
  const int e = kk & 31;
  return (kk >> 5) * 32 + ((e >> 1) & 3) * 8 + 2 * ((e >> 3) & 3) + (e & 1);
}

template <int NT, bool kF32, int PRO, int EPI, int U>
__global__ void __launch_bounds__(kGemvThreads) k_gemv_q4(const GemvArgs a) {
  constexpr int BM = 4 * NT;  // tokens this instantiation can hold
  using SV = typename ScaleT<kF32>::V;
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int B = a.batch;
  const int64_t rt = blockIdx.x;
  const int ky = blockIdx.y;
  const int64_t KP = a.w.kp;
  const int64_t pb = (int64_t)ky * a.pairs_per_chunk;
  const int64_t pe = min(pb + a.pairs_per_chunk, KP);
  const int kbc = (int)(2 * a.pairs_per_chunk);
  const int plane = kbc * 64 + 64;  // bytes per x plane (64 B pad staggers banks)
  uint8_t* xs = smem;
  float* red = reinterpret_cast<float*>(smem + (size_t)2 * B * plane);  // [warps][16][B]
  float* fin = red + kGemvWarps * 16 * B;                               // [16][B]
  float* tok_inv = fin + 16 * B;                                        // RMSNorm 1/rms per token
  float* exps = tok_inv + kGemvMaxBatch;                                // [B][kbc] 2^-s per block
  float* wred = exps + B * kbc;                                         // [warps][BM]
  int* flag = reinterpret_cast<int*>(wred + kGemvWarps * BM);

  const int64_t npairs = pe - pb;
  const int64_t per_warp = (npairs + kGemvWarps - 1) / kGemvWarps;
  const int64_t wp0 = pb + warp * per_warp;
  const int64_t wp1 = min(wp0 + per_warp, pe);
  const uint4* nibp = a.w.nib + rt * KP * 32 + lane;
  const SV* sclp = reinterpret_cast<const SV*>(a.w.scales) + rt * KP * 8 + g;

  // Weights do not depend on the previous kernel: start streaming them now.
  uint4 wv[U];
  SV sv[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (wp0 + u < wp1) {
      wv[u] = ldg_stream_v4(nibp + (wp0 + u) * 32);
      sv[u] = ScaleT<kF32>::load(sclp + (wp0 + u) * 8);
    }
  pdl_wait();

  // ---- prologue ------------------------------------------------------------
  const int64_t K = a.w.cols;
  const int64_t k0 = pb * 64, k1 = min(pe * 64, K);
  if (PRO == kProRmsNorm) {
    // RMSNorm statistics (inference/math.rs:53-63) from the producer's
    // per-tile partial sums of squares of x.
    float ss[BM];
#pragma unroll
    for (int b = 0; b < BM; ++b) {
      ss[b] = 0.0f;
      if (b < B)
        for (int i = tid; i < a.n_ss_in; i += kGemvThreads) ss[b] += a.ss_in[b * a.n_ss_in + i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss[b] += __shfl_xor_sync(0xFFFFFFFFu, ss[b], o);
    }
    if (lane == 0)
#pragma unroll
      for (int b = 0; b < BM; ++b) wred[warp * BM + b] = ss[b];
    __syncthreads();
    if (tid < B) {
      float s_tot = 0.0f;
      for (int w = 0; w < kGemvWarps; ++w) s_tot += wred[w * BM + tid];
      tok_inv[tid] = __fdiv_rn(1.0f, sqrtf(__fdiv_rn(s_tot, (float)K) + a.eps));
    }
    __syncthreads();
  }
  // ---- split x into f16 hi/lo planes, one power-of-two scale per (token, block) --
  // Eight threads share a 32-column block; each loads 4 values (one 16-byte
  // load), four blocks per thread are in flight per round.
  {
    constexpr int UNR = 4;
    const int tasks = B * kbc;
    const int rounds = (tasks + 32 * UNR - 1) / (32 * UNR);
    const int sub = tid & 7;
    const bool vec_ok = ((a.x_stride & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0);
    for (int r = 0; r < rounds; ++r) {
      float4 v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int task = (r * UNR + u) * 32 + (tid >> 3);
        v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (task < tasks) {
          const int b = task / kbc, kb = task - b * kbc;
          const int64_t k = k0 + (int64_t)kb * 32 + sub * 4;
          const float* xr = a.x + b * a.x_stride;
          if (vec_ok && k + 3 < k1) {
            v[u] = __ldg(reinterpret_cast<const float4*>(xr + k));
          } else {
            if (k < k1) v[u].x = xr[k];
            if (k + 1 < k1) v[u].y = xr[k + 1];
            if (k + 2 < k1) v[u].z = xr[k + 2];
            if (k + 3 < k1) v[u].w = xr[k + 3];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int task = (r * UNR + u) * 32 + (tid >> 3);
        const bool live = task < tasks;
        const int b = live ? task / kbc : 0;
        const int kb = live ? task - b * kbc : 0;
        const int64_t k = k0 + (int64_t)kb * 32 + sub * 4;
        float xv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        if (PRO == kProRmsNorm && live) {
          const float inv = tok_inv[b];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (k + i < k1) xv[i] = (xv[i] * inv) * __half2float(__ushort_as_half(a.norm_w[k + i]));
        }
        float m = fmaxf(fmaxf(fabsf(xv[0]), fabsf(xv[1])), fmaxf(fabsf(xv[2]), fabsf(xv[3])));
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 4));
        // scale so the block max lands in [2^14, 2^15): hi+lo then carry ~22 bits
        const int eb = (int)((__float_as_uint(m) >> 23) & 0xFFu);
        const int sc = (m == 0.0f) ? 0 : min(max(14 - (eb - 127), -120), 120);
        const float up = __uint_as_float((uint32_t)(127 + sc) << 23);
        if (live) {
          __half* ph = reinterpret_cast<__half*>(xs + (2 * b) * plane);
          __half* pl = reinterpret_cast<__half*>(xs + (2 * b + 1) * plane);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float sv = xv[i] * up;
            const __half hi = __float2half_rn(sv);
            const int pos = xs_pos(kb * 32 + sub * 4 + i);
            ph[pos] = hi;
            pl[pos] = __float2half_rn(sv - __half2float(hi));
          }
          if (sub == 0) exps[b * kbc + kb] = __uint_as_float((uint32_t)(127 - sc) << 23);
        }
      }
    }
  }
  __syncthreads();

  // ---- main loop: stream weights, unpack to f16 fragments, mma -----------------
  float tot[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) tot[j][0] = tot[j][1] = tot[j][2] = tot[j][3] = 0.0f;
  for (int64_t p = wp0; p < wp1; p += U) {
    if (p != wp0) {
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (p + u < wp1) {
          wv[u] = ldg_stream_v4(nibp + (p + u) * 32);
          sv[u] = ScaleT<kF32>::load(sclp + (p + u) * 8);
        }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (p + u < wp1) {
        const int kb_rel = (int)(2 * (p + u - pb));
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
          unpack_word(blk ? wv[u].z : wv[u].x, a0, a1, a2, a3);  // row g
          unpack_word(blk ? wv[u].w : wv[u].y, c0, c1, c2, c3);  // row g+8
          float dg, dg8;
          ScaleT<kF32>::get(sv[u], blk, dg, dg8);
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const int col = 8 * j + g;
            uint4 bf = make_uint4(0u, 0u, 0u, 0u);
            if (col < 2 * B) bf = *reinterpret_cast<const uint4*>(xs + col * plane + (kb_rel + blk) * 64 + t * 16);
            const int tok = 4 * j + t;  // this lane's accumulator columns 2t, 2t+1 = token tok (hi, lo)
            const float ex = tok < B ? exps[tok * kbc + kb_rel + blk] : 0.0f;
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            mma16816(acc, a0, c0, a1, c1, bf.x, bf.y, acc);
            mma16816(acc, a2, c2, a3, c3, bf.z, bf.w, acc);
            const float de = dg * ex, d8e = dg8 * ex;
            tot[j][0] = fmaf(de, acc[0], tot[j][0]);
            tot[j][1] = fmaf(de, acc[1], tot[j][1]);
            tot[j][2] = fmaf(d8e, acc[2], tot[j][2]);
            tot[j][3] = fmaf(d8e, acc[3], tot[j][3]);
          }
        }
      }
    }
  }
  pdl_launch_dependents();

  // ---- epilogue: columns -> tokens, warps -> tile, chunks -> row ------------------
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int b = 4 * j + t;
    if (b < B) {
      red[(warp * 16 + g) * B + b] = tot[j][0] + tot[j][1];
      red[(warp * 16 + g + 8) * B + b] = tot[j][2] + tot[j][3];
    }
  }
  __syncthreads();
  const int64_t rows_pad = a.w.r16 * 16;
  for (int i = tid; i < 16 * B; i += kGemvThreads) {
    const int r = i / B, b = i - r * B;
    float v = 0.0f;
    for (int w = 0; w < kGemvWarps; ++w) v += red[(w * 16 + r) * B + b];
    if (a.ksplit == 1) fin[i] = v;
    else a.partial[((int64_t)ky * rows_pad + rt * 16 + r) * B + b] = v;
  }
  if (a.ksplit > 1) {
    __threadfence();
    __syncthreads();
    if (tid == 0) *flag = (atomicAdd(&a.counters[rt], 1) == a.ksplit - 1);
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    for (int i = tid; i < 16 * B; i += kGemvThreads) {
      const int r = i / B, b = i - r * B;
      float v = 0.0f;
      for (int c = 0; c < a.ksplit; ++c) v += __ldcg(&a.partial[((int64_t)c * rows_pad + rt * 16 + r) * B + b]);
      fin[i] = v;
    }
    if (tid == 0) a.counters[rt] = 0;
  }
  __syncthreads();
  if (EPI == kEpiSwiglu) {
    // rows g < 8 of the tile are gate rows 8rt+g, rows g+8 the matching up rows.
    for (int i = tid; i < 8 * B; i += kGemvThreads) {
      const int r = i / B, b = i - r * B;
      const int64_t o = rt * 8 + r;
      if (o < a.w.rows / 2) a.y[b * a.y_stride + o] = silu_ref(fin[r * B + b]) * fin[(r + 8) * B + b];
    }
  } else {
    for (int i = tid; i < 16 * B; i += kGemvThreads) {
      const int r = i / B, b = i - r * B;
      const int64_t R = rt * 16 + r;
      float h = 0.0f;
      if (R < a.w.rows) {
        float* dst = a.y + b * a.y_stride + R;
        h = (EPI == kEpiAdd) ? *dst + fin[i] : fin[i];  // residual: hidden[i] += out[i]
        *dst = h;
      }
      if (a.ss_out) fin[i] = h;
    }
    if (a.ss_out) {
      // per-tile partial sum of squares of the new values, for the next
      // kernel's RMSNorm prologue
      __syncthreads();
      if (tid < B) {
        float s2 = 0.0f;
        for (int r = 0; r < 16; ++r) s2 = fmaf(fin[r * B + tid], fin[r * B + tid], s2);
        a.ss_out[tid * a.w.r16 + rt] = s2;
      }
    }
  }
}

using GemvKernel = void (*)(const GemvArgs);

template <int NT>
GemvKernel pick_kernel(bool f32s, int pro, int epi) {
  constexpr int U = NT == 1 ? 8 : 4;
  if (f32s) return (pro == kProPlain && epi == kEpiStore) ? k_gemv_q4<NT, true, kProPlain, kEpiStore, U> : nullptr;
  if (pro == kProPlain) {
    if (epi == kEpiStore) return k_gemv_q4<NT, false, kProPlain, kEpiStore, U>;
    if (epi == kEpiAdd) return k_gemv_q4<NT, false, kProPlain, kEpiAdd, U>;
    return k_gemv_q4<NT, false, kProPlain, kEpiSwiglu, U>;
  }
  if (epi == kEpiStore) return k_gemv_q4<NT, false, kProRmsNorm, kEpiStore, U>;
  if (epi == kEpiAdd) return k_gemv_q4<NT, false, kProRmsNorm, kEpiAdd, U>;
  return k_gemv_q4<NT, false, kProRmsNorm, kEpiSwiglu, U>;
}

}  // namespace

GemvPlan gemv_plan(const Q4Tiled& w, int batch) {
  GemvPlan p{};
  p.nt = (batch + 3) / 4;
  int64_t max_kbc = ((int64_t)kXsBudget / (2 * batch) - 64) / 64;
  int64_t ppc = std::max<int64_t>(1, max_kbc / 2);
  ppc = std::min<int64_t>(ppc, w.kp);
  p.ksplit = (int)((w.kp + ppc - 1) / ppc);
  p.pairs_per_chunk = (w.kp + p.ksplit - 1) / p.ksplit;
  const int64_t plane = 2 * p.pairs_per_chunk * 64 + 64;
  p.smem = (size_t)2 * batch * plane + (size_t)(kGemvWarps * 16 * batch + 16 * batch + kGemvMaxBatch) * 4 +
           (size_t)batch * (2 * p.pairs_per_chunk) * 4 + (size_t)kGemvWarps * (4 * p.nt) * 4 + 16;
  return p;
}

int gemv_workspace_reserve(GemvWorkspace& ws, const Q4Tiled& w, const GemvPlan& plan, int batch) {
  if (plan.ksplit <= 1) return AH_OK;
  const size_t need = (size_t)plan.ksplit * w.r16 * 16 * batch;
  if (ws.partial_floats < need) {
    if (ws.partial) cudaFree(ws.partial);
    ws.partial = nullptr;
    ws.partial_floats = 0;
    if (cudaMalloc(&ws.partial, need * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      return fail(AH_ENOMEM, "gemv workspace: cudaMalloc of %zu floats failed", need);
    }
    ws.partial_floats = need;
  }
  if (ws.n_counters < w.r16) {
    if (ws.counters) cudaFree(ws.counters);
    ws.counters = nullptr;
    ws.n_counters = 0;
    if (cudaMalloc(&ws.counters, (size_t)w.r16 * sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      return fail(AH_ENOMEM, "gemv workspace: counter allocation failed");
    }
    AH_CUDA_TRY(cudaMemset(ws.counters, 0, (size_t)w.r16 * sizeof(int)));
    ws.n_counters = w.r16;
  }
  return AH_OK;
}

void gemv_workspace_free(GemvWorkspace& ws) {
  if (ws.partial) cudaFree(ws.partial);
  if (ws.counters) cudaFree(ws.counters);
  ws = GemvWorkspace{};
}

int gemv_launch(GemvArgs a, int pro, int epi, GemvWorkspace& ws, cudaStream_t st, bool pdl) {
  AH_REQUIRE(a.batch >= 1 && a.batch <= kGemvMaxBatch, "gemv: batch must be 1..16");
  AH_REQUIRE(pro != kProRmsNorm || (a.norm_w != nullptr && a.ss_in != nullptr && a.n_ss_in > 0),
             "gemv: RMSNorm prologue needs a norm weight and the producer's partial sums of squares");
  AH_REQUIRE(epi != kEpiSwiglu || a.w.rows % 16 == 0, "gemv: SwiGLU epilogue needs interleaved rows %% 16 == 0");
  const GemvPlan plan = gemv_plan(a.w, a.batch);
  if (plan.ksplit > 1) {
    if (ws.partial_floats < (size_t)plan.ksplit * a.w.r16 * 16 * a.batch || ws.n_counters < a.w.r16) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(st, &cs);
      AH_REQUIRE(cs == cudaStreamCaptureStatusNone, "gemv: k-split workspace must be reserved before graph capture");
      int rc = gemv_workspace_reserve(ws, a.w, plan, a.batch);
      if (rc) return rc;
    }
  }
  a.pairs_per_chunk = plan.pairs_per_chunk;
  a.ksplit = plan.ksplit;
  a.partial = ws.partial;
  a.counters = ws.counters;
  GemvKernel kern = nullptr;
  switch (plan.nt) {
    case 1: kern = pick_kernel<1>(a.w.f32_scales, pro, epi); break;
    case 2: kern = pick_kernel<2>(a.w.f32_scales, pro, epi); break;
    case 3: kern = pick_kernel<3>(a.w.f32_scales, pro, epi); break;
    default: kern = pick_kernel<4>(a.w.f32_scales, pro, epi); break;
  }
  if (!kern) return fail(AH_EUNSUPPORTED, "gemv: engine-format weights support only the plain GEMV");
  {
    // Raise the kernel's dynamic shared-memory cap once per (device, kernel, size).
    static std::mutex mu;
    static std::vector<std::pair<std::pair<int, void*>, size_t>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    bool found = false;
    for (auto& e : done)
      if (e.first.first == dev && e.first.second == (void*)kern) {
        found = true;
        if (e.second < plan.smem) {
          AH_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem));
          e.second = plan.smem;
        }
      }
    if (!found) {
      AH_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem));
      done.push_back({{dev, (void*)kern}, plan.smem});
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)a.w.r16, (unsigned)plan.ksplit, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AH_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return AH_OK;
}

}  // namespace ah

// ---------------------------------------------------------------------------
// Generic engine-format GEMV (any group size), straight from the reference's
// storage: one warp per row, lanes stride over groups.  Used for the literal
// device-pointer drop-in of gemv_4bit_into; the tiled handle path is the fast one.
// ---------------------------------------------------------------------------
namespace ah {
namespace {
__global__ void __launch_bounds__(256) k_gemv_engine_generic(float* __restrict__ out, const float* __restrict__ scales,
                                                             const uint8_t* __restrict__ packed,
                                                             const float* __restrict__ x, int64_t rows, int64_t cols,
                                                             int64_t gs) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t n_gpr = (cols + gs - 1) / gs;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    float sum = 0.0f;
    const int64_t row_off = r * cols;
    for (int64_t j = lane; j < cols; j += 32) {
      const int64_t lin = row_off + j;
      const uint32_t byte = packed[lin >> 1];
      const uint32_t nib = (lin & 1) ? (byte >> 4) & 0xFu : byte & 0xFu;
      const float wv = __fmul_rn((float)(int)nib - 8.0f, scales[r * n_gpr + j / gs]);
      sum = __fadd_rn(sum, __fmul_rn(wv, x[j]));  // no contraction, as in math.rs:412-413
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) out[r] = sum;
  }
}
__global__ void k_zero(float* p, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = 0.0f;
}
}  // namespace
}  // namespace ah

extern "C" {

int ah_q4w_from_q4_0(const void* blocks, int64_t rows, int64_t cols, AhQ4Weight** out, void* stream) {
  const void* srcs[1] = {blocks};
  int64_t r[1] = {rows};
  return q4w_create_q4_0_multi(srcs, r, 1, 0, cols, out, as_stream(stream));
}

int ah_q4w_from_engine(const float* scales, const uint8_t* packed, int64_t rows, int64_t cols, AhQ4Weight** out,
                       void* stream) {
  AH_REQUIRE(scales && packed, "q4w_from_engine: null source");
  RowSource s{};
  s.mode = 0;
  s.rows[0] = rows;
  s.eng_s[0] = scales;
  s.eng_p[0] = packed;
  return q4w_create(s, true, rows, cols, out, as_stream(stream));
}

int ah_q4w_destroy(AhQ4Weight* w) {
  if (!w) return AH_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(w->device);
  cudaFree(w->nib_alloc);
  cudaFree(w->scale_alloc);
  gemv_workspace_free(w->ws);
  cudaSetDevice(cur);
  delete w;
  return AH_OK;
}

int ah_q4w_shape(const AhQ4Weight* w, int64_t* rows, int64_t* cols) {
  AH_REQUIRE(w && rows && cols, "q4w_shape: null argument");
  *rows = w->t.rows;
  *cols = w->t.cols;
  return AH_OK;
}

int64_t ah_q4w_weight_bytes(const AhQ4Weight* w) { return w ? w->weight_bytes : 0; }

int ah_q4w_gemv(const AhQ4Weight* wc, const float* x, float* y, int batch, void* stream) {
  AH_REQUIRE(wc && x && y, "q4w_gemv: null argument");
  AH_REQUIRE(batch >= 1 && batch <= kGemvMaxBatch, "q4w_gemv: batch must be 1..16");
  AhQ4Weight* w = const_cast<AhQ4Weight*>(wc);
  GemvArgs a{};
  a.w = w->t;
  a.x = x;
  a.x_stride = w->t.cols;
  a.y = y;
  a.y_stride = w->t.rows;
  a.batch = batch;
  std::lock_guard<std::mutex> lk(w->mu);
  return gemv_launch(a, kProPlain, kEpiStore, w->ws, as_stream(stream), true);
}

int ah_gemv_4bit_into(float* out, const float* scales, const uint8_t* packed, const float* x, int64_t rows,
                      int64_t cols, int64_t gs, void* stream) {
  cudaStream_t st = as_stream(stream);
  AH_REQUIRE(rows >= 0 && cols >= 0, "gemv_4bit_into: negative shape");
  if (rows == 0) return AH_OK;
  AH_REQUIRE(out != nullptr, "gemv_4bit_into: null out");
  if (cols == 0 || x == nullptr) {  // inference/math.rs:264-267
    k_zero<<<(int)std::min<int64_t>((rows + 255) / 256, 1024), 256, 0, st>>>(out, rows);
    AH_LAUNCH_CHECK();
    return AH_OK;
  }
  AH_REQUIRE(scales && packed, "gemv_4bit_into: null weights");
  if (gs < 1) gs = 1;
  int64_t grid = std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 8);
  k_gemv_engine_generic<<<(int)grid, 256, 0, st>>>(out, scales, packed, x, rows, cols, gs);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_matvec_4bit_into(float* out, const float* scales, const uint8_t* packed, const float* x, int64_t dim, int64_t gs,
                        void* stream) {
  return ah_gemv_4bit_into(out, scales, packed, x, dim, dim, gs, stream);
}

}  // extern "C"
