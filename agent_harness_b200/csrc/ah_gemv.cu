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
  // device staging for host-buffer calls (ah_q4w_gemv_host), allocated on the
  // first such call for the largest batch; mu serialises those calls
  void* stage = nullptr;
  // the pull + GEMV of the last pinned-buffer call as one graph, reused while
  // the caller passes the same buffers and batch
  cudaGraphExec_t host_graph = nullptr;
  cudaStream_t host_cap = nullptr;
  const void* hg_x = nullptr;
  const void* hg_y = nullptr;
  int hg_batch = 0;
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
        const int e = 2 * t + (pp >> 2) + 16 * (pp & 1) + 8 * ((pp >> 1) & 1);
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

int q4w_alloc(int64_t rows, int64_t cols, bool engine, AhQ4Weight** out) {
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
  if (ah::dev_malloc(&w->nib_alloc, nib_bytes) != cudaSuccess || ah::dev_malloc(&w->scale_alloc, sc_bytes) != cudaSuccess) {
    cudaGetLastError();
    if (w->nib_alloc) cudaFree(w->nib_alloc);
    if (w->scale_alloc) cudaFree(w->scale_alloc);
    delete w;
    return fail(AH_ENOMEM, "q4w_create: cudaMalloc of %zu bytes failed", nib_bytes + sc_bytes);
  }
  w->t.nib = static_cast<const uint4*>(w->nib_alloc);
  w->t.scales = w->scale_alloc;
  w->weight_bytes = engine ? rows * ((cols + 1) / 2) + rows * nb * 4 : rows * nb * 18;
  *out = w;
  return AH_OK;
}

int q4w_create(const RowSource& src, bool engine, int64_t rows, int64_t cols, AhQ4Weight** out, cudaStream_t st) {
  AhQ4Weight* w = nullptr;
  const int rc = q4w_alloc(rows, cols, engine, &w);
  if (rc != AH_OK) return rc;
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

int q4w_create_engine_multi(const float* const* scales, const uint8_t* const* packed, const int64_t* src_rows,
                            int nsrc, int mode, int64_t cols, AhQ4Weight** out, cudaStream_t st) {
  AH_REQUIRE(nsrc >= 1 && nsrc <= 3, "q4w_create: 1..3 sources");
  RowSource s{};
  s.mode = mode;
  int64_t rows = 0;
  for (int k = 0; k < nsrc; ++k) {
    AH_REQUIRE(scales[k] != nullptr && packed[k] != nullptr && src_rows[k] > 0, "q4w_create: null source");
    s.eng_s[k] = scales[k];
    s.eng_p[k] = packed[k];
    s.rows[k] = src_rows[k];
    rows += src_rows[k];
  }
  if (mode == 1) {
    AH_REQUIRE(nsrc == 2 && src_rows[0] == src_rows[1] && src_rows[0] % 8 == 0,
               "q4w_create: interleave needs two sources of equal rows, rows %% 8 == 0");
  }
  return q4w_create(s, true, rows, cols, out, st);
}

const Q4Tiled& q4w_tiled(const AhQ4Weight* w) { return w->t; }
uint4* q4w_nib_mut(AhQ4Weight* w) { return static_cast<uint4*>(w->nib_alloc); }
void* q4w_scales_mut(AhQ4Weight* w) { return w->scale_alloc; }

// ---------------------------------------------------------------------------
// The fused GEMV kernel
// ---------------------------------------------------------------------------
namespace {


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

// ---------------------------------------------------------------------------
// The fused GEMV.  A thread-block cluster of kGemvCluster CTAs walks row groups
// of kGemvWarps 16-row tiles (128 rows) over the full K; cluster CTA c takes
// K-chunk c (ppc = ceil(kp/8) block pairs).  Each CTA splits its chunk of x
// into shared memory once, and for every row group its warp w multiplies row
// tile w against it, so the main loop reads only local shared memory; weights
// stream HBM -> registers, and the next row group's are in flight while the
// current one is reduced.  The chunk partials of row tile r meet in cluster CTA
// r, which sums them over DSMEM in chunk order (deterministic; no global
// scratch, fences or atomics) and runs the epilogue.  The grid holds at most
// as many clusters as are resident at once (persistent).
// ---------------------------------------------------------------------------
template <bool kF32, int U>
__device__ __forceinline__ void load_pairs(uint4 (&w)[U], typename ScaleT<kF32>::V (&sv)[U],
                                           const uint4* nibp, const typename ScaleT<kF32>::V* sclp, int p, int np) {
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (p + u < np) {
      w[u] = ldg_stream_v4(nibp + (p + u) * 32);
      sv[u] = ScaleT<kF32>::load(sclp + (p + u) * 8);
    }
}

template <int NT, bool kF32, int U>
__device__ __forceinline__ void mma_pairs(float (&tot)[NT][4], const uint4 (&w)[U],
                                          const typename ScaleT<kF32>::V (&sv)[U], int p, int np, int B,
                                          int g, int t, const uint8_t* xs, const float4* blk_info, int plane,
                                          int kbc, int kb0) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (p + u < np) {
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        // nibbles -> exact f16 subnormals n*2^-24 (k-step 0) and n*2^-20 (k-step 1)
        const uint32_t w0 = blk ? w[u].z : w[u].x;  // row g
        const uint32_t w8 = blk ? w[u].w : w[u].y;  // row g+8
        const uint32_t w0s = w0 >> 8, w8s = w8 >> 8;
        const uint32_t s0a0 = w0 & 0x000F000Fu, s0a1 = w8 & 0x000F000Fu;
        const uint32_t s0a2 = w0s & 0x000F000Fu, s0a3 = w8s & 0x000F000Fu;
        const uint32_t s1a0 = w0 & 0x00F000F0u, s1a1 = w8 & 0x00F000F0u;
        const uint32_t s1a2 = w0s & 0x00F000F0u, s1a3 = w8s & 0x00F000F0u;
        float dg, dg8;
        ScaleT<kF32>::get(sv[u], blk, dg, dg8);
        const int kb = kb0 + 2 * (p + u) + blk;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int col = 8 * j + g;
          uint4 bf = make_uint4(0u, 0u, 0u, 0u);
          if (col < 2 * B) bf = *reinterpret_cast<const uint4*>(xs + col * plane + kb * 64 + t * 16);
          const int tok = 4 * j + t;  // accumulator columns 2t, 2t+1 = token tok (hi, lo)
          const float4 bi = tok < B ? blk_info[tok * (kbc + 1) + kb] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          float acc[4] = {bi.y, bi.z, bi.y, bi.z};  // -8 * sum(x) start value, rows g and g+8
          mma16816(acc, s0a0, s0a1, s0a2, s0a3, bf.x, bf.y, acc);
          mma16816(acc, s1a0, s1a1, s1a2, s1a3, bf.z, bf.w, acc);
          const float de = dg * bi.x, d8e = dg8 * bi.x;
          tot[j][0] = fmaf(de, acc[0], tot[j][0]);
          tot[j][1] = fmaf(de, acc[1], tot[j][1]);
          tot[j][2] = fmaf(d8e, acc[2], tot[j][2]);
          tot[j][3] = fmaf(d8e, acc[3], tot[j][3]);
        }
      }
    }
  }
}

// RMSNorm statistics (inference/math.rs:53-63): 1/rms per token from the
// producer's partial sums of squares of x.
template <int BM, int PRO>
__device__ __forceinline__ void rms_stats(const GemvArgs& a, float* wred, float* tok_inv, int tid, int lane,
                                          int warp) {
  const int B = a.batch;
  const int64_t K = a.w.cols;
  if (PRO == kProRmsNorm) {
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
      tok_inv[tid] = __fdiv_rn(1.0f, sqrtf(__fdiv_rn(s_tot, (float)K) + a.eps));  // inference/math.rs:59
    }
    __syncthreads();
  }
}

// Splits columns [k0, k1) of x (block-relative 0 .. kbc*32) into f16 hi/lo
// planes.  Eight threads share a (token, 32-column block) task; each loads 4
// values.  Per block this also records {2^(24-s), -8*2^-24*sum(hi),
// -8*2^-24*sum(lo)}: the exponent that undoes the power-of-two scaling and the
// accumulator start value that applies the -8 nibble offset inside the tensor core.
template <int PRO>
__device__ __forceinline__ void split_x(const GemvArgs& a, uint8_t* xs, float4* blk_info, int plane, int kbc,
                                        int64_t k0, int64_t k1, const float* tok_inv, int tid, int warp) {
  const int B = a.batch;
  {
    constexpr int UNR = 2;
    const int tasks = B * kbc;
    const int rounds = (tasks + 32 * UNR - 1) / (32 * UNR);
    const int sub = tid & 7;
    const int e0 = sub * 4;                  // this thread's first column in the block
    const int stp = e0 >> 4, reg = (e0 & 15) >> 3;
    const int tA = ((e0 & 15) >> 1) & 3;     // fragment owner of values 0,1 (values 2,3: tA+1)
    const int halfA = tA * 4 + stp * 2 + reg;  // half2 index of values 0,1 within the block
    const float pre = stp ? 0.0625f : 1.0f;  // k-step-1 columns meet A values 16x larger
    const bool vec_ok = ((a.x_stride & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15u) == 0);
    for (int r = 0; r < rounds; ++r) {
      if ((r * UNR) * 32 + warp * 4 >= tasks) break;  // warp-uniform: nothing left for this warp
      float4 v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int task = (r * UNR + u) * 32 + (tid >> 3);
        v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (task < tasks) {
          const int b = task / kbc, kb = task - b * kbc;
          const int64_t k = k0 + (int64_t)kb * 32 + e0;
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
        if ((r * UNR + u) * 32 + warp * 4 >= tasks) break;  // warp-uniform
        const int task = (r * UNR + u) * 32 + (tid >> 3);
        const bool tl = task < tasks;
        const int b = tl ? task / kbc : 0, kb = tl ? task - b * kbc : 0;
        const int64_t k = k0 + (int64_t)kb * 32 + e0;
        float xv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        if (PRO == kProRmsNorm && tl) {
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
        const int sc = (m == 0.0f) ? 0 : min(max(14 - (eb - 127), -100), 100);
        const float up = __uint_as_float((uint32_t)(127 + sc) << 23) * pre;
        const float2 s01 = make_float2(xv[0] * up, xv[1] * up), s23 = make_float2(xv[2] * up, xv[3] * up);
        const __half2 h01 = __float22half2_rn(s01), h23 = __float22half2_rn(s23);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __float22half2_rn(make_float2(s01.x - f01.x, s01.y - f01.y));
        const __half2 l23 = __float22half2_rn(make_float2(s23.x - f23.x, s23.y - f23.y));
        const float2 g01 = __half22float2(l01), g23 = __half22float2(l23);
        // threads 4..7 hold the k-step-1 columns, stored /16: their sums count 16x
        const float wsum = stp ? 16.0f : 1.0f;
        float shi = ((f01.x + f01.y) + (f23.x + f23.y)) * wsum;
        float slo = ((g01.x + g01.y) + (g23.x + g23.y)) * wsum;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          shi += __shfl_xor_sync(0xFFFFFFFFu, shi, o);
          slo += __shfl_xor_sync(0xFFFFFFFFu, slo, o);
        }
        if (tl) {
          __half2* ph = reinterpret_cast<__half2*>(xs + (2 * b) * plane) + kb * 16 + halfA;
          __half2* pl = reinterpret_cast<__half2*>(xs + (2 * b + 1) * plane) + kb * 16 + halfA;
          ph[0] = h01;
          ph[4] = h23;
          pl[0] = l01;
          pl[4] = l23;
          if (sub == 0) {
            const float c = -8.0f * 5.9604644775390625e-8f;  // -8 * 2^-24
            blk_info[b * (kbc + 1) + kb] = make_float4(__uint_as_float((uint32_t)(127 + 24 - sc) << 23), c * shi, c * slo,
                                                 0.0f);
          }
        }
      }
    }
  }
}

template <int NT, bool kF32, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, kGemvMinBlocks<NT>) k_gemv_q4(const GemvArgs a) {
  constexpr int BM = 4 * NT;  // tokens this instantiation can hold
  using SV = typename ScaleT<kF32>::V;
  constexpr int U = kGemvBatchPairs<NT>;  // block pairs per register batch
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int B = a.batch;
  const int crank = (int)cluster_ctarank();  // = K-chunk
  const int64_t n_rg = (a.w.r16 + kGemvWarps - 1) / kGemvWarps;
  const int64_t n_cl = gridDim.x / kGemvCluster;
  int64_t rg = blockIdx.x / kGemvCluster;
  int64_t rt = rg * kGemvWarps + warp;  // this warp's row tile
  bool warp_live = rt < a.w.r16;
  const int64_t KP = a.w.kp;
  const int ppc = (int)a.pairs_per_chunk;
  const int kbc = 2 * ppc;          // blocks per chunk
  const int plane = kbc * 64 + 64;  // bytes per x plane (64 B pad staggers banks)
  uint8_t* xs = smem;                                                           // [2B][plane]
  float4* blk_info = reinterpret_cast<float4*>(smem + (size_t)2 * B * plane);  // [B][kbc+1]: rows padded
                                                                                // so tokens hit different banks
  float* part = reinterpret_cast<float*>(blk_info + B * (kbc + 1));             // [warps][16][B]
  float* tok_inv = part + kGemvWarps * 16 * B;                                  // [16]
  float* wred = tok_inv + kGemvMaxBatch;                                        // [warps][BM], then [16][B]
  float* slots = wred + kGemvWarps * BM + 16 * B;  // [2][cluster][16][B] pushed chunk partials
  int64_t iter = 0;

  // Weights do not depend on the previous kernel: start streaming them now
  // (two batches of kGemvU pairs in flight per lane).
  const int64_t PE = a.pair_end > 0 ? a.pair_end : KP;  // this launch's K window [pair_begin, PE)
  const int64_t p0 = a.pair_begin + (int64_t)crank * ppc;
  const int np = (int)max((int64_t)0, min(p0 + ppc, PE) - p0);
  const uint4* nibp = a.w.nib + (rt * KP + p0) * 32 + lane;
  const SV* sclp = reinterpret_cast<const SV*>(a.w.scales) + (rt * KP + p0) * 8 + g;
  const int64_t tile_nib = KP * 32 * kGemvWarps * n_cl;  // uint4 stride to the next row group of this CTA
  const int64_t tile_scl = KP * 8 * kGemvWarps * n_cl;
  uint4 wa[U], wb[U];
  SV sa[U], sb[U];
  if (warp_live) {
    load_pairs<kF32, U>(wa, sa, nibp, sclp, 0, np);
    load_pairs<kF32, U>(wb, sb, nibp, sclp, U, np);
  }
  // A grid resident in one wave lets the next kernel launch now, so its weight
  // prefetch overlaps this kernel; larger grids trigger after the main loop.
  if (a.early_trigger) pdl_launch_dependents();
  pdl_wait();

  const int64_t K = a.w.cols;
  rms_stats<BM, PRO>(a, wred, tok_inv, tid, lane, warp);
  split_x<PRO>(a, xs, blk_info, plane, kbc, p0 * 64, min(min(p0 * 64 + (int64_t)ppc * 64, PE * 64), K), tok_inv, tid,
               warp);
  __syncthreads();

  // ---- row groups: main loop (local), DSMEM reduction, epilogue ------------------
  for (; rg < n_rg; rg += n_cl) {
    float tot[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) tot[j][0] = tot[j][1] = tot[j][2] = tot[j][3] = 0.0f;
    if (warp_live) {
      for (int p = 0; p < np; p += 2 * U) {
        mma_pairs<NT, kF32, U>(tot, wa, sa, p, np, B, g, t, xs, blk_info, plane, kbc, 0);
        if (p + 2 * U < np) load_pairs<kF32, U>(wa, sa, nibp, sclp, p + 2 * U, np);
        mma_pairs<NT, kF32, U>(tot, wb, sb, p + U, np, B, g, t, xs, blk_info, plane, kbc, 0);
        if (p + 3 * U < np) load_pairs<kF32, U>(wb, sb, nibp, sclp, p + 3 * U, np);
      }
    }
    // prefetch the next row group's first two batches while this one is reduced
    const int64_t rg_next = rg + n_cl;
    const int64_t rt_next = rg_next * kGemvWarps + warp;
    const bool next_live = rg_next < n_rg && rt_next < a.w.r16;
    nibp += tile_nib;
    sclp += tile_scl;
    if (next_live) {
      load_pairs<kF32, U>(wa, sa, nibp, sclp, 0, np);
      load_pairs<kF32, U>(wb, sb, nibp, sclp, U, np);
    }
    if (rg_next >= n_rg && !a.early_trigger) pdl_launch_dependents();

    // push the chunk partials to their owners: row tile `warp` of this group is
    // finalised by cluster CTA `warp`, which gathers chunk c's partial in its
    // slot c (slots double-buffered by row-group parity).  One cluster barrier
    // then makes every push visible; afterwards each CTA reads only its own
    // shared memory, so no second barrier guards the slots or the exit.
    float* slot_base = slots + (size_t)(iter & 1) * kGemvCluster * 16 * B;
    if (warp_live) {
      const uint32_t dst = mapa_shared(smem_u32(slot_base + crank * 16 * B), (uint32_t)warp);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int b = 4 * j + t;  // columns 2t (hi) and 2t+1 (lo) of tile j
        if (b < B) {
          st_dsmem_f32(dst + (uint32_t)((g * B + b) * 4), tot[j][0] + tot[j][1]);
          st_dsmem_f32(dst + (uint32_t)(((g + 8) * B + b) * 4), tot[j][2] + tot[j][3]);
        }
      }
    }
    cluster_arrive();
    cluster_wait();  // every push into this CTA's slots has landed
    const int64_t my_rt = rg * kGemvWarps + crank;  // the row tile this CTA finalises
    const bool fin_live = my_rt < a.w.r16;
    float* fin = wred;  // [16][B]
    if (fin_live) {
      for (int i = tid; i < 16 * B; i += kGemvThreads) {
        float v = 0.0f;
#pragma unroll
        for (int c = 0; c < kGemvCluster; ++c) v += slot_base[c * 16 * B + i];  // chunk order
        fin[i] = v;
      }
    }
    __syncthreads();
    if (fin_live) {
      if (EPI == kEpiSwiglu) {
        // tile rows r < 8 are gate rows 8rt+r, rows r+8 the matching up rows
        for (int i = tid; i < 8 * B; i += kGemvThreads) {
          const int r = i / B, b = i - r * B;
          const int64_t o = my_rt * 8 + r;
          if (o < a.w.rows / 2) a.y[b * a.y_stride + o] = silu_ref(fin[r * B + b]) * fin[(r + 8) * B + b];
        }
      } else {
        for (int i = tid; i < 16 * B; i += kGemvThreads) {
          const int r = i / B, b = i - r * B;
          const int64_t R = my_rt * 16 + r;
          float h = 0.0f;
          if (R < a.w.rows) {
            if (EPI == kEpiStore && a.n_peer > 0) {
              h = fin[i];
              for (int p = 0; p < a.n_peer; ++p) a.peer_y[p][R * a.peer_row + b] = h;  // NVLink stores
            } else {
              float* d = a.y + b * a.y_stride + R;
              h = (EPI == kEpiAdd) ? *d + fin[i] : fin[i];  // residual: hidden[i] += out[i]
              *d = h;
            }
          }
          fin[i] = h;
        }
        // peer slots: the stores reach the other GPUs before this grid completes
        if (EPI == kEpiStore && a.n_peer > 0) __threadfence_system();
        if (a.ss_out) {
          // per-tile partial sum of squares of the values written (next RMSNorm)
          __syncthreads();
          if (tid < B) {
            float q = 0.0f;
            for (int r = 0; r < 16; ++r) q = fmaf(fin[r * B + tid], fin[r * B + tid], q);
            a.ss_out[tid * a.w.r16 + my_rt] = q;
          }
        }
      }
    }
    __syncthreads();  // fin is reused by the next row group
    rt = rt_next;
    warp_live = next_live;
    ++iter;
  }
}

// Persistent full-K CTAs for GEMVs with many row tiles (FFN gate/up, the
// fused QKV, the LM head): each CTA splits all of x into shared memory once,
// then walks row tiles rt = blockIdx.x, +gridDim.x, ...; its eight warps take
// the eight K-chunks of the tile and meet in local shared memory, so a tile
// costs one CTA barrier instead of a cluster exchange.  A tile's nibble and
// scale planes are contiguous in HBM (KP x 512 B and KP x 8 scale entries), so
// each arrives by two bulk copies into one of n_stages shared-memory stages,
// completing on the stage's mbarrier: n_stages tiles per CTA are in flight
// while earlier ones are multiplied and reduced, and the first n_stages are
// requested before the kernel waits for its predecessor (weights do not
// change).  A stage is refilled once every warp has read it.
template <int NT, bool kF32, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) k_gemv_q4_rows(const GemvArgs a) {
  constexpr int BM = 4 * NT;
  using SV = typename ScaleT<kF32>::V;
  constexpr int U = kGemvBatchPairs<NT>;  // block pairs read from the stage per batch
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int B = a.batch;
  const int64_t KP = a.w.kp, r16 = a.w.r16;
  const int ppc = (int)a.pairs_per_chunk;  // pairs per warp = ceil(kp / 8)
  const int kbc = 2 * (int)KP;             // the whole K
  const int plane = kbc * 64 + 64;
  const int S = a.n_stages;
  const uint32_t nib_bytes = (uint32_t)KP * 512u, scl_bytes = (uint32_t)KP * 8u * (uint32_t)sizeof(SV);
  const uint32_t stage_bytes = nib_bytes + scl_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint8_t* base = smem + (size_t)S * stage_bytes + (((size_t)S * 8 + 15) & ~(size_t)15);
  uint8_t* xs = base;                                                           // [2B][plane]
  float4* blk_info = reinterpret_cast<float4*>(base + (size_t)2 * B * plane);  // [B][kbc+1]: rows padded
                                                                                // so tokens hit different banks
  float* part = reinterpret_cast<float*>(blk_info + B * (kbc + 1));             // [warps][16][B]
  float* tok_inv = part + kGemvWarps * 16 * B;                                  // [16]
  float* wred = tok_inv + kGemvMaxBatch;                                        // [warps][BM], then [16][B]
  float* part_odd = wred + kGemvWarps * BM + 16 * B;                            // partials of odd tiles
  const int64_t p0 = (int64_t)warp * ppc;
  const int np = (int)max((int64_t)0, min(p0 + ppc, KP) - p0);
  const int64_t my_tiles = r16 > (int64_t)blockIdx.x ? (r16 - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int64_t issued = 0;  // tiles requested (thread 0)
  auto request = [&](int64_t i) {
    const int s = (int)(i % S);
    const int64_t rt = blockIdx.x + i * gridDim.x;
    uint8_t* dst = smem + (size_t)s * stage_bytes;
    mbar_arrive_expect_tx(&full[s], stage_bytes);
    bulk_g2s(dst, a.w.nib + rt * KP * 32, nib_bytes, &full[s]);
    bulk_g2s(dst + nib_bytes, reinterpret_cast<const SV*>(a.w.scales) + rt * KP * 8, scl_bytes, &full[s]);
  };
  if (tid == 0)
    for (; issued < S && issued < my_tiles; ++issued) request(issued);
  if (a.early_trigger) pdl_launch_dependents();
  pdl_wait();
  rms_stats<BM, PRO>(a, wred, tok_inv, tid, lane, warp);
  split_x<PRO>(a, xs, blk_info, plane, kbc, 0, a.w.cols, tok_inv, tid, warp);
  __syncthreads();
  float* fin = wred;  // [16][B]
  int64_t k = 0;
  for (; k < my_tiles; ++k) {
    const int64_t rt = blockIdx.x + k * gridDim.x;
    const int s = (int)(k % S);
    // warp-uniform, so a warp runs its mma.sync with all lanes or not at all
    const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full[s], (uint32_t)((k / S) & 1), a.err, 0x601));
    if (ok) {
      const uint4* snib = reinterpret_cast<const uint4*>(smem + (size_t)s * stage_bytes) + p0 * 32 + lane;
      const SV* sscl = reinterpret_cast<const SV*>(smem + (size_t)s * stage_bytes + nib_bytes) + p0 * 8 + g;
      float tot[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) tot[j][0] = tot[j][1] = tot[j][2] = tot[j][3] = 0.0f;
      for (int p = 0; p < np; p += U) {
        uint4 w[U];
        SV sv[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (p + u < np) {
            w[u] = snib[(p + u) * 32];
            sv[u] = sscl[(p + u) * 8];
          }
        mma_pairs<NT, kF32, U>(tot, w, sv, p, np, B, g, t, xs, blk_info, plane, kbc, (int)(2 * p0));
      }
      float* pw = (k & 1) ? part_odd : part;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int b = 4 * j + t;  // columns 2t (hi) and 2t+1 (lo) of tile j
        if (b < B) {
          pw[(warp * 16 + g) * B + b] = tot[j][0] + tot[j][1];
          pw[(warp * 16 + g + 8) * B + b] = tot[j][2] + tot[j][3];
        }
      }
    }
    // one barrier: stage s read by every warp (refill it), the partials are in
    // place, and every wait succeeded
    if (__syncthreads_or(!ok)) break;
    if (tid == 0 && issued < my_tiles) {
      fence_proxy_async_smem();
      request(issued);
      ++issued;
    }
    if (k + 1 == my_tiles && !a.early_trigger) pdl_launch_dependents();
    // warp k % 8 reduces tile k and runs its epilogue while the other warps
    // go on to tile k + 1 (partials alternate between two buffers; the next
    // barrier waits for this warp)
    if (warp == (int)(k & (kGemvWarps - 1))) {
      const float* pk = (k & 1) ? part_odd : part;
      for (int i = lane; i < 16 * B; i += 32) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) v += pk[w * 16 * B + i];  // K-chunk order
        fin[i] = v;
      }
      __syncwarp();
      if (EPI == kEpiSwiglu) {
        for (int i = lane; i < 8 * B; i += 32) {
          const int r = i / B, b = i - r * B;
          const int64_t o = rt * 8 + r;
          if (o < a.w.rows / 2) a.y[b * a.y_stride + o] = silu_ref(fin[r * B + b]) * fin[(r + 8) * B + b];
        }
      } else {
        for (int i = lane; i < 16 * B; i += 32) {
          const int r = i / B, b = i - r * B;
          const int64_t R = rt * 16 + r;
          float h = 0.0f;
          if (R < a.w.rows) {
            if (EPI == kEpiStore && a.n_peer > 0) {
              h = fin[i];
              for (int p = 0; p < a.n_peer; ++p) a.peer_y[p][R * a.peer_row + b] = h;  // NVLink stores
            } else {
              float* d = a.y + b * a.y_stride + R;
              h = (EPI == kEpiAdd) ? *d + fin[i] : fin[i];  // residual: hidden[i] += out[i]
              *d = h;
            }
          }
          fin[i] = h;
        }
        // peer slots: the stores reach the other GPUs before this grid completes
        if (EPI == kEpiStore && a.n_peer > 0) __threadfence_system();
        if (a.ss_out) {
          __syncwarp();
          if (lane < B) {
            float q = 0.0f;
            for (int r = 0; r < 16; ++r) q = fmaf(fin[r * B + lane], fin[r * B + lane], q);
            a.ss_out[lane * a.w.r16 + rt] = q;
          }
        }
      }
      __syncwarp();
    }
  }
  // A wait gave up: let the copies still in flight land (bounded) before exiting.
  if (k < my_tiles && tid == 0)
    for (int64_t j = k; j < issued; ++j) mbar_wait_bounded(&full[j % S], (uint32_t)((j / S) & 1), a.err, 0x602);
}

using GemvKernel = void (*)(const GemvArgs);
#define AH_TRY_GEMV(expr)         \
  do {                            \
    int _rc = (expr);             \
    if (_rc != AH_OK) return _rc; \
  } while (0)

// Every prologue / epilogue for both scale formats: Q4_0 blocks (f16 scales)
// and the engine format of quantize() (f32 scales).
template <int NT, bool kRows, bool F>
GemvKernel pick_format(int pro, int epi) {
#define AH_K(P, E) (kRows ? k_gemv_q4_rows<NT, F, P, E> : k_gemv_q4<NT, F, P, E>)
  if (pro == kProPlain) {
    if (epi == kEpiStore) return AH_K(kProPlain, kEpiStore);
    if (epi == kEpiAdd) return AH_K(kProPlain, kEpiAdd);
    return AH_K(kProPlain, kEpiSwiglu);
  }
  if (epi == kEpiStore) return AH_K(kProRmsNorm, kEpiStore);
  if (epi == kEpiAdd) return AH_K(kProRmsNorm, kEpiAdd);
  return AH_K(kProRmsNorm, kEpiSwiglu);
#undef AH_K
}

template <int NT, bool kRows>
GemvKernel pick_kernel(bool f32s, int pro, int epi) {
  return f32s ? pick_format<NT, kRows, true>(pro, epi) : pick_format<NT, kRows, false>(pro, epi);
}

}  // namespace

GemvPlan gemv_plan(const Q4Tiled& w, int batch, bool rows_mode, int64_t kp_window) {
  GemvPlan p{};
  p.nt = (batch + 3) / 4;
  p.rows_mode = rows_mode;
  const int64_t kp = kp_window > 0 ? kp_window : w.kp;
  p.pairs_per_chunk = (kp + kGemvCluster - 1) / kGemvCluster;  // one K-chunk per warp (rows) or cluster CTA
  p.ksplit = 1;
  const int64_t kbc = rows_mode ? 2 * w.kp : 2 * p.pairs_per_chunk;
  const int64_t plane = kbc * 64 + 64;
  p.smem = (size_t)2 * batch * plane + (size_t)batch * (kbc + 1) * 16 + (size_t)kGemvWarps * 16 * batch * 4 +
           (size_t)kGemvMaxBatch * 4 + (size_t)kGemvWarps * (4 * p.nt) * 4 + (size_t)16 * batch * 4 + 16;
  if (!rows_mode) p.smem += (size_t)2 * kGemvCluster * 16 * batch * 4;  // DSMEM partial slots
  if (rows_mode) p.smem += (size_t)kGemvWarps * 16 * batch * 4;  // partials of odd tiles
  p.smem_base = p.smem;
  p.n_stages = 0;
  if (rows_mode) {  // tile stages (nibbles + scales) and their mbarriers in front
    const size_t stage = (size_t)w.kp * 512 + (size_t)w.kp * 8 * (w.f32_scales ? 16 : 8);
    int n = 0;
    while (n < kGemvMaxStages &&
           (size_t)(n + 1) * stage + (((size_t)(n + 1) * 8 + 15) & ~(size_t)15) + p.smem_base <= (size_t)kGemvRowsCtaSmem)
      ++n;
    if (n >= 2) {
      p.n_stages = n;
      p.smem = (size_t)n * stage + (((size_t)n * 8 + 15) & ~(size_t)15) + p.smem_base;
    }
  }
  return p;
}

GemvPlan gemv_plan(const Q4Tiled& w, int batch) { return gemv_plan(w, batch, false, 0); }

namespace {
GemvKernel select_kernel(const GemvPlan& plan, bool f32s, int pro, int epi) {
  if (plan.rows_mode) {
    switch (plan.nt) {
      case 1: return pick_kernel<1, true>(f32s, pro, epi);
      case 2: return pick_kernel<2, true>(f32s, pro, epi);
      case 3: return pick_kernel<3, true>(f32s, pro, epi);
      default: return pick_kernel<4, true>(f32s, pro, epi);
    }
  }
  switch (plan.nt) {
    case 1: return pick_kernel<1, false>(f32s, pro, epi);
    case 2: return pick_kernel<2, false>(f32s, pro, epi);
    case 3: return pick_kernel<3, false>(f32s, pro, epi);
    default: return pick_kernel<4, false>(f32s, pro, epi);
  }
}

// Per (device, kernel, smem): raises the dynamic shared-memory cap once and
// caches how many clusters (cluster mode) or CTAs (rows mode) fit in one wave.
int kernel_setup(GemvKernel kern, const GemvPlan& plan, int* capacity) {
  static std::mutex mu;
  struct Entry { int dev; void* k; size_t smem; int cap; };
  static std::vector<Entry> cache;
  struct Cap { int dev; void* k; size_t smem; };  // the largest cap set per (device, kernel)
  static std::vector<Cap> caps;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  for (auto& e : cache)
    if (e.dev == dev && e.k == (void*)kern && e.smem == plan.smem) {
      *capacity = e.cap;
      return AH_OK;
    }
  // the attribute is per kernel: raise it, never lower it below a size an
  // earlier plan of the same kernel still launches with
  Cap* cp = nullptr;
  for (auto& c : caps)
    if (c.dev == dev && c.k == (void*)kern) cp = &c;
  if (!cp || cp->smem < plan.smem) {
    AH_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem));
    if (cp) cp->smem = plan.smem;
    else caps.push_back({dev, (void*)kern, plan.smem});
  }
  int n = 0;
  if (plan.rows_mode) {
    AH_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kGemvThreads, plan.smem));
    n *= sm_count();
  } else {
    cudaLaunchConfig_t q{};
    q.gridDim = dim3(kGemvCluster, 1, 1);
    q.blockDim = dim3(kGemvThreads, 1, 1);
    q.dynamicSmemBytes = plan.smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kGemvCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    q.attrs = attr;
    q.numAttrs = 1;
    AH_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &q));
  }
  cache.push_back({dev, (void*)kern, plan.smem, n});
  *capacity = n;
  return AH_OK;
}

// Cluster mode for GEMVs whose row groups fit in one wave (one pass each) and
// for those with fewer than two row tiles per resident rows-mode CTA; rows mode
// for many-tile GEMVs whose full-K split of x fits comfortably in shared
// memory beside at least two tile stages (it is then amortised over several
// tiles per CTA).
int choose_plan(const Q4Tiled& w, int batch, int pro, int epi, GemvPlan* plan, GemvKernel* kern, int* cap,
                int64_t kp_window = 0) {
  GemvPlan pc = gemv_plan(w, batch, false, kp_window);
  if (pc.smem > (size_t)kGemvSmemLimit)
    return fail(AH_EUNSUPPORTED, "gemv: batch %d x %lld columns needs %zu B of shared memory per CTA (limit %d)",
                batch, (long long)w.cols, pc.smem, kGemvSmemLimit);
  GemvKernel kc = select_kernel(pc, w.f32_scales, pro, epi);
  if (!kc) return fail(AH_EUNSUPPORTED, "gemv: no kernel for prologue %d / epilogue %d", pro, epi);
  int ccap = 0;
  AH_TRY_GEMV(kernel_setup(kc, pc, &ccap));
  const int64_t n_rg = (w.r16 + kGemvWarps - 1) / kGemvWarps;
  GemvPlan pr = gemv_plan(w, batch, true);
  if (kp_window == 0 && n_rg > ccap && pr.smem_base <= (size_t)kGemvRowsSmem && pr.n_stages >= 2 && aligned16(w.nib) &&
      aligned16(w.scales)) {
    GemvKernel kr = select_kernel(pr, w.f32_scales, pro, epi);
    int rcap = 0;
    AH_TRY_GEMV(kernel_setup(kr, pr, &rcap));
    if (rcap > 0 && w.r16 >= 2 * (int64_t)rcap) {  // the stages pay off from two tiles per CTA
      *plan = pr;
      *kern = kr;
      *cap = rcap;
      return AH_OK;
    }
  }
  AH_REQUIRE(ccap > 0, "gemv: no cluster of this kernel fits on the device");
  *plan = pc;
  *kern = kc;
  *cap = ccap;
  return AH_OK;
}
}  // namespace

namespace {
// The largest token count (<= batch) whose split of x fits one CTA's shared
// memory; larger batches run as several launches over token slices.
int max_sub_batch(const Q4Tiled& w, int batch) {
  for (int b = batch; b >= 1; --b)
    if (gemv_plan(w, b, false).smem <= (size_t)kGemvSmemLimit) return b;
  return 0;
}
int gemv_launch_one(GemvArgs a, int pro, int epi, cudaStream_t st, bool pdl);
}  // namespace

namespace {
// K windows for a batch whose split of x does not fit one CTA: the fewest
// windows (each launch then covers kp_window block pairs) whose plan fits, or 0.
// Only for epilogues that can accumulate (store, then residual adds) into a
// local y; SwiGLU and the peer scatter need the whole sum and take token slices.
int64_t k_window(const Q4Tiled& w, int batch, int epi, int n_peer) {
  if (epi == kEpiSwiglu || n_peer > 0) return 0;
  for (int64_t nw = 2; nw <= 16; ++nw) {
    const int64_t win = (w.kp + nw - 1) / nw;
    if (gemv_plan(w, batch, false, win).smem <= (size_t)kGemvSmemLimit) return win;
  }
  return 0;
}
}  // namespace

int gemv_prepare(const Q4Tiled& w, int batch, int pro, int epi) {
  AH_REQUIRE(batch >= 1 && batch <= kGemvMaxBatch, "gemv: batch must be 1..16");
  const int sb = max_sub_batch(w, batch);
  AH_REQUIRE(sb >= 1, "gemv: %lld columns do not fit one CTA even for one token", (long long)w.cols);
  GemvPlan plan;
  GemvKernel kern;
  int cap;
  if (sb < batch) {
    // the peer scatter never combines with windows; the decoder's o / down
    // GEMVs under tensor parallelism take token slices, prepared below
    const int64_t win = k_window(w, batch, epi, 0);
    if (win > 0) {
      AH_TRY_GEMV(choose_plan(w, batch, pro, epi, &plan, &kern, &cap, win));
      AH_TRY_GEMV(choose_plan(w, batch, pro, kEpiAdd, &plan, &kern, &cap, win));
    }
  }
  AH_TRY_GEMV(choose_plan(w, sb, pro, epi, &plan, &kern, &cap));
  if (batch % sb) AH_TRY_GEMV(choose_plan(w, batch % sb, pro, epi, &plan, &kern, &cap));
  return AH_OK;
}

int gemv_launch(GemvArgs a, int pro, int epi, cudaStream_t st, bool pdl) {
  AH_REQUIRE(a.batch >= 1 && a.batch <= kGemvMaxBatch, "gemv: batch must be 1..16");
  const int sb = max_sub_batch(a.w, a.batch);
  AH_REQUIRE(sb >= 1, "gemv: %lld columns do not fit one CTA even for one token", (long long)a.w.cols);
  if (sb == a.batch) return gemv_launch_one(a, pro, epi, st, pdl);
  const int64_t win = k_window(a.w, a.batch, epi, a.n_peer);
  if (win > 0) {
    // K windows: every weight byte is read once; the first window stores (or
    // adds, for a residual epilogue) and the later ones add into y; the last
    // writes the sums of squares of the final values
    for (int64_t pb = 0, i = 0; pb < a.w.kp; pb += win, ++i) {
      GemvArgs s = a;
      s.pair_begin = pb;
      s.pair_end = std::min(pb + win, a.w.kp);
      if (s.pair_end < a.w.kp) s.ss_out = nullptr;
      AH_TRY_GEMV(gemv_launch_one(s, pro, i == 0 ? epi : kEpiAdd, st, pdl));
    }
    return AH_OK;
  }
  // token slices: every per-token operand moves by the slice start
  for (int b0 = 0; b0 < a.batch; b0 += sb) {
    GemvArgs s = a;
    s.batch = std::min(sb, a.batch - b0);
    s.x = a.x + (int64_t)b0 * a.x_stride;
    s.y = a.y + (int64_t)b0 * a.y_stride;
    if (a.ss_in) s.ss_in = a.ss_in + (int64_t)b0 * a.n_ss_in;
    if (a.ss_out) s.ss_out = a.ss_out + (int64_t)b0 * a.w.r16;
    for (int p = 0; p < a.n_peer; ++p) s.peer_y[p] = a.peer_y[p] + b0;
    AH_TRY_GEMV(gemv_launch_one(s, pro, epi, st, pdl));
  }
  return AH_OK;
}

namespace {
int gemv_launch_one(GemvArgs a, int pro, int epi, cudaStream_t st, bool pdl) {
  AH_REQUIRE(a.batch >= 1 && a.batch <= kGemvMaxBatch, "gemv: batch must be 1..16");
  AH_REQUIRE(pro != kProRmsNorm || (a.norm_w != nullptr && a.ss_in != nullptr && a.n_ss_in > 0),
             "gemv: RMSNorm prologue needs a norm weight and the producer's partial sums of squares");
  AH_REQUIRE(a.x != nullptr && a.y != nullptr, "gemv: null activation or output");
  AH_REQUIRE(epi != kEpiSwiglu || a.w.rows % 16 == 0, "gemv: SwiGLU epilogue needs interleaved rows %% 16 == 0");
  GemvPlan plan;
  GemvKernel kern;
  int cap = 0;
  const int64_t kp_window = a.pair_end > 0 ? a.pair_end - a.pair_begin : 0;
  AH_TRY_GEMV(choose_plan(a.w, a.batch, pro, epi, &plan, &kern, &cap, kp_window));
  a.pairs_per_chunk = plan.pairs_per_chunk;
  a.n_stages = plan.n_stages;
  a.err = device_error_word();
  AH_REQUIRE(!plan.rows_mode || a.err, "gemv: device error word unavailable");
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (plan.rows_mode) {
    const int64_t n = std::min<int64_t>(a.w.r16, cap);
    a.early_trigger = a.w.r16 <= cap ? 1 : 0;
    cfg.gridDim = dim3((unsigned)n, 1, 1);
  } else {
    const int64_t n_rg = (a.w.r16 + kGemvWarps - 1) / kGemvWarps;  // row groups
    const int64_t n_clusters = std::min<int64_t>(n_rg, cap);
    a.early_trigger = n_rg <= cap ? 1 : 0;
    cfg.gridDim = dim3((unsigned)(n_clusters * kGemvCluster), 1, 1);
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = kGemvCluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  ++na;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (inject_failure(AH_INJECT_LAUNCH)) return fail(AH_ECUDA, "gemv: kernel launch failed (injected)");
  AH_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return AH_OK;
}
}  // namespace

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
                                                             int64_t gs, int64_t row0, int64_t byte0) {
  // out[r] for global row row0 + r; scales start at row row0; packed holds the
  // bytes from byte0 on (the nibble of linear index i is in byte i / 2)
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t n_gpr = (cols + gs - 1) / gs;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    float sum = 0.0f;
    const int64_t row_off = (row0 + r) * cols;
    for (int64_t j = lane; j < cols; j += 32) {
      const int64_t lin = row_off + j;
      const uint32_t byte = packed[(lin >> 1) - byte0];
      const uint32_t nib = (lin & 1) ? (byte >> 4) & 0xFu : byte & 0xFu;
      const float wv = __fmul_rn((float)(int)nib - 8.0f, scales[r * n_gpr + j / gs]);
      sum = __fadd_rn(sum, __fmul_rn(wv, x[j]));  // no contraction, as in math.rs:412-413
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) out[r] = sum;
  }
}
// The gate and up GEMVs of inference/ffn.rs:155-174 in one pass over x (one
// warp per FFN row, engine format as stored): scratch_gate[i] = gate_i . x,
// scratch_up[i] = up_i . x, scratch_act[i] = silu(gate) * up (math.rs:83-95).
__global__ void __launch_bounds__(256) k_gate_up_silu_engine(
    float* __restrict__ sg, float* __restrict__ su, float* __restrict__ act, const float* __restrict__ g_s,
    const uint8_t* __restrict__ g_p, const float* __restrict__ u_s, const uint8_t* __restrict__ u_p,
    const float* __restrict__ x, int64_t n_ff, int64_t n_embd, int64_t gs) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t n_gpr = (n_embd + gs - 1) / gs;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_ff; r += warps) {
    float a = 0.0f, b = 0.0f;
    const int64_t row_off = r * n_embd;
    for (int64_t j = lane; j < n_embd; j += 32) {
      const int64_t lin = row_off + j;
      const int sh = (lin & 1) ? 4 : 0;
      const float xv = x[j];
      const int64_t si = r * n_gpr + j / gs;
      const float wg = __fmul_rn((float)(int)((g_p[lin >> 1] >> sh) & 0xFu) - 8.0f, g_s[si]);
      const float wu = __fmul_rn((float)(int)((u_p[lin >> 1] >> sh) & 0xFu) - 8.0f, u_s[si]);
      a = __fadd_rn(a, __fmul_rn(wg, xv));
      b = __fadd_rn(b, __fmul_rn(wu, xv));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
      b += __shfl_xor_sync(0xFFFFFFFFu, b, o);
    }
    if (lane == 0) {
      sg[r] = a;
      su[r] = b;
      act[r] = silu_ref(a) * b;
    }
  }
}
// Copies n floats from device-mapped (pinned) host memory over the bus:
// avoids the copy engine's start-up for the small activation vectors.
__global__ void __launch_bounds__(256) k_pull_f32(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}
// The device address of a pinned, device-mapped host buffer, or null (pageable).
const void* mapped_host_ptr(const void* p) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}
__global__ void k_zero(float* p, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = 0.0f;
}
}  // namespace
int gemv_rows_window(float* out, const float* scales, const uint8_t* packed, const float* x, int64_t rows,
                     int64_t cols, int64_t gs, int64_t row0, int64_t byte0, cudaStream_t st) {
  const int64_t grid = std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 8);
  k_gemv_engine_generic<<<(int)grid, 256, 0, st>>>(out, scales, packed, x, rows, cols, gs, row0, byte0);
  AH_LAUNCH_CHECK();
  return AH_OK;
}
namespace {
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
  if (w->stage) cudaFree(w->stage);
  if (w->host_graph) cudaGraphExecDestroy(w->host_graph);
  if (w->host_cap) cudaStreamDestroy(w->host_cap);
  cudaSetDevice(cur);
  delete w;
  return AH_OK;
}

int ah_q4w_gemv_host(const AhQ4Weight* cw, const float* x_host, float* y_host, int batch, void* stream) {
  AH_REQUIRE(cw && x_host && y_host, "q4w_gemv_host: null argument");
  AH_REQUIRE(batch >= 1 && batch <= kGemvMaxBatch, "q4w_gemv_host: batch must be 1..16");
  AhQ4Weight* w = const_cast<AhQ4Weight*>(cw);
  std::lock_guard<std::mutex> lk(w->mu);
  const size_t x_max = ((size_t)kGemvMaxBatch * w->t.cols * 4 + 255) / 256 * 256;
  if (!w->stage) {
    if (ah::dev_malloc(&w->stage, x_max + (size_t)kGemvMaxBatch * w->t.rows * 4) != cudaSuccess) {
      cudaGetLastError();
      w->stage = nullptr;
      return fail(AH_ENOMEM, "q4w_gemv_host: staging allocation failed");
    }
  }
  float* xd = static_cast<float*>(w->stage);
  float* yd = reinterpret_cast<float*>(static_cast<uint8_t*>(w->stage) + x_max);
  cudaStream_t st = as_stream(stream);
  // pinned host buffers are reached directly: a small kernel pulls x over the
  // bus and the GEMV stores y into the mapped buffer; pageable ones go
  // through the copy engine
  const int64_t nx = (int64_t)batch * w->t.cols;
  const float* xm = static_cast<const float*>(mapped_host_ptr(x_host));
  float* ym = static_cast<float*>(const_cast<void*>(mapped_host_ptr(y_host)));
  const int pull_grid = (int)std::min<int64_t>((nx + 1023) / 1024, 64);
  if (xm && ym) {  // both pinned: one graph launch for the pull and the GEMV
    if (!w->host_graph || w->hg_x != xm || w->hg_y != ym || w->hg_batch != batch) {
      if (w->host_graph) cudaGraphExecDestroy(w->host_graph);
      w->host_graph = nullptr;
      AH_TRY_GEMV(gemv_prepare(w->t, batch, kProPlain, kEpiStore));  // kernel attributes before the capture
      if (!w->host_cap) AH_CUDA_TRY(cudaStreamCreateWithFlags(&w->host_cap, cudaStreamNonBlocking));
      cudaGraph_t g = nullptr;
      AH_CUDA_TRY(cudaStreamBeginCapture(w->host_cap, cudaStreamCaptureModeThreadLocal));
      k_pull_f32<<<pull_grid, 256, 0, w->host_cap>>>(xd, xm, nx);
      const int rc = ah_q4w_gemv(w, xd, ym, batch, w->host_cap);
      const cudaError_t e = cudaStreamEndCapture(w->host_cap, &g);
      if (rc != AH_OK || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return rc != AH_OK ? rc : fail(AH_ECUDA, "q4w_gemv_host: capture failed: %s", cudaGetErrorString(e));
      }
      const cudaError_t ei = cudaGraphInstantiate(&w->host_graph, g, 0);
      cudaGraphDestroy(g);
      if (ei != cudaSuccess) {
        w->host_graph = nullptr;
        return fail(AH_ECUDA, "q4w_gemv_host: graph instantiate: %s", cudaGetErrorString(ei));
      }
      w->hg_x = xm;
      w->hg_y = ym;
      w->hg_batch = batch;
    }
    AH_CUDA_TRY(cudaGraphLaunch(w->host_graph, st));
    AH_CUDA_TRY(cudaStreamSynchronize(st));
    return AH_OK;
  }
  if (xm) {
    k_pull_f32<<<pull_grid, 256, 0, st>>>(xd, xm, nx);
    AH_LAUNCH_CHECK();
  } else {
    AH_CUDA_TRY(cudaMemcpyAsync(xd, x_host, (size_t)nx * 4, cudaMemcpyHostToDevice, st));
  }
  const int rc = ah_q4w_gemv(w, xd, ym ? ym : yd, batch, stream);
  if (rc != AH_OK) return rc;
  if (!ym) AH_CUDA_TRY(cudaMemcpyAsync(y_host, yd, (size_t)batch * w->t.rows * 4, cudaMemcpyDeviceToHost, st));
  AH_CUDA_TRY(cudaStreamSynchronize(st));
  return AH_OK;
}

int ah_q4w_shape(const AhQ4Weight* w, int64_t* rows, int64_t* cols) {
  AH_REQUIRE(w && rows && cols, "q4w_shape: null argument");
  *rows = w->t.rows;
  *cols = w->t.cols;
  return AH_OK;
}

int64_t ah_q4w_weight_bytes(const AhQ4Weight* w) { return w ? w->weight_bytes : 0; }

int ah_q4w_planes(const AhQ4Weight* w, const void** nib, size_t* nib_bytes, const void** scales, size_t* scale_bytes,
                  int* f32_scales) {
  AH_REQUIRE(w && nib && nib_bytes && scales && scale_bytes && f32_scales, "q4w_planes: null argument");
  *nib = w->nib_alloc;
  *nib_bytes = (size_t)w->t.r16 * w->t.kp * 32 * 16;
  *scales = w->scale_alloc;
  *scale_bytes = (size_t)w->t.r16 * w->t.kp * 8 * (w->t.f32_scales ? 16 : 8);
  *f32_scales = w->t.f32_scales ? 1 : 0;
  return AH_OK;
}

int ah_q4w_gemv(const AhQ4Weight* w, const float* x, float* y, int batch, void* stream) {
  AH_REQUIRE(w && x && y, "q4w_gemv: null argument");
  AH_REQUIRE(batch >= 1 && batch <= kGemvMaxBatch, "q4w_gemv: batch must be 1..16");
  GemvArgs a{};
  a.w = w->t;
  a.x = x;
  a.x_stride = w->t.cols;
  a.y = y;
  a.y_stride = w->t.rows;
  a.batch = batch;
  return gemv_launch(a, kProPlain, kEpiStore, as_stream(stream), true);
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
  k_gemv_engine_generic<<<(int)grid, 256, 0, st>>>(out, scales, packed, x, rows, cols, gs, 0, 0);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_matvec_4bit_into(float* out, const float* scales, const uint8_t* packed, const float* x, int64_t dim, int64_t gs,
                        void* stream) {
  return ah_gemv_4bit_into(out, scales, packed, x, dim, dim, gs, stream);
}

int ah_gemv_4bit_rows(float* out, const float* scales, const uint8_t* packed, const float* x, int64_t row_start,
                      int64_t row_end, int64_t cols, int64_t gs, void* stream) {
  AH_REQUIRE(row_start >= 0 && row_end >= row_start && cols >= 0, "gemv_4bit_rows: bad row range or shape");
  const int64_t rows = row_end - row_start;
  if (rows == 0) return AH_OK;
  AH_REQUIRE(out != nullptr, "gemv_4bit_rows: null out");
  cudaStream_t st = as_stream(stream);
  if (cols == 0) {  // every row sums nothing (math.rs:395-418 with cols = 0)
    k_zero<<<(int)std::min<int64_t>((rows + 255) / 256, 1024), 256, 0, st>>>(out, rows);
    AH_LAUNCH_CHECK();
    return AH_OK;
  }
  AH_REQUIRE(scales && packed && x, "gemv_4bit_rows: null input");
  if (gs < 1) gs = 1;
  const int64_t n_gpr = (cols + gs - 1) / gs;
  const int64_t grid = std::min<int64_t>((rows + 7) / 8, (int64_t)sm_count() * 8);
  k_gemv_engine_generic<<<(int)grid, 256, 0, st>>>(out, scales + row_start * n_gpr, packed, x, rows, cols, gs,
                                                   row_start, 0);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_swiglu_4bit_into(float* out, const float* input, const float* gate_scales, const uint8_t* gate_packed,
                        const float* up_scales, const uint8_t* up_packed, const float* down_scales,
                        const uint8_t* down_packed, int64_t n_embd, int64_t n_ff, int64_t gs, float* scratch_gate,
                        float* scratch_up, float* scratch_act, void* stream) {
  AH_REQUIRE(n_embd >= 0 && n_ff >= 0, "swiglu_4bit_into: negative shape");
  cudaStream_t st = as_stream(stream);
  if (gs < 1) gs = 1;
  if (n_ff > 0) {
    AH_REQUIRE(scratch_gate && scratch_up && scratch_act, "swiglu_4bit_into: null scratch");
    if (n_embd == 0 || input == nullptr) {  // gemv_4bit_into on empty x: zeros (math.rs:264-267)
      for (float* z : {scratch_gate, scratch_up, scratch_act}) {
        k_zero<<<(int)std::min<int64_t>((n_ff + 255) / 256, 1024), 256, 0, st>>>(z, n_ff);
        AH_LAUNCH_CHECK();
      }
    } else {
      AH_REQUIRE(gate_scales && gate_packed && up_scales && up_packed, "swiglu_4bit_into: null gate/up weights");
      const int64_t grid = std::min<int64_t>((n_ff + 7) / 8, (int64_t)sm_count() * 8);
      k_gate_up_silu_engine<<<(int)grid, 256, 0, st>>>(scratch_gate, scratch_up, scratch_act, gate_scales,
                                                        gate_packed, up_scales, up_packed, input, n_ff, n_embd, gs);
      AH_LAUNCH_CHECK();
    }
  }
  if (n_embd == 0) return AH_OK;
  return ah_gemv_4bit_into(out, down_scales, down_packed, n_ff > 0 ? scratch_act : nullptr, n_embd, n_ff, gs,
                           stream);
}

int ah_q4w_from_engine_gate_up(const float* gate_scales, const uint8_t* gate_packed, const float* up_scales,
                               const uint8_t* up_packed, int64_t n_ff, int64_t n_embd, AhQ4Weight** out,
                               void* stream) {
  const float* sc[2] = {gate_scales, up_scales};
  const uint8_t* pk[2] = {gate_packed, up_packed};
  const int64_t r[2] = {n_ff, n_ff};
  AH_REQUIRE(n_ff % 8 == 0, "q4w_from_engine_gate_up: n_ff must be a multiple of 8");
  return q4w_create_engine_multi(sc, pk, r, 2, 1, n_embd, out, as_stream(stream));
}

int ah_q4w_from_q4_0_gate_up(const void* gate_blocks, const void* up_blocks, int64_t n_ff, int64_t n_embd,
                             AhQ4Weight** out, void* stream) {
  const void* srcs[2] = {gate_blocks, up_blocks};
  const int64_t r[2] = {n_ff, n_ff};
  AH_REQUIRE(n_ff % 8 == 0, "q4w_from_q4_0_gate_up: n_ff must be a multiple of 8");
  return q4w_create_q4_0_multi(srcs, r, 2, 1, n_embd, out, as_stream(stream));
}

int ah_q4w_swiglu(const AhQ4Weight* gate_up, const AhQ4Weight* down, const float* x, float* act, float* out,
                  int batch, void* stream) {
  AH_REQUIRE(gate_up && down && x && act && out, "q4w_swiglu: null argument");
  AH_REQUIRE(batch >= 1 && batch <= kGemvMaxBatch, "q4w_swiglu: batch must be 1..16");
  const Q4Tiled& gu = gate_up->t;
  const Q4Tiled& dn = down->t;
  AH_REQUIRE(gu.rows % 16 == 0 && dn.cols == gu.rows / 2 && dn.rows == gu.cols,
             "q4w_swiglu: gate/up must be [2*n_ff][n_embd] (n_ff %% 8 == 0) and down [n_embd][n_ff]");
  GemvArgs a{};
  a.w = gu;
  a.x = x;
  a.x_stride = gu.cols;
  a.y = act;
  a.y_stride = gu.rows / 2;
  a.batch = batch;
  const int rc = gemv_launch(a, kProPlain, kEpiSwiglu, as_stream(stream), true);
  if (rc != AH_OK) return rc;
  GemvArgs d{};
  d.w = dn;
  d.x = act;
  d.x_stride = dn.cols;
  d.y = out;
  d.y_stride = dn.rows;
  d.batch = batch;
  return gemv_launch(d, kProPlain, kEpiStore, as_stream(stream), true);
}

}  // extern "C"
