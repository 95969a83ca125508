// ah_prefill.cu — row kernels of the decoder's prompt prefill.  The prompt is
// processed in chunks of positions; for each chunk and layer the projections
// run as tcgen05 GEMMs (ah_gemm_tc.cu) and these kernels do the rest: rows are
// (sequence, position) pairs, row r = b * cnt + i for position p0 + i.
#include <algorithm>
#include <cmath>

#include "ah_prefill.cuh"
#include "ah_sm100.cuh"

namespace ah {
namespace {

__device__ __forceinline__ float silu_f(float x) {  // inference/math.rs:83-95
  const float sg = x >= 0.0f ? __fdiv_rn(1.0f, 1.0f + expf(-x)) : __fdiv_rn(expf(x), 1.0f + expf(x));
  return x * sg;
}

__global__ void __launch_bounds__(256) k_embed_rows(const uint16_t* __restrict__ emb, const int* __restrict__ prompt,
                                                    PrefillRows pr, int d, int vocab, float* __restrict__ hidden) {
  const int64_t r = blockIdx.y;
  const int b = (int)(r / pr.cnt), i = (int)(r - (int64_t)b * pr.cnt);
  const int t = prompt[(size_t)b * pr.n_prompt + pr.p0 + i];
  const int tv = (t >= 0 && t < vocab) ? t : 0;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < d; c += gridDim.x * blockDim.x)
    hidden[r * d + c] = f16_bits_to_f32(emb[(size_t)tv * d + c]);
}

__global__ void __launch_bounds__(256) k_rmsnorm_rows(const float* __restrict__ x, const uint16_t* __restrict__ w,
                                                      float eps, int d, float* __restrict__ out) {
  const int64_t r = blockIdx.x;
  const float* xr = x + r * d;
  float ss = 0.0f;
  for (int c = threadIdx.x; c < d; c += blockDim.x) ss = fmaf(xr[c], xr[c], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  __shared__ float red[8];
  __shared__ float inv;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
    inv = __fdiv_rn(1.0f, sqrtf(__fdiv_rn(s, (float)d) + eps));  // inference/math.rs:59
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x)
    out[r * d + c] = (xr[c] * inv) * __half2float(__ushort_as_half(w[c]));
}

// grid (rows), block 128: RoPE on the nh local q heads (in place) and the nkv k
// heads, then k and v rounded to f16 into the cache.
__global__ void __launch_bounds__(128) k_rope_append_rows(float* __restrict__ qkv, int ld,
                                                          const float2* __restrict__ rope, uint16_t* __restrict__ kc,
                                                          uint16_t* __restrict__ vc, int layer, int n_layer, int nh,
                                                          int nkv, int hd, int max_seq, PrefillRows pr) {
  const int64_t r = blockIdx.x;
  const int b = (int)(r / pr.cnt), i = (int)(r - (int64_t)b * pr.cnt);
  const int pos = pr.p0 + i;
  const int half = hd / 2, dq = nh * hd, dkv = nkv * hd;
  float* row = qkv + r * ld;
  const float2* cs = rope + (size_t)pos * half;
  // RoPE on adjacent pairs (2k, 2k+1), theta_k = pos * base^(-k/half) (math.rs:119-151)
  for (int e = threadIdx.x; e < (nh + nkv) * half; e += blockDim.x) {
    const int hh = e / half, k = e - hh * half;
    float* p = row + hh * hd + 2 * k;  // q heads first, then the k heads (at dq)
    const float x0 = p[0], x1 = p[1];
    const float2 c = cs[k];
    const float y0 = x0 * c.x - x1 * c.y, y1 = x0 * c.y + x1 * c.x;
    if (hh < nh) {
      p[0] = y0;
      p[1] = y1;
    } else {
      const int h = hh - nh;
      uint16_t* kr = kc + ((((size_t)b * n_layer + layer) * nkv + h) * max_seq + pos) * hd;
      kr[2 * k] = __half_as_ushort(__float2half_rn(y0));
      kr[2 * k + 1] = __half_as_ushort(__float2half_rn(y1));
    }
  }
  for (int e = threadIdx.x; e < dkv; e += blockDim.x) {
    const int h = e / hd, c = e - h * hd;
    uint16_t* vr = vc + ((((size_t)b * n_layer + layer) * nkv + h) * max_seq + pos) * hd;
    vr[c] = __half_as_ushort(__float2half_rn(row[dq + dkv + e]));
  }
}

__global__ void __launch_bounds__(256) k_add_rows(float* __restrict__ h, const float* __restrict__ p, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    h[i] += p[i];  // residual: hidden[i] += out[i]
}

__global__ void __launch_bounds__(256) k_swiglu_rows(const float* __restrict__ gu, int64_t rows, int nff,
                                                     float* __restrict__ act) {
  const int64_t n = rows * nff;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / nff;
    const int i = (int)(e - r * nff);
    const float* g = gu + r * (2 * (int64_t)nff) + (i >> 3) * 16 + (i & 7);
    act[e] = silu_f(g[0]) * g[8];
  }
}

// Causal attention of a chunk's queries over the f16 KV cache, f32 arithmetic
// as in the decode step (q after RoPE in f32, k and v as cached).  grid
// (ceil(cnt / 64), nh, B), 256 threads: CTA (t, hq, b) takes queries
// p0 + 64t .. +63 of head hq and walks the cache rows 0 .. last query in tiles
// of 64 keys with an online softmax.  Thread (ty, tx) = (tid / 16, tid % 16)
// holds the 4 x 4 score block rows 4ty.., keys 4tx.. and the output rows
// 4ty.. x columns tx*HD/16..; q and k sit transposed in shared memory so a
// score block reads one float4 of each per head dimension.
constexpr int kQT = 64, kKT = 64;

template <int HD>
struct PfSmem {
  static constexpr int kQt = HD * kQT;          // floats: q^T [HD][64]
  static constexpr int kKt = HD * kKT;          // k^T [HD][64]
  static constexpr int kV = kKT * HD;           // v [64][HD]
  static constexpr int kP = kQT * (kKT + 4);    // p [64][68]
  static constexpr size_t kBytes = sizeof(float) * (size_t)(kQt + kKt + kV + kP);
};

template <int HD>
__global__ void __launch_bounds__(256) k_prefill_attn(const float* __restrict__ qkv, int ld,
                                                      const uint16_t* __restrict__ kc,
                                                      const uint16_t* __restrict__ vc, int layer, int n_layer,
                                                      int nh, int nkv, int max_seq, float scale, PrefillRows pr,
                                                      float* __restrict__ out, int ld_out) {
  constexpr int CW = HD / 16;  // output columns per thread
  extern __shared__ __align__(16) float sm[];
  float* Qt = sm;
  float* Kt = Qt + PfSmem<HD>::kQt;
  float* Vs = Kt + PfSmem<HD>::kKt;
  float* Ps = Vs + PfSmem<HD>::kV;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int q0 = blockIdx.x * kQT;  // first query of the tile, within the chunk
  const int nq = min(kQT, pr.cnt - q0);
  const int G = nh / nkv, hk = hq / G;
  const int qpos_last = pr.p0 + q0 + nq - 1;  // causal limit of the tile
  const size_t head_off = (((size_t)b * n_layer + layer) * nkv + hk) * max_seq * HD;
  const uint16_t* kh = kc + head_off;
  const uint16_t* vh = vc + head_off;
  // q tile, transposed
  for (int e = tid; e < kQT * HD; e += 256) {
    const int i = e / HD, c = e - i * HD;
    Qt[c * kQT + i] = i < nq ? qkv[((int64_t)b * pr.cnt + q0 + i) * ld + hq * HD + c] : 0.0f;
  }
  float m[4], l[4], o[4][CW];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < CW; ++c) o[i][c] = 0.0f;
  }
  const int n_kt = qpos_last / kKT + 1;
  for (int kt = 0; kt < n_kt; ++kt) {
    const int k0 = kt * kKT;
    __syncthreads();  // the previous tile's k, v and p are consumed
    for (int e = tid; e < kKT * HD; e += 256) {
      const int j = e / HD, c = e - j * HD;
      const bool live = k0 + j <= qpos_last;
      const float kv = live ? __half2float(__ushort_as_half(kh[(size_t)(k0 + j) * HD + c])) : 0.0f;
      const float vv = live ? __half2float(__ushort_as_half(vh[(size_t)(k0 + j) * HD + c])) : 0.0f;
      Kt[c * kKT + j] = kv;
      Vs[j * HD + c] = vv;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 8
    for (int c = 0; c < HD; ++c) {
      const float4 qv = *reinterpret_cast<const float4*>(Qt + c * kQT + 4 * ty);
      const float4 kv = *reinterpret_cast<const float4*>(Kt + c * kKT + 4 * tx);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qa[i], ka[j], s[i][j]);
    }
    // causal mask, online softmax (each row's 64 keys live in 16 lanes)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qp = pr.p0 + q0 + 4 * ty + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kp = k0 + 4 * tx + j;
        s[i][j] = kp <= qp ? s[i][j] * scale : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
      const float mn = fmaxf(m[i], mx);
      const float alpha = mn == -INFINITY ? 1.0f : expf(m[i] - mn);
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = mn == -INFINITY ? 0.0f : expf(s[i][j] - mn);
        Ps[(4 * ty + i) * (kKT + 4) + 4 * tx + j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xFFFFFFFFu, rs, off);
      l[i] = l[i] * alpha + rs;
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < CW; ++c) o[i][c] *= alpha;
    }
    __syncthreads();
    // o += p . v
#pragma unroll 4
    for (int j = 0; j < kKT; ++j) {
      float vv[CW];
      if constexpr (CW % 4 == 0) {  // 16-byte aligned: tx * CW * 4 bytes
#pragma unroll
        for (int c = 0; c < CW; c += 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(Vs + j * HD + tx * CW + c);
          vv[c] = t4.x;
          vv[c + 1] = t4.y;
          vv[c + 2] = t4.z;
          vv[c + 3] = t4.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < CW; ++c) vv[c] = Vs[j * HD + tx * CW + c];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float p = Ps[(4 * ty + i) * (kKT + 4) + j];
#pragma unroll
        for (int c = 0; c < CW; ++c) o[i][c] = fmaf(p, vv[c], o[i][c]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = 4 * ty + i;
    if (qi < nq) {
      float* orow = out + ((int64_t)b * pr.cnt + q0 + qi) * ld_out + hq * HD + tx * CW;
      const float inv = 1.0f / l[i];
#pragma unroll
      for (int c = 0; c < CW; ++c) orow[c] = o[i][c] * inv;
    }
  }
}

}  // namespace

int prefill_embed(const uint16_t* emb, const int* prompt, const PrefillRows& pr, int d, int vocab, float* hidden,
                  cudaStream_t st) {
  const int64_t rows = (int64_t)pr.batch * pr.cnt;
  AH_REQUIRE(rows <= 65535 * 16, "prefill: too many rows per chunk");
  k_embed_rows<<<dim3((d + 255) / 256 < 8 ? (d + 255) / 256 : 8, (unsigned)rows), 256, 0, st>>>(emb, prompt, pr, d,
                                                                                               vocab, hidden);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int prefill_rmsnorm(const float* x, const uint16_t* w, float eps, int64_t rows, int d, float* out, cudaStream_t st) {
  k_rmsnorm_rows<<<(unsigned)rows, 256, 0, st>>>(x, w, eps, d, out);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int prefill_rope_append(float* qkv, int ld, const float2* rope, uint16_t* kc, uint16_t* vc, int layer, int n_layer,
                        int nh, int nkv, int hd, int max_seq, const PrefillRows& pr, cudaStream_t st) {
  k_rope_append_rows<<<(unsigned)((int64_t)pr.batch * pr.cnt), 128, 0, st>>>(qkv, ld, rope, kc, vc, layer, n_layer,
                                                                              nh, nkv, hd, max_seq, pr);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

template <int HD>
int launch_attn(const float* qkv, int ld, const uint16_t* kc, const uint16_t* vc, int layer, int n_layer, int nh,
                int nkv, int max_seq, float scale, const PrefillRows& pr, float* out, int ld_out, cudaStream_t st) {
  auto kern = k_prefill_attn<HD>;
  static bool configured[64] = {};
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    AH_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PfSmem<HD>::kBytes));
    configured[dev] = true;
  }
  const dim3 grid((unsigned)((pr.cnt + kQT - 1) / kQT), (unsigned)nh, (unsigned)pr.batch);
  kern<<<grid, 256, PfSmem<HD>::kBytes, st>>>(qkv, ld, kc, vc, layer, n_layer, nh, nkv, max_seq, scale, pr, out,
                                              ld_out);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int prefill_attention(const float* qkv, int ld, const uint16_t* kc, const uint16_t* vc, int layer, int n_layer,
                      int nh, int nkv, int hd, int max_seq, float scale, const PrefillRows& pr, float* out,
                      int ld_out, cudaStream_t st) {
  switch (hd) {
    case 32: return launch_attn<32>(qkv, ld, kc, vc, layer, n_layer, nh, nkv, max_seq, scale, pr, out, ld_out, st);
    case 64: return launch_attn<64>(qkv, ld, kc, vc, layer, n_layer, nh, nkv, max_seq, scale, pr, out, ld_out, st);
    case 96: return launch_attn<96>(qkv, ld, kc, vc, layer, n_layer, nh, nkv, max_seq, scale, pr, out, ld_out, st);
    case 128: return launch_attn<128>(qkv, ld, kc, vc, layer, n_layer, nh, nkv, max_seq, scale, pr, out, ld_out, st);
    default: return fail(AH_EUNSUPPORTED, "prefill attention: head_dim %d", hd);
  }
}

int prefill_add(float* hidden, const float* part, int64_t n, cudaStream_t st) {
  const int64_t g = std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
  k_add_rows<<<(unsigned)g, 256, 0, st>>>(hidden, part, n);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int prefill_swiglu(const float* gu, int64_t rows, int nff, float* act, cudaStream_t st) {
  const int64_t n = rows * nff;
  const int64_t g = std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
  k_swiglu_rows<<<(unsigned)g, 256, 0, st>>>(gu, rows, nff, act);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

}  // namespace ah
