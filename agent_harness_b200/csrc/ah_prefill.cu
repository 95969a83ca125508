// ah_prefill.cu — row kernels of the decoder's prompt prefill.  The prompt is
// processed in chunks of positions; for each chunk and layer the projections
// run as tcgen05 GEMMs (ah_gemm_tc.cu) and these kernels do the rest: rows are
// (sequence, position) pairs, row r = b * cnt + i for position p0 + i.
#include <algorithm>
#include <cmath>

#include <mutex>

#include "ah_gemv.cuh"
#include "ah_prefill.cuh"
#include "ah_sm100.cuh"

namespace ah {
namespace {

__global__ void __launch_bounds__(256) k_embed_rows(const uint16_t* __restrict__ emb, const int* __restrict__ prompt,
                                                    PrefillRows pr, int d, int vocab, float* __restrict__ hidden) {
  const int64_t r = blockIdx.y;
  const int b = (int)(r / pr.cnt), i = (int)(r - (int64_t)b * pr.cnt);
  const int t = prompt[(size_t)b * pr.n_prompt + pr.p0 + i];
  const int tv = (t >= 0 && t < vocab) ? t : 0;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < d; c += gridDim.x * blockDim.x)
    hidden[r * d + c] = f16_bits_to_f32(emb[(size_t)tv * d + c]);
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


// ---- causal attention on the tensor cores (head_dim 64 / 128) ---------------------
// The same attention as k_prefill_attn on mma.sync m16n8k16: CTA (t, hq, b)
// takes queries p0 + 64t .. +63 of head hq, four warps of 16 query rows each,
// and walks the cache rows 0 .. its last query in tiles of 64 keys.  K / V
// tiles (f16, as cached) arrive by cp.async into two buffers (the next tile
// loads while this one is used) in 128-byte rows with a 16-byte-chunk XOR
// swizzle, so the fragment loads are conflict-free.  S = Q K^T with q split
// into f16 hi + lo (per row scaled by a power of two into [2^14, 2^15)), an
// online softmax per row in registers, then O += P V with P split into hi +
// lo as well: against the f16 cache the products keep f32 accuracy, as in
// the decode attention.  P is the S accumulator itself (its C fragment
// layout is the A fragment layout of the next MMA).
constexpr int kTcQ = 64;  // queries per CTA (4 warps x 16 rows)
constexpr int kTcK = 64;  // keys per tile
constexpr int kTcThreads = 128;

template <int HD>
struct PfTcSmem {
  static constexpr int kHalves = HD / 64;                   // 128-byte column halves per row
  static constexpr int kHalfBytes = kTcK * 128;             // one half of a K or V tile
  static constexpr int kTile = 2 * kHalves * kHalfBytes;    // K then V
  static constexpr size_t kBytes = 2 * (size_t)kTile;       // two tile buffers
};

__device__ __forceinline__ uint32_t pf_swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }
__device__ __forceinline__ void pf_cp_async16(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
__device__ __forceinline__ void pf_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pf_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint32_t pf_pack(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// x = hi + lo with hi, lo f16 (lo holds the rounding error of hi)
__device__ __forceinline__ void pf_split(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  hi = pf_pack(h0, h1);
  lo = pf_pack(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1)));
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads) k_prefill_attn_tc(const float* __restrict__ qkv, int ld,
                                                                const uint16_t* __restrict__ kc,
                                                                const uint16_t* __restrict__ vc, int layer,
                                                                int n_layer, int nh, int nkv, int max_seq, float scale,
                                                                PrefillRows pr, float* __restrict__ out, int ld_out) {
  using S = PfTcSmem<HD>;
  constexpr int KS = HD / 16;  // 16-wide k-steps over the head dims (S = Q K^T)
  constexpr int NT = HD / 8;   // n8 tiles over the head dims (O)
  constexpr int CH = HD / 8;   // 16-byte chunks per K / V row
  extern __shared__ __align__(128) uint8_t smx[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int q0 = blockIdx.x * kTcQ;
  const int nq = min(kTcQ, pr.cnt - q0);
  const int G = nh / nkv, hk = hq / G;
  const int qpos_last = pr.p0 + q0 + nq - 1;  // causal limit of the CTA
  const size_t head_off = (((size_t)b * n_layer + layer) * nkv + hk) * (size_t)max_seq * HD;
  const uint16_t* kh = kc + head_off;
  const uint16_t* vh = vc + head_off;
  const int n_kt = qpos_last / kTcK + 1;

  // tile kt into buffer buf: rows past the causal limit are zero (finite P . V)
  auto load_tile = [&](int kt, int buf) {
    uint8_t* base = smx + (size_t)buf * S::kTile;
    const int k0 = kt * kTcK;
    for (int i = tid; i < kTcK * CH; i += kTcThreads) {
      const int r = i / CH, c = i - r * CH;
      const uint32_t off = (uint32_t)(c >> 3) * S::kHalfBytes + pf_swz(r, c & 7);
      uint8_t* dk = base + off;
      uint8_t* dv = base + S::kHalves * S::kHalfBytes + off;
      if (k0 + r <= qpos_last) {
        pf_cp_async16(dk, kh + (size_t)(k0 + r) * HD + c * 8);
        pf_cp_async16(dv, vh + (size_t)(k0 + r) * HD + c * 8);
      } else {
        *reinterpret_cast<uint4*>(dk) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(dv) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    pf_cp_commit();
  };
  load_tile(0, 0);

  // this warp's query rows r0 = 16 warp + g and r1 = r0 + 8 as A fragments
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  const bool l0 = r0 < nq, l1 = r1 < nq;
  const float* qrow0 = qkv + ((int64_t)b * pr.cnt + q0 + (l0 ? r0 : 0)) * ld + hq * HD;
  const float* qrow1 = qkv + ((int64_t)b * pr.cnt + q0 + (l1 ? r1 : 0)) * ld + hq * HD;
  float2 qa[KS][2], qb[KS][2];
  float ma = 0.0f, mb = 0.0f;
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int d = kk * 16 + hh * 8 + 2 * t;
      qa[kk][hh] = l0 ? *reinterpret_cast<const float2*>(qrow0 + d) : make_float2(0.0f, 0.0f);
      qb[kk][hh] = l1 ? *reinterpret_cast<const float2*>(qrow1 + d) : make_float2(0.0f, 0.0f);
      ma = fmaxf(ma, fmaxf(fabsf(qa[kk][hh].x), fabsf(qa[kk][hh].y)));
      mb = fmaxf(mb, fmaxf(fabsf(qb[kk][hh].x), fabsf(qb[kk][hh].y)));
    }
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {  // the four threads of a row
    ma = fmaxf(ma, __shfl_xor_sync(0xFFFFFFFFu, ma, o));
    mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
  }
  auto pow2_scale = [](float m) {
    int ex = 0;
    if (m > 0.0f) frexpf(m, &ex);
    return ldexpf(1.0f, m > 0.0f ? min(15 - ex, 100) : 0);
  };
  const float sa = pow2_scale(ma), sb = pow2_scale(mb);
  uint32_t qh[KS][4], ql[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    pf_split(qa[kk][0].x * sa, qa[kk][0].y * sa, qh[kk][0], ql[kk][0]);  // row g, dims 2t
    pf_split(qb[kk][0].x * sb, qb[kk][0].y * sb, qh[kk][1], ql[kk][1]);  // row g + 8
    pf_split(qa[kk][1].x * sa, qa[kk][1].y * sa, qh[kk][2], ql[kk][2]);  // row g, dims 8 + 2t
    pf_split(qb[kk][1].x * sb, qb[kk][1].y * sb, qh[kk][3], ql[kk][3]);
  }
  const float mult0 = scale / sa, mult1 = scale / sb;
  const int qp0 = pr.p0 + q0 + r0, qp1 = pr.p0 + q0 + r1;
  const int warp_qlast = pr.p0 + q0 + warp * 16 + 15;

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, s0 = 0.0f, s1 = 0.0f;
  for (int kt = 0; kt < n_kt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kt) {
      load_tile(kt + 1, buf ^ 1);
      pf_cp_wait<1>();  // tile kt has landed (tile kt + 1 may be in flight)
    } else {
      pf_cp_wait<0>();
    }
    __syncthreads();
    const int k0 = kt * kTcK;
    if (k0 <= warp_qlast) {  // warp-uniform: a tile wholly past this warp's queries is skipped
      const uint8_t* base = smx + (size_t)buf * S::kTile;
      const uint32_t kb = smem_u32(base), vb = smem_u32(base + S::kHalves * S::kHalfBytes);
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // keys k0 + 8j .. +7
        sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
        for (int k2 = 0; k2 < HD / 32; ++k2) {
          const int d0 = k2 * 32 + (lane >> 3) * 8;  // matrix lane/8: dims d0 .. d0 + 7
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + (uint32_t)(d0 >> 6) * S::kHalfBytes + pf_swz(8 * j + (lane & 7), (d0 & 63) >> 3), b0, b1, b2, b3);
          mma16816(sc[j], qh[2 * k2][0], qh[2 * k2][1], qh[2 * k2][2], qh[2 * k2][3], b0, b1, sc[j]);
          mma16816(sc[j], ql[2 * k2][0], ql[2 * k2][1], ql[2 * k2][2], ql[2 * k2][3], b0, b1, sc[j]);
          mma16816(sc[j], qh[2 * k2 + 1][0], qh[2 * k2 + 1][1], qh[2 * k2 + 1][2], qh[2 * k2 + 1][3], b2, b3, sc[j]);
          mma16816(sc[j], ql[2 * k2 + 1][0], ql[2 * k2 + 1][1], ql[2 * k2 + 1][2], ql[2 * k2 + 1][3], b2, b3, sc[j]);
        }
      }
      // causal mask and the online softmax of rows r0 (c0, c1) and r1 (c2, c3)
      float x0 = -INFINITY, x1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = k0 + 8 * j + 2 * t + e;
          sc[j][e] = key <= qp0 ? sc[j][e] * mult0 : -INFINITY;
          sc[j][2 + e] = key <= qp1 ? sc[j][2 + e] * mult1 : -INFINITY;
          x0 = fmaxf(x0, sc[j][e]);
          x1 = fmaxf(x1, sc[j][2 + e]);
        }
#pragma unroll
      for (int o2 = 1; o2 <= 2; o2 <<= 1) {
        x0 = fmaxf(x0, __shfl_xor_sync(0xFFFFFFFFu, x0, o2));
        x1 = fmaxf(x1, __shfl_xor_sync(0xFFFFFFFFu, x1, o2));
      }
      const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
      const float al0 = n0 == -INFINITY ? 1.0f : expf(m0 - n0), al1 = n1 == -INFINITY ? 1.0f : expf(m1 - n1);
      float r0s = 0.0f, r1s = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p0v = n0 == -INFINITY ? 0.0f : expf(sc[j][e] - n0);
          const float p1v = n1 == -INFINITY ? 0.0f : expf(sc[j][2 + e] - n1);
          sc[j][e] = p0v;
          sc[j][2 + e] = p1v;
          r0s += p0v;
          r1s += p1v;
        }
#pragma unroll
      for (int o2 = 1; o2 <= 2; o2 <<= 1) {
        r0s += __shfl_xor_sync(0xFFFFFFFFu, r0s, o2);
        r1s += __shfl_xor_sync(0xFFFFFFFFu, r1s, o2);
      }
      s0 = s0 * al0 + r0s;
      s1 = s1 * al1 + r1s;
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        o[n][0] *= al0;
        o[n][1] *= al0;
        o[n][2] *= al1;
        o[n][3] *= al1;
      }
      // O += P V over the tile's four 16-key steps
      const int mi = lane >> 3;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t ph[4], pl[4];
        pf_split(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);          // row g, keys 16kk + 2t
        pf_split(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);          // row g + 8
        pf_split(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);  // row g, keys 16kk + 8 + 2t
        pf_split(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
        const int key = 16 * kk + ((mi & 1) << 3) + (lane & 7);
#pragma unroll
        for (int n2 = 0; n2 < HD / 16; ++n2) {
          const int d0 = n2 * 16 + ((mi >> 1) << 3);
          uint32_t v0, v1, v2, v3;
          ldsm_x4_trans(vb + (uint32_t)(d0 >> 6) * S::kHalfBytes + pf_swz(key, (d0 & 63) >> 3), v0, v1, v2, v3);
          mma16816(o[2 * n2], ph[0], ph[1], ph[2], ph[3], v0, v1, o[2 * n2]);
          mma16816(o[2 * n2], pl[0], pl[1], pl[2], pl[3], v0, v1, o[2 * n2]);
          mma16816(o[2 * n2 + 1], ph[0], ph[1], ph[2], ph[3], v2, v3, o[2 * n2 + 1]);
          mma16816(o[2 * n2 + 1], pl[0], pl[1], pl[2], pl[3], v2, v3, o[2 * n2 + 1]);
        }
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
  const float inv0 = 1.0f / s0, inv1 = 1.0f / s1;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int d = hq * HD + n * 8 + 2 * t;
    if (l0)
      *reinterpret_cast<float2*>(out + ((int64_t)b * pr.cnt + q0 + r0) * ld_out + d) =
          make_float2(o[n][0] * inv0, o[n][1] * inv0);
    if (l1)
      *reinterpret_cast<float2*>(out + ((int64_t)b * pr.cnt + q0 + r1) * ld_out + d) =
          make_float2(o[n][2] * inv1, o[n][3] * inv1);
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

int prefill_rope_append(float* qkv, int ld, const float2* rope, uint16_t* kc, uint16_t* vc, int layer, int n_layer,
                        int nh, int nkv, int hd, int max_seq, const PrefillRows& pr, cudaStream_t st) {
  k_rope_append_rows<<<(unsigned)((int64_t)pr.batch * pr.cnt), 128, 0, st>>>(qkv, ld, rope, kc, vc, layer, n_layer,
                                                                              nh, nkv, hd, max_seq, pr);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

template <int HD>
int launch_attn_tc(const float* qkv, int ld, const uint16_t* kc, const uint16_t* vc, int layer, int n_layer, int nh,
                   int nkv, int max_seq, float scale, const PrefillRows& pr, float* out, int ld_out,
                   cudaStream_t st) {
  auto kern = k_prefill_attn_tc<HD>;
  constexpr int kMaxDevices = 64;
  static std::once_flag once[kMaxDevices];
  static cudaError_t set_rc[kMaxDevices];
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  AH_REQUIRE(dev >= 0 && dev < kMaxDevices, "prefill attention: device %d out of range", dev);
  std::call_once(once[dev], [&] {
    set_rc[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PfTcSmem<HD>::kBytes);
  });
  if (set_rc[dev] != cudaSuccess)
    return fail(AH_ECUDA, "prefill attention: cudaFuncSetAttribute: %s", cudaGetErrorString(set_rc[dev]));
  AH_REQUIRE((ld % 2) == 0 && (ld_out % 2) == 0, "prefill attention: odd row strides");
  const dim3 grid((unsigned)((pr.cnt + kTcQ - 1) / kTcQ), (unsigned)nh, (unsigned)pr.batch);
  kern<<<grid, kTcThreads, PfTcSmem<HD>::kBytes, st>>>(qkv, ld, kc, vc, layer, n_layer, nh, nkv, max_seq, scale, pr,
                                                        out, ld_out);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

template <int HD>
int launch_attn(const float* qkv, int ld, const uint16_t* kc, const uint16_t* vc, int layer, int n_layer, int nh,
                int nkv, int max_seq, float scale, const PrefillRows& pr, float* out, int ld_out, cudaStream_t st) {
  if constexpr (HD == 64 || HD == 128)
    return launch_attn_tc<HD>(qkv, ld, kc, vc, layer, n_layer, nh, nkv, max_seq, scale, pr, out, ld_out, st);
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


}  // namespace ah
