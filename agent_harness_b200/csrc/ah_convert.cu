// ah_convert.cu — f16/bf16 <-> f32 conversion and block dequantisation
// (Q8_0, Q4_0, the engine's INT4 SoA format) for sm_100a.
//
// All of these are HBM-streaming kernels: 128-bit loads and streaming 128-bit
// stores, grids sized to a multiple of the SM count.  The AoS block formats
// (34-byte Q8_0, 18-byte Q4_0 blocks are not 16-byte aligned) are staged tile
// by tile into shared memory with bulk (TMA) copies on an mbarrier ring, so the
// global reads stay fully coalesced and overlap with the unpacking of the
// previous tile.  Results are bit-exact against the reference's scalar
// semantics, NaN bit patterns included (see x86_mul in ah_common.cuh).
#include "ah_common.cuh"
#include "ah_sm100.cuh"

namespace ah {
namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t work_items, int per_sm = 8) {
  int64_t g = (work_items + kThreads - 1) / kThreads;
  int64_t cap = (int64_t)sm_count() * per_sm;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

// ---------------------------------------------------------------------------
// f16 / bf16 -> f32
// ---------------------------------------------------------------------------
template <bool kBf16>
__device__ __forceinline__ float half_bits_to_f32(uint32_t h) {
  if (kBf16) return __uint_as_float(h << 16);  // formats/gguf.rs:124-126
  return f16_bits_to_f32(h);                   // formats/gguf.rs:93-120
}

template <bool kBf16>
__device__ __forceinline__ void cvt8(const uint4& v, float4* dst) {
  float4 a, b;
  a.x = half_bits_to_f32<kBf16>(v.x & 0xFFFFu); a.y = half_bits_to_f32<kBf16>(v.x >> 16);
  a.z = half_bits_to_f32<kBf16>(v.y & 0xFFFFu); a.w = half_bits_to_f32<kBf16>(v.y >> 16);
  b.x = half_bits_to_f32<kBf16>(v.z & 0xFFFFu); b.y = half_bits_to_f32<kBf16>(v.z >> 16);
  b.z = half_bits_to_f32<kBf16>(v.w & 0xFFFFu); b.w = half_bits_to_f32<kBf16>(v.w >> 16);
  st_cs_f4(dst, a);
  st_cs_f4(dst + 1, b);
}

// 8 halves per 16-byte load; four loads in flight per thread.
template <bool kBf16>
__global__ void __launch_bounds__(kThreads) k_half_to_f32_vec(const uint4* __restrict__ src, float4* __restrict__ dst,
                                                              int64_t n8) {
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (U - 1) * stride < n8; i += U * stride) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < U; ++u) cvt8<kBf16>(v[u], dst + 2 * (i + u * stride));
  }
  for (; i < n8; i += stride) cvt8<kBf16>(__ldcs(src + i), dst + 2 * i);
}

// Byte-addressed fallback (any alignment) and tail.
template <bool kBf16>
__global__ void __launch_bounds__(kThreads) k_half_to_f32_scalar(const uint8_t* __restrict__ src,
                                                                 float* __restrict__ dst, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t h = (uint32_t)src[2 * i] | ((uint32_t)src[2 * i + 1] << 8);
    dst[i] = half_bits_to_f32<kBf16>(h);
  }
}

template <class F>
int launch_dequant_blocks(const void* blocks, float* out, int64_t n, cudaStream_t st);
template <bool kBf16>
struct HalfFmt;

// The bulk-copy ring for 16-byte aligned buffers of at least one tile; the
// register-batched kernel and the byte-addressed one cover the rest.
template <bool kBf16>
int launch_half_to_f32(const void* src, float* dst, int64_t n, cudaStream_t st) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(src && dst && n > 0, "half_to_f32: null pointer or negative n");
  if (aligned16(src) && aligned16(dst) && n >= (int64_t)HalfFmt<kBf16>::kTileBlocks * 32)
    return launch_dequant_blocks<HalfFmt<kBf16>>(src, dst, n, st);
  int64_t done = 0;
  if (aligned16(src) && aligned16(dst)) {
    int64_t n8 = n / 8;
    if (n8 > 0) {
      k_half_to_f32_vec<kBf16><<<grid_for(n8), kThreads, 0, st>>>(static_cast<const uint4*>(src),
                                                                   reinterpret_cast<float4*>(dst), n8);
      AH_LAUNCH_CHECK();
    }
    done = n8 * 8;
  }
  if (done < n) {
    k_half_to_f32_scalar<kBf16><<<grid_for(n - done), kThreads, 0, st>>>(
        static_cast<const uint8_t*>(src) + 2 * done, dst + done, n - done);
    AH_LAUNCH_CHECK();
  }
  return AH_OK;
}

// ---------------------------------------------------------------------------
// f32 -> f16 (IEEE RNE; NaN -> sign | 0x7E00 | top payload bits)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f32_to_f16_bits(float f) {
  uint32_t x = __float_as_uint(f);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return ((x >> 16) & 0x8000u) | 0x7E00u | ((x >> 13) & 0x3FFu);
  return __half_as_ushort(__float2half_rn(f));
}

__global__ void __launch_bounds__(kThreads) k_f32_to_f16_vec(const float4* __restrict__ src, uint2* __restrict__ dst,
                                                             int64_t n4) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = __ldcs(src + i);
    uint2 o;
    o.x = f32_to_f16_bits(v.x) | (f32_to_f16_bits(v.y) << 16);
    o.y = f32_to_f16_bits(v.z) | (f32_to_f16_bits(v.w) << 16);
    dst[i] = o;
  }
}

__global__ void __launch_bounds__(kThreads) k_f32_to_f16_scalar(const float* __restrict__ src,
                                                                uint16_t* __restrict__ dst, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = (uint16_t)f32_to_f16_bits(src[i]);
}

// ---------------------------------------------------------------------------
// AoS block dequantisation with bulk-copy staging
// ---------------------------------------------------------------------------
constexpr int kStages = 4;

struct Q8Fmt {  // formats/gguf.rs:460-479, types/dtype.rs:77-83
  static constexpr int kBlockBytes = 34;
  static constexpr int kTileBlocks = 128;  // 4352 B in (16-byte multiple), 16 KB out
  // float4 `f` of a tile: 4 consecutive elements of block f/8.
  static __device__ __forceinline__ float4 unpack(const uint8_t* tile, int f) {
    const uint8_t* bp = tile + (f >> 3) * kBlockBytes;
    const int e0 = (f & 7) * 4;
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(bp));
    const uint32_t q01 = *reinterpret_cast<const uint16_t*>(bp + 2 + e0);
    const uint32_t q23 = *reinterpret_cast<const uint16_t*>(bp + 4 + e0);
    float4 v;
    v.x = x86_mul(d, (float)(int8_t)(q01 & 0xFFu));
    v.y = x86_mul(d, (float)(int8_t)(q01 >> 8));
    v.z = x86_mul(d, (float)(int8_t)(q23 & 0xFFu));
    v.w = x86_mul(d, (float)(int8_t)(q23 >> 8));
    return v;
  }
  static __device__ __forceinline__ float element(const uint8_t* blocks, int64_t e) {
    const uint8_t* bp = blocks + (e >> 5) * kBlockBytes;
    const uint32_t dbits = (uint32_t)bp[0] | ((uint32_t)bp[1] << 8);
    return x86_mul(f16_bits_to_f32(dbits), (float)(int8_t)bp[2 + (e & 31)]);
  }
};

struct Q4Fmt {  // formats/gguf.rs:480-502, types/dtype.rs:69-75
  static constexpr int kBlockBytes = 18;
  static constexpr int kTileBlocks = 256;  // 4608 B in, 32 KB out
  static __device__ __forceinline__ float4 unpack(const uint8_t* tile, int f) {
    const uint8_t* bp = tile + (f >> 3) * kBlockBytes;
    const int e0 = (f & 7) * 4;
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(bp));
    const uint32_t b = *reinterpret_cast<const uint16_t*>(bp + 2 + (e0 >> 1));
    float4 v;  // byte i: low nibble = element 2i, high nibble = element 2i+1
    v.x = x86_mul(d, (float)(int)(b & 0xFu) - 8.0f);
    v.y = x86_mul(d, (float)(int)((b >> 4) & 0xFu) - 8.0f);
    v.z = x86_mul(d, (float)(int)((b >> 8) & 0xFu) - 8.0f);
    v.w = x86_mul(d, (float)(int)((b >> 12) & 0xFu) - 8.0f);
    return v;
  }
  static __device__ __forceinline__ float element(const uint8_t* blocks, int64_t e) {
    const uint8_t* bp = blocks + (e >> 5) * kBlockBytes;
    const uint32_t dbits = (uint32_t)bp[0] | ((uint32_t)bp[1] << 8);
    const int i = (int)(e & 31);
    const uint32_t byte = bp[2 + (i >> 1)];
    const uint32_t nib = (i & 1) ? (byte >> 4) : (byte & 0xFu);
    return x86_mul(f16_bits_to_f32(dbits), (float)(int)nib - 8.0f);
  }
};

// f16 / bf16 as a "block" format of 32 halves (64 bytes): the conversion then
// streams through the same bulk-copy ring as the quantised blocks.
template <bool kBf16>
struct HalfFmt {
  static constexpr int kBlockBytes = 64;
  static constexpr int kTileBlocks = 128;  // 8 KB in, 16 KB out
  static __device__ __forceinline__ float4 unpack(const uint8_t* tile, int f) {
    const uint2 h = *reinterpret_cast<const uint2*>(tile + f * 8);
    float4 v;
    v.x = half_bits_to_f32<kBf16>(h.x & 0xFFFFu);
    v.y = half_bits_to_f32<kBf16>(h.x >> 16);
    v.z = half_bits_to_f32<kBf16>(h.y & 0xFFFFu);
    v.w = half_bits_to_f32<kBf16>(h.y >> 16);
    return v;
  }
  static __device__ __forceinline__ float element(const uint8_t* src, int64_t e) {
    return half_bits_to_f32<kBf16>((uint32_t)src[2 * e] | ((uint32_t)src[2 * e + 1] << 8));
  }
};

// The engine's SoA format (quantization.rs:365-404, group 32): "blocks" of
// 16 nibble bytes, with the group's f32 scale in a second array staged beside
// them (kAuxBytes per block).
struct EngineFmt {
  static constexpr int kBlockBytes = 16;
  static constexpr int kAuxBytes = 4;
  static constexpr int kTileBlocks = 256;  // 4 KB nibbles + 1 KB scales in, 32 KB out
  static __device__ __forceinline__ float4 unpack(const uint8_t* tile, const uint8_t* aux, int f) {
    const float s = reinterpret_cast<const float*>(aux)[f >> 3];
    const uint32_t b = *reinterpret_cast<const uint16_t*>(tile + (f >> 3) * 16 + (f & 7) * 2);
    float4 v;  // element 2i in the low nibble of byte i (quantization.rs:444-452)
    v.x = x86_mul(s, (float)(int)(b & 0xFu) - 8.0f);
    v.y = x86_mul(s, (float)(int)((b >> 4) & 0xFu) - 8.0f);
    v.z = x86_mul(s, (float)(int)((b >> 8) & 0xFu) - 8.0f);
    v.w = x86_mul(s, (float)(int)((b >> 12) & 0xFu) - 8.0f);
    return v;
  }
};

template <class F, class = void>
struct AuxOf {
  static constexpr int kBytes = 0;
};
template <class F>
struct AuxOf<F, decltype((void)F::kAuxBytes)> {
  static constexpr int kBytes = F::kAuxBytes;
};

// Persistent CTAs walk whole tiles t = blockIdx.x + k*gridDim.x.  Thread 0
// keeps kStages bulk copies in flight; every thread unpacks the tile in shared
// memory and streams its float4s out.
template <class F>
__global__ void __launch_bounds__(kThreads) k_dequant_blocks_tma(const uint8_t* __restrict__ blocks,
                                                                 float* __restrict__ out, int64_t n_tiles,
                                                                 int* __restrict__ err,
                                                                 const void* __restrict__ aux_src = nullptr) {
  constexpr int kTileBytes = F::kTileBlocks * F::kBlockBytes;
  constexpr int kAuxTile = F::kTileBlocks * AuxOf<F>::kBytes;  // second source per tile (0: none)
  constexpr int kF4PerTile = F::kTileBlocks * 8;
  static_assert(kTileBytes % 16 == 0 && kAuxTile % 16 == 0, "bulk copies move 16-byte multiples");
  __shared__ __align__(128) uint8_t buf[kStages][kTileBytes];
  __shared__ __align__(128) uint8_t aux[kStages][kAuxTile > 0 ? kAuxTile : 16];
  __shared__ __align__(8) uint64_t full[kStages];
  const uint8_t* auxg = static_cast<const uint8_t*>(aux_src);
  const int tid = threadIdx.x;
  const int64_t my_tiles =
      n_tiles > (int64_t)blockIdx.x ? (n_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int64_t issued = 0;
  if (tid == 0) {
    for (; issued < kStages && issued < my_tiles; ++issued) {
      const int64_t t = blockIdx.x + issued * gridDim.x;
      mbar_arrive_expect_tx(&full[issued], kTileBytes + kAuxTile);
      bulk_g2s(buf[issued], blocks + t * kTileBytes, kTileBytes, &full[issued]);
      if (kAuxTile > 0) bulk_g2s(aux[issued], auxg + t * kAuxTile, kAuxTile, &full[issued]);
    }
  }
  int64_t k = 0;
  for (; k < my_tiles; ++k) {
    const int s = (int)(k % kStages);
    const uint32_t parity = (uint32_t)((k / kStages) & 1);
    const bool ok = mbar_wait_bounded(&full[s], parity, err, 0x101);
    if (__syncthreads_or(!ok)) break;
    const int64_t t = blockIdx.x + k * gridDim.x;
    float4* o = reinterpret_cast<float4*>(out + t * (int64_t)F::kTileBlocks * 32);
#pragma unroll
    for (int j = 0; j < kF4PerTile / kThreads; ++j) {
      const int f = tid + j * kThreads;
      if constexpr (kAuxTile > 0)
        st_cs_f4(o + f, F::unpack(buf[s], aux[s], f));
      else
        st_cs_f4(o + f, F::unpack(buf[s], f));
    }
    __syncthreads();  // stage s fully consumed
    if (tid == 0 && issued < my_tiles) {
      const int64_t tn = blockIdx.x + issued * gridDim.x;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&full[s], kTileBytes + kAuxTile);
      bulk_g2s(buf[s], blocks + tn * kTileBytes, kTileBytes, &full[s]);
      if (kAuxTile > 0) bulk_g2s(aux[s], auxg + tn * kAuxTile, kAuxTile, &full[s]);
      ++issued;
    }
  }
  // A wait gave up: drain the copies still in flight (bounded) before exiting.
  if (k < my_tiles && tid == 0) {
    for (int64_t j = k; j < issued; ++j)
      mbar_wait_bounded(&full[j % kStages], (uint32_t)((j / kStages) & 1), err, 0x102);
  }
}

// Element-wise path: tails, misaligned pointers, and partial last blocks.
template <class F>
__global__ void __launch_bounds__(kThreads) k_dequant_blocks_scalar(const uint8_t* __restrict__ blocks,
                                                                    float* __restrict__ out, int64_t e_begin,
                                                                    int64_t e_end) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = e_begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < e_end; e += stride)
    out[e] = F::element(blocks, e);
}

template <class F>
int launch_dequant_blocks(const void* blocks, float* out, int64_t n, cudaStream_t st) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(blocks && out && n > 0, "dequant: null pointer or negative n");
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  int64_t done = 0;
  if (aligned16(b) && aligned16(out)) {
    const int64_t n_tiles = n / ((int64_t)F::kTileBlocks * 32);
    if (n_tiles > 0) {
      int64_t g = (int64_t)sm_count() * 4;
      if (g > n_tiles) g = n_tiles;
      int* err = device_error_word();
      AH_REQUIRE(err != nullptr, "dequant: device error word unavailable");
      k_dequant_blocks_tma<F><<<(int)g, kThreads, 0, st>>>(b, out, n_tiles, err);
      AH_LAUNCH_CHECK();
    }
    done = n_tiles * F::kTileBlocks * 32;
  }
  if (done < n) {
    k_dequant_blocks_scalar<F><<<grid_for(n - done), kThreads, 0, st>>>(b, out, done, n);
    AH_LAUNCH_CHECK();
  }
  return AH_OK;
}

// ---------------------------------------------------------------------------
// Engine INT4 format: f32 scales per group + linear nibbles
// (models/quantization.rs:444-452: out[i] = (nib(i) - 8) * scales[i / gs]).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_dequant_engine_gs32(const float* __restrict__ scales,
                                                                  const uint32_t* __restrict__ packed,
                                                                  float4* __restrict__ out, int64_t n8) {
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i < n8; i += U * stride) {
    uint32_t w[U];
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = i + u * stride;
      if (j < n8) { w[u] = __ldcs(packed + j); s[u] = __ldg(scales + (j >> 2)); }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = i + u * stride;
      if (j < n8) {
        float4 a, b;
        a.x = x86_mul(s[u], (float)(int)(w[u] & 0xFu) - 8.0f);
        a.y = x86_mul(s[u], (float)(int)((w[u] >> 4) & 0xFu) - 8.0f);
        a.z = x86_mul(s[u], (float)(int)((w[u] >> 8) & 0xFu) - 8.0f);
        a.w = x86_mul(s[u], (float)(int)((w[u] >> 12) & 0xFu) - 8.0f);
        b.x = x86_mul(s[u], (float)(int)((w[u] >> 16) & 0xFu) - 8.0f);
        b.y = x86_mul(s[u], (float)(int)((w[u] >> 20) & 0xFu) - 8.0f);
        b.z = x86_mul(s[u], (float)(int)((w[u] >> 24) & 0xFu) - 8.0f);
        b.w = x86_mul(s[u], (float)(int)(w[u] >> 28) - 8.0f);
        st_cs_f4(out + 2 * j, a);
        st_cs_f4(out + 2 * j + 1, b);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_dequant_engine_any(const float* __restrict__ scales,
                                                                 const uint8_t* __restrict__ packed,
                                                                 float* __restrict__ out, int64_t e_begin,
                                                                 int64_t n, int64_t gs) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = e_begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint32_t byte = packed[i >> 1];
    const uint32_t nib = (i & 1) ? (byte >> 4) & 0xFu : byte & 0xFu;
    out[i] = x86_mul(scales[i / gs], (float)(int)nib - 8.0f);
  }
}

// Q6_K "approximate, for stats" branch (formats/gguf.rs:503-529):
// out = ((i8)raw[off + 6 + i%128]) * d / 127.
__global__ void __launch_bounds__(kThreads) k_dequant_q6k_approx(const uint8_t* __restrict__ raw,
                                                                 float* __restrict__ out, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
    const int64_t b = e >> 8;
    const int i = (int)(e & 255);
    const uint8_t* bp = raw + b * 210;
    const float d = f16_bits_to_f32((uint32_t)bp[0] | ((uint32_t)bp[1] << 8));
    float p = x86_mul(d, (float)(int8_t)bp[6 + (i & 127)]);
    out[e] = (p != p) ? p : __fdiv_rn(p, 127.0f);
  }
}

}  // namespace
}  // namespace ah

using namespace ah;

extern "C" {

int ah_f16_to_f32(const uint16_t* src, float* dst, int64_t n, void* stream) {
  return launch_half_to_f32<false>(src, dst, n, as_stream(stream));
}

int ah_bf16_to_f32(const uint16_t* src, float* dst, int64_t n, void* stream) {
  return launch_half_to_f32<true>(src, dst, n, as_stream(stream));
}

int ah_f32_to_f16(const float* src, uint16_t* dst, int64_t n, void* stream) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(src && dst && n > 0, "f32_to_f16: null pointer or negative n");
  cudaStream_t st = as_stream(stream);
  int64_t done = 0;
  if (aligned16(src) && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      k_f32_to_f16_vec<<<grid_for(n4), kThreads, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                          reinterpret_cast<uint2*>(dst), n4);
      AH_LAUNCH_CHECK();
    }
    done = n4 * 4;
  }
  if (done < n) {
    k_f32_to_f16_scalar<<<grid_for(n - done), kThreads, 0, st>>>(src + done, dst + done, n - done);
    AH_LAUNCH_CHECK();
  }
  return AH_OK;
}

int ah_dequant_q8_0_f32(const void* blocks, float* out, int64_t n, void* stream) {
  return launch_dequant_blocks<Q8Fmt>(blocks, out, n, as_stream(stream));
}

int ah_dequant_q4_0_f32(const void* blocks, float* out, int64_t n, void* stream) {
  return launch_dequant_blocks<Q4Fmt>(blocks, out, n, as_stream(stream));
}

int ah_dequant_layer(const float* scales, const uint8_t* packed, float* out, int64_t n, int64_t gs, void* stream) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(scales && packed && out && n > 0 && gs > 0, "dequant_layer: bad arguments");
  cudaStream_t st = as_stream(stream);
  int64_t done = 0;
  if (gs == 32 && aligned16(packed) && aligned16(scales) && aligned16(out) &&
      n >= (int64_t)EngineFmt::kTileBlocks * 32) {
    // whole tiles through the bulk-copy ring (nibbles and scales on one mbarrier)
    const int64_t n_tiles = n / ((int64_t)EngineFmt::kTileBlocks * 32);
    int64_t g = (int64_t)sm_count() * 4;
    if (g > n_tiles) g = n_tiles;
    int* err = device_error_word();
    AH_REQUIRE(err != nullptr, "dequant_layer: device error word unavailable");
    k_dequant_blocks_tma<EngineFmt><<<(int)g, kThreads, 0, st>>>(packed, out, n_tiles, err, scales);
    AH_LAUNCH_CHECK();
    done = n_tiles * EngineFmt::kTileBlocks * 32;
  }
  if (done < n && gs == 32 && (reinterpret_cast<uintptr_t>(packed) & 3u) == 0 && aligned16(out)) {
    const int64_t n8 = (n - done) / 8;  // done is a multiple of 32: groups stay whole
    if (n8 > 0) {
      k_dequant_engine_gs32<<<grid_for(n8), kThreads, 0, st>>>(scales + done / 32,
                                                               reinterpret_cast<const uint32_t*>(packed + done / 2),
                                                               reinterpret_cast<float4*>(out + done), n8);
      AH_LAUNCH_CHECK();
    }
    done += n8 * 8;
  }
  if (done < n) {
    k_dequant_engine_any<<<grid_for(n - done), kThreads, 0, st>>>(scales, packed, out, done, n, gs);
    AH_LAUNCH_CHECK();
  }
  return AH_OK;
}

int ah_dequantize_to_f32(const void* raw, int64_t raw_bytes, uint32_t dtype, int64_t element_count, float* out,
                         int64_t* n_out, void* stream) {
  AH_REQUIRE(n_out != nullptr && raw_bytes >= 0 && element_count >= 0, "dequantize_to_f32: bad arguments");
  cudaStream_t st = as_stream(stream);
  *n_out = 0;
  switch (dtype) {
    case AH_DTYPE_F32: {
      const int64_t k = raw_bytes / 4;
      if (k > 0) AH_CUDA_TRY(cudaMemcpyAsync(out, raw, (size_t)k * 4, cudaMemcpyDeviceToDevice, st));
      *n_out = k;
      return AH_OK;
    }
    case AH_DTYPE_F16: *n_out = raw_bytes / 2; return launch_half_to_f32<false>(raw, out, raw_bytes / 2, st);
    case AH_DTYPE_BF16: *n_out = raw_bytes / 2; return launch_half_to_f32<true>(raw, out, raw_bytes / 2, st);
    case AH_DTYPE_Q8_0: {
      const int64_t full = raw_bytes / 34, rem = raw_bytes % 34;
      int64_t avail = full * 32 + (rem >= 2 ? (rem - 2 < 32 ? rem - 2 : 32) : 0);
      const int64_t k = avail < element_count ? avail : element_count;
      *n_out = k;
      return launch_dequant_blocks<Q8Fmt>(raw, out, k, st);
    }
    case AH_DTYPE_Q4_0: {
      const int64_t nb = (element_count + 31) / 32;
      int64_t k = element_count;
      if (raw_bytes < nb * 18) {
        const int64_t b = raw_bytes / 18;  // first block not fully present
        if (b * 18 + 2 <= raw_bytes)
          return fail(AH_EINVAL, "dequantize_to_f32: truncated Q4_0 block %lld (the reference panics here)",
                      (long long)b);
        k = b * 32 < element_count ? b * 32 : element_count;
      }
      *n_out = k;
      return launch_dequant_blocks<Q4Fmt>(raw, out, k, st);
    }
    case AH_DTYPE_Q6_K: {
      const int64_t full = raw_bytes / 210;
      const int64_t k = full * 256 < element_count ? full * 256 : element_count;
      *n_out = k;
      if (k > 0) {
        k_dequant_q6k_approx<<<grid_for(k), kThreads, 0, st>>>(static_cast<const uint8_t*>(raw), out, k);
        AH_LAUNCH_CHECK();
      }
      return AH_OK;
    }
    default:
      *n_out = element_count;
      if (element_count > 0) AH_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)element_count * 4, st));
      return AH_OK;
  }
}

}  // extern "C"
