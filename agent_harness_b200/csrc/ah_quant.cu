// ah_quant.cu — quantisers (the engine's INT4 format and the Q8_0/Q4_0 block
// formats) and the seeded synthetic-input generators, for sm_100a.
//
// Quantisation is a load-time pass (inference/mod.rs:184-314 runs it once per
// tensor), so these kernels favour exactness over speed: every arithmetic step
// uses the IEEE round-to-nearest intrinsic the Rust reference's scalar code
// performs, so the packed bytes and scales are bit-identical to the CPU oracle.
#include "ah_common.cuh"

namespace ah {
namespace {

constexpr int kThreads = 256;

inline int grid_cap(int64_t items, int per_sm = 16) {
  int64_t g = (items + kThreads - 1) / kThreads;
  int64_t cap = (int64_t)sm_count() * per_sm;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t f32_to_f16_rne(float f) {
  uint32_t x = __float_as_uint(f);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return ((x >> 16) & 0x8000u) | 0x7E00u | ((x >> 13) & 0x3FFu);
  return __half_as_ushort(__float2half_rn(f));
}

// --- engine format, group size 32: one warp per group (quantization.rs:369-404) ---
__global__ void __launch_bounds__(kThreads) k_quantize_q4_gs32(const float* __restrict__ w, int64_t n,
                                                               float* __restrict__ scales,
                                                               uint8_t* __restrict__ packed) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t n_groups = (n + 31) / 32;
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < n_groups; g += warps) {
    const int64_t idx = g * 32 + lane;
    const bool live = idx < n;
    const float v = live ? w[idx] : 0.0f;
    const float max_abs = warp_max(live ? fabsf(v) : 0.0f);
    const float scale = max_abs > 0.0f ? __fdiv_rn(max_abs, 7.0f) : 0.0f;
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    int q = scale > 0.0f ? rust_f32_as_i32(roundf(__fmul_rn(v, inv))) : 0;
    q = min(max(q, -8), 7) + 8;
    const int hi = __shfl_down_sync(0xFFFFFFFFu, q, 1);
    if (lane == 0) scales[g] = scale;
    if (live && (lane & 1) == 0) packed[idx >> 1] = (uint8_t)(q | ((idx + 1 < n ? hi : 0) << 4));
  }
}

// --- engine format, any group size: scales, then one thread per packed byte ---
__global__ void __launch_bounds__(kThreads) k_quantize_q4_scales(const float* __restrict__ w, int64_t n, int64_t gs,
                                                                 float* __restrict__ scales) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n_groups = (n + gs - 1) / gs;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n_groups; g += stride) {
    const int64_t s = g * gs, e = s + gs < n ? s + gs : n;
    float max_abs = 0.0f;
    for (int64_t i = s; i < e; ++i) max_abs = fmaxf(max_abs, fabsf(w[i]));
    scales[g] = max_abs > 0.0f ? __fdiv_rn(max_abs, 7.0f) : 0.0f;
  }
}

__device__ __forceinline__ int q4_nibble(float v, float scale) {
  const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
  int q = scale > 0.0f ? rust_f32_as_i32(roundf(__fmul_rn(v, inv))) : 0;
  return min(max(q, -8), 7) + 8;
}

__global__ void __launch_bounds__(kThreads) k_quantize_q4_bytes(const float* __restrict__ w, int64_t n, int64_t gs,
                                                                const float* __restrict__ scales,
                                                                uint8_t* __restrict__ packed) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nbytes = (n + 1) / 2;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nbytes; b += stride) {
    const int64_t i0 = 2 * b, i1 = i0 + 1;
    int lo = q4_nibble(w[i0], scales[i0 / gs]);
    int hi = i1 < n ? q4_nibble(w[i1], scales[i1 / gs]) : 0;
    packed[b] = (uint8_t)(lo | (hi << 4));
  }
}

// --- Q8_0 / Q4_0 blocks, one warp per block ---
template <bool kQ4>
__device__ __forceinline__ void quantize_block(float v, bool live, int lane, uint8_t* blk) {
  const float amax = warp_max(live ? fabsf(v) : 0.0f);
  const uint32_t d16 = f32_to_f16_rne(__fdiv_rn(amax, kQ4 ? 8.0f : 127.0f));
  const float d = __half2float(__ushort_as_half((unsigned short)d16));
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  if (kQ4) {
    int q = live ? rust_f32_as_i32(roundf(__fmul_rn(v, id))) + 8 : 8;
    q = min(max(q, 0), 15);
    const int hi = __shfl_down_sync(0xFFFFFFFFu, q, 1);
    if (lane == 0) *reinterpret_cast<uint16_t*>(blk) = (uint16_t)d16;
    if ((lane & 1) == 0) blk[2 + (lane >> 1)] = (uint8_t)(q | (hi << 4));
  } else {
    int q = live ? rust_f32_as_i32(roundf(__fmul_rn(v, id))) : 0;
    q = min(max(q, -127), 127);
    if (lane == 0) *reinterpret_cast<uint16_t*>(blk) = (uint16_t)d16;
    blk[2 + lane] = (uint8_t)(int8_t)q;
  }
}

template <bool kQ4>
__global__ void __launch_bounds__(kThreads) k_quantize_blocks(const float* __restrict__ w, int64_t n,
                                                              uint8_t* __restrict__ blocks) {
  constexpr int kBytes = kQ4 ? 18 : 34;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nb = (n + 31) / 32;
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nb; b += warps) {
    const int64_t idx = b * 32 + lane;
    const bool live = idx < n;
    quantize_block<kQ4>(live ? w[idx] : 0.0f, live, lane, blocks + b * kBytes);
  }
}

// --- synthetic inputs ---
__global__ void __launch_bounds__(kThreads) k_fill_normal(float* __restrict__ out, int64_t n, float mean, float std,
                                                          uint64_t key, int64_t off) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = __fadd_rn(mean, __fmul_rn(std, normal_at(key, (uint64_t)(i + off))));
}

__global__ void __launch_bounds__(kThreads) k_synth_f16(uint16_t* __restrict__ out, int64_t n, float mean, float std,
                                                        uint64_t key, int64_t off) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = (uint16_t)f32_to_f16_rne(__fadd_rn(mean, __fmul_rn(std, normal_at(key, (uint64_t)(i + off)))));
}

__global__ void __launch_bounds__(kThreads) k_synth_q4_0(uint8_t* __restrict__ blocks, int64_t row0, int64_t rows,
                                                         int64_t col0, int64_t cols, int64_t full_cols, float std,
                                                         uint64_t key) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t bpr = cols / 32;
  const int64_t nb = rows * bpr;
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nb; b += warps) {
    const int64_t r = b / bpr, cb = b % bpr;
    const uint64_t gi = (uint64_t)(row0 + r) * (uint64_t)full_cols + (uint64_t)(col0 + cb * 32 + lane);
    quantize_block<true>(__fmul_rn(std, normal_at(key, gi)), true, lane, blocks + b * 18);
  }
}

}  // namespace
}  // namespace ah

using namespace ah;

extern "C" {

int ah_quantize_q4(const float* w, int64_t n, int64_t gs, float* scales, uint8_t* packed, void* stream) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(w && scales && packed && n > 0, "quantize_q4: bad arguments");
  if (gs < 1) gs = 1;  // quantization.rs:370 group_size.max(1)
  cudaStream_t st = as_stream(stream);
  if (gs == 32) {
    k_quantize_q4_gs32<<<grid_cap((n + 31) / 32 * 32), kThreads, 0, st>>>(w, n, scales, packed);
    AH_LAUNCH_CHECK();
    return AH_OK;
  }
  k_quantize_q4_scales<<<grid_cap((n + gs - 1) / gs), kThreads, 0, st>>>(w, n, gs, scales);
  AH_LAUNCH_CHECK();
  k_quantize_q4_bytes<<<grid_cap((n + 1) / 2), kThreads, 0, st>>>(w, n, gs, scales, packed);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_quantize_q8_0(const float* w, int64_t n, void* blocks, void* stream) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(w && blocks && n > 0 && (reinterpret_cast<uintptr_t>(blocks) & 1u) == 0,
             "quantize_q8_0: bad arguments (blocks must be 2-byte aligned)");
  k_quantize_blocks<false><<<grid_cap((n + 31) / 32 * 32), kThreads, 0, as_stream(stream)>>>(
      w, n, static_cast<uint8_t*>(blocks));
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_quantize_q4_0(const float* w, int64_t n, void* blocks, void* stream) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(w && blocks && n > 0 && (reinterpret_cast<uintptr_t>(blocks) & 1u) == 0,
             "quantize_q4_0: bad arguments (blocks must be 2-byte aligned)");
  k_quantize_blocks<true><<<grid_cap((n + 31) / 32 * 32), kThreads, 0, as_stream(stream)>>>(
      w, n, static_cast<uint8_t*>(blocks));
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_fill_normal(float* out, int64_t n, float mean, float std, uint64_t seed, int64_t off, void* stream) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(out && n > 0 && off >= 0, "fill_normal: bad arguments");
  k_fill_normal<<<grid_cap(n), kThreads, 0, as_stream(stream)>>>(out, n, mean, std, splitmix64(seed), off);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_synth_f16(uint16_t* out, int64_t n, float mean, float std, uint64_t seed, int64_t off, void* stream) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(out && n > 0 && off >= 0, "synth_f16: bad arguments");
  k_synth_f16<<<grid_cap(n), kThreads, 0, as_stream(stream)>>>(out, n, mean, std, splitmix64(seed), off);
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_synth_q4_0(void* blocks, int64_t row0, int64_t rows, int64_t col0, int64_t cols, int64_t full_cols, float std,
                  uint64_t seed, void* stream) {
  if (rows == 0 || cols == 0) return AH_OK;
  AH_REQUIRE(blocks && rows > 0 && cols > 0 && cols % 32 == 0 && col0 % 32 == 0 && col0 + cols <= full_cols &&
                 row0 >= 0 && (reinterpret_cast<uintptr_t>(blocks) & 1u) == 0,
             "synth_q4_0: bad arguments");
  k_synth_q4_0<<<grid_cap(rows * cols), kThreads, 0, as_stream(stream)>>>(static_cast<uint8_t*>(blocks), row0, rows,
                                                                          col0, cols, full_cols, std,
                                                                          splitmix64(seed));
  AH_LAUNCH_CHECK();
  return AH_OK;
}

}  // extern "C"
