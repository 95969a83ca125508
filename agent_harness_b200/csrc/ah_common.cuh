// ah_common.cuh — shared helpers for the sm_100a kernels and the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/ah_cuda.h"

namespace ah {

// ---- errors ------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);

#define AH_CUDA_TRY(expr)                                                                    \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    if (_e != cudaSuccess) return ::ah::fail(AH_ECUDA, "%s: %s (%s:%d)", #expr,             \
                                             cudaGetErrorString(_e), __FILE__, __LINE__);     \
  } while (0)

#define AH_LAUNCH_CHECK()                                                                    \
  do {                                                                                       \
    cudaError_t _e = cudaGetLastError();                                                     \
    if (_e != cudaSuccess) return ::ah::fail(AH_ECUDA, "kernel launch: %s (%s:%d)",          \
                                             cudaGetErrorString(_e), __FILE__, __LINE__);     \
  } while (0)

#define AH_REQUIRE(cond, ...)                                                                \
  do {                                                                                       \
    if (!(cond)) return ::ah::fail(AH_EINVAL, __VA_ARGS__);                                  \
  } while (0)

// ---- device facts --------------------------------------------------------------
int sm_count();  // SM count of the current device (cached per device)
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per-device error word (a zero-initialised __device__ variable of this
// library's module) that kernels with bounded waits set when a wait gives up;
// read and cleared by ah_check_device_error.  Looking it up allocates nothing.
int* device_error_word();

// Every device allocation of the library goes through here: counted for
// ah_device_alloc_count, and failed on request by ah_debug_inject_failure.
cudaError_t dev_malloc(void** p, size_t bytes);
template <typename T>
inline cudaError_t dev_malloc(T** p, size_t bytes) {
  void* v = nullptr;
  const cudaError_t e = dev_malloc(&v, bytes);
  *p = static_cast<T*>(v);
  return e;
}
// True when an armed injection of this AH_INJECT_* kind fires on this call.
bool inject_failure(int kind);
// Codes in the error word: 0x5xxx input indices a kernel found out of range
// (AH_EINVAL); every other code is a bounded wait that gave up (AH_ETIMEOUT).
constexpr int kDeviceIndexError = 0x5000;

// ---- bit-exact scalar semantics ------------------------------------------------
// f16 bits -> f32 with the reference's NaN rule (formats/gguf.rs:93-120): every
// NaN becomes f32::NAN (0x7FC00000) with the half's sign; all other values are
// exact, which the hardware conversion already is.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  float v = __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
  if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu)) v = __uint_as_float(((h & 0x8000u) << 16) | 0x7FC00000u);
  return v;
}

// The x86 SSE product the reference's Rust code compiles to: a NaN operand is
// returned quieted (its sign and payload kept); inf*0 gives the default NaN
// 0xFFC00000.  `a` may be NaN, `q` never is (a small integer).
__device__ __forceinline__ float x86_mul(float a, float q) {
  float p = __fmul_rn(a, q);
  if (p != p) {
    uint32_t ab = __float_as_uint(a);
    p = (a != a) ? __uint_as_float(ab | 0x00400000u) : __uint_as_float(0xFFC00000u);
  }
  return p;
}

__device__ __forceinline__ int rust_f32_as_i32(float v) {
  // Rust `as i32`: saturating, NaN -> 0 (values here are already bounded).
  if (v != v) return 0;
  return __float2int_rz(v);
}

// ---- counter-based normal generator (synthetic inputs) -----------------------------
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Element i of the stream keyed by `key` (= splitmix64(seed)): Box-Muller on the
// pair i>>1 with u1 in (0,1], u2 in [0,1); even i takes the cosine branch.
__device__ __forceinline__ float normal_at(uint64_t key, uint64_t i) {
  uint64_t z = splitmix64(key + (i >> 1));
  float u1 = (float)((z >> 40) + 1) * (1.0f / 16777216.0f);
  float u2 = (float)(z & 0xFFFFFFull) * (1.0f / 16777216.0f);
  float r = sqrtf(-2.0f * logf(u1));
  float s, c;
  sincospif(2.0f * u2, &s, &c);
  return (i & 1) ? r * s : r * c;
}

}  // namespace ah
