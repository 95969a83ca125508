// ah_runtime.cu — status/error plumbing, device facts and the host-slice
// staging used by the ah_host_* drop-in entries.
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <vector>

#include "ah_common.cuh"

namespace ah {

static thread_local char t_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return status;
}

// The error word lives in the module's own device memory (one per device
// context, zero at module load), so reaching it allocates nothing: even an
// entry whose contract is to allocate nothing may report a timeout through it.
__device__ int g_device_error_word;

int* device_error_word() {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static int* words[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!words[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    words[dev] = static_cast<int*>(p);
  }
  return words[dev];
}

// ---- device allocations: one counted entry, with host-side failure injection ----
static std::atomic<int64_t> g_alloc_count{0};
static std::atomic<int64_t> g_inject[4];  // countdown per AH_INJECT_* kind (0: disarmed)

bool inject_failure(int kind) {
  if (kind < 1 || kind > 3) return false;
  int64_t v = g_inject[kind].load();
  while (v > 0) {
    if (g_inject[kind].compare_exchange_weak(v, v - 1)) return v == 1;
  }
  return false;
}

cudaError_t dev_malloc(void** p, size_t bytes) {
  *p = nullptr;
  if (inject_failure(AH_INJECT_ALLOC)) return cudaErrorMemoryAllocation;
  const cudaError_t e = cudaMalloc(p, bytes);
  if (e == cudaSuccess) g_alloc_count.fetch_add(1);
  return e;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace ah

using namespace ah;

extern "C" {

const char* ah_strerror(int status) {
  switch (status) {
    case AH_OK: return "ok";
    case AH_EINVAL: return "invalid argument";
    case AH_ENOMEM: return "out of memory";
    case AH_ECUDA: return "CUDA error";
    case AH_ENCCL: return "NCCL error";
    case AH_ETIMEOUT: return "device-side wait timed out";
    case AH_EUNSUPPORTED: return "unsupported";
    default: return "unknown status";
  }
}

const char* ah_last_error(void) { return t_last_error; }

int ah_version(void) { return 1; }

int ah_device_init(int device) {
  AH_CUDA_TRY(cudaSetDevice(device));
  AH_CUDA_TRY(cudaFree(nullptr));  // establish the primary context
  (void)sm_count();
  if (!device_error_word()) return fail(AH_ECUDA, "device_init: the device error word is unavailable");
  return AH_OK;
}

int ah_check_device_error(void* stream) {
  int* w = device_error_word();
  if (!w) return fail(AH_ECUDA, "check_device_error: the device error word is unavailable");
  int v = 0;
  AH_CUDA_TRY(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, as_stream(stream)));
  AH_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  if (v != 0) {
    const int zero = 0;
    AH_CUDA_TRY(cudaMemcpyAsync(w, &zero, sizeof(int), cudaMemcpyHostToDevice, as_stream(stream)));
    AH_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    if ((v & 0xF000) == kDeviceIndexError)
      return fail(AH_EINVAL, "a device-side index check failed (code 0x%x)", v);
    return fail(AH_ETIMEOUT, "a bounded device-side wait gave up (code 0x%x)", v);
  }
  return AH_OK;
}

int64_t ah_packed_bytes(int64_t n) { return n < 0 ? 0 : (n + 1) / 2; }
int64_t ah_n_groups(int64_t n, int64_t gs) { return (n < 0 || gs <= 0) ? 0 : (n + gs - 1) / gs; }
int64_t ah_quantized_bytes(int64_t n, int64_t gs) { return ah_n_groups(n, gs) * 4 + ah_packed_bytes(n); }

int64_t ah_device_alloc_count(void) { return g_alloc_count.load(); }

int ah_debug_inject_failure(int kind, int64_t nth) {
  AH_REQUIRE(kind >= AH_INJECT_ALLOC && kind <= AH_INJECT_LAUNCH, "inject_failure: unknown kind %d", kind);
  AH_REQUIRE(nth >= 0, "inject_failure: negative count");
  g_inject[kind].store(nth);
  return AH_OK;
}

}  // extern "C"
