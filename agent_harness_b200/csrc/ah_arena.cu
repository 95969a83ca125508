// ah_arena.cu — a paged virtual tensor arena on CUDA virtual memory management,
// the B200 form of memory_controller/virtual_tensor_arena.rs:23-257.
//
// The reference reserves a sparse Vulkan buffer and binds fixed-size pages of
// GPU memory into it (commit_page), routes a page to host memory when the GPU
// is out of memory, unbinds pages (evict_page: Move to the host or Drop), and
// runs gemv_4bit_into on a page (execute_layer_math; its GPU branch is empty).
// Here:
//   * the arena is one reserved virtual address range (cuMemAddressReserve),
//     so a page's device address never changes while its backing comes and goes;
//   * commit maps one physical allocation of page_bytes (cuMemCreate + cuMemMap
//     + cuMemSetAccess) at the page's address; an out-of-memory result, or a
//     full page budget (the caller's cap on GPU-resident pages, which stands in
//     for device exhaustion), routes the page to the host pool instead;
//   * evict waits for the device, copies a GPU page's bytes into the host pool
//     on Move, then unmaps and releases the physical allocation;
//   * the page GEMV runs on the device either way: GPU pages through their
//     arena address, host pages through the pinned host pool over the bus.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <new>
#include <vector>

#include "ah_common.cuh"

struct AhArena {
  int device = 0;
  CUdeviceptr base = 0;
  size_t total = 0, page_bytes = 0;
  int64_t n_pages = 0, budget = -1, gpu_pages = 0;
  std::vector<int> residency;                        // AH_PAGE_*
  std::vector<CUmemGenericAllocationHandle> handle;  // GPU pages
  std::vector<char> cpu_offset;                      // the reference's cpu_offset is Some
  std::mutex mu;
};

namespace ah {
namespace {

struct VmmApi {
  PFN_cuMemAddressReserve reserve = nullptr;
  PFN_cuMemAddressFree free_va = nullptr;
  PFN_cuMemCreate create = nullptr;
  PFN_cuMemRelease release = nullptr;
  PFN_cuMemMap map = nullptr;
  PFN_cuMemUnmap unmap = nullptr;
  PFN_cuMemSetAccess access = nullptr;
  PFN_cuMemGetAllocationGranularity granularity = nullptr;
  bool ok = false;
};

template <typename F>
bool entry(const char* name, F* fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return false;
  }
  *fn = reinterpret_cast<F>(p);
  return true;
}

// Driver entry points through the runtime (no -lcuda), resolved once.
const VmmApi& vmm() {
  static VmmApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    api.ok = entry("cuMemAddressReserve", &api.reserve) && entry("cuMemAddressFree", &api.free_va) &&
             entry("cuMemCreate", &api.create) && entry("cuMemRelease", &api.release) && entry("cuMemMap", &api.map) &&
             entry("cuMemUnmap", &api.unmap) && entry("cuMemSetAccess", &api.access) &&
             entry("cuMemGetAllocationGranularity", &api.granularity);
  });
  return api;
}

CUmemAllocationProp device_prop(int dev) {
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = dev;
  return p;
}

int vmm_fail(const char* what, CUresult r) { return fail(AH_ECUDA, "arena: %s failed (CUresult %d)", what, (int)r); }

// Unmaps and releases a GPU page (the caller holds the lock and has synchronised).
int unbind(AhArena* a, int64_t page) {
  const VmmApi& v = vmm();
  const CUdeviceptr va = a->base + (CUdeviceptr)page * a->page_bytes;
  CUresult r = v.unmap(va, a->page_bytes);
  if (r != CUDA_SUCCESS) return vmm_fail("cuMemUnmap", r);
  r = v.release(a->handle[page]);
  if (r != CUDA_SUCCESS) return vmm_fail("cuMemRelease", r);
  a->handle[page] = 0;
  a->gpu_pages -= 1;
  return AH_OK;
}

}  // namespace
}  // namespace ah

using namespace ah;

extern "C" {

int ah_arena_page_granularity(size_t* bytes) {
  AH_REQUIRE(bytes, "arena: null out");
  const VmmApi& v = vmm();
  if (!v.ok) return fail(AH_ECUDA, "arena: the driver's virtual memory entry points are unavailable");
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  CUmemAllocationProp p = device_prop(dev);
  const CUresult r = v.granularity(bytes, &p, CU_MEM_ALLOC_GRANULARITY_MINIMUM);
  if (r != CUDA_SUCCESS) return vmm_fail("cuMemGetAllocationGranularity", r);
  return AH_OK;
}

int ah_arena_create(size_t total_virtual_bytes, size_t page_bytes, int64_t gpu_page_budget, AhArena** out) {
  AH_REQUIRE(out, "arena: null out");
  *out = nullptr;
  size_t g = 0;
  const int rc = ah_arena_page_granularity(&g);
  if (rc != AH_OK) return rc;
  AH_REQUIRE(page_bytes > 0 && page_bytes % g == 0, "arena: page_bytes must be a multiple of %zu", g);
  AH_REQUIRE(total_virtual_bytes >= page_bytes && total_virtual_bytes % page_bytes == 0,
             "arena: total_virtual_bytes must be a positive multiple of page_bytes");
  AhArena* a = new (std::nothrow) AhArena();
  if (!a) return fail(AH_ENOMEM, "arena: host allocation");
  cudaGetDevice(&a->device);
  a->total = total_virtual_bytes;
  a->page_bytes = page_bytes;
  a->n_pages = (int64_t)(total_virtual_bytes / page_bytes);
  a->budget = gpu_page_budget;
  a->residency.assign(a->n_pages, AH_PAGE_UNMAPPED);
  a->handle.assign(a->n_pages, 0);
  a->cpu_offset.assign(a->n_pages, 0);
  const CUresult r = vmm().reserve(&a->base, total_virtual_bytes, g, 0, 0);
  if (r != CUDA_SUCCESS) {
    delete a;
    return vmm_fail("cuMemAddressReserve", r);
  }
  *out = a;
  return AH_OK;
}

int ah_arena_destroy(AhArena* a) {
  if (!a) return AH_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(a->device);
  cudaDeviceSynchronize();
  int rc = AH_OK;
  for (int64_t p = 0; p < a->n_pages; ++p)
    if (a->residency[p] == AH_PAGE_GPU && rc == AH_OK) rc = unbind(a, p);
  if (a->base) vmm().free_va(a->base, a->total);
  cudaSetDevice(cur);
  delete a;
  return rc;
}

int ah_arena_commit_page(AhArena* a, int64_t page) {
  AH_REQUIRE(a && page >= 0 && page < a->n_pages, "arena: page %lld out of range", (long long)page);
  std::lock_guard<std::mutex> lk(a->mu);
  if (a->residency[page] != AH_PAGE_UNMAPPED) return AH_OK;  // virtual_tensor_arena.rs:81-83
  auto route_to_cpu = [&] {                                  // :142-147
    a->residency[page] = AH_PAGE_CPU;
    a->cpu_offset[page] = 1;
    return AH_OK;
  };
  if (a->budget >= 0 && a->gpu_pages >= a->budget) return route_to_cpu();
  const VmmApi& v = vmm();
  CUmemAllocationProp prop = device_prop(a->device);
  CUmemGenericAllocationHandle h = 0;
  CUresult r = v.create(&h, a->page_bytes, &prop, 0);
  if (r == CUDA_ERROR_OUT_OF_MEMORY) return route_to_cpu();
  if (r != CUDA_SUCCESS) return vmm_fail("cuMemCreate", r);
  const CUdeviceptr va = a->base + (CUdeviceptr)page * a->page_bytes;
  r = v.map(va, a->page_bytes, 0, h, 0);
  if (r != CUDA_SUCCESS) {
    v.release(h);
    return r == CUDA_ERROR_OUT_OF_MEMORY ? route_to_cpu() : vmm_fail("cuMemMap", r);
  }
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = a->device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = v.access(va, a->page_bytes, &acc, 1);
  if (r != CUDA_SUCCESS) {
    v.unmap(va, a->page_bytes);
    v.release(h);
    return vmm_fail("cuMemSetAccess", r);
  }
  a->handle[page] = h;
  a->residency[page] = AH_PAGE_GPU;
  a->gpu_pages += 1;
  return AH_OK;
}

int ah_arena_evict_page(AhArena* a, int64_t page, int move, void* host_pool, void* stream) {
  AH_REQUIRE(a && page >= 0 && page < a->n_pages, "arena: page %lld out of range", (long long)page);
  std::lock_guard<std::mutex> lk(a->mu);
  const bool gpu = a->residency[page] == AH_PAGE_GPU;
  if (gpu) {
    // nothing may still read or write the page when it is unmapped
    AH_CUDA_TRY(cudaDeviceSynchronize());
    if (move) {
      AH_REQUIRE(host_pool, "arena: Move needs the host pool");
      const CUdeviceptr va = a->base + (CUdeviceptr)page * a->page_bytes;
      AH_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(host_pool) + (size_t)page * a->page_bytes,
                                  reinterpret_cast<const void*>(va), a->page_bytes, cudaMemcpyDeviceToHost,
                                  as_stream(stream)));
      AH_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
      a->cpu_offset[page] = 1;  // virtual_tensor_arena.rs:159-163
    }
    const int rc = unbind(a, page);
    if (rc != AH_OK) return rc;
  }
  if (move) {
    a->residency[page] = AH_PAGE_CPU;  // :195-197 (a page never on the GPU keeps no cpu offset)
  } else {
    a->residency[page] = AH_PAGE_UNMAPPED;  // :191-194
    a->cpu_offset[page] = 0;
  }
  return AH_OK;
}

int ah_arena_page_state(const AhArena* ca, int64_t page, int* residency, void** dev_ptr) {
  AH_REQUIRE(ca && residency && page >= 0 && page < ca->n_pages, "arena: page %lld out of range", (long long)page);
  AhArena* a = const_cast<AhArena*>(ca);
  std::lock_guard<std::mutex> lk(a->mu);
  *residency = a->residency[page];
  if (dev_ptr)
    *dev_ptr = a->residency[page] == AH_PAGE_GPU ? reinterpret_cast<void*>(a->base + (CUdeviceptr)page * a->page_bytes)
                                                 : nullptr;
  return AH_OK;
}

int ah_arena_gemv_4bit(AhArena* a, int64_t page, const void* host_pool, float* out, const float* scales,
                       const float* x, int64_t rows, int64_t cols, int64_t group_size, void* stream) {
  AH_REQUIRE(a && page >= 0 && page < a->n_pages, "arena: page %lld out of range", (long long)page);
  AH_REQUIRE(rows >= 0 && cols >= 0 && (size_t)((rows * cols + 1) / 2) <= a->page_bytes,
             "arena: a %lld x %lld packed matrix does not fit one page", (long long)rows, (long long)cols);
  const uint8_t* packed = nullptr;
  // the lock is held through the (asynchronous) launch: an eviction takes it,
  // then waits for the device before unmapping, so the page stays mapped for
  // every GEMV enqueued on it
  std::lock_guard<std::mutex> lk(a->mu);
  {
    switch (a->residency[page]) {
      case AH_PAGE_UNMAPPED:  // virtual_tensor_arena.rs:231-232 panics
        return fail(AH_EINVAL, "arena: page %lld is unmapped", (long long)page);
      case AH_PAGE_GPU:
        packed = reinterpret_cast<const uint8_t*>(a->base + (CUdeviceptr)page * a->page_bytes);
        break;
      default: {
        AH_REQUIRE(a->cpu_offset[page], "arena: page %lld is host resident without data (:253-254)",
                   (long long)page);
        AH_REQUIRE(host_pool, "arena: host-resident page %lld needs the host pool", (long long)page);
        cudaPointerAttributes at{};
        const cudaError_t e = cudaPointerGetAttributes(&at, host_pool);
        if (e != cudaSuccess || at.type != cudaMemoryTypeHost || !at.devicePointer) {
          cudaGetLastError();
          return fail(AH_EINVAL, "arena: the host pool must be pinned (device-mapped) host memory");
        }
        packed = static_cast<const uint8_t*>(at.devicePointer) + (size_t)page * a->page_bytes;
      }
    }
  }
  return ah_gemv_4bit_into(out, scales, packed, x, rows, cols, group_size, stream);
}

}  // extern "C"
