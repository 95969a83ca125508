// ah_probe.cu — a measurement kernel behind the batched GEMV's design: the
// cost of one tcgen05.mma (kind::f16, K = 16) by N, by where A lives (tensor
// or shared memory) and for the CTA-pair form (cta_group::2, M = 256).
//
// One cluster of two CTAs; one thread issues kProbeIters MMAs into one
// accumulator and times issue and completion with clock64 and %globaltimer.
// Operands are left uninitialised: only the time is read.  Every address is
// inside the CTA's allocation (B <= 32 KB and A <= 16 KB of shared memory,
// D in tensor-memory columns 0..255, A in columns 256..287); the completion
// wait is bounded.
#include "ah_common.cuh"
#include "ah_sm100.cuh"
#include "ah_tc.cuh"

namespace ah {
namespace {

constexpr int kProbeIters = 256;
constexpr int kProbeSmem = 50 * 1024;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// mode 0: cta_group::1, A from shared memory, M = 64
// mode 1: cta_group::1, A from tensor memory, M = 128
// mode 2: cta_group::2, A from tensor memory, M = 256 (N >= 32)
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1) k_probe_mma(long long* out, int n, int mode) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5;
  const uint32_t rank = cluster_ctarank();
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    if (mode == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&slot)),
                   "r"(512)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      tmem_alloc(&slot, 512);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_arrive();
  cluster_wait();
  tc_fence_after();
  const uint32_t tmem = slot;
  const bool issuer = threadIdx.x == 0 && (mode != 2 || rank == 0);
  if (issuer) {
    const int m = mode == 0 ? 64 : (mode == 1 ? 128 : 256);
    const uint32_t idesc = idesc_f16(m, n);
    const uint64_t bdesc = sw128_desc(smem_u32(sm));          // B: n (or n/2) rows x 128 B
    const uint64_t adesc = sw128_desc(smem_u32(sm + 32768));  // A (M = 64): 64 rows x 128 B
    const long long t0 = clock64();
    const unsigned long long g0 = globaltimer_ns();
    for (int i = 0; i < kProbeIters; ++i) {
      const uint32_t kk = (uint32_t)(i & 3);
      if (mode == 0) {
        mma_f16(tmem, adesc + kk * 2, bdesc + kk * 2, idesc, i > 0);
      } else if (mode == 1) {
        mma_f16_ts(tmem, tmem + 256 + kk * 8, bdesc + kk * 2, idesc, i > 0);
      } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(
                tmem),
            "r"(tmem + 256 + kk * 8), "l"(bdesc + kk * 2), "r"(idesc), "r"((uint32_t)(i > 0)), "r"(0u)
            : "memory");
      }
    }
    const long long t1 = clock64();
    if (mode == 2) {
      // the leader's barrier only; the peer CTA meets it at the cluster barrier below
      asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(&bar))
                   : "memory");
    } else {
      mma_commit(&bar);
    }
    mbar_wait_bounded(&bar, 0, nullptr, 0, 1u << 26);
    const long long t2 = clock64();
    const unsigned long long g2 = globaltimer_ns();
    if (blockIdx.x == 0) {
      out[0] = t1 - t0;
      out[1] = t2 - t0;
      out[2] = (long long)(g2 - g0);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_arrive();
  cluster_wait();
  if (warp == 0) {
    tc_fence_after();
    if (mode == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    else
      tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace ah

extern "C" {

// Times kProbeIters back-to-back tcgen05.mma (kind::f16, K = 16, one
// accumulator) on one SM (or one SM pair for mode 2): out[0] = issue cycles,
// out[1] = cycles to completion, out[2] = nanoseconds to completion.
AH_API int ah_debug_tc_mma_rate(int mode, int n, long long* out_host) {
  AH_REQUIRE(out_host != nullptr, "ah_debug_tc_mma_rate: null output");
  AH_REQUIRE(mode >= 0 && mode <= 2, "ah_debug_tc_mma_rate: mode must be 0, 1 or 2");
  const int n_min = mode == 2 ? 32 : (mode == 0 ? 8 : 16);
  AH_REQUIRE(n >= n_min && n <= 256 && n % n_min == 0, "ah_debug_tc_mma_rate: N %d outside the form's range", n);
  void* d = nullptr;
  AH_CUDA_TRY(ah::dev_malloc(&d, 4 * sizeof(long long)));
  int rc = AH_OK;
  cudaError_t e = cudaFuncSetAttribute(ah::k_probe_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, ah::kProbeSmem);
  if (e == cudaSuccess) {
    ah::k_probe_mma<<<2, 128, ah::kProbeSmem>>>(static_cast<long long*>(d), n, mode);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(out_host, d, 3 * sizeof(long long), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) rc = ah::fail(AH_ECUDA, "ah_debug_tc_mma_rate: %s", cudaGetErrorString(e));
  cudaFree(d);
  return rc;
}

}  // extern "C"
