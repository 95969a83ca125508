// ah_sample.cu — temperature + top-k sampling of the next token on the device
// (inference/sampling.rs:17-64, called by generate with top_k 40 whenever the
// temperature is above 0, inference/mod.rs:552-553).
//
// Per sequence (one CTA of 1024 threads over its logits row):
//   1. the top-k logits by a radix select on order-preserving integer keys
//      (four 8-bit digit passes, histograms in shared memory with warp-
//      aggregated atomics), ties at the threshold taken in index order, the
//      candidates sorted by (value descending, index ascending);
//   2. the reference's arithmetic in its order over the sorted candidates:
//      p_i = exp((v_i - max) / T), sum, then the CDF scan cdf += p_i / sum
//      against a uniform r in [0, 1) with 24 random bits.
// The reference draws r from a clock-seeded xorshift; here r comes from a
// counter-based hash of (seed, step, sequence), so a run is reproducible and
// the oracle can be given the same r.  Top-k by logit equals the reference's
// top-k by probability (exp is monotone) except where distinct logits give
// equal probabilities, whose order the reference leaves unspecified.
//
// Under tensor parallelism each rank's CTA selects the top-k of its vocab
// slice (global indices), the candidates are all-gathered, and k_sample_merge
// ranks the W * k candidates and samples: every rank picks the same token.
#include <cfloat>
#include <climits>

#include "ah_common.cuh"
#include "ah_sample.cuh"
#include "ah_sm100.cuh"

namespace ah {

__host__ __device__ uint64_t sample_mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__host__ __device__ float sample_uniform(uint64_t seed, int64_t step, int seq) {
  const uint64_t x = sample_mix64(seed ^ sample_mix64((uint64_t)step * 0x100000001B3ull + (uint64_t)seq));
  return (float)(x & 0xFFFFFFull) / 16777216.0f;  // 24 bits, as the reference maps its draw
}

namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleUnroll = 8;  // loads in flight per thread per sweep
constexpr int kSampleSweep = kSampleThreads * kSampleUnroll;

// Larger float -> larger key; -0 and +0 share a key; NaN maps below every
// number (never a candidate ahead of a number).
__device__ __forceinline__ uint32_t order_key(float v) {
  if (v != v) return 0u;
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// (key desc, index asc): a strict order for distinct indices
__device__ __forceinline__ bool cand_before(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Warp 0: the bin of hist[0..256) (descending) where the count of keys
// reaches `remaining`; misc[0] = bin, misc[1] = remaining left inside it,
// misc[4] = the bin's count.  The bins hold at least `remaining` keys.
__device__ __forceinline__ void find_bin(const int* hist, int remaining, int* misc) {
  const int lane = threadIdx.x & 31;
  int c[8], s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c[j] = hist[255 - 8 * lane - j];
    s += c[j];
  }
  int x = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  int cum = x - s;  // keys in the bins above this lane's eight
  if (cum < remaining && remaining <= x) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (cum >= 0 && cum + c[j] >= remaining) {
        misc[0] = 255 - 8 * lane - j;
        misc[1] = remaining - cum;
        misc[4] = c[j];
        cum = -1 - (1 << 30);  // found: stop
      } else if (cum >= 0) {
        cum += c[j];
      }
    }
  }
}

// The k largest of row[0 .. n) (k <= kSampleMaxK, k <= n) into cv / ci sorted
// by (value desc, index asc); global index = local + idx_base.  Whole-CTA.
__device__ void topk_row(const float* __restrict__ row, int64_t n, int k, int64_t idx_base, float* cv, int* ci,
                         int* hist, int* misc) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t prefix = 0, pmask = 0;
  int remaining = k;
  for (int digit = 3; digit >= 0; --digit) {
    for (int i = tid; i < 256; i += kSampleThreads) hist[i] = 0;
    __syncthreads();
    const int sh = digit * 8;
    for (int64_t i0 = 0; i0 < n; i0 += kSampleSweep) {
      float v[kSampleUnroll];
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        const int64_t i = i0 + (int64_t)u * kSampleThreads + tid;
        v[u] = i < n ? __ldg(row + i) : __int_as_float(0x7FC00000);
      }
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        const int64_t i = i0 + (int64_t)u * kSampleThreads + tid;
        int bin = -1;
        if (i < n) {
          const uint32_t key = order_key(v[u]);
          if ((key & pmask) == prefix) bin = (int)((key >> sh) & 0xFFu);
        }
        // warp-aggregated: one atomic per distinct bin of the warp
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, bin);
        if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
      }
    }
    __syncthreads();
    if (tid < 32) find_bin(hist, remaining, misc);
    __syncthreads();
    prefix |= (uint32_t)misc[0] << sh;
    pmask |= 0xFFu << sh;
    remaining = misc[1];
    __syncthreads();
  }
  // prefix is the k-th largest key: every key above it, then `remaining`
  // keys equal to it -- all of them when that is how many there are (the
  // usual case), else the first in index order
  const bool all_ties = misc[4] == remaining;
  __syncthreads();
  if (tid == 0) {
    misc[2] = 0;  // slots taken above the threshold
    misc[3] = 0;  // slots taken at the threshold
  }
  __syncthreads();
  const int k_above = k - remaining;
  if (all_ties) {
    for (int64_t i0 = 0; i0 < n; i0 += kSampleSweep) {
      float v[kSampleUnroll];
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        const int64_t i = i0 + (int64_t)u * kSampleThreads + tid;
        v[u] = i < n ? __ldg(row + i) : __int_as_float(0x7FC00000);
      }
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        const int64_t i = i0 + (int64_t)u * kSampleThreads + tid;
        const uint32_t key = order_key(v[u]);
        if (i < n && key >= prefix) {
          const int slot = key > prefix ? atomicAdd(&misc[2], 1) : k_above + atomicAdd(&misc[3], 1);
          cv[slot] = v[u];
          ci[slot] = (int)(i + idx_base);
        }
      }
    }
  } else {
    for (int64_t i0 = 0; i0 < n; i0 += kSampleThreads) {
      const int64_t i = i0 + tid;
      bool above = false, at = false;
      float v = 0.0f;
      if (i < n) {
        v = row[i];
        const uint32_t key = order_key(v);
        above = key > prefix;
        at = key == prefix;
      }
      if (above) {
        const int slot = atomicAdd(&misc[2], 1);
        cv[slot] = v;
        ci[slot] = (int)(i + idx_base);
      }
      // ordered: a block-wide exclusive scan of the tie flags of this slice
      const unsigned tie = __ballot_sync(0xFFFFFFFFu, at);
      if (lane == 0) hist[tid >> 5] = __popc(tie);
      __syncthreads();
      if (tid < 32) {
        const int c = hist[tid];
        int x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
          if (lane >= o) x += y;
        }
        hist[32 + tid] = x - c;  // exclusive offset of warp tid
        if (tid == 31) hist[64] = x;
      }
      __syncthreads();
      if (at) {
        const int r = misc[3] + hist[32 + (tid >> 5)] + __popc(tie & ((1u << lane) - 1u));
        if (r < remaining) {
          cv[k_above + r] = v;
          ci[k_above + r] = (int)(i + idx_base);
        }
      }
      __syncthreads();
      if (tid == 0) misc[3] += hist[64];
      __syncthreads();
      if (misc[3] >= remaining && misc[2] >= k_above) break;  // every slot taken
    }
  }
  __syncthreads();
  // rank sort of the k candidates: (value desc, index asc)
  float v = 0.0f;
  int ix = 0, rank = 0;
  if (tid < k) {
    v = cv[tid];
    ix = ci[tid];
    const uint32_t key = order_key(v);
    for (int j = 0; j < k; ++j) rank += cand_before(order_key(cv[j]), ci[j], key, ix) ? 1 : 0;
  }
  __syncthreads();
  if (tid < k) {
    cv[rank] = v;
    ci[rank] = ix;
  }
  __syncthreads();
}

// sampling.rs:17-64 over k sorted candidates (thread 0)
__device__ int sample_sorted(const float* cv, const int* ci, int k, float temperature, float r) {
  const float max_logit = cv[0];
  const float inv_temp = 1.0f / temperature;
  float sum = 0.0f;
  for (int j = 0; j < k; ++j) sum += expf((cv[j] - max_logit) * inv_temp);
  if (sum == 0.0f) return ci[0];
  const float inv = 1.0f / sum;
  float cdf = 0.0f;
  for (int j = 0; j < k; ++j) {
    cdf += expf((cv[j] - max_logit) * inv_temp) * inv;
    if (r < cdf) return ci[j];
  }
  return ci[k - 1];
}

// One CTA per sequence: local top-k of its logits row; with `cand` null it
// samples and writes the token, else it writes the sorted candidates.
__global__ void __launch_bounds__(kSampleThreads) k_sample_topk(const float* __restrict__ logits, int64_t ld,
                                                                int64_t n, int k, int64_t idx_base, float temperature,
                                                                uint64_t seed, int64_t step, const int* step_dev,
                                                                SampleCand* cand, int* tok, int* tok_log, int batch) {
  __shared__ float cv[kSampleMaxK];
  __shared__ int ci[kSampleMaxK];
  __shared__ int hist[256];
  __shared__ int misc[5];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const int ke = (int)(k < n ? k : n);
  topk_row(logits + (size_t)b * ld, n, ke, idx_base, cv, ci, hist, misc);
  if (threadIdx.x != 0) return;
  if (cand) {
    for (int j = 0; j < k; ++j)
      cand[(size_t)b * k + j] = j < ke ? SampleCand{cv[j], ci[j]} : SampleCand{-INFINITY, INT_MAX};
    return;
  }
  const int64_t st = step_dev ? (int64_t)*step_dev : step;
  const int next = sample_sorted(cv, ci, ke, temperature, sample_uniform(seed, st, b));
  tok[b] = next;
  if (tok_log) tok_log[(size_t)st * batch + b] = next;
}

// The W ranks' k candidates per sequence ([W][B][k]) -> the global top-k,
// then the sample (one CTA of 256 threads per sequence).
__global__ void __launch_bounds__(256) k_sample_merge(const SampleCand* __restrict__ all, int world, int batch, int k,
                                                      float temperature, uint64_t seed, const int* step_dev,
                                                      int* tok, int* tok_log) {
  __shared__ float cv[kSampleMaxK];
  __shared__ int ci[kSampleMaxK];
  __shared__ SampleCand sc[kSampleMaxRanks * kSampleMaxK];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const int m = world * k;
  for (int i = threadIdx.x; i < m; i += blockDim.x) sc[i] = all[((size_t)(i / k) * batch + b) * k + (i % k)];
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    const SampleCand c = sc[i];
    const uint32_t key = order_key(c.v);
    int rank = 0;
    for (int j = 0; j < m; ++j) rank += cand_before(order_key(sc[j].v), sc[j].i, key, c.i) ? 1 : 0;
    if (rank < k) {
      cv[rank] = c.v;
      ci[rank] = c.i;
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  int ke = 0;
  while (ke < k && ci[ke] != INT_MAX) ++ke;
  const int64_t st = *step_dev;
  const int next = ke == 0 ? 0 : sample_sorted(cv, ci, ke, temperature, sample_uniform(seed, st, b));
  tok[b] = next;
  tok_log[(size_t)st * batch + b] = next;
}

}  // namespace

int sample_launch(const float* logits, int64_t ld, int batch, int64_t n, int k, int64_t idx_base, float temperature,
                  uint64_t seed, int64_t step, const int* step_dev, SampleCand* cand, int* tok, int* tok_log,
                  cudaStream_t st, bool pdl) {
  AH_REQUIRE(batch >= 1 && n >= 1 && ld >= n, "sample: bad shape");
  AH_REQUIRE(k >= 1 && k <= kSampleMaxK, "sample: top_k must be 1..%d", kSampleMaxK);
  AH_REQUIRE(cand || temperature > 0.0f, "sample: temperature must be above 0");
  AH_REQUIRE(n <= (int64_t)INT_MAX - idx_base, "sample: vocabulary too large");
  return launch_pdl(k_sample_topk, dim3((unsigned)batch), dim3(kSampleThreads), 0, st, logits, ld, n, k, idx_base,
                    temperature, seed, step, step_dev, cand, tok, tok_log, batch);
}

int sample_merge_launch(const SampleCand* all, int world, int batch, int k, float temperature, uint64_t seed,
                        const int* step_dev, int* tok, int* tok_log, cudaStream_t st) {
  AH_REQUIRE(world >= 1 && world <= kSampleMaxRanks && k >= 1 && k <= kSampleMaxK, "sample merge: bad shape");
  return launch_pdl(k_sample_merge, dim3((unsigned)batch), dim3(256), 0, st, all, world, batch, k, temperature, seed,
                    step_dev, tok, tok_log);
}

}  // namespace ah

extern "C" {

AH_API int ah_sample_logits(const float* logits_dev, int64_t ld, int batch, int64_t vocab, float temperature,
                            int top_k, uint64_t seed, int64_t step, int32_t* out_dev, void* stream) {
  AH_REQUIRE(logits_dev && out_dev, "ah_sample_logits: null pointer");
  AH_REQUIRE(temperature > 0.0f, "ah_sample_logits: temperature must be above 0 (0 is greedy: take the argmax)");
  return ah::sample_launch(logits_dev, ld, batch, vocab, top_k, 0, temperature, seed, step, nullptr, nullptr,
                           out_dev, nullptr, ah::as_stream(stream), false);
}

AH_API float ah_sample_uniform(uint64_t seed, int64_t step, int seq) { return ah::sample_uniform(seed, step, seq); }

}  // extern "C"
