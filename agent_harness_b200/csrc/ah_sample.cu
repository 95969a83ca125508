// ah_sample.cu — temperature + top-k sampling of the next token on the device
// (inference/sampling.rs:17-64, called by generate with top_k 40 whenever the
// temperature is above 0, inference/mod.rs:552-553).
//
// Per sequence:
//   1. the top-k logits by a radix select on order-preserving integer keys
//      (four 8-bit digit passes, histograms in shared memory, the lanes
//      sharing lane 0's bin counted by one ballot), ties at the threshold
//      taken in index order, the candidates sorted by (value descending,
//      index ascending).  With a
//      workspace the row is split into slices of kSampleSlice logits, one CTA
//      each (k_sample_part), and one CTA per row selects the top-k of the
//      slices' candidates (k_sample_reduce); without one, one CTA walks the
//      whole row (k_sample_topk);
//   2. the reference's arithmetic in its order over the sorted candidates:
//      p_i = exp((v_i - max) / T), sum, then the CDF scan cdf += p_i / sum
//      against a uniform r in [0, 1) with 24 random bits.
// The reference draws r from a clock-seeded xorshift; here r comes from a
// counter-based hash of (seed, step, sequence), so a run is reproducible and
// the oracle can be given the same r.  Top-k by logit equals the reference's
// top-k by probability (exp is monotone) except where distinct logits give
// equal probabilities, whose order the reference leaves unspecified.
//
// Under tensor parallelism each rank selects the top-k of its vocab slice
// (global indices), the candidates are all-gathered, and k_sample_merge ranks
// the W * k candidates and samples: every rank picks the same token.
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

constexpr int kSampleThreads = 1024;  // whole-row CTAs
constexpr int kPartThreads = 512;     // slice CTAs
constexpr int kReduceThreads = 256;   // CTAs over a row's slice candidates
constexpr int kSampleUnroll = 8;      // loads in flight per thread per sweep
constexpr int kMergeParts = 64;       // slices per row the reduce merges as sorted lists

// Larger float -> larger key; -0 and +0 share a key; NaN maps below every
// number (never a candidate ahead of a number).
__device__ __forceinline__ uint32_t order_key(float v) {
  if (v != v) return 0u;
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// The value of a key (-0 comes back as +0, NaN as a NaN).
__device__ __forceinline__ float key_value(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// (key desc, index asc): a strict order for distinct indices
__device__ __forceinline__ bool cand_before(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Shared state of a top-k: two histograms (passes alternate), two sets of
// pass results, the candidates, their probabilities.
struct TopkSmem {
  int hist[2][256];
  int pass[2][4];  // bin, remaining inside it, the bin's count
  int slots[2];    // slots taken above / at the threshold
  float cv[kSampleMaxK];
  int ci[kSampleMaxK];
  float pv[kSampleMaxK];
};

// Warp 0: the bin of hist[0..256) (descending) where the count of keys
// reaches `remaining`; out[0] = bin, out[1] = remaining left inside it,
// out[2] = the bin's count.  The bins hold at least `remaining` keys.
__device__ __forceinline__ void find_bin(const int* hist, int remaining, int* out) {
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
    bool found = false;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (!found && cum + c[j] >= remaining) {
        out[0] = 255 - 8 * lane - j;
        out[1] = remaining - cum;
        out[2] = c[j];
        found = true;
      }
      cum += c[j];
    }
  }
}

// The k largest of row[0 .. n) (1 <= k <= kSampleMaxK, k <= n) into sm.cv /
// sm.ci sorted by (value desc, index asc); index = local + idx_base.  Whole CTA
// of kT threads.  kRes > 0: the row (at most kRes sweeps of kT *
// kSampleUnroll values) is read once into registers as keys; 0: every pass
// reads it again (from L2 after the first).
template <int kT, int kRes>
__device__ void topk_row(const float* __restrict__ row, int64_t n, int k, int64_t idx_base, TopkSmem& sm) {
  constexpr int kSweep = kT * kSampleUnroll;
  constexpr int kWarps = kT / 32;
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t kr[kRes > 0 ? kRes : 1][kSampleUnroll];
  if constexpr (kRes > 0) {
#pragma unroll
    for (int r = 0; r < kRes; ++r)
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        const int64_t i = (int64_t)r * kSweep + u * kT + tid;
        kr[r][u] = i < n ? order_key(__ldg(row + i)) : 0u;
      }
  }
  // fn(i, key) for each of this thread's elements (i may be >= n), every
  // lane of the warp together; rounds wholly past n are skipped
  auto each = [&](auto&& fn) {
    if constexpr (kRes > 0) {
#pragma unroll
      for (int r = 0; r < kRes; ++r)
#pragma unroll
        for (int u = 0; u < kSampleUnroll; ++u) {
          const int64_t base = (int64_t)r * kSweep + u * kT;
          if (base < n) fn(base + tid, kr[r][u]);
        }
    } else {
      for (int64_t i0 = 0; i0 < n; i0 += kSweep) {
        float v[kSampleUnroll];
#pragma unroll
        for (int u = 0; u < kSampleUnroll; ++u) {
          const int64_t i = i0 + (int64_t)u * kT + tid;
          v[u] = i < n ? __ldg(row + i) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kSampleUnroll; ++u) {
          const int64_t base = i0 + (int64_t)u * kT;
          if (base < n) fn(base + tid, order_key(v[u]));
        }
      }
    }
  };
  for (int i = tid; i < 2 * 256; i += kT) (&sm.hist[0][0])[i] = 0;
  if (tid < 2) sm.slots[tid] = 0;
  __syncthreads();
  uint32_t prefix = 0, pmask = 0;
  int remaining = k, tie_count = 0;
#pragma unroll 1
  for (int q = 0; q < 4; ++q) {
    const int sh = (3 - q) * 8;
    int* h = sm.hist[q & 1];
    each([&](int64_t i, uint32_t key) {
      const int bin = (i < n && (key & pmask) == prefix) ? (int)((key >> sh) & 0xFFu) : -1;
      // lane 0's bin (usually the warp's commonest: the leading digits of
      // neighbouring logits agree) with one atomic for all its lanes; the
      // other lanes' bins one atomic each
      const int lead = __shfl_sync(0xFFFFFFFFu, bin, 0);
      const unsigned same = __ballot_sync(0xFFFFFFFFu, bin == lead);
      if (lane == 0 && lead >= 0) atomicAdd(&h[lead], __popc(same));
      if (bin >= 0 && bin != lead) atomicAdd(&h[bin], 1);
    });
    __syncthreads();
    if (tid < 32) find_bin(h, remaining, sm.pass[q & 1]);
    // the other histogram was last read by the previous pass's search
    int* h2 = sm.hist[(q + 1) & 1];
    for (int i = tid; i < 256; i += kT) h2[i] = 0;
    __syncthreads();
    prefix |= (uint32_t)sm.pass[q & 1][0] << sh;
    pmask |= 0xFFu << sh;
    remaining = sm.pass[q & 1][1];
    tie_count = sm.pass[q & 1][2];
  }
  // prefix is the k-th largest key: every key above it, then `remaining`
  // keys equal to it -- all of them when that is how many there are (the
  // usual case), else the first in index order
  const int k_above = k - remaining;
  if (tie_count == remaining) {
    each([&](int64_t i, uint32_t key) {
      if (i < n && key >= prefix) {
        const int slot = key > prefix ? atomicAdd(&sm.slots[0], 1) : k_above + atomicAdd(&sm.slots[1], 1);
        sm.cv[slot] = key_value(key);
        sm.ci[slot] = (int)(i + idx_base);
      }
    });
  } else {
    int* scan = sm.hist[0];  // the histograms are done with
    for (int64_t i0 = 0; i0 < n; i0 += kT) {
      const int64_t i = i0 + tid;
      uint32_t key = 0;
      bool above = false, at = false;
      if (i < n) {
        key = order_key(row[i]);
        above = key > prefix;
        at = key == prefix;
      }
      if (above) {
        const int slot = atomicAdd(&sm.slots[0], 1);
        sm.cv[slot] = key_value(key);
        sm.ci[slot] = (int)(i + idx_base);
      }
      // ordered: a block-wide exclusive scan of the tie flags of this slice
      const unsigned tie = __ballot_sync(0xFFFFFFFFu, at);
      if (lane == 0) scan[tid >> 5] = __popc(tie);
      __syncthreads();
      if (tid < 32) {
        const int c = tid < kWarps ? scan[tid] : 0;
        int x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
          if (lane >= o) x += y;
        }
        scan[32 + tid] = x - c;  // exclusive offset of warp tid
        if (tid == 31) scan[64] = x;
      }
      __syncthreads();
      if (at) {
        const int r = sm.slots[1] + scan[32 + (tid >> 5)] + __popc(tie & ((1u << lane) - 1u));
        if (r < remaining) {
          sm.cv[k_above + r] = key_value(key);
          sm.ci[k_above + r] = (int)(i + idx_base);
        }
      }
      __syncthreads();
      if (tid == 0) sm.slots[1] += scan[64];
      __syncthreads();
      if (sm.slots[1] >= remaining && sm.slots[0] >= k_above) break;  // every slot taken
    }
  }
  __syncthreads();
  // rank sort of the k candidates: (value desc, index asc)
  float v = 0.0f;
  int ix = 0, rank = 0;
  if (tid < k) {
    v = sm.cv[tid];
    ix = sm.ci[tid];
    const uint32_t key = order_key(v);
#pragma unroll 8
    for (int j = 0; j < k; ++j) rank += cand_before(order_key(sm.cv[j]), sm.ci[j], key, ix) ? 1 : 0;
  }
  __syncthreads();
  if (tid < k) {
    sm.cv[rank] = v;
    sm.ci[rank] = ix;
  }
  __syncthreads();
}

// sampling.rs:17-64 over k sorted candidates (whole CTA; the pick is valid
// in thread 0): p_j = exp((v_j - max) / T) in parallel, then the sum and the
// CDF scan in the reference's order.
__device__ int sample_pick(TopkSmem& sm, int k, float temperature, float r) {
  const float max_logit = sm.cv[0];
  const float inv_temp = 1.0f / temperature;
  if ((int)threadIdx.x < k) sm.pv[threadIdx.x] = expf((sm.cv[threadIdx.x] - max_logit) * inv_temp);
  __syncthreads();
  if (threadIdx.x != 0) return 0;
  float sum = 0.0f;
  for (int j = 0; j < k; ++j) sum += sm.pv[j];
  if (sum == 0.0f) return sm.ci[0];
  const float inv = 1.0f / sum;
  float cdf = 0.0f;
  for (int j = 0; j < k; ++j) {
    cdf += sm.pv[j] * inv;
    if (r < cdf) return sm.ci[j];
  }
  return sm.ci[k - 1];
}

// Whole CTA, after the top-k of row b (ke <= k entries): either the k
// candidates to `cand` (no candidate: -inf, INT_MAX), or the sample to
// tok[b] and tok_log[step * batch + b].
__device__ void sample_finish(TopkSmem& sm, int ke, int k, int b, float temperature, uint64_t seed, int64_t step,
                              const int* step_dev, SampleCand* cand, int* tok, int* tok_log, int batch) {
  const int t = threadIdx.x;
  if (cand) {
    if (t < k) cand[(size_t)b * k + t] = t < ke ? SampleCand{sm.cv[t], sm.ci[t]} : SampleCand{-INFINITY, INT_MAX};
    return;
  }
  const int64_t st = step_dev ? (int64_t)*step_dev : step;
  const int next = sample_pick(sm, ke, temperature, sample_uniform(seed, st, b));
  if (t == 0) {
    tok[b] = next;
    if (tok_log) tok_log[(size_t)st * batch + b] = next;
  }
}

// One CTA per sequence over its whole row.
__global__ void __launch_bounds__(kSampleThreads) k_sample_topk(const float* __restrict__ logits, int64_t ld,
                                                                int64_t n, int k, int64_t idx_base, float temperature,
                                                                uint64_t seed, int64_t step, const int* step_dev,
                                                                SampleCand* cand, int* tok, int* tok_log, int batch) {
  __shared__ TopkSmem sm;
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const int ke = (int)(k < n ? k : n);
  topk_row<kSampleThreads, 0>(logits + (size_t)b * ld, n, ke, idx_base, sm);
  sample_finish(sm, ke, k, b, temperature, seed, step, step_dev, cand, tok, tok_log, batch);
}

// Slice p of row b (blockIdx.x = p, blockIdx.y = b): its top-k to
// part_v / part_i [b][p][k].  Slices hold kSampleSlice logits, the last one
// the rest as well (fewer than 2 * kSampleSlice), so each has >= k.
__global__ void __launch_bounds__(kPartThreads) k_sample_part(const float* __restrict__ logits, int64_t ld, int64_t n,
                                                              int k, int64_t idx_base, float* part_v, int* part_i) {
  __shared__ TopkSmem sm;
  pdl_launch_dependents();
  pdl_wait();
  const int p = blockIdx.x, b = blockIdx.y, parts = gridDim.x;
  const int64_t lo = (int64_t)p * kSampleSlice;
  const int64_t len = p == parts - 1 ? n - lo : kSampleSlice;
  topk_row<kPartThreads, 2>(logits + (size_t)b * ld + lo, len, k, idx_base + lo, sm);
  const int t = threadIdx.x;
  if (t < k) {
    const size_t o = ((size_t)b * parts + p) * k + t;
    part_v[o] = sm.cv[t];
    part_i[o] = sm.ci[t];
  }
}

// Warp 0: the top ke of the parts' sorted candidate lists (mv / mi [p][k],
// each sorted by (value desc, index asc), parts <= 2 * 32) by a k-way merge:
// lane l holds the heads of lists l and l + 32, and each step a butterfly
// over the lanes picks the winner, which its list's lane replaces by the
// list's next entry.  The result is sorted, as topk_row's.
__device__ void merge_lists(const float* mv, const int* mi, int parts, int k, int ke, TopkSmem& sm) {
  const int lane = threadIdx.x & 31;
  int pos0 = 0, pos1 = 0;
  uint32_t k0 = 0u, k1 = 0u;
  int i0 = INT_MAX, i1 = INT_MAX;  // exhausted lists: (key 0, index INT_MAX) loses to every entry
  const int p0 = lane, p1 = lane + 32;
  if (p0 < parts) {
    k0 = order_key(mv[p0 * k]);
    i0 = mi[p0 * k];
  }
  if (p1 < parts) {
    k1 = order_key(mv[p1 * k]);
    i1 = mi[p1 * k];
  }
  for (int j = 0; j < ke; ++j) {
    const bool second = cand_before(k1, i1, k0, i0);
    uint32_t bk = second ? k1 : k0;
    int bi = second ? i1 : i0;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const uint32_t ok = __shfl_xor_sync(0xFFFFFFFFu, bk, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (cand_before(ok, oi, bk, bi)) {
        bk = ok;
        bi = oi;
      }
    }
    if (lane == 0) {
      sm.cv[j] = key_value(bk);
      sm.ci[j] = bi;
    }
    // vocabulary indices are distinct: only the winner's list moves
    if (bi != INT_MAX) {
      if (!second && i0 == bi) {
        ++pos0;
        k0 = pos0 < k ? order_key(mv[p0 * k + pos0]) : 0u;
        i0 = pos0 < k ? mi[p0 * k + pos0] : INT_MAX;
      } else if (second && i1 == bi) {
        ++pos1;
        k1 = pos1 < k ? order_key(mv[p1 * k + pos1]) : 0u;
        i1 = pos1 < k ? mi[p1 * k + pos1] : INT_MAX;
      }
    }
  }
}

// Row b's parts * k slice candidates -> its top-k (position order among equal
// values is index order: slices ascend, each sorted), then the sample or the
// candidates as k_sample_topk.  Up to kMergeParts slices: staged in shared
// memory and merged by one warp; more: a radix select over them.
__global__ void __launch_bounds__(kReduceThreads) k_sample_reduce(const float* __restrict__ part_v,
                                                                  const int* __restrict__ part_i, int parts, int k,
                                                                  int64_t n, float temperature, uint64_t seed,
                                                                  int64_t step, const int* step_dev, SampleCand* cand,
                                                                  int* tok, int* tok_log, int batch) {
  __shared__ TopkSmem sm;
  __shared__ float mv[kMergeParts * kSampleMaxK];
  __shared__ int mi[kMergeParts * kSampleMaxK];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const int64_t m = (int64_t)parts * k;
  const int ke = (int)(k < n ? k : n);
  if (parts <= kMergeParts) {
    for (int i = threadIdx.x; i < (int)m; i += kReduceThreads) {
      mv[i] = part_v[(size_t)b * m + i];
      mi[i] = part_i[(size_t)b * m + i];
    }
    __syncthreads();
    if (threadIdx.x < 32) merge_lists(mv, mi, parts, k, ke, sm);
  } else {
    if (m <= 2 * kReduceThreads * kSampleUnroll)
      topk_row<kReduceThreads, 2>(part_v + (size_t)b * m, m, ke, 0, sm);
    else
      topk_row<kReduceThreads, 0>(part_v + (size_t)b * m, m, ke, 0, sm);
    if ((int)threadIdx.x < ke) sm.ci[threadIdx.x] = part_i[(size_t)b * m + sm.ci[threadIdx.x]];
  }
  __syncthreads();
  sample_finish(sm, ke, k, b, temperature, seed, step, step_dev, cand, tok, tok_log, batch);
}

// The W ranks' k candidates per sequence ([W][B][k]) -> the global top-k,
// then the sample (one CTA of 256 threads per sequence).
__global__ void __launch_bounds__(256) k_sample_merge(const SampleCand* __restrict__ all, int world, int batch, int k,
                                                      float temperature, uint64_t seed, const int* step_dev,
                                                      int* tok, int* tok_log) {
  __shared__ TopkSmem sm;
  __shared__ SampleCand sc[kSampleMaxRanks * kSampleMaxK];
  __shared__ int n_real;
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
      sm.cv[rank] = c.v;
      sm.ci[rank] = c.i;
    }
  }
  __syncthreads();
  // the entries without a vocabulary index (a rank's slice shorter than k)
  // share one rank behind every number: the candidates end at the first
  if (threadIdx.x == 0) {
    int e = 0;
    while (e < k && sm.ci[e] != INT_MAX) ++e;
    n_real = e;
  }
  __syncthreads();
  const int ke = n_real;
  const int64_t st = *step_dev;
  const int next = ke == 0 ? 0 : sample_pick(sm, ke, temperature, sample_uniform(seed, st, b));
  if (threadIdx.x == 0) {
    tok[b] = next;
    tok_log[(size_t)st * batch + b] = next;
  }
}

// slices of a split row (fewer than 2: one CTA per row)
int64_t sample_parts(int64_t n) { return n / kSampleSlice; }

}  // namespace

size_t sample_workspace_bytes(int batch, int64_t n) {
  const int64_t parts = sample_parts(n);
  if (parts <= 1 || batch < 1) return 0;
  return (size_t)batch * (size_t)parts * kSampleMaxK * (sizeof(float) + sizeof(int));
}

int sample_launch(const float* logits, int64_t ld, int batch, int64_t n, int k, int64_t idx_base, float temperature,
                  uint64_t seed, int64_t step, const int* step_dev, SampleCand* cand, int* tok, int* tok_log,
                  void* ws, size_t ws_bytes, cudaStream_t st) {
  AH_REQUIRE(batch >= 1 && n >= 1 && ld >= n, "sample: bad shape");
  AH_REQUIRE(batch <= 65535 || !ws, "sample: more than 65535 rows with a workspace");
  AH_REQUIRE(k >= 1 && k <= kSampleMaxK, "sample: top_k must be 1..%d", kSampleMaxK);
  AH_REQUIRE(cand || temperature > 0.0f, "sample: temperature must be above 0");
  AH_REQUIRE(idx_base >= 0 && n <= (int64_t)INT_MAX - idx_base, "sample: vocabulary too large");
  const int64_t parts = sample_parts(n);
  if (!ws || parts <= 1) {
    return launch_pdl(k_sample_topk, dim3((unsigned)batch), dim3(kSampleThreads), 0, st, logits, ld, n, k,
                      idx_base, temperature, seed, step, step_dev, cand, tok, tok_log, batch);
  }
  const size_t need = (size_t)batch * (size_t)parts * (size_t)k * (sizeof(float) + sizeof(int));
  AH_REQUIRE(ws_bytes >= need, "sample: workspace of %zu bytes, %zu needed", ws_bytes, need);
  AH_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 15) == 0, "sample: workspace must be 16-byte aligned");
  float* part_v = static_cast<float*>(ws);
  int* part_i = reinterpret_cast<int*>(part_v + (size_t)batch * parts * k);
  if (launch_pdl(k_sample_part, dim3((unsigned)parts, (unsigned)batch), dim3(kPartThreads), 0, st, logits, ld, n, k,
                 idx_base, part_v, part_i) != AH_OK)
    return AH_ECUDA;
  return launch_pdl(k_sample_reduce, dim3((unsigned)batch), dim3(kReduceThreads), 0, st, (const float*)part_v,
                    (const int*)part_i, (int)parts, k, n, temperature, seed, step, step_dev, cand, tok, tok_log,
                    batch);
}

int sample_merge_launch(const SampleCand* all, int world, int batch, int k, float temperature, uint64_t seed,
                        const int* step_dev, int* tok, int* tok_log, cudaStream_t st) {
  AH_REQUIRE(world >= 1 && world <= kSampleMaxRanks && k >= 1 && k <= kSampleMaxK, "sample merge: bad shape");
  return launch_pdl(k_sample_merge, dim3((unsigned)batch), dim3(256), 0, st, all, world, batch, k, temperature, seed,
                    step_dev, tok, tok_log);
}

}  // namespace ah

extern "C" {

AH_API size_t ah_sample_workspace_bytes(int batch, int64_t vocab) { return ah::sample_workspace_bytes(batch, vocab); }

AH_API int ah_sample_logits(const float* logits_dev, int64_t ld, int batch, int64_t vocab, float temperature,
                            int top_k, uint64_t seed, int64_t step, int32_t* out_dev, void* workspace,
                            size_t workspace_bytes, void* stream) {
  AH_REQUIRE(logits_dev && out_dev, "ah_sample_logits: null pointer");
  AH_REQUIRE(temperature > 0.0f, "ah_sample_logits: temperature must be above 0 (0 is greedy: take the argmax)");
  return ah::sample_launch(logits_dev, ld, batch, vocab, top_k, 0, temperature, seed, step, nullptr, nullptr,
                           out_dev, nullptr, workspace, workspace_bytes, ah::as_stream(stream));
}

AH_API float ah_sample_uniform(uint64_t seed, int64_t step, int seq) { return ah::sample_uniform(seed, step, seq); }

}  // extern "C"
