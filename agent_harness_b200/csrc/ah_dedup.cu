// ah_dedup.cu — DedupCount weight decoding (models/dedup/) for sm_100a.
//
// The reference decodes every element as
//   value = prefix + tail / divisor + avg_precision_lost, negated by a sign bit
// where prefix and tail come from per-tensor lookups (decompressor.rs:7-85,
// global_lookup.rs:89-113).  Those lookups are tiny, per-tensor host work, so
// they are flattened here into f32 value tables:
//   local   pre[p] = prefix_int / 10^pd, tl[t] = tail / 10^(pd+td)  (two 1-D tables)
//   global  tab[p][t] = global_prefix[gp(p)] + tails_for_prefix[gp][gt(p,t)] / divisor
//   remap   tab[p][t] = global_prefix[gp(p)] + tails_for_prefix[gp][remap[t]] / divisor
// each with one extra fallback row / column that reproduces the reference's
// `.get(i).copied().unwrap_or(0)` for out-of-range indices.  The device side is
// then a pure gather, HBM-bound at 2 + 2 + 1/8 bytes in and 4 bytes out per
// element; the table adds are the reference's own f32 operations, in its order.
//
// The load-time path (inference/mod.rs:255-271: decompress, quantise, write)
// runs as one kernel: each warp decodes eight 32-element groups, quantises them
// exactly as quantization.rs:369-404 does, and writes nibbles and f32 scales
// straight into the tiled GEMV layout — no f32 tensor in HBM, 4.75 bytes per
// element in total.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "ah_common.cuh"
#include "ah_gemv_impl.cuh"

#define AH_TRY_DEDUP(expr)      \
  do {                          \
    const int _rc = (expr);     \
    if (_rc != AH_OK) return _rc; \
  } while (0)

struct AhDedupTable {
  int device = 0;
  int mode = 0;          // kLocal, kGlobal, kRemap
  int64_t n_prefix = 0;  // table rows before the fallback row
  int64_t n_tail = 0;    // table columns before the fallback column
  float avg = 0.0f;      // avg_precision_lost
  float* d_pre = nullptr;   // local: [n_prefix + 1]
  float* d_tail = nullptr;  // local: [n_tail + 1]
  float* d_tab = nullptr;   // global / remap: [(n_prefix + 1) * (n_tail + 1)]
};

namespace ah {
namespace {

enum DedupMode : int { kLocal = 0, kGlobal = 1, kRemap = 2 };
constexpr int kThreads = 256;
constexpr int kMaxDigits = 10;                 // 10^n exact in f32 for n <= 10
constexpr int64_t kMaxTableEntries = 1 << 26;  // 256 MB of f32
constexpr int kErrPrefixIndex = kDeviceIndexError | 0x101;  // remap: prefix index past the tensor's prefixes

// 10f32.powi(n), exact for n <= kMaxDigits.
float pow10f_i(int n) {
  float r = 1.0f;
  for (int i = 0; i < n; ++i) r *= 10.0f;
  return r;
}
uint32_t pow10u(int n) {
  uint32_t r = 1;
  for (int i = 0; i < n; ++i) r *= 10u;
  return r;
}
// Rust `f as u32`: saturating, NaN -> 0.
uint32_t sat_u32(float f) {
  if (!(f > 0.0f)) return 0;
  if (f >= 4294967295.0f) return 4294967295u;
  return (uint32_t)f;
}
// First global prefix gi with (g[gi] * scale).round() as u32 == norm (`iter().position`), or -1.
int64_t find_global_prefix(const float* g, int64_t n_gp, float scale, uint32_t norm) {
  for (int64_t gi = 0; gi < n_gp; ++gi)
    if (sat_u32(std::round(g[gi] * scale)) == norm) return gi;
  return -1;
}
uint32_t norm_prefix(uint16_t pv, int scale_diff) {
  return scale_diff > 0 ? (uint32_t)pv * pow10u(scale_diff) : (uint32_t)pv;
}

struct DedupArgs {
  const uint16_t* pidx;  // sandbag.prefix_idx
  const uint16_t* tidx;  // sandbag.tail_idx
  const uint8_t* signs;  // sandbag.sign_bits
  int64_t n_pidx, n_tidx, n_sign;
  const float* pre;  // local tables
  const float* tl;
  const float* tab;  // 2-D table
  int64_t np, nt;    // fallback row / column index
  float avg;
  int* err;
};

// Decode tables larger than this stay in global memory (L1 / L2 gathers);
// smaller ones are staged in shared memory, where a warp's 32 random lookups
// cost a few bank wavefronts instead of one L1 wavefront per distinct sector.
constexpr int kSmemTableBytes = 64 * 1024;

// The value tables a kernel reads: staged in shared memory (kSmem) or global.
struct DedupTables {
  const float* pre;
  const float* tl;
  const float* tab;
};

template <bool k2d, bool kSmem>
__device__ __forceinline__ DedupTables stage_tables(const DedupArgs& a) {
  if (!kSmem) return DedupTables{a.pre, a.tl, a.tab};
  extern __shared__ float dsm[];
  if (k2d) {
    const int64_t n = (a.np + 1) * (a.nt + 1);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dsm[i] = __ldg(a.tab + i);
    __syncthreads();
    return DedupTables{nullptr, nullptr, dsm};
  }
  const int64_t n1 = a.np + 1, n2 = a.nt + 1;
  for (int64_t i = threadIdx.x; i < n1; i += blockDim.x) dsm[i] = __ldg(a.pre + i);
  for (int64_t i = threadIdx.x; i < n2; i += blockDim.x) dsm[n1 + i] = __ldg(a.tl + i);
  __syncthreads();
  return DedupTables{dsm, dsm + n1, nullptr};
}

// value = table lookup + avg_precision_lost, negated when `neg` (bit 0) is set.
// Table indices fit 32 bits: at most 65536 + 1 per side and 2^26 entries.
template <bool k2d>
__device__ __forceinline__ float dedup_value(const DedupArgs& a, const DedupTables& tb, uint32_t p, uint32_t t,
                                             uint32_t neg) {
  const uint32_t pp = min(p, (uint32_t)a.np), tt = min(t, (uint32_t)a.nt);
  const float v = k2d ? tb.tab[pp * (uint32_t)(a.nt + 1) + tt] : __fadd_rn(tb.pre[pp], tb.tl[tt]);
  return __uint_as_float(__float_as_uint(__fadd_rn(v, a.avg)) ^ (neg << 31));  // value += avg; -value
}

__device__ __forceinline__ void unpack4(uint2 u, uint32_t (&o)[4]) {
  o[0] = u.x & 0xFFFFu;
  o[1] = u.x >> 16;
  o[2] = u.y & 0xFFFFu;
  o[3] = u.y >> 16;
}
__device__ __forceinline__ void unpack8(uint4 u, uint32_t (&o)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    o[2 * k] = w[k] & 0xFFFFu;
    o[2 * k + 1] = w[k] >> 16;
  }
}

// decompress_all / _global / _with_remap: one thread per 8 elements (one sign byte).
template <bool k2d, bool kSmem, bool kStrict>
__global__ void __launch_bounds__(kThreads) k_dedup_decompress(const DedupArgs a, int64_t count,
                                                               float* __restrict__ out, int vec) {
  const DedupTables tb = stage_tables<k2d, kSmem>(a);
  const int64_t n8 = (count + 7) / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t g8 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g8 < n8; g8 += stride) {
    const int64_t i0 = g8 * 8;
    uint32_t p[8], t[8];
    if (vec && i0 + 8 <= a.n_pidx) {
      unpack8(ldg_stream_v4(reinterpret_cast<const uint4*>(a.pidx + i0)), p);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) p[k] = i0 + k < a.n_pidx ? a.pidx[i0 + k] : 0u;
    }
    if (vec && i0 + 8 <= a.n_tidx) {
      unpack8(ldg_stream_v4(reinterpret_cast<const uint4*>(a.tidx + i0)), t);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = i0 + k < a.n_tidx ? a.tidx[i0 + k] : 0u;
    }
    const uint32_t sb = g8 < a.n_sign ? a.signs[g8] : 0u;
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      o[k] = dedup_value<k2d>(a, tb, p[k], t[k], (sb >> k) & 1u);
      if (kStrict && i0 + k < count && p[k] >= (uint32_t)a.np) atomicExch(a.err, kErrPrefixIndex);
    }
    if (vec && i0 + 8 <= count) {
      reinterpret_cast<float4*>(out + i0)[0] = make_float4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<float4*>(out + i0)[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (i0 + k < count) out[i0 + k] = o[k];
    }
  }
}

// Decode + quantise + tiled write.  A warp takes row R and blocks b0..b0+7
// (32 elements each); lane 4s+l holds elements 8l..8l+7 of block b0+s.  The
// tiled word t of a 16-row tile packs, for lane (g, t) of the MMA fragment,
// element e = 2t + (pp>>2) + 16(pp&1) + 8((pp>>1)&1) in nibble pp (the layout
// the GEMV reads); for element 8l + j that is word j>>1, nibble
// ((j&1)<<2) | ((l&1)<<1) | (l>>1).  Rows past `rows` and blocks past cols/32
// are written as zero weights (nibble 8, scale 0).  Each warp loads its next
// item's indices before it decodes the current one.
struct Q4wItem {
  uint4 p, t;   // eight prefix / tail indices
  uint32_t sb;  // their sign bits
  bool live;
};

__device__ __forceinline__ Q4wItem q4w_load(const DedupArgs& a, int64_t it, int64_t items, int64_t quads,
                                            int64_t rows, int64_t cols, int sub, int l4) {
  Q4wItem x{};
  if (it >= items) return x;
  const int64_t R = it / quads, b = (it - R * quads) * 8 + sub;
  x.live = R < rows && b < cols / 32;
  if (!x.live) return x;
  const int64_t i0 = R * cols + b * 32 + l4 * 8;
  if (i0 + 8 <= a.n_pidx) {
    x.p = ldg_stream_v4(reinterpret_cast<const uint4*>(a.pidx + i0));
  } else {
    uint32_t v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = i0 + k < a.n_pidx ? a.pidx[i0 + k] : 0u;
    x.p = make_uint4(v[0] | v[1] << 16, v[2] | v[3] << 16, v[4] | v[5] << 16, v[6] | v[7] << 16);
  }
  if (i0 + 8 <= a.n_tidx) {
    x.t = ldg_stream_v4(reinterpret_cast<const uint4*>(a.tidx + i0));
  } else {
    uint32_t v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = i0 + k < a.n_tidx ? a.tidx[i0 + k] : 0u;
    x.t = make_uint4(v[0] | v[1] << 16, v[2] | v[3] << 16, v[4] | v[5] << 16, v[6] | v[7] << 16);
  }
  x.sb = (i0 >> 3) < a.n_sign ? a.signs[i0 >> 3] : 0u;
  return x;
}

template <bool k2d, bool kSmem, bool kStrict>
__global__ void __launch_bounds__(kThreads) k_dedup_q4w(const DedupArgs a, uint32_t* __restrict__ nib,
                                                        float* __restrict__ scales, int64_t rows, int64_t cols,
                                                        int64_t r16, int64_t kp) {
  const DedupTables tb = stage_tables<k2d, kSmem>(a);
  const int lane = threadIdx.x & 31, sub = lane >> 2, l4 = lane & 3;
  const int64_t quads = (2 * kp + 7) / 8;  // 8-block groups per row (blocks past 2 kp are skipped)
  const int64_t items = r16 * 16 * quads;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t it = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  Q4wItem cur = q4w_load(a, it, items, quads, rows, cols, sub, l4);
  for (; it < items; it += warps) {
    const Q4wItem nxt = q4w_load(a, it + warps, items, quads, rows, cols, sub, l4);
    const int64_t R = it / quads, b = (it - R * quads) * 8 + sub;
    float v[8];
    uint32_t p[8], t[8];
    unpack8(cur.p, p);
    unpack8(cur.t, t);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[k] = cur.live ? dedup_value<k2d>(a, tb, p[k], t[k], (cur.sb >> k) & 1u) : 0.0f;
      if (kStrict && cur.live && p[k] >= (uint32_t)a.np) atomicExch(a.err, kErrPrefixIndex);
    }
    // quantise the 32-element group (quantization.rs:369-404): scale = max|w| / 7,
    // q = clamp(round(w * (1 / scale)), -8, 7) + 8
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) m = fmaxf(m, fabsf(v[k]));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
    const float scale = m > 0.0f ? __fdiv_rn(m, 7.0f) : 0.0f;
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    const int pp0 = ((l4 & 1) << 1) | (l4 >> 1);  // nibble of even j; odd j adds 4
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      int q0 = scale > 0.0f ? rust_f32_as_i32(roundf(__fmul_rn(v[2 * k], inv))) : 0;
      int q1 = scale > 0.0f ? rust_f32_as_i32(roundf(__fmul_rn(v[2 * k + 1], inv))) : 0;
      q0 = min(max(q0, -8), 7) + 8;
      q1 = min(max(q1, -8), 7) + 8;
      w[k] = ((uint32_t)q0 << (4 * pp0)) | ((uint32_t)q1 << (4 * (pp0 + 4)));
      w[k] |= __shfl_xor_sync(0xFFFFFFFFu, w[k], 1);
      w[k] |= __shfl_xor_sync(0xFFFFFFFFu, w[k], 2);
    }
    if (b < 2 * kp) {
      const int64_t rt = R >> 4;
      const int r = (int)(R & 15), g = r & 7, half = r >> 3;
      const int64_t tp = rt * kp + (b >> 1);
      const int wi = (int)(b & 1) * 2 + half;
      const uint32_t word = l4 == 0 ? w[0] : l4 == 1 ? w[1] : l4 == 2 ? w[2] : w[3];
      nib[((tp * 32 + g * 4 + l4) * 4) + wi] = word;  // lane l writes word l
      if (l4 == 0) scales[(tp * 8 + g) * 4 + wi] = scale;
    }
    cur = nxt;
  }
}

// Shared-memory bytes of the table staging, or 0 when the tables stay global.
size_t table_smem_bytes(const AhDedupTable* t) {
  const size_t n = t->mode == kLocal ? (size_t)(t->n_prefix + 1) + (size_t)(t->n_tail + 1)
                                     : (size_t)(t->n_prefix + 1) * (size_t)(t->n_tail + 1);
  return n * 4 <= (size_t)kSmemTableBytes ? n * 4 : 0;
}

template <typename K>
int allow_smem(K kern, size_t bytes) {
  AH_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return AH_OK;
}

// The kernel variant for a table: 1-D (local) or 2-D lookups, staged in shared
// memory when small enough, with the prefix-index check only for remap tables.
struct DecompressKernel {
  template <bool k2d, bool kSmem, bool kStrict>
  static auto get() { return k_dedup_decompress<k2d, kSmem, kStrict>; }
};
struct Q4wKernel {
  template <bool k2d, bool kSmem, bool kStrict>
  static auto get() { return k_dedup_q4w<k2d, kSmem, kStrict>; }
};

template <typename KS, bool k2d, bool kSmem, bool kStrict, typename... Args>
int launch_variant(size_t smem, int grid, cudaStream_t st, Args... args) {
  auto kern = KS::template get<k2d, kSmem, kStrict>();
  if (kSmem) AH_TRY_DEDUP(allow_smem(kern, smem));
  kern<<<grid, kThreads, kSmem ? smem : 0, st>>>(args...);
  return AH_OK;
}

template <typename KS, typename... Args>
int launch_table_kernel(const AhDedupTable* t, int grid, cudaStream_t st, Args... args) {
  const size_t smem = table_smem_bytes(t);
  if (t->mode == kLocal)
    return smem ? launch_variant<KS, false, true, false>(smem, grid, st, args...)
                : launch_variant<KS, false, false, false>(smem, grid, st, args...);
  if (t->mode == kGlobal)
    return smem ? launch_variant<KS, true, true, false>(smem, grid, st, args...)
                : launch_variant<KS, true, false, false>(smem, grid, st, args...);
  return smem ? launch_variant<KS, true, true, true>(smem, grid, st, args...)
              : launch_variant<KS, true, false, true>(smem, grid, st, args...);
}

int grid_for(int64_t threads_needed) {
  int64_t g = (threads_needed + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sm_count() * 8;
  return (int)std::max<int64_t>(1, std::min(g, cap));
}

int check_digits(int a, int b) {
  AH_REQUIRE(a >= 0 && b >= 0 && a + b <= kMaxDigits, "dedup: digit counts %d + %d outside 0..%d", a, b,
             kMaxDigits);
  return AH_OK;
}

int upload(AhDedupTable* t, float** dst, const std::vector<float>& src) {
  if (ah::dev_malloc(dst, src.size() * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    *dst = nullptr;
    return fail(AH_ENOMEM, "dedup: cudaMalloc of %zu bytes failed", src.size() * sizeof(float));
  }
  AH_CUDA_TRY(cudaMemcpy(*dst, src.data(), src.size() * sizeof(float), cudaMemcpyHostToDevice));
  (void)t;
  return AH_OK;
}

int finish(AhDedupTable* t, int rc, AhDedupTable** out) {
  if (rc != AH_OK) {
    ah_dedup_table_destroy(t);
    return rc;
  }
  *out = t;
  return AH_OK;
}

DedupArgs make_args(const AhDedupTable* t, const uint16_t* pidx, int64_t n_pidx, const uint16_t* tidx,
                    int64_t n_tidx, const uint8_t* signs, int64_t n_sign) {
  DedupArgs a{};
  a.pidx = pidx;
  a.tidx = tidx;
  a.signs = signs;
  a.n_pidx = pidx ? n_pidx : 0;
  a.n_tidx = tidx ? n_tidx : 0;
  a.n_sign = signs ? n_sign : 0;
  a.pre = t->d_pre;
  a.tl = t->d_tail;
  a.tab = t->d_tab;
  a.np = t->n_prefix;
  a.nt = t->n_tail;
  a.avg = t->avg;
  a.err = device_error_word();
  return a;
}

int check_sandbag(const AhDedupTable* t, int64_t n_pidx, int64_t n_tidx, int64_t n_sign, int64_t count) {
  AH_REQUIRE(count >= 0 && n_pidx >= 0 && n_tidx >= 0 && n_sign >= 0, "dedup: negative length");
  if (t->mode == kRemap)  // the remap path indexes the sandbag directly (global_lookup.rs:96-108)
    AH_REQUIRE(count <= n_pidx && count <= n_tidx && (count + 7) / 8 <= n_sign,
               "dedup: sandbag arrays shorter than count %lld", (long long)count);
  return AH_OK;
}

}  // namespace
}  // namespace ah

using namespace ah;

extern "C" {

int ah_dedup_table_local(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values, int64_t n_tail,
                         int prefix_digits, int tail_digits, float avg_precision_lost, AhDedupTable** out) {
  AH_REQUIRE(out, "dedup_table: null out");
  *out = nullptr;
  AH_REQUIRE(n_prefix >= 0 && n_prefix <= 65536 && n_tail >= 0 && n_tail <= 65536,
             "dedup_table: at most 65536 prefixes and tails");
  AH_REQUIRE((prefixes || n_prefix == 0) && (tail_values || n_tail == 0), "dedup_table: null table");
  AH_TRY_DEDUP(check_digits(prefix_digits, tail_digits));
  AhDedupTable* t = new (std::nothrow) AhDedupTable();
  if (!t) return fail(AH_ENOMEM, "dedup_table: host allocation");
  cudaGetDevice(&t->device);
  t->mode = kLocal;
  t->n_prefix = n_prefix;
  t->n_tail = n_tail;
  t->avg = avg_precision_lost;
  // decompressor.rs:8-9,15-20: prefix_int as f32 / prefix_scale, tail as f32 / divisor
  const float prefix_scale = pow10f_i(prefix_digits), divisor = pow10f_i(prefix_digits + tail_digits);
  std::vector<float> pre((size_t)n_prefix + 1, 0.0f), tl((size_t)n_tail + 1, 0.0f);
  for (int64_t k = 0; k < n_prefix; ++k) pre[k] = (float)prefixes[k] / prefix_scale;
  for (int64_t k = 0; k < n_tail; ++k) tl[k] = (float)tail_values[k] / divisor;
  int rc = upload(t, &t->d_pre, pre);
  if (rc == AH_OK) rc = upload(t, &t->d_tail, tl);
  return finish(t, rc, out);
}

int ah_dedup_table_global(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values, int64_t n_tail,
                          int prefix_digits, int tail_digits, float avg_precision_lost, int g_prefix_digits,
                          const float* g_prefixes, int64_t n_gp, const uint32_t* g_tail_off, const uint32_t* g_tails,
                          AhDedupTable** out) {
  AH_REQUIRE(out, "dedup_table: null out");
  *out = nullptr;
  AH_REQUIRE(n_prefix >= 0 && n_prefix <= 65536 && n_tail >= 0 && n_tail <= 65536,
             "dedup_table: at most 65536 prefixes and tails");
  AH_REQUIRE((prefixes || n_prefix == 0) && (tail_values || n_tail == 0), "dedup_table: null table");
  AH_REQUIRE(n_gp >= 1 && g_prefixes && g_tail_off && (g_tails || g_tail_off[n_gp] == 0),
             "dedup_table: the global table needs at least one prefix (the reference indexes row 0)");
  AH_TRY_DEDUP(check_digits(g_prefix_digits, tail_digits));
  AH_TRY_DEDUP(check_digits(prefix_digits, 0));
  AH_REQUIRE((n_prefix + 1) * (n_tail + 1) <= kMaxTableEntries, "dedup_table: %lld x %lld lookup table too large",
             (long long)n_prefix, (long long)n_tail);
  const float tail_divisor = pow10f_i(g_prefix_digits + tail_digits);
  const float gt_scale = pow10f_i(g_prefix_digits);
  const int scale_diff = g_prefix_digits - prefix_digits;
  // prefix_lookup: pv -> gi, the first insert wins (decompressor.rs:37-48)
  std::vector<int32_t> plook(65536, -1);
  for (int64_t k = 0; k < n_prefix; ++k) {
    const uint16_t pv = prefixes[k];
    if (plook[pv] < 0) {
      const int64_t gi = find_global_prefix(g_prefixes, n_gp, gt_scale, norm_prefix(pv, scale_diff));
      if (gi >= 0) plook[pv] = (int32_t)gi;
    }
  }
  // rows: p < n_prefix with tail_lookup (:50-61, value -> last index in the row);
  // row n_prefix is an out-of-range p_idx (pv reads 0, no tail key)
  std::vector<float> tab((size_t)(n_prefix + 1) * (n_tail + 1));
  std::vector<int32_t> last(65536, -1);
  for (int64_t cp = 0; cp <= n_prefix; ++cp) {
    const uint16_t pv = cp < n_prefix ? prefixes[cp] : 0;
    const int64_t gp = plook[pv] >= 0 ? plook[pv] : 0;
    const uint32_t r0 = g_tail_off[gp], r1 = g_tail_off[gp + 1];
    AH_REQUIRE(r1 > r0, "dedup_table: global tail row %lld is empty (the reference panics)", (long long)gp);
    if (cp < n_prefix)
      for (uint32_t q = r0; q < r1; ++q)
        if (g_tails[q] < 65536u) last[g_tails[q]] = (int32_t)(q - r0);
    for (int64_t ct = 0; ct <= n_tail; ++ct) {
      const int64_t gt = (cp < n_prefix && ct < n_tail && last[tail_values[ct]] >= 0) ? last[tail_values[ct]] : 0;
      tab[(size_t)cp * (n_tail + 1) + ct] = g_prefixes[gp] + (float)g_tails[r0 + gt] / tail_divisor;
    }
    if (cp < n_prefix)
      for (uint32_t q = r0; q < r1; ++q)
        if (g_tails[q] < 65536u) last[g_tails[q]] = -1;
  }
  AhDedupTable* t = new (std::nothrow) AhDedupTable();
  if (!t) return fail(AH_ENOMEM, "dedup_table: host allocation");
  cudaGetDevice(&t->device);
  t->mode = kGlobal;
  t->n_prefix = n_prefix;
  t->n_tail = n_tail;
  t->avg = avg_precision_lost;
  return finish(t, upload(t, &t->d_tab, tab), out);
}

int ah_dedup_table_remap(const uint16_t* prefixes, int64_t n_prefix, int prefix_digits, int tail_digits,
                         float avg_precision_lost, int g_prefix_digits, const float* g_prefixes, int64_t n_gp,
                         const uint32_t* g_tail_off, const uint32_t* g_tails, const uint16_t* remap, int64_t n_remap,
                         AhDedupTable** out) {
  AH_REQUIRE(out, "dedup_table: null out");
  *out = nullptr;
  AH_REQUIRE(n_prefix >= 0 && n_prefix <= 65536 && n_remap >= 0 && n_remap <= 65536,
             "dedup_table: at most 65536 prefixes and remap entries");
  AH_REQUIRE((prefixes || n_prefix == 0) && (remap || n_remap == 0), "dedup_table: null table");
  AH_REQUIRE(n_gp >= 1 && g_prefixes && g_tail_off && (g_tails || g_tail_off[n_gp] == 0),
             "dedup_table: the global table needs at least one prefix (the reference indexes row 0)");
  AH_TRY_DEDUP(check_digits(g_prefix_digits, tail_digits));
  AH_TRY_DEDUP(check_digits(prefix_digits, 0));
  AH_REQUIRE((n_prefix + 1) * (n_remap + 1) <= kMaxTableEntries, "dedup_table: %lld x %lld lookup table too large",
             (long long)n_prefix, (long long)n_remap);
  // global_lookup.rs:91-108: gp = first matching global prefix (else 0), the tail
  // through the remap (missing entries read 0)
  const float divisor = pow10f_i(g_prefix_digits + tail_digits);
  const float gt_scale = pow10f_i(g_prefix_digits);
  const int scale_diff = g_prefix_digits - prefix_digits;
  std::vector<float> tab((size_t)(n_prefix + 1) * (n_remap + 1), 0.0f);
  for (int64_t cp = 0; cp < n_prefix; ++cp) {
    const int64_t gi = find_global_prefix(g_prefixes, n_gp, gt_scale, norm_prefix(prefixes[cp], scale_diff));
    const int64_t gp = gi >= 0 ? gi : 0;
    const uint32_t r0 = g_tail_off[gp], len = g_tail_off[gp + 1] - r0;
    for (int64_t ct = 0; ct <= n_remap; ++ct) {
      const uint32_t mapped = ct < n_remap ? remap[ct] : 0u;
      const uint32_t tail = mapped < len ? g_tails[r0 + mapped] : 0u;
      tab[(size_t)cp * (n_remap + 1) + ct] = g_prefixes[gp] + (float)tail / divisor;
    }
  }
  AhDedupTable* t = new (std::nothrow) AhDedupTable();
  if (!t) return fail(AH_ENOMEM, "dedup_table: host allocation");
  cudaGetDevice(&t->device);
  t->mode = kRemap;
  t->n_prefix = n_prefix;
  t->n_tail = n_remap;
  t->avg = avg_precision_lost;
  return finish(t, upload(t, &t->d_tab, tab), out);
}

int ah_dedup_table_destroy(AhDedupTable* t) {
  if (!t) return AH_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(t->device);
  if (t->d_pre) cudaFree(t->d_pre);
  if (t->d_tail) cudaFree(t->d_tail);
  if (t->d_tab) cudaFree(t->d_tab);
  cudaSetDevice(cur);
  delete t;
  return AH_OK;
}

int ah_dedup_decompress_f32(const AhDedupTable* t, const uint16_t* prefix_idx, int64_t n_pidx,
                            const uint16_t* tail_idx, int64_t n_tidx, const uint8_t* sign_bits, int64_t n_sign,
                            int64_t count, float* out, void* stream) {
  AH_REQUIRE(t, "dedup_decompress: null table");
  AH_TRY_DEDUP(check_sandbag(t, n_pidx, n_tidx, n_sign, count));
  if (count == 0) return AH_OK;
  AH_REQUIRE(out, "dedup_decompress: null output");
  const DedupArgs a = make_args(t, prefix_idx, n_pidx, tail_idx, n_tidx, sign_bits, n_sign);
  AH_REQUIRE(a.err, "dedup_decompress: device error word unavailable");
  const int vec = aligned16(prefix_idx) && aligned16(tail_idx) && aligned16(out);
  const int grid = grid_for((count + 7) / 8);
  AH_TRY_DEDUP(launch_table_kernel<DecompressKernel>(t, grid, as_stream(stream), a, count, out, vec));
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_dedup_into_q4w(const AhDedupTable* t, const uint16_t* prefix_idx, int64_t n_pidx, const uint16_t* tail_idx,
                      int64_t n_tidx, const uint8_t* sign_bits, int64_t n_sign, AhQ4Weight* w, void* stream) {
  AH_REQUIRE(t && w, "dedup_into_q4w: null argument");
  const Q4Tiled& tw = q4w_tiled(w);
  const int64_t rows = tw.rows, cols = tw.cols;
  AH_REQUIRE(tw.f32_scales && cols % 32 == 0,
             "dedup_into_q4w: the weight must be engine format (f32 scales) with cols a multiple of 32");
  AH_TRY_DEDUP(check_sandbag(t, n_pidx, n_tidx, n_sign, rows * cols));
  AH_REQUIRE(((uintptr_t)prefix_idx & 7u) == 0 && ((uintptr_t)tail_idx & 7u) == 0,
             "dedup_into_q4w: index arrays must be 8-byte aligned");
  const DedupArgs a = make_args(t, prefix_idx, n_pidx, tail_idx, n_tidx, sign_bits, n_sign);
  AH_REQUIRE(a.err, "dedup_into_q4w: device error word unavailable");
  const int64_t warps = tw.r16 * 16 * ((2 * tw.kp + 7) / 8);
  const int grid = grid_for(warps * 32);
  uint32_t* nib = reinterpret_cast<uint32_t*>(q4w_nib_mut(w));
  float* sc = static_cast<float*>(q4w_scales_mut(w));
  AH_TRY_DEDUP(launch_table_kernel<Q4wKernel>(t, grid, as_stream(stream), a, nib, sc, rows, cols, tw.r16, tw.kp));
  AH_LAUNCH_CHECK();
  return AH_OK;
}

int ah_dedup_to_q4w(const AhDedupTable* t, const uint16_t* prefix_idx, int64_t n_pidx, const uint16_t* tail_idx,
                    int64_t n_tidx, const uint8_t* sign_bits, int64_t n_sign, int64_t rows, int64_t cols,
                    AhQ4Weight** out, void* stream) {
  AH_REQUIRE(t && out, "dedup_to_q4w: null argument");
  *out = nullptr;
  AH_REQUIRE(rows > 0 && cols > 0 && cols % 32 == 0, "dedup_to_q4w: rows > 0 and cols a multiple of 32 required");
  AH_TRY_DEDUP(check_sandbag(t, n_pidx, n_tidx, n_sign, rows * cols));
  AhQ4Weight* w = nullptr;
  AH_TRY_DEDUP(q4w_alloc(rows, cols, true, &w));
  const int rc = ah_dedup_into_q4w(t, prefix_idx, n_pidx, tail_idx, n_tidx, sign_bits, n_sign, w, stream);
  if (rc != AH_OK) {
    ah_q4w_destroy(w);
    return rc;
  }
  *out = w;
  return AH_OK;
}

int ah_host_dedup_decompress_all(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values,
                                 int64_t n_tail, int64_t count, int prefix_digits, int tail_digits,
                                 float avg_precision_lost, const uint16_t* prefix_idx, int64_t n_pidx,
                                 const uint16_t* tail_idx, int64_t n_tidx, const uint8_t* sign_bits, int64_t n_sign,
                                 float* out) {
  AH_REQUIRE(count >= 0, "dedup_decompress_all: negative count");
  if (count == 0) return AH_OK;
  AH_REQUIRE(out, "dedup_decompress_all: null output");
  AhDedupTable* t = nullptr;
  AH_TRY_DEDUP(ah_dedup_table_local(prefixes, n_prefix, tail_values, n_tail, prefix_digits, tail_digits,
                                    avg_precision_lost, &t));
  n_pidx = prefix_idx ? std::min(n_pidx, count) : 0;  // entries past count are never read
  n_tidx = tail_idx ? std::min(n_tidx, count) : 0;
  n_sign = sign_bits ? std::min(n_sign, (count + 7) / 8) : 0;
  uint16_t *dp = nullptr, *dt = nullptr;
  uint8_t* ds = nullptr;
  float* dout = nullptr;
  int rc = AH_OK;
  if (ah::dev_malloc(&dp, std::max<int64_t>(n_pidx, 1) * 2) != cudaSuccess ||
      ah::dev_malloc(&dt, std::max<int64_t>(n_tidx, 1) * 2) != cudaSuccess ||
      ah::dev_malloc(&ds, std::max<int64_t>(n_sign, 1)) != cudaSuccess ||
      ah::dev_malloc(&dout, (size_t)count * 4) != cudaSuccess) {
    cudaGetLastError();
    rc = fail(AH_ENOMEM, "dedup_decompress_all: device allocation failed");
  }
  if (rc == AH_OK && n_pidx && cudaMemcpy(dp, prefix_idx, n_pidx * 2, cudaMemcpyHostToDevice) != cudaSuccess)
    rc = fail(AH_ECUDA, "dedup_decompress_all: upload failed");
  if (rc == AH_OK && n_tidx && cudaMemcpy(dt, tail_idx, n_tidx * 2, cudaMemcpyHostToDevice) != cudaSuccess)
    rc = fail(AH_ECUDA, "dedup_decompress_all: upload failed");
  if (rc == AH_OK && n_sign && cudaMemcpy(ds, sign_bits, n_sign, cudaMemcpyHostToDevice) != cudaSuccess)
    rc = fail(AH_ECUDA, "dedup_decompress_all: upload failed");
  if (rc == AH_OK) rc = ah_dedup_decompress_f32(t, dp, n_pidx, dt, n_tidx, ds, n_sign, count, dout, nullptr);
  if (rc == AH_OK && cudaMemcpy(out, dout, (size_t)count * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = fail(AH_ECUDA, "dedup_decompress_all: download failed");
  cudaFree(dp);
  cudaFree(dt);
  cudaFree(ds);
  cudaFree(dout);
  ah_dedup_table_destroy(t);
  return rc;
}

}  // extern "C"
