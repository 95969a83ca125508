// ah_ssm.cu — the gated delta-net SSM block (inference/ssm.rs:171-296), one
// token step on the device.
//
// Three launches per step, all on the caller's stream, each allowed to start
// while the previous one drains (programmatic dependent launch):
//   k_ssm_gemv (4 segments)  qkv_mixed = Wqkv x, each row's channel going
//                            straight through the depthwise conv1d over the
//                            (d_conv - 1)-step window, SiLU and the window shift
//                            (math.rs:165-190); z = Wgate x;
//                            beta = sigmoid(Wbeta x); gate = softplus(Walpha x + dt_bias) * a
//   k_ssm_delta              per value head and 16-row slice of its state: L2 norm
//                            of q and k (their key head), S *= exp(gate); sk = S k;
//                            delta = (v - sk) beta; S += delta k^T; o = S q / sqrt(d);
//                            the head's last slice to finish applies the gated
//                            RMSNorm of o times silu(z)
//   k_ssm_gemv (1 segment)   out = Wout result
// The recurrence is row-parallel: row i of a head's state needs only k, q, v_i
// and beta, so one warp owns each row and S streams through HBM once per step
// (2 x 4 B per state element).  The projections are HBM-bound f32 GEMVs, a
// warp (or, for short wide matrices, a few warps) per row.  Sums are warp trees
// rather than the reference's sequential loops, so results agree to f32
// rounding, not bit for bit; the state update uses separately rounded multiply
// and add, as the Rust code does.
#include <algorithm>

#include "ah_common.cuh"
#include "ah_sm100.cuh"

#define AH_TRY_SSM(expr)          \
  do {                            \
    const int _rc = (expr);       \
    if (_rc != AH_OK) return _rc; \
  } while (0)

namespace ah {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxHeadDim = 256;  // head_k_dim = head_v_dim

__device__ __forceinline__ float sigmoid_ref(float x) {  // math.rs:88-96
  if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
  const float e = expf(x);
  return e / (1.0f + e);
}
__device__ __forceinline__ float silu_ssm(float x) { return x * sigmoid_ref(x); }      // math.rs:83-86
__device__ __forceinline__ float softplus_ref(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }  // :98-104

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
// Sum over the CTA; every thread gets the result.  `red` holds one float per warp.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

enum SegEpi : int { kSegPlain = 0, kSegSigmoid = 1, kSegSoftplusGate = 2, kSegConv = 3 };
struct GemvSeg {
  const float* w;  // [rows][cols]
  float* y;        // [rows]
  int rows;
  int epi;
  const float* bias;  // softplus gate: dt_bias
  const float* mul;   // softplus gate: a
};
struct SsmGemvArgs {
  GemvSeg seg[4];
  int nseg;
  int cols;
  int vec;    // float4 loads (cols % 4 == 0, 16-byte aligned rows and x)
  int split;  // warps per row (1, 2, 4 or 8): each sums a contiguous share of the columns
  const float* x;
  // kSegConv: conv_out[c] = silu(sum_k state[k][c] w[c][k] + y_c w[c][d_conv-1]),
  // then the window moves one step (math.rs:165-190)
  const float* conv_w;  // [channels][d_conv]
  float* conv_state;    // [(d_conv - 1)][channels]
  int d_conv;
  int* zero;  // [nzero] set to 0 once the previous launch on the stream is complete
  int nzero;
};

constexpr int kGemvBatch = 8;  // float4 loads in flight per lane

__device__ __forceinline__ float4 ldg4_or0(const float4* p, int j, int hi) {
  return j < hi ? __ldg(p + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
}

// `split` warps per output row over the concatenated segments; a CTA covers
// 8 / split rows.  Each lane issues kGemvBatch independent float4 weight loads
// before it consumes them, and the first batch is fetched before the launch
// waits for the previous kernel on the stream (weights do not change during
// the step), so the weight stream starts while the producer of x drains.
__global__ void __launch_bounds__(kThreads) k_ssm_gemv(const SsmGemvArgs a) {
  __shared__ float part[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int S = a.split;
  int total = 0;
  for (int s = 0; s < a.nseg; ++s) total += a.seg[s].rows;
  const int r = blockIdx.x * ((kThreads / 32) / S) + warp / S, piece = warp % S;
  const bool live = r < total;
  int s = 0, rr = r;
  if (live)
    while (rr >= a.seg[s].rows) rr -= a.seg[s++].rows;
  const GemvSeg& g = a.seg[s];
  const float* row = g.w + (int64_t)(live ? rr : 0) * a.cols;
  float acc = 0.0f;
  if (a.vec) {
    const int n4 = a.cols / 4, share = (n4 + S - 1) / S;
    const int lo = min(piece * share, n4), hi = live ? min(lo + share, n4) : lo;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    float4 w[kGemvBatch];
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u) w[u] = ldg4_or0(r4, lo + lane + 32 * u, hi);
    pdl_wait();
    for (int j0 = lo + lane;;) {
#pragma unroll
      for (int u = 0; u < kGemvBatch; ++u) {
        const float4 x = ldg4_or0(x4, j0 + 32 * u, hi);
        acc += w[u].x * x.x + w[u].y * x.y + w[u].z * x.z + w[u].w * x.w;
      }
      j0 += 32 * kGemvBatch;
      if (j0 >= hi) break;
#pragma unroll
      for (int u = 0; u < kGemvBatch; ++u) w[u] = ldg4_or0(r4, j0 + 32 * u, hi);
    }
  } else {
    pdl_wait();
    const int share = (a.cols + S - 1) / S;
    const int lo = min(piece * share, a.cols), hi = live ? min(lo + share, a.cols) : lo;
    for (int j = lo + lane; j < hi; j += 32) acc += __ldg(row + j) * __ldg(a.x + j);
  }
  pdl_launch_dependents();
  if (a.zero && blockIdx.x == 0)
    for (int i = threadIdx.x; i < a.nzero; i += blockDim.x) a.zero[i] = 0;
  acc = warp_sum(acc);
  if (S > 1) {  // the row's pieces in column order
    if (lane == 0) part[warp] = acc;
    __syncthreads();
    if (piece != 0) return;
    acc = part[warp];
    for (int p = 1; p < S; ++p) acc += part[warp + p];
  }
  if (!live || lane != 0) return;
  if (g.epi == kSegSigmoid) {
    acc = sigmoid_ref(acc);
  } else if (g.epi == kSegSoftplusGate) {
    acc = softplus_ref(acc + g.bias[rr]) * g.mul[rr];
  } else if (g.epi == kSegConv) {
    const int c = rr, ch = g.rows, dc = a.d_conv;
    float sum = 0.0f;
    for (int k = 0; k < dc - 1; ++k) sum += a.conv_state[(int64_t)k * ch + c] * a.conv_w[(int64_t)c * dc + k];
    sum += acc * a.conv_w[(int64_t)c * dc + (dc - 1)];
    for (int k = 0; k + 1 < dc - 1; ++k) a.conv_state[(int64_t)k * ch + c] = a.conv_state[(int64_t)(k + 1) * ch + c];
    if (dc > 1) a.conv_state[(int64_t)(dc - 2) * ch + c] = acc;
    acc = silu_ssm(sum);
  }
  g.y[rr] = acc;
}

struct DeltaArgs {
  const float* conv_out;  // [2 key_dim + value_dim]: q | k | v
  const float* z;         // [value_dim]
  const float* beta;      // [nv]
  const float* gate;      // [nv]
  const float* norm_w;    // [D]
  float* state;           // [nv][D][D]
  float* obuf;            // [value_dim]: o = S q, before the gated norm
  float* result;          // [value_dim]
  int* done;              // [nv]: row slices of the head finished this step (zeroed by the projection launch)
  int D, nk, nv, rows_per_cta;
  float eps, scale;
};

constexpr int kDeltaRowsPerWarp = 2;

// CTA (h, c): value head h (its key head is h / (nv / nk)), state rows
// [c * rows_per_cta, (c + 1) * rows_per_cta), kDeltaRowsPerWarp rows per warp
// at once.  The state rows are fetched first, so their HBM latency overlaps
// the L2 norms of q and k.  The last CTA of a head to finish (a counter per
// head, after a device-scope fence) applies the gated RMSNorm of the head's
// o (math.rs:53-63) times silu(z).
__global__ void __launch_bounds__(kThreads) k_ssm_delta(const DeltaArgs a) {
  constexpr int E = kMaxHeadDim / 32, RW = kDeltaRowsPerWarp;
  __shared__ float qs[kMaxHeadDim], kn[kMaxHeadDim], red[kThreads / 32];
  __shared__ int last;
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.y * a.rows_per_cta, r1 = min(r0 + a.rows_per_cta, a.D);
  const int D = a.D, key_dim = a.nk * D;
  const int src = h / (a.nv / a.nk);
  float* S = a.state + (int64_t)h * D * D;
  pdl_wait();
  const int row0 = r0 + warp * RW;
  float s[RW][E];
#pragma unroll
  for (int t = 0; t < RW; ++t)
#pragma unroll
    for (int e = 0; e < E; ++e)
      s[t][e] = (row0 + t < r1 && lane + 32 * e < D) ? S[(int64_t)(row0 + t) * D + lane + 32 * e] : 0.0f;
  const float* q = a.conv_out + (int64_t)src * D;
  const float* k = a.conv_out + key_dim + (int64_t)src * D;
  const float* v = a.conv_out + 2 * key_dim + (int64_t)h * D;
  // L2 norm per key head (math.rs:71-80): x / max(sqrt(sum x^2), eps); q then scaled
  float sq = 0.0f, sk2 = 0.0f;
  for (int i = tid; i < D; i += blockDim.x) {
    sq += q[i] * q[i];
    sk2 += k[i] * k[i];
  }
  const float nq = block_sum(sq, red);
  const float nkk = block_sum(sk2, red);
  const float iq = 1.0f / fmaxf(sqrtf(nq), a.eps), ik = 1.0f / fmaxf(sqrtf(nkk), a.eps);
  for (int i = tid; i < D; i += blockDim.x) {
    qs[i] = (q[i] * iq) * a.scale;
    kn[i] = k[i] * ik;
  }
  __syncthreads();
  pdl_launch_dependents();
  const float decay = expf(a.gate[h]), beta = a.beta[h];
#pragma unroll
  for (int t = 0; t < RW; ++t) {
    const int i = row0 + t;
    if (i >= r1) break;  // warp-uniform
    float dot = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (lane + 32 * e < D) {
        s[t][e] *= decay;
        dot += s[t][e] * kn[lane + 32 * e];
      }
    const float delta = (v[i] - warp_sum(dot)) * beta;
    float od = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (lane + 32 * e < D) {
        s[t][e] = __fadd_rn(s[t][e], __fmul_rn(delta, kn[lane + 32 * e]));  // S += delta k^T, unfused like the reference
        S[(int64_t)i * D + lane + 32 * e] = s[t][e];
        od += s[t][e] * qs[lane + 32 * e];
      }
    od = warp_sum(od);
    if (lane == 0) a.obuf[(int64_t)h * D + i] = od;
  }
  // the last row slice of head h to finish normalises the head
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.done[h], 1) == (int)gridDim.y - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* o = a.obuf + (int64_t)h * D;
  float ss = 0.0f;
  for (int i = tid; i < D; i += blockDim.x) {
    const float oi = __ldcg(o + i);
    ss += oi * oi;
  }
  const float tot = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(tot / (float)D + a.eps);
  for (int i = tid; i < D; i += blockDim.x)
    a.result[(int64_t)h * D + i] = (__ldcg(o + i) * inv * a.norm_w[i]) * silu_ssm(a.z[(int64_t)h * D + i]);
}

struct SsmDims {
  int64_t d, D, nk, nv, key_dim, value_dim, conv_dim, d_conv;
};

inline int64_t pad4(int64_t n) { return (n + 3) / 4 * 4; }

int ssm_dims(const AhSsmConfig* c, SsmDims* s) {
  AH_REQUIRE(c, "ssm: null config");
  AH_REQUIRE(c->n_embd > 0 && c->d_state > 0 && c->n_group > 0 && c->dt_rank > 0 && c->d_inner > 0 && c->d_conv >= 1,
             "ssm: non-positive dimension");
  AH_REQUIRE(c->d_inner % c->dt_rank == 0 && c->d_inner / c->dt_rank == c->d_state,
             "ssm: head_v_dim (d_inner / dt_rank) must equal head_k_dim (d_state), as ssm.rs:239 asserts");
  AH_REQUIRE(c->dt_rank % c->n_group == 0, "ssm: dt_rank must be a multiple of n_group");
  AH_REQUIRE(c->d_state <= kMaxHeadDim, "ssm: head dim at most %d", kMaxHeadDim);
  s->d = c->n_embd;
  s->D = c->d_state;
  s->nk = c->n_group;
  s->nv = c->dt_rank;
  s->key_dim = s->D * s->nk;
  s->value_dim = s->D * s->nv;
  s->conv_dim = 2 * s->key_dim + s->value_dim;
  s->d_conv = c->d_conv;
  return AH_OK;
}

// conv_out | z | result | obuf | beta | gate | per-head counters (int)
size_t ws_floats(const SsmDims& s) {
  return (size_t)(pad4(s.conv_dim) + 3 * pad4(s.value_dim) + 3 * pad4(s.nv));
}

bool aligned16f(const float* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Warps per row: one while the rows alone give every SM two CTAs' worth of
// warps, else up to 8, so that short, wide matrices still keep enough loads in
// flight.
int launch_gemv(SsmGemvArgs g, int total_rows, cudaStream_t st) {
  const int warps_per_cta = kThreads / 32;
  const int want = 2 * sm_count() * warps_per_cta;
  g.split = 1;
  while (g.split < warps_per_cta && total_rows * g.split < want && g.cols / (4 * 32 * g.split) >= 2 * kGemvBatch)
    g.split *= 2;
  const int rows_per_cta = warps_per_cta / g.split;
  return launch_pdl(k_ssm_gemv, dim3((unsigned)((total_rows + rows_per_cta - 1) / rows_per_cta)), dim3(kThreads), 0,
                    st, g);
}

}  // namespace
}  // namespace ah

using namespace ah;

extern "C" {

int ah_ssm_workspace_bytes(const AhSsmConfig* cfg, size_t* bytes) {
  AH_REQUIRE(bytes, "ssm_workspace_bytes: null out");
  SsmDims s;
  const int rc = ssm_dims(cfg, &s);
  if (rc != AH_OK) return rc;
  *bytes = ws_floats(s) * sizeof(float);
  return AH_OK;
}

int ah_ssm_forward(const AhSsmConfig* cfg, const AhSsmWeights* w, float* conv_state, float* ssm_state,
                   const float* x, float* out, void* workspace, size_t workspace_bytes, void* stream) {
  SsmDims s;
  const int rc = ssm_dims(cfg, &s);
  if (rc != AH_OK) return rc;
  AH_REQUIRE(w && w->wqkv && w->wqkv_gate && w->conv1d && w->dt_bias && w->a && w->alpha && w->beta && w->norm &&
                 w->out,
             "ssm_forward: null weight");
  AH_REQUIRE(ssm_state && x && out && (conv_state || s.d_conv == 1), "ssm_forward: null state or vector");
  AH_REQUIRE(workspace && workspace_bytes >= ws_floats(s) * sizeof(float) && aligned16f((const float*)workspace),
             "ssm_forward: workspace of %zu bytes (16-byte aligned) required", ws_floats(s) * sizeof(float));
  cudaStream_t st = as_stream(stream);
  float* ws = static_cast<float*>(workspace);
  float* cout = ws;
  float* z = cout + pad4(s.conv_dim);
  float* res = z + pad4(s.value_dim);
  float* obuf = res + pad4(s.value_dim);
  float* beta = obuf + pad4(s.value_dim);
  float* gate = beta + pad4(s.nv);
  int* done = reinterpret_cast<int*>(gate + pad4(s.nv));
  // input projections with the conv1d + SiLU + window shift fused into the
  // qkv rows, beta and the decay gate, in one launch (ssm.rs:184-207)
  SsmGemvArgs g{};
  g.x = x;
  g.cols = (int)s.d;
  g.nseg = 4;
  g.seg[0] = GemvSeg{w->wqkv, cout, (int)s.conv_dim, kSegConv, nullptr, nullptr};
  g.seg[1] = GemvSeg{w->wqkv_gate, z, (int)s.value_dim, kSegPlain, nullptr, nullptr};
  g.seg[2] = GemvSeg{w->beta, beta, (int)s.nv, kSegSigmoid, nullptr, nullptr};
  g.seg[3] = GemvSeg{w->alpha, gate, (int)s.nv, kSegSoftplusGate, w->dt_bias, w->a};
  g.vec = s.d % 4 == 0 && aligned16f(x) && aligned16f(w->wqkv) && aligned16f(w->wqkv_gate) &&
          aligned16f(w->beta) && aligned16f(w->alpha);
  g.conv_w = w->conv1d;
  g.conv_state = conv_state;
  g.d_conv = (int)s.d_conv;
  g.zero = done;
  g.nzero = (int)s.nv;
  AH_TRY_SSM(launch_gemv(g, (int)(s.conv_dim + s.value_dim + 2 * s.nv), st));
  // L2 norms, gated delta rule, gated RMSNorm (ssm.rs:216-292)
  DeltaArgs da{};
  da.conv_out = cout;
  da.z = z;
  da.beta = beta;
  da.gate = gate;
  da.norm_w = w->norm;
  da.state = ssm_state;
  da.obuf = obuf;
  da.result = res;
  da.done = done;
  da.D = (int)s.D;
  da.nk = (int)s.nk;
  da.nv = (int)s.nv;
  da.rows_per_cta = (kThreads / 32) * kDeltaRowsPerWarp;  // the heads' rows spread over many SMs
  da.eps = cfg->rms_eps;
  da.scale = 1.0f / sqrtf((float)s.D);
  AH_TRY_SSM(launch_pdl(k_ssm_delta, dim3((unsigned)s.nv, (unsigned)((s.D + da.rows_per_cta - 1) / da.rows_per_cta)),
                        dim3(kThreads), 0, st, da));
  // output projection (ssm.rs:295)
  SsmGemvArgs go{};
  go.x = res;
  go.cols = (int)s.value_dim;
  go.nseg = 1;
  go.seg[0] = GemvSeg{w->out, out, (int)s.d, kSegPlain, nullptr, nullptr};
  go.vec = s.value_dim % 4 == 0 && aligned16f(w->out) && aligned16f(out);
  return launch_gemv(go, (int)s.d, st);
}

}  // extern "C"
