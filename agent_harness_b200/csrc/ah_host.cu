// ah_host.cu — the host-slice drop-ins: the reference's Rust functions take
// host slices and return when the result is in the caller's buffer, so these
// upload, run the device kernel and download, synchronously, on a per-thread
// stream, with device staging buffers cached per thread and device.
#include <cstring>
#include <vector>

#include "ah_common.cuh"

namespace ah {
// the engine-format GEMV over a window of rows whose bytes start at byte0 (ah_gemv.cu)
int gemv_rows_window(float* out, const float* scales, const uint8_t* packed, const float* x, int64_t rows,
                     int64_t cols, int64_t gs, int64_t row0, int64_t byte0, cudaStream_t st);
namespace {

struct Staging {
  int device = -1;
  cudaStream_t stream = nullptr;
  std::vector<void*> bufs;
  std::vector<size_t> caps;
  ~Staging() {
    for (void* p : bufs)
      if (p) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
  }
};

thread_local Staging t_stage;

int stage_ready() {
  int dev = 0;
  AH_CUDA_TRY(cudaGetDevice(&dev));
  if (t_stage.device != dev) {
    for (void* p : t_stage.bufs)
      if (p) cudaFree(p);
    t_stage.bufs.clear();
    t_stage.caps.clear();
    if (t_stage.stream) cudaStreamDestroy(t_stage.stream);
    t_stage.stream = nullptr;
    AH_CUDA_TRY(cudaStreamCreateWithFlags(&t_stage.stream, cudaStreamNonBlocking));
    t_stage.device = dev;
  }
  return AH_OK;
}

// Device buffer `slot` of at least `bytes` (256-byte aligned).
int stage_buf(int slot, size_t bytes, void** out) {
  if ((int)t_stage.bufs.size() <= slot) {
    t_stage.bufs.resize(slot + 1, nullptr);
    t_stage.caps.resize(slot + 1, 0);
  }
  if (bytes == 0) bytes = 16;
  if (t_stage.caps[slot] < bytes) {
    if (t_stage.bufs[slot]) cudaFree(t_stage.bufs[slot]);
    t_stage.bufs[slot] = nullptr;
    t_stage.caps[slot] = 0;
    if (ah::dev_malloc(&t_stage.bufs[slot], bytes) != cudaSuccess) {
      cudaGetLastError();
      return fail(AH_ENOMEM, "host staging: cudaMalloc of %zu bytes failed", bytes);
    }
    t_stage.caps[slot] = bytes;
  }
  *out = t_stage.bufs[slot];
  return AH_OK;
}

#define AH_TRY(expr)            \
  do {                          \
    int _rc = (expr);           \
    if (_rc != AH_OK) return _rc; \
  } while (0)

int upload(int slot, const void* host, size_t bytes, void** dev) {
  AH_TRY(stage_buf(slot, bytes, dev));
  if (bytes) AH_CUDA_TRY(cudaMemcpyAsync(*dev, host, bytes, cudaMemcpyHostToDevice, t_stage.stream));
  return AH_OK;
}

int finish_download(void* host, const void* dev, size_t bytes) {
  if (bytes) AH_CUDA_TRY(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, t_stage.stream));
  AH_CUDA_TRY(cudaStreamSynchronize(t_stage.stream));
  return AH_OK;
}

}  // namespace
}  // namespace ah

using namespace ah;

extern "C" {

int ah_host_gemv_4bit_into(float* out, const float* scales, const uint8_t* packed, const float* x, size_t rows,
                           size_t cols, size_t gs) {
  if (rows == 0) return AH_OK;
  AH_REQUIRE(out != nullptr, "host_gemv_4bit_into: null out");
  if (cols == 0 || x == nullptr) {  // inference/math.rs:264-267
    memset(out, 0, rows * sizeof(float));
    return AH_OK;
  }
  AH_REQUIRE(scales && packed, "host_gemv_4bit_into: null weights");
  const size_t g = gs < 1 ? 1 : gs;
  const size_t n_gpr = (cols + g - 1) / g;
  AH_TRY(stage_ready());
  void *ds, *dp, *dx, *dy;
  AH_TRY(upload(0, scales, rows * n_gpr * sizeof(float), &ds));
  AH_TRY(upload(1, packed, (rows * cols + 1) / 2, &dp));
  AH_TRY(upload(2, x, cols * sizeof(float), &dx));
  AH_TRY(stage_buf(3, rows * sizeof(float), &dy));
  AH_TRY(ah_gemv_4bit_into(static_cast<float*>(dy), static_cast<const float*>(ds), static_cast<const uint8_t*>(dp),
                           static_cast<const float*>(dx), (int64_t)rows, (int64_t)cols, (int64_t)g, t_stage.stream));
  return finish_download(out, dy, rows * sizeof(float));
}

int ah_host_gemv_4bit_worker_scalar(float* out, const float* scales, const uint8_t* packed, const float* x,
                                    size_t row_start, size_t row_end, size_t cols, size_t gs) {
  AH_REQUIRE(row_end >= row_start, "host_gemv_4bit_worker_scalar: row_end < row_start");
  const size_t rows = row_end - row_start;
  if (rows == 0) return AH_OK;
  AH_REQUIRE(out != nullptr, "host_gemv_4bit_worker_scalar: null out");
  if (cols == 0) {
    memset(out, 0, rows * sizeof(float));
    return AH_OK;
  }
  AH_REQUIRE(scales && packed && x, "host_gemv_4bit_worker_scalar: null input");
  const size_t g = gs < 1 ? 1 : gs;
  const size_t n_gpr = (cols + g - 1) / g;
  // only the rows the worker reads: their scales and the bytes holding their nibbles
  const size_t b0 = (row_start * cols) >> 1, b1 = (row_end * cols + 1) >> 1;
  AH_TRY(stage_ready());
  void *ds, *dp, *dx, *dy;
  AH_TRY(upload(0, scales + row_start * n_gpr, rows * n_gpr * sizeof(float), &ds));
  AH_TRY(upload(1, packed + b0, b1 - b0, &dp));
  AH_TRY(upload(2, x, cols * sizeof(float), &dx));
  AH_TRY(stage_buf(3, rows * sizeof(float), &dy));
  AH_TRY(gemv_rows_window(static_cast<float*>(dy), static_cast<const float*>(ds), static_cast<const uint8_t*>(dp),
                          static_cast<const float*>(dx), (int64_t)rows, (int64_t)cols, (int64_t)g, (int64_t)row_start,
                          (int64_t)b0, t_stage.stream));
  return finish_download(out, dy, rows * sizeof(float));
}

int ah_host_swiglu_4bit_into(float* out, const float* input, const float* gate_scales, const uint8_t* gate_packed,
                             const float* up_scales, const uint8_t* up_packed, const float* down_scales,
                             const uint8_t* down_packed, size_t n_embd, size_t n_ff, size_t gs, float* scratch_gate,
                             float* scratch_up, float* scratch_act) {
  if (n_embd == 0 && n_ff == 0) return AH_OK;
  AH_REQUIRE(n_embd == 0 || out != nullptr, "host_swiglu_4bit_into: null out");
  AH_REQUIRE(n_ff == 0 || (scratch_gate && scratch_up && scratch_act), "host_swiglu_4bit_into: null scratch");
  const size_t g = gs < 1 ? 1 : gs;
  AH_TRY(stage_ready());
  void *dgs = nullptr, *dgp = nullptr, *dus = nullptr, *dup = nullptr, *dds = nullptr, *ddp = nullptr, *dx = nullptr;
  void *dout = nullptr, *dsg = nullptr, *dsu = nullptr, *dsa = nullptr;
  const size_t ff_sc = n_ff * ((n_embd + g - 1) / g), dn_sc = n_embd * ((n_ff + g - 1) / g);
  if (n_ff && n_embd) {
    AH_REQUIRE(gate_scales && gate_packed && up_scales && up_packed && input, "host_swiglu_4bit_into: null input");
    AH_TRY(upload(0, gate_scales, ff_sc * 4, &dgs));
    AH_TRY(upload(1, gate_packed, (n_ff * n_embd + 1) / 2, &dgp));
    AH_TRY(upload(2, up_scales, ff_sc * 4, &dus));
    AH_TRY(upload(3, up_packed, (n_ff * n_embd + 1) / 2, &dup));
    AH_TRY(upload(4, input, n_embd * 4, &dx));
    AH_REQUIRE(down_scales && down_packed, "host_swiglu_4bit_into: null down weights");
    AH_TRY(upload(5, down_scales, dn_sc * 4, &dds));
    AH_TRY(upload(6, down_packed, (n_embd * n_ff + 1) / 2, &ddp));
  }
  AH_TRY(stage_buf(7, n_embd * 4, &dout));
  AH_TRY(stage_buf(8, n_ff * 4, &dsg));
  AH_TRY(stage_buf(9, n_ff * 4, &dsu));
  AH_TRY(stage_buf(10, n_ff * 4, &dsa));
  AH_TRY(ah_swiglu_4bit_into(static_cast<float*>(dout), static_cast<const float*>(dx), static_cast<const float*>(dgs),
                             static_cast<const uint8_t*>(dgp), static_cast<const float*>(dus),
                             static_cast<const uint8_t*>(dup), static_cast<const float*>(dds),
                             static_cast<const uint8_t*>(ddp), (int64_t)n_embd, (int64_t)n_ff, (int64_t)g,
                             static_cast<float*>(dsg), static_cast<float*>(dsu), static_cast<float*>(dsa),
                             t_stage.stream));
  if (n_ff) {
    AH_CUDA_TRY(cudaMemcpyAsync(scratch_gate, dsg, n_ff * 4, cudaMemcpyDeviceToHost, t_stage.stream));
    AH_CUDA_TRY(cudaMemcpyAsync(scratch_up, dsu, n_ff * 4, cudaMemcpyDeviceToHost, t_stage.stream));
    AH_CUDA_TRY(cudaMemcpyAsync(scratch_act, dsa, n_ff * 4, cudaMemcpyDeviceToHost, t_stage.stream));
  }
  return finish_download(out, dout, n_embd * 4);
}

int ah_host_dequant_layer(const float* scales, const uint8_t* packed, float* result, size_t n, size_t gs) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(scales && packed && result && gs > 0, "host_dequant_layer: bad arguments");
  AH_TRY(stage_ready());
  void *ds, *dp, *dr;
  AH_TRY(upload(0, scales, ((n + gs - 1) / gs) * sizeof(float), &ds));
  AH_TRY(upload(1, packed, (n + 1) / 2, &dp));
  AH_TRY(stage_buf(2, n * sizeof(float), &dr));
  AH_TRY(ah_dequant_layer(static_cast<const float*>(ds), static_cast<const uint8_t*>(dp), static_cast<float*>(dr),
                          (int64_t)n, (int64_t)gs, t_stage.stream));
  return finish_download(result, dr, n * sizeof(float));
}

int ah_host_quantize(const float* weights, size_t n, size_t gs, float* scales, uint8_t* packed) {
  if (n == 0) return AH_OK;
  AH_REQUIRE(weights && scales && packed, "host_quantize: bad arguments");
  const size_t g = gs < 1 ? 1 : gs;
  AH_TRY(stage_ready());
  void *dw, *ds, *dp;
  AH_TRY(upload(0, weights, n * sizeof(float), &dw));
  AH_TRY(stage_buf(1, ((n + g - 1) / g) * sizeof(float), &ds));
  AH_TRY(stage_buf(2, (n + 1) / 2, &dp));
  AH_TRY(ah_quantize_q4(static_cast<const float*>(dw), (int64_t)n, (int64_t)g, static_cast<float*>(ds),
                        static_cast<uint8_t*>(dp), t_stage.stream));
  AH_CUDA_TRY(cudaMemcpyAsync(scales, ds, ((n + g - 1) / g) * sizeof(float), cudaMemcpyDeviceToHost, t_stage.stream));
  return finish_download(packed, dp, (n + 1) / 2);
}

int ah_host_f16_bytes_to_f32(const uint8_t* src, size_t n_bytes, float* out) {
  const size_t n = n_bytes / 2;
  if (n == 0) return AH_OK;
  AH_REQUIRE(src && out, "host_f16_bytes_to_f32: bad arguments");
  AH_TRY(stage_ready());
  void *ds, *dd;
  AH_TRY(upload(0, src, n * 2, &ds));
  AH_TRY(stage_buf(1, n * sizeof(float), &dd));
  AH_TRY(ah_f16_to_f32(static_cast<const uint16_t*>(ds), static_cast<float*>(dd), (int64_t)n, t_stage.stream));
  return finish_download(out, dd, n * sizeof(float));
}

int ah_host_bf16_bytes_to_f32(const uint8_t* src, size_t n_bytes, float* out) {
  const size_t n = n_bytes / 2;
  if (n == 0) return AH_OK;
  AH_REQUIRE(src && out, "host_bf16_bytes_to_f32: bad arguments");
  AH_TRY(stage_ready());
  void *ds, *dd;
  AH_TRY(upload(0, src, n * 2, &ds));
  AH_TRY(stage_buf(1, n * sizeof(float), &dd));
  AH_TRY(ah_bf16_to_f32(static_cast<const uint16_t*>(ds), static_cast<float*>(dd), (int64_t)n, t_stage.stream));
  return finish_download(out, dd, n * sizeof(float));
}

int ah_host_dequantize_to_f32(const uint8_t* raw, size_t raw_bytes, uint32_t dtype, size_t element_count, float* out,
                              size_t* n_out) {
  AH_REQUIRE(n_out && (raw || raw_bytes == 0), "host_dequantize_to_f32: bad arguments");
  AH_TRY(stage_ready());
  void *dr, *dd;
  AH_TRY(upload(0, raw, raw_bytes, &dr));
  const size_t cap = element_count > raw_bytes / 2 ? element_count : raw_bytes / 2;
  AH_TRY(stage_buf(1, cap * sizeof(float), &dd));
  int64_t k = 0;
  AH_TRY(ah_dequantize_to_f32(dr, (int64_t)raw_bytes, dtype, (int64_t)element_count, static_cast<float*>(dd), &k,
                              t_stage.stream));
  *n_out = (size_t)k;
  AH_REQUIRE(out != nullptr || k == 0, "host_dequantize_to_f32: null out");
  return finish_download(out, dd, (size_t)k * sizeof(float));
}

}  // extern "C"
