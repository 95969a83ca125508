/*
 * ah_cuda.h — C ABI of agent_harness_b200, the B200 (sm_100a) implementation of
 * agent_harness's quantized-weight hot path.
 *
 * Every entry point returns an int status (AH_OK = 0, negative on error) and
 * never aborts; ah_last_error() returns the calling thread's last message.
 * Pointers named *_dev are device pointers; `stream` is a cudaStream_t passed
 * as void* (NULL = legacy default stream).  Device-pointer entries are
 * asynchronous on `stream`.  Entries named ah_host_* take HOST slices exactly as
 * the reference's Rust functions do, and are synchronous (upload, compute,
 * download).  "Reference:" lines cite the agent_harness function each entry
 * replaces (paths relative to the agent_harness source tree).
 */
#ifndef AH_CUDA_H
#define AH_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AH_API __attribute__((visibility("default")))
#else
#define AH_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define AH_OK 0
#define AH_EINVAL (-1)       /* bad shape, size, alignment or argument        */
#define AH_ENOMEM (-2)       /* device or pinned allocation failed            */
#define AH_ECUDA (-3)        /* a CUDA runtime call failed                    */
#define AH_ENCCL (-4)        /* an NCCL call failed                           */
#define AH_ETIMEOUT (-5)     /* a bounded device-side wait gave up            */
#define AH_EUNSUPPORTED (-6) /* valid request this build does not implement   */

/* GGML dtype codes accepted by ah_dequantize_to_f32 (formats/gguf.rs:57-74). */
#define AH_DTYPE_F32 0u
#define AH_DTYPE_F16 1u
#define AH_DTYPE_Q4_0 2u
#define AH_DTYPE_Q8_0 8u
#define AH_DTYPE_Q6_K 13u
#define AH_DTYPE_BF16 30u

/* Bytes per 32-element block (types/dtype.rs:69-83). */
#define AH_Q4_0_BLOCK_BYTES 18
#define AH_Q8_0_BLOCK_BYTES 34
#define AH_GROUP_SIZE 32 /* models/quantization.rs:365 GROUP_SIZE */

/* ---- runtime --------------------------------------------------------------- */
AH_API const char* ah_strerror(int status);
AH_API const char* ah_last_error(void);
AH_API int ah_version(void);
/* Makes `device` current for the calling thread and caches its properties. */
AH_API int ah_device_init(int device);
/* Reads and clears the device-side error word that bounded waits set
 * (AH_ETIMEOUT when a wait gave up since the last call). */
AH_API int ah_check_device_error(void* stream);

/* ---- diagnostics (no reference counterpart) --------------------------------- */
/* Device allocations (cudaMalloc) the library has made since it was loaded,
 * over all threads and devices: a caller can check that an entry allocates
 * nothing by reading it before and after the call. */
AH_API int64_t ah_device_alloc_count(void);
/* Host-side failure injection for tests: the nth library call of `kind` from
 * now on (1 = the next one) fails as if the underlying call had failed, and
 * its status travels to the caller as usual (ah_last_error names the
 * injection); nth = 0 disarms.  Nothing is injected on the device. */
#define AH_INJECT_ALLOC 1  /* a device allocation       -> AH_ENOMEM */
#define AH_INJECT_NCCL 2   /* ncclCommInitRank          -> AH_ENCCL  */
#define AH_INJECT_LAUNCH 3 /* a fused GEMV kernel launch -> AH_ECUDA  */
AH_API int ah_debug_inject_failure(int kind, int64_t nth);
/* Runs the tensor-parallel decoder's peer all-reduce step once on caller device
 * buffers: waits (bounded, ~0.4 s) until flags[r] >= *seq for every rank r <
 * world, then hidden[b][i] += sum_r slots[r][i][b] (rank order) and writes the
 * per-16-row sums of squares ss[b][d/16].  A flag that never reaches *seq makes
 * the wait give up: ah_check_device_error then returns AH_ETIMEOUT and hidden
 * is left as it was.  For tests of the bounded wait on one GPU. */
AH_API int ah_debug_residual_add_peer(float* hidden, const float* slots, int world, int batch, int d, float* ss,
                                      const unsigned* flags, const unsigned* seq, void* stream);
/* Diagnostic (no reference counterpart): times 256 back-to-back tcgen05.mma
 * (kind::f16, K = 16, one accumulator) on one SM -- mode 0: A from shared
 * memory, M = 64; mode 1: A from tensor memory, M = 128; mode 2: the CTA-pair
 * form, M = 256 over two SMs (N a multiple of 32).  out_host[0] = issue
 * cycles, [1] = cycles to completion, [2] = nanoseconds to completion.  The
 * batched decode GEMV's design rests on these costs. */
AH_API int ah_debug_tc_mma_rate(int mode, int n, long long* out_host);

/* ---- sizes (models/quantization.rs:423-435) -------------------------------- */
AH_API int64_t ah_packed_bytes(int64_t n_elements);
AH_API int64_t ah_n_groups(int64_t n_elements, int64_t group_size);
AH_API int64_t ah_quantized_bytes(int64_t n_elements, int64_t group_size);

/* ---- conversions (device pointers) ------------------------------------------ */
/* Reference: formats/gguf.rs:93-120 f16_to_f32 (IEEE; NaN -> +-0x7FC00000);
 * also the defined semantics of models/avx512_kernel.rs:212-232 f16_bytes_to_f32. */
AH_API int ah_f16_to_f32(const uint16_t* src_dev, float* dst_dev, int64_t n, void* stream);
/* Reference: formats/gguf.rs:124-126 bf16_to_f32; avx512_kernel.rs:236-255. */
AH_API int ah_bf16_to_f32(const uint16_t* src_dev, float* dst_dev, int64_t n, void* stream);
/* No reference counterpart (the reference never narrows): IEEE RNE f32 -> f16. */
AH_API int ah_f32_to_f16(const float* src_dev, uint16_t* dst_dev, int64_t n, void* stream);

/* ---- block dequantisation (device pointers; bit-exact incl. NaN bits) -------- */
/* Reference: formats/gguf.rs:460-479 (Q8_0 branch of dequantize_to_f32).
 * `blocks_dev` holds ceil(n/32) 34-byte blocks {u16 d; i8 qs[32]}. */
AH_API int ah_dequant_q8_0_f32(const void* blocks_dev, float* out_dev, int64_t n, void* stream);
/* Reference: formats/gguf.rs:480-502 (Q4_0 branch); 18-byte blocks
 * {u16 d; u8 qs[16]}, byte i = element 2i (low nibble), 2i+1 (high nibble). */
AH_API int ah_dequant_q4_0_f32(const void* blocks_dev, float* out_dev, int64_t n, void* stream);
/* Reference: models/quantization.rs:439-454 dequant_layer (scalar semantics,
 * :444-452): out[i] = (nib(i) - 8) * scales[i / group_size]. */
AH_API int ah_dequant_layer(const float* scales_dev, const uint8_t* packed_dev, float* out_dev, int64_t n,
                     int64_t group_size, void* stream);
/* Reference: formats/gguf.rs:434-535 GGUFFile::dequantize_to_f32 — dispatch on
 * the GGML dtype code.  *n_out receives the element count the reference's Vec
 * would hold (F32/F16/BF16: raw_bytes / elem size; Q8_0: limited by raw_bytes;
 * unknown dtype: n zeros).  A truncated Q4_0 block (where the reference panics)
 * returns AH_EINVAL.  Q6_K follows the reference's approximate branch. */
AH_API int ah_dequantize_to_f32(const void* raw_dev, int64_t raw_bytes, uint32_t dtype, int64_t element_count,
                         float* out_dev, int64_t* n_out, void* stream);

/* ---- quantisers (device pointers) -------------------------------------------- */
/* Reference: models/quantization.rs:369-404 quantize (and inference/math.rs:223-253):
 * per group scale = absmax/7 (f32), q = clamp(round(w/scale),-8,7)+8, low nibble =
 * even index.  scales_dev: ceil(n/gs) floats; packed_dev: ceil(n/2) bytes. */
AH_API int ah_quantize_q4(const float* w_dev, int64_t n, int64_t group_size, float* scales_dev, uint8_t* packed_dev,
                   void* stream);
/* No reference quantiser exists for these block formats (their dequant is
 * formats/gguf.rs:459-502): d = f16(absmax/127), q = clamp(round(w/d),-127,127). */
AH_API int ah_quantize_q8_0(const float* w_dev, int64_t n, void* blocks_dev, void* stream);
/* d = f16(absmax/8), q = clamp(round(w/d)+8, 0, 15), reference nibble order. */
AH_API int ah_quantize_q4_0(const float* w_dev, int64_t n, void* blocks_dev, void* stream);

/* ---- synthetic data (no reference counterpart: seeded benchmark inputs) -------- */
/* out[i] = mean + std * N(0,1) from a counter-based generator keyed by (seed, i + index_offset). */
AH_API int ah_fill_normal(float* out_dev, int64_t n, float mean, float std, uint64_t seed, int64_t index_offset,
                   void* stream);
/* Rows [row0, row0+rows) and columns [col0, col0+cols) of a logical matrix with
 * `full_cols` columns drawn as ah_fill_normal(seed) in row-major order, quantised
 * straight to Q4_0 blocks (cols % 32 == 0, col0 % 32 == 0). */
AH_API int ah_synth_q4_0(void* blocks_dev, int64_t row0, int64_t rows, int64_t col0, int64_t cols, int64_t full_cols,
                  float std, uint64_t seed, void* stream);
/* Same for f16 values mean + std*N(0,1) (embeddings, norm weights). */
AH_API int ah_synth_f16(uint16_t* out_dev, int64_t n, float mean, float std, uint64_t seed, int64_t index_offset,
                 void* stream);

/* ---- fused Q4 GEMV ------------------------------------------------------------ */
/* Opaque device-resident quantised weight in the GEMV's tiled layout (rows
 * padded to 16, columns to 64; nibbles and scales in separate planes). */
typedef struct AhQ4Weight AhQ4Weight;

/* Reference: inference/mod.rs:184-314 decompress_all_parallel's per-tensor
 * quantise + store step — here an upload-and-repack of an already-quantised
 * tensor into device memory owned by the handle.  Source pointers are DEVICE
 * pointers in the reference formats. */
AH_API int ah_q4w_from_q4_0(const void* blocks_dev, int64_t rows, int64_t cols, AhQ4Weight** out, void* stream);
AH_API int ah_q4w_from_engine(const float* scales_dev, const uint8_t* packed_dev, int64_t rows, int64_t cols,
                       AhQ4Weight** out, void* stream);
AH_API int ah_q4w_destroy(AhQ4Weight* w);
AH_API int ah_q4w_shape(const AhQ4Weight* w, int64_t* rows, int64_t* cols);
/* Bytes the algorithm must read per GEMV (nibbles + scales, unpadded). */
AH_API int64_t ah_q4w_weight_bytes(const AhQ4Weight* w);
/* Reference: inference/math.rs:255-295 gemv_4bit_into(out, ..., x, ...) with
 * host slices, for a weight already resident: copies x_host [batch][cols] to
 * the device, runs ah_q4w_gemv, copies y_host [batch][rows] back and waits for
 * the stream.  Pinned (device-mapped) host buffers are read and written by the
 * kernels over the bus, the pull of x and the GEMV replayed as one graph while
 * the caller keeps passing the same buffers; pageable ones go through the copy
 * engine.  The
 * device staging is allocated on the first call for each weight; calls on one
 * weight from several host threads are serialised. */
AH_API int ah_q4w_gemv_host(const AhQ4Weight* w, const float* x_host, float* y_host, int batch, void* stream);
/* Read-only view of a resident weight's device planes (no reference
 * counterpart): the tiled nibbles, the scales (f16x4 or, for f32_scales,
 * float4 per row pair of a block pair) and their sizes in bytes. */
AH_API int ah_q4w_planes(const AhQ4Weight* w, const void** nib, size_t* nib_bytes, const void** scales,
                         size_t* scale_bytes, int* f32_scales);

/* Reference: inference/math.rs:255-295 gemv_4bit_into (batch 1) and its
 * token-by-token use in inference/mod.rs:411-538, batched to `batch` <= 16
 * tokens: y[b][r] = sum_j W[r][j] * x[b][j], f32 accumulate, dequantised
 * weights never written to memory.  x_dev: [batch][cols] f32, y_dev: [batch][rows].
 */
AH_API int ah_q4w_gemv(const AhQ4Weight* w, const float* x_dev, float* y_dev, int batch, void* stream);

/* ---- prefill GEMM (tcgen05 tensor cores) -------------------------------------------- */
/* Reference: the prompt prefill of inference/mod.rs:547-562, which runs
 * forward() token by token (mod.rs:550) and so one inference/math.rs:255-295
 * gemv_4bit_into per token and projection; here all m tokens at once:
 * c[i][r] = sum_j W[r][j] * a[i][j], a_dev [m][lda] f32 (lda >= cols), c_dev
 * [m][ldc] f32 (ldc >= rows).  Tensor-core operands are f16: W as d*(q-8)
 * rounded once, a per row scaled by a power of two into f16 range; f32
 * accumulation.  `workspace_dev` (1024-byte aligned, at least
 * ah_q4w_gemm_workspace_bytes(w, m) bytes) holds the converted activations;
 * calls on different streams need different workspaces.  m == 0 is a no-op. */
AH_API int ah_q4w_gemm_workspace_bytes(const AhQ4Weight* w, int64_t m, size_t* bytes);
AH_API int ah_q4w_gemm(const AhQ4Weight* w, const float* a_dev, int64_t lda, int64_t m, float* c_dev, int64_t ldc,
                       void* workspace_dev, size_t workspace_bytes, void* stream);
/* ah_q4w_gemm with the prefill step's fusions, for an engine that runs a
 * block's projections over many tokens:
 *   norm_w_dev (f16 bits, cols entries; may be null): each a row is first
 *     RMS-normalised, inference/math.rs:53-63 rms_norm_into with `eps`;
 *   epilogue 0: c = a . W^T;
 *   epilogue 1: w is an interleaved gate/up weight (ah_q4w_from_*_gate_up,
 *     2 * n_ff rows) and c [m][ldc >= n_ff] = silu(gate) * up, the
 *     activation of inference/ffn.rs:155-174 swiglu_4bit_into for every row;
 *   epilogue 2: c += a . W^T, the residual adds of inference/mod.rs:505-545
 *     (an f32 add per element; subnormal sums flush to zero).
 * Same precision and workspace as ah_q4w_gemm. */
AH_API int ah_q4w_gemm_ex(const AhQ4Weight* w, const float* a_dev, int64_t lda, int64_t m, float* c_dev, int64_t ldc,
                          int epilogue, const uint16_t* norm_w_dev, float eps, void* workspace_dev,
                          size_t workspace_bytes, void* stream);
/* No counterpart in the reference: ah_q4w_gemm without a caller workspace.  The
 * workspace lives in a fixed 8 MiB static device buffer per device (at 4096
 * columns: up to 768 tokens); larger requests return AH_EINVAL before any
 * launch.  Calls that overlap in time on one device race on that buffer.  The
 * call allocates nothing, on its first call on a device (even before
 * ah_device_init) as on later ones: the buffer and the device error word are
 * module variables whose addresses are looked up, not allocated. */
AH_API int ah_q4w_gemm_noalloc(const AhQ4Weight* w, const float* a_dev, int64_t lda, int64_t m, float* c_dev,
                               int64_t ldc, void* stream);

/* Replaces, for 1..16 tokens at once, the reference's gemv_4bit_into
 * (inference/math.rs:255-295) per token, like ah_q4w_gemv, on the 5th-
 * generation tensor cores: y_dev[b][y_stride] (+)= W . x_dev[b][x_stride] for
 * b < batch.  W is dequantised as d*(q-8) rounded once to f16 and each x row is
 * scaled by a power of two and rounded to f16 (the ah_q4w_gemm precision); f32
 * accumulation.  accumulate != 0 adds into y instead of storing.
 * `workspace_dev` (1024-byte aligned, at least ah_q4w_gemv_tc_workspace_bytes(w)
 * bytes) holds the converted tokens and the partial sums of row blocks that
 * several CTAs share; calls on different streams need different workspaces. */
AH_API int ah_q4w_gemv_tc_workspace_bytes(const AhQ4Weight* w, size_t* bytes);
AH_API int ah_q4w_gemv_tc(const AhQ4Weight* w, const float* x_dev, int64_t x_stride, int batch, float* y_dev,
                          int64_t y_stride, int accumulate, void* workspace_dev, size_t workspace_bytes,
                          void* stream);

/* Reference: inference/math.rs:255-295 gemv_4bit_into on the engine format as
 * stored (f32 scales [rows][ceil(cols/gs)], linear nibbles), device pointers, any
 * group size; empty input -> zero output (math.rs:264-267). */
AH_API int ah_gemv_4bit_into(float* out_dev, const float* scales_dev, const uint8_t* packed_dev, const float* x_dev,
                      int64_t rows, int64_t cols, int64_t group_size, void* stream);
/* Reference: inference/math.rs:205-214 matvec_4bit_into (square). */
AH_API int ah_matvec_4bit_into(float* out_dev, const float* scales_dev, const uint8_t* packed_dev, const float* x_dev,
                        int64_t dim, int64_t group_size, void* stream);

/* Reference: inference/math.rs:382-418 gemv_4bit_parallel_worker_scalar(out,
 * global_scales, global_packed, x, row_start, row_end, cols, gs): rows
 * [row_start, row_end) of the engine-format matrix whose full planes are
 * scales_dev / packed_dev; out_dev holds row_end - row_start values. */
AH_API int ah_gemv_4bit_rows(float* out_dev, const float* scales_dev, const uint8_t* packed_dev, const float* x_dev,
                             int64_t row_start, int64_t row_end, int64_t cols, int64_t group_size, void* stream);

/* ---- SwiGLU feed-forward block ------------------------------------------------------ */
/* Reference: inference/ffn.rs:155-174 swiglu_4bit_into (the quantized branch of
 * FfnBlock::forward, ffn.rs:72-111), device pointers, engine format as stored,
 * any group size: scratch_gate = gate.input, scratch_up = up.input (one fused
 * pass over input), scratch_act = silu(gate) * up, out = down.scratch_act.
 * gate/up: [n_ff][n_embd]; down: [n_embd][n_ff]. */
AH_API int ah_swiglu_4bit_into(float* out_dev, const float* input_dev, const float* gate_scales_dev,
                               const uint8_t* gate_packed_dev, const float* up_scales_dev,
                               const uint8_t* up_packed_dev, const float* down_scales_dev,
                               const uint8_t* down_packed_dev, int64_t n_embd, int64_t n_ff, int64_t group_size,
                               float* scratch_gate_dev, float* scratch_up_dev, float* scratch_act_dev, void* stream);
/* The same block on resident tiled weights, as the decoder runs it: gate and up
 * interleaved in one weight (8 rows of each per 16-row tile) so one fused GEMV
 * writes act = silu(gate) * up straight from its epilogue, then the down GEMV.
 * Built from the engine format (group 32) or Q4_0 blocks; n_ff % 8 == 0.
 * x [batch][n_embd] -> act [batch][n_ff] -> out [batch][n_embd], batch <= 16. */
AH_API int ah_q4w_from_engine_gate_up(const float* gate_scales_dev, const uint8_t* gate_packed_dev,
                                      const float* up_scales_dev, const uint8_t* up_packed_dev, int64_t n_ff,
                                      int64_t n_embd, AhQ4Weight** out, void* stream);
AH_API int ah_q4w_from_q4_0_gate_up(const void* gate_blocks_dev, const void* up_blocks_dev, int64_t n_ff,
                                    int64_t n_embd, AhQ4Weight** out, void* stream);
AH_API int ah_q4w_swiglu(const AhQ4Weight* gate_up, const AhQ4Weight* down, const float* x_dev, float* act_dev,
                         float* out_dev, int batch, void* stream);

/* ---- Llama-shaped decoder ----------------------------------------------------------- */
/* Reference: inference/config.rs:6-58 ModelConfig (the fields the decoder uses;
 * rope sections default to [head_dim/2, 0, 0, 0] as config.rs:170-172 does). */
typedef struct {
  int32_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, vocab_size;
  int32_t max_seq;    /* KV-cache capacity per sequence (inference/kv_cache.rs:24 uses 4096) */
  int32_t max_batch;  /* sequences decoded together, 1..16 */
  float rope_freq_base, rms_eps;
} AhModelConfig;

typedef struct AhModel AhModel;

/* Tensor kinds for ah_model_load_tensor (GGUF names in inference/mod.rs:392-538). */
#define AH_T_TOK_EMBD 0   /* token_embd.weight   f16 [vocab][n_embd]             */
#define AH_T_ATTN_NORM 1  /* blk.L.attn_norm     f16 [n_embd]                    */
#define AH_T_FFN_NORM 2   /* blk.L.ffn_norm      f16 [n_embd]                    */
#define AH_T_OUT_NORM 3   /* output_norm.weight  f16 [n_embd]                    */
#define AH_T_WQ 4         /* blk.L.attn_q        Q4_0 [n_head*head_dim][n_embd]  */
#define AH_T_WK 5         /* blk.L.attn_k        Q4_0 [n_head_kv*head_dim][n_embd] */
#define AH_T_WV 6         /* blk.L.attn_v        Q4_0 [n_head_kv*head_dim][n_embd] */
#define AH_T_WO 7         /* blk.L.attn_output   Q4_0 [n_embd][n_head*head_dim]  */
#define AH_T_WGATE 8      /* blk.L.ffn_gate      Q4_0 [n_ff][n_embd]             */
#define AH_T_WUP 9        /* blk.L.ffn_up        Q4_0 [n_ff][n_embd]             */
#define AH_T_WDOWN 10     /* blk.L.ffn_down      Q4_0 [n_embd][n_ff]             */
#define AH_T_LM_HEAD 11   /* output.weight       Q4_0 [vocab][n_embd]            */

/* Reference: inference/mod.rs:70-331 InferenceEngine::open_with_progress's
 * device side: allocates the weight arena, f16 KV cache [batch][layer][kv_head]
 * [max_seq][head_dim] and activations on the current device. */
AH_API int ah_model_create(const AhModelConfig* cfg, AhModel** out);
/* Tensor parallelism (no reference counterpart: the reference runs on one CPU).
 * Rank `rank` of `world` (one process or thread per GPU, each with its own
 * current device) holds heads [rank*n_head/world, ...), the matching kv heads,
 * FFN rows and vocab rows: q/k/v, gate/up and the LM head are split by rows,
 * o and down by columns, with one NCCL all-reduce per attention and MLP block
 * and an all-gather of per-shard argmax candidates.  `nccl_id` is the
 * 128-byte id from ah_nccl_unique_id on one rank, shared by the caller.
 * world must divide n_head_kv, n_ff and vocab_size.  ah_model_load_tensor then
 * takes this rank's slices; ah_model_forward writes this rank's vocab slice
 * of the logits [batch][vocab/world]; generated tokens are identical on all
 * ranks.  ah_model_create(cfg) equals ah_model_create_tp(cfg, 0, 1, ...). */
AH_API int ah_nccl_unique_id(void* id_out, size_t bytes);
AH_API int ah_model_create_tp(const AhModelConfig* cfg, int rank, int world, const void* nccl_id, AhModel** out);
/* Block all-reduce over NVLink peer memory instead of NCCL (no reference
 * counterpart): the o / down GEMVs store their partials straight into every
 * rank's receive slots, a flag per rank publishes completion, and each rank
 * sums the slots in rank order (bounded waits; a missing rank gives
 * AH_ETIMEOUT from ah_check_device_error).  Every rank passes its 64-byte
 * ah_model_ipc_handle to all ranks; ah_model_ipc_open takes the world's handles
 * in rank order.  Ranks must be processes on GPUs with peer access. */
AH_API int ah_model_ipc_handle(AhModel* m, void* handle_out, size_t bytes);
AH_API int ah_model_ipc_open(AhModel* m, const void* handles, size_t bytes);
/* Loads a projection (AH_T_WQ .. AH_T_LM_HEAD) in the engine format that
 * models/quantization.rs:369-404 quantize(weights, 32) returns: scales_dev
 * [rows * cols / 32] f32 and packed_dev [rows * cols / 2] (even element in the
 * low nibble), as inference/mod.rs:255-271 writes them per tensor.  The GEMVs
 * then run on f32 scales (inference/math.rs:255-418 arithmetic).  q/k/v and
 * gate/up of a layer must share one format. */
AH_API int ah_model_load_tensor_engine(AhModel* m, int kind, int layer, const float* scales_dev,
                                       const uint8_t* packed_dev, void* stream);
/* Loads an f32 tensor as the reference's loader does (inference/mod.rs:255-271):
 * projections are quantized on the device with quantize(weights, 32) and
 * loaded in the engine format; embeddings and norms are stored as f16 (round
 * to nearest even), the decoder's storage for them. */
AH_API int ah_model_load_tensor_f32(AhModel* m, int kind, int layer, const float* data_dev, void* stream);
/* This rank's shard: heads, kv heads, FFN rows and vocab rows it holds. */
AH_API int ah_model_shard(const AhModel* m, int* rank, int* world, int* n_head, int* n_head_kv, int* n_ff,
                          int* vocab);
AH_API int ah_model_destroy(AhModel* m);
/* Loads one tensor from device memory (f16 bits or Q4_0 blocks, per kind);
 * Q4_0 projections are repacked into the GEMV layout (q|k|v fused, gate/up
 * interleaved).  Layer is ignored for the model-level kinds. */
AH_API int ah_model_load_tensor(AhModel* m, int kind, int layer, const void* data_dev, void* stream);
/* Seeded synthetic weights (no reference counterpart): every projection Q4_0 of
 * N(0, w_std), embeddings f16 N(0, emb_std), norm weights f16 1 + N(0, norm_std);
 * tensor t of layer l draws from seed ah_model_tensor_seed(seed, kind, l). */
AH_API int ah_model_init_random(AhModel* m, uint64_t seed, float w_std, float emb_std, float norm_std);
AH_API uint64_t ah_model_tensor_seed(uint64_t seed, int kind, int layer);
/* Reference: inference/mod.rs:547-562 generate with temperature 0 (greedy,
 * sampling.rs:4-14 argmax), for `batch` sequences in lock step.  `prompt` is
 * [batch][n_prompt] host int32; the prompt is consumed as ah_model_set_prefill
 * selects (GEMM prefill by default, or forward() token by token as the
 * reference does, mod.rs:550), then `n_new` greedy steps write their tokens to
 * `out_tokens` [n_new][batch] (host).  Resets the KV cache. */
AH_API int ah_model_generate(AhModel* m, const int32_t* prompt, int batch, int n_prompt, int n_new,
                             int32_t* out_tokens, void* stream);
/* How ah_model_generate consumes the prompt (no reference counterpart: the
 * reference always runs one forward() per prompt token, inference/mod.rs:550).
 * mode 1 (default): prompts of 9 tokens or more go through the prefill GEMMs
 * (tcgen05) in chunks of up to 2048 rows (sequences x positions) with a causal
 * attention over the f16 KV cache, and the last prompt token through the
 * decode step; mode 0: token by token, as the reference.  Both leave the same
 * state (KV cache, position) up to rounding. */
AH_API int ah_model_set_prefill(AhModel* m, int mode);
/* Which GEMV the decode steps use (no reference counterpart): in steps of at
 * least `min_batch` sequences (default 9) a projection runs on the tcgen05
 * batched GEMV (ah_q4w_gemv_tc precision: f16 operands, f32 accumulation)
 * where that is the faster one -- from 20 MB of Q4 weights at 9-12 sequences,
 * 5 MB at 13-16 -- and on the mma.sync GEMV (ah_q4w_gemv)
 * otherwise.  1: every projection of every step on the tcgen05 GEMV; 17:
 * never. */
AH_API int ah_model_set_batched_gemv(AhModel* m, int min_batch);
/* Next-token choice of the decode steps.  temperature 0 (the default): greedy,
 * sampling.rs:4-14.  temperature > 0: inference/mod.rs:552-553 with top_k
 * (the reference passes 40; 1..64 here): the top_k logits of each sequence,
 * then sampling.rs:17-64's exp / sum / CDF scan in the reference's order, with
 * the uniform r = ah_sample_uniform(seed, position, sequence) in place of the
 * reference's clock-seeded xorshift (sampling.rs:67-86), so runs repeat.
 * Under tensor parallelism every rank picks the same token. */
AH_API int ah_model_set_sampling(AhModel* m, float temperature, int top_k, uint64_t seed);
/* Lower-level stepping (same semantics): reset, feed one token per sequence
 * (forward(), inference/mod.rs:333-545) and read the logits [batch][vocab]. */
AH_API int ah_model_reset(AhModel* m, int batch, void* stream);
AH_API int ah_model_forward(AhModel* m, const int32_t* tokens_dev, float* logits_dev, void* stream);
/* Runs `n` greedy decode steps from the current state as one CUDA graph per
 * step (captured on first use); the first step consumes the argmax of the
 * last forward's logits.  Tokens land in out_tokens_dev [n][batch]. */
AH_API int ah_model_decode(AhModel* m, int n, int32_t* out_tokens_dev, void* stream);
/* Current position (tokens consumed per sequence). */
AH_API int ah_model_position(const AhModel* m, int* pos);

/* ---- Sampling (inference/sampling.rs) ----------------------------------------------
 * Replaces sampling.rs:17-64 sample(logits, temperature, top_k) for `batch`
 * rows of logits_dev [batch][ld] (device f32, vocab <= ld): out_dev[b] (device
 * int32) = the token that sample() returns for row b when its rand_val() draw
 * is ah_sample_uniform(seed, step, b).  top_k in 1..64; temperature > 0.
 * Candidates are ranked by logit, ties by lower index.  With a device
 * workspace of ah_sample_workspace_bytes(batch, vocab) bytes (16-byte
 * aligned; any contents; one per stream) rows of 8192 logits or more are
 * split over CTAs of 4096 logits (0 bytes: no split at this vocabulary); with
 * workspace null, one CTA takes each row (large batches).  Both give the same
 * tokens. */
AH_API size_t ah_sample_workspace_bytes(int batch, int64_t vocab);
AH_API int ah_sample_logits(const float* logits_dev, int64_t ld, int batch, int64_t vocab, float temperature,
                            int top_k, uint64_t seed, int64_t step, int32_t* out_dev, void* workspace,
                            size_t workspace_bytes, void* stream);
/* The uniform draw in [0, 1) (24 bits, as sampling.rs:84-85 maps its xorshift
 * state) of sequence `seq` at step `step`: a counter-based hash of the three. */
AH_API float ah_sample_uniform(uint64_t seed, int64_t step, int seq);

/* ---- DedupCount weight decoding (models/dedup/) --------------------------------------
 * A decode table holds one tensor's lookups flattened to f32 values on the
 * device; the sandbag arrays (prefix_idx, tail_idx: u16; sign_bits: one bit per
 * element, LSB first) are device arrays that may be shorter than `count`
 * (missing entries read 0, as the reference's .get(i).unwrap_or(0) does). */
typedef struct AhDedupTable AhDedupTable;
/* Replaces the per-element arithmetic of dedup/decompressor.rs:7-27
 * DedupCountTensor::decompress_all: prefix_int / 10^pd + tail / 10^(pd+td). */
AH_API int ah_dedup_table_local(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values, int64_t n_tail,
                                int prefix_digits, int tail_digits, float avg_precision_lost, AhDedupTable** out);
/* Replaces dedup/decompressor.rs:29-85 DedupCountTensor::decompress_all_global's
 * prefix and tail lookups against a GlobalTable (dedup/types.rs:23-28) given as
 * g_prefixes[n_gp] and tails_for_prefix in CSR form (g_tail_off[n_gp + 1]). */
AH_API int ah_dedup_table_global(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values,
                                 int64_t n_tail, int prefix_digits, int tail_digits, float avg_precision_lost,
                                 int g_prefix_digits, const float* g_prefixes, int64_t n_gp, const uint32_t* g_tail_off,
                                 const uint32_t* g_tails, AhDedupTable** out);
/* Replaces dedup/global_lookup.rs:89-113 GlobalTable::decompress_with_remap's
 * lookups for a ChunkRemap (global_tail_indices = remap[n_remap]).  A prefix
 * index past the tensor's prefixes (a panic in the reference) sets the device
 * error word: ah_check_device_error then returns AH_EINVAL. */
AH_API int ah_dedup_table_remap(const uint16_t* prefixes, int64_t n_prefix, int prefix_digits, int tail_digits,
                                float avg_precision_lost, int g_prefix_digits, const float* g_prefixes, int64_t n_gp,
                                const uint32_t* g_tail_off, const uint32_t* g_tails, const uint16_t* remap,
                                int64_t n_remap, AhDedupTable** out);
AH_API int ah_dedup_table_destroy(AhDedupTable* t);
/* decompress_all / decompress_all_global / decompress_with_remap on device
 * arrays: out[count] f32 (count: the tensor's count; for a remap table, the
 * sandbag's count, and the arrays must hold that many entries). */
AH_API int ah_dedup_decompress_f32(const AhDedupTable* t, const uint16_t* prefix_idx, int64_t n_prefix_idx,
                                   const uint16_t* tail_idx, int64_t n_tail_idx, const uint8_t* sign_bits,
                                   int64_t n_sign_bytes, int64_t count, float* out, void* stream);
/* Load path of inference/mod.rs:255-271 (decompress_tensor_global_single, then
 * quantization.rs:369-404 quantize with group 32) in one pass: decodes a
 * [rows][cols] tensor (cols % 32 == 0) and writes a resident engine-format
 * weight (f32 scales) in the GEMV's tiled layout, bit-identical to quantize()
 * of the decoded values followed by ah_q4w_from_engine. */
AH_API int ah_dedup_to_q4w(const AhDedupTable* t, const uint16_t* prefix_idx, int64_t n_prefix_idx,
                           const uint16_t* tail_idx, int64_t n_tail_idx, const uint8_t* sign_bits,
                           int64_t n_sign_bytes, int64_t rows, int64_t cols, AhQ4Weight** out, void* stream);
/* The same into an existing engine-format weight of the tensor's shape (a
 * resident arena slot reloaded in place; allocates nothing). */
AH_API int ah_dedup_into_q4w(const AhDedupTable* t, const uint16_t* prefix_idx, int64_t n_prefix_idx,
                             const uint16_t* tail_idx, int64_t n_tail_idx, const uint8_t* sign_bits,
                             int64_t n_sign_bytes, AhQ4Weight* w, void* stream);

/* ---- paged virtual tensor arena (memory_controller/virtual_tensor_arena.rs) ------------ */
/* Page residency (PageResidency, virtual_tensor_arena.rs:5-10). */
#define AH_PAGE_UNMAPPED 0
#define AH_PAGE_GPU 1
#define AH_PAGE_CPU 2
typedef struct AhArena AhArena;
/* Minimum page size (the device's physical allocation granularity). */
AH_API int ah_arena_page_granularity(size_t* bytes);
/* Replaces VirtualTensorArena::new (:34-68): a reserved virtual range of
 * total_virtual_bytes on the current device in pages of page_bytes, all
 * unmapped.  gpu_page_budget caps GPU-resident pages (-1: no cap); a commit
 * past it is routed to the host as an out-of-memory commit is. */
AH_API int ah_arena_create(size_t total_virtual_bytes, size_t page_bytes, int64_t gpu_page_budget, AhArena** out);
AH_API int ah_arena_destroy(AhArena* a);
/* Replaces commit_page (:70-140): maps physical GPU memory at the page's fixed
 * address, or routes the page to the host pool on out-of-memory (:142-147);
 * pages already committed are left as they are. */
AH_API int ah_arena_commit_page(AhArena* a, int64_t page);
/* Replaces evict_page (:149-212): move != 0 copies a GPU page's bytes into
 * host_pool + page * page_bytes and marks it host resident; move == 0 drops
 * it (unmapped).  Waits for the device first: nothing may still use the page. */
AH_API int ah_arena_evict_page(AhArena* a, int64_t page, int move, void* host_pool, void* stream);
/* The page's residency and, when GPU resident, its device address. */
AH_API int ah_arena_page_state(const AhArena* a, int64_t page, int* residency, void** dev_ptr);
/* Replaces execute_layer_math (:216-257): gemv_4bit_into (inference/math.rs:
 * 255-295) with the page's bytes as `packed`, on the device either way: a GPU
 * page through its address, a host page through host_pool (pinned) over the
 * bus.  out, scales and x are device pointers; an unmapped page is AH_EINVAL. */
AH_API int ah_arena_gemv_4bit(AhArena* a, int64_t page, const void* host_pool, float* out, const float* scales,
                              const float* x, int64_t rows, int64_t cols, int64_t group_size, void* stream);

/* ---- gated delta-net SSM block (inference/ssm.rs) ------------------------------------ */
/* ModelConfig's SSM fields (inference/config.rs:31-39): head_k_dim = d_state,
 * num_k_heads = n_group, num_v_heads = dt_rank, head_v_dim = d_inner / dt_rank
 * (must equal d_state), conv kernel d_conv. */
typedef struct {
  int32_t n_embd, d_state, n_group, dt_rank, d_inner, d_conv;
  float rms_eps;
} AhSsmConfig;
/* SsmBlock's weights (ssm.rs:25-44), device f32, row-major as the reference
 * multiplies them: wqkv [conv_dim][n_embd], wqkv_gate [value_dim][n_embd],
 * conv1d [conv_dim][d_conv], dt_bias / a [dt_rank], alpha / beta
 * [dt_rank][n_embd], norm [head_v_dim], out [n_embd][value_dim]
 * (conv_dim = 2 * n_group * d_state + value_dim, value_dim = d_inner). */
typedef struct {
  const float *wqkv, *wqkv_gate, *conv1d, *dt_bias, *a, *alpha, *beta, *norm, *out;
} AhSsmWeights;
/* Device workspace one step needs (caller-allocated, 16-byte aligned, any
 * contents).  It holds the step's intermediates and per-head completion
 * counters, so one workspace serves one step at a time: steps that share it run
 * on one stream. */
AH_API int ah_ssm_workspace_bytes(const AhSsmConfig* cfg, size_t* bytes);
/* Replaces inference/ssm.rs:171-296 SsmBlock::forward(input, state, config):
 * one token, x [n_embd] -> out [n_embd], updating the state in place:
 * conv_state [(d_conv - 1)][conv_dim] and ssm_state [dt_rank][d_state][d_state]
 * (SsmState::new zero-initialises both, ssm.rs:78-91).  head_dim at most 256. */
AH_API int ah_ssm_forward(const AhSsmConfig* cfg, const AhSsmWeights* w, float* conv_state, float* ssm_state,
                          const float* x, float* out, void* workspace, size_t workspace_bytes, void* stream);

/* ---- host-slice drop-ins (synchronous; reference signatures) ---------------------- */
/* Reference: dedup/decompressor.rs:7-27 DedupCountTensor::decompress_all(&self,
 * sandbag) -> Vec<f32> (count = self.count; host arrays in, out[count]). */
AH_API int ah_host_dedup_decompress_all(const uint16_t* prefixes, int64_t n_prefix, const uint16_t* tail_values,
                                        int64_t n_tail, int64_t count, int prefix_digits, int tail_digits,
                                        float avg_precision_lost, const uint16_t* prefix_idx, int64_t n_prefix_idx,
                                        const uint16_t* tail_idx, int64_t n_tail_idx, const uint8_t* sign_bits,
                                        int64_t n_sign_bytes, float* out);
/* Reference: inference/math.rs:255-295 gemv_4bit_into(out, scales, packed, x, rows, cols, gs). */
AH_API int ah_host_gemv_4bit_into(float* out, const float* scales, const uint8_t* packed, const float* x, size_t rows,
                           size_t cols, size_t group_size);
/* Reference: inference/math.rs:382-418 gemv_4bit_parallel_worker_scalar(out, global_scales,
 * global_packed, x, row_start, row_end, cols, gs); out[row_end - row_start]. */
AH_API int ah_host_gemv_4bit_worker_scalar(float* out, const float* scales, const uint8_t* packed, const float* x,
                                           size_t row_start, size_t row_end, size_t cols, size_t group_size);
/* Reference: inference/ffn.rs:155-174 swiglu_4bit_into(out, input, gate_scales, gate_packed,
 * up_scales, up_packed, down_scales, down_packed, n_embd, n_ff, gs, scratch_gate, scratch_up,
 * scratch_act); the three scratch slices receive the reference's intermediates. */
AH_API int ah_host_swiglu_4bit_into(float* out, const float* input, const float* gate_scales,
                                    const uint8_t* gate_packed, const float* up_scales, const uint8_t* up_packed,
                                    const float* down_scales, const uint8_t* down_packed, size_t n_embd, size_t n_ff,
                                    size_t group_size, float* scratch_gate, float* scratch_up, float* scratch_act);
/* Reference: models/quantization.rs:439-454 dequant_layer(scales, packed, result, gs). */
AH_API int ah_host_dequant_layer(const float* scales, const uint8_t* packed, float* result, size_t n, size_t group_size);
/* Reference: models/quantization.rs:369-404 quantize(weights, gs) -> (scales, packed). */
AH_API int ah_host_quantize(const float* weights, size_t n, size_t group_size, float* scales, uint8_t* packed);
/* Reference: models/avx512_kernel.rs:212-232 f16_bytes_to_f32 (defined semantics). */
AH_API int ah_host_f16_bytes_to_f32(const uint8_t* src, size_t n_bytes, float* out);
/* Reference: models/avx512_kernel.rs:236-255 bf16_bytes_to_f32. */
AH_API int ah_host_bf16_bytes_to_f32(const uint8_t* src, size_t n_bytes, float* out);
/* Reference: formats/gguf.rs:434-535 GGUFFile::dequantize_to_f32(raw, dtype, n). */
AH_API int ah_host_dequantize_to_f32(const uint8_t* raw, size_t raw_bytes, uint32_t dtype, size_t element_count,
                              float* out, size_t* n_out);

#ifdef __cplusplus
}
#endif
#endif /* AH_CUDA_H */
