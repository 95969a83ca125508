// ah_prefill.cuh — the row kernels of the decoder's prompt prefill (many
// tokens per launch, the projections run as tcgen05 GEMMs): embedding rows,
// RMSNorm rows, RoPE + f16 KV-cache append, causal attention over the cache,
// residual add and SwiGLU of the interleaved gate/up output.
#pragma once

#include "ah_common.cuh"

namespace ah {

// Prompt rows r = b * cnt + i hold token prompt[b * n_prompt + p0 + i].
struct PrefillRows {
  int batch;     // sequences
  int cnt;       // positions of this chunk per sequence
  int p0;        // first position of the chunk
  int n_prompt;  // prompt length (row stride of the prompt array)
};

// hidden[r] = f16 -> f32 (token_embd[token of row r]) (inference/mod.rs:392-397)
int prefill_embed(const uint16_t* emb, const int* prompt, const PrefillRows& pr, int d, int vocab, float* hidden,
                  cudaStream_t st);
// RoPE (per head, adjacent pairs) on q in place and on k; k and v rounded to
// f16 into the cache at positions p0 + i: cache [B][L][nkv][max_seq][hd]
int prefill_rope_append(float* qkv, int ld, const float2* rope, uint16_t* kc, uint16_t* vc, int layer, int n_layer,
                        int nh, int nkv, int hd, int max_seq, const PrefillRows& pr, cudaStream_t st);
// out[r][hq*hd + c] = sum_{j <= p} softmax_j(q . k_j * scale) v_j over the
// cache rows of row r's sequence (inference/mod.rs:469-502, GQA kv head hq / G)
int prefill_attention(const float* qkv, int ld, const uint16_t* kc, const uint16_t* vc, int layer, int n_layer,
                      int nh, int nkv, int hd, int max_seq, float scale, const PrefillRows& pr, float* out,
                      int ld_out, cudaStream_t st);
// hidden += part
int prefill_add(float* hidden, const float* part, int64_t n, cudaStream_t st);

}  // namespace ah
