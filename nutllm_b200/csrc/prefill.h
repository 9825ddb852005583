#pragma once
/* Row-wise kernels of the batched prefill (prefill.cu); fp16 buffers are
 * passed as uint16_t. */
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace nut {

cudaError_t gather_rows(const float *emb, const int32_t *tokens, int M, int dim, int vocab,
                        float *h, cudaStream_t s);
/* out[m][k] = fp16(rmsnorm(h[m]) * w) for k < dim, 0 for dim <= k < Kp. */
cudaError_t rmsnorm_rows(const float *h, const float *w, int M, int dim, int Kp, uint16_t *out,
                         cudaStream_t s);
/* RoPE of q and k rows of qkv [M][ldq] in place, k and v rows appended to
 * the cache at positions start .. start + M - 1. */
cudaError_t rope_kv_rows(float *qkv, int M, int ldq, int start, const float *rope_cos,
                         const float *rope_sin, int heads, int kv_heads, int hd, int dim, int kvd,
                         float *kcache, float *vcache, int layer, int max_seq, cudaStream_t s);
/* Shapes attention_prefill takes: G = heads / kv_heads divides 64,
 * head_dim a multiple of 4 up to 128, ldq a multiple of 4. */
bool attention_prefill_supported(int heads, int kv_heads, int hd, int ldq);
/* Causal attention of nseq prompts of n tokens each at positions start ..
 * start + n - 1: row b = sq n + t of qkv [nseq n][ldq] (q of head h at
 * columns h hd) is token t of sequence seq0 + sq and attends to positions
 * 0 .. start + t of that sequence's cache, laid out
 * [layer][cache_seqs][kv_heads][max_seq][hd] (cache_seqs = 1: one
 * sequence).  ctx fp16 [nseq n][Kp], columns h hd + d; with zero_q the q
 * rows are zeroed once read. */
cudaError_t attention_prefill(float *qkv, int n, int nseq, int ldq, int seq0, int cache_seqs,
                              int start, const float *kcache, const float *vcache, int layer,
                              int heads, int kv_heads, int hd, int max_seq, int Kp,
                              uint16_t *ctx, bool zero_q, cudaStream_t s);
/* x[m][k] = 0 for dim <= k < Kp. */
cudaError_t zero_tail(uint16_t *x, int M, int dim, int Kp, cudaStream_t s);
/* act fp16 [M][Kp] = silu(gate) * up from gu [M][2 ffn] (groups of 8);
 * with clear_src the gate/up values are zeroed once read. */
cudaError_t swiglu_rows(const float *gu, int M, int ffn, int Kp, uint16_t *act, cudaStream_t s,
                        bool clear_src = false);

} // namespace nut
