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
size_t attention_rows_smem(int hd, int max_seq);
/* Causal attention of every (token, head) over the cache; ctx fp16 [M][Kp]. */
cudaError_t attention_rows(const float *qkv, int M, int ldq, int start, const float *kcache,
                           const float *vcache, int layer, int heads, int kv_heads, int hd,
                           int dim, int max_seq, int Kp, uint16_t *ctx, cudaStream_t s);
/* act fp16 [M][Kp] = silu(gate) * up from gu [M][2 ffn] (groups of 8);
 * with clear_src the gate/up values are zeroed once read. */
cudaError_t swiglu_rows(const float *gu, int M, int ffn, int Kp, uint16_t *act, cudaStream_t s,
                        bool clear_src = false);

} // namespace nut
