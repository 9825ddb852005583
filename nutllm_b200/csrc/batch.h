#pragma once
/* Row kernels of the batched (multi-sequence) decode step (batch.cu).  A
 * batch of B independent sequences advances one token per step, all at the
 * same position, which is read from device memory so that a captured step
 * can be replayed for every position.  The KV cache of a batch is fp32
 * [layer][sequence][kv_head][max_seq][head_dim]: the reference's per-model
 * layout (src/kvcache.cpp:196-205) repeated per sequence. */
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace nut {

/* h[b] += part[b] (when part is not null and add is set; part is then
 * zeroed for the next split-K GEMM that adds into it), then out[b][k] =
 * fp16(rmsnorm(h[b]) * w) for k < dim and 0 for dim <= k < Kp
 * (src/ops.cpp:111-134, eps 1e-5). */
cudaError_t add_rmsnorm_rows(float *h, float *part, bool add, const float *w, int B, int dim,
                             int Kp, uint16_t *out, cudaStream_t s);

/* RoPE (interleaved pairs, src/quant_model.cpp:26-37) of the q and k rows
 * of qkv [B][ldq] (q: heads * hd values, then k and v: kv_heads * hd each)
 * at position *pos, and the k and v rows appended to the batch cache (their
 * qkv entries are zeroed once cached, for the next split-K GEMM). */
cudaError_t rope_kv_batch(float *qkv, int B, int ldq, const int *pos, const float *rope_cos,
                          const float *rope_sin, int heads, int kv_heads, int hd,
                          float *kcache, float *vcache, int layer, int max_seq,
                          cudaStream_t s, int rows = 0, int pf_n = 0, int seq0 = 0);
/* Prefill form (rows > 0, pf_n > 0): qkv row m is position
 * m % pf_n of sequence seq0 + m / pf_n (B is still the batch the cache
 * holds).  The prefill's causal attention is attention_prefill (prefill.h). */

/* Attention of every (sequence, head) at position *pos over cached
 * positions 0 .. *pos (attention_step, src/quant_model.cpp:68-105: scores
 * q.k / sqrt(hd), softmax, weighted values; GQA head -> kv head by
 * head / (heads / kv_heads)); context fp16 [B][Kp], zero padded.  The q
 * entries of qkv are zeroed once read. */
cudaError_t attention_batch(const float *qkv, int B, int ldq, const int *pos,
                            const float *kcache, const float *vcache, int layer, int heads,
                            int kv_heads, int hd, int max_seq, int Kp, uint16_t *ctx,
                            cudaStream_t s);

/* Per row b: the first-index argmax of logits[b][0, V) as a 64-bit key
 * (order-preserving value bits << 32 | ~(v0 + index)), so that the maximum
 * key over any split of the vocabulary is the global first-index argmax
 * (std::max_element, src/generate.cpp:28-30).  Chunks of a row combine by
 * atomic max into keys[b], which must be zero on entry (keys_to_ids leaves
 * it zero).  With `clear` the logits are zeroed once read. */
cudaError_t argmax_keys(const float *logits, int B, int V, int v0, unsigned long long *keys,
                        bool clear, cudaStream_t s);
/* ids[b] = token of keys[b] (then keys[b] = 0); also appended to
 * out[b * ld + step] when out is not null. */
cudaError_t keys_to_ids(unsigned long long *keys, int B, int32_t *ids, int32_t *out,
                        int ld, const int *step, cudaStream_t s);
/* ids[b] = prompts[b * n + *step] (the next prompt column). */
cudaError_t prompt_column(const int32_t *prompts, int B, int n, const int *step, int32_t *ids,
                          cudaStream_t s);
/* *pos += 1 and *step += 1 (advances a captured step's position). */
cudaError_t advance(int *pos, int *step, cudaStream_t s);

/* Seeded synthetic weights generated on the device (benchmark shapes too
 * large to build on the host): normal(0, sigma) fp32 values, and fp16
 * values q * scale of random symmetric INT4 blocks (q uniform in [-7, 7],
 * one fp16 scale per 32 consecutive values of a row, near sigma * 2.5 / 7),
 * i.e. the dequantised form of a random INT4 block-32 matrix. */
cudaError_t synth_normal_dev(uint64_t seed, uint64_t stream, float sigma, float *out, size_t n,
                             cudaStream_t s);
cudaError_t synth_int4_f16_dev(uint64_t seed, uint64_t stream, float sigma, int rows, int cols,
                               int ld, uint16_t *out, cudaStream_t s);
/* The same random INT4 block-32 matrix [rows][cols] written directly in the
 * packed layout of gemm_q4 (K = cols rounded up to 64, zero past cols and
 * rows). */
cudaError_t synth_q4_packed_dev(uint64_t seed, uint64_t stream, float sigma, int rows,
                                int cols, int K, uint8_t *out, cudaStream_t s);

} // namespace nut

namespace nut {

/* One-shot all-reduce (sum, fp32) of n floats over `world` ranks through
 * peer memory (NVLink), one call per rank, every rank with the same n and
 * the same sequence of calls.  Rank r's receive area recv[r] is
 * [2][world][n] floats (double-buffered by call parity) and its flags
 * [world][chunks] words; recv and flags hold every rank's pointers (IPC
 * mappings of the peers', this rank's own).  CTA c pushes chunk c of x into
 * every rank's area with plain stores, fences at system scope, raises its
 * flag on every rank, waits (bounded by limit_ns; *error = 1 on timeout)
 * for chunk c of every rank and writes their sum, in rank order, to out.
 * epochs [chunks] counts this rank's calls per chunk. */
constexpr int kArChunks = 128;
cudaError_t peer_all_reduce(const float *x, float *out, int n, float *const *recv,
                            unsigned *const *flags, int rank, int world, unsigned *epochs,
                            int *error, uint64_t limit_ns, cudaStream_t s);

} // namespace nut
