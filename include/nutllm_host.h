/* nutllm_host.h — C entry points of libnutllm.so, the C++17 host library
 * (load-time quantiser, llama2.c loader, generation and seeded synthetic
 * inputs; the C++ API itself is declared in nutllm_b200/host/, one header
 * per reference header).  Status codes are the
 * nut_status values of nutllm_cuda.h. */
#ifndef NUTLLM_HOST_H
#define NUTLLM_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Message of the calling thread's last host-library failure. */
const char *nut_host_last_error(void);

/* QuantizedMatrix::quantize (reference src/quant.cpp:154-197) into caller
 * buffers: data holds rows*cols (INT8) or (rows*cols+1)/2 (INT4) bytes,
 * scales (rows*cols+31)/32 fp16 bit patterns.  type: 0 INT8, 1 INT4. */
int nut_host_quantize(const float *source, int64_t rows, int64_t cols,
                      int32_t type, uint8_t *data, uint16_t *scales);

/* fp16 encoding of one positive scale as the quantiser rounds it. */
int nut_host_scale_to_half(float value, uint16_t *bits);

/* load_llama2c_quantized_model + generate_tokens_cached (reference
 * include/llama2.hpp:27-29, include/generate.hpp:29-36): loads a llama2.c
 * checkpoint, quantises it (type 0 INT8, 1 INT4; type 2 keeps fp32
 * weights: load_llama2c_model and the ModelWeights overload of
 * generate_tokens_cached, src/generate.cpp:128-172) and generates up to
 * max_tokens ids after the prompt on the current device, stopping at eos
 * (token 1) like the reference.  temperature <= 0 is greedy; otherwise
 * top-p sampling with std::mt19937(seed).  ids has room for max_tokens;
 * stats (may be NULL) receives GenerationStats. */
struct nut_generation_stats;
int nut_host_llama2c_generate(const char *path, int32_t type, const int32_t *prompt,
                              int64_t n, int64_t max_tokens, float temperature,
                              float top_p, uint32_t seed, int32_t *ids, int64_t *n_out,
                              struct nut_generation_stats *stats);

/* Loads a llama2.c checkpoint on the host only and describes it: config
 * (9 values in nut_config order: layers, heads, dim, head_dim, ffn_dim,
 * vocab_size, max_seq, eos_token, kv_heads), whether the classifier is the
 * embedding table, storage_bytes(), and a 64-bit FNV-1a digest of every
 * loaded byte in this order: embeddings; per layer the data then scales of
 * query, key, value, output, gate, up, down (type 2: the fp32 [in][out]
 * matrices), then the attention and ffn norms; the final norm; the
 * classifier when it is separate. */
int nut_host_llama2c_inspect(const char *path, int32_t type, int64_t *config,
                             int32_t *tied, uint64_t *storage_bytes, uint64_t *digest);

/* Llama2Tokenizer (reference include/llama2.hpp:11-25): loads `path` with
 * `vocab` entries and encodes text (bos / eos flags) into ids (room for
 * `cap`; *n_out = count), or decodes ids into text (room for `cap` bytes,
 * not NUL-terminated; *len_out = length). */
int nut_host_tokenizer_encode(const char *path, int64_t vocab, const char *text,
                              int64_t text_len, int32_t bos, int32_t eos, int32_t *ids,
                              int64_t cap, int64_t *n_out);
int nut_host_tokenizer_decode(const char *path, int64_t vocab, const int32_t *ids, int64_t n,
                              char *out, int64_t cap, int64_t *len_out);

/* Safetensors fp32 checkpoints (reference include/loader.hpp:11-62,
 * src/loader.cpp:286-498): load_model(path) described as
 * nut_host_llama2c_inspect describes a llama2.c file (config, storage_bytes,
 * FNV-1a digest of embeddings, per layer the [in][out] query, key, value,
 * output, gate, up, down then both norms, the final norm, lm_head), and
 * load_model + generation on the current device: cached != 0 calls
 * generate_tokens_cached (src/generate.cpp:128-172), cached == 0
 * generate_tokens (:101-126), each with its own checks and messages. */
int nut_host_safetensors_inspect(const char *path, int64_t *config, uint64_t *storage_bytes,
                                 uint64_t *digest);
int nut_host_safetensors_generate(const char *path, const int32_t *prompt, int64_t n,
                                  int64_t max_tokens, float temperature, float top_p,
                                  uint32_t seed, int32_t cached, int32_t *ids, int64_t *n_out);

/* Byte-level BPE Tokenizer (reference include/tokenizer.hpp:9-24):
 * Tokenizer::load(vocab_path, merges_path).encode(text) into ids (room for
 * `cap`; *n_out = count), or decode(ids) into out (room for `cap` bytes, not
 * NUL-terminated; *len_out = length). */
int nut_host_bpe_encode(const char *vocab_path, const char *merges_path, const char *text,
                        int64_t text_len, int32_t *ids, int64_t cap, int64_t *n_out);
int nut_host_bpe_decode(const char *vocab_path, const char *merges_path, const int32_t *ids,
                        int64_t n, char *out, int64_t cap, int64_t *len_out);

/* The generation token choice (choose_token, reference
 * src/generate.cpp:25-73) over `steps` rows of logits [steps][vocab] with
 * one std::mt19937(seed) shared by the steps, as one generation uses it. */
int nut_host_choose_tokens(const float *logits, int64_t steps, int64_t vocab,
                           float temperature, float top_p, uint32_t seed, int64_t *tokens);

/* Seeded synthetic inputs (documented in nutllm_b200/host/synth.cpp). */
void nut_synth_normal(uint64_t seed, uint64_t stream, float sigma, float *out,
                      size_t n);
void nut_synth_tokens(uint64_t seed, uint64_t stream, int lo, int hi, int *out,
                      size_t n);

#ifdef __cplusplus
}
#endif
#endif /* NUTLLM_HOST_H */
