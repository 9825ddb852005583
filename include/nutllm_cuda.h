/* nutllm_cuda.h — C ABI of libnutcuda.so, the B200 (sm_100a) token loop.
 *
 * Plain pointers and sizes only.  Every entry point returns a nut_status;
 * nut_last_error() gives the calling thread's message for the last failure,
 * formatted "component: reason" like the reference's exceptions.  The status
 * codes map one-to-one onto the exception classes the reference throws for
 * the same conditions, so a C++ wrapper can re-throw the same type.
 *
 * Citations are to the reference project (MokiMeow/nutllm) interface each
 * entry point replaces.
 */
#ifndef NUTLLM_CUDA_H
#define NUTLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nut_status {
    NUT_OK = 0,
    NUT_INVALID_ARGUMENT = 1, /* std::invalid_argument */
    NUT_OUT_OF_RANGE = 2,     /* std::out_of_range */
    NUT_LENGTH_ERROR = 3,     /* std::length_error */
    NUT_RUNTIME_ERROR = 4,    /* std::runtime_error, CUDA failures included */
    NUT_RANGE_ERROR = 5,      /* std::range_error */
    NUT_DEVICE_TIMEOUT = 6    /* a bounded device-side wait gave up */
} nut_status;

/* QuantType (include/quant.hpp:9-12). */
enum { NUT_QUANT_INT8 = 0, NUT_QUANT_INT4 = 1 };

/* ModelConfig (include/model.hpp:8-24); kv_heads 0 means kv_heads = heads. */
typedef struct nut_config {
    int64_t layers, heads, dim, head_dim, ffn_dim, vocab_size, max_seq,
        eos_token, kv_heads;
} nut_config;

/* Host view of a QuantizedMatrix's storage (include/quant.hpp:14-50):
 * [rows][cols] row-major, flattened blocks of block_size (must be 32)
 * weights, INT8 one byte per weight or INT4 two's-complement nibbles with
 * the even flattened index in the low nibble, one fp16 scale (bits) per
 * block. */
typedef struct nut_qmatrix_view {
    const uint8_t *data;
    const uint16_t *scales;
    int64_t rows, cols, block_size;
    int32_t type;
} nut_qmatrix_view;

/* QuantizedLayerWeights (include/quant_model.hpp:9-29): projections are
 * [out][in]: query (dim x dim), key/value (kv_dim x dim), output
 * (dim x dim), gate/up (ffn x dim), down (dim x ffn). */
typedef struct nut_layer_view {
    nut_qmatrix_view query, key, value, output, gate, up, down;
    const float *attention_norm, *ffn_norm; /* [dim] each */
} nut_layer_view;

/* QuantizedModelWeights (include/quant_model.hpp:31-46).  lm_head is
 * ignored when tied_embeddings is set (output_weights() == embeddings). */
typedef struct nut_model_view {
    nut_config config;
    int32_t quant_type;
    int32_t tied_embeddings;
    const float *embeddings; /* [vocab][dim] */
    const float *final_norm; /* [dim] */
    const float *lm_head;    /* [vocab][dim] */
    const nut_layer_view *layers;
    int64_t n_layers;
} nut_model_view;

/* fp32 ModelWeights / LayerWeights (include/loader.hpp, include/model.hpp:
 * 26-38) for the `--quant fp32` path: every projection fp32 and [out][in]
 * (the llama2.c storage; the reference's own ModelWeights holds them
 * transposed, [in][out]). */
typedef struct nut_layer_f32_view {
    const float *query, *key, *value, *output, *gate, *up, *down;
    const float *attention_norm, *ffn_norm; /* [dim] each */
} nut_layer_f32_view;

typedef struct nut_model_f32_view {
    nut_config config;
    int32_t tied_embeddings;
    const float *embeddings; /* [vocab][dim] */
    const float *final_norm; /* [dim] */
    const float *lm_head;    /* [vocab][dim], ignored when tied */
    const nut_layer_f32_view *layers;
    int64_t n_layers;
} nut_model_f32_view;

/* GenerationStats (include/generate.hpp:19-24), device-event timed. */
typedef struct nut_generation_stats {
    int64_t prefill_tokens, generated_tokens;
    double prefill_seconds, decode_seconds;
} nut_generation_stats;

typedef struct nut_qmatrix nut_qmatrix;
typedef struct nut_model nut_model;
typedef struct nut_kv nut_kv;

/* Message of the calling thread's last failure ("" if none). */
const char *nut_last_error(void);

/* Number of visible CUDA devices. */
nut_status nut_device_count(int *count);

/* ---- QuantizedMatrix device mirror (src/quant.cpp:154-321) ---------- */

/* Uploads one quantised matrix to `device`. */
nut_status nut_qmatrix_create(const nut_qmatrix_view *view, int device,
                              nut_qmatrix **out);
nut_status nut_qmatrix_destroy(nut_qmatrix *matrix);
/* Reads the device copy back in the reference storage layout. */
nut_status nut_qmatrix_download(const nut_qmatrix *matrix, uint8_t *data,
                                uint16_t *scales);
/* matvec_quantized_threaded (src/quant.cpp:262-321) with HOST buffers:
 * y[rows] = Q x[cols].  Synchronous. */
nut_status nut_qmatvec(nut_qmatrix *matrix, const float *x, float *y);
/* The same product on DEVICE buffers, enqueued on `stream` (a
 * cudaStream_t, NULL = the legacy default stream). */
nut_status nut_qmatvec_async(nut_qmatrix *matrix, const float *x_device,
                             float *y_device, void *stream);

/* Prefill form of the quantised product on DEVICE buffers, enqueued on
 * `stream`: Y[tokens][rows] = X[tokens][cols] Q^T.  Runs on the 5th-gen
 * tensor cores with fp16 operands (Q dequantised once, q * scale rounded to
 * fp16, and cached with the matrix; X rounded to fp16 per call, saturating
 * at +-65504) and fp32 accumulation, so |Y - exact| <= 2^-10 sum_k
 * |x_k q_k s_k| per element (plus fp16's subnormal step below 2^-14).
 * The reference has no batched quantised product: prefill_quantized
 * (src/quant_model.cpp:208-220) runs matvec_quantized_threaded per token;
 * this entry point is that loop over a batch of tokens.  Device-side
 * timeouts are reported by the next nut_qmatrix_error call. */
nut_status nut_qmatrix_gemm(nut_qmatrix *matrix, const float *x_device, int64_t tokens,
                            float *y_device, void *stream);
/* Synchronises the matrix's work and reports a device-side timeout of an
 * earlier asynchronous call (NUT_DEVICE_TIMEOUT), clearing it. */
nut_status nut_qmatrix_error(nut_qmatrix *matrix);

/* ---- fp32 kernels of the reference's benches -------------------------- */

/* matmul_threaded (src/threading.cpp:163-181, include/matmul.hpp:32) on
 * DEVICE buffers: c[m][n] = a[m][k] b[k][n], row-major, every output the
 * k-sequential fused multiply-add chain of the reference build (results
 * are bit-identical).  Enqueued on `stream`. */
nut_status nut_matmul_f32(const float *a, const float *b, float *c, int64_t m, int64_t k,
                          int64_t n, void *stream);
/* matvec_threaded (src/threading.cpp:183-198, include/matmul.hpp:34) on
 * DEVICE buffers: output[r] = sum_c matrix[r][c] vector[c], each row a
 * sequential sum of rounded products (bit-identical to the reference). */
nut_status nut_matvec_f32(const float *matrix, const float *vector, float *output,
                          int64_t rows, int64_t cols, void *stream);

/* ---- Model weights (include/quant_model.hpp:31-46) ------------------- */

/* Copies a QuantizedModelWeights image to `device` (layout private to the
 * library).  Fails with NUT_INVALID_ARGUMENT for an invalid config or a
 * layer whose shape does not match it (src/quant_model.cpp:161-166). */
/* decode_token / prefill_tokens over fp32 weights (src/kvcache.cpp:237-284)
 * as a nut_model: the KV cache, decode, prefill, logits and greedy
 * generation calls below take it like a quantised model (one position per
 * pass; fp32 matvecs with the reference's matvec_threaded order; the fp32
 * reference projects with linear_threaded, so parity is by tolerance). */
nut_status nut_model_create_f32(const nut_model_f32_view *view, int device, nut_model **out);
nut_status nut_model_create(const nut_model_view *view, int device,
                            nut_model **out);
/* The same model built in steps, so a loader can overlap reading and
 * quantising layer l + 1 on the host with the upload of layer l:
 * nut_model_begin takes a view whose `layers` may be NULL (the fp32
 * tensors and the configuration are uploaded and checked), then
 * nut_model_add_layer appends layers 0, 1, ... in order (each packed into
 * tiles and copied to the device before it returns; the host buffers may be
 * reused afterwards), and nut_model_finish completes the model once
 * config.layers layers were added.  A model cannot back a KV cache before
 * it is finished; nut_model_destroy releases it at any step.  nut_model_add_layer
 * may be called from another host thread than nut_model_begin, one call at
 * a time.  Same checks, classes and messages as nut_model_create
 * (reference QuantizedModelWeights construction, include/quant_model.hpp:
 * 31-53, with src/quant_model.cpp:158-172's layer-count check). */
nut_status nut_model_begin(const nut_model_view *view, int device, nut_model **out);
nut_status nut_model_add_layer(nut_model *model, const nut_layer_view *layer);
nut_status nut_model_finish(nut_model *model);
nut_status nut_model_destroy(nut_model *model);
/* QuantizedModelWeights::storage_bytes (src/quant_model.cpp:140-156). */
nut_status nut_model_storage_bytes(const nut_model *model, uint64_t *bytes);

/* The CUDA stream (a cudaStream_t) on which every call with this model
 * enqueues its work, for callers that time or order that work with their
 * own CUDA events.  No counterpart in the reference (its loop is host
 * code). */
nut_status nut_model_stream(const nut_model *model, void **stream);

/* Prompts of at least min_tokens tokens (default 64; 0 = never) are
 * prefilled as one batch: every projection of every layer as one GEMM on
 * the tensor cores with fp16 operands (weights dequantised once, rounded to
 * fp16; fp32 accumulation), instead of the per-token loop of
 * prefill_quantized (src/quant_model.cpp:208-220).  Hidden states and the
 * KV cache then carry fp16 rounding (a looser bound than the per-token
 * path's parity); set 0 to keep every prompt on the per-token path.  The
 * batch's causal attention runs in tiles that share their keys and values;
 * shapes those tiles do not take (head_dim above 128 or not a multiple of
 * 4) keep the per-token path whatever the threshold.  Applies to
 * nut_prefill and nut_generate_greedy.  No counterpart in the reference. */
nut_status nut_model_set_prefill_threshold(nut_model *model, int64_t min_tokens);

/* Total kernels this library has launched in this process (all devices),
 * for callers that account for launches per step.  No counterpart in the
 * reference. */
nut_status nut_launch_count(uint64_t *count);

/* ---- KV cache and decode state (include/kvcache.hpp:8-31) ------------ */

/* KVCache(config) (src/kvcache.cpp:173-177): fp32 keys and values of
 * capacity config.max_seq, resident on the model's device, plus the
 * sequence's decode state (last hidden vector, logits). */
nut_status nut_kv_create(nut_model *model, nut_kv **out);
nut_status nut_kv_destroy(nut_kv *kv);
nut_status nut_kv_reset(nut_kv *kv);                   /* KVCache::reset */
nut_status nut_kv_length(const nut_kv *kv, int64_t *length);
nut_status nut_kv_set_length(nut_kv *kv, int64_t length); /* :231-235 */
nut_status nut_kv_memory_bytes(const nut_kv *kv, uint64_t *bytes);
/* KVCache::store (src/kvcache.cpp:216-229): writes the keys and values of
 * every kv head (kv_heads x head_dim floats each, host) at (layer,
 * position); the length is unchanged. */
nut_status nut_kv_write(nut_kv *kv, int64_t layer, int64_t position, const float *keys,
                        const float *values);
/* KVCache::key / KVCache::value (src/kvcache.cpp:207-214): copies one
 * head_dim vector of each to the host (either pointer may be NULL). */
nut_status nut_kv_read(const nut_kv *kv, int64_t layer, int64_t head,
                       int64_t position, float *key, float *value);

/* ---- Token loop -------------------------------------------------------- */

/* decode_quantized_token (src/quant_model.cpp:158-206): runs one token
 * through every layer at position kv length, appends its keys and values
 * and advances the length.  hidden (dim floats, host) may be NULL; the
 * pre-final-norm hidden vector stays on the device for nut_logits. */
nut_status nut_decode_token(nut_model *model, nut_kv *kv, int32_t token,
                            float *hidden);
/* prefill_quantized (src/quant_model.cpp:208-220): resets the cache and
 * feeds the prompt; hidden (dim floats, host) may be NULL. */
nut_status nut_prefill(nut_model *model, nut_kv *kv, const int32_t *tokens,
                       int64_t n, float *hidden);
/* Final rmsnorm + fp32 lm_head + first-index argmax over the last hidden
 * vector (src/generate.cpp:197-201).  Either output may be NULL. */
nut_status nut_logits(nut_model *model, nut_kv *kv, float *logits,
                      int32_t *argmax);
/* Greedy generate_tokens_cached (src/generate.cpp:174-216): prefill, then
 * up to max_tokens greedy steps, the whole loop on the device.  With
 * stop_at_eos set, a chosen eos_token ends the loop without being emitted
 * (the reference behaviour); with it clear, exactly max_tokens ids are
 * produced (the parity-harness form).  ids has room for max_tokens;
 * logits (max_tokens x vocab, host) and stats may be NULL. */
nut_status nut_generate_greedy(nut_model *model, nut_kv *kv,
                               const int32_t *prompt, int64_t n,
                               int64_t max_tokens, int32_t stop_at_eos,
                               int32_t *ids, int64_t *n_generated,
                               float *logits, nut_generation_stats *stats);

/* ---- Batched decode, tensor parallel ----------------------------------- */

/* B independent sequences generated in lockstep (BASELINE's 7B-shape
 * configuration: batch 64, equal prompt lengths), sharded over `world`
 * ranks, one process per GPU: rank r holds heads [r H/world, (r+1) H/world)
 * of Wq/Wk/Wv and the matching Wo columns, hidden units
 * [r F/world, (r+1) F/world) of Wgate/Wup and the matching Wdown columns,
 * and classifier rows [r V/world, (r+1) V/world); Wo and Wdown partial
 * outputs are summed with one NCCL all-reduce each per layer, the argmax
 * with a 64-bit max all-reduce (first-index tie rule of std::max_element).
 * Heads, kv heads and ffn / 32 must divide by world.  No reference
 * counterpart: the reference generates one sequence at a time on the CPU
 * (src/generate.cpp:174-216); this is that loop for a batch, with the
 * projections as fp16 tensor-core GEMMs (dequantised weights and fp16
 * activations, so logits follow the prefill GEMM's stated bound). */
typedef struct nut_batch nut_batch;

/* ncclGetUniqueId for rank 0 to share with the others (size >= 128). */
nut_status nut_tp_unique_id(uint8_t *id, int64_t size);
/* This rank's shard of a host model (every rank passes the whole view);
 * nccl_id may be NULL when world == 1. */
nut_status nut_batch_create(const nut_model_view *view, int device, int64_t batch, int rank,
                            int world, const uint8_t *nccl_id, nut_batch **out);
/* The same with seeded synthetic weights generated on the device (random
 * INT4 block-32 projections, N(0, 0.02) embeddings and classifier, unit norm
 * gains), for shapes too large to build on the host. */
nut_status nut_batch_create_synthetic(const nut_config *config, uint64_t seed, int device,
                                      int64_t batch, int rank, int world,
                                      const uint8_t *nccl_id, nut_batch **out);
void nut_batch_destroy(nut_batch *batch);
/* info[8] = {batch, heads, kv heads, ffn units, first vocabulary row, vocabulary
 * rows (all of this rank), weight bytes held, world}. */
nut_status nut_batch_info(const nut_batch *batch, int64_t *info);
nut_status nut_batch_stream(nut_batch *batch, void **stream);
/* Peer-memory all-reduce in place of NCCL for the Wo and Wdown sums: each
 * rank exports an IPC handle of its receive area (size >= 64 bytes per
 * handle), the ranks exchange them (e.g. an all-gather on the host), and
 * each opens everyone's handles [world][stride bytes].  Collective, world
 * <= 8, one process per GPU; the argmax still uses NCCL. */
nut_status nut_batch_ipc_handle(nut_batch *batch, uint8_t *handle, int64_t size);
nut_status nut_batch_open_peers(nut_batch *batch, const uint8_t *handles, int64_t stride);
/* Prompts of at least min_tokens tokens (default 16; 0 = never) are
 * prefilled as GEMMs over chunks of whole sequences (causal attention per
 * sequence, in tiles that share their keys and values) instead of one
 * position per pass; shapes the tiles do not take (per-rank head_dim above
 * 128 or not a multiple of 4) keep one position per pass. */
nut_status nut_batch_set_prefill_threshold(nut_batch *batch, int64_t min_tokens);
/* This rank's shard without creating anything (host only): shard[8] =
 * {first head, heads, first kv head, kv heads, first ffn unit, ffn units,
 * first vocabulary row, vocabulary rows}. */
nut_status nut_tp_shard(const nut_config *config, int rank, int world, int64_t *shard);
/* Prompts [batch][n] (host), then `steps` greedy tokens per sequence
 * without an eos stop: ids [batch][steps] (host).  logits [steps][batch]
 * [this rank's vocabulary rows] (host) may be NULL.  Collective: every rank
 * calls it with the same arguments. */
nut_status nut_batch_generate(nut_batch *batch, const int32_t *prompts, int64_t n,
                              int64_t steps, int32_t *ids, float *logits,
                              nut_generation_stats *stats);

/* One call of the peer-memory all-reduce (fp32 sum of n floats, n % 4 ==
 * 0) that the tensor-parallel decoder can use in place of NCCL, on
 * caller-owned buffers: recv[q] / flags[q] are rank q's receive area
 * ([2][world][n] floats) and flag words ([world][NUT_PEER_AR_CHUNKS]), as
 * this process addresses them (its own, or IPC mappings of the peers'),
 * zeroed before the first call; epochs [NUT_PEER_AR_CHUNKS] and error [1]
 * are this rank's, zeroed before the first call.  Every rank makes the same
 * sequence of calls with the same n.  Each wait for a peer's chunk gives up
 * after limit_ns nanoseconds: the call then returns NUT_DEVICE_TIMEOUT (the
 * kernel has ended; the device stays usable) and clears the error word.
 * Synchronises `stream` to read the error word.  The reference has no
 * multi-GPU path; like its RowExecutor, which hands a worker's failure back
 * to the caller (src/threading.cpp:58-74,91-99), a failed wait is reported
 * to the caller instead of hanging. */
#define NUT_PEER_AR_CHUNKS 128
nut_status nut_peer_all_reduce(const float *x, float *out, int64_t n, float *const *recv,
                               unsigned *const *flags, int rank, int world, unsigned *epochs,
                               int *error, int64_t limit_ns, void *stream);

/* ---- Greedy head without allocation ------------------------------------ */

/* Largest batch of nut_greedy_head_static. */
#define NUT_GREEDY_HEAD_MAX_BATCH 64

/* Final rmsnorm + fp32 classifier + first-index argmax of `batch` hidden
 * vectors, with every buffer in caller-provided DEVICE memory and no
 * allocation of any kind.  It is for callers that cannot call cudaMalloc
 * or cudaFree: code whose device memory is handed out by a host runtime's
 * own arena, or that issues GPU work where allocating is not allowed, and
 * which therefore cannot create the nut_model / nut_kv objects whose
 * buffers the rest of this ABI owns.  The kernels' only scratch, one
 * 64-bit argmax accumulator per batch row, is a fixed array of
 * NUT_GREEDY_HEAD_MAX_BATCH entries in this library's device memory, which
 * every GPU that loads the library keeps until the process exits; a larger
 * batch fails with NUT_LENGTH_ERROR.  The first call on a device resolves
 * the array's address (with that device current) and should come before
 * any stream capture.  Every call shares the array and clears the rows it
 * uses: calls whose work overlaps on the GPU race, so the caller must
 * serialise them.  A cudaDeviceReset() after the first call on a device is
 * not supported.
 *   hidden [batch][dim], final_norm [dim], weights [vocab][dim] (fp32),
 *   logits [batch][vocab] (may be NULL), argmax [batch] (int32);
 *   enqueued on `stream` (a cudaStream_t, NULL = legacy default stream).
 * Pointers need only their element's alignment (4 bytes; others fail with
 * NUT_INVALID_ARGUMENT); 16-byte-aligned weights with dim % 4 == 0 are read
 * as float4.  This entry point has no counterpart in the reference;
 * nut_logits is this library's model-handle form of the same head. */
nut_status nut_greedy_head_static(const float *hidden, const float *final_norm,
                                  const float *weights, int64_t batch, int64_t vocab,
                                  int64_t dim, float *logits, int32_t *argmax,
                                  void *stream);

#ifdef __cplusplus
}
#endif
#endif /* NUTLLM_CUDA_H */
