/* Test infrastructure only: the CPU checker for the nutllm token loop.
 *
 * A plain-C restatement of the reference's quantised decoder forward
 * (MokiMeow/nutllm, paths relative to that project).  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it, and
 * only as the thing results are checked against — never as a product path.
 */
#ifndef NUT_ORACLE_H
#define NUT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_INT8 = 0, ORC_INT4 = 1 };

/* Status codes mirror the reference's exception classes. */
enum {
    ORC_OK = 0,
    ORC_INVALID_ARGUMENT = 1, /* std::invalid_argument */
    ORC_OUT_OF_RANGE = 2,     /* std::out_of_range */
    ORC_LENGTH = 3,           /* std::length_error */
    ORC_RUNTIME = 4,          /* std::runtime_error */
    ORC_RANGE = 5             /* std::range_error */
};

typedef struct {
    int64_t layers, heads, dim, head_dim, ffn_dim, vocab_size, max_seq,
        eos_token, kv_heads;
} orc_config;

typedef struct {
    const uint8_t *data;
    const uint16_t *scales;
    int64_t rows, cols;
} orc_qmatrix;

typedef struct {
    orc_qmatrix q, k, v, o, gate, up, down; /* [out][in], block 32 */
    const float *attention_norm, *ffn_norm;
} orc_layer;

typedef struct {
    orc_config config;
    int type;
    const float *embeddings; /* [vocab][dim] */
    const float *final_norm; /* [dim] */
    const float *lm_head;    /* [vocab][dim]; == embeddings when tied */
    const orc_layer *layers;
} orc_model;

typedef struct {
    float *keys, *values; /* [layers][kv_heads][max_seq][head_dim] each */
    int64_t length;
} orc_kv;

const char *orc_last_error(void);

uint16_t orc_half_from_float(float value, int *status);
float orc_half_to_float(uint16_t value);
int orc_quantize(const float *source, int64_t rows, int64_t cols, int type,
                 uint8_t *data, uint16_t *scales);
int orc_qmatvec(int type, int64_t rows, int64_t cols, const uint8_t *data,
                const uint16_t *scales, const float *x, float *y);
void orc_set_threads(int threads);
void orc_rmsnorm(const float *x, const float *w, float *out, int64_t n,
                 float eps);
void orc_rope(float *values, int64_t dims, int64_t position);
void orc_matvec_f32(const float *w, int64_t rows, int64_t cols,
                    const float *x, float *y);
/* matmul_threaded (src/threading.cpp:163-181): c[m][n] = a[m][k] b[k][n]. */
void orc_matmul_f32(const float *a, const float *b, int64_t m, int64_t k, int64_t n,
                    float *c);
int64_t orc_argmax(const float *values, int64_t n);
int orc_decode_token(const orc_model *model, orc_kv *kv, int token,
                     float *hidden);
int orc_logits(const orc_model *model, const float *hidden, float *logits,
               int64_t *argmax);
int orc_generate(const orc_model *model, orc_kv *kv, const int *prompt,
                 int64_t n, int64_t steps, int *ids, float *logits,
                 float *prefill_hidden);

/* Token sampling of generate_tokens_cached (src/generate.cpp:25-73) with the
 * random source the reference uses: std::mt19937 seeded with `seed`, drawn
 * through std::uniform_real_distribution<double>.  orc_choose_tokens runs
 * `steps` choices over rows of logits [steps][vocab] with one generator.
 * orc_generate_sampled is the reference's quantised generate_tokens_cached
 * loop (src/generate.cpp:174-216): prefill, then while fewer than
 * max_tokens ids and the cache is not full: logits, choose, stop at eos,
 * decode.  Greedy when temperature <= 0. */
/* n values of std::uniform_real_distribution<float>(lo, hi) drawn from
 * std::mt19937(seed) (libstdc++'s generate_canonical). */
void orc_uniform_floats(uint32_t seed, float lo, float hi, int64_t n, float *out);

int orc_choose_tokens(const float *logits, int64_t steps, int64_t vocab,
                      float temperature, float top_p, uint32_t seed,
                      int64_t *tokens);
int orc_generate_sampled(const orc_model *model, orc_kv *kv, const int *prompt,
                         int64_t n, int64_t max_tokens, float temperature,
                         float top_p, uint32_t seed, int *ids, int64_t *n_out);

/* The benchmark's seeded synthetic inputs (the same documented generator
 * as the product's host library): n N(0, sigma^2) floats of `stream`, and n
 * token ids uniform in [lo, hi]. */
void orc_synth_normal(uint64_t seed, uint64_t stream, float sigma, float *out, int64_t n);
void orc_synth_tokens(uint64_t seed, uint64_t stream, int lo, int hi, int *out, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
