/* Test infrastructure only: the CPU checker for the nutllm token loop.
 *
 * A plain-C restatement of the reference's INT8/INT4 block-32 quantised
 * decoder forward (MokiMeow/nutllm; every function cites the file:line it
 * follows).  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may load this library, and only to check or to time a CPU baseline.
 *
 * Floating-point order follows the reference's x86 build (g++ -O3 -mavx2
 * -mfma): the block dot products accumulate in eight fp32 lanes with fused
 * multiply-adds and a sequential lane sum, exactly as the AVX2 kernels do.
 * The file is compiled with -ffp-contract=off so that every fused
 * multiply-add here is an explicit fmaf/fma call.
 */
#include "nut_oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static _Thread_local char g_error[256];

/* Rows are split into contiguous ranges over host threads, as
 * run_threaded_rows does (src/threading.cpp:134-157); every row is computed
 * by one thread in a fixed order, so results do not depend on the count. */
typedef void (*row_fn)(void *ctx, int64_t begin, int64_t end);
typedef struct {
    row_fn fn;
    void *ctx;
    int64_t begin, end;
} row_task;

static int g_threads = 0;

void orc_set_threads(int threads) { g_threads = threads; }

static void *row_worker(void *arg) {
    row_task *t = arg;
    t->fn(t->ctx, t->begin, t->end);
    return NULL;
}

static void parallel_rows(int64_t rows, row_fn fn, void *ctx) {
    int threads = g_threads > 0 ? g_threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (threads > 64)
        threads = 64;
    if (rows < 64 || threads <= 1) {
        fn(ctx, 0, rows);
        return;
    }
    if (threads > rows)
        threads = (int)rows;
    pthread_t ids[64];
    row_task tasks[64];
    int started[64] = {0};
    for (int i = 1; i < threads; i++) {
        tasks[i] = (row_task){fn, ctx, rows * i / threads,
                              rows * (i + 1) / threads};
        started[i] =
            pthread_create(&ids[i], NULL, row_worker, &tasks[i]) == 0;
    }
    fn(ctx, 0, rows / threads);
    for (int i = 1; i < threads; i++) {
        if (started[i])
            pthread_join(ids[i], NULL);
        else /* no thread could be started: run the range here */
            fn(ctx, tasks[i].begin, tasks[i].end);
    }
}

static int fail(int status, const char *message) {
    snprintf(g_error, sizeof g_error, "%s", message);
    return status;
}

const char *orc_last_error(void) { return g_error; }

/* positive_float_to_half, src/quant.cpp:23-47.  Finite positive scale to
 * fp16 bits; the mantissa is rounded with lround (ties away from zero). */
uint16_t orc_half_from_float(float value, int *status) {
    *status = ORC_OK;
    if (!(value > 0.0f) || !isfinite(value)) {
        *status = fail(ORC_INVALID_ARGUMENT,
                       "quantize: scale must be finite positive");
        return 0;
    }
    if (value > 65504.0f) {
        *status = fail(ORC_RANGE, "quantize: scale exceeds fp16");
        return 0;
    }
    if (value < ldexpf(1.0f, -14)) {
        long mantissa = lround(ldexp((double)value, 24));
        if (mantissa < 1)
            mantissa = 1;
        if (mantissa > 1023)
            mantissa = 1023;
        return (uint16_t)mantissa;
    }
    int exponent = 0;
    const double fraction = frexp((double)value, &exponent);
    exponent--;
    long mantissa = lround((fraction * 2.0 - 1.0) * 1024.0);
    if (mantissa == 1024) {
        mantissa = 0;
        exponent++;
    }
    if (exponent > 15) {
        *status = fail(ORC_RANGE, "quantize: rounded scale exceeds fp16");
        return 0;
    }
    return (uint16_t)(((exponent + 15) << 10) | mantissa);
}

/* positive_half_to_float, src/quant.cpp:49-56. */
float orc_half_to_float(uint16_t value) {
    const unsigned exponent = (value >> 10) & 0x1f;
    const unsigned mantissa = value & 0x3ff;
    if (exponent == 0)
        return ldexpf((float)mantissa, -24);
    return ldexpf(1.0f + (float)mantissa / 1024.0f, (int)exponent - 15);
}

/* QuantizedMatrix::quantize, src/quant.cpp:154-197.  Blocks of 32 run over
 * the flattened row-major array (a block may span rows).  INT4 packs the
 * even flattened index in the low nibble (src/quant.cpp:1-5). */
int orc_quantize(const float *source, int64_t rows, int64_t cols, int type,
                 uint8_t *data, uint16_t *scales) {
    if (source == NULL)
        return fail(ORC_INVALID_ARGUMENT, "quantize: null source");
    if (rows <= 0 || cols <= 0)
        return fail(ORC_INVALID_ARGUMENT, "quantize: invalid dimensions");
    const int64_t n = rows * cols;
    const int64_t blocks = (n + 31) / 32;
    const int limit = type == ORC_INT8 ? 127 : 7;
    if (type == ORC_INT4)
        memset(data, 0, (size_t)((n + 1) / 2));
    for (int64_t b = 0; b < blocks; b++) {
        const int64_t begin = b * 32;
        const int64_t end = begin + 32 < n ? begin + 32 : n;
        float maximum = 0.0f;
        for (int64_t i = begin; i < end; i++) {
            if (!isfinite(source[i]))
                return fail(ORC_INVALID_ARGUMENT,
                            "quantize: non-finite source weight");
            const float a = fabsf(source[i]);
            if (a > maximum)
                maximum = a;
        }
        const float exact =
            maximum == 0.0f ? ldexpf(1.0f, -24) : maximum / (float)limit;
        int status = ORC_OK;
        scales[b] = orc_half_from_float(exact, &status);
        if (status != ORC_OK)
            return status;
        const float stored = orc_half_to_float(scales[b]);
        for (int64_t i = begin; i < end; i++) {
            long q = lroundf(source[i] / stored);
            if (q < -limit)
                q = -limit;
            if (q > limit)
                q = limit;
            if (type == ORC_INT8) {
                data[i] = (uint8_t)((unsigned)q & 0xffu);
            } else {
                const uint8_t nibble = (uint8_t)q & 0x0f;
                if (i % 2 == 0)
                    data[i / 2] = (uint8_t)((data[i / 2] & 0xf0) | nibble);
                else
                    data[i / 2] =
                        (uint8_t)((data[i / 2] & 0x0f) | (nibble << 4));
            }
        }
    }
    return ORC_OK;
}

/* quantized_value, src/quant.cpp:199-209. */
static int qvalue(int type, const uint8_t *data, int64_t index) {
    if (type == ORC_INT8)
        return data[index] >= 128 ? (int)data[index] - 256 : (int)data[index];
    const uint8_t packed = data[index / 2];
    const unsigned nibble = index % 2 == 0 ? packed & 0x0f : (packed >> 4);
    return nibble >= 8 ? (int)nibble - 16 : (int)nibble;
}

/* horizontal_sum, src/quant.cpp:66-73: lanes summed left to right. */
static float lane_sum(const float lanes[8]) {
    float total = 0.0f;
    for (int j = 0; j < 8; j++)
        total += lanes[j];
    return total;
}

/* One output row of matvec_quantized_threaded, src/quant.cpp:262-321.
 * Block-aligned rows take the AVX2 order of dot_int8_blocks /
 * dot_int4_blocks (src/quant.cpp:75-129): element (q * scale) rounded to
 * fp32, fused into lane (index mod 8).  Other shapes take the scalar double
 * path (src/quant.cpp:289-317). */
static float qdot_row(int type, int64_t row, int64_t cols, const uint8_t *data,
                      const uint16_t *scales, const float *x) {
    if (cols % 32 == 0) {
        float lanes[8] = {0};
        const int64_t base = row * cols;
        for (int64_t b = 0; b < cols / 32; b++) {
            const float scale = orc_half_to_float(scales[base / 32 + b]);
            for (int i = 0; i < 32; i++) {
                const int64_t col = b * 32 + i;
                const float value =
                    (float)qvalue(type, data, base + col) * scale;
                lanes[i % 8] = fmaf(value, x[col], lanes[i % 8]);
            }
        }
        return lane_sum(lanes);
    }
    double sum = 0.0;
    const int64_t begin = row * cols, end = begin + cols;
    for (int64_t index = begin; index < end; index++) {
        const float scale = orc_half_to_float(scales[index / 32]);
        sum += (double)((float)qvalue(type, data, index) * scale) *
               (double)x[index - begin];
    }
    return (float)sum;
}

typedef struct {
    int type;
    int64_t cols;
    const uint8_t *data;
    const uint16_t *scales;
    const float *x;
    float *y;
} qmv_ctx;

static void qmv_rows(void *arg, int64_t begin, int64_t end) {
    const qmv_ctx *c = arg;
    for (int64_t r = begin; r < end; r++)
        c->y[r] = qdot_row(c->type, r, c->cols, c->data, c->scales, c->x);
}

int orc_qmatvec(int type, int64_t rows, int64_t cols, const uint8_t *data,
                const uint16_t *scales, const float *x, float *y) {
    if (x == NULL || y == NULL)
        return fail(ORC_INVALID_ARGUMENT, "quantized matvec: null pointer");
    qmv_ctx ctx = {type, cols, data, scales, x, y};
    parallel_rows(rows, qmv_rows, &ctx);
    return ORC_OK;
}

/* rmsnorm, src/ops.cpp:111-134: squares in eight fp32 lanes (each square
 * rounded before it is added, as the AVX2 mul/add pair), a sequential lane
 * sum, a sequential tail, then x * scale * w with the scale in fp32. */
void orc_rmsnorm(const float *x, const float *w, float *out, int64_t n,
                 float eps) {
    float lanes[8] = {0};
    int64_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; j++)
            lanes[j] += x[i + j] * x[i + j];
    float squares = lane_sum(lanes);
    for (; i < n; i++)
        squares += x[i] * x[i];
    const float scale = 1.0f / sqrtf(squares / (float)n + eps);
    for (int64_t k = 0; k < n; k++)
        out[k] = x[k] * scale * w[k];
}

/* silu, src/ops.cpp:136-138. */
static float silu(float v) { return v / (1.0f + expf(-v)); }

/* rotate_vector, src/quant_model.cpp:26-37: interleaved pairs, angles in
 * double, cos/sin rounded to fp32, theta 10000.  Each product is rounded
 * before the add/subtract (the reference build pairs them unfused). */
void orc_rope(float *values, int64_t dims, int64_t position) {
    for (int64_t pair = 0; pair < dims; pair += 2) {
        const double frequency = pow(10000.0, -(double)pair / (double)dims);
        const float c = (float)cos((double)position * frequency);
        const float s = (float)sin((double)position * frequency);
        const float even = values[pair], odd = values[pair + 1];
        values[pair] = even * c - odd * s;
        values[pair + 1] = even * s + odd * c;
    }
}

/* matvec_threaded, src/threading.cpp:183-198: one sequential fp32 sum per
 * row.  The reference build vectorises the products 8 at a time (then 4 at
 * a time once, if 4 or more columns remain) and keeps the sum sequential
 * and unfused; the scalar loop over the last cols % 4 columns is contracted
 * into fused multiply-adds. */
typedef struct {
    const float *w, *x;
    int64_t cols;
    float *y;
} mv_ctx;

static void mv_rows(void *arg, int64_t begin, int64_t end) {
    const mv_ctx *c = arg;
    const int64_t rem = c->cols % 8;
    const int64_t unfused = c->cols - rem + (rem >= 4 ? 4 : 0);
    for (int64_t r = begin; r < end; r++) {
        const float *row = c->w + r * c->cols;
        float sum = 0.0f;
        int64_t k = 0;
        for (; k < unfused; k++)
            sum += row[k] * c->x[k];
        for (; k < c->cols; k++)
            sum = fmaf(row[k], c->x[k], sum);
        c->y[r] = sum;
    }
}

void orc_matvec_f32(const float *w, int64_t rows, int64_t cols,
                    const float *x, float *y) {
    mv_ctx ctx = {w, x, cols, y};
    parallel_rows(rows, mv_rows, &ctx);
}

/* matmul_threaded, src/threading.cpp:163-181: C = A B (row-major), C
 * zeroed, then for each row and each inner index k in order the row of B
 * scaled by a[row][k] is added into the output row.  The reference build
 * vectorises the column loop and contracts each update into one fused
 * multiply-add, so every output is a k-sequential chain of fmaf. */
typedef struct {
    const float *a, *b;
    int64_t k, n;
    float *c;
} mm_ctx;

static void mm_rows(void *arg, int64_t begin, int64_t end) {
    const mm_ctx *x = arg;
    for (int64_t r = begin; r < end; r++) {
        float *out = x->c + r * x->n;
        for (int64_t j = 0; j < x->n; j++)
            out[j] = 0.0f;
        for (int64_t k = 0; k < x->k; k++) {
            const float v = x->a[r * x->k + k];
            const float *w = x->b + k * x->n;
            for (int64_t j = 0; j < x->n; j++)
                out[j] = fmaf(v, w[j], out[j]);
        }
    }
}

void orc_matmul_f32(const float *a, const float *b, int64_t m, int64_t k, int64_t n,
                    float *c) {
    mm_ctx ctx = {a, b, k, n, c};
    parallel_rows(m, mm_rows, &ctx);
}

/* std::max_element as used by choose_token, src/generate.cpp:28-30: the
 * first index holding the largest value. */
int64_t orc_argmax(const float *values, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; i++)
        if (values[best] < values[i])
            best = i;
    return best;
}

static int64_t kv_offset(const orc_config *c, int64_t layer, int64_t head,
                         int64_t pos) {
    /* KVCache::offset, src/kvcache.cpp:196-205. */
    return ((layer * c->kv_heads + head) * c->max_seq + pos) * c->head_dim;
}

/* attention_step, src/quant_model.cpp:45-108. */
static int attention_step(const orc_model *m, const orc_layer *w,
                          int64_t layer, int64_t pos, const float *normalized,
                          orc_kv *kv, float *out) {
    const orc_config *c = &m->config;
    const int64_t d = c->head_dim, kvd = c->kv_heads * d;
    float *q = malloc(sizeof(float) * (size_t)c->dim);
    float *k = malloc(sizeof(float) * (size_t)kvd);
    float *v = malloc(sizeof(float) * (size_t)kvd);
    float *ctx = calloc((size_t)c->dim, sizeof(float));
    float *scores = malloc(sizeof(float) * (size_t)(pos + 1));
    if (!q || !k || !v || !ctx || !scores) {
        free(q), free(k), free(v), free(ctx), free(scores);
        return fail(ORC_RUNTIME, "oracle: out of memory");
    }
    orc_qmatvec(m->type, w->q.rows, w->q.cols, w->q.data, w->q.scales,
                normalized, q);
    orc_qmatvec(m->type, w->k.rows, w->k.cols, w->k.data, w->k.scales,
                normalized, k);
    orc_qmatvec(m->type, w->v.rows, w->v.cols, w->v.data, w->v.scales,
                normalized, v);
    for (int64_t h = 0; h < c->heads; h++)
        orc_rope(q + h * d, d, pos);
    for (int64_t h = 0; h < c->kv_heads; h++)
        orc_rope(k + h * d, d, pos);
    for (int64_t h = 0; h < c->kv_heads; h++) { /* KVCache::store */
        memcpy(kv->keys + kv_offset(c, layer, h, pos), k + h * d,
               sizeof(float) * (size_t)d);
        memcpy(kv->values + kv_offset(c, layer, h, pos), v + h * d,
               sizeof(float) * (size_t)d);
    }
    const float scale = 1.0f / sqrtf((float)d);
    const int64_t group = c->heads / c->kv_heads;
    for (int64_t h = 0; h < c->heads; h++) {
        const int64_t kvh = h / group;
        const float *qh = q + h * d;
        float maximum = -INFINITY;
        for (int64_t p = 0; p <= pos; p++) {
            const float *key = kv->keys + kv_offset(c, layer, kvh, p);
            double dot = 0.0;
            for (int64_t i = 0; i < d; i++)
                dot += (double)qh[i] * (double)key[i];
            scores[p] = (float)dot * scale;
            if (scores[p] > maximum)
                maximum = scores[p];
        }
        double total = 0.0;
        for (int64_t p = 0; p <= pos; p++) {
            scores[p] = expf(scores[p] - maximum);
            total += scores[p];
        }
        for (int64_t i = 0; i < d; i++) {
            double sum = 0.0;
            for (int64_t p = 0; p <= pos; p++) {
                const float *value = kv->values + kv_offset(c, layer, kvh, p);
                sum += (double)(scores[p] / (float)total) * (double)value[i];
            }
            ctx[h * d + i] = (float)sum;
        }
    }
    orc_qmatvec(m->type, w->o.rows, w->o.cols, w->o.data, w->o.scales, ctx,
                out);
    free(q), free(k), free(v), free(ctx), free(scores);
    return ORC_OK;
}

/* decode_quantized_token, src/quant_model.cpp:158-206.  Returns the hidden
 * state before the final norm. */
int orc_decode_token(const orc_model *m, orc_kv *kv, int token,
                     float *hidden) {
    const orc_config *c = &m->config;
    if (token < 0 || token >= c->vocab_size)
        return fail(ORC_OUT_OF_RANGE, "quantized decode: token out of range");
    if (kv->length >= c->max_seq)
        return fail(ORC_LENGTH, "quantized decode: context is full");
    const int64_t pos = kv->length, dim = c->dim, ffn = c->ffn_dim;
    memcpy(hidden, m->embeddings + (int64_t)token * dim,
           sizeof(float) * (size_t)dim);
    float *normalized = malloc(sizeof(float) * (size_t)dim);
    float *delta = malloc(sizeof(float) * (size_t)dim);
    float *gate = malloc(sizeof(float) * (size_t)ffn);
    float *up = malloc(sizeof(float) * (size_t)ffn);
    if (!normalized || !delta || !gate || !up) {
        free(normalized), free(delta), free(gate), free(up);
        return fail(ORC_RUNTIME, "oracle: out of memory");
    }
    int status = ORC_OK;
    for (int64_t l = 0; l < c->layers && status == ORC_OK; l++) {
        const orc_layer *w = &m->layers[l];
        orc_rmsnorm(hidden, w->attention_norm, normalized, dim, 1e-5f);
        status = attention_step(m, w, l, pos, normalized, kv, delta);
        for (int64_t i = 0; i < dim; i++)
            hidden[i] += delta[i];
        orc_rmsnorm(hidden, w->ffn_norm, normalized, dim, 1e-5f);
        orc_qmatvec(m->type, w->gate.rows, w->gate.cols, w->gate.data,
                    w->gate.scales, normalized, gate);
        orc_qmatvec(m->type, w->up.rows, w->up.cols, w->up.data,
                    w->up.scales, normalized, up);
        for (int64_t i = 0; i < ffn; i++)
            gate[i] = silu(gate[i]) * up[i];
        orc_qmatvec(m->type, w->down.rows, w->down.cols, w->down.data,
                    w->down.scales, gate, delta);
        for (int64_t i = 0; i < dim; i++)
            hidden[i] += delta[i];
    }
    free(normalized), free(delta), free(gate), free(up);
    if (status == ORC_OK)
        kv->length = pos + 1;
    return status;
}

/* Final rmsnorm + fp32 lm_head + first-index argmax, the head of the greedy
 * loop in generate_tokens_cached (src/generate.cpp:197-201). */
int orc_logits(const orc_model *m, const float *hidden, float *logits,
               int64_t *argmax) {
    const orc_config *c = &m->config;
    float *normalized = malloc(sizeof(float) * (size_t)c->dim);
    if (!normalized)
        return fail(ORC_RUNTIME, "oracle: out of memory");
    orc_rmsnorm(hidden, m->final_norm, normalized, c->dim, 1e-5f);
    orc_matvec_f32(m->lm_head, c->vocab_size, c->dim, normalized, logits);
    free(normalized);
    if (argmax)
        *argmax = orc_argmax(logits, c->vocab_size);
    return ORC_OK;
}

/* prefill_quantized (src/quant_model.cpp:208-220) followed by `steps` greedy
 * tokens of generate_tokens_cached (src/generate.cpp:195-207) without the
 * eos stop.  logits (steps x vocab) and prefill_hidden (dim) may be NULL. */
int orc_generate(const orc_model *m, orc_kv *kv, const int *prompt,
                 int64_t n, int64_t steps, int *ids, float *logits,
                 float *prefill_hidden) {
    const orc_config *c = &m->config;
    if (n <= 0 || n > c->max_seq)
        return fail(ORC_INVALID_ARGUMENT, "quantized prefill: invalid prompt");
    kv->length = 0;
    float *hidden = malloc(sizeof(float) * (size_t)c->dim);
    float *row = malloc(sizeof(float) * (size_t)c->vocab_size);
    if (!hidden || !row) {
        free(hidden), free(row);
        return fail(ORC_RUNTIME, "oracle: out of memory");
    }
    int status = ORC_OK;
    for (int64_t i = 0; i < n && status == ORC_OK; i++)
        status = orc_decode_token(m, kv, prompt[i], hidden);
    if (status == ORC_OK && prefill_hidden)
        memcpy(prefill_hidden, hidden, sizeof(float) * (size_t)c->dim);
    for (int64_t s = 0; s < steps && status == ORC_OK; s++) {
        int64_t best = 0;
        orc_logits(m, hidden, row, &best);
        if (logits)
            memcpy(logits + s * c->vocab_size, row,
                   sizeof(float) * (size_t)c->vocab_size);
        ids[s] = (int)best;
        status = orc_decode_token(m, kv, (int)best, hidden);
    }
    free(hidden), free(row);
    return status;
}

/* ---- Sampling ----------------------------------------------------------
 *
 * The reference draws with std::mt19937 and
 * std::uniform_real_distribution<double>, so the checker restates both:
 *   MT19937 — Matsumoto & Nishimura, "Mersenne Twister: a 623-dimensionally
 *   equidistributed uniform pseudo-random number generator", ACM TOMACS 8(1),
 *   1998 (the 32-bit generator with the 1812433253 seeding recurrence that
 *   C++11 [rand.eng.mers] specifies for mt19937);
 *   uniform_real_distribution<double>(a, b) in GNU libstdc++ (the library
 *   the reference is built against): generate_canonical<double, 53> takes
 *   two 32-bit draws g1, g2 and returns (g1 + g2 * 2^32) / 2^64, replaced by
 *   the largest double below 1 if it rounds up to 1; the draw is then
 *   canonical * (b - a) + a. */

typedef struct {
    uint32_t mt[624];
    int next;
} orc_mt19937;

static void mt_seed(orc_mt19937 *g, uint32_t seed) {
    g->mt[0] = seed;
    for (uint32_t i = 1; i < 624; i++)
        g->mt[i] = 1812433253u * (g->mt[i - 1] ^ (g->mt[i - 1] >> 30)) + i;
    g->next = 624;
}

static uint32_t mt_draw(orc_mt19937 *g) {
    if (g->next >= 624) {
        for (int i = 0; i < 624; i++) {
            const uint32_t y = (g->mt[i] & 0x80000000u) | (g->mt[(i + 1) % 624] & 0x7fffffffu);
            g->mt[i] = g->mt[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        g->next = 0;
    }
    uint32_t y = g->mt[g->next++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

static double uniform_double(orc_mt19937 *g, double lo, double hi) {
    double sum = (double)mt_draw(g);
    sum += (double)mt_draw(g) * 4294967296.0;
    double canonical = sum / 18446744073709551616.0;
    if (canonical >= 1.0)
        canonical = nextafter(1.0, 0.0);
    return canonical * (hi - lo) + lo;
}

/* std::uniform_real_distribution<float>(lo, hi) over std::mt19937(seed) as
 * libstdc++ computes it: generate_canonical<float, 24> takes one 32-bit
 * draw x, u = float(x) / 2^32 (u = 1 is replaced by the float below 1),
 * then u * (hi - lo) + lo in float.  The reference's self-tests fill their
 * matrices this way (src/quant_selftest.cpp:16-21). */
void orc_uniform_floats(uint32_t seed, float lo, float hi, int64_t n, float *out) {
    orc_mt19937 g;
    mt_seed(&g, seed);
    for (int64_t i = 0; i < n; i++) {
        float u = (float)mt_draw(&g) / 4294967296.0f;
        if (u >= 1.0f)
            u = nextafterf(1.0f, 0.0f);
        out[i] = u * (hi - lo) + lo;
    }
}

/* Probability order: larger weight first, lower token id on ties. */
static const float *g_sort_weights;
static int by_weight(const void *a, const void *b) {
    const int64_t i = *(const int64_t *)a, j = *(const int64_t *)b;
    const float wi = g_sort_weights[i], wj = g_sort_weights[j];
    if (wi != wj)
        return wi > wj ? -1 : 1;
    return i < j ? -1 : (i > j);
}

/* choose_token (src/generate.cpp:25-73). */
static int choose_one(const float *logits, int64_t vocab, float temperature, float top_p,
                      orc_mt19937 *g, float *weight, int64_t *order, int64_t *token) {
    if (vocab <= 0)
        return fail(ORC_INVALID_ARGUMENT, "sampling: empty logits");
    const int64_t best = orc_argmax(logits, vocab);
    if (temperature <= 0.0f) {
        *token = best;
        return ORC_OK;
    }
    if (!isfinite(temperature) || top_p <= 0.0f || top_p > 1.0f)
        return fail(ORC_INVALID_ARGUMENT, "sampling: invalid temperature or top-p");
    const float peak = logits[best];
    double total = 0.0;
    for (int64_t t = 0; t < vocab; t++) {
        const float p = expf((logits[t] - peak) / temperature);
        if (!isfinite(p))
            return fail(ORC_RUNTIME, "sampling: non-finite probability");
        weight[t] = p;
        order[t] = t;
        total += p;
    }
    if (!(total > 0.0))
        return fail(ORC_RUNTIME, "sampling: zero probability mass");
    g_sort_weights = weight;
    qsort(order, (size_t)vocab, sizeof(int64_t), by_weight);
    const double cutoff = (double)top_p * total;
    double nucleus = 0.0;
    int64_t count = 0;
    do {
        nucleus += weight[order[count]];
        count++;
    } while (count < vocab && nucleus < cutoff);
    const double target = uniform_double(g, 0.0, nucleus);
    double cumulative = 0.0;
    for (int64_t k = 0; k < count; k++) {
        cumulative += weight[order[k]];
        if (target <= cumulative) {
            *token = order[k];
            return ORC_OK;
        }
    }
    *token = order[count - 1];
    return ORC_OK;
}

int orc_choose_tokens(const float *logits, int64_t steps, int64_t vocab,
                      float temperature, float top_p, uint32_t seed,
                      int64_t *tokens) {
    orc_mt19937 g;
    mt_seed(&g, seed);
    float *weight = malloc(sizeof(float) * (size_t)(vocab > 0 ? vocab : 1));
    int64_t *order = malloc(sizeof(int64_t) * (size_t)(vocab > 0 ? vocab : 1));
    int status = (weight && order) ? ORC_OK : fail(ORC_RUNTIME, "oracle: out of memory");
    for (int64_t s = 0; s < steps && status == ORC_OK; s++)
        status = choose_one(logits + s * vocab, vocab, temperature, top_p, &g, weight, order,
                            &tokens[s]);
    free(weight), free(order);
    return status;
}

int orc_generate_sampled(const orc_model *m, orc_kv *kv, const int *prompt,
                         int64_t n, int64_t max_tokens, float temperature,
                         float top_p, uint32_t seed, int *ids, int64_t *n_out) {
    const orc_config *c = &m->config;
    if (n <= 0 || n > c->max_seq)
        return fail(ORC_INVALID_ARGUMENT, "generation: invalid prompt length");
    kv->length = 0;
    *n_out = 0;
    float *hidden = malloc(sizeof(float) * (size_t)c->dim);
    float *row = malloc(sizeof(float) * (size_t)c->vocab_size);
    float *weight = malloc(sizeof(float) * (size_t)c->vocab_size);
    int64_t *order = malloc(sizeof(int64_t) * (size_t)c->vocab_size);
    int status = (hidden && row && weight && order) ? ORC_OK
                                                    : fail(ORC_RUNTIME, "oracle: out of memory");
    for (int64_t i = 0; i < n && status == ORC_OK; i++)
        status = orc_decode_token(m, kv, prompt[i], hidden);
    orc_mt19937 g;
    mt_seed(&g, seed);
    while (status == ORC_OK && *n_out < max_tokens && kv->length < c->max_seq) {
        int64_t token = 0;
        orc_logits(m, hidden, row, NULL);
        status = choose_one(row, c->vocab_size, temperature, top_p, &g, weight, order, &token);
        if (status != ORC_OK || token == c->eos_token)
            break;
        ids[(*n_out)++] = (int)token;
        status = orc_decode_token(m, kv, (int)token, hidden);
    }
    free(hidden), free(row), free(weight), free(order);
    return status;
}

/* ---- seeded synthetic inputs ------------------------------------------
 *
 * The benchmark's documented counter-based generator (the reference has no
 * seeded N(0, sigma) initialiser), restated here so the reference's CPU
 * baseline can be fed the same bytes without loading this repository's own
 * libraries:
 *   key     = splitmix64(seed ^ splitmix64(stream))   (Steele, Lea, Flood 2014)
 *   u1, u2  = 53-bit uniforms in (0, 1] of splitmix64(key + 2j), (key + 2j + 1)
 *   z0, z1  = Box-Muller in double, out[2j] = float(sigma z0), out[2j+1] =
 *             float(sigma z1)
 * Token ids: lo + splitmix64(splitmix64(seed ^ splitmix64(stream ^
 * "token")) + i) mod (hi - lo + 1). */

static uint64_t orc_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static double orc_unit53(uint64_t bits) {
    return (double)((bits >> 11) + 1) * (1.0 / 9007199254740992.0);
}

typedef struct {
    uint64_t key;
    double sigma;
    float *out;
    int64_t n;
} synth_ctx;

static void synth_pairs(void *arg, int64_t begin, int64_t end) {
    const synth_ctx *s = arg;
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t pair = begin; pair < end; pair++) {
        const double u1 = orc_unit53(orc_splitmix64(s->key + 2 * (uint64_t)pair));
        const double u2 = orc_unit53(orc_splitmix64(s->key + 2 * (uint64_t)pair + 1));
        const double r = sqrt(-2.0 * log(u1));
        const double t = two_pi * u2;
        const int64_t i = 2 * pair;
        s->out[i] = (float)(s->sigma * (r * cos(t)));
        if (i + 1 < s->n)
            s->out[i + 1] = (float)(s->sigma * (r * sin(t)));
    }
}

void orc_synth_normal(uint64_t seed, uint64_t stream, float sigma, float *out, int64_t n) {
    synth_ctx s = {orc_splitmix64(seed ^ orc_splitmix64(stream)), (double)sigma, out, n};
    parallel_rows((n + 1) / 2, synth_pairs, &s);
}

void orc_synth_tokens(uint64_t seed, uint64_t stream, int lo, int hi, int *out, int64_t n) {
    const uint64_t key = orc_splitmix64(seed ^ orc_splitmix64(stream ^ 0x746f6b656eull));
    const uint64_t span = (uint64_t)((int64_t)hi - (int64_t)lo + 1);
    for (int64_t i = 0; i < n; i++)
        out[i] = (int)((int64_t)lo + (int64_t)(orc_splitmix64(key + (uint64_t)i) % span));
}
