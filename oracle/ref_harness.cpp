/* Test infrastructure only — never linked into the product.
 *
 * C entry points over the UNMODIFIED reference sources, compiled from where
 * they lie by oracle/Makefile into oracle/_ref/libnutref.so.  The tests use it
 * to pin the C restatement (nut_oracle.c) and to generate golden vectors; the
 * benchmark's reference arm times the reference's own CPU token loop through
 * it.  Nothing here re-implements reference arithmetic: every number comes
 * from the reference's own functions.
 *
 *   QuantizedMatrix::quantize            src/quant.cpp:154-197
 *   matvec_quantized_threaded            src/quant.cpp:262-321
 *   decode_quantized_token               src/quant_model.cpp:158-206
 *   prefill_quantized                    src/quant_model.cpp:208-220
 *   greedy loop of generate_tokens_cached src/generate.cpp:195-207 (driven
 *     directly, without the eos stop, as the parity harness must do)
 *   matvec_threaded / matmul_threaded    src/threading.cpp:163-198
 *   load_llama2c_quantized_model         src/llama2.cpp:339-412
 *   generate_tokens_cached (quantised)   src/generate.cpp:174-216
 *   Llama2Tokenizer::encode              src/llama2.cpp:455-514
 *
 * Reading the private byte and scale arrays needs access to QuantizedMatrix
 * internals, so this translation unit alone compiles quant.hpp with private
 * members made public (layout unchanged).
 */
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <map>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#define private public
#include "quant.hpp"
#undef private
#include "generate.hpp"
#include "kvcache.hpp"
#include "llama2.hpp"
#include "loader.hpp"
#include "tokenizer.hpp"
#include "matmul.hpp"
#include "ops.hpp"
#include "quant_model.hpp"

namespace {

thread_local std::string g_error;

template <typename F> int guarded(F &&body) {
    try {
        body();
        return 0;
    } catch (const std::invalid_argument &e) {
        g_error = e.what();
        return 1;
    } catch (const std::out_of_range &e) {
        g_error = e.what();
        return 2;
    } catch (const std::length_error &e) {
        g_error = e.what();
        return 3;
    } catch (const std::range_error &e) {
        g_error = e.what();
        return 5;
    } catch (const std::exception &e) {
        g_error = e.what();
        return 4;
    }
}

QuantType to_type(int t) {
    if (t == 0)
        return QuantType::int8;
    if (t == 1)
        return QuantType::int4;
    throw std::invalid_argument("ref harness: unknown quant type");
}

ModelConfig to_config(const int64_t *c) {
    ModelConfig config;
    config.layers = size_t(c[0]);
    config.heads = size_t(c[1]);
    config.dim = size_t(c[2]);
    config.head_dim = size_t(c[3]);
    config.ffn_dim = size_t(c[4]);
    config.vocab_size = size_t(c[5]);
    config.max_seq = size_t(c[6]);
    config.eos_token = size_t(c[7]);
    config.kv_heads = size_t(c[8]);
    return config;
}

QuantizedMatrix from_bytes(int type, size_t rows, size_t cols,
                           const uint8_t *data, const uint16_t *scales) {
    QuantizedMatrix m(rows, cols, 32, to_type(type));
    std::memcpy(m.data_.data(), data, m.data_.size());
    std::memcpy(m.scales_.data(), scales, m.scales_.size() * 2);
    return m;
}

struct RefModel {
    std::unique_ptr<QuantizedModelWeights> weights;
};

/* The greedy token loop of generate_tokens_cached (src/generate.cpp:184-207)
 * minus the eos stop: final rmsnorm -> fp32 lm_head (matvec_threaded) ->
 * first-index argmax (std::max_element) -> decode_quantized_token. */
void greedy(const QuantizedModelWeights &model, const std::vector<int> &prompt,
            size_t steps, size_t threads, int *ids, float *logits_out,
            float *prefill_hidden, double *prefill_s, double *decode_s) {
    KVCache cache(model.config);
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<float> last = prefill_quantized(model, prompt, cache, threads);
    const auto t1 = std::chrono::steady_clock::now();
    if (prefill_hidden)
        std::memcpy(prefill_hidden, last.data(), last.size() * 4);
    std::vector<float> normalized(model.config.dim);
    std::vector<float> logits(model.config.vocab_size);
    for (size_t step = 0; step < steps; step++) {
        rmsnorm(last.data(), model.final_norm.data(), normalized.data(),
                model.config.dim, 1e-5f);
        matvec_threaded(model.output_weights(), normalized.data(),
                        logits.data(), threads);
        const size_t token = size_t(
            std::max_element(logits.begin(), logits.end()) - logits.begin());
        if (logits_out)
            std::memcpy(logits_out + step * logits.size(), logits.data(),
                        logits.size() * 4);
        ids[step] = int(token);
        last = decode_quantized_token(model, int(token), cache, threads);
    }
    const auto t2 = std::chrono::steady_clock::now();
    if (prefill_s)
        *prefill_s = std::chrono::duration<double>(t1 - t0).count();
    if (decode_s)
        *decode_s = std::chrono::duration<double>(t2 - t1).count();
}

} // namespace

extern "C" {

const char *ref_last_error(void) { return g_error.c_str(); }

int ref_quantize(const float *src, size_t rows, size_t cols, int type,
                 uint8_t *data, size_t data_len, uint16_t *scales,
                 size_t scales_len) {
    return guarded([&] {
        QuantizedMatrix m =
            QuantizedMatrix::quantize(src, rows, cols, to_type(type));
        if (m.data_.size() != data_len || m.scales_.size() != scales_len)
            throw std::invalid_argument("ref harness: output size mismatch");
        std::memcpy(data, m.data_.data(), data_len);
        std::memcpy(scales, m.scales_.data(), scales_len * 2);
    });
}

int ref_qmatrix_info(const float *src, size_t rows, size_t cols, int type,
                     size_t *storage_bytes, float *values, float *bounds) {
    return guarded([&] {
        QuantizedMatrix m =
            QuantizedMatrix::quantize(src, rows, cols, to_type(type));
        *storage_bytes = m.storage_bytes();
        for (size_t r = 0; r < rows; r++)
            for (size_t c = 0; c < cols; c++) {
                if (values)
                    values[r * cols + c] = m.value(r, c);
                if (bounds)
                    bounds[r * cols + c] = m.error_bound(r, c);
            }
    });
}

int ref_qmatvec(int type, size_t rows, size_t cols, const uint8_t *data,
                const uint16_t *scales, const float *x, float *y,
                size_t threads) {
    return guarded([&] {
        QuantizedMatrix m = from_bytes(type, rows, cols, data, scales);
        matvec_quantized_threaded(m, x, y, threads);
    });
}

/* Times `reps` back-to-back quantised matvecs; returns seconds per call. */
int ref_qmatvec_time(int type, size_t rows, size_t cols, const uint8_t *data,
                     const uint16_t *scales, const float *x, float *y,
                     size_t threads, size_t reps, double *seconds) {
    return guarded([&] {
        QuantizedMatrix m = from_bytes(type, rows, cols, data, scales);
        matvec_quantized_threaded(m, x, y, threads);
        const auto t0 = std::chrono::steady_clock::now();
        for (size_t i = 0; i < reps; i++)
            matvec_quantized_threaded(m, x, y, threads);
        *seconds = std::chrono::duration<double>(
                       std::chrono::steady_clock::now() - t0)
                       .count() /
                   double(reps);
    });
}

int ref_rmsnorm(const float *x, const float *w, float *out, size_t n,
                float eps) {
    return guarded([&] { rmsnorm(x, w, out, n, eps); });
}

int ref_matvec_threaded(const float *w, size_t rows, size_t cols,
                        const float *x, float *y, size_t threads) {
    return guarded([&] {
        Matrix m(rows, cols);
        std::memcpy(m.data(), w, rows * cols * 4);
        matvec_threaded(m, x, y, threads);
    });
}

int ref_matmul_threaded(const float *a, const float *b, float *c, size_t m,
                        size_t k, size_t n, size_t threads, size_t reps,
                        double *seconds) {
    return guarded([&] {
        Matrix A(m, k), B(k, n), C(m, n);
        std::memcpy(A.data(), a, m * k * 4);
        std::memcpy(B.data(), b, k * n * 4);
        matmul_threaded(A, B, C, threads);
        const auto t0 = std::chrono::steady_clock::now();
        for (size_t i = 0; i < reps; i++)
            matmul_threaded(A, B, C, threads);
        if (seconds)
            *seconds = std::chrono::duration<double>(
                           std::chrono::steady_clock::now() - t0)
                           .count() /
                       double(reps ? reps : 1);
        std::memcpy(c, C.data(), m * n * 4);
    });
}

int ref_matvec_time(const float *w, size_t rows, size_t cols, const float *x,
                    float *y, size_t threads, size_t reps, double *seconds) {
    return guarded([&] {
        Matrix m(rows, cols);
        std::memcpy(m.data(), w, rows * cols * 4);
        matvec_threaded(m, x, y, threads);
        const auto t0 = std::chrono::steady_clock::now();
        for (size_t i = 0; i < reps; i++)
            matvec_threaded(m, x, y, threads);
        *seconds = std::chrono::duration<double>(
                       std::chrono::steady_clock::now() - t0)
                       .count() /
                   double(reps);
    });
}

int ref_model_new(const int64_t *config, int type, int tied, void **out) {
    return guarded([&] {
        auto model = std::make_unique<RefModel>();
        model->weights = std::make_unique<QuantizedModelWeights>(
            to_config(config), to_type(type), tied == 0);
        model->weights->tied_embeddings = tied != 0;
        *out = model.release();
    });
}

void ref_model_free(void *model) { delete static_cast<RefModel *>(model); }

int ref_model_set_embeddings(void *model, const float *embeddings) {
    return guarded([&] {
        auto &w = *static_cast<RefModel *>(model)->weights;
        std::memcpy(w.embeddings.data(), embeddings, w.embeddings.size() * 4);
    });
}

int ref_model_set_final(void *model, const float *final_norm,
                        const float *lm_head) {
    return guarded([&] {
        auto &w = *static_cast<RefModel *>(model)->weights;
        std::memcpy(w.final_norm.data(), final_norm, w.final_norm.size() * 4);
        if (!w.tied_embeddings)
            std::memcpy(w.lm_head.data(), lm_head, w.lm_head.size() * 4);
    });
}

/* Adds a layer from fp32 [out][in] projections, quantised by the reference's
 * own quantiser.  Order of `mats`: q, k, v, o, gate, up, down. */
int ref_model_add_layer(void *model, const float *const *mats,
                        const float *attention_norm, const float *ffn_norm) {
    return guarded([&] {
        auto &w = *static_cast<RefModel *>(model)->weights;
        const ModelConfig &c = w.config;
        const size_t shapes[7][2] = {
            {c.dim, c.dim},     {c.kv_dim(), c.dim}, {c.kv_dim(), c.dim},
            {c.dim, c.dim},     {c.ffn_dim, c.dim},  {c.ffn_dim, c.dim},
            {c.dim, c.ffn_dim}};
        std::vector<QuantizedMatrix> q;
        for (int i = 0; i < 7; i++)
            q.push_back(QuantizedMatrix::quantize(mats[i], shapes[i][0],
                                                  shapes[i][1], w.quant_type));
        w.layers.emplace_back(
            std::move(q[0]), std::move(q[1]), std::move(q[2]), std::move(q[3]),
            std::move(q[4]), std::move(q[5]), std::move(q[6]),
            std::vector<float>(attention_norm, attention_norm + c.dim),
            std::vector<float>(ffn_norm, ffn_norm + c.dim));
    });
}

int ref_model_storage_bytes(void *model, size_t *bytes) {
    return guarded([&] {
        *bytes = static_cast<RefModel *>(model)->weights->storage_bytes();
    });
}

/* Copies out the quantised bytes and fp16 scales of one projection
 * (which: 0..6 = q k v o gate up down). */
int ref_model_layer_bytes(void *model, size_t layer, int which, uint8_t *data,
                          size_t data_len, uint16_t *scales,
                          size_t scales_len) {
    return guarded([&] {
        auto &w = *static_cast<RefModel *>(model)->weights;
        const QuantizedLayerWeights &l = w.layers.at(layer);
        const QuantizedMatrix *mats[7] = {&l.query, &l.key,  &l.value,
                                          &l.output, &l.gate, &l.up,
                                          &l.down};
        if (which < 0 || which > 6)
            throw std::out_of_range("ref harness: projection index");
        const QuantizedMatrix &m = *mats[which];
        if (m.data_.size() != data_len || m.scales_.size() != scales_len)
            throw std::invalid_argument("ref harness: output size mismatch");
        std::memcpy(data, m.data_.data(), data_len);
        std::memcpy(scales, m.scales_.data(), scales_len * 2);
    });
}

int ref_generate(void *model, const int *prompt, size_t n, size_t steps,
                 size_t threads, int *ids, float *logits,
                 float *prefill_hidden, double *prefill_s, double *decode_s) {
    return guarded([&] {
        auto &w = *static_cast<RefModel *>(model)->weights;
        greedy(w, std::vector<int>(prompt, prompt + n), steps, threads, ids,
               logits, prefill_hidden, prefill_s, decode_s);
    });
}

/* Per-token hidden states (pre final norm) of prefill, then `steps` greedy
 * tokens: out_hidden holds (n + steps) rows of dim floats. */
int ref_trace(void *model, const int *prompt, size_t n, size_t steps,
              size_t threads, float *out_hidden) {
    return guarded([&] {
        auto &w = *static_cast<RefModel *>(model)->weights;
        const ModelConfig &c = w.config;
        KVCache cache(c);
        std::vector<float> h;
        for (size_t i = 0; i < n; i++) {
            h = decode_quantized_token(w, prompt[i], cache, threads);
            std::memcpy(out_hidden + i * c.dim, h.data(), c.dim * 4);
        }
        std::vector<float> normalized(c.dim), logits(c.vocab_size);
        for (size_t s = 0; s < steps; s++) {
            rmsnorm(h.data(), w.final_norm.data(), normalized.data(), c.dim,
                    1e-5f);
            matvec_threaded(w.output_weights(), normalized.data(),
                            logits.data(), threads);
            const int token = int(std::max_element(logits.begin(),
                                                   logits.end()) -
                                  logits.begin());
            h = decode_quantized_token(w, token, cache, threads);
            std::memcpy(out_hidden + (n + s) * c.dim, h.data(), c.dim * 4);
        }
    });
}

/* The reference's own end-to-end path on a llama2.c checkpoint:
 * load_llama2c_quantized_model + generate_tokens_cached (eos stop; greedy
 * for temperature <= 0, else its top-p sampler with std::mt19937(seed)). */
int ref_llama2c_generate(const char *path, int type, const int *prompt,
                         size_t n, size_t max_tokens, float temperature,
                         float top_p, unsigned seed, int *ids, size_t *n_out) {
    return guarded([&] {
        SamplingConfig sampling;
        sampling.max_tokens = max_tokens;
        sampling.temperature = temperature;
        sampling.top_p = top_p;
        sampling.seed = seed;
        const std::vector<int> tokens(prompt, prompt + n);
        /* type 2: the fp32 loader and the ModelWeights overload */
        const std::vector<int> out =
            type == 2 ? generate_tokens_cached(load_llama2c_model(path), tokens, sampling)
                      : generate_tokens_cached(
                            load_llama2c_quantized_model(path, to_type(type)), tokens,
                            sampling);
        std::copy(out.begin(), out.end(), ids);
        *n_out = out.size();
    });
}

/* The reference loader's result, described as nut_host_llama2c_inspect
 * describes the build's: config, tied flag, storage_bytes() and a 64-bit
 * FNV-1a digest of embeddings; per layer data+scales of q k v o gate up
 * down, attention norm, ffn norm; final norm; separate classifier. */
int ref_llama2c_inspect(const char *path, int type, int64_t *config,
                        int *tied, uint64_t *storage_bytes, uint64_t *digest) {
    return guarded([&] {
        uint64_t h = 0xcbf29ce484222325ull;
        auto add = [&h](const void *p, size_t bytes) {
            const unsigned char *b = static_cast<const unsigned char *>(p);
            for (size_t i = 0; i < bytes; i++) {
                h ^= b[i];
                h *= 0x100000001b3ull;
            }
        };
        auto describe = [&](const ModelConfig &c, bool is_tied, size_t bytes) {
            const size_t v[9] = {c.layers,     c.heads,   c.dim,
                                 c.head_dim,   c.ffn_dim, c.vocab_size,
                                 c.max_seq,    c.eos_token, c.kv_heads};
            for (int i = 0; i < 9; i++)
                config[i] = int64_t(v[i]);
            *tied = is_tied ? 1 : 0;
            *storage_bytes = bytes;
        };
        if (type == 2) {
            const ModelWeights m = load_llama2c_model(path);
            describe(m.config, m.tied_embeddings, m.storage_bytes());
            add(m.embeddings.data(), m.embeddings.size() * 4);
            for (const LayerWeights &l : m.layers) {
                for (const Matrix *q : {&l.query, &l.key, &l.value, &l.output,
                                        &l.gate, &l.up, &l.down})
                    add(q->data(), q->size() * 4);
                add(l.attention_norm.data(), l.attention_norm.size() * 4);
                add(l.ffn_norm.data(), l.ffn_norm.size() * 4);
            }
            add(m.final_norm.data(), m.final_norm.size() * 4);
            if (!m.tied_embeddings)
                add(m.lm_head.data(), m.lm_head.size() * 4);
            *digest = h;
            return;
        }
        const QuantizedModelWeights m =
            load_llama2c_quantized_model(path, to_type(type));
        describe(m.config, m.tied_embeddings, m.storage_bytes());
        add(m.embeddings.data(), m.embeddings.size() * 4);
        for (const QuantizedLayerWeights &l : m.layers) {
            for (const QuantizedMatrix *q : {&l.query, &l.key, &l.value,
                                             &l.output, &l.gate, &l.up,
                                             &l.down}) {
                add(q->data_.data(), q->data_.size());
                add(q->scales_.data(), q->scales_.size() * 2);
            }
            add(l.attention_norm.data(), l.attention_norm.size() * 4);
            add(l.ffn_norm.data(), l.ffn_norm.size() * 4);
        }
        add(m.final_norm.data(), m.final_norm.size() * 4);
        if (!m.tied_embeddings)
            add(m.lm_head.data(), m.lm_head.size() * 4);
        *digest = h;
    });
}

/* load_model(path) described like ref_llama2c_inspect (type 2 digest
 * order: embeddings, per layer the [in][out] q k v o gate up down and both
 * norms, final norm, lm_head). */
int ref_safetensors_inspect(const char *path, int64_t *config, uint64_t *storage_bytes,
                            uint64_t *digest) {
    return guarded([&] {
        const ModelWeights m = load_model(path);
        const ModelConfig &c = m.config;
        const size_t v[9] = {c.layers,     c.heads,   c.dim,       c.head_dim, c.ffn_dim,
                             c.vocab_size, c.max_seq, c.eos_token, c.kv_heads};
        for (int i = 0; i < 9; i++)
            config[i] = int64_t(v[i]);
        *storage_bytes = m.storage_bytes();
        uint64_t h = 0xcbf29ce484222325ull;
        auto add = [&h](const void *p, size_t bytes) {
            const unsigned char *b = static_cast<const unsigned char *>(p);
            for (size_t i = 0; i < bytes; i++) {
                h ^= b[i];
                h *= 0x100000001b3ull;
            }
        };
        add(m.embeddings.data(), m.embeddings.size() * 4);
        for (const LayerWeights &l : m.layers) {
            for (const Matrix *q : {&l.query, &l.key, &l.value, &l.output, &l.gate, &l.up,
                                    &l.down})
                add(q->data(), q->size() * 4);
            add(l.attention_norm.data(), l.attention_norm.size() * 4);
            add(l.ffn_norm.data(), l.ffn_norm.size() * 4);
        }
        add(m.final_norm.data(), m.final_norm.size() * 4);
        if (!m.tied_embeddings)
            add(m.lm_head.data(), m.lm_head.size() * 4);
        *digest = h;
    });
}

/* load_model + generate_tokens_cached (cached != 0) or generate_tokens. */
int ref_safetensors_generate(const char *path, const int *prompt, size_t n,
                             size_t max_tokens, float temperature, float top_p,
                             unsigned seed, int cached, int *ids, size_t *n_out) {
    return guarded([&] {
        const ModelWeights model = load_model(path);
        SamplingConfig sampling;
        sampling.max_tokens = max_tokens;
        sampling.temperature = temperature;
        sampling.top_p = top_p;
        sampling.seed = seed;
        const std::vector<int> tokens(prompt, prompt + n);
        const std::vector<int> out = cached ? generate_tokens_cached(model, tokens, sampling)
                                            : generate_tokens(model, tokens, sampling);
        std::copy(out.begin(), out.end(), ids);
        *n_out = out.size();
    });
}

/* Tokenizer::load(vocab, merges).encode(text) / .decode(ids). */
int ref_bpe_encode(const char *vocab_path, const char *merges_path, const char *text,
                   size_t text_len, int *ids, size_t capacity, size_t *n_out) {
    return guarded([&] {
        const Tokenizer t = Tokenizer::load(vocab_path, merges_path);
        const std::vector<int> out = t.encode(std::string(text, text_len));
        if (out.size() > capacity)
            throw std::length_error("harness: capacity");
        std::copy(out.begin(), out.end(), ids);
        *n_out = out.size();
    });
}

int ref_bpe_decode(const char *vocab_path, const char *merges_path, const int *ids, size_t n,
                   char *out, size_t capacity, size_t *len_out) {
    return guarded([&] {
        const Tokenizer t = Tokenizer::load(vocab_path, merges_path);
        const std::string text = t.decode(std::vector<int>(ids, ids + n));
        if (text.size() > capacity)
            throw std::length_error("harness: capacity");
        std::memcpy(out, text.data(), text.size());
        *len_out = text.size();
    });
}

/* Llama2Tokenizer::load(path, vocab).encode(text, bos, eos). */
int ref_llama2c_encode2(const char *tokenizer_path, size_t vocab, const char *text,
                        size_t text_len, int bos, int eos, int *ids, size_t capacity,
                        size_t *n_out) {
    return guarded([&] {
        const Llama2Tokenizer tok = Llama2Tokenizer::load(tokenizer_path, vocab);
        const std::vector<int> out =
            tok.encode(std::string(text, text_len), bos != 0, eos != 0);
        if (out.size() > capacity)
            throw std::length_error("ref harness: encode capacity");
        std::copy(out.begin(), out.end(), ids);
        *n_out = out.size();
    });
}

/* Llama2Tokenizer::load(path, vocab).decode(ids) into out (not terminated). */
int ref_llama2c_decode(const char *tokenizer_path, size_t vocab, const int *ids,
                       size_t n, char *out, size_t capacity, size_t *len_out) {
    return guarded([&] {
        const Llama2Tokenizer tok = Llama2Tokenizer::load(tokenizer_path, vocab);
        const std::string text = tok.decode(std::vector<int>(ids, ids + n));
        if (text.size() > capacity)
            throw std::length_error("ref harness: decode capacity");
        std::memcpy(out, text.data(), text.size());
        *len_out = text.size();
    });
}

/* Llama2Tokenizer::load(path, vocab).encode(text, bos, false). */
int ref_llama2c_encode(const char *tokenizer_path, size_t vocab,
                       const char *text, int bos, int *ids, size_t capacity,
                       size_t *n_out) {
    return guarded([&] {
        const Llama2Tokenizer tok = Llama2Tokenizer::load(tokenizer_path, vocab);
        const std::vector<int> out = tok.encode(text, bos != 0, false);
        if (out.size() > capacity)
            throw std::length_error("ref harness: encode capacity");
        std::copy(out.begin(), out.end(), ids);
        *n_out = out.size();
    });
}

} // extern "C"
