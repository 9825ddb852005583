/* C entry points of the host library (include/nutllm_host.h). */
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/nutllm_cuda.h"
#include "../../include/nutllm_host.h"
#include "generate.hpp"
#include "llama2.hpp"
#include "quant.hpp"
#include "quant_model.hpp"
#include "tokenizer.hpp"

namespace {

thread_local std::string g_error;

template <typename F> int guarded(F &&body) {
    try {
        body();
        return NUT_OK;
    } catch (const std::invalid_argument &e) {
        g_error = e.what();
        return NUT_INVALID_ARGUMENT;
    } catch (const std::out_of_range &e) {
        g_error = e.what();
        return NUT_OUT_OF_RANGE;
    } catch (const std::length_error &e) {
        g_error = e.what();
        return NUT_LENGTH_ERROR;
    } catch (const std::range_error &e) {
        g_error = e.what();
        return NUT_RANGE_ERROR;
    } catch (const std::exception &e) {
        g_error = e.what();
        return NUT_RUNTIME_ERROR;
    }
}

QuantType quant_type(int32_t type) {
    if (type != 0 && type != 1)
        throw std::invalid_argument("quantize: unknown type");
    return type == 0 ? QuantType::int8 : QuantType::int4;
}

/* The loader type that selects load_llama2c_model (fp32 weights). */
constexpr int32_t kFp32 = 2;

void describe(const ModelConfig &c, bool is_tied, size_t bytes, int64_t *config, int32_t *tied,
              uint64_t *storage_bytes) {
    if (config != nullptr) {
        const size_t v[9] = {c.layers,     c.heads,   c.dim,       c.head_dim, c.ffn_dim,
                             c.vocab_size, c.max_seq, c.eos_token, c.kv_heads};
        for (int i = 0; i < 9; i++)
            config[i] = int64_t(v[i]);
    }
    if (tied != nullptr)
        *tied = is_tied ? 1 : 0;
    if (storage_bytes != nullptr)
        *storage_bytes = uint64_t(bytes);
}

/* 64-bit FNV-1a over a byte stream. */
struct Fnv1a {
    uint64_t h = 0xcbf29ce484222325ull;
    void add(const void *p, size_t n) {
        const unsigned char *b = static_cast<const unsigned char *>(p);
        for (size_t i = 0; i < n; i++) {
            h ^= b[i];
            h *= 0x100000001b3ull;
        }
    }
    template <typename T> void add(const std::vector<T> &v) { add(v.data(), v.size() * sizeof(T)); }
};

/* embeddings; per layer the seven [in][out] matrices then both norms; the
 * final norm; the classifier when it is separate */
uint64_t fp32_digest(const ModelWeights &m) {
    Fnv1a f;
    f.add(m.embeddings.data(), m.embeddings.size() * sizeof(float));
    for (const LayerWeights &l : m.layers) {
        for (const Matrix *q : {&l.query, &l.key, &l.value, &l.output, &l.gate, &l.up, &l.down})
            f.add(q->data(), q->size() * sizeof(float));
        f.add(l.attention_norm);
        f.add(l.ffn_norm);
    }
    f.add(m.final_norm);
    if (!m.tied_embeddings)
        f.add(m.lm_head.data(), m.lm_head.size() * sizeof(float));
    return f.h;
}

} // namespace

extern "C" {

const char *nut_host_last_error(void) { return g_error.c_str(); }

int nut_host_quantize(const float *source, int64_t rows, int64_t cols,
                      int32_t type, uint8_t *data, uint16_t *scales) {
    return guarded([&] {
        if (type != 0 && type != 1)
            throw std::invalid_argument("quantize: unknown type");
        if (rows <= 0 || cols <= 0)
            throw std::invalid_argument("quantize: invalid dimensions");
        if (data == nullptr || scales == nullptr)
            throw std::invalid_argument("quantize: null output");
        const QuantizedMatrix m = QuantizedMatrix::quantize(
            source, size_t(rows), size_t(cols),
            type == 0 ? QuantType::int8 : QuantType::int4);
        std::memcpy(data, m.data().data(), m.data().size());
        std::memcpy(scales, m.scales().data(), m.scales().size() * 2);
    });
}

int nut_host_scale_to_half(float value, uint16_t *bits) {
    return guarded([&] { *bits = quant_scale_to_half(value); });
}

int nut_host_llama2c_generate(const char *path, int32_t type, const int32_t *prompt,
                              int64_t n, int64_t max_tokens, float temperature,
                              float top_p, uint32_t seed, int32_t *ids, int64_t *n_out,
                              nut_generation_stats *stats) {
    return guarded([&] {
        if (path == nullptr || prompt == nullptr || n_out == nullptr || max_tokens < 0 ||
            (max_tokens > 0 && ids == nullptr) || n < 0)
            throw std::invalid_argument("generation: invalid argument");
        SamplingConfig sampling;
        sampling.max_tokens = size_t(max_tokens);
        sampling.temperature = temperature;
        sampling.top_p = top_p;
        sampling.seed = seed;
        GenerationStats st;
        const std::vector<int> tokens(prompt, prompt + n);
        const std::vector<int> out =
            type == kFp32 ? generate_tokens_cached(load_llama2c_model(path), tokens, sampling, &st)
                          : generate_tokens_cached(
                                load_llama2c_quantized_model(path, quant_type(type)), tokens,
                                sampling, &st);
        std::copy(out.begin(), out.end(), ids);
        *n_out = int64_t(out.size());
        if (stats != nullptr) {
            stats->prefill_tokens = int64_t(st.prefill_tokens);
            stats->generated_tokens = int64_t(st.generated_tokens);
            stats->prefill_seconds = st.prefill_seconds;
            stats->decode_seconds = st.decode_seconds;
        }
    });
}

int nut_host_llama2c_inspect(const char *path, int32_t type, int64_t *config,
                             int32_t *tied, uint64_t *storage_bytes, uint64_t *digest) {
    return guarded([&] {
        if (path == nullptr)
            throw std::invalid_argument("llama2 checkpoint: null path");
        if (type == kFp32) {
            const ModelWeights m = load_llama2c_model(path);
            describe(m.config, m.tied_embeddings, m.storage_bytes(), config, tied,
                     storage_bytes);
            if (digest != nullptr)
                *digest = fp32_digest(m);
            return;
        }
        const QuantizedModelWeights m = load_llama2c_quantized_model(path, quant_type(type));
        describe(m.config, m.tied_embeddings, m.storage_bytes(), config, tied, storage_bytes);
        if (digest != nullptr) {
            Fnv1a f;
            f.add(m.embeddings.data(), m.embeddings.size() * sizeof(float));
            for (const QuantizedLayerWeights &l : m.layers) {
                for (const QuantizedMatrix *q :
                     {&l.query, &l.key, &l.value, &l.output, &l.gate, &l.up, &l.down}) {
                    f.add(q->data());
                    f.add(q->scales());
                }
                f.add(l.attention_norm);
                f.add(l.ffn_norm);
            }
            f.add(m.final_norm);
            if (!m.tied_embeddings)
                f.add(m.lm_head.data(), m.lm_head.size() * sizeof(float));
            *digest = f.h;
        }
    });
}

int nut_host_choose_tokens(const float *logits, int64_t steps, int64_t vocab,
                           float temperature, float top_p, uint32_t seed, int64_t *tokens) {
    return guarded([&] {
        if (steps < 0 || vocab < 0 || (steps > 0 && (logits == nullptr || tokens == nullptr)))
            throw std::invalid_argument("sampling: invalid argument");
        SamplingConfig sampling;
        sampling.temperature = temperature;
        sampling.top_p = top_p;
        sampling.seed = seed;
        std::mt19937 rng(seed);
        std::vector<float> row(static_cast<size_t>(vocab));
        for (int64_t s = 0; s < steps; s++) {
            std::copy(logits + s * vocab, logits + (s + 1) * vocab, row.begin());
            tokens[s] = int64_t(choose_token(row, sampling, rng));
        }
    });
}

int nut_host_tokenizer_encode(const char *path, int64_t vocab, const char *text,
                              int64_t text_len, int32_t bos, int32_t eos, int32_t *ids,
                              int64_t cap, int64_t *n_out) {
    return guarded([&] {
        if (path == nullptr || (text == nullptr && text_len > 0) || n_out == nullptr ||
            vocab < 0 || text_len < 0)
            throw std::invalid_argument("llama2 tokenizer: invalid argument");
        const Llama2Tokenizer t = Llama2Tokenizer::load(path, size_t(vocab));
        const std::vector<int> out =
            t.encode(std::string(text, size_t(text_len)), bos != 0, eos != 0);
        if (int64_t(out.size()) > cap || (cap > 0 && ids == nullptr))
            throw std::length_error("llama2 tokenizer: output buffer too small");
        std::copy(out.begin(), out.end(), ids);
        *n_out = int64_t(out.size());
    });
}

int nut_host_tokenizer_decode(const char *path, int64_t vocab, const int32_t *ids, int64_t n,
                              char *out, int64_t cap, int64_t *len_out) {
    return guarded([&] {
        if (path == nullptr || (ids == nullptr && n > 0) || len_out == nullptr || vocab < 0 ||
            n < 0)
            throw std::invalid_argument("llama2 tokenizer: invalid argument");
        const Llama2Tokenizer t = Llama2Tokenizer::load(path, size_t(vocab));
        const std::string text = t.decode(std::vector<int>(ids, ids + n));
        if (int64_t(text.size()) > cap || (cap > 0 && out == nullptr))
            throw std::length_error("llama2 tokenizer: output buffer too small");
        std::memcpy(out, text.data(), text.size());
        *len_out = int64_t(text.size());
    });
}

int nut_host_safetensors_inspect(const char *path, int64_t *config, uint64_t *storage_bytes,
                                 uint64_t *digest) {
    return guarded([&] {
        if (path == nullptr)
            throw std::invalid_argument("safetensors: null path");
        const ModelWeights m = load_model(path);
        describe(m.config, false, m.storage_bytes(), config, nullptr, storage_bytes);
        if (digest != nullptr)
            *digest = fp32_digest(m);
    });
}

int nut_host_safetensors_generate(const char *path, const int32_t *prompt, int64_t n,
                                  int64_t max_tokens, float temperature, float top_p,
                                  uint32_t seed, int32_t cached, int32_t *ids, int64_t *n_out) {
    return guarded([&] {
        if (path == nullptr || (prompt == nullptr && n > 0) || n_out == nullptr ||
            max_tokens < 0 || (max_tokens > 0 && ids == nullptr) || n < 0)
            throw std::invalid_argument("generation: invalid argument");
        const ModelWeights model = load_model(path);
        SamplingConfig sampling;
        sampling.max_tokens = size_t(max_tokens);
        sampling.temperature = temperature;
        sampling.top_p = top_p;
        sampling.seed = seed;
        const std::vector<int> tokens(prompt, prompt + n);
        const std::vector<int> out = cached ? generate_tokens_cached(model, tokens, sampling)
                                            : generate_tokens(model, tokens, sampling);
        std::copy(out.begin(), out.end(), ids);
        *n_out = int64_t(out.size());
    });
}

int nut_host_bpe_encode(const char *vocab_path, const char *merges_path, const char *text,
                        int64_t text_len, int32_t *ids, int64_t cap, int64_t *n_out) {
    return guarded([&] {
        if (vocab_path == nullptr || merges_path == nullptr || n_out == nullptr ||
            (text == nullptr && text_len > 0) || text_len < 0)
            throw std::invalid_argument("tokenizer: invalid argument");
        const Tokenizer t = Tokenizer::load(vocab_path, merges_path);
        const std::vector<int> out = t.encode(std::string(text, size_t(text_len)));
        if (int64_t(out.size()) > cap || (cap > 0 && ids == nullptr))
            throw std::length_error("tokenizer: output buffer too small");
        std::copy(out.begin(), out.end(), ids);
        *n_out = int64_t(out.size());
    });
}

int nut_host_bpe_decode(const char *vocab_path, const char *merges_path, const int32_t *ids,
                        int64_t n, char *out, int64_t cap, int64_t *len_out) {
    return guarded([&] {
        if (vocab_path == nullptr || merges_path == nullptr || len_out == nullptr ||
            (ids == nullptr && n > 0) || n < 0)
            throw std::invalid_argument("tokenizer: invalid argument");
        const Tokenizer t = Tokenizer::load(vocab_path, merges_path);
        const std::string text = t.decode(std::vector<int>(ids, ids + n));
        if (int64_t(text.size()) > cap || (cap > 0 && out == nullptr))
            throw std::length_error("tokenizer: output buffer too small");
        std::memcpy(out, text.data(), text.size());
        *len_out = int64_t(text.size());
    });
}

} // extern "C"
