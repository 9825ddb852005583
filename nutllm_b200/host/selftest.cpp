/* Self-tests of the C++ host API against a llama2.c checkpoint, in the
 * style of the reference's own self-tests (src/kvcache_selftest.cpp,
 * src/loader_selftest.cpp): each check prints "ok" or "FAIL" and the
 * program exits 1 if any failed.
 *
 *   nutllm_selftest <checkpoint.bin> <int8|int4> <prompt ids...>
 *
 * It exercises the calls a reference caller makes — KVCache,
 * load_llama2c_quantized_model, prefill_quantized, decode_quantized_token,
 * generate_tokens_cached — and the exception classes of their failures. */
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "generate.hpp"
#include "kvcache.hpp"
#include "llama2.hpp"
#include "quant_model.hpp"

namespace {

int g_failed = 0;

void report(bool ok, const std::string &what) {
    std::printf("  %s %s\n", ok ? "ok" : "FAIL", what.c_str());
    if (!ok)
        g_failed++;
}

template <typename E> bool throws(const std::function<void()> &f, const char *message) {
    try {
        f();
    } catch (const E &e) {
        return message == nullptr || std::strstr(e.what(), message) != nullptr;
    } catch (...) {
        return false;
    }
    return false;
}

/* Final rmsnorm + fp32 classifier + first-index argmax on the host. */
int host_argmax(const QuantizedModelWeights &m, const std::vector<float> &hidden) {
    const size_t dim = m.config.dim;
    float ss = 0.0f;
    for (float v : hidden)
        ss += v * v;
    const float scale = 1.0f / std::sqrt(ss / float(dim) + 1e-5f);
    std::vector<float> x(dim);
    for (size_t i = 0; i < dim; i++)
        x[i] = hidden[i] * scale * m.final_norm[i];
    const Matrix &w = m.output_weights();
    int best = 0;
    float best_v = -INFINITY;
    for (size_t r = 0; r < m.config.vocab_size; r++) {
        float acc = 0.0f;
        for (size_t c = 0; c < dim; c++)
            acc += w.at(r, c) * x[c];
        if (acc > best_v) {
            best_v = acc;
            best = int(r);
        }
    }
    return best;
}

} // namespace

int main(int argc, char **argv) {
    if (argc < 4) {
        std::fprintf(stderr, "usage: %s <checkpoint.bin> <int8|int4> <prompt ids...>\n",
                     argv[0]);
        return 2;
    }
    const QuantType type = std::strcmp(argv[2], "int8") == 0 ? QuantType::int8 : QuantType::int4;
    std::vector<int> prompt;
    for (int i = 3; i < argc; i++)
        prompt.push_back(std::atoi(argv[i]));

    try {
        const QuantizedModelWeights model = load_llama2c_quantized_model(argv[1], type);
        const ModelConfig &c = model.config;
        report(model.layers.size() == c.layers && c.eos_token == 1 &&
                   model.storage_bytes() > 0 &&
                   (model.tied_embeddings ==
                    (model.output_weights().data() == model.embeddings.data())),
               "llama2.c loader: config, eos 1, classifier binding");

        /* prefill + decode through KVCache */
        KVCache cache(c);
        report(cache.length() == 0 && cache.capacity() == c.max_seq &&
                   cache.memory_bytes() ==
                       2 * c.layers * c.effective_kv_heads() * c.max_seq * c.head_dim * 4 &&
                   cache.compatible(c),
               "kv cache: empty, capacity, memory_bytes, compatible");
        std::vector<float> hidden = prefill_quantized(model, prompt, cache, 1);
        report(cache.length() == prompt.size() && hidden.size() == c.dim,
               "prefill_quantized: cache length and hidden size");

        /* the greedy loop written against the API, as a caller would */
        std::vector<int> manual;
        const size_t steps = std::min<size_t>(6, c.max_seq - prompt.size());
        for (size_t s = 0; s < steps; s++) {
            const int token = host_argmax(model, hidden);
            if (size_t(token) == c.eos_token)
                break;
            manual.push_back(token);
            hidden = decode_quantized_token(model, token, cache, 1);
        }
        SamplingConfig greedy;
        greedy.max_tokens = steps;
        GenerationStats stats;
        const std::vector<int> generated = generate_tokens_cached(model, prompt, greedy, &stats);
        report(generated == manual && stats.prefill_tokens == prompt.size() &&
                   stats.generated_tokens == generated.size() && stats.decode_seconds >= 0.0,
               "generate_tokens_cached: same ids as prefill + decode_quantized_token");

        /* the same prompt again from a reset cache gives the same state, up
         * to the order of the split-K float reductions (device atomics) */
        KVCache again(c);
        const std::vector<float> h1 = prefill_quantized(model, prompt, again, 1);
        const std::vector<float> h2 = prefill_quantized(model, prompt, again, 1);
        bool close = h1.size() == h2.size();
        float worst = 0.0f;
        for (size_t i = 0; close && i < h1.size(); i++) {
            worst = std::max(worst, std::fabs(h1[i] - h2[i]));
            close = std::fabs(h1[i] - h2[i]) <= 1e-4f + 1e-4f * std::fabs(h1[i]);
        }
        report(close && again.length() == prompt.size(),
               "prefill_quantized: resets the cache and repeats (max |diff| " +
                   std::to_string(worst) + ")");

        /* key / value / store / set_length */
        const size_t kvh = c.effective_kv_heads(), hd = c.head_dim;
        std::vector<float> k(kvh * hd), v(kvh * hd);
        for (size_t i = 0; i < k.size(); i++) {
            k[i] = float(i) * 0.25f - 3.0f;
            v[i] = 7.0f - float(i) * 0.5f;
        }
        again.store(c.layers - 1, prompt.size(), k.data(), v.data());
        bool round_trip = true;
        for (size_t h = 0; h < kvh; h++) {
            const float *kk = again.key(c.layers - 1, h, prompt.size());
            round_trip = round_trip && std::memcmp(kk, k.data() + h * hd, hd * 4) == 0;
            const float *vv = again.value(c.layers - 1, h, prompt.size());
            round_trip = round_trip && std::memcmp(vv, v.data() + h * hd, hd * 4) == 0;
        }
        report(round_trip && again.length() == prompt.size(),
               "kv cache: store then key/value round trip, length unchanged");
        report(throws<std::out_of_range>([&] { again.key(c.layers, 0, 0); },
                                         "kv cache: index out of range") &&
                   throws<std::out_of_range>([&] { again.value(0, kvh, 0); },
                                             "kv cache: index out of range") &&
                   throws<std::invalid_argument>(
                       [&] { again.store(0, 0, nullptr, v.data()); }, "kv cache: null source") &&
                   throws<std::length_error>([&] { again.set_length(c.max_seq + 1); },
                                             "kv cache: context exceeds capacity"),
               "kv cache: out_of_range / invalid_argument / length_error");

        /* decode errors, with the reference's classes */
        report(throws<std::invalid_argument>(
                   [&] { decode_quantized_token(model, 2, again, 0); },
                   "quantized decode: zero threads") &&
                   throws<std::out_of_range>(
                       [&] { decode_quantized_token(model, int(c.vocab_size), again, 1); },
                       "quantized decode: token out of range") &&
                   throws<std::out_of_range>([&] { decode_quantized_token(model, -1, again, 1); },
                                             "quantized decode: token out of range") &&
                   throws<std::invalid_argument>(
                       [&] { prefill_quantized(model, {}, again, 1); },
                       "quantized prefill: invalid prompt"),
               "decode/prefill: zero threads, token range, empty prompt");
        again.set_length(c.max_seq);
        report(throws<std::length_error>([&] { decode_quantized_token(model, 2, again, 1); },
                                         "quantized decode: context is full"),
               "decode: full context is a length_error");
        ModelConfig other = c;
        other.max_seq = c.max_seq + 1;
        KVCache mismatched(other);
        report(!mismatched.compatible(c) &&
                   throws<std::invalid_argument>(
                       [&] { decode_quantized_token(model, 2, mismatched, 1); },
                       "quantized decode: cache configuration mismatch"),
               "decode: incompatible cache is rejected");

        /* sampling: the same seed repeats, generation errors */
        SamplingConfig sampled;
        sampled.max_tokens = steps;
        sampled.temperature = 0.9f;
        sampled.top_p = 0.8f;
        sampled.seed = 42;
        report(generate_tokens_cached(model, prompt, sampled) ==
                   generate_tokens_cached(model, prompt, sampled),
               "generate_tokens_cached: seeded sampling repeats");
        SamplingConfig no_threads;
        no_threads.threads = 0;
        report(throws<std::invalid_argument>(
                   [&] { generate_tokens_cached(model, prompt, no_threads); },
                   "generation: zero threads") &&
                   throws<std::invalid_argument>(
                       [&] { generate_tokens_cached(model, {}, greedy); },
                       "generation: invalid prompt length"),
               "generate_tokens_cached: zero threads, empty prompt");
    } catch (const std::exception &e) {
        std::printf("  FAIL unexpected exception: %s\n", e.what());
        g_failed++;
    }
    std::printf("%s\n", g_failed == 0 ? "all host API checks passed" : "host API checks FAILED");
    return g_failed == 0 ? 0 : 1;
}
