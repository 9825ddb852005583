/* generate_tokens_cached for quantised and fp32 models over the C ABI, and the
 * host token sampler.  The sampler keeps the reference's arithmetic
 * (src/generate.cpp:25-73) step for step, because a seeded draw only picks
 * the same token when every intermediate value is the same:
 *   w_i   = float exp(float(logit_i - max) / temperature)    (float)
 *   mass  = sum of w_i in token order                          (double)
 *   order = tokens by w descending, ties by lower id
 *   keep the shortest prefix of `order` (at least one token) whose running
 *   double sum reaches top_p * mass; draw u ~ U[0, kept) from
 *   std::uniform_real_distribution<double> over std::mt19937(seed), and
 *   return the first kept token whose running sum is >= u. */
#include "generate.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <numeric>
#include <stdexcept>

#include "device.hpp"
#include "kvcache.hpp"
#include "loader.hpp"
#include "quant_model.hpp"

size_t choose_token(const std::vector<float> &logits, const SamplingConfig &sampling,
                    std::mt19937 &rng) {
    const size_t n = logits.size();
    if (n == 0)
        throw std::invalid_argument("sampling: empty logits");
    const size_t best = size_t(std::max_element(logits.begin(), logits.end()) - logits.begin());
    if (sampling.temperature <= 0.0f)
        return best;
    if (!std::isfinite(sampling.temperature) || !(sampling.top_p > 0.0f) ||
        sampling.top_p > 1.0f)
        throw std::invalid_argument("sampling: invalid temperature or top-p");

    const float peak = logits[best];
    std::vector<float> weight(n);
    double mass = 0.0;
    for (size_t i = 0; i < n; i++) {
        const float w = std::exp((logits[i] - peak) / sampling.temperature);
        if (!std::isfinite(w))
            throw std::runtime_error("sampling: non-finite probability");
        weight[i] = w;
        mass += w;
    }
    if (!(mass > 0.0))
        throw std::runtime_error("sampling: zero probability mass");

    std::vector<uint32_t> order(n);
    std::iota(order.begin(), order.end(), 0u);
    std::sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        return weight[a] != weight[b] ? weight[a] > weight[b] : a < b;
    });

    const double cutoff = double(sampling.top_p) * mass;
    double kept = 0.0;
    size_t keep = 0;
    do
        kept += weight[order[keep++]];
    while (keep < n && kept < cutoff);

    const double target = std::uniform_real_distribution<double>(0.0, kept)(rng);
    double running = 0.0;
    for (size_t i = 0; i < keep; i++) {
        running += weight[order[i]];
        if (target <= running)
            return order[i];
    }
    return order[keep - 1];
}

namespace {

double seconds_since(std::chrono::steady_clock::time_point start) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
}

/* Both model kinds run the loop through one nut_model. */
std::vector<int> generate_greedy(nut_model *m, const std::vector<int> &prompt,
                                 const SamplingConfig &sampling, KVCache &cache,
                                 GenerationStats *stats) {
    nut_kv *kv = cache.device(m);
    const std::vector<int32_t> ids32(prompt.begin(), prompt.end());
    std::vector<int32_t> out(std::max<size_t>(sampling.max_tokens, 1));
    int64_t produced = 0;
    nut_generation_stats st{};
    nutdev::check(nut_generate_greedy(m, kv, ids32.data(), int64_t(ids32.size()),
                                      int64_t(sampling.max_tokens), 1, out.data(),
                                      &produced, nullptr, &st));
    if (stats != nullptr) {
        stats->prefill_tokens = prompt.size();
        stats->generated_tokens = size_t(produced);
        stats->prefill_seconds = st.prefill_seconds;
        stats->decode_seconds = st.decode_seconds;
    }
    return std::vector<int>(out.begin(), out.begin() + produced);
}

/* `prefill` fills the cache from the prompt (the model kind's own prefill
 * and messages). */
template <typename Prefill>
std::vector<int> generate_sampled(nut_model *m, const ModelConfig &config,
                                  const std::vector<int> &prompt,
                                  const SamplingConfig &sampling, KVCache &cache,
                                  GenerationStats *stats, Prefill &&prefill) {
    const auto prefill_start = std::chrono::steady_clock::now();
    prefill();
    const double prefill_seconds = seconds_since(prefill_start);

    nut_kv *kv = cache.device(m);
    std::vector<float> logits(config.vocab_size);
    std::vector<int> generated;
    std::mt19937 rng(sampling.seed);
    const auto decode_start = std::chrono::steady_clock::now();
    while (generated.size() < sampling.max_tokens && cache.length() < cache.capacity()) {
        nutdev::check(nut_logits(m, kv, logits.data(), nullptr));
        const size_t token = choose_token(logits, sampling, rng);
        if (token == config.eos_token)
            break;
        generated.push_back(int(token));
        nutdev::check(nut_decode_token(m, kv, int32_t(token), nullptr));
    }
    if (stats != nullptr) {
        stats->prefill_tokens = prompt.size();
        stats->generated_tokens = generated.size();
        stats->prefill_seconds = prefill_seconds;
        stats->decode_seconds = seconds_since(decode_start);
    }
    return generated;
}

void check_generation(const ModelConfig &config, const std::vector<int> &prompt,
                      const SamplingConfig &sampling) {
    config.validate();
    if (prompt.empty() || prompt.size() > config.max_seq)
        throw std::invalid_argument("generation: invalid prompt length");
    if (sampling.threads == 0)
        throw std::invalid_argument("generation: zero threads");
}

} // namespace

std::vector<int> generate_tokens_cached(const QuantizedModelWeights &model,
                                        const std::vector<int> &prompt,
                                        const SamplingConfig &sampling,
                                        GenerationStats *stats) {
    check_generation(model.config, prompt, sampling);
    KVCache cache(model.config);
    if (sampling.temperature <= 0.0f)
        return generate_greedy(model.device(), prompt, sampling, cache, stats);
    return generate_sampled(model.device(), model.config, prompt, sampling, cache, stats,
                            [&] { prefill_quantized(model, prompt, cache, sampling.threads); });
}

/* The fp32 overload (src/generate.cpp:128-172): prefill_tokens, then per
 * step final norm + classifier, choice, decode_token. */
std::vector<int> generate_tokens_cached(const ModelWeights &model,
                                        const std::vector<int> &prompt,
                                        const SamplingConfig &sampling,
                                        GenerationStats *stats) {
    check_generation(model.config, prompt, sampling);
    KVCache cache(model.config);
    if (sampling.temperature <= 0.0f)
        return generate_greedy(model.device(), prompt, sampling, cache, stats);
    return generate_sampled(model.device(), model.config, prompt, sampling, cache, stats,
                            [&] { prefill_tokens(model, prompt, cache, sampling.threads); });
}

std::vector<int> generate_tokens(const ModelWeights &model, const std::vector<int> &prompt,
                                 const SamplingConfig &sampling) {
    model.config.validate();
    if (prompt.empty())
        throw std::invalid_argument("generation: prompt cannot be empty");
    if (sampling.threads == 0)
        throw std::invalid_argument("generation: zero threads");
    if (prompt.size() > model.config.max_seq)
        throw std::length_error("generation: prompt exceeds context");
    return generate_tokens_cached(model, prompt, sampling, nullptr);
}
