#pragma once
/* Generation — host side of the drop-in for the reference's
 * include/generate.hpp:11-36 (both overloads of generate_tokens_cached,
 * src/generate.cpp:128-216).
 *
 * temperature <= 0 (greedy) runs the whole loop on the device
 * (nut_generate_greedy: prefill, then final norm + classifier + argmax and
 * the next token's forward in one persistent launch), and the statistics
 * are device-event times.  temperature > 0 reads each step's logits back
 * and draws on the host with the reference's sampler, so a given seed picks
 * the same ids as the reference for the same logits; its statistics are
 * wall-clock, as in the reference. */
#include <cstddef>
#include <cstdint>
#include <random>
#include <vector>

struct QuantizedModelWeights;
struct ModelWeights;

struct SamplingConfig {
    size_t max_tokens = 32;
    float temperature = 0.0f;
    float top_p = 1.0f;
    uint32_t seed = 1;
    size_t threads = 1;
};

struct GenerationStats {
    size_t prefill_tokens = 0;
    size_t generated_tokens = 0;
    double prefill_seconds = 0.0;
    double decode_seconds = 0.0;
};

std::vector<int> generate_tokens_cached(const QuantizedModelWeights &model,
                                        const std::vector<int> &prompt,
                                        const SamplingConfig &sampling,
                                        GenerationStats *stats = nullptr);
/* The fp32-weight overload (src/generate.cpp:128-172), same loop. */
std::vector<int> generate_tokens_cached(const ModelWeights &model,
                                        const std::vector<int> &prompt,
                                        const SamplingConfig &sampling,
                                        GenerationStats *stats = nullptr);

/* generate_tokens (src/generate.cpp:101-126): the reference recomputes the
 * whole prefix every step; here the same loop runs through the device KV
 * cache (the same ids up to rounding order — the reference's own selftest
 * holds the two equal, src/kvcache_selftest.cpp:97-115).  Checks and
 * messages are generate_tokens' own. */
std::vector<int> generate_tokens(const ModelWeights &model, const std::vector<int> &prompt,
                                 const SamplingConfig &sampling);

/* The token choice of one step (src/generate.cpp:25-73): first-index argmax
 * for temperature <= 0; otherwise a draw from the smallest set of most
 * probable tokens whose probability reaches top_p.  Exposed for tests. */
size_t choose_token(const std::vector<float> &logits, const SamplingConfig &sampling,
                    std::mt19937 &rng);
