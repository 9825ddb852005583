#pragma once
/* Model shape, as the reference's ModelConfig (include/model.hpp:8-24,
 * validate at src/attention.cpp:15-27). */
#include <cstddef>
#include <limits>
#include <stdexcept>

struct ModelConfig {
    size_t layers = 0;
    size_t heads = 0;
    size_t dim = 0;
    size_t head_dim = 0;
    size_t ffn_dim = 0;
    size_t vocab_size = 0;
    size_t max_seq = 0;
    size_t eos_token = 0;
    size_t kv_heads = 0;

    size_t effective_kv_heads() const { return kv_heads == 0 ? heads : kv_heads; }
    size_t kv_dim() const { return effective_kv_heads() * head_dim; }

    /* heads * head_dim == dim, even head_dim, heads divisible by kv heads,
     * eos inside the vocabulary; std::invalid_argument otherwise. */
    void validate() const {
        const size_t kv = effective_kv_heads();
        if (layers == 0 || heads == 0 || dim == 0 || head_dim == 0 ||
            ffn_dim == 0 || vocab_size == 0 || max_seq == 0 ||
            heads > std::numeric_limits<size_t>::max() / head_dim ||
            heads * head_dim != dim || head_dim % 2 != 0 ||
            eos_token >= vocab_size || kv == 0 || kv > heads ||
            heads % kv != 0 ||
            kv > std::numeric_limits<size_t>::max() / head_dim)
            throw std::invalid_argument("model config: invalid dimensions");
    }
};
