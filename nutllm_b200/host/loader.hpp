#pragma once
/* fp32 decoder weights and their per-token forward — host side of the
 * drop-in for the reference's LayerWeights (include/model.hpp:26-38),
 * ModelWeights (include/loader.hpp:46-60) and prefill_tokens / decode_token
 * (include/kvcache.hpp:33-38).
 *
 * Matrices keep the reference's storage, [in][out] (query [dim][dim], key
 * and value [dim][kv_dim], gate and up [dim][ffn], down [ffn][dim]), so
 * loaders fill them unchanged; the first prefill or decode uploads them
 * once, transposed to [out][in] rows for the device matvec
 * (nut_model_create_f32).  thread_count must be non-zero, as in the
 * reference; the device ignores it. */
#include <cstddef>
#include <memory>
#include <vector>

#include "kvcache.hpp"
#include "model.hpp"
#include "tensor.hpp"

struct nut_model;

struct LayerWeights {
    explicit LayerWeights(const ModelConfig &config);

    Matrix query;
    Matrix key;
    Matrix value;
    Matrix output;
    Matrix gate;
    Matrix up;
    Matrix down;
    std::vector<float> attention_norm;
    std::vector<float> ffn_norm;
};

struct ModelWeights {
    ModelConfig config;
    Matrix embeddings;
    std::vector<LayerWeights> layers;
    std::vector<float> final_norm;
    Matrix lm_head;
    bool tied_embeddings = false;

    explicit ModelWeights(const ModelConfig &model_config, bool allocate_lm_head = true);
    const Matrix &output_weights() const { return tied_embeddings ? embeddings : lm_head; }
    size_t storage_bytes() const;

    /* The device image (uploaded on first use; later changes to the host
     * weights are not seen by it). */
    nut_model *device() const;

private:
    mutable std::shared_ptr<nut_model> device_;
};

/* The hidden rows of every prompt position after the last layer (the
 * reference's prefill_tokens result, [tokens][dim]); the cache holds the
 * prompt afterwards. */
Matrix prefill_tokens(const ModelWeights &model, const std::vector<int> &tokens,
                      KVCache &cache, size_t thread_count = 1);
std::vector<float> decode_token(const ModelWeights &model, int token, KVCache &cache,
                                size_t thread_count = 1);
