#pragma once
/* Quantised decoder weights and the per-token forward — host side of the
 * drop-in for the reference's include/quant_model.hpp:9-53.
 *
 * The weights stay in host memory in the reference's storage (so existing
 * loaders fill them unchanged); the first prefill or decode uploads them
 * once to the current device (nut_model_create) and every later call runs
 * the token loop there.  thread_count is accepted for interface parity and
 * must be non-zero, as in the reference; the device ignores it. */
#include <cstddef>
#include <memory>
#include <vector>

#include "kvcache.hpp"
#include "model.hpp"
#include "quant.hpp"
#include "tensor.hpp"

struct nut_model;

struct QuantizedLayerWeights {
    QuantizedLayerWeights(QuantizedMatrix query_weight, QuantizedMatrix key_weight,
                          QuantizedMatrix value_weight, QuantizedMatrix output_weight,
                          QuantizedMatrix gate_weight, QuantizedMatrix up_weight,
                          QuantizedMatrix down_weight, std::vector<float> attention_norm_weight,
                          std::vector<float> ffn_norm_weight);

    QuantizedMatrix query;
    QuantizedMatrix key;
    QuantizedMatrix value;
    QuantizedMatrix output;
    QuantizedMatrix gate;
    QuantizedMatrix up;
    QuantizedMatrix down;
    std::vector<float> attention_norm;
    std::vector<float> ffn_norm;
};

struct QuantizedModelWeights {
    ModelConfig config;
    Matrix embeddings;
    std::vector<QuantizedLayerWeights> layers;
    std::vector<float> final_norm;
    Matrix lm_head;
    bool tied_embeddings = false;
    QuantType quant_type;

    QuantizedModelWeights(const ModelConfig &model_config, QuantType type,
                          bool allocate_lm_head);
    const Matrix &output_weights() const { return tied_embeddings ? embeddings : lm_head; }
    size_t storage_bytes() const;

    /* The device image (uploaded on first use; later changes to the host
     * weights are not seen by it). */
    nut_model *device() const;
    /* Takes ownership of a finished device image of these weights (built
     * by a streaming loader), so first use does not upload them again. */
    void adopt_device(nut_model *model);

private:
    mutable std::shared_ptr<nut_model> device_;
};

/* Builds the device image of a model while a loader is still producing its
 * layers: the constructor uploads the fp32 tensors (nut_model_begin) when a
 * device is present, add(l) queues layer l for a background thread that
 * packs and uploads it (nut_model_add_layer) while the loader reads and
 * quantises the next one, and finish() waits for the thread, completes the
 * image (nut_model_finish) and gives it to the weights.  Without a device,
 * or if any device step fails, it stands aside and the weights keep the
 * upload-on-first-use path (which then reports the failure). */
class StreamingUpload {
public:
    explicit StreamingUpload(const QuantizedModelWeights &model);
    ~StreamingUpload();
    StreamingUpload(const StreamingUpload &) = delete;
    StreamingUpload &operator=(const StreamingUpload &) = delete;
    void add(size_t layer);
    void finish(QuantizedModelWeights &model);
    bool active() const;

private:
    struct State;
    std::unique_ptr<State> state_;
};

std::vector<float> prefill_quantized(const QuantizedModelWeights &model,
                                     const std::vector<int> &tokens, KVCache &cache,
                                     size_t thread_count);
std::vector<float> decode_quantized_token(const QuantizedModelWeights &model, int token,
                                          KVCache &cache, size_t thread_count);
