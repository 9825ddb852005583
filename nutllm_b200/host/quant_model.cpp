/* QuantizedModelWeights over the C ABI (nut_model): the host image is
 * described by a nut_model_view (pointers into this object's own storage)
 * and uploaded once.  Errors keep the reference's classes and messages
 * (src/quant_model.cpp:140-220). */
#include "quant_model.hpp"

#include <condition_variable>
#include <deque>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <utility>

#include "device.hpp"

QuantizedLayerWeights::QuantizedLayerWeights(
    QuantizedMatrix query_weight, QuantizedMatrix key_weight, QuantizedMatrix value_weight,
    QuantizedMatrix output_weight, QuantizedMatrix gate_weight, QuantizedMatrix up_weight,
    QuantizedMatrix down_weight, std::vector<float> attention_norm_weight,
    std::vector<float> ffn_norm_weight)
    : query(std::move(query_weight)), key(std::move(key_weight)),
      value(std::move(value_weight)), output(std::move(output_weight)),
      gate(std::move(gate_weight)), up(std::move(up_weight)), down(std::move(down_weight)),
      attention_norm(std::move(attention_norm_weight)),
      ffn_norm(std::move(ffn_norm_weight)) {}

QuantizedModelWeights::QuantizedModelWeights(const ModelConfig &model_config, QuantType type,
                                             bool allocate_lm_head)
    : config(model_config), embeddings(model_config.vocab_size, model_config.dim),
      final_norm(model_config.dim, 1.0f), quant_type(type) {
    config.validate();
    if (allocate_lm_head)
        lm_head = Matrix(config.vocab_size, config.dim);
    tied_embeddings = !allocate_lm_head;
}

size_t QuantizedModelWeights::storage_bytes() const {
    /* the quantised projections, the fp32 norms, embeddings, final norm and
     * (if separate) the classifier */
    size_t bytes = embeddings.size() * sizeof(float) + final_norm.size() * sizeof(float);
    if (!tied_embeddings)
        bytes += lm_head.size() * sizeof(float);
    for (const QuantizedLayerWeights &l : layers) {
        for (const QuantizedMatrix *m : {&l.query, &l.key, &l.value, &l.output, &l.gate,
                                         &l.up, &l.down})
            bytes += m->storage_bytes();
        bytes += (l.attention_norm.size() + l.ffn_norm.size()) * sizeof(float);
    }
    return bytes;
}

namespace {

nut_qmatrix_view view_of(const QuantizedMatrix &m) {
    nut_qmatrix_view v{};
    v.data = m.data().data();
    v.scales = m.scales().data();
    v.rows = int64_t(m.rows());
    v.cols = int64_t(m.cols());
    v.block_size = int64_t(m.block_size());
    v.type = m.type() == QuantType::int8 ? NUT_QUANT_INT8 : NUT_QUANT_INT4;
    return v;
}

/* The host-side checks of decode_quantized_token, in the reference's order
 * (src/quant_model.cpp:161-172); token range and a full context are
 * checked by the C ABI with the same classes and messages. */
void check_decode(const QuantizedModelWeights &model, const KVCache &cache,
                  size_t thread_count) {
    model.config.validate();
    if (!cache.compatible(model.config))
        throw std::invalid_argument("quantized decode: cache configuration mismatch");
    if (model.layers.size() != model.config.layers)
        throw std::invalid_argument("quantized decode: layer count mismatch");
    if (thread_count == 0)
        throw std::invalid_argument("quantized decode: zero threads");
}

nut_layer_view layer_view(const QuantizedLayerWeights &l) {
    nut_layer_view v{};
    v.query = view_of(l.query);
    v.key = view_of(l.key);
    v.value = view_of(l.value);
    v.output = view_of(l.output);
    v.gate = view_of(l.gate);
    v.up = view_of(l.up);
    v.down = view_of(l.down);
    v.attention_norm = l.attention_norm.data();
    v.ffn_norm = l.ffn_norm.data();
    return v;
}

/* The fp32 tensors and configuration; `layers` is left to the caller. */
nut_model_view model_view(const QuantizedModelWeights &w) {
    const ModelConfig &config = w.config;
    nut_model_view v{};
    v.config = nut_config{int64_t(config.layers),    int64_t(config.heads),
                          int64_t(config.dim),       int64_t(config.head_dim),
                          int64_t(config.ffn_dim),   int64_t(config.vocab_size),
                          int64_t(config.max_seq),   int64_t(config.eos_token),
                          int64_t(config.kv_heads)};
    v.quant_type = w.quant_type == QuantType::int8 ? NUT_QUANT_INT8 : NUT_QUANT_INT4;
    v.tied_embeddings = w.tied_embeddings ? 1 : 0;
    v.embeddings = w.embeddings.data();
    v.final_norm = w.final_norm.data();
    v.lm_head = w.tied_embeddings ? nullptr : w.lm_head.data();
    v.n_layers = int64_t(config.layers);
    return v;
}

} // namespace

nut_model *QuantizedModelWeights::device() const {
    if (device_)
        return device_.get();
    if (layers.size() != config.layers)
        throw std::invalid_argument("quantized decode: layer count mismatch");
    std::vector<nut_layer_view> lv(layers.size());
    for (size_t i = 0; i < layers.size(); i++)
        lv[i] = layer_view(layers[i]);
    nut_model_view v = model_view(*this);
    v.layers = lv.data();
    v.n_layers = int64_t(lv.size());
    nut_model *m = nullptr;
    nutdev::check(nut_model_create(&v, nutdev::current_device(), &m));
    device_.reset(m, [](nut_model *p) { nut_model_destroy(p); });
    return m;
}

void QuantizedModelWeights::adopt_device(nut_model *m) {
    device_.reset(m, [](nut_model *p) { nut_model_destroy(p); });
}

/* ---- streaming upload ---------------------------------------------------- */

struct StreamingUpload::State {
    const QuantizedModelWeights *weights = nullptr;
    nut_model *model = nullptr;
    std::mutex lock;
    std::condition_variable wake;
    std::deque<size_t> queue;
    bool closing = false;
    bool failed = false;
    std::thread worker;

    void run() {
        for (;;) {
            size_t l = 0;
            {
                std::unique_lock<std::mutex> g(lock);
                wake.wait(g, [&] { return closing || !queue.empty(); });
                if (queue.empty())
                    return;
                l = queue.front();
                queue.pop_front();
            }
            if (failed)
                continue;
            const nut_layer_view v = layer_view(weights->layers[l]);
            if (nut_model_add_layer(model, &v) != NUT_OK) {
                std::lock_guard<std::mutex> g(lock);
                failed = true;
            }
        }
    }
    void stop() {
        {
            std::lock_guard<std::mutex> g(lock);
            closing = true;
        }
        wake.notify_all();
        if (worker.joinable())
            worker.join();
    }
};

StreamingUpload::StreamingUpload(const QuantizedModelWeights &weights)
    : state_(new State) {
    int count = 0;
    if (nut_device_count(&count) != NUT_OK || count <= 0)
        return;
    const nut_model_view v = model_view(weights);
    nut_model *m = nullptr;
    if (nut_model_begin(&v, nutdev::current_device(), &m) != NUT_OK)
        return;
    state_->weights = &weights;
    state_->model = m;
    state_->worker = std::thread([s = state_.get()] { s->run(); });
}

StreamingUpload::~StreamingUpload() {
    state_->stop();
    if (state_->model != nullptr)
        nut_model_destroy(state_->model);
}

bool StreamingUpload::active() const { return state_->model != nullptr; }

void StreamingUpload::add(size_t layer) {
    if (state_->model == nullptr)
        return;
    {
        std::lock_guard<std::mutex> g(state_->lock);
        state_->queue.push_back(layer);
    }
    state_->wake.notify_one();
}

void StreamingUpload::finish(QuantizedModelWeights &weights) {
    state_->stop();
    nut_model *m = state_->model;
    if (m == nullptr)
        return;
    state_->model = nullptr;
    if (state_->failed || weights.layers.size() != weights.config.layers ||
        nut_model_finish(m) != NUT_OK) {
        nut_model_destroy(m); /* first use uploads again and reports the error */
        return;
    }
    weights.adopt_device(m);
}

std::vector<float> prefill_quantized(const QuantizedModelWeights &model,
                                     const std::vector<int> &tokens, KVCache &cache,
                                     size_t thread_count) {
    if (tokens.empty() || tokens.size() > cache.capacity())
        throw std::invalid_argument("quantized prefill: invalid prompt");
    check_decode(model, cache, thread_count);
    nut_model *m = model.device();
    nut_kv *kv = cache.device(m);
    std::vector<float> hidden(model.config.dim);
    std::vector<int32_t> ids(tokens.begin(), tokens.end());
    nutdev::check(nut_prefill(m, kv, ids.data(), int64_t(ids.size()), hidden.data()));
    return hidden;
}

std::vector<float> decode_quantized_token(const QuantizedModelWeights &model, int token,
                                          KVCache &cache, size_t thread_count) {
    check_decode(model, cache, thread_count);
    nut_model *m = model.device();
    nut_kv *kv = cache.device(m);
    std::vector<float> hidden(model.config.dim);
    nutdev::check(nut_decode_token(m, kv, int32_t(token), hidden.data()));
    return hidden;
}
