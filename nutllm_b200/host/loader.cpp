/* ModelWeights over the C ABI (nut_model_create_f32).  Errors keep the
 * reference's classes and messages (src/kvcache.cpp:237-284,
 * src/loader.cpp:401-440). */
#include "loader.hpp"

#include <limits>
#include <stdexcept>

#include "device.hpp"

LayerWeights::LayerWeights(const ModelConfig &config)
    : query(config.dim, config.dim), key(config.dim, config.kv_dim()),
      value(config.dim, config.kv_dim()), output(config.dim, config.dim),
      gate(config.dim, config.ffn_dim), up(config.dim, config.ffn_dim),
      down(config.ffn_dim, config.dim), attention_norm(config.dim, 1.0f),
      ffn_norm(config.dim, 1.0f) {
    config.validate();
}

ModelWeights::ModelWeights(const ModelConfig &model_config, bool allocate_lm_head)
    : config(model_config), embeddings(model_config.vocab_size, model_config.dim),
      final_norm(model_config.dim, 1.0f) {
    config.validate();
    if (allocate_lm_head)
        lm_head = Matrix(config.vocab_size, config.dim);
    layers.reserve(config.layers);
    for (size_t l = 0; l < config.layers; l++)
        layers.emplace_back(config);
}

size_t ModelWeights::storage_bytes() const {
    size_t elements = 0;
    auto add = [&elements](size_t v) {
        if (v > std::numeric_limits<size_t>::max() - elements)
            throw std::overflow_error("model: storage size overflow");
        elements += v;
    };
    add(embeddings.size());
    add(final_norm.size());
    add(lm_head.size());
    for (const LayerWeights &l : layers) {
        for (const Matrix *m : {&l.query, &l.key, &l.value, &l.output, &l.gate, &l.up, &l.down})
            add(m->size());
        add(l.attention_norm.size());
        add(l.ffn_norm.size());
    }
    if (elements > std::numeric_limits<size_t>::max() / sizeof(float))
        throw std::overflow_error("model: storage size overflow");
    return elements * sizeof(float);
}

namespace {

/* [in][out] -> [out][in] */
std::vector<float> rows_of(const Matrix &m) {
    std::vector<float> t(m.size());
    const size_t in = m.rows(), out = m.cols();
    for (size_t i = 0; i < in; i++)
        for (size_t o = 0; o < out; o++)
            t[o * in + i] = m.data()[i * out + o];
    return t;
}

void check_model(const ModelWeights &model, const KVCache &cache, size_t thread_count) {
    model.config.validate();
    if (!cache.compatible(model.config))
        throw std::invalid_argument("kv cache: model configuration mismatch");
    if (model.layers.size() != model.config.layers)
        throw std::invalid_argument("kv cache: layer count mismatch");
    if (thread_count == 0)
        throw std::invalid_argument("kv cache: zero threads");
}

} // namespace

nut_model *ModelWeights::device() const {
    if (device_)
        return device_.get();
    if (layers.size() != config.layers)
        throw std::invalid_argument("kv cache: layer count mismatch");
    const ModelConfig &c = config;
    auto shaped = [](const Matrix &m, size_t rows, size_t cols) {
        if (m.rows() != rows || m.cols() != cols)
            throw std::invalid_argument("model: weight shape mismatch");
    };
    std::vector<std::vector<float>> store;
    store.reserve(layers.size() * 7);
    std::vector<nut_layer_f32_view> lv(layers.size());
    for (size_t i = 0; i < layers.size(); i++) {
        const LayerWeights &l = layers[i];
        shaped(l.query, c.dim, c.dim);
        shaped(l.key, c.dim, c.kv_dim());
        shaped(l.value, c.dim, c.kv_dim());
        shaped(l.output, c.dim, c.dim);
        shaped(l.gate, c.dim, c.ffn_dim);
        shaped(l.up, c.dim, c.ffn_dim);
        shaped(l.down, c.ffn_dim, c.dim);
        if (l.attention_norm.size() != c.dim || l.ffn_norm.size() != c.dim)
            throw std::invalid_argument("model: weight shape mismatch");
        const float **dst[7] = {&lv[i].query, &lv[i].key, &lv[i].value, &lv[i].output,
                                &lv[i].gate,  &lv[i].up,  &lv[i].down};
        const Matrix *src[7] = {&l.query, &l.key, &l.value, &l.output, &l.gate, &l.up, &l.down};
        for (int j = 0; j < 7; j++) {
            store.push_back(rows_of(*src[j]));
            *dst[j] = store.back().data();
        }
        lv[i].attention_norm = l.attention_norm.data();
        lv[i].ffn_norm = l.ffn_norm.data();
    }
    nut_model_f32_view v{};
    v.config = nut_config{int64_t(c.layers),     int64_t(c.heads),   int64_t(c.dim),
                          int64_t(c.head_dim),   int64_t(c.ffn_dim), int64_t(c.vocab_size),
                          int64_t(c.max_seq),    int64_t(c.eos_token),
                          int64_t(c.kv_heads)};
    v.tied_embeddings = tied_embeddings ? 1 : 0;
    v.embeddings = embeddings.data();
    v.final_norm = final_norm.data();
    v.lm_head = tied_embeddings ? nullptr : lm_head.data();
    v.layers = lv.data();
    v.n_layers = int64_t(lv.size());
    nut_model *m = nullptr;
    nutdev::check(nut_model_create_f32(&v, nutdev::current_device(), &m));
    device_.reset(m, [](nut_model *p) { nut_model_destroy(p); });
    return m;
}

Matrix prefill_tokens(const ModelWeights &model, const std::vector<int> &tokens,
                      KVCache &cache, size_t thread_count) {
    model.config.validate();
    if (!cache.compatible(model.config))
        throw std::invalid_argument("kv cache: model configuration mismatch");
    if (model.layers.size() != model.config.layers)
        throw std::invalid_argument("kv cache: layer count mismatch");
    if (tokens.empty() || tokens.size() > model.config.max_seq)
        throw std::invalid_argument("kv cache: invalid prefill length");
    if (thread_count == 0)
        throw std::invalid_argument("kv cache: zero threads");
    for (int t : tokens)
        if (t < 0 || size_t(t) >= model.config.vocab_size)
            throw std::out_of_range("kv cache: token id out of range");
    nut_model *m = model.device();
    nut_kv *kv = cache.device(m);
    cache.reset();
    /* one pass per position; each pass leaves that position's row */
    Matrix rows(tokens.size(), model.config.dim);
    for (size_t i = 0; i < tokens.size(); i++)
        nutdev::check(nut_decode_token(m, kv, int32_t(tokens[i]),
                                       rows.data() + i * model.config.dim));
    return rows;
}

std::vector<float> decode_token(const ModelWeights &model, int token, KVCache &cache,
                                size_t thread_count) {
    check_model(model, cache, thread_count);
    nut_model *m = model.device();
    nut_kv *kv = cache.device(m);
    std::vector<float> hidden(model.config.dim);
    nutdev::check(nut_decode_token(m, kv, int32_t(token), hidden.data()));
    return hidden;
}
