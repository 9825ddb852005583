/* KVCache over the device cache of the C ABI (nut_kv).  Error classes and
 * messages follow the reference (src/kvcache.cpp:173-235). */
#include "kvcache.hpp"

#include <stdexcept>

#include "device.hpp"

KVCache::KVCache(const ModelConfig &config) : config_(config) { config_.validate(); }

size_t KVCache::length() const {
    if (!kv_)
        return pending_length_;
    int64_t n = 0;
    nutdev::check(nut_kv_length(kv_.get(), &n));
    return size_t(n);
}

size_t KVCache::memory_bytes() const {
    /* keys and values, fp32, [layers][kv_heads][max_seq][head_dim] each */
    return 2 * config_.layers * config_.effective_kv_heads() * config_.max_seq *
           config_.head_dim * sizeof(float);
}

bool KVCache::compatible(const ModelConfig &config) const {
    return config.layers == config_.layers && config.max_seq == config_.max_seq &&
           config.kv_dim() == config_.kv_dim() && config.head_dim == config_.head_dim;
}

void KVCache::reset() {
    pending_length_ = 0;
    if (kv_)
        nutdev::check(nut_kv_reset(kv_.get()));
}

void KVCache::set_length(size_t length) {
    if (length > capacity())
        throw std::length_error("kv cache: context exceeds capacity");
    if (!kv_) {
        pending_length_ = length;
        return;
    }
    nutdev::check(nut_kv_set_length(kv_.get(), int64_t(length)));
}

nut_kv *KVCache::device(nut_model *model) {
    if (model == nullptr)
        throw std::invalid_argument("kv cache: null model");
    if (kv_ && model_ == model)
        return kv_.get();
    nut_kv *kv = nullptr;
    nutdev::check(nut_kv_create(model, &kv));
    kv_.reset(kv, [](nut_kv *p) { nut_kv_destroy(p); });
    model_ = model;
    if (pending_length_ != 0)
        nutdev::check(nut_kv_set_length(kv, int64_t(pending_length_)));
    return kv;
}

const float *KVCache::key(size_t layer, size_t head, size_t position) const {
    if (!kv_)
        throw std::logic_error("kv cache: not bound to a model yet");
    scratch_.resize(config_.head_dim);
    nutdev::check(nut_kv_read(kv_.get(), int64_t(layer), int64_t(head), int64_t(position),
                              scratch_.data(), nullptr));
    return scratch_.data();
}

const float *KVCache::value(size_t layer, size_t head, size_t position) const {
    if (!kv_)
        throw std::logic_error("kv cache: not bound to a model yet");
    scratch_.resize(config_.head_dim);
    nutdev::check(nut_kv_read(kv_.get(), int64_t(layer), int64_t(head), int64_t(position),
                              nullptr, scratch_.data()));
    return scratch_.data();
}

void KVCache::store(size_t layer, size_t position, const float *key, const float *value) {
    if (key == nullptr || value == nullptr)
        throw std::invalid_argument("kv cache: null source");
    if (!kv_)
        throw std::logic_error("kv cache: not bound to a model yet");
    nutdev::check(nut_kv_write(kv_.get(), int64_t(layer), int64_t(position), key, value));
}
