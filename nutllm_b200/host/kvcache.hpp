#pragma once
/* KVCache — host side of the drop-in for the reference's include/kvcache.hpp:
 * 8-31 (src/kvcache.cpp:173-235).  The keys and values live on the device
 * (nut_kv, fp32 [layer][kv_head][max_seq][head_dim], the reference layout);
 * this object owns that device cache once it is first used with a model,
 * and key() / value() copy one vector back into host scratch (valid until
 * the next key() / value() call on this object). */
#include <cstddef>
#include <memory>
#include <vector>

#include "model.hpp"

struct nut_kv;
struct nut_model;

class KVCache {
public:
    explicit KVCache(const ModelConfig &config);

    size_t length() const;
    size_t capacity() const { return config_.max_seq; }
    size_t memory_bytes() const;
    bool compatible(const ModelConfig &config) const;
    void reset();

    const float *key(size_t layer, size_t head, size_t position) const;
    const float *value(size_t layer, size_t head, size_t position) const;
    void store(size_t layer, size_t position, const float *key, const float *value);
    void set_length(size_t length);

    /* The device cache bound to `model` (created on first use; a cache used
     * with another model of the same shape starts empty on it). */
    nut_kv *device(nut_model *model);

private:
    ModelConfig config_;
    nut_model *model_ = nullptr;
    std::shared_ptr<nut_kv> kv_;
    size_t pending_length_ = 0; /* length set before a device cache exists */
    mutable std::vector<float> scratch_;
};
