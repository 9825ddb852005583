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
#include <map>
#include <memory>
#include <string>
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

/* Safetensors checkpoints (include/loader.hpp:11-45, src/loader.cpp:24-498).
 *
 * SafeTensorFile maps the file read-only and parses its header: a
 * little-endian uint64 length, then that many bytes of JSON — an object
 * whose "__metadata__" member maps names to strings and whose other
 * members describe one F32 tensor each ({"dtype": "F32", "shape": [..],
 * "data_offsets": [begin, end]}, byte offsets after the header).  The JSON
 * accepted is the reference's subset: objects (duplicate keys rejected),
 * arrays, strings with the escapes \" \\ \/ \b \f \n \r \t, and
 * unsigned decimal integers.  Tensor views point into the mapping, which
 * lives as long as the SafeTensorFile (or a copy of its storage).
 *
 * load_model reads a Llama-style fp32 checkpoint: config from the metadata
 * strings nutllm.{layers, heads, dim, head_dim, ffn_dim, vocab_size,
 * max_seq, eos_token} (decimal), tensors model.embed_tokens.weight,
 * model.layers.N.self_attn.{q,k,v,o}_proj.weight,
 * model.layers.N.mlp.{gate,up,down}_proj.weight ([out][in], transposed into
 * the [in][out] matrices), model.layers.N.{input,post_attention}_layernorm
 * .weight, model.norm.weight and lm_head.weight.  Errors keep the
 * reference's classes and messages. */
struct TensorView {
    const float *data = nullptr;
    std::vector<size_t> shape;
    size_t elements = 0;
};

class SafeTensorFile {
public:
    static SafeTensorFile load(const std::string &path);

    SafeTensorFile();
    ~SafeTensorFile();
    SafeTensorFile(SafeTensorFile &&) noexcept;
    SafeTensorFile &operator=(SafeTensorFile &&) noexcept;
    SafeTensorFile(const SafeTensorFile &) = delete;
    SafeTensorFile &operator=(const SafeTensorFile &) = delete;

    TensorView tensor(const std::string &name) const;
    const std::string &metadata(const std::string &name) const;

private:
    struct Mapping;
    struct Entry {
        std::vector<size_t> shape;
        size_t begin = 0, end = 0;
    };
    std::shared_ptr<Mapping> mapping_;
    std::map<std::string, Entry> tensors_;
    std::map<std::string, std::string> metadata_;
    size_t payload_ = 0; /* first payload byte */
};

ModelWeights load_model(const std::string &path);
