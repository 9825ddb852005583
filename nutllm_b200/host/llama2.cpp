/* llama2.c loader.  The checks and their exception classes and messages
 * follow the reference (src/llama2.cpp:133-150,199-298) so callers see the
 * same errors; reading is positioned std::ifstream reads of one tensor at a
 * time.  The quantised loader goes layer by layer: a layer's seven
 * projections are quantised by seven host threads (each matrix on its own,
 * so the bytes do not depend on the split) while the previous layer is
 * packed and uploaded to the device in the background. */
#include "llama2.hpp"

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <exception>
#include <fstream>
#include <limits>
#include <memory>
#include <stdexcept>
#include <thread>
#include <utility>
#include <vector>

namespace {

constexpr size_t kHeaderBytes = 7 * sizeof(int32_t);

size_t mul_checked(size_t a, size_t b, const char *what) {
    if (a != 0 && b > std::numeric_limits<size_t>::max() / a)
        throw std::length_error(std::string("llama2 checkpoint: ") + what + " overflows");
    return a * b;
}

void add_checked(size_t &sum, size_t v) {
    if (v > std::numeric_limits<size_t>::max() - sum)
        throw std::length_error("llama2 checkpoint: size overflows");
    sum += v;
}

size_t dimension(int32_t v, const char *name) {
    if (v <= 0)
        throw std::runtime_error(std::string("llama2 checkpoint: invalid ") + name);
    return size_t(v);
}

/* Section offsets, in floats from the end of the header. */
struct Sections {
    ModelConfig config;
    bool shared_classifier = false;
    size_t embeddings = 0, attention_norms = 0, wq = 0, wk = 0, wv = 0, wo = 0,
           ffn_norms = 0, w1 = 0, w2 = 0, w3 = 0, final_norm = 0, classifier = 0;
};

class Checkpoint {
public:
    explicit Checkpoint(const std::string &path) : in_(path, std::ios::binary) {
        if (!in_)
            throw std::runtime_error("llama2 checkpoint: cannot open " + path);
        in_.seekg(0, std::ios::end);
        const std::streamoff end = in_.tellg();
        if (end < 0)
            throw std::runtime_error("llama2 checkpoint: cannot stat " + path);
        size_ = size_t(end);
        if (size_ == 0)
            throw std::runtime_error("llama2 checkpoint: empty file");
    }

    size_t size() const { return size_; }

    /* count floats starting `first` floats after the header. */
    void read(float *dst, size_t first, size_t count) {
        const size_t at = kHeaderBytes + mul_checked(first, sizeof(float), "read");
        const size_t bytes = mul_checked(count, sizeof(float), "read");
        if (at > size_ || bytes > size_ - at)
            throw std::runtime_error("llama2 checkpoint: read outside file");
        in_.clear();
        in_.seekg(std::streamoff(at));
        in_.read(reinterpret_cast<char *>(dst), std::streamsize(bytes));
        if (!in_)
            throw std::runtime_error("llama2 checkpoint: read failed");
    }

    void header(int32_t (&h)[7]) {
        if (size_ < kHeaderBytes)
            throw std::runtime_error("llama2 checkpoint: truncated header");
        in_.seekg(0);
        in_.read(reinterpret_cast<char *>(h), kHeaderBytes);
        if (!in_)
            throw std::runtime_error("llama2 checkpoint: read failed");
    }

private:
    std::ifstream in_;
    size_t size_ = 0;
};

Sections parse(Checkpoint &file) {
    int32_t h[7];
    file.header(h);
    const size_t dim = dimension(h[0], "dimension");
    const size_t ffn = dimension(h[1], "ffn dimension");
    const size_t layers = dimension(h[2], "layer count");
    const size_t heads = dimension(h[3], "head count");
    const size_t kv_heads = dimension(h[4], "kv head count");
    if (h[5] == 0 || h[5] == std::numeric_limits<int32_t>::min())
        throw std::runtime_error("llama2 checkpoint: invalid vocabulary");
    const size_t vocab = size_t(h[5] > 0 ? h[5] : -h[5]);
    const size_t max_seq = dimension(h[6], "context length");
    if (dim % heads != 0)
        throw std::runtime_error("llama2 checkpoint: heads do not divide dimension");

    Sections s;
    s.config.layers = layers;
    s.config.heads = heads;
    s.config.dim = dim;
    s.config.head_dim = dim / heads;
    s.config.ffn_dim = ffn;
    s.config.vocab_size = vocab;
    s.config.max_seq = max_seq;
    s.config.eos_token = 1;
    s.config.kv_heads = kv_heads;
    s.config.validate();
    s.shared_classifier = h[5] > 0;

    const size_t emb = mul_checked(vocab, dim, "embeddings");
    const size_t norms = mul_checked(layers, dim, "norms");
    const size_t att = mul_checked(layers, mul_checked(dim, dim, "attention matrix"),
                                   "attention weights");
    const size_t kv = mul_checked(layers, mul_checked(dim, s.config.kv_dim(), "kv matrix"),
                                  "kv weights");
    const size_t ff = mul_checked(layers, mul_checked(dim, ffn, "ffn matrix"), "ffn weights");
    const size_t rope = mul_checked(max_seq, s.config.head_dim, "rope frequencies");

    size_t at = 0;
    auto section = [&](size_t count) {
        const size_t here = at;
        add_checked(at, count);
        return here;
    };
    s.embeddings = section(emb);
    s.attention_norms = section(norms);
    s.wq = section(att);
    s.wk = section(kv);
    s.wv = section(kv);
    s.wo = section(att);
    s.ffn_norms = section(norms);
    s.w1 = section(ff);
    s.w2 = section(ff);
    s.w3 = section(ff);
    s.final_norm = section(dim);
    section(rope);
    s.classifier = s.shared_classifier ? s.embeddings : section(emb);
    if (at > (std::numeric_limits<size_t>::max() - kHeaderBytes) / sizeof(float))
        throw std::length_error("llama2 checkpoint: file size overflows");
    if (file.size() != kHeaderBytes + at * sizeof(float))
        throw std::runtime_error("llama2 checkpoint: size does not match configuration");
    return s;
}

/* The seven projections of layer l, read from their sections and
 * quantised by one host thread each (each matrix is quantised on its own,
 * so the bytes do not depend on the split).  `raw` keeps seven fp32
 * buffers across layers. */
QuantizedLayerWeights quantize_layer(Checkpoint &file, const Sections &s, size_t l,
                                     QuantType type, std::vector<std::vector<float>> &raw) {
    const ModelConfig &c = s.config;
    struct Proj {
        size_t first, rows, cols;
    };
    const size_t att = mul_checked(c.dim, c.dim, "quantized projection");
    const size_t kv = mul_checked(c.kv_dim(), c.dim, "quantized projection");
    const size_t ff = mul_checked(c.ffn_dim, c.dim, "quantized projection");
    /* query key value output gate up down, [out][in] as stored */
    const Proj p[7] = {{s.wq + l * att, c.dim, c.dim},     {s.wk + l * kv, c.kv_dim(), c.dim},
                       {s.wv + l * kv, c.kv_dim(), c.dim}, {s.wo + l * att, c.dim, c.dim},
                       {s.w1 + l * ff, c.ffn_dim, c.dim},  {s.w3 + l * ff, c.ffn_dim, c.dim},
                       {s.w2 + l * ff, c.dim, c.ffn_dim}};
    raw.resize(7);
    for (int j = 0; j < 7; j++) {
        raw[j].resize(p[j].rows * p[j].cols);
        file.read(raw[j].data(), p[j].first, raw[j].size());
    }
    std::vector<std::unique_ptr<QuantizedMatrix>> done(7);
    std::vector<std::exception_ptr> errors(7);
    std::vector<std::thread> pool;
    for (int j = 0; j < 7; j++)
        pool.emplace_back([&, j] {
            try {
                done[j].reset(new QuantizedMatrix(
                    QuantizedMatrix::quantize(raw[j].data(), p[j].rows, p[j].cols, type)));
            } catch (...) {
                errors[j] = std::current_exception();
            }
        });
    for (std::thread &t : pool)
        t.join();
    for (int j = 0; j < 7; j++)
        if (errors[j])
            std::rethrow_exception(errors[j]);
    std::vector<float> an(c.dim), fn(c.dim);
    file.read(an.data(), s.attention_norms + l * c.dim, c.dim);
    file.read(fn.data(), s.ffn_norms + l * c.dim, c.dim);
    return QuantizedLayerWeights(std::move(*done[0]), std::move(*done[1]), std::move(*done[2]),
                                 std::move(*done[3]), std::move(*done[4]), std::move(*done[5]),
                                 std::move(*done[6]), std::move(an), std::move(fn));
}

/* One stored [out][in] projection of a layer into the reference's
 * [in][out] Matrix (transpose_external, src/llama2.cpp:300-337). */
void read_transposed(Checkpoint &file, size_t first, Matrix &dst, std::vector<float> &raw) {
    const size_t in = dst.rows(), out = dst.cols();
    raw.resize(in * out);
    file.read(raw.data(), first, raw.size());
    for (size_t o = 0; o < out; o++)
        for (size_t i = 0; i < in; i++)
            dst.data()[i * out + o] = raw[o * in + i];
}

} // namespace

ModelWeights load_llama2c_model(const std::string &path) {
    Checkpoint file(path);
    const Sections s = parse(file);
    const ModelConfig &c = s.config;
    ModelWeights model(c, !s.shared_classifier);
    model.tied_embeddings = s.shared_classifier;
    file.read(model.embeddings.data(), s.embeddings, c.vocab_size * c.dim);
    file.read(model.final_norm.data(), s.final_norm, c.dim);
    if (!s.shared_classifier)
        file.read(model.lm_head.data(), s.classifier, c.vocab_size * c.dim);
    const size_t att = c.dim * c.dim, kv = c.dim * c.kv_dim(), ff = c.dim * c.ffn_dim;
    std::vector<float> raw;
    for (size_t l = 0; l < c.layers; l++) {
        LayerWeights &d = model.layers[l];
        file.read(d.attention_norm.data(), s.attention_norms + l * c.dim, c.dim);
        file.read(d.ffn_norm.data(), s.ffn_norms + l * c.dim, c.dim);
        read_transposed(file, s.wq + l * att, d.query, raw);
        read_transposed(file, s.wk + l * kv, d.key, raw);
        read_transposed(file, s.wv + l * kv, d.value, raw);
        read_transposed(file, s.wo + l * att, d.output, raw);
        read_transposed(file, s.w1 + l * ff, d.gate, raw);
        read_transposed(file, s.w2 + l * ff, d.down, raw);
        read_transposed(file, s.w3 + l * ff, d.up, raw);
    }
    return model;
}

/* Streams to the device while it loads: the fp32 tensors first (their
 * device copy starts at once), then layer by layer, each quantised on the
 * host while a background thread packs and uploads the previous one
 * (StreamingUpload), so on a GPU host the returned weights already carry
 * their device image.  The host storage and the checks are those of the
 * reference loader (src/llama2.cpp:339-412). */
QuantizedModelWeights load_llama2c_quantized_model(const std::string &path, QuantType type) {
    Checkpoint file(path);
    const Sections s = parse(file);
    const ModelConfig &c = s.config;
    QuantizedModelWeights model(c, type, !s.shared_classifier);
    model.tied_embeddings = s.shared_classifier;
    file.read(model.embeddings.data(), s.embeddings, c.vocab_size * c.dim);
    file.read(model.final_norm.data(), s.final_norm, c.dim);
    if (!s.shared_classifier)
        file.read(model.lm_head.data(), s.classifier, c.vocab_size * c.dim);
    model.layers.reserve(c.layers); /* the uploader reads earlier layers in place */
    StreamingUpload upload(model);
    std::vector<std::vector<float>> raw;
    for (size_t l = 0; l < c.layers; l++) {
        model.layers.push_back(quantize_layer(file, s, l, type, raw));
        upload.add(l);
    }
    upload.finish(model);
    return model;
}

/* ---- tokenizer -------------------------------------------------------- */

Llama2Tokenizer Llama2Tokenizer::load(const std::string &path, size_t vocab_size) {
    if (vocab_size == 0 || vocab_size > size_t(std::numeric_limits<int>::max()))
        throw std::invalid_argument("llama2 tokenizer: invalid vocabulary");
    std::ifstream in(path, std::ios::binary);
    if (!in)
        throw std::runtime_error("llama2 tokenizer: cannot open " + path);
    uint32_t max_len = 0;
    in.read(reinterpret_cast<char *>(&max_len), sizeof max_len);
    if (!in || max_len == 0)
        throw std::runtime_error("llama2 tokenizer: invalid header");
    Llama2Tokenizer t;
    t.max_length_ = max_len;
    t.pieces_.reserve(vocab_size);
    t.scores_.reserve(vocab_size);
    for (size_t id = 0; id < vocab_size; id++) {
        float score = 0.0f;
        int32_t len = 0;
        in.read(reinterpret_cast<char *>(&score), sizeof score);
        in.read(reinterpret_cast<char *>(&len), sizeof len);
        if (!in || !std::isfinite(score) || len <= 0 || size_t(len) > t.max_length_)
            throw std::runtime_error("llama2 tokenizer: malformed vocabulary entry");
        std::string piece(size_t(len), '\0');
        in.read(&piece[0], len);
        if (!in)
            throw std::runtime_error("llama2 tokenizer: truncated token");
        t.scores_.push_back(score);
        t.pieces_.push_back(std::move(piece));
    }
    if (in.peek() != std::char_traits<char>::eof())
        throw std::runtime_error("llama2 tokenizer: trailing data");
    t.ids_.reserve(t.pieces_.size());
    for (size_t id = 0; id < t.pieces_.size(); id++)
        t.ids_.emplace(t.pieces_[id], int(id)); /* keeps the first id of a piece */
    return t;
}

int Llama2Tokenizer::find(const std::string &piece) const {
    const auto it = ids_.find(piece);
    return it == ids_.end() ? -1 : it->second;
}

std::vector<int> Llama2Tokenizer::encode(const std::string &text, bool bos, bool eos) const {
    std::vector<int> out;
    out.reserve(text.size() + 3);
    if (bos)
        out.push_back(1);
    if (!text.empty()) {
        const int space = find(" ");
        if (space < 0)
            throw std::runtime_error("llama2 tokenizer: dummy prefix token missing");
        out.push_back(space);
    }
    /* one token per UTF-8 character: a lead byte and up to three
     * continuation bytes (10xxxxxx) */
    size_t i = 0;
    while (i < text.size()) {
        size_t j = i + 1;
        while (j < text.size() && j - i < 4 &&
               (static_cast<unsigned char>(text[j]) & 0xC0u) == 0x80u)
            j++;
        const std::string ch = text.substr(i, j - i);
        const int id = find(ch);
        if (id >= 0) {
            out.push_back(id);
        } else {
            for (unsigned char c : ch) {
                if (size_t(c) + 3 >= pieces_.size())
                    throw std::runtime_error("llama2 tokenizer: byte fallback unavailable");
                out.push_back(int(c) + 3);
            }
        }
        i = j;
    }
    /* merge the best-scoring adjacent pair until none forms a token */
    for (;;) {
        size_t at = out.size();
        int merged = -1;
        float best = -std::numeric_limits<float>::infinity();
        for (size_t k = 0; k + 1 < out.size(); k++) {
            const int id = find(pieces_[size_t(out[k])] + pieces_[size_t(out[k + 1])]);
            if (id >= 0 && scores_[size_t(id)] > best) {
                best = scores_[size_t(id)];
                at = k;
                merged = id;
            }
        }
        if (at == out.size())
            break;
        out[at] = merged;
        out.erase(out.begin() + std::ptrdiff_t(at) + 1);
    }
    if (eos)
        out.push_back(2);
    return out;
}

std::string Llama2Tokenizer::decode(const std::vector<int> &tokens) const {
    auto hex = [](char c) -> int {
        if (c >= '0' && c <= '9')
            return c - '0';
        if (c >= 'a' && c <= 'f')
            return c - 'a' + 10;
        if (c >= 'A' && c <= 'F')
            return c - 'A' + 10;
        return -1;
    };
    std::string text;
    size_t k = 0;
    int prev = -1;
    if (!tokens.empty() && tokens[0] == 1) {
        prev = 1;
        k = 1;
    }
    for (; k < tokens.size(); k++) {
        const int id = tokens[k];
        if (id < 0 || size_t(id) >= pieces_.size())
            throw std::out_of_range("llama2 tokenizer: token id out of range");
        std::string piece = pieces_[size_t(id)];
        if (prev == 1 && !piece.empty() && piece[0] == ' ')
            piece.erase(0, 1);
        if (piece.size() == 6 && piece.compare(0, 3, "<0x") == 0 && piece[5] == '>') {
            const int hi = hex(piece[3]), lo = hex(piece[4]);
            if (hi >= 0 && lo >= 0)
                piece.assign(1, char((hi << 4) | lo));
        }
        text += piece;
        prev = id;
    }
    return text;
}
