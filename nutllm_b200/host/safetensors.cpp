/* Safetensors reader and the fp32 Llama checkpoint loader (load_model),
 * host side of the reference's src/loader.cpp:24-498.  The accepted JSON
 * language, the order of the checks and the error texts follow the
 * reference, so a file either loads in both or fails in both with the same
 * message; the code is this library's own. */
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>
#include <utility>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "loader.hpp"

namespace {

/* One JSON value of the header language. */
struct Node {
    enum Kind { kText, kInteger, kList, kDict } kind = kDict;
    std::string text;
    uint64_t integer = 0;
    std::vector<Node> list;
    std::map<std::string, Node> dict;
};

class HeaderParser {
public:
    HeaderParser(const char *p, size_t n) : p_(p), n_(n) {}

    Node document() {
        Node v = value();
        skip_space();
        if (at_ != n_)
            bad("trailing content");
        return v;
    }

private:
    [[noreturn]] void bad(const char *what) const {
        throw std::runtime_error(std::string("safetensors: malformed JSON: ") + what);
    }
    bool more() const { return at_ < n_; }
    char peek() const { return p_[at_]; }
    char next() {
        if (!more())
            bad("unexpected end");
        return p_[at_++];
    }
    void skip_space() {
        while (more() && (peek() == ' ' || peek() == '\t' || peek() == '\n' || peek() == '\r'))
            at_++;
    }

    Node value() {
        skip_space();
        if (!more())
            bad("missing value");
        const char c = peek();
        Node v;
        if (c == '"') {
            v.kind = Node::kText;
            v.text = string();
        } else if (c == '{') {
            v = dict();
        } else if (c == '[') {
            v = list();
        } else if (c >= '0' && c <= '9') {
            v.kind = Node::kInteger;
            while (more() && peek() >= '0' && peek() <= '9') {
                const uint64_t d = uint64_t(peek() - '0');
                if (v.integer > (std::numeric_limits<uint64_t>::max() - d) / 10)
                    bad("integer overflow");
                v.integer = v.integer * 10 + d;
                at_++;
            }
        } else {
            bad("unsupported value");
        }
        return v;
    }

    std::string string() {
        if (next() != '"')
            bad("expected string");
        std::string out;
        while (more()) {
            const char c = next();
            if (c == '"')
                return out;
            if (static_cast<unsigned char>(c) < 0x20)
                bad("control character in string");
            if (c != '\\') {
                out += c;
                continue;
            }
            static const char kFrom[] = "\"\\/bfnrt";
            static const char kTo[] = "\"\\/\b\f\n\r\t";
            const char e = next();
            const char *hit = e != '\0' ? std::strchr(kFrom, e) : nullptr;
            if (hit == nullptr)
                bad("unsupported string escape");
            out += kTo[hit - kFrom];
        }
        bad("unterminated string");
    }

    Node list() {
        Node v;
        v.kind = Node::kList;
        at_++; /* '[' */
        skip_space();
        if (more() && peek() == ']') {
            at_++;
            return v;
        }
        for (;;) {
            v.list.push_back(value());
            skip_space();
            const char d = next();
            if (d == ']')
                return v;
            if (d != ',')
                bad("expected array delimiter");
        }
    }

    Node dict() {
        Node v;
        v.kind = Node::kDict;
        at_++; /* '{' */
        skip_space();
        if (more() && peek() == '}') {
            at_++;
            return v;
        }
        for (;;) {
            skip_space();
            if (!more() || peek() != '"')
                bad("expected object key");
            std::string key = string();
            skip_space();
            if (next() != ':')
                bad("expected colon");
            Node member = value();
            if (!v.dict.emplace(std::move(key), std::move(member)).second)
                bad("duplicate object key");
            skip_space();
            const char d = next();
            if (d == '}')
                return v;
            if (d != ',')
                bad("expected object delimiter");
        }
    }

    const char *p_;
    size_t n_;
    size_t at_ = 0;
};

const Node &field(const Node &obj, const char *name, Node::Kind kind) {
    if (obj.kind != Node::kDict)
        throw std::runtime_error("safetensors: expected object");
    auto it = obj.dict.find(name);
    if (it == obj.dict.end() || it->second.kind != kind)
        throw std::runtime_error(std::string("safetensors: missing or invalid ") + name);
    return it->second;
}

size_t as_size(uint64_t v, const char *label) {
    if (v > std::numeric_limits<size_t>::max())
        throw std::runtime_error(std::string("safetensors: ") + label +
                                 " exceeds address space");
    return size_t(v);
}

size_t count_of(const std::vector<size_t> &shape) {
    if (shape.empty())
        throw std::runtime_error("safetensors: scalar tensors unsupported");
    size_t n = 1;
    for (size_t d : shape) {
        if (d == 0 || n > std::numeric_limits<size_t>::max() / d)
            throw std::runtime_error("safetensors: invalid tensor shape");
        n *= d;
    }
    return n;
}

size_t decimal(const std::string &text, const std::string &name) {
    if (text.empty())
        throw std::runtime_error("model metadata: empty " + name);
    size_t v = 0;
    for (char c : text) {
        if (c < '0' || c > '9')
            throw std::runtime_error("model metadata: invalid " + name);
        const size_t d = size_t(c - '0');
        if (v > (std::numeric_limits<size_t>::max() - d) / 10)
            throw std::runtime_error("model metadata: overflow in " + name);
        v = v * 10 + d;
    }
    return v;
}

} // namespace

struct SafeTensorFile::Mapping {
    int fd = -1;
    void *base = MAP_FAILED;
    size_t size = 0;
    const unsigned char *bytes() const { return static_cast<const unsigned char *>(base); }
    ~Mapping() {
        if (base != MAP_FAILED)
            munmap(base, size);
        if (fd >= 0)
            close(fd);
    }
};

SafeTensorFile::SafeTensorFile() = default;
SafeTensorFile::~SafeTensorFile() = default;
SafeTensorFile::SafeTensorFile(SafeTensorFile &&) noexcept = default;
SafeTensorFile &SafeTensorFile::operator=(SafeTensorFile &&) noexcept = default;

SafeTensorFile SafeTensorFile::load(const std::string &path) {
    SafeTensorFile f;
    f.mapping_ = std::make_shared<Mapping>();
    Mapping &m = *f.mapping_;
    m.fd = open(path.c_str(), O_RDONLY);
    if (m.fd < 0)
        throw std::runtime_error("safetensors: cannot open " + path + ": " +
                                 std::strerror(errno));
    struct stat st {};
    if (fstat(m.fd, &st) != 0 || st.st_size < 0)
        throw std::runtime_error("safetensors: cannot stat " + path);
    m.size = size_t(st.st_size);
    if (m.size == 0)
        throw std::runtime_error("safetensors: empty file");
    m.base = mmap(nullptr, m.size, PROT_READ, MAP_PRIVATE, m.fd, 0);
    if (m.base == MAP_FAILED)
        throw std::runtime_error("safetensors: mmap failed");

    if (m.size < 8)
        throw std::runtime_error("safetensors: truncated length prefix");
    uint64_t header = 0;
    for (int b = 7; b >= 0; b--)
        header = (header << 8) | m.bytes()[b];
    const size_t hsize = as_size(header, "header");
    if (hsize == 0 || hsize > m.size - 8)
        throw std::runtime_error("safetensors: truncated header");
    f.payload_ = 8 + hsize;

    const Node root =
        HeaderParser(reinterpret_cast<const char *>(m.bytes() + 8), hsize).document();
    if (root.kind != Node::kDict)
        throw std::runtime_error("safetensors: root must be an object");
    for (const auto &kv : root.dict) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind != Node::kDict)
                throw std::runtime_error("safetensors: invalid metadata");
            for (const auto &md : kv.second.dict) {
                if (md.second.kind != Node::kText)
                    throw std::runtime_error("safetensors: metadata values must be strings");
                f.metadata_.emplace(md.first, md.second.text);
            }
            continue;
        }
        const Node &dtype = field(kv.second, "dtype", Node::kText);
        const Node &shape = field(kv.second, "shape", Node::kList);
        const Node &offsets = field(kv.second, "data_offsets", Node::kList);
        if (dtype.text != "F32")
            throw std::runtime_error("safetensors: only F32 is supported");
        Entry e;
        for (const Node &d : shape.list) {
            if (d.kind != Node::kInteger)
                throw std::runtime_error("safetensors: invalid shape");
            e.shape.push_back(as_size(d.integer, "shape dimension"));
        }
        if (offsets.list.size() != 2 || offsets.list[0].kind != Node::kInteger ||
            offsets.list[1].kind != Node::kInteger)
            throw std::runtime_error("safetensors: invalid data offsets");
        e.begin = as_size(offsets.list[0].integer, "data offset");
        e.end = as_size(offsets.list[1].integer, "data offset");
        const size_t n = count_of(e.shape);
        if (n > std::numeric_limits<size_t>::max() / sizeof(float) || e.begin > e.end ||
            e.end - e.begin != n * sizeof(float) || e.end > m.size - f.payload_ ||
            (f.payload_ + e.begin) % alignof(float) != 0)
            throw std::runtime_error("safetensors: invalid tensor extent");
        f.tensors_.emplace(kv.first, std::move(e));
    }
    if (f.tensors_.empty())
        throw std::runtime_error("safetensors: no tensors");
    return f;
}

TensorView SafeTensorFile::tensor(const std::string &name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end())
        throw std::runtime_error("model: missing tensor " + name);
    TensorView v;
    v.data = reinterpret_cast<const float *>(mapping_->bytes() + payload_ + it->second.begin);
    v.shape = it->second.shape;
    v.elements = count_of(v.shape);
    return v;
}

const std::string &SafeTensorFile::metadata(const std::string &name) const {
    auto it = metadata_.find(name);
    if (it == metadata_.end())
        throw std::runtime_error("model metadata: missing " + name);
    return it->second;
}

namespace {

void vector_from(const TensorView &t, std::vector<float> &dst, const std::string &name) {
    if (t.shape != std::vector<size_t>{dst.size()})
        throw std::runtime_error("model: wrong shape for " + name);
    std::memcpy(dst.data(), t.data, dst.size() * sizeof(float));
}

void matrix_from(const TensorView &t, Matrix &dst, const std::string &name) {
    if (t.shape != std::vector<size_t>{dst.rows(), dst.cols()})
        throw std::runtime_error("model: wrong shape for " + name);
    std::memcpy(dst.data(), t.data, dst.size() * sizeof(float));
}

/* [out][in] tensor into an [in][out] matrix */
void transposed_from(const TensorView &t, Matrix &dst, const std::string &name) {
    if (t.shape != std::vector<size_t>{dst.cols(), dst.rows()})
        throw std::runtime_error("model: wrong shape for " + name);
    const size_t out = t.shape[0], in = t.shape[1];
    for (size_t o = 0; o < out; o++)
        for (size_t i = 0; i < in; i++)
            dst.data()[i * out + o] = t.data[o * in + i];
}

} // namespace

ModelWeights load_model(const std::string &path) {
    const SafeTensorFile f = SafeTensorFile::load(path);
    ModelConfig c;
    size_t *fields[8] = {&c.layers,     &c.heads,   &c.dim,     &c.head_dim,
                         &c.ffn_dim,    &c.vocab_size, &c.max_seq, &c.eos_token};
    const char *keys[8] = {"layers",     "heads",   "dim",     "head_dim",
                           "ffn_dim",    "vocab_size", "max_seq", "eos_token"};
    for (int i = 0; i < 8; i++)
        *fields[i] = decimal(f.metadata(std::string("nutllm.") + keys[i]), keys[i]);
    c.validate();
    ModelWeights model(c);
    matrix_from(f.tensor("model.embed_tokens.weight"), model.embeddings,
                "model.embed_tokens.weight");
    for (size_t l = 0; l < c.layers; l++) {
        LayerWeights &w = model.layers[l];
        const std::string pre = "model.layers." + std::to_string(l);
        const std::pair<const char *, Matrix *> proj[7] = {
            {".self_attn.q_proj.weight", &w.query}, {".self_attn.k_proj.weight", &w.key},
            {".self_attn.v_proj.weight", &w.value}, {".self_attn.o_proj.weight", &w.output},
            {".mlp.gate_proj.weight", &w.gate},     {".mlp.up_proj.weight", &w.up},
            {".mlp.down_proj.weight", &w.down}};
        for (const auto &p : proj)
            transposed_from(f.tensor(pre + p.first), *p.second, pre + p.first);
        vector_from(f.tensor(pre + ".input_layernorm.weight"), w.attention_norm,
                    pre + ".input_layernorm.weight");
        vector_from(f.tensor(pre + ".post_attention_layernorm.weight"), w.ffn_norm,
                    pre + ".post_attention_layernorm.weight");
    }
    vector_from(f.tensor("model.norm.weight"), model.final_norm, "model.norm.weight");
    matrix_from(f.tensor("lm_head.weight"), model.lm_head, "lm_head.weight");
    return model;
}
