#pragma once
/* llama2.c checkpoint loaders — host side of the drop-in for the reference's
 * load_llama2c_model and load_llama2c_quantized_model (include/llama2.hpp:
 * 27-29, src/llama2.cpp:199-412).
 *
 * File format (llama2.c "legacy" export): seven int32 — dim, ffn_dim,
 * layers, heads, kv_heads, vocab (negative: separate classifier follows),
 * max_seq — then fp32 tensors in this order: embeddings [vocab][dim],
 * attention norms [layers][dim], wq [layers][dim][dim], wk and wv
 * [layers][kv_dim][dim], wo [layers][dim][dim], ffn norms [layers][dim],
 * w1 (gate) [layers][ffn][dim], w2 (down) [layers][dim][ffn], w3 (up)
 * [layers][ffn][dim], final norm [dim], RoPE tables [max_seq][head_dim]
 * (skipped), and the classifier [vocab][dim] when vocab < 0.  Projections
 * are [out][in] as stored; eos is token 1.  Each projection is quantised
 * per block of 32 on the host exactly as QuantizedMatrix::quantize does. */
#include <string>
#include <unordered_map>
#include <vector>

#include "loader.hpp"
#include "quant.hpp"
#include "quant_model.hpp"

QuantizedModelWeights load_llama2c_quantized_model(const std::string &path, QuantType type);
/* The fp32 loader (src/llama2.cpp:300-337): the same file into ModelWeights,
 * projections transposed to the reference's [in][out] storage. */
ModelWeights load_llama2c_model(const std::string &path);

/* The llama2.c tokenizer (include/llama2.hpp:11-25, src/llama2.cpp:414-543),
 * host text I/O around the token loop.
 *
 * File: uint32 maximum token length, then per id a float score, an int32
 * byte length and the bytes.  encode: BOS (1) if asked, the " " token when
 * the text is non-empty, one token per UTF-8 character (or, for a character
 * with no token, one byte-fallback id byte + 3 per byte), then repeatedly
 * the adjacent pair whose concatenation is a token with the highest score
 * (the first such pair on ties) is merged, then EOS (2) if asked.  decode:
 * skips a leading BOS, drops one leading space of the piece after a BOS,
 * and turns "<0xHH>" pieces into that byte.  Errors keep the reference's
 * classes and messages. */
class Llama2Tokenizer {
public:
    static Llama2Tokenizer load(const std::string &path, size_t vocab_size);

    std::vector<int> encode(const std::string &text, bool bos = true, bool eos = false) const;
    std::string decode(const std::vector<int> &tokens) const;
    size_t vocabulary_size() const { return pieces_.size(); }

private:
    int find(const std::string &piece) const;

    std::vector<std::string> pieces_;
    std::vector<float> scores_;
    std::unordered_map<std::string, int> ids_; /* first id of each piece */
    size_t max_length_ = 0;
};
