#pragma once
/* llama2.c checkpoint loader — host side of the drop-in for the reference's
 * load_llama2c_quantized_model (include/llama2.hpp:27-29,
 * src/llama2.cpp:199-298,339-412).
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

#include "quant.hpp"
#include "quant_model.hpp"

QuantizedModelWeights load_llama2c_quantized_model(const std::string &path, QuantType type);
