#pragma once
/* Byte-level BPE tokenizer — host side of the reference's Tokenizer
 * (include/tokenizer.hpp:9-24, src/tokenizer.cpp).
 *
 * Files: the vocabulary has one "id hex" line per token, ids contiguous
 * from 0; the merges file one "left-hex right-hex" pair per non-empty line,
 * in rank order.  Tokens are byte strings (hex-encoded, so any byte can
 * appear).  encode starts from one symbol per byte and, while some adjacent
 * pair is a merge, takes the lowest-ranked such pair and joins every
 * non-overlapping occurrence of it from left to right; each final symbol
 * must be a token.  decode concatenates the tokens' bytes.  Errors keep the
 * reference's classes and messages. */
#include <map>
#include <string>
#include <utility>
#include <vector>

class Tokenizer {
public:
    Tokenizer(std::vector<std::string> vocabulary,
              std::vector<std::pair<std::string, std::string>> merges);

    static Tokenizer load(const std::string &vocabulary_path, const std::string &merges_path);

    std::vector<int> encode(const std::string &text) const;
    std::string decode(const std::vector<int> &tokens) const;
    size_t vocabulary_size() const { return tokens_.size(); }

private:
    std::vector<std::string> tokens_;
    std::map<std::string, int> ids_;
    std::map<std::pair<std::string, std::string>, size_t> rank_;
};
