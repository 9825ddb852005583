/* Byte-level BPE tokenizer (src/tokenizer.cpp), this library's own code. */
#include "tokenizer.hpp"

#include <fstream>
#include <limits>
#include <stdexcept>

namespace {

std::string unhex(const std::string &s) {
    auto nibble = [](char c) {
        if (c >= '0' && c <= '9')
            return c - '0';
        if (c >= 'a' && c <= 'f')
            return c - 'a' + 10;
        if (c >= 'A' && c <= 'F')
            return c - 'A' + 10;
        return -1;
    };
    if (s.empty() || s.size() % 2 != 0)
        throw std::runtime_error("tokenizer: malformed hex token");
    std::string out(s.size() / 2, '\0');
    for (size_t i = 0; i < out.size(); i++) {
        const int hi = nibble(s[2 * i]), lo = nibble(s[2 * i + 1]);
        if (hi < 0 || lo < 0)
            throw std::runtime_error("tokenizer: malformed hex token");
        out[i] = char(hi * 16 + lo);
    }
    return out;
}

bool blank(char c) {
    return c == ' ' || c == '\t' || c == '\n' || c == '\v' || c == '\f' || c == '\r';
}

/* The next blank-delimited word of `line` from `at` (empty at the end). */
std::string word(const std::string &line, size_t &at) {
    while (at < line.size() && blank(line[at]))
        at++;
    const size_t from = at;
    while (at < line.size() && !blank(line[at]))
        at++;
    return line.substr(from, at - from);
}

/* A vocabulary line "id hex ...": the id as a formatted unsigned read takes
 * it (optional sign, then decimal digits; a minus sign wraps modulo 2^64,
 * overflow fails), then the next word is the token.  Lines are parsed here
 * rather than through stream extraction so that the result does not depend
 * on the process's locale state. */
bool vocab_line(const std::string &line, size_t &id, std::string &hex) {
    size_t at = 0;
    while (at < line.size() && blank(line[at]))
        at++;
    bool negative = false;
    if (at < line.size() && (line[at] == '+' || line[at] == '-'))
        negative = line[at++] == '-';
    const size_t digits = at;
    unsigned long long v = 0;
    bool overflow = false;
    while (at < line.size() && line[at] >= '0' && line[at] <= '9') {
        const unsigned d = unsigned(line[at++] - '0');
        if (v > (std::numeric_limits<unsigned long long>::max() - d) / 10)
            overflow = true;
        else
            v = v * 10 + d;
    }
    if (at == digits || overflow)
        return false;
    id = size_t(negative ? 0ull - v : v);
    hex = word(line, at);
    return !hex.empty();
}

} // namespace

Tokenizer::Tokenizer(std::vector<std::string> vocabulary,
                     std::vector<std::pair<std::string, std::string>> merges)
    : tokens_(std::move(vocabulary)) {
    if (tokens_.empty())
        throw std::invalid_argument("tokenizer: empty vocabulary");
    for (size_t id = 0; id < tokens_.size(); id++)
        if (id > size_t(std::numeric_limits<int>::max()) || tokens_[id].empty() ||
            !ids_.emplace(tokens_[id], int(id)).second)
            throw std::invalid_argument("tokenizer: empty or duplicate token");
    for (size_t r = 0; r < merges.size(); r++) {
        const auto &m = merges[r];
        if (m.first.empty() || m.second.empty() || !rank_.emplace(m, r).second)
            throw std::invalid_argument("tokenizer: invalid duplicate merge");
        if (ids_.count(m.first + m.second) == 0)
            throw std::invalid_argument("tokenizer: merged token missing from vocabulary");
    }
}

Tokenizer Tokenizer::load(const std::string &vocabulary_path, const std::string &merges_path) {
    std::ifstream vf(vocabulary_path);
    if (!vf)
        throw std::runtime_error("tokenizer: cannot open vocabulary");
    std::vector<std::string> vocab;
    std::string line;
    while (std::getline(vf, line)) {
        size_t id = 0;
        std::string hex;
        if (!vocab_line(line, id, hex) || id != vocab.size())
            throw std::runtime_error("tokenizer: vocabulary ids must be contiguous");
        vocab.push_back(unhex(hex));
    }
    if (!vf.eof())
        throw std::runtime_error("tokenizer: failed reading vocabulary");

    std::ifstream mf(merges_path);
    if (!mf)
        throw std::runtime_error("tokenizer: cannot open merges");
    std::vector<std::pair<std::string, std::string>> merges;
    while (std::getline(mf, line)) {
        if (line.empty())
            continue;
        size_t at = 0;
        const std::string a = word(line, at), b = word(line, at);
        if (a.empty() || b.empty() || !word(line, at).empty())
            throw std::runtime_error("tokenizer: malformed merge");
        merges.emplace_back(unhex(a), unhex(b));
    }
    if (!mf.eof())
        throw std::runtime_error("tokenizer: failed reading merges");
    return Tokenizer(std::move(vocab), std::move(merges));
}

std::vector<int> Tokenizer::encode(const std::string &text) const {
    std::vector<std::string> sym;
    sym.reserve(text.size());
    for (char c : text)
        sym.emplace_back(1, c);
    for (;;) {
        /* the lowest-ranked adjacent merge */
        const std::pair<std::string, std::string> *best = nullptr;
        size_t best_rank = std::numeric_limits<size_t>::max();
        for (size_t i = 0; i + 1 < sym.size(); i++) {
            auto it = rank_.find({sym[i], sym[i + 1]});
            if (it != rank_.end() && it->second < best_rank) {
                best_rank = it->second;
                best = &it->first;
            }
        }
        if (best == nullptr)
            break;
        /* join every non-overlapping occurrence, left to right */
        std::vector<std::string> out;
        out.reserve(sym.size());
        for (size_t i = 0; i < sym.size(); i++) {
            if (i + 1 < sym.size() && sym[i] == best->first && sym[i + 1] == best->second) {
                out.push_back(sym[i] + sym[i + 1]);
                i++;
            } else {
                out.push_back(std::move(sym[i]));
            }
        }
        sym = std::move(out);
    }
    std::vector<int> ids;
    ids.reserve(sym.size());
    for (const std::string &s : sym) {
        auto it = ids_.find(s);
        if (it == ids_.end())
            throw std::runtime_error("tokenizer: input byte absent from vocabulary");
        ids.push_back(it->second);
    }
    return ids;
}

std::string Tokenizer::decode(const std::vector<int> &tokens) const {
    std::string out;
    for (int t : tokens) {
        if (t < 0 || size_t(t) >= tokens_.size())
            throw std::out_of_range("tokenizer: token id out of range");
        out += tokens_[size_t(t)];
    }
    return out;
}
