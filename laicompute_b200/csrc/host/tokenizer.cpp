// Gpt2Tokenizer (reference src/tokenizer.cpp:10-14), re-implemented.
//
// Behaviour kept from the reference: the vocabulary and merge ranks come from
// tokenizer.ggml.tokens / tokenizer.ggml.merges; "<|...|>" tokens are matched
// literally in the text; the text between them is byte-encoded with the GPT-2
// byte->code-point table and merged greedily by lowest merge rank (leftmost
// on equal ranks) without a pre-tokenisation regex; unknown symbols map to
// unk; decode() drops "<|...|>" tokens. Where several special tokens match at
// one position the longest one wins (the reference takes whichever its hash
// map visits first).
#include "laic/tokenizer.hpp"

#include <algorithm>
#include <array>
#include <stdexcept>

namespace laic {
namespace {

// GPT-2 bytes_to_unicode: printable bytes keep their value, the rest map to 256+k.
const std::array<uint32_t, 256>& byte_to_cp() {
    static const std::array<uint32_t, 256> table = [] {
        std::array<uint32_t, 256> t{};
        std::array<bool, 256> direct{};
        for (int b = 33; b <= 126; ++b) direct[b] = true;
        for (int b = 161; b <= 172; ++b) direct[b] = true;
        for (int b = 174; b <= 255; ++b) direct[b] = true;
        uint32_t extra = 0;
        for (int b = 0; b < 256; ++b) t[b] = direct[b] ? uint32_t(b) : 256 + extra++;
        return t;
    }();
    return table;
}

void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) s.push_back(char(cp));
    else if (cp < 0x800) { s.push_back(char(0xC0 | (cp >> 6))); s.push_back(char(0x80 | (cp & 63))); }
    else if (cp < 0x10000) {
        s.push_back(char(0xE0 | (cp >> 12))); s.push_back(char(0x80 | ((cp >> 6) & 63))); s.push_back(char(0x80 | (cp & 63)));
    } else {
        s.push_back(char(0xF0 | (cp >> 18))); s.push_back(char(0x80 | ((cp >> 12) & 63)));
        s.push_back(char(0x80 | ((cp >> 6) & 63))); s.push_back(char(0x80 | (cp & 63)));
    }
}

// Split into UTF-8 symbols (a truncated sequence at the end becomes one-byte symbols).
std::vector<std::string> symbols(const std::string& s) {
    std::vector<std::string> out;
    for (size_t i = 0; i < s.size();) {
        const unsigned char c = s[i];
        size_t n = c < 0x80 ? 1 : (c & 0xE0) == 0xC0 ? 2 : (c & 0xF0) == 0xE0 ? 3 : 4;
        if (i + n > s.size()) n = 1;
        out.push_back(s.substr(i, n));
        i += n;
    }
    return out;
}

bool is_special(const std::string& t) { return t.size() > 2 && t.compare(0, 2, "<|") == 0; }

}  // namespace

void Gpt2Tokenizer::load(const GgufModel& m) {
    tokens_ = m.strings("tokenizer.ggml.tokens");
    if (tokens_.empty()) throw std::runtime_error("GGUF has no tokenizer vocabulary");
    ids_.clear();
    specials_.clear();
    for (uint32_t i = 0; i < tokens_.size(); ++i) {
        ids_.emplace(tokens_[i], i);
        if (is_special(tokens_[i])) specials_.emplace_back(tokens_[i], i);
    }
    std::stable_sort(specials_.begin(), specials_.end(),
                     [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
    ranks_.clear();
    const auto& merges = m.strings("tokenizer.ggml.merges");
    for (uint32_t i = 0; i < merges.size(); ++i) ranks_[merges[i]] = i;
    bos_ = uint32_t(m.u64("tokenizer.ggml.bos_token_id", 0));
    eos_ = uint32_t(m.u64("tokenizer.ggml.eos_token_id", 0));
    unk_ = uint32_t(m.u64("tokenizer.ggml.unknown_token_id", 0));
    add_bos_ = m.u64("tokenizer.ggml.add_bos_token", 0) != 0;
    if (m.str("tokenizer.ggml.model", "") != "gpt2") throw std::runtime_error("M7 currently supports GPT-2 tokenizers only");
}

std::vector<uint32_t> Gpt2Tokenizer::encode(const std::string& text) const {
    std::vector<uint32_t> out;
    if (add_bos_) out.push_back(bos_);
    auto special_at = [&](size_t p) -> const std::pair<std::string, uint32_t>* {
        for (const auto& s : specials_)
            if (text.compare(p, s.first.size(), s.first) == 0) return &s;
        return nullptr;
    };
    const auto& b2c = byte_to_cp();
    size_t pos = 0;
    while (pos < text.size()) {
        if (const auto* s = special_at(pos)) {
            out.push_back(s->second);
            pos += s->first.size();
            continue;
        }
        size_t end = pos;
        while (end < text.size() && !special_at(end)) ++end;
        std::string piece;
        for (size_t i = pos; i < end; ++i) put_utf8(piece, b2c[(unsigned char)text[i]]);
        std::vector<std::string> syms = symbols(piece);
        while (syms.size() > 1) {
            uint32_t best = UINT32_MAX;
            size_t at = 0;
            for (size_t i = 0; i + 1 < syms.size(); ++i) {
                auto it = ranks_.find(syms[i] + " " + syms[i + 1]);
                if (it != ranks_.end() && it->second < best) { best = it->second; at = i; }
            }
            if (best == UINT32_MAX) break;
            syms[at] += syms[at + 1];
            syms.erase(syms.begin() + long(at) + 1);
        }
        for (const auto& s : syms) {
            auto it = ids_.find(s);
            out.push_back(it == ids_.end() ? unk_ : it->second);
        }
        pos = end;
    }
    return out;
}

std::string Gpt2Tokenizer::decode(uint32_t id) const {
    if (id >= tokens_.size()) return {};
    const std::string& t = tokens_[id];
    if (is_special(t)) return {};
    static const std::array<int, 512> c2b = [] {
        std::array<int, 512> r{};
        r.fill(-1);
        const auto& t = byte_to_cp();
        for (int b = 0; b < 256; ++b) r[t[b]] = b;
        return r;
    }();
    std::string out;
    for (const std::string& sym : symbols(t)) {
        const unsigned char c0 = sym[0];
        uint32_t cp = c0 < 0x80 ? c0 : (c0 & 0xE0) == 0xC0 ? (c0 & 31) : (c0 & 0xF0) == 0xE0 ? (c0 & 15) : (c0 & 7);
        for (size_t i = 1; i < sym.size(); ++i) cp = (cp << 6) | (uint32_t(sym[i]) & 63);
        if (cp < c2b.size() && c2b[cp] >= 0) out.push_back(char(c2b[cp]));
        else out += sym;
    }
    return out;
}

}  // namespace laic
