// Byte-level BPE tokenizer of a JFM package (host only), behind the
// reference's tokenizer interface (runtime/tokenization/tokenizer.hpp:9-16).
//
// The reference tokenizes with llama.cpp's vocabulary loaded from the
// package's metadata.gguf (runtime/adapters/llama_cpp_tokenizer.cpp:44-126):
// tokenize(text, add_special = true, parse_special = true),
// token_to_piece(token, lstrip 0, special = true), is_eog. This file restates
// the published algorithm those Qwen2-family ("gpt2" model, "qwen2" or
// "llama-bpe" pre-tokenizer) vocabularies use:
//   1. special tokens (control and user-defined entries of
//      tokenizer.ggml.token_type) are cut out of the text first, longest
//      first;
//   2. each remaining fragment is split by the pre-tokenizer pattern
//        (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,D}|
//         ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
//      (D = 1 for qwen2, 3 for llama-bpe), evaluated here as a hand-written
//      scanner over code points with the alternatives tried in order;
//   3. each piece's UTF-8 bytes become the GPT-2 byte-to-unicode characters
//      and are merged by tokenizer.ggml.merges rank, lowest first;
//   4. BOS / EOS are added when tokenizer.ggml.add_bos_token /
//      add_eos_token say so.
// End-of-generation tokens are the EOS, EOT and EOM ids and the vocabulary
// entries named like the end-of-turn tokens of the common chat templates.
#include "jetsonfabric/tokenizer.hpp"
#include "jfb/jfb_tokenizer.h"

#include "engine/gguf_meta.hpp"

#include <algorithm>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

struct CodeRange {
    std::uint32_t lo, hi;
};

#include "unicode_ranges.inc"

template <std::size_t N>
bool in_ranges(const CodeRange (&r)[N], std::uint32_t cp) {
    std::size_t lo = 0, hi = N;
    while (lo < hi) {
        const std::size_t mid = (lo + hi) / 2;
        if (cp < r[mid].lo) hi = mid;
        else if (cp > r[mid].hi) lo = mid + 1;
        else return true;
    }
    return false;
}

bool is_letter(std::uint32_t cp) { return cp < 0x110000 && in_ranges(kLetters, cp); }
bool is_number(std::uint32_t cp) { return cp < 0x110000 && in_ranges(kNumbers, cp); }
bool is_space(std::uint32_t cp) { return cp < 0x110000 && in_ranges(kWhiteSpace, cp); }
bool is_newline(std::uint32_t cp) { return cp == '\r' || cp == '\n'; }

struct CodePoint {
    std::uint32_t cp;  // 0x110000 + byte for a byte that starts no valid UTF-8 sequence
    std::uint32_t begin, end;
};

std::vector<CodePoint> decode_utf8(std::string_view s) {
    std::vector<CodePoint> out;
    out.reserve(s.size());
    const auto * b = reinterpret_cast<const unsigned char *>(s.data());
    const std::size_t n = s.size();
    std::size_t i = 0;
    auto cont = [&](std::size_t k) { return k < n && (b[k] & 0xC0) == 0x80; };
    while (i < n) {
        std::uint32_t cp = 0x110000u + b[i];
        std::size_t len = 1;
        if (b[i] < 0x80) {
            cp = b[i];
        } else if ((b[i] & 0xE0) == 0xC0 && cont(i + 1)) {
            const std::uint32_t v = (std::uint32_t(b[i] & 0x1F) << 6) | (b[i + 1] & 0x3F);
            if (v >= 0x80) cp = v, len = 2;
        } else if ((b[i] & 0xF0) == 0xE0 && cont(i + 1) && cont(i + 2)) {
            const std::uint32_t v = (std::uint32_t(b[i] & 0x0F) << 12) | (std::uint32_t(b[i + 1] & 0x3F) << 6) | (b[i + 2] & 0x3F);
            if (v >= 0x800 && (v < 0xD800 || v > 0xDFFF)) cp = v, len = 3;
        } else if ((b[i] & 0xF8) == 0xF0 && cont(i + 1) && cont(i + 2) && cont(i + 3)) {
            const std::uint32_t v = (std::uint32_t(b[i] & 0x07) << 18) | (std::uint32_t(b[i + 1] & 0x3F) << 12) |
                                    (std::uint32_t(b[i + 2] & 0x3F) << 6) | (b[i + 3] & 0x3F);
            if (v >= 0x10000 && v <= 0x10FFFF) cp = v, len = 4;
        }
        out.push_back({cp, std::uint32_t(i), std::uint32_t(i + len)});
        i += len;
    }
    return out;
}

void append_utf8(std::string & out, std::uint32_t cp) {
    if (cp < 0x80) {
        out.push_back(char(cp));
    } else if (cp < 0x800) {
        out.push_back(char(0xC0 | (cp >> 6)));
        out.push_back(char(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
        out.push_back(char(0xE0 | (cp >> 12)));
        out.push_back(char(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(char(0x80 | (cp & 0x3F)));
    } else {
        out.push_back(char(0xF0 | (cp >> 18)));
        out.push_back(char(0x80 | ((cp >> 12) & 0x3F)));
        out.push_back(char(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(char(0x80 | (cp & 0x3F)));
    }
}

// GPT-2's byte-to-unicode table: the printable bytes '!'..'~', 0xA1..0xAC
// and 0xAE..0xFF stand for themselves; the other 68 bytes, in increasing
// order, become U+0100, U+0101, ...
std::uint32_t byte_char(std::uint8_t b) {
    static const std::vector<std::uint32_t> table = [] {
        std::vector<std::uint32_t> t(256);
        std::uint32_t next = 256;
        for (int v = 0; v < 256; ++v) {
            const bool keep = (v >= '!' && v <= '~') || (v >= 0xA1 && v <= 0xAC) || (v >= 0xAE && v <= 0xFF);
            t[std::size_t(v)] = keep ? std::uint32_t(v) : next++;
        }
        return t;
    }();
    return table[b];
}

// Pieces [begin, end) (code point indices) of the pre-tokenizer pattern.
std::vector<std::pair<std::size_t, std::size_t>> pre_tokenize(const std::vector<CodePoint> & c, std::size_t digits) {
    std::vector<std::pair<std::size_t, std::size_t>> out;
    const std::size_t n = c.size();
    auto cp = [&](std::size_t k) { return c[k].cp; };
    auto lower = [](std::uint32_t v) { return v >= 'A' && v <= 'Z' ? v + 32 : v; };
    std::size_t i = 0;
    while (i < n) {
        // (?i:'s|'t|'re|'ve|'m|'ll|'d)
        if (cp(i) == '\'' && i + 1 < n) {
            const std::uint32_t a = lower(cp(i + 1));
            if (a == 's' || a == 't' || a == 'm' || a == 'd') {
                out.emplace_back(i, i + 2);
                i += 2;
                continue;
            }
            if (i + 2 < n) {
                const std::uint32_t b = lower(cp(i + 2));
                if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) {
                    out.emplace_back(i, i + 3);
                    i += 3;
                    continue;
                }
            }
        }
        // [^\r\n\p{L}\p{N}]?\p{L}+
        {
            std::size_t j = i;
            if (!is_newline(cp(j)) && !is_letter(cp(j)) && !is_number(cp(j)) && j + 1 < n && is_letter(cp(j + 1))) ++j;
            if (is_letter(cp(j))) {
                std::size_t k = j;
                while (k < n && is_letter(cp(k))) ++k;
                out.emplace_back(i, k);
                i = k;
                continue;
            }
        }
        // \p{N}{1,digits}
        if (is_number(cp(i))) {
            std::size_t k = i;
            while (k < n && k - i < digits && is_number(cp(k))) ++k;
            out.emplace_back(i, k);
            i = k;
            continue;
        }
        // ' '?[^\s\p{L}\p{N}]+[\r\n]*
        {
            const std::size_t j = i + (cp(i) == ' ' ? 1 : 0);
            auto other = [&](std::size_t k) { return !is_space(cp(k)) && !is_letter(cp(k)) && !is_number(cp(k)); };
            if (j < n && other(j)) {
                std::size_t k = j;
                while (k < n && other(k)) ++k;
                while (k < n && is_newline(cp(k))) ++k;
                out.emplace_back(i, k);
                i = k;
                continue;
            }
        }
        // \s*[\r\n]+ | \s+(?!\S) | \s+
        if (is_space(cp(i))) {
            std::size_t k = i, last_newline = n;
            while (k < n && is_space(cp(k))) {
                if (is_newline(cp(k))) last_newline = k;
                ++k;
            }
            std::size_t end;
            if (last_newline != n) end = last_newline + 1;  // up to the last line break of the run
            else if (k == n || k - i == 1) end = k;          // at the end, or a single blank before text
            else end = k - 1;                                // leave one blank to the following word
            out.emplace_back(i, end);
            i = end;
            continue;
        }
        out.emplace_back(i, i + 1);
        ++i;
    }
    return out;
}

enum TokenType : std::int64_t { kNormal = 1, kUnknown = 2, kControl = 3, kUserDefined = 4, kUnused = 5, kByte = 6 };

class BpeTokenizer final : public jetsonfabric::runtime::tokenization::Tokenizer {
public:
    explicit BpeTokenizer(const jfb::engine::GgufMetadata & meta) {
        const auto * model = meta.find("tokenizer.ggml.model");
        if (model == nullptr || model->type != jfb::engine::GgufType::STRING) {
            throw std::invalid_argument("package metadata has no tokenizer.ggml.model");
        }
        if (model->s != "gpt2") {
            throw std::invalid_argument("tokenizer model '" + model->s + "' is not supported (byte-level BPE 'gpt2' only)");
        }
        const auto * pre = meta.find("tokenizer.ggml.pre");
        const std::string pre_name = pre != nullptr && pre->type == jfb::engine::GgufType::STRING ? pre->s : "default";
        if (pre_name == "qwen2") digits_ = 1;
        else if (pre_name == "llama-bpe" || pre_name == "llama3") digits_ = 3;
        else throw std::invalid_argument("pre-tokenizer '" + pre_name + "' is not supported (qwen2, llama-bpe)");

        const auto * tokens = meta.find("tokenizer.ggml.tokens");
        if (tokens == nullptr || tokens->type != jfb::engine::GgufType::ARRAY ||
            tokens->element != jfb::engine::GgufType::STRING || tokens->strings.empty()) {
            throw std::invalid_argument("package metadata has no tokenizer.ggml.tokens");
        }
        text_ = tokens->strings;
        if (text_.size() > std::size_t(INT32_MAX)) throw std::invalid_argument("vocabulary is too large");
        type_.assign(text_.size(), kNormal);
        if (const auto * types = meta.find("tokenizer.ggml.token_type")) {
            if (types->integers.size() != text_.size()) throw std::invalid_argument("tokenizer.ggml.token_type does not match the vocabulary");
            type_ = types->integers;
        }
        id_.reserve(text_.size());
        for (std::size_t t = 0; t < text_.size(); ++t) id_.emplace(text_[t], std::int32_t(t));

        for (int b = 0; b < 256; ++b) {
            std::string s;
            append_utf8(s, byte_char(std::uint8_t(b)));
            const auto it = id_.find(s);
            if (it == id_.end()) throw std::invalid_argument("vocabulary lacks the byte-level token of byte " + std::to_string(b));
            byte_token_[b] = it->second;
        }
        const auto * merges = meta.find("tokenizer.ggml.merges");
        if (merges == nullptr || merges->element != jfb::engine::GgufType::STRING) {
            throw std::invalid_argument("package metadata has no tokenizer.ggml.merges");
        }
        merge_.reserve(merges->strings.size());
        for (std::size_t r = 0; r < merges->strings.size(); ++r) {
            const std::string & m = merges->strings[r];
            const std::size_t sp = m.find(' ', 1);
            if (sp == std::string::npos) throw std::invalid_argument("malformed merge '" + m + "'");
            const std::string left = m.substr(0, sp), right = m.substr(sp + 1);
            const auto l = id_.find(left), rr = id_.find(right), lr = id_.find(left + right);
            if (l == id_.end() || rr == id_.end() || lr == id_.end()) continue;  // not reachable in this vocabulary
            merge_.emplace(key(l->second, rr->second), std::make_pair(std::int32_t(r), lr->second));
        }

        auto id_key = [&](const char * k) -> std::int32_t {
            const auto * v = meta.find(k);
            if (v == nullptr) return -1;
            const std::int64_t x = v->type == jfb::engine::GgufType::I32 || v->type == jfb::engine::GgufType::I64 ? v->i : std::int64_t(v->u);
            return x >= 0 && x < std::int64_t(text_.size()) ? std::int32_t(x) : -1;
        };
        auto flag = [&](const char * k) {
            const auto * v = meta.find(k);
            return v != nullptr && v->type == jfb::engine::GgufType::BOOL && v->u != 0;
        };
        bos_ = id_key("tokenizer.ggml.bos_token_id");
        eos_ = id_key("tokenizer.ggml.eos_token_id");
        add_bos_ = flag("tokenizer.ggml.add_bos_token") && bos_ >= 0;
        add_eos_ = flag("tokenizer.ggml.add_eos_token") && eos_ >= 0;
        for (const char * k : {"tokenizer.ggml.eos_token_id", "tokenizer.ggml.eot_token_id", "tokenizer.ggml.eom_token_id"}) {
            const std::int32_t t = id_key(k);
            if (t >= 0) end_.insert(t);
        }
        static const char * const kEndTexts[] = {"<|endoftext|>", "<|im_end|>", "<|eot_id|>", "<|eom_id|>", "<|end|>",
                                                 "<end_of_turn>", "<|end_of_text|>", "<EOT>"};
        for (const char * e : kEndTexts) {
            const auto it = id_.find(e);
            if (it != id_.end()) end_.insert(it->second);
        }
        for (std::size_t t = 0; t < text_.size(); ++t) {
            if ((type_[t] == kControl || type_[t] == kUserDefined) && !text_[t].empty()) special_.push_back(std::int32_t(t));
        }
        std::stable_sort(special_.begin(), special_.end(),
                         [&](std::int32_t a, std::int32_t b) { return text_[std::size_t(a)].size() > text_[std::size_t(b)].size(); });
    }

    std::vector<std::int32_t> tokenize(std::string_view text) const override {
        // fragments: special token ids, or raw text
        struct Fragment {
            std::int32_t special;  // -1 for text
            std::size_t begin, end;
        };
        std::vector<Fragment> frags{{-1, 0, text.size()}};
        for (const std::int32_t s : special_) {
            const std::string & st = text_[std::size_t(s)];
            std::vector<Fragment> next;
            for (const Fragment & f : frags) {
                if (f.special >= 0) {
                    next.push_back(f);
                    continue;
                }
                std::size_t at = f.begin;
                while (at < f.end) {
                    const std::size_t hit = text.substr(0, f.end).find(st, at);
                    if (hit == std::string_view::npos) break;
                    if (hit > at) next.push_back({-1, at, hit});
                    next.push_back({s, hit, hit + st.size()});
                    at = hit + st.size();
                }
                if (at < f.end) next.push_back({-1, at, f.end});
            }
            frags.swap(next);
        }
        std::vector<std::int32_t> out;
        if (add_bos_) out.push_back(bos_);
        for (const Fragment & f : frags) {
            if (f.special >= 0) {
                out.push_back(f.special);
                continue;
            }
            const std::string_view part = text.substr(f.begin, f.end - f.begin);
            const std::vector<CodePoint> cps = decode_utf8(part);
            for (const auto & [b, e] : pre_tokenize(cps, digits_)) encode_piece(part.substr(cps[b].begin, cps[e - 1].end - cps[b].begin), out);
        }
        if (add_eos_) out.push_back(eos_);
        if (out.empty()) throw std::invalid_argument("native prompt tokenization produced no tokens");
        return out;
    }

    std::string token_piece(std::int32_t token) const override {
        if (token < 0 || std::size_t(token) >= text_.size()) throw std::invalid_argument("token id " + std::to_string(token) + " is outside the vocabulary");
        const std::string & t = text_[std::size_t(token)];
        switch (type_[std::size_t(token)]) {
        case kNormal: {
            // byte-level characters back to bytes
            std::string out;
            for (const CodePoint & c : decode_utf8(t)) {
                const int b = byte_of(c.cp);
                if (b >= 0) out.push_back(char(b));
                else out.append(t, c.begin, c.end - c.begin);
            }
            return out;
        }
        case kByte: {
            unsigned v = 0;
            if (t.size() == 6 && std::sscanf(t.c_str(), "<0x%02X>", &v) == 1) return std::string(1, char(v));
            return t;
        }
        case kUnused: return {};
        default: return t;  // control (special = true), user-defined, unknown: their text
        }
    }

    bool is_end_token(std::int32_t token) const override { return token == -1 || end_.count(token) != 0; }

private:
    static std::uint64_t key(std::int32_t a, std::int32_t b) { return (std::uint64_t(std::uint32_t(a)) << 32) | std::uint32_t(b); }

    static int byte_of(std::uint32_t cp) {
        static const std::unordered_map<std::uint32_t, int> inverse = [] {
            std::unordered_map<std::uint32_t, int> m;
            for (int b = 0; b < 256; ++b) m.emplace(byte_char(std::uint8_t(b)), b);
            return m;
        }();
        const auto it = inverse.find(cp);
        return it == inverse.end() ? -1 : it->second;
    }

    // Byte-level BPE of one pre-tokenizer piece: the lowest-rank adjacent pair
    // is merged wherever it occurs (left to right), until no pair merges. A
    // merge creates only pairs of higher rank than its own, so this equals
    // merging one lowest-rank occurrence at a time.
    void encode_piece(std::string_view bytes, std::vector<std::int32_t> & out) const {
        std::vector<std::int32_t> sym;
        sym.reserve(bytes.size());
        for (const char ch : bytes) sym.push_back(byte_token_[std::uint8_t(ch)]);
        std::vector<std::int32_t> next;
        while (sym.size() > 1) {
            std::int32_t best = INT32_MAX, merged = -1;
            std::uint64_t best_key = 0;
            for (std::size_t i = 0; i + 1 < sym.size(); ++i) {
                const auto it = merge_.find(key(sym[i], sym[i + 1]));
                if (it != merge_.end() && it->second.first < best) {
                    best = it->second.first;
                    merged = it->second.second;
                    best_key = it->first;
                }
            }
            if (merged < 0) break;
            next.clear();
            for (std::size_t i = 0; i < sym.size();) {
                if (i + 1 < sym.size() && key(sym[i], sym[i + 1]) == best_key) {
                    next.push_back(merged);
                    i += 2;
                } else {
                    next.push_back(sym[i]);
                    ++i;
                }
            }
            sym.swap(next);
        }
        out.insert(out.end(), sym.begin(), sym.end());
    }

    std::vector<std::string> text_;
    std::vector<std::int64_t> type_;
    std::unordered_map<std::string, std::int32_t> id_;
    std::unordered_map<std::uint64_t, std::pair<std::int32_t, std::int32_t>> merge_;  // pair -> (rank, merged id)
    std::int32_t byte_token_[256] = {};
    std::vector<std::int32_t> special_;  // control and user-defined tokens, longest first
    std::unordered_set<std::int32_t> end_;
    std::int32_t bos_ = -1, eos_ = -1;
    bool add_bos_ = false, add_eos_ = false;
    std::size_t digits_ = 1;
};

}  // namespace

namespace jetsonfabric::native {

std::unique_ptr<runtime::tokenization::Tokenizer> open_gguf_tokenizer(const void * metadata, std::size_t size) {
    if (metadata == nullptr || size == 0) throw std::invalid_argument("native model metadata is empty");
    try {
        const jfb::engine::GgufMetadata meta(std::span<const std::byte>(static_cast<const std::byte *>(metadata), size), true);
        return std::make_unique<BpeTokenizer>(meta);
    } catch (const std::invalid_argument &) {
        throw;
    } catch (const std::exception & e) {
        throw std::invalid_argument(std::string("native model metadata is not valid GGUF: ") + e.what());
    }
}

std::unique_ptr<runtime::tokenization::Tokenizer> open_package_tokenizer(const std::string & package_path) {
    std::ifstream in(package_path + "/metadata.gguf", std::ios::binary);
    if (!in) throw std::invalid_argument("native model package is missing metadata.gguf");
    const std::vector<char> bytes{std::istreambuf_iterator<char>(in), std::istreambuf_iterator<char>()};
    return open_gguf_tokenizer(bytes.data(), bytes.size());
}

}  // namespace jetsonfabric::native

// ---- C ABI -----------------------------------------------------------------------

struct jfb_tokenizer {
    std::unique_ptr<jetsonfabric::runtime::tokenization::Tokenizer> impl;
};

namespace {

jfb_status tok_status(jfb_status_code code, const char * message) {
    jfb_status s{};
    s.code = code;
    if (message != nullptr) std::snprintf(s.message, sizeof(s.message), "%s", message);
    return s;
}

template <class F>
jfb_status guarded(F && f) {
    try {
        f();
        return tok_status(JFB_STATUS_OK, nullptr);
    } catch (const std::invalid_argument & e) {
        return tok_status(JFB_STATUS_INVALID_ARGUMENT, e.what());
    } catch (const std::bad_alloc &) {
        return tok_status(JFB_STATUS_OUT_OF_MEMORY, "out of memory");
    } catch (const std::exception & e) {
        return tok_status(JFB_STATUS_EXECUTION_FAILED, e.what());
    }
}

}  // namespace

extern "C" jfb_status jfb_tokenizer_open(const char * package_dir, jfb_tokenizer ** out) {
    if (package_dir == nullptr || out == nullptr) return tok_status(JFB_STATUS_INVALID_ARGUMENT, "package directory and handle are required");
    *out = nullptr;
    return guarded([&] {
        auto t = std::make_unique<jfb_tokenizer>();
        t->impl = jetsonfabric::native::open_package_tokenizer(package_dir);
        *out = t.release();
    });
}

extern "C" void jfb_tokenizer_close(jfb_tokenizer * tokenizer) { delete tokenizer; }

extern "C" jfb_status jfb_tokenizer_tokenize(const jfb_tokenizer * tokenizer, const char * text, size_t length,
                                             int32_t * tokens, size_t capacity, size_t * count) {
    if (tokenizer == nullptr || (text == nullptr && length > 0) || count == nullptr || (tokens == nullptr && capacity > 0)) {
        return tok_status(JFB_STATUS_INVALID_ARGUMENT, "tokenizer, text and count are required");
    }
    return guarded([&] {
        const std::vector<std::int32_t> ids = tokenizer->impl->tokenize(std::string_view(text == nullptr ? "" : text, length));
        *count = ids.size();
        std::copy_n(ids.begin(), std::min(ids.size(), capacity), tokens);
    });
}

extern "C" jfb_status jfb_tokenizer_token_piece(const jfb_tokenizer * tokenizer, int32_t token, char * piece,
                                                size_t capacity, size_t * length) {
    if (tokenizer == nullptr || length == nullptr || (piece == nullptr && capacity > 0)) {
        return tok_status(JFB_STATUS_INVALID_ARGUMENT, "tokenizer and length are required");
    }
    return guarded([&] {
        const std::string p = tokenizer->impl->token_piece(token);
        *length = p.size();
        if (capacity > 0) std::memcpy(piece, p.data(), std::min(p.size(), capacity));
    });
}

extern "C" int jfb_tokenizer_is_end_token(const jfb_tokenizer * tokenizer, int32_t token) {
    return tokenizer != nullptr && tokenizer->impl->is_end_token(token) ? 1 : 0;
}
