// Text tokenizer of a JFM package, behind the reference's tokenizer interface
// (runtime/tokenization/tokenizer.hpp:9-16, kept with the same namespace,
// names and meaning).
//
// The reference loads llama.cpp's vocabulary from the package's metadata.gguf
// (runtime/adapters/llama_cpp_tokenizer.cpp:44-81) and calls
// tokenize(text, add_special = true, parse_special = true), token_to_piece(
// token, lstrip 0, special = true) and is_eog (:86-126). open_package_tokenizer
// reads the same GGUF keys (tokenizer.ggml.model, .pre, .tokens, .token_type,
// .merges, special token ids, add_bos/add_eos flags) and implements the
// byte-level BPE those models use ("gpt2" vocabularies with the "qwen2" or
// "llama-bpe" pre-tokenizer), without llama.cpp.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

namespace jetsonfabric::runtime::tokenization {

class Tokenizer {
public:
    virtual ~Tokenizer() = default;

    virtual std::vector<std::int32_t> tokenize(std::string_view text) const = 0;
    virtual std::string token_piece(std::int32_t token) const = 0;
    virtual bool is_end_token(std::int32_t token) const = 0;
};

}  // namespace jetsonfabric::runtime::tokenization

namespace jetsonfabric::native {

// The tokenizer of the package at `package_path` (its metadata.gguf).
// Throws std::invalid_argument when the metadata is missing or malformed, or
// describes a vocabulary this implementation does not support; tokenize()
// throws std::invalid_argument when the text produces no tokens, as the
// reference adapter does (llama_cpp_tokenizer.cpp:91-93).
std::unique_ptr<runtime::tokenization::Tokenizer> open_package_tokenizer(const std::string & package_path);

// The same from the bytes of a metadata.gguf.
std::unique_ptr<runtime::tokenization::Tokenizer> open_gguf_tokenizer(const void * metadata, std::size_t size);

}  // namespace jetsonfabric::native
