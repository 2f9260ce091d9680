// GGUF v2/v3 key/value reader for the metadata segment of a JFM package
// (metadata.gguf holds the source file's bytes [0, data_offset): header,
// key/values and tensor directory). Only the key/values are decoded; the
// engine takes tensor shapes from the JFM records.
//
// Replaces the reference's use of GGML's gguf parser
// (runtime/engines/native/src/qwen2_metadata.cpp). Layout per the GGUF
// specification: "GGUF", u32 version, u64 tensor count, u64 kv count, then
// kv records (u64-length string key, u32 type, value).
#pragma once

#include <cstdint>
#include <cstring>
#include <map>
#include <span>
#include <stdexcept>
#include <string>
#include <variant>
#include <vector>

namespace jfb::engine {

enum class GgufType : std::uint32_t {
    U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STRING = 8, ARRAY = 9,
    U64 = 10, I64 = 11, F64 = 12,
};

struct GgufValue {
    GgufType type = GgufType::U8;
    std::uint64_t u = 0;   // unsigned / bool payload; element count of an array
    std::int64_t i = 0;    // signed payload
    double f = 0.0;        // float payload
    std::string s;         // string payload
    // arrays, kept only when the reader is asked to: string elements, or
    // integer and bool elements (as int64)
    GgufType element = GgufType::U8;
    std::vector<std::string> strings;
    std::vector<std::int64_t> integers;
};

class GgufMetadata {
public:
    explicit GgufMetadata(std::span<const std::byte> blob, bool keep_arrays = false)
        : data_(blob), keep_arrays_(keep_arrays) {
        if (blob.size() < 24 || std::memcmp(blob.data(), "GGUF", 4) != 0) {
            throw std::runtime_error("JFM metadata is not a GGUF header");
        }
        pos_ = 4;
        const std::uint32_t version = read<std::uint32_t>();
        if (version < 2 || version > 3) throw std::runtime_error("unsupported GGUF version " + std::to_string(version));
        (void) read<std::uint64_t>();  // tensor count
        const std::uint64_t kv_count = read<std::uint64_t>();
        if (kv_count > 1000000) throw std::runtime_error("GGUF key/value count is implausible");
        for (std::uint64_t n = 0; n < kv_count; ++n) {
            std::string key = read_string();
            const auto type = static_cast<GgufType>(read<std::uint32_t>());
            GgufValue value = read_value(type);
            values_.emplace(std::move(key), std::move(value));
        }
    }

    const GgufValue * find(const std::string & key) const {
        const auto it = values_.find(key);
        return it == values_.end() ? nullptr : &it->second;
    }

private:
    template <typename T>
    T read() {
        if (pos_ + sizeof(T) > data_.size()) throw std::runtime_error("GGUF metadata is truncated");
        T v;
        std::memcpy(&v, data_.data() + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }

    std::string read_string() {
        const std::uint64_t n = read<std::uint64_t>();
        if (n > data_.size() - pos_) throw std::runtime_error("GGUF string is truncated");
        std::string s(reinterpret_cast<const char *>(data_.data() + pos_), n);
        pos_ += n;
        return s;
    }

    GgufValue read_value(GgufType type) {
        GgufValue v;
        v.type = type;
        switch (type) {
        case GgufType::U8: v.u = read<std::uint8_t>(); break;
        case GgufType::I8: v.i = read<std::int8_t>(); break;
        case GgufType::U16: v.u = read<std::uint16_t>(); break;
        case GgufType::I16: v.i = read<std::int16_t>(); break;
        case GgufType::U32: v.u = read<std::uint32_t>(); break;
        case GgufType::I32: v.i = read<std::int32_t>(); break;
        case GgufType::F32: v.f = read<float>(); break;
        case GgufType::BOOL: v.u = read<std::uint8_t>(); break;
        case GgufType::STRING: v.s = read_string(); break;
        case GgufType::U64: v.u = read<std::uint64_t>(); break;
        case GgufType::I64: v.i = read<std::int64_t>(); break;
        case GgufType::F64: v.f = read<double>(); break;
        case GgufType::ARRAY: {
            const auto element = static_cast<GgufType>(read<std::uint32_t>());
            const std::uint64_t count = read<std::uint64_t>();
            if (element == GgufType::ARRAY) throw std::runtime_error("nested GGUF arrays are not supported");
            if (count > data_.size()) throw std::runtime_error("GGUF array is truncated");
            v.element = element;
            for (std::uint64_t k = 0; k < count; ++k) {
                GgufValue e = read_value(element);
                if (!keep_arrays_) continue;
                if (element == GgufType::STRING) v.strings.push_back(std::move(e.s));
                else if (element == GgufType::F32 || element == GgufType::F64) v.integers.push_back(std::int64_t(e.f));
                else v.integers.push_back(e.type == GgufType::I8 || e.type == GgufType::I16 || e.type == GgufType::I32 ||
                                                  e.type == GgufType::I64
                                              ? e.i
                                              : std::int64_t(e.u));
            }
            v.u = count;
            break;
        }
        default: throw std::runtime_error("unknown GGUF value type");
        }
        return v;
    }

    std::span<const std::byte> data_;
    bool keep_arrays_ = false;
    std::size_t pos_ = 0;
    std::map<std::string, GgufValue> values_;
};

}  // namespace jfb::engine
