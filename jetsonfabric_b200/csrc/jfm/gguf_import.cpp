// GGUF -> JFM v2 importer without GGML (host only).
//
// Replaces the reference's GGML-based compiler
// (runtime/compiler/jf_model_compile.cpp:547-645) with the same package
// contract (docs/jfm-v2-format.md):
//   - metadata.gguf is the exact source prefix [0, data offset);
//   - tensors go, in GGUF directory order, to layer-NNNNN.jfs ("blk.N."),
//     input.jfs ("token_embd."), output.jfs ("output." / "output_norm.") or
//     shared.jfs (anything else); every layer and the input must be
//     non-empty and output.weight must exist (tied embeddings are rejected,
//     jf_model_compile.cpp:382-410);
//   - segment files: 64-byte header, 80-byte index records with the name
//     padded to 8 bytes, payloads 64-byte aligned, file padded to 64 bytes
//     (jf_model_compile.cpp:420-505);
//   - the manifest records every segment's sizes and SHA-256 and the source
//     file's size and SHA-256 (jf_model_compile.cpp:585-608);
//   - the package is built in an exclusive staging directory next to the
//     output and published with one no-replace rename, so readers see either
//     no package or a complete one (jf_model_compile.cpp:113-151,
//     docs/native-engine.md:90-93); the source is locked shared and hashed
//     again at the end to catch concurrent modification
//     (jf_model_compile.cpp:917-921).
//
// The GGUF reader follows the published GGUF v2/v3 layout: magic "GGUF",
// version, tensor and key/value counts, typed key/values (arrays of scalars or
// strings), then the tensor directory (name, dimensions, GGML type id,
// offset) and the data section at the next `general.alignment` boundary
// (default 32). GGML type ids map to the stable JFM ids by the public
// ggml_type numbering; block geometry comes from the JFM table
// (jf_tensor_type_layout), which the reference also requires the pinned
// GGML to agree with (jf_model_compile.cpp:336-350).
#include "sha256_stream.h"

#include "jetsonfabric/engine.h"
#include "jfb/jfb_model.h"

#include <fcntl.h>
#include <sys/file.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <limits>
#include <optional>
#include <stdexcept>
#include <string>
#include <string_view>
#include <unordered_set>
#include <vector>

#ifndef RENAME_NOREPLACE
#define RENAME_NOREPLACE (1 << 0)
#endif

namespace {

namespace fs = std::filesystem;

struct ImportError : std::runtime_error {
    jfb_status_code code;
    ImportError(jfb_status_code c, const std::string & m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(jfb_status_code code, const char * fmt, ...) {
    char buf[512];
    va_list args;
    va_start(args, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, args);
    va_end(args);
    throw ImportError(code, buf);
}

std::uint64_t add_checked(std::uint64_t a, std::uint64_t b, const char * what) {
    if (a > std::numeric_limits<std::uint64_t>::max() - b) fail(JFB_STATUS_FORMAT_ERROR, "%s overflows uint64", what);
    return a + b;
}

std::uint64_t mul_checked(std::uint64_t a, std::uint64_t b, const char * what) {
    if (a != 0 && b > std::numeric_limits<std::uint64_t>::max() / a) {
        fail(JFB_STATUS_FORMAT_ERROR, "%s overflows uint64", what);
    }
    return a * b;
}

std::uint64_t align_up(std::uint64_t v, std::uint64_t a) {
    return add_checked(v, a - 1, "aligned size") / a * a;
}

// ---- source file ---------------------------------------------------------------

class Source {
public:
    explicit Source(const char * path) {
        fd_ = ::open(path, O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
        if (fd_ < 0) fail(JFB_STATUS_INVALID_ARGUMENT, "could not open input GGUF %s: %s", path, std::strerror(errno));
        struct stat st {};
        if (::fstat(fd_, &st) != 0 || !S_ISREG(st.st_mode) || st.st_size < 0) {
            ::close(fd_);
            fail(JFB_STATUS_INVALID_ARGUMENT, "input is not a regular GGUF file: %s", path);
        }
        if (::flock(fd_, LOCK_SH) != 0) {
            ::close(fd_);
            fail(JFB_STATUS_IO_ERROR, "could not lock input GGUF %s", path);
        }
        size_ = static_cast<std::uint64_t>(st.st_size);
    }
    ~Source() {
        (void) ::flock(fd_, LOCK_UN);
        ::close(fd_);
    }
    Source(const Source &) = delete;
    Source & operator=(const Source &) = delete;

    std::uint64_t size() const { return size_; }

    void read(std::uint64_t offset, void * dst, std::size_t n) const {
        auto * out = static_cast<std::uint8_t *>(dst);
        while (n > 0) {
            const ssize_t got = ::pread(fd_, out, n, static_cast<off_t>(offset));
            if (got < 0 && errno == EINTR) continue;
            if (got <= 0) fail(JFB_STATUS_FORMAT_ERROR, "GGUF is truncated at byte %llu", (unsigned long long) offset);
            out += got;
            offset += static_cast<std::uint64_t>(got);
            n -= static_cast<std::size_t>(got);
        }
    }

    // SHA-256 of the whole file.
    std::array<std::uint8_t, 32> digest() const {
        jfb_sha256_stream h;
        jfb_sha256_stream_begin(&h);
        std::vector<std::uint8_t> buf(8u << 20);
        for (std::uint64_t at = 0; at < size_;) {
            const std::size_t n = static_cast<std::size_t>(std::min<std::uint64_t>(buf.size(), size_ - at));
            read(at, buf.data(), n);
            jfb_sha256_stream_feed(&h, buf.data(), n);
            at += n;
        }
        std::array<std::uint8_t, 32> d{};
        jfb_sha256_stream_end(&h, d.data());
        return d;
    }

private:
    int fd_ = -1;
    std::uint64_t size_ = 0;
};

// Sequential little-endian reads from the source, buffered.
class Cursor {
public:
    explicit Cursor(const Source & src) : src_(src) {}
    std::uint64_t position() const { return pos_; }

    void bytes(void * dst, std::size_t n) {
        if (n > src_.size() || pos_ > src_.size() - n) {
            fail(JFB_STATUS_FORMAT_ERROR, "GGUF metadata runs past the end of the file (byte %llu)",
                 (unsigned long long) pos_);
        }
        auto * out = static_cast<std::uint8_t *>(dst);
        while (n > 0) {
            if (pos_ < buf_start_ || pos_ >= buf_start_ + buf_.size()) refill();
            const std::size_t off = static_cast<std::size_t>(pos_ - buf_start_);
            const std::size_t take = std::min(n, buf_.size() - off);
            std::memcpy(out, buf_.data() + off, take);
            out += take;
            pos_ += take;
            n -= take;
        }
    }
    template <class T>
    T scalar() {
        T v;
        std::uint8_t raw[sizeof(T)];
        bytes(raw, sizeof(T));
        std::memcpy(&v, raw, sizeof(T));  // little-endian host
        return v;
    }
    std::string string(const char * what) {
        const std::uint64_t n = scalar<std::uint64_t>();
        if (n > (1u << 30)) fail(JFB_STATUS_FORMAT_ERROR, "GGUF %s string length %llu is unsupported", what, (unsigned long long) n);
        std::string s(static_cast<std::size_t>(n), '\0');
        bytes(s.data(), s.size());
        return s;
    }
    void skip(std::uint64_t n) {
        if (n > src_.size() || pos_ > src_.size() - n) fail(JFB_STATUS_FORMAT_ERROR, "GGUF metadata runs past the end of the file");
        pos_ += n;
    }

private:
    void refill() {
        buf_start_ = pos_;
        const std::size_t n = static_cast<std::size_t>(std::min<std::uint64_t>(1u << 20, src_.size() - pos_));
        buf_.resize(n);
        src_.read(pos_, buf_.data(), n);
    }
    const Source & src_;
    std::uint64_t pos_ = 0, buf_start_ = 0;
    std::vector<std::uint8_t> buf_;
};

// ---- GGUF metadata -----------------------------------------------------------------

enum GgufType : std::uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

std::size_t scalar_size(std::uint32_t t) {
    switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
    }
}

// The key/values the importer needs, as read; every other value is skipped.
struct Value {
    std::uint32_t type = 0;
    std::int64_t integer = 0;   // integer types
    bool has_integer = false;
    std::string text;           // kString
};

struct Tensor {
    std::string name;
    std::uint32_t type = 0;  // JFM id
    std::uint32_t rank = 0;
    std::array<std::uint64_t, 4> shape{1, 1, 1, 1};
    std::int32_t layer = -1;
    std::uint64_t source_offset = 0, size = 0, package_offset = 0;
    std::uint32_t block_elements = 0, block_bytes = 0;
};

// Public ggml_type numbering -> stable JFM type (0 = unknown).
std::uint32_t jfm_type_of(std::uint32_t ggml_id) {
    switch (ggml_id) {
    case 0: return JF_TENSOR_F32;
    case 1: return JF_TENSOR_F16;
    case 2: return JF_TENSOR_Q4_0;
    case 3: return JF_TENSOR_Q4_1;
    case 6: return JF_TENSOR_Q5_0;
    case 7: return JF_TENSOR_Q5_1;
    case 8: return JF_TENSOR_Q8_0;
    case 9: return JF_TENSOR_Q8_1;
    case 10: return JF_TENSOR_Q2_K;
    case 11: return JF_TENSOR_Q3_K;
    case 12: return JF_TENSOR_Q4_K;
    case 13: return JF_TENSOR_Q5_K;
    case 14: return JF_TENSOR_Q6_K;
    case 15: return JF_TENSOR_Q8_K;
    case 16: return JF_TENSOR_IQ2_XXS;
    case 17: return JF_TENSOR_IQ2_XS;
    case 18: return JF_TENSOR_IQ3_XXS;
    case 19: return JF_TENSOR_IQ1_S;
    case 20: return JF_TENSOR_IQ4_NL;
    case 21: return JF_TENSOR_IQ3_S;
    case 22: return JF_TENSOR_IQ2_S;
    case 23: return JF_TENSOR_IQ4_XS;
    case 24: return JF_TENSOR_I8;
    case 25: return JF_TENSOR_I16;
    case 26: return JF_TENSOR_I32;
    case 27: return JF_TENSOR_I64;
    case 28: return JF_TENSOR_F64;
    case 29: return JF_TENSOR_IQ1_M;
    case 30: return JF_TENSOR_BF16;
    case 34: return JF_TENSOR_TQ1_0;
    case 35: return JF_TENSOR_TQ2_0;
    case 39: return JF_TENSOR_MXFP4;
    default: return 0;
    }
}

// "blk.<decimal>." -> layer index; other names -> none; malformed "blk." names fail.
std::optional<std::uint32_t> layer_of(std::string_view name) {
    constexpr std::string_view prefix = "blk.";
    if (name.substr(0, prefix.size()) != prefix) return std::nullopt;
    std::size_t i = prefix.size();
    if (i >= name.size() || name[i] < '0' || name[i] > '9') {
        fail(JFB_STATUS_FORMAT_ERROR, "invalid block tensor name: %.*s", int(name.size()), name.data());
    }
    std::uint64_t v = 0;
    for (; i < name.size() && name[i] >= '0' && name[i] <= '9'; ++i) {
        v = v * 10 + std::uint64_t(name[i] - '0');
        if (v > std::numeric_limits<std::uint32_t>::max()) {
            fail(JFB_STATUS_FORMAT_ERROR, "block index overflows in tensor %.*s", int(name.size()), name.data());
        }
    }
    if (i >= name.size() || name[i] != '.') {
        fail(JFB_STATUS_FORMAT_ERROR, "invalid block tensor name: %.*s", int(name.size()), name.data());
    }
    return std::uint32_t(v);
}

struct Gguf {
    std::vector<Value> wanted;              // parallel to the wanted keys
    std::vector<Tensor> tensors;
    std::uint64_t data_offset = 0;
};

Gguf read_gguf(const Source & src, const std::vector<std::string> & keys) {
    Cursor c(src);
    char magic[4];
    c.bytes(magic, 4);
    if (std::memcmp(magic, "GGUF", 4) != 0) fail(JFB_STATUS_FORMAT_ERROR, "input is not a GGUF file (bad magic)");
    const std::uint32_t version = c.scalar<std::uint32_t>();
    if (version != 2 && version != 3) fail(JFB_STATUS_FORMAT_ERROR, "GGUF version %u is not supported (2 or 3)", version);
    const std::uint64_t n_tensors = c.scalar<std::uint64_t>();
    const std::uint64_t n_kv = c.scalar<std::uint64_t>();
    if (n_tensors > (1u << 24) || n_kv > (1u << 24)) fail(JFB_STATUS_FORMAT_ERROR, "GGUF counts are implausible");

    Gguf g;
    g.wanted.resize(keys.size());
    std::uint64_t alignment = 32;
    std::unordered_set<std::string> seen_keys;
    for (std::uint64_t k = 0; k < n_kv; ++k) {
        const std::string key = c.string("key");
        if (!seen_keys.insert(key).second) fail(JFB_STATUS_FORMAT_ERROR, "duplicate GGUF key %s", key.c_str());
        const std::uint32_t type = c.scalar<std::uint32_t>();
        const auto slot = std::find(keys.begin(), keys.end(), key);
        Value * out = slot == keys.end() ? nullptr : &g.wanted[std::size_t(slot - keys.begin())];
        if (out != nullptr) out->type = type + 1;  // + 1: present
        if (type == kString) {
            std::string s = c.string("value");
            if (out != nullptr) out->text = std::move(s);
        } else if (type == kArray) {
            const std::uint32_t et = c.scalar<std::uint32_t>();
            const std::uint64_t count = c.scalar<std::uint64_t>();
            if (et == kString) {
                for (std::uint64_t e = 0; e < count; ++e) c.skip(c.scalar<std::uint64_t>());
            } else if (scalar_size(et) != 0) {
                c.skip(mul_checked(count, scalar_size(et), "GGUF array"));
            } else {
                fail(JFB_STATUS_FORMAT_ERROR, "GGUF key %s has an array of unsupported type %u", key.c_str(), et);
            }
        } else if (scalar_size(type) != 0) {
            std::uint8_t raw[8] = {};
            c.bytes(raw, scalar_size(type));
            std::int64_t iv = 0;
            bool is_int = true;
            switch (type) {
            case kU8: iv = raw[0]; break;
            case kI8: iv = std::int8_t(raw[0]); break;
            case kU16: { std::uint16_t v; std::memcpy(&v, raw, 2); iv = v; break; }
            case kI16: { std::int16_t v; std::memcpy(&v, raw, 2); iv = v; break; }
            case kU32: { std::uint32_t v; std::memcpy(&v, raw, 4); iv = v; break; }
            case kI32: { std::int32_t v; std::memcpy(&v, raw, 4); iv = v; break; }
            case kU64: {
                std::uint64_t v; std::memcpy(&v, raw, 8);
                iv = v > std::uint64_t(std::numeric_limits<std::int64_t>::max()) ? -1 : std::int64_t(v);
                break;
            }
            case kI64: { std::int64_t v; std::memcpy(&v, raw, 8); iv = v; break; }
            default: is_int = false; break;
            }
            if (out != nullptr && is_int) {
                out->integer = iv;
                out->has_integer = true;
            }
            if (key == "general.alignment") {
                if (type != kU32) fail(JFB_STATUS_FORMAT_ERROR, "general.alignment must be a uint32");
                if (iv <= 0 || (iv & (iv - 1)) != 0) fail(JFB_STATUS_FORMAT_ERROR, "general.alignment %lld is not a power of two", (long long) iv);
                alignment = std::uint64_t(iv);
            }
        } else {
            fail(JFB_STATUS_FORMAT_ERROR, "GGUF key %s has unsupported value type %u", key.c_str(), type);
        }
    }

    std::unordered_set<std::string> seen_tensors;
    g.tensors.reserve(std::size_t(n_tensors));
    for (std::uint64_t t = 0; t < n_tensors; ++t) {
        Tensor x;
        x.name = c.string("tensor name");
        if (x.name.empty() || x.name.size() > 1024) fail(JFB_STATUS_FORMAT_ERROR, "GGUF tensor name length is unsupported");
        if (!seen_tensors.insert(x.name).second) fail(JFB_STATUS_FORMAT_ERROR, "duplicate GGUF tensor %s", x.name.c_str());
        const std::uint32_t n_dims = c.scalar<std::uint32_t>();
        if (n_dims == 0 || n_dims > 4) fail(JFB_STATUS_FORMAT_ERROR, "tensor %s has %u dimensions", x.name.c_str(), n_dims);
        for (std::uint32_t d = 0; d < n_dims; ++d) {
            x.shape[d] = c.scalar<std::uint64_t>();
            if (x.shape[d] == 0 || x.shape[d] > std::uint64_t(std::numeric_limits<std::int64_t>::max())) {
                fail(JFB_STATUS_FORMAT_ERROR, "tensor has an invalid shape: %s", x.name.c_str());
            }
        }
        const std::uint32_t ggml_type = c.scalar<std::uint32_t>();
        x.type = jfm_type_of(ggml_type);
        if (x.type == 0) fail(JFB_STATUS_UNSUPPORTED, "tensor %s has GGML type id %u, unknown to this importer", x.name.c_str(), ggml_type);
        if (jf_tensor_type_layout(x.type, &x.block_elements, &x.block_bytes).code != JF_STATUS_OK) {
            fail(JFB_STATUS_UNSUPPORTED, "tensor %s has a type without JFM v2 geometry", x.name.c_str());
        }
        x.source_offset = c.scalar<std::uint64_t>();  // relative to the data section for now
        if (x.shape[0] % x.block_elements != 0) {
            fail(JFB_STATUS_FORMAT_ERROR, "tensor %s: dimension 0 (%llu) is not a multiple of its block (%u)",
                 x.name.c_str(), (unsigned long long) x.shape[0], x.block_elements);
        }
        std::uint64_t size = mul_checked(x.shape[0] / x.block_elements, x.block_bytes, "tensor size");
        for (int d = 1; d < 4; ++d) size = mul_checked(size, x.shape[d], "tensor size");
        x.size = size;
        // rank: the last dimension above one (trailing ones dropped)
        x.rank = 1;
        for (std::uint32_t d = 1; d < 4; ++d) if (x.shape[d] > 1) x.rank = d + 1;
        g.tensors.push_back(std::move(x));
    }
    g.data_offset = align_up(c.position(), alignment);
    if (g.data_offset > src.size()) fail(JFB_STATUS_FORMAT_ERROR, "GGUF metadata offset is outside the source file");
    for (Tensor & x : g.tensors) {
        if (x.source_offset % alignment != 0) fail(JFB_STATUS_FORMAT_ERROR, "tensor %s is not aligned to %llu", x.name.c_str(), (unsigned long long) alignment);
        x.source_offset = add_checked(g.data_offset, x.source_offset, "GGUF tensor offset");
        if (x.source_offset > src.size() || x.size > src.size() - x.source_offset) {
            fail(JFB_STATUS_FORMAT_ERROR, "tensor exceeds the source GGUF: %s", x.name.c_str());
        }
    }
    return g;
}

// ---- package --------------------------------------------------------------------------

enum : std::uint32_t { kShared = 0, kInput = 1, kLayer = 2, kOutput = 3, kMetadata = 4 };

struct Segment {
    std::uint32_t kind = kShared;
    std::int32_t layer = -1;
    std::string path;
    std::vector<Tensor> tensors;
    std::uint64_t tensor_bytes = 0, file_size = 0;
    std::array<std::uint8_t, 32> sha{};
};

Segment make_segment(std::uint32_t kind, std::int32_t layer, std::string path) {
    Segment s;
    s.kind = kind;
    s.layer = layer;
    s.path = std::move(path);
    return s;
}

struct Bytes {
    std::vector<std::uint8_t> data;
    void u32(std::uint32_t v) { for (int i = 0; i < 4; ++i) data.push_back(std::uint8_t(v >> (8 * i))); }
    void u64(std::uint64_t v) { for (int i = 0; i < 8; ++i) data.push_back(std::uint8_t(v >> (8 * i))); }
    void raw(const void * p, std::size_t n) {
        const auto * b = static_cast<const std::uint8_t *>(p);
        data.insert(data.end(), b, b + n);
    }
    void pad(std::size_t a) { while (data.size() % a != 0) data.push_back(0); }
};

std::vector<Segment> collect(std::vector<Tensor> tensors, std::uint32_t layers) {
    Segment shared = make_segment(kShared, -1, "shared.jfs");
    Segment input = make_segment(kInput, -1, "input.jfs");
    Segment output = make_segment(kOutput, -1, "output.jfs");
    std::vector<Segment> per_layer(layers);
    for (std::uint32_t l = 0; l < layers; ++l) {
        char path[32];
        std::snprintf(path, sizeof(path), "layer-%05u.jfs", l);
        per_layer[l] = make_segment(kLayer, std::int32_t(l), path);
    }
    bool has_output_weight = false;
    for (Tensor & t : tensors) {
        const std::string_view name = t.name;
        if (const auto l = layer_of(name)) {
            if (*l >= layers) fail(JFB_STATUS_FORMAT_ERROR, "tensor block exceeds model block count: %s", t.name.c_str());
            t.layer = std::int32_t(*l);
            per_layer[*l].tensors.push_back(std::move(t));
        } else if (name.substr(0, 11) == "token_embd.") {
            input.tensors.push_back(std::move(t));
        } else if (name.substr(0, 7) == "output." || name.substr(0, 12) == "output_norm.") {
            has_output_weight = has_output_weight || name == "output.weight";
            output.tensors.push_back(std::move(t));
        } else {
            shared.tensors.push_back(std::move(t));
        }
    }
    std::vector<Segment> out;
    out.push_back(make_segment(kMetadata, -1, "metadata.gguf"));
    if (!shared.tensors.empty()) out.push_back(std::move(shared));
    if (input.tensors.empty()) fail(JFB_STATUS_FORMAT_ERROR, "GGUF contains no input embedding tensors");
    out.push_back(std::move(input));
    for (Segment & s : per_layer) {
        if (s.tensors.empty()) fail(JFB_STATUS_FORMAT_ERROR, "GGUF contains no tensors for %s", s.path.c_str());
        out.push_back(std::move(s));
    }
    if (!has_output_weight) {
        fail(JFB_STATUS_UNSUPPORTED, "tied output embeddings are not supported by JFM v2; output.weight is required");
    }
    out.push_back(std::move(output));
    return out;
}

class Writer {
public:
    Writer(const fs::path & path) : path_(path) {
        fd_ = ::open(path.c_str(), O_WRONLY | O_CREAT | O_EXCL | O_CLOEXEC, 0644);
        if (fd_ < 0) fail(JFB_STATUS_IO_ERROR, "could not create %s: %s", path.c_str(), std::strerror(errno));
        jfb_sha256_stream_begin(&hash_);
    }
    ~Writer() {
        if (fd_ >= 0) ::close(fd_);
    }
    void write(const void * p, std::size_t n) {
        const auto * b = static_cast<const std::uint8_t *>(p);
        jfb_sha256_stream_feed(&hash_, b, n);
        size_ += n;
        while (n > 0) {
            const ssize_t w = ::write(fd_, b, n);
            if (w < 0 && errno == EINTR) continue;
            if (w <= 0) fail(JFB_STATUS_IO_ERROR, "could not write %s: %s", path_.c_str(), std::strerror(errno));
            b += w;
            n -= std::size_t(w);
        }
    }
    void zeros(std::uint64_t n) {
        static const std::uint8_t z[4096] = {};
        while (n > 0) {
            const std::size_t k = std::size_t(std::min<std::uint64_t>(n, sizeof(z)));
            write(z, k);
            n -= k;
        }
    }
    void copy(const Source & src, std::uint64_t offset, std::uint64_t n, std::vector<std::uint8_t> & buf) {
        while (n > 0) {
            const std::size_t k = std::size_t(std::min<std::uint64_t>(n, buf.size()));
            src.read(offset, buf.data(), k);
            write(buf.data(), k);
            offset += k;
            n -= k;
        }
    }
    std::uint64_t size() const { return size_; }
    std::array<std::uint8_t, 32> finish() {
        if (::fsync(fd_) != 0) fail(JFB_STATUS_IO_ERROR, "could not sync %s: %s", path_.c_str(), std::strerror(errno));
        if (::close(fd_) != 0) {
            fd_ = -1;
            fail(JFB_STATUS_IO_ERROR, "could not finish %s", path_.c_str());
        }
        fd_ = -1;
        std::array<std::uint8_t, 32> d{};
        jfb_sha256_stream_end(&hash_, d.data());
        return d;
    }

private:
    fs::path path_;
    int fd_ = -1;
    std::uint64_t size_ = 0;
    jfb_sha256_stream hash_{};
};

constexpr std::uint64_t kAlign = 64;

void write_tensor_segment(const Source & src, const fs::path & dir, Segment & s, std::vector<std::uint8_t> & buf) {
    std::uint64_t index_bytes = 0;
    for (const Tensor & t : s.tensors) index_bytes = add_checked(index_bytes, align_up(80 + t.name.size(), 8), "segment index");
    std::uint64_t cursor = align_up(add_checked(64, index_bytes, "segment header"), kAlign);
    s.tensor_bytes = 0;
    for (Tensor & t : s.tensors) {
        t.package_offset = cursor;
        cursor = align_up(add_checked(cursor, t.size, "segment payload"), kAlign);
        s.tensor_bytes = add_checked(s.tensor_bytes, t.size, "segment tensor bytes");
    }
    Bytes head;
    head.raw("JFSEGM02", 8);
    head.u32(2);
    head.u32(std::uint32_t(s.tensors.size()));
    head.u64(index_bytes);
    head.u64(s.tensor_bytes);
    head.data.resize(64, 0);
    for (const Tensor & t : s.tensors) {
        head.u32(t.type);
        head.u32(t.rank);
        head.u32(std::uint32_t(t.layer));
        head.u32(0);
        for (std::uint64_t d : t.shape) head.u64(d);
        head.u64(t.package_offset);
        head.u64(t.size);
        head.u32(std::uint32_t(t.name.size()));
        head.u32(t.block_elements);
        head.u32(t.block_bytes);
        head.u32(0);
        head.raw(t.name.data(), t.name.size());
        head.pad(8);
    }
    if (head.data.size() != 64 + index_bytes) fail(JFB_STATUS_EXECUTION_FAILED, "internal segment index size mismatch");
    head.pad(kAlign);
    Writer w(dir / s.path);
    w.write(head.data.data(), head.data.size());
    for (const Tensor & t : s.tensors) {
        w.zeros(t.package_offset - w.size());
        w.copy(src, t.source_offset, t.size, buf);
    }
    w.zeros(cursor - w.size());
    s.file_size = w.size();
    s.sha = w.finish();
}

void sync_dir(const fs::path & dir) {
    const int fd = ::open(dir.c_str(), O_RDONLY | O_DIRECTORY | O_CLOEXEC);
    if (fd < 0 || ::fsync(fd) != 0) {
        const int e = errno;
        if (fd >= 0) ::close(fd);
        fail(JFB_STATUS_IO_ERROR, "could not sync directory %s: %s", dir.c_str(), std::strerror(e));
    }
    ::close(fd);
}

// The exclusive staging directory; removed unless published.
class Staging {
public:
    explicit Staging(const fs::path & out) : out_(out) {
        fs::path parent = out.parent_path();
        if (parent.empty()) parent = ".";
        std::error_code ec;
        if (!fs::is_directory(parent, ec)) fail(JFB_STATUS_INVALID_ARGUMENT, "output parent is not a directory: %s", parent.c_str());
        dir_ = parent / (out.filename().string() + ".tmp." + std::to_string(::getpid()));
        if (::mkdir(dir_.c_str(), 0755) != 0) {
            fail(JFB_STATUS_IO_ERROR, "could not create exclusive staging directory %s: %s", dir_.c_str(), std::strerror(errno));
        }
        parent_ = parent;
    }
    ~Staging() {
        if (!published_) {
            std::error_code ec;
            fs::remove_all(dir_, ec);
        }
    }
    const fs::path & path() const { return dir_; }
    void publish() {
        if (::syscall(SYS_renameat2, AT_FDCWD, dir_.c_str(), AT_FDCWD, out_.c_str(), RENAME_NOREPLACE) != 0) {
            const int e = errno;
            fail(e == EEXIST ? JFB_STATUS_INVALID_ARGUMENT : JFB_STATUS_IO_ERROR,
                 "atomic no-replace publication of %s failed: %s", out_.c_str(), std::strerror(e));
        }
        published_ = true;
        sync_dir(parent_);
    }

private:
    fs::path out_, dir_, parent_;
    bool published_ = false;
};

jfb_status ok_status() {
    jfb_status s{};
    s.code = JFB_STATUS_OK;
    return s;
}

jfb_status error_status(jfb_status_code code, const char * message) {
    jfb_status s{};
    s.code = code;
    std::snprintf(s.message, sizeof(s.message), "%s", message);
    return s;
}

void import(const char * gguf_path, const char * package_dir, jfb_import_report * report) {
    const fs::path out(package_dir);
    std::error_code ec;
    if (fs::exists(fs::symlink_status(out, ec))) fail(JFB_STATUS_INVALID_ARGUMENT, "output already exists: %s", package_dir);
    Source src(gguf_path);
    const std::vector<std::string> keys = {"general.architecture", "split.count"};
    Gguf g = read_gguf(src, keys);
    if (g.wanted[1].type != 0 && (!g.wanted[1].has_integer || g.wanted[1].integer < 0)) {
        fail(JFB_STATUS_FORMAT_ERROR, "GGUF metadata split.count is not a non-negative integer");
    }
    if (g.wanted[1].type != 0 && g.wanted[1].integer > 1) {
        fail(JFB_STATUS_UNSUPPORTED, "split GGUF inputs are not supported; merge the shards first");
    }
    if (g.wanted[0].type != kString + 1) fail(JFB_STATUS_FORMAT_ERROR, "GGUF metadata is missing string general.architecture");
    const std::string arch = g.wanted[0].text;
    // the block count key depends on the architecture: read the metadata again for it
    const std::vector<std::string> arch_keys = {arch + ".block_count"};
    const Gguf ga = read_gguf(src, arch_keys);
    const Value & bc = ga.wanted[0];
    if (bc.type == 0) fail(JFB_STATUS_FORMAT_ERROR, "GGUF metadata is missing %s.block_count", arch.c_str());
    if (!bc.has_integer || bc.integer < 0) fail(JFB_STATUS_FORMAT_ERROR, "GGUF metadata %s.block_count is not a non-negative integer", arch.c_str());
    if (bc.integer == 0 || bc.integer > 4096) fail(JFB_STATUS_FORMAT_ERROR, "GGUF block count is invalid");
    const std::uint32_t layers = std::uint32_t(bc.integer);

    const std::array<std::uint8_t, 32> source_sha = src.digest();
    std::vector<Segment> segments = collect(std::move(g.tensors), layers);

    Staging staging(out);
    std::vector<std::uint8_t> buf(8u << 20);
    {
        Segment & meta = segments.front();
        Writer w(staging.path() / meta.path);
        w.copy(src, 0, g.data_offset, buf);
        meta.file_size = w.size();
        meta.sha = w.finish();
    }
    for (std::size_t i = 1; i < segments.size(); ++i) write_tensor_segment(src, staging.path(), segments[i], buf);
    if (src.digest() != source_sha) fail(JFB_STATUS_IO_ERROR, "input GGUF changed while the package was being written");

    Bytes m;
    m.raw("JFMODEL2", 8);
    m.u32(2);
    m.u32(layers);
    m.u64(src.size());
    m.raw(source_sha.data(), 32);
    m.u32(std::uint32_t(segments.size()));
    m.u32(0);
    std::uint64_t tensor_count = 0, tensor_bytes = 0, package_bytes = 0;
    for (const Segment & s : segments) {
        m.u32(s.kind);
        m.u32(std::uint32_t(s.layer));
        m.u64(s.tensors.size());
        m.u64(s.tensor_bytes);
        m.u64(s.file_size);
        m.raw(s.sha.data(), 32);
        m.u32(std::uint32_t(s.path.size()));
        m.u32(0);
        m.raw(s.path.data(), s.path.size());
        tensor_count += s.tensors.size();
        tensor_bytes += s.tensor_bytes;
        package_bytes += s.file_size;
    }
    {
        Writer w(staging.path() / "manifest.jfm");
        w.write(m.data.data(), m.data.size());
        package_bytes += w.size();
        (void) w.finish();
    }
    sync_dir(staging.path());
    staging.publish();
    if (report != nullptr) {
        std::memset(report, 0, sizeof(*report));
        report->layer_count = layers;
        report->tensor_count = tensor_count;
        report->tensor_bytes = tensor_bytes;
        report->package_bytes = package_bytes;
        std::memcpy(report->source_sha256, source_sha.data(), 32);
        std::snprintf(report->architecture, sizeof(report->architecture), "%s", arch.c_str());
    }
}

}  // namespace

extern "C" jfb_status jfb_import_gguf(const char * gguf_path, const char * package_dir, jfb_import_report * report) {
    if (gguf_path == nullptr || package_dir == nullptr || package_dir[0] == '\0') {
        return error_status(JFB_STATUS_INVALID_ARGUMENT, "input GGUF and output package paths are required");
    }
    try {
        import(gguf_path, package_dir, report);
        return ok_status();
    } catch (const ImportError & e) {
        return error_status(e.code, e.what());
    } catch (const std::bad_alloc &) {
        return error_status(JFB_STATUS_OUT_OF_MEMORY, "out of memory while importing GGUF");
    } catch (const std::exception & e) {
        return error_status(JFB_STATUS_IO_ERROR, e.what());
    }
}
