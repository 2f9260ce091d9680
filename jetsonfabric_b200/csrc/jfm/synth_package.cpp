// Seeded synthetic Qwen2 JFM v2 package writer (host only).
//
// Writes the package topology the reference loader and engine expect
// (docs/jfm-v2-format.md; tensor names and shapes from
// runtime/engines/native/src/qwen2_architecture.cpp:80-118):
//   metadata.gguf   GGUF v3 header, key/values and tensor directory (no data)
//   input.jfs       token_embd.weight                     [h, V]
//   layer-NNNNN.jfs blk.i.{attn_norm, attn_q(+bias), attn_k(+bias),
//                   attn_v(+bias), attn_output, ffn_norm, ffn_gate, ffn_up,
//                   ffn_down}
//   output.jfs      output_norm.weight [h], output.weight [h, V]
// "Tied" configurations still get a materialised output.weight, because the
// engine requires one (qwen2_architecture.cpp:96-98).
//
// Weights are N(0, std) from a counter-based generator (SplitMix64 + Box-Muller),
// so every element depends only on (seed, tensor name, index) and the output
// is identical for any thread count.
#include "half.hpp"
#include "kquant_encode.hpp"

#include "jetsonfabric/engine.h"
#include "jfb/jfb_model.h"

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <functional>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

namespace fs = std::filesystem;

struct WriterError : std::runtime_error {
    jfb_status_code code;
    WriterError(jfb_status_code c, const std::string & m) : std::runtime_error(m), code(c) {}
};

// ---- little-endian byte building -------------------------------------------

struct Bytes {
    std::vector<std::uint8_t> data;
    void u8(std::uint8_t v) { data.push_back(v); }
    void u32(std::uint32_t v) { for (int i = 0; i < 4; ++i) data.push_back(static_cast<std::uint8_t>(v >> (8 * i))); }
    void i32(std::int32_t v) { u32(static_cast<std::uint32_t>(v)); }
    void u64(std::uint64_t v) { for (int i = 0; i < 8; ++i) data.push_back(static_cast<std::uint8_t>(v >> (8 * i))); }
    void f32(float v) { u32(jfb::float_bits(v)); }
    void raw(const void * p, std::size_t n) {
        const auto * b = static_cast<const std::uint8_t *>(p);
        data.insert(data.end(), b, b + n);
    }
    void pad(std::size_t alignment) { while (data.size() % alignment != 0) data.push_back(0); }
    void gguf_string(const std::string & s) { u64(s.size()); raw(s.data(), s.size()); }
};

// ---- tensor plan ------------------------------------------------------------

struct TensorPlan {
    std::string name;
    std::uint32_t type = JF_TENSOR_F32;   // JFM id
    std::uint64_t cols = 1;               // shape[0] (input dimension)
    std::uint64_t rows = 1;               // shape[1]
    std::uint32_t rank = 1;
    int32_t layer = -1;
    enum Fill { Normal, NormWeight, Bias, Constant, RowScaled } fill = Normal;
    float constant = 0.0f;                // Constant value, or RowScaled scale
};

std::uint32_t ggml_type_id(std::uint32_t jfm_type) {
    switch (jfm_type) {
    case JF_TENSOR_F32: return 0;
    case JF_TENSOR_F16: return 1;
    case JF_TENSOR_Q2_K: return 10;
    case JF_TENSOR_Q4_K: return 12;
    case JF_TENSOR_Q6_K: return 14;
    default: throw WriterError(JFB_STATUS_UNSUPPORTED, "synthetic writer cannot emit JFM type " + std::to_string(jfm_type));
    }
}

std::uint64_t payload_bytes(const TensorPlan & t) {
    std::uint32_t be = 0, bb = 0;
    const jf_status s = jf_tensor_type_layout(t.type, &be, &bb);
    if (s.code != JF_STATUS_OK || t.cols % be != 0) {
        throw WriterError(JFB_STATUS_INVALID_ARGUMENT, "tensor " + t.name + " does not fit its storage blocks");
    }
    return t.cols / be * bb * t.rows;
}

// ---- random numbers ---------------------------------------------------------

std::uint64_t splitmix64(std::uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

std::uint64_t name_hash(const std::string & name, std::uint64_t seed) {
    std::uint64_t h = 0xcbf29ce484222325ull ^ seed;  // FNV-1a, seeded
    for (unsigned char c : name) h = (h ^ c) * 0x100000001b3ull;
    return splitmix64(h);
}

// Two standard normals per counter value (Box-Muller), element i uses pair i/2.
inline void normal_pair(std::uint64_t stream, std::uint64_t even_index, float * z0, float * z1) {
    const std::uint64_t bits = splitmix64(stream + (even_index >> 1) * 0xd1b54a32d192ed03ull);
    const double u1 = (static_cast<double>(bits >> 32) + 0.5) * (1.0 / 4294967296.0);
    const double u2 = static_cast<double>(bits & 0xffffffffull) * (1.0 / 4294967296.0);
    const double radius = std::sqrt(-2.0 * std::log(u1));
    const double angle = 6.283185307179586476925286766559 * u2;
    *z0 = static_cast<float>(radius * std::cos(angle));
    *z1 = static_cast<float>(radius * std::sin(angle));
}

inline float normal_at(std::uint64_t stream, std::uint64_t index) {
    float z0, z1;
    normal_pair(stream, index & ~1ull, &z0, &z1);
    return (index & 1) ? z1 : z0;
}

void fill_row(const TensorPlan & t, const jfb_synth_spec & spec, std::uint64_t row, float * out) {
    const std::uint64_t stream = name_hash(t.name, spec.seed);
    const std::uint64_t base = row * t.cols;
    for (std::uint64_t c = 0; c < t.cols; ++c) {
        switch (t.fill) {
        case TensorPlan::Normal:
            if (((base + c) & 1) == 0 && c + 1 < t.cols) {
                float z0, z1;
                normal_pair(stream, base + c, &z0, &z1);
                out[c] = spec.weight_std * z0;
                out[c + 1] = spec.weight_std * z1;
                ++c;
            } else {
                out[c] = spec.weight_std * normal_at(stream, base + c);
            }
            break;
        case TensorPlan::NormWeight:
            out[c] = spec.draw_norms ? 1.0f + spec.weight_std * normal_at(stream, base + c) : 1.0f;
            break;
        case TensorPlan::Bias:
            out[c] = spec.draw_biases ? spec.weight_std * normal_at(stream, base + c) : 0.0f;
            break;
        case TensorPlan::Constant: out[c] = t.constant; break;
        case TensorPlan::RowScaled: out[c] = t.constant * static_cast<float>(row + 1); break;
        }
    }
}

void encode_row(std::uint32_t type, const float * values, std::uint64_t count, std::uint8_t * out) {
    switch (type) {
    case JF_TENSOR_F32: std::memcpy(out, values, count * 4); break;
    case JF_TENSOR_F16:
        for (std::uint64_t i = 0; i < count; ++i) {
            const std::uint16_t h = jfb::float_to_half_rne(values[i]);
            std::memcpy(out + 2 * i, &h, 2);
        }
        break;
    case JF_TENSOR_Q4_K:
        for (std::uint64_t b = 0; b < count / 256; ++b) jfb::kquant::encode_q4_k(values + 256 * b, out + 144 * b);
        break;
    case JF_TENSOR_Q6_K:
        for (std::uint64_t b = 0; b < count / 256; ++b) jfb::kquant::encode_q6_k(values + 256 * b, out + 210 * b);
        break;
    case JF_TENSOR_Q2_K:
        for (std::uint64_t b = 0; b < count / 256; ++b) jfb::kquant::encode_q2_k(values + 256 * b, out + 84 * b);
        break;
    default: throw WriterError(JFB_STATUS_UNSUPPORTED, "unsupported tensor type");
    }
}

void parallel_for(std::uint64_t count, unsigned threads, const std::function<void(std::uint64_t, std::uint64_t)> & body,
                  std::uint64_t fixed_chunk = 0) {
    threads = static_cast<unsigned>(std::max<std::uint64_t>(1, std::min<std::uint64_t>(threads, count)));
    if (threads == 1) {
        body(0, count);
        return;
    }
    std::vector<std::thread> pool;
    std::atomic<std::uint64_t> next{0};
    const std::uint64_t chunk = fixed_chunk != 0 ? fixed_chunk : std::max<std::uint64_t>(1, count / (threads * 8));
    std::exception_ptr failure;
    std::atomic<bool> failed{false};
    for (unsigned t = 0; t < threads; ++t) {
        pool.emplace_back([&] {
            for (;;) {
                const std::uint64_t begin = next.fetch_add(chunk);
                if (begin >= count || failed.load()) return;
                try {
                    body(begin, std::min(count, begin + chunk));
                } catch (...) {
                    if (!failed.exchange(true)) failure = std::current_exception();
                    return;
                }
            }
        });
    }
    for (auto & th : pool) th.join();
    if (failure) std::rethrow_exception(failure);
}

std::vector<std::uint8_t> materialise(const TensorPlan & t, const jfb_synth_spec & spec, unsigned threads) {
    std::vector<std::uint8_t> bytes(payload_bytes(t));
    const std::uint64_t row_bytes = bytes.size() / t.rows;
    parallel_for(t.rows, threads, [&](std::uint64_t begin, std::uint64_t end) {
        std::vector<float> row(t.cols);
        for (std::uint64_t r = begin; r < end; ++r) {
            fill_row(t, spec, r, row.data());
            encode_row(t.type, row.data(), t.cols, bytes.data() + r * row_bytes);
        }
    });
    return bytes;
}

// ---- package assembly -------------------------------------------------------

struct SegmentRecord {
    std::uint32_t kind;
    std::int32_t layer;
    std::uint64_t tensor_count = 0;
    std::uint64_t payload = 0;
    std::uint64_t file_size = 0;
    std::uint8_t digest[32] = {};
    std::string path;
};

void write_file(const fs::path & path, const std::vector<std::uint8_t> & bytes) {
    std::ofstream out(path, std::ios::binary | std::ios::trunc);
    if (!out) throw WriterError(JFB_STATUS_IO_ERROR, "could not create " + path.string());
    out.write(reinterpret_cast<const char *>(bytes.data()), static_cast<std::streamsize>(bytes.size()));
    if (!out) throw WriterError(JFB_STATUS_IO_ERROR, "could not write " + path.string());
}

SegmentRecord write_tensor_segment(const fs::path & dir, std::uint32_t kind, std::int32_t layer,
                                   const std::string & path, const std::vector<TensorPlan> & tensors,
                                   const jfb_synth_spec & spec, unsigned threads) {
    Bytes index;
    std::vector<std::uint64_t> sizes;
    std::uint64_t index_bytes = 0;
    for (const TensorPlan & t : tensors) {
        sizes.push_back(payload_bytes(t));
        index_bytes += (80 + t.name.size() + 7) / 8 * 8;
    }
    const std::uint64_t data_start = (64 + index_bytes + 63) / 64 * 64;
    std::uint64_t cursor = data_start;
    std::vector<std::uint64_t> offsets;
    for (std::size_t i = 0; i < tensors.size(); ++i) {
        offsets.push_back(cursor);
        cursor = (cursor + sizes[i] + 63) / 64 * 64;
    }
    const std::uint64_t file_size = cursor;
    std::uint64_t payload_total = 0;
    for (std::uint64_t s : sizes) payload_total += s;

    std::vector<std::uint8_t> file(file_size, 0);
    Bytes header;
    header.raw("JFSEGM02", 8);
    header.u32(2);
    header.u32(static_cast<std::uint32_t>(tensors.size()));
    header.u64(index_bytes);
    header.u64(payload_total);
    header.data.resize(64, 0);
    for (std::size_t i = 0; i < tensors.size(); ++i) {
        const TensorPlan & t = tensors[i];
        std::uint32_t be = 0, bb = 0;
        (void) jf_tensor_type_layout(t.type, &be, &bb);
        header.u32(t.type);
        header.u32(t.rank);
        header.i32(layer);
        header.u32(0);
        header.u64(t.cols);
        header.u64(t.rank >= 2 ? t.rows : 1);
        header.u64(1);
        header.u64(1);
        header.u64(offsets[i]);
        header.u64(sizes[i]);
        header.u32(static_cast<std::uint32_t>(t.name.size()));
        header.u32(be);
        header.u32(bb);
        header.u32(0);
        header.raw(t.name.data(), t.name.size());
        header.pad(8);
    }
    std::memcpy(file.data(), header.data.data(), header.data.size());
    for (std::size_t i = 0; i < tensors.size(); ++i) {
        const std::vector<std::uint8_t> payload = materialise(tensors[i], spec, threads);
        std::memcpy(file.data() + offsets[i], payload.data(), payload.size());
    }
    write_file(dir / path, file);
    SegmentRecord record;
    record.kind = kind;
    record.layer = layer;
    record.tensor_count = tensors.size();
    record.payload = payload_total;
    record.file_size = file_size;
    record.path = path;
    jf_sha256_buffer(file.data(), file.size(), record.digest);
    return record;
}

struct Plan {
    std::vector<TensorPlan> input, output;
    std::vector<std::vector<TensorPlan>> layers;
    std::uint32_t layer_count, hidden, heads, kv_heads, ffn, vocab, context;
    float rope_base, rms_eps;
};

Plan make_plan(const jfb_synth_spec & s) {
    Plan p;
    if (s.kind == JFB_SYNTH_REFERENCE_FIXTURE) {
        p.layer_count = 2; p.hidden = 4; p.heads = 1; p.kv_heads = 1; p.ffn = 8; p.vocab = 8;
        p.context = 16; p.rope_base = 10000.0f; p.rms_eps = 1.0e-5f;
    } else {
        p.layer_count = s.layer_count; p.hidden = s.embedding_length; p.heads = s.head_count;
        p.kv_heads = s.kv_head_count; p.ffn = s.feed_forward_length; p.vocab = s.vocabulary_size;
        p.context = s.context_length; p.rope_base = s.rope_freq_base; p.rms_eps = s.rms_epsilon;
    }
    if (p.layer_count == 0 || p.hidden == 0 || p.heads == 0 || p.kv_heads == 0 || p.ffn == 0 ||
        p.vocab == 0 || p.context == 0 || p.hidden % p.heads != 0 || p.heads % p.kv_heads != 0) {
        throw WriterError(JFB_STATUS_INVALID_ARGUMENT, "synthetic model dimensions are inconsistent");
    }
    const std::uint64_t h = p.hidden, f = p.ffn, V = p.vocab;
    const std::uint64_t kvd = h / p.heads * p.kv_heads;
    const bool fixture = s.kind == JFB_SYNTH_REFERENCE_FIXTURE;
    auto matrix = [&](const std::string & name, std::uint32_t type, std::uint64_t cols, std::uint64_t rows, int layer) {
        TensorPlan t;
        t.name = name; t.type = type; t.cols = cols; t.rows = rows; t.rank = 2; t.layer = layer;
        t.fill = fixture ? TensorPlan::Constant : TensorPlan::Normal;
        t.constant = 0.01f;
        return t;
    };
    auto vector = [&](const std::string & name, std::uint64_t n, int layer, TensorPlan::Fill fill) {
        TensorPlan t;
        t.name = name; t.type = JF_TENSOR_F32; t.cols = n; t.rank = 1; t.layer = layer;
        t.fill = fixture ? TensorPlan::Constant : fill;
        t.constant = fill == TensorPlan::NormWeight ? 1.0f : 0.0f;
        return t;
    };
    const std::uint32_t layer_type = fixture ? JF_TENSOR_F32 : s.layer_type;
    TensorPlan embd = matrix("token_embd.weight", fixture ? JF_TENSOR_F32 : s.embedding_type, h, V, -1);
    if (fixture) { embd.fill = TensorPlan::RowScaled; embd.constant = 0.1f; }
    p.input.push_back(embd);
    p.output.push_back(vector("output_norm.weight", h, -1, TensorPlan::NormWeight));
    TensorPlan head = matrix("output.weight", fixture ? JF_TENSOR_F32 : s.output_type, h, V, -1);
    if (fixture) { head.fill = TensorPlan::RowScaled; head.constant = 0.01f; }
    p.output.push_back(head);
    const std::uint32_t L = p.layer_count;
    for (std::uint32_t i = 0; i < L; ++i) {
        const bool more_bits = i < L / 8 || i >= 7 * L / 8 || (i >= L / 8 && (i - L / 8) % 3 == 2);
        const std::uint32_t vd_type = (!fixture && s.more_bits_q6k && more_bits) ? JF_TENSOR_Q6_K : layer_type;
        const std::string b = "blk." + std::to_string(i) + ".";
        const int l = static_cast<int>(i);
        std::vector<TensorPlan> layer;
        layer.push_back(vector(b + "attn_norm.weight", h, l, TensorPlan::NormWeight));
        layer.push_back(matrix(b + "attn_q.weight", layer_type, h, h, l));
        layer.push_back(vector(b + "attn_q.bias", h, l, TensorPlan::Bias));
        layer.push_back(matrix(b + "attn_k.weight", layer_type, h, kvd, l));
        layer.push_back(vector(b + "attn_k.bias", kvd, l, TensorPlan::Bias));
        layer.push_back(matrix(b + "attn_v.weight", vd_type, h, kvd, l));
        layer.push_back(vector(b + "attn_v.bias", kvd, l, TensorPlan::Bias));
        layer.push_back(matrix(b + "attn_output.weight", layer_type, h, h, l));
        layer.push_back(vector(b + "ffn_norm.weight", h, l, TensorPlan::NormWeight));
        layer.push_back(matrix(b + "ffn_gate.weight", layer_type, h, f, l));
        layer.push_back(matrix(b + "ffn_up.weight", layer_type, h, f, l));
        layer.push_back(matrix(b + "ffn_down.weight", vd_type, f, h, l));
        p.layers.push_back(layer);
    }
    return p;
}

std::vector<std::uint8_t> gguf_metadata(const Plan & p, const jfb_synth_spec & spec, std::uint64_t * data_bytes) {
    std::vector<const TensorPlan *> order;
    for (const auto & t : p.input) order.push_back(&t);
    for (const auto & t : p.output) order.push_back(&t);
    for (const auto & layer : p.layers) for (const auto & t : layer) order.push_back(&t);
    Bytes g;
    g.raw("GGUF", 4);
    g.u32(3);
    g.u64(order.size());
    const bool fixture = spec.kind == JFB_SYNTH_REFERENCE_FIXTURE;
    const std::uint64_t kv_count = fixture ? 10 : 12;
    g.u64(kv_count);
    auto kv_u32 = [&](const char * key, std::uint32_t v) { g.gguf_string(key); g.u32(4); g.u32(v); };
    auto kv_f32 = [&](const char * key, float v) { g.gguf_string(key); g.u32(6); g.f32(v); };
    g.gguf_string("general.architecture"); g.u32(8); g.gguf_string("qwen2");
    kv_u32("qwen2.block_count", p.layer_count);
    kv_u32("qwen2.context_length", p.context);
    kv_u32("qwen2.embedding_length", p.hidden);
    kv_u32("qwen2.feed_forward_length", p.ffn);
    kv_u32("qwen2.attention.head_count", p.heads);
    kv_u32("qwen2.attention.head_count_kv", p.kv_heads);
    kv_u32("qwen2.rope.dimension_count", p.hidden / p.heads);
    kv_f32("qwen2.rope.freq_base", p.rope_base);
    kv_f32("qwen2.attention.layer_norm_rms_epsilon", p.rms_eps);
    if (!fixture) {
        g.gguf_string("jetsonfabric.synthetic.seed"); g.u32(10); g.u64(spec.seed);
        kv_f32("jetsonfabric.synthetic.weight_std", spec.weight_std);
    }
    std::uint64_t offset = 0;
    for (const TensorPlan * t : order) {
        g.gguf_string(t->name);
        g.u32(t->rank);
        g.u64(t->cols);
        if (t->rank >= 2) g.u64(t->rows);
        g.u32(ggml_type_id(t->type));
        g.u64(offset);
        offset = (offset + payload_bytes(*t) + 31) / 32 * 32;
    }
    g.pad(32);
    *data_bytes = offset;
    return g.data;
}

void write_package(const jfb_synth_spec & spec, const fs::path & dir, jfb_synth_report * report) {
    const Plan plan = make_plan(spec);
    unsigned threads = spec.threads != 0 ? spec.threads : std::max(1u, std::thread::hardware_concurrency());
    std::error_code ec;
    fs::create_directories(dir, ec);
    if (ec) throw WriterError(JFB_STATUS_IO_ERROR, "could not create package directory: " + ec.message());

    std::uint64_t data_bytes = 0;
    const std::vector<std::uint8_t> meta = gguf_metadata(plan, spec, &data_bytes);
    write_file(dir / "metadata.gguf", meta);
    std::vector<SegmentRecord> segments;
    SegmentRecord meta_record;
    meta_record.kind = 4;
    meta_record.layer = -1;
    meta_record.file_size = meta.size();
    meta_record.path = "metadata.gguf";
    jf_sha256_buffer(meta.data(), meta.size(), meta_record.digest);
    segments.push_back(meta_record);
    // One task per segment file (generate, encode, hash, write), the two
    // vocabulary-sized segments first and row-parallel, layers one per thread.
    const std::size_t task_count = plan.layer_count + 2u;
    std::vector<SegmentRecord> written(task_count);
    parallel_for(task_count, threads, [&](std::uint64_t begin, std::uint64_t end) {
        for (std::uint64_t task = begin; task < end; ++task) {
            if (task == 0) {
                written[0] = write_tensor_segment(dir, 1, -1, "input.jfs", plan.input, spec, std::max(1u, threads / 2));
            } else if (task == 1) {
                written[task_count - 1] = write_tensor_segment(dir, 3, -1, "output.jfs", plan.output, spec, std::max(1u, threads / 2));
            } else {
                const std::uint32_t i = static_cast<std::uint32_t>(task - 2);
                char name[32];
                std::snprintf(name, sizeof(name), "layer-%05u.jfs", i);
                written[1 + i] = write_tensor_segment(dir, 2, static_cast<std::int32_t>(i), name, plan.layers[i], spec, 1);
            }
        }
    }, 1);
    segments.insert(segments.end(), written.begin(), written.end());

    // Synthetic packages have no source GGUF file; the manifest's source
    // identity is the SHA-256 of metadata.gguf followed by every segment
    // digest in manifest order, and the source size is the size the GGUF
    // would have (header plus 32-byte aligned tensor data).
    std::vector<std::uint8_t> identity(meta);
    for (const auto & s : segments) identity.insert(identity.end(), s.digest, s.digest + 32);
    std::uint8_t source_digest[32];
    jf_sha256_buffer(identity.data(), identity.size(), source_digest);

    Bytes manifest;
    manifest.raw("JFMODEL2", 8);
    manifest.u32(2);
    manifest.u32(plan.layer_count);
    manifest.u64(meta.size() + data_bytes);
    manifest.raw(source_digest, 32);
    manifest.u32(static_cast<std::uint32_t>(segments.size()));
    manifest.u32(0);
    std::uint64_t weight_bytes = 0, tensor_count = 0, file_bytes = 0;
    for (const auto & s : segments) {
        manifest.u32(s.kind);
        manifest.i32(s.layer);
        manifest.u64(s.tensor_count);
        manifest.u64(s.payload);
        manifest.u64(s.file_size);
        manifest.raw(s.digest, 32);
        manifest.u32(static_cast<std::uint32_t>(s.path.size()));
        manifest.u32(0);
        manifest.raw(s.path.data(), s.path.size());
        weight_bytes += s.payload;
        tensor_count += s.tensor_count;
        file_bytes += s.file_size;
    }
    write_file(dir / "manifest.jfm", manifest.data);
    if (report != nullptr) {
        report->weight_bytes = weight_bytes;
        report->tensor_count = tensor_count;
        report->file_bytes = file_bytes;
    }
}

jfb_status make_status(jfb_status_code code, const char * message) {
    jfb_status s;
    s.code = code;
    std::snprintf(s.message, sizeof(s.message), "%s", message);
    return s;
}

}  // namespace

extern "C" jfb_status jfb_write_synthetic_package(const jfb_synth_spec * spec, const char * directory,
                                                  jfb_synth_report * report) {
    if (spec == nullptr || directory == nullptr || directory[0] == '\0') {
        return make_status(JFB_STATUS_INVALID_ARGUMENT, "spec and directory are required");
    }
    try {
        write_package(*spec, fs::path(directory), report);
        return make_status(JFB_STATUS_OK, "");
    } catch (const WriterError & e) {
        return make_status(e.code, e.what());
    } catch (const std::exception & e) {
        return make_status(JFB_STATUS_EXECUTION_FAILED, e.what());
    }
}

extern "C" jfb_status jfb_quantize_blocks(std::uint32_t type, const float * values, std::size_t count,
                                          void * blocks, std::size_t capacity) {
    if (values == nullptr || blocks == nullptr || count % 256 != 0) {
        return make_status(JFB_STATUS_INVALID_ARGUMENT, "values, blocks and a multiple of 256 elements are required");
    }
    std::size_t block_bytes = 0;
    switch (type) {
    case JF_TENSOR_Q2_K: block_bytes = 84; break;
    case JF_TENSOR_Q4_K: block_bytes = 144; break;
    case JF_TENSOR_Q6_K: block_bytes = 210; break;
    default: return make_status(JFB_STATUS_UNSUPPORTED, "only Q2_K, Q4_K and Q6_K are encodable");
    }
    if (capacity < count / 256 * block_bytes) return make_status(JFB_STATUS_INVALID_ARGUMENT, "block buffer too small");
    try {
        encode_row(type, values, count, static_cast<std::uint8_t *>(blocks));
    } catch (const std::exception & e) {
        return make_status(JFB_STATUS_EXECUTION_FAILED, e.what());
    }
    return make_status(JFB_STATUS_OK, "");
}

extern "C" const char * jfb_status_code_name(jfb_status_code code) {
    switch (code) {
    case JFB_STATUS_OK: return "ok";
    case JFB_STATUS_INVALID_ARGUMENT: return "invalid_argument";
    case JFB_STATUS_IO_ERROR: return "io_error";
    case JFB_STATUS_FORMAT_ERROR: return "format_error";
    case JFB_STATUS_NOT_FOUND: return "not_found";
    case JFB_STATUS_OUT_OF_MEMORY: return "out_of_memory";
    case JFB_STATUS_EXECUTION_FAILED: return "execution_failed";
    case JFB_STATUS_CUDA_ERROR: return "cuda_error";
    case JFB_STATUS_UNSUPPORTED: return "unsupported";
    case JFB_STATUS_TIMEOUT: return "timeout";
    }
    return "unknown";
}
