// Device-resident Qwen2 stage (see qwen2_stage.hpp).
//
// Forward pass per layer (reference graph qwen2_architecture.cpp:575-583),
// R rows over S sequences, all launches on the model's stream:
//   rmsnorm+quant(attn_norm) -> Q, K, V matmuls (+bias) -> RoPE + F16 KV append
//   -> attention (+Q8_K of the result) -> O matmul (+residual)
//   -> rmsnorm+quant(ffn_norm) -> gate, up matmuls -> SwiGLU (+Q8_K)
//   -> down matmul (+residual)
// then either the activations (intermediate stage) or, per sequence, the last
// row through output_norm, the LM head (+bias) and argmax (final stage,
// 584-597).
#include "qwen2_stage.hpp"

#include "gguf_meta.hpp"
#include "jetsonfabric/engine.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <iomanip>
#include <sstream>
#include <string>
#include <stdexcept>
#include <unordered_map>

namespace jfb::engine {

void cuda_check(cudaError_t e, const char * what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void jfb_check(const jfb_status & s) {
    if (s.code == JFB_STATUS_OK) return;
    if (s.code == JFB_STATUS_INVALID_ARGUMENT) throw std::invalid_argument(s.message);
    throw std::runtime_error(s.message);
}

namespace {

// Activation rows from which K-quant matmuls run on the tensor cores.
constexpr std::uint32_t kTensorCoreMinRows = 8;

}  // namespace

namespace {

// ---- hyper-parameters (reference qwen2_metadata.cpp:14-123) -----------------

const GgufValue & require_key(const GgufMetadata & g, const char * key) {
    const GgufValue * v = g.find(key);
    if (v == nullptr) throw std::runtime_error(std::string("missing GGUF metadata key ") + key);
    return *v;
}

std::uint32_t require_u32(const GgufMetadata & g, const char * key) {
    const GgufValue & v = require_key(g, key);
    if (v.type != GgufType::U32) throw std::runtime_error(std::string("GGUF metadata key is not uint32: ") + key);
    return static_cast<std::uint32_t>(v.u);
}

std::uint32_t optional_u32(const GgufMetadata & g, const char * key, std::uint32_t fallback) {
    const GgufValue * v = g.find(key);
    if (v == nullptr) return fallback;
    if (v->type != GgufType::U32) throw std::runtime_error(std::string("GGUF metadata key is not uint32: ") + key);
    return static_cast<std::uint32_t>(v->u);
}

float require_f32(const GgufMetadata & g, const char * key) {
    const GgufValue & v = require_key(g, key);
    if (v.type != GgufType::F32) throw std::runtime_error(std::string("GGUF metadata key is not float32: ") + key);
    return static_cast<float>(v.f);
}

}  // namespace

Qwen2HParams load_qwen2_hparams(std::span<const std::byte> blob) {
    const GgufMetadata g(blob);
    const GgufValue & arch = require_key(g, "general.architecture");
    if (arch.type != GgufType::STRING || arch.s != "qwen2") {
        throw std::runtime_error("native execution currently supports only qwen2 GGUF models");
    }
    if (const GgufValue * t = g.find("qwen2.rope.scaling.type")) {
        if (t->type != GgufType::STRING) throw std::runtime_error("Qwen2 RoPE scaling type is not a string");
        if (t->s != "none" && t->s != "linear") {
            throw std::runtime_error("native Qwen2 does not support RoPE scaling type " + t->s);
        }
    }
    if (const GgufValue * f = g.find("qwen2.rope.scaling.factor")) {
        if (f->type != GgufType::F32 || std::fabs(f->f - 1.0) > 1.0e-6) {
            throw std::runtime_error("native Qwen2 does not support scaled RoPE factors");
        }
    }
    Qwen2HParams p;
    p.info.architecture = "qwen2";
    p.info.layer_count = require_u32(g, "qwen2.block_count");
    p.info.embedding_length = require_u32(g, "qwen2.embedding_length");
    p.feed_forward_length = require_u32(g, "qwen2.feed_forward_length");
    p.head_count = require_u32(g, "qwen2.attention.head_count");
    p.kv_head_count = require_u32(g, "qwen2.attention.head_count_kv");
    p.info.context_length = require_u32(g, "qwen2.context_length");
    const std::uint32_t head_length = p.head_count == 0 ? 0 : p.info.embedding_length / p.head_count;
    p.rope_dimension_count = optional_u32(g, "qwen2.rope.dimension_count", head_length);
    p.rope_frequency_base = require_f32(g, "qwen2.rope.freq_base");
    p.rms_epsilon = require_f32(g, "qwen2.attention.layer_norm_rms_epsilon");
    // validate_hparams (qwen2_metadata.cpp:70-88)
    if (p.info.layer_count == 0 || p.info.embedding_length == 0 || p.feed_forward_length == 0 ||
        p.head_count == 0 || p.kv_head_count == 0 || p.info.context_length == 0) {
        throw std::runtime_error("Qwen2 metadata dimensions must be positive");
    }
    if (p.info.embedding_length % p.head_count != 0 || p.head_count % p.kv_head_count != 0) {
        throw std::runtime_error("Qwen2 attention dimensions are inconsistent");
    }
    if (p.rope_dimension_count != head_length || p.rms_epsilon <= 0.0f || p.rope_frequency_base <= 0.0f) {
        throw std::runtime_error("Qwen2 RoPE or RMS metadata is unsupported");
    }
    return p;
}

// ---- weights ----------------------------------------------------------------

namespace {

struct JfmModel {
    jf_model * m = nullptr;
    ~JfmModel() { if (m) jf_model_close(m); }
};

void jf_require(const jf_status & s, const char * what) {
    if (s.code != JF_STATUS_OK) throw std::runtime_error(std::string(what) + ": " + s.message);
}

std::string hex(const std::uint8_t * d, std::size_t n) {
    std::ostringstream o;
    o << std::hex << std::setfill('0');
    for (std::size_t i = 0; i < n; ++i) o << std::setw(2) << unsigned(d[i]);
    return o.str();
}

std::uint64_t align256(std::uint64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

namespace {

// Algorithmic bytes of one matmul launch: the weight's encoded bytes (GGML
// block size), the activations it reads (Q8_K planes or f32), the bias or
// residual it reads and the f32 outputs it writes.
double matmul_bytes(const jfb_weight & w, std::uint32_t n, std::uint32_t epilogue) {
    std::uint64_t block_bytes = 0;
    switch (w.type) {
    case JF_TENSOR_Q4_K: block_bytes = 144; break;
    case JF_TENSOR_Q6_K: block_bytes = 210; break;
    case JF_TENSOR_Q2_K: block_bytes = 84; break;
    default: break;
    }
    double weight = block_bytes ? double(w.rows) * (w.cols / 256) * block_bytes
                                : double(w.rows) * w.cols * (w.type == JF_TENSOR_F16 ? 2.0 : 4.0);
    double act = block_bytes ? double(n) * (w.cols + w.cols / 256 * 4.0 + w.cols / 16 * 2.0) : double(n) * w.cols * 4.0;
    double out = double(n) * w.rows * 4.0;
    double extra = epilogue == JFB_EPILOGUE_BIAS ? double(w.rows) * 4.0
                 : epilogue == JFB_EPILOGUE_RESIDUAL ? double(n) * w.rows * 4.0 : 0.0;
    return weight + act + out + extra;
}

}  // namespace

DeviceModel::DeviceModel(const std::string & package_path, std::uint32_t layer_start, std::uint32_t layer_end) {
    cuda_check(cudaGetDevice(&device_), "query CUDA device");
    kv_pool_ = std::make_shared<KvPool>(device_);
    cudaDeviceProp prop{};
    cuda_check(cudaGetDeviceProperties(&prop, device_), "query CUDA device properties");
    device_name_ = prop.name;

    // TensorStore opens the package with hash verification on
    // (reference tensor_store.cpp:67-79).
    JfmModel model;
    const jf_stage_plan plan{layer_start, layer_end, 1, 0};
    jf_require(jf_model_open(package_path.c_str(), &plan, &model.m), "open JFM package");
    const void * meta = nullptr;
    std::size_t meta_size = 0;
    jf_require(jf_model_get_gguf_metadata(model.m, &meta, &meta_size), "read JFM metadata");
    hp_ = load_qwen2_hparams(std::span<const std::byte>(static_cast<const std::byte *>(meta), meta_size));
    std::uint8_t digest[32];
    jf_require(jf_model_get_source_sha256(model.m, digest), "read JFM source identity");
    source_sha256_ = hex(digest, 32);
    const jf_model_stats stats = jf_model_get_stats(model.m);
    layer_start_ = stats.layer_start;
    layer_end_ = stats.layer_end;
    weight_bytes_ = stats.selected_weight_bytes;
    total_weight_bytes_ = stats.total_weight_bytes;
    tensor_count_ = stats.selected_tensor_count;
    if (stats.layer_count != hp_.info.layer_count) throw std::runtime_error("JFM layer count disagrees with GGUF metadata");

    std::unordered_map<std::string, jf_tensor_view> views;
    for (std::size_t i = 0; i < jf_model_tensor_count(model.m); ++i) {
        jf_tensor_view v{};
        jf_require(jf_model_tensor_at(model.m, i, &v), "read JFM tensor");
        views.emplace(std::string(v.name, v.name_length), v);
    }
    auto find = [&](const std::string & n) -> const jf_tensor_view * {
        const auto it = views.find(n);
        return it == views.end() ? nullptr : &it->second;
    };
    auto require = [&](const std::string & n) -> const jf_tensor_view & {
        const jf_tensor_view * v = find(n);
        if (v == nullptr) throw std::runtime_error("required native tensor is missing: " + n);
        return *v;
    };
    const jf_tensor_view * vocab_src = find("token_embd.weight");
    if (vocab_src == nullptr) vocab_src = find("output.weight");
    vocab_ = vocab_src == nullptr ? 0u : static_cast<std::uint32_t>(vocab_src->shape[1]);

    // shape contract (qwen2_architecture.cpp:80-118)
    const std::uint64_t h = hp_.info.embedding_length, kvd = hp_.kv_dim(), f = hp_.feed_forward_length;
    auto require_shape = [&](const std::string & n, std::initializer_list<std::uint64_t> dims) {
        const jf_tensor_view & v = require(n);
        if (v.rank != dims.size()) throw std::runtime_error("native Qwen2 tensor has wrong rank: " + n);
        std::size_t d = 0;
        for (std::uint64_t e : dims) {
            if (v.shape[d++] != e) throw std::runtime_error("native Qwen2 tensor has wrong shape: " + n);
        }
    };
    if (layer_start_ >= layer_end_ || layer_end_ > hp_.info.layer_count) {
        throw std::runtime_error("native Qwen2 layer range is invalid");
    }
    if (first_stage()) require_shape("token_embd.weight", {h, vocab_});
    if (last_stage()) {
        require_shape("output_norm.weight", {h});
        require_shape("output.weight", {h, vocab_});
        if (find("output.bias") != nullptr) require_shape("output.bias", {vocab_});
    }
    for (std::uint32_t l = layer_start_; l < layer_end_; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        require_shape(p + "attn_norm.weight", {h});
        require_shape(p + "attn_q.weight", {h, h});
        require_shape(p + "attn_q.bias", {h});
        require_shape(p + "attn_k.weight", {h, kvd});
        require_shape(p + "attn_k.bias", {kvd});
        require_shape(p + "attn_v.weight", {h, kvd});
        require_shape(p + "attn_v.bias", {kvd});
        require_shape(p + "attn_output.weight", {h, h});
        require_shape(p + "ffn_norm.weight", {h});
        require_shape(p + "ffn_gate.weight", {h, f});
        require_shape(p + "ffn_up.weight", {h, f});
        require_shape(p + "ffn_down.weight", {f, h});
    }

    // Fusion groups: a layer's Q/K/V and gate/up stacked by rows into one
    // matrix when they share a K-quant type, so a tensor-core launch covers
    // the group; the members become row views of it.
    struct Group {
        std::string name;
        std::vector<std::string> members;
        std::uint32_t type = 0, cols = 0, rows = 0;
        std::uint64_t raw_bytes = 0, offset = 0;
    };
    std::vector<Group> groups;
    std::unordered_map<std::string, std::size_t> grouped;  // member -> group
    auto is_kq = [](std::uint32_t t) { return t == JF_TENSOR_Q4_K || t == JF_TENSOR_Q6_K || t == JF_TENSOR_Q2_K; };
    for (std::uint32_t l = layer_start_; l < layer_end_; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        // (Q/K when V has another type, as on the layers whose V the Q4_K_M
        // map keeps in Q6_K)
        bool qkv_stacked = false;
        for (const auto & [gname, members] : std::vector<std::pair<std::string, std::vector<std::string>>>{
                 {p + "attn_qkv", {p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"}},
                 {p + "attn_qk", {p + "attn_q.weight", p + "attn_k.weight"}},
                 {p + "ffn_gate_up", {p + "ffn_gate.weight", p + "ffn_up.weight"}}}) {
            if (gname == p + "attn_qk" && qkv_stacked) continue;
            Group g;
            g.name = gname;
            g.members = members;
            bool ok = true;
            for (const std::string & m : members) {
                const jf_tensor_view & v = require(m);
                if (!is_kq(v.type) || (g.type != 0 && (v.type != g.type || v.shape[0] != g.cols))) ok = false;
                g.type = v.type;
                g.cols = static_cast<std::uint32_t>(v.shape[0]);
                g.rows += static_cast<std::uint32_t>(v.shape[1]);
                g.raw_bytes += v.size;
            }
            if (!ok) continue;
            if (gname == p + "attn_qkv") qkv_stacked = true;
            for (const std::string & m : members) grouped[m] = groups.size();
            groups.push_back(g);
        }
    }

    // One device arena for the whole stage; matrices in the planar layout.
    struct Placement {
        const jf_tensor_view * view;
        std::uint64_t offset;
        bool matrix;
    };
    std::vector<Placement> placements;
    std::uint64_t cursor = 0, max_raw = 0;
    std::unordered_map<std::string, std::size_t> index;
    for (Group & g : groups) {
        g.offset = cursor;
        cursor = align256(cursor + jfb_weight_device_bytes(g.type, g.rows, g.cols));
        max_raw = std::max<std::uint64_t>(max_raw, g.raw_bytes);
    }
    for (const auto & [name, v] : views) {
        if (grouped.count(name) != 0) continue;
        const bool matrix = v.rank == 2;
        std::uint64_t bytes;
        if (matrix) {
            bytes = jfb_weight_device_bytes(v.type, static_cast<std::uint32_t>(v.shape[1]),
                                            static_cast<std::uint32_t>(v.shape[0]));
            if (bytes == 0) throw std::runtime_error("unsupported tensor type for " + name);
            max_raw = std::max<std::uint64_t>(max_raw, v.size);
        } else {
            if (v.type != JF_TENSOR_F32) throw std::runtime_error("native Qwen2 vector tensor must be F32: " + name);
            bytes = v.size;
        }
        index[name] = placements.size();
        placements.push_back({&v, cursor, matrix});
        cursor = align256(cursor + bytes);
    }
    arena_bytes_ = cursor;
    cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "create CUDA stream");
    cuda_check(cudaMalloc(&arena_, arena_bytes_), "allocate native model weights on the device");
    void * staging = nullptr;
    if (max_raw > 0) cuda_check(cudaMalloc(&staging, max_raw), "allocate weight staging buffer");
    std::unordered_map<std::string, jfb_weight> matrices;
    for (const auto & [name, i] : index) {
        const Placement & pl = placements[i];
        std::uint8_t * dst = static_cast<std::uint8_t *>(arena_) + pl.offset;
        if (!pl.matrix) {
            cuda_check(cudaMemcpyAsync(dst, pl.view->data, pl.view->size, cudaMemcpyHostToDevice, stream_),
                       "upload native tensor");
            continue;
        }
        cuda_check(cudaMemcpyAsync(staging, pl.view->data, pl.view->size, cudaMemcpyHostToDevice, stream_),
                   "upload native tensor");
        jfb_weight w{};
        jfb_check(jfb_weight_repack(pl.view->type, static_cast<std::uint32_t>(pl.view->shape[1]),
                                    static_cast<std::uint32_t>(pl.view->shape[0]), staging, dst, &w, stream_));
        matrices[name] = w;
        cuda_check(cudaStreamSynchronize(stream_), "repack native tensor");  // staging is reused
    }
    std::unordered_map<std::string, jfb_weight> fused;
    for (const Group & g : groups) {
        std::uint64_t at = 0;
        for (const std::string & m : g.members) {
            const jf_tensor_view & v = require(m);
            cuda_check(cudaMemcpyAsync(static_cast<std::uint8_t *>(staging) + at, v.data, v.size, cudaMemcpyHostToDevice,
                                       stream_),
                       "upload native tensor");
            at += v.size;
        }
        jfb_weight w{};
        jfb_check(jfb_weight_repack(g.type, g.rows, g.cols, staging, static_cast<std::uint8_t *>(arena_) + g.offset, &w,
                                    stream_));
        fused[g.name] = w;
        std::uint32_t row = 0;
        for (const std::string & m : g.members) {
            const std::uint32_t rows = static_cast<std::uint32_t>(require(m).shape[1]);
            jfb_weight view{};
            jfb_check(jfb_weight_row_view(&w, row, rows, &view));
            matrices[m] = view;
            row += rows;
        }
        cuda_check(cudaStreamSynchronize(stream_), "repack native tensor");  // staging is reused
    }
    cuda_check(cudaStreamSynchronize(stream_), "upload native weights");
    if (staging != nullptr) cudaFree(staging);

    // RoPE coefficients, computed once on the host with the C library's
    // cosf/sinf exactly as GGML's rope cache does, then kept on the device.
    {
        const std::uint32_t positions = hp_.info.context_length, pairs = hp_.rope_dimension_count / 2;
        std::vector<float> table(std::size_t(positions) * pairs * 2);
        jfb_rope_table_host(table.data(), positions, hp_.rope_dimension_count, hp_.rope_frequency_base);
        cuda_check(cudaMalloc(&rope_table_, table.size() * sizeof(float)), "allocate rope table");
        cuda_check(cudaMemcpy(rope_table_, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice),
                   "upload rope table");
    }

    auto vec = [&](const std::string & n) -> const float * {
        const auto it = index.find(n);
        if (it == index.end()) return nullptr;
        return reinterpret_cast<const float *>(static_cast<std::uint8_t *>(arena_) + placements[it->second].offset);
    };
    auto mat = [&](const std::string & n) -> jfb_weight {
        const auto it = matrices.find(n);
        if (it == matrices.end()) throw std::runtime_error("required native tensor is missing: " + n);
        return it->second;
    };
    if (first_stage()) token_embd_ = mat("token_embd.weight");
    if (last_stage()) {
        output_ = mat("output.weight");
        output_norm_ = vec("output_norm.weight");
        output_bias_ = vec("output.bias");
    }
    for (std::uint32_t l = layer_start_; l < layer_end_; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        LayerWeights w;
        w.q = mat(p + "attn_q.weight");
        w.k = mat(p + "attn_k.weight");
        w.v = mat(p + "attn_v.weight");
        w.o = mat(p + "attn_output.weight");
        w.gate = mat(p + "ffn_gate.weight");
        w.up = mat(p + "ffn_up.weight");
        w.down = mat(p + "ffn_down.weight");
        w.attn_norm = vec(p + "attn_norm.weight");
        w.q_bias = vec(p + "attn_q.bias");
        w.k_bias = vec(p + "attn_k.bias");
        w.v_bias = vec(p + "attn_v.bias");
        w.ffn_norm = vec(p + "ffn_norm.weight");
        if (const auto it = fused.find(p + "attn_qkv"); it != fused.end()) w.qkv = it->second;
        if (const auto it = fused.find(p + "attn_qk"); it != fused.end()) w.qk = it->second;
        if (const auto it = fused.find(p + "ffn_gate_up"); it != fused.end()) w.gate_up = it->second;
        layer_weights_.push_back(w);
    }
}

DeviceModel::~DeviceModel() {
    if (arena_ != nullptr) cudaFree(arena_);
    if (rope_table_ != nullptr) cudaFree(rope_table_);
    if (stream_ != nullptr) cudaStreamDestroy(stream_);
}

// ---- KV cache ----------------------------------------------------------------

namespace {
constexpr std::uint64_t kKvMinChunk = 64ull << 20;    // smallest chunk taken from the device
constexpr std::uint64_t kKvMaxChunk = 2ull << 30;     // largest chunk (unless one cache is larger)
constexpr std::uint64_t kKvFreeMargin = 512ull << 20;  // device memory a new chunk must leave free
}  // namespace

KvPool::~KvPool() {
    for (void * c : chunks_) cudaFree(c);
}

std::uint64_t KvPool::reserved_bytes() const {
    std::lock_guard lock(mu_);
    return reserved_;
}

void * KvPool::acquire(std::uint64_t bytes) {
    std::lock_guard lock(mu_);
    auto it = free_.find(bytes);
    if (it != free_.end() && !it->second.empty()) {
        void * p = it->second.back();
        it->second.pop_back();
        return p;
    }
    if (left_ < bytes) {
        // a new chunk: room for about eight more caches of this size
        std::uint64_t want = std::max(bytes, std::min(kKvMaxChunk, std::max(kKvMinChunk, 8 * bytes)));
        int prev = -1;
        cuda_check(cudaGetDevice(&prev), "query the current device");
        cuda_check(cudaSetDevice(device_), "select the stage device");
        std::size_t free_bytes = 0, total_bytes = 0;
        cudaError_t e = cudaMemGetInfo(&free_bytes, &total_bytes);
        if (e == cudaSuccess && free_bytes < want + kKvFreeMargin) want = bytes;  // only what this cache needs
        void * chunk = nullptr;
        if (e == cudaSuccess && free_bytes >= want + kKvFreeMargin) e = cudaMalloc(&chunk, want);
        else if (e == cudaSuccess) e = cudaErrorMemoryAllocation;
        cudaSetDevice(prev);
        if (e != cudaSuccess || chunk == nullptr) {
            (void) cudaGetLastError();
            throw std::runtime_error("could not allocate native Qwen2 KV cache");
        }
        chunks_.push_back(chunk);
        reserved_ += want;
        // the unused tail of the previous chunk serves no later cache of this
        // size; keep it for smaller ones
        if (left_ >= 256) free_[left_].push_back(cursor_);
        cursor_ = static_cast<std::uint8_t *>(chunk);
        left_ = want;
    }
    void * p = cursor_;
    cursor_ += bytes;
    left_ -= bytes;
    return p;
}

void KvPool::release(void * p, std::uint64_t bytes) {
    std::lock_guard lock(mu_);
    free_[bytes].push_back(p);
}

KvCache::KvCache(const DeviceModel & model, std::uint32_t capacity) : pool_(model.kv_pool()), capacity_(capacity) {
    const std::uint64_t elems = std::uint64_t(model.layers()) * capacity * model.hparams().kv_dim();
    const std::uint64_t half = align256(elems * sizeof(std::uint16_t));
    bytes_ = 2 * elems * sizeof(std::uint16_t);
    block_ = 2 * half;
    auto * base = static_cast<std::uint8_t *>(pool_->acquire(block_));
    k_ = reinterpret_cast<std::uint16_t *>(base);
    v_ = reinterpret_cast<std::uint16_t *>(base + half);
    // the reference clears its cache buffer at allocation (qwen2_architecture.cpp:1091)
    const cudaError_t e = cudaMemsetAsync(base, 0, block_, model.stream());
    if (e != cudaSuccess) {
        pool_->release(base, block_);
        cuda_check(e, "clear KV cache");
    }
}

KvCache::~KvCache() {
    if (k_ != nullptr) pool_->release(k_, block_);
}

// ---- stage forward ----------------------------------------------------------

Qwen2Stage::Qwen2Stage(DeviceModel & model) : m_(model) {
    // rows per device pass: a larger batched prefill runs as several passes,
    // which bounds the activation scratch (about 330 KB per row at the 7B
    // widths); JFB_MAX_PASS_ROWS overrides the default
    if (const char * v = std::getenv("JFB_MAX_PASS_ROWS")) {
        const long n = std::strtol(v, nullptr, 10);
        if (n < 1 || n > (1L << 24)) throw std::invalid_argument("JFB_MAX_PASS_ROWS must be between 1 and 16777216");
        max_pass_rows_ = static_cast<std::uint32_t>(n);
    }
    // JFB_MATMUL_PATH selects between the two bit-identical K-quant matmuls:
    // "auto" (default), "cuda-core" or "tensor-core".
    if (const char * path = std::getenv("JFB_MATMUL_PATH")) {
        const std::string v(path);
        if (v == "cuda-core") matmul_path_ = 1;
        else if (v == "tensor-core") matmul_path_ = 2;
        else if (v != "auto" && !v.empty()) throw std::invalid_argument("JFB_MATMUL_PATH must be auto, cuda-core or tensor-core");
    }
}

void Qwen2Stage::check_device_errors() {
    if (tc_error_host_ == nullptr || *tc_error_host_ == 0) return;
    const int code = *tc_error_host_;
    *tc_error_host_ = 0;
    // an aborted launch may leave stream-K arrival counters mid-count
    if (tc_workspace_ != nullptr) cudaMemset(tc_workspace_, 0, tc_workspace_bytes_);
    throw std::runtime_error("native Qwen2 tensor-core matmul stalled: pipeline wait " + std::to_string(code) +
                             " timed out");
}

Qwen2Stage::~Qwen2Stage() {
    free_scratch();
    if (attn_scratch_ != nullptr) cudaFree(attn_scratch_);
    if (meta_uploaded_ != nullptr) cudaEventDestroy(meta_uploaded_);
    for (const TimedLaunch & t : timed_) {
        cudaEventDestroy(t.start);
        cudaEventDestroy(t.stop);
    }
    for (cudaEvent_t e : event_pool_) cudaEventDestroy(e);
    if (tc_error_host_ != nullptr) cudaFreeHost(const_cast<int *>(tc_error_host_));
}

cudaEvent_t Qwen2Stage::take_event() {
    if (!event_pool_.empty()) {
        cudaEvent_t e = event_pool_.back();
        event_pool_.pop_back();
        return e;
    }
    cudaEvent_t e;
    cuda_check(cudaEventCreate(&e), "create timing event");
    return e;
}

KernelTiming Qwen2Stage::collect_timing() {
    KernelTiming t;
    for (const TimedLaunch & l : timed_) {
        cuda_check(cudaEventSynchronize(l.stop), "wait for timed launch");
        float ms = 0.0f;
        cuda_check(cudaEventElapsedTime(&ms, l.start, l.stop), "read timing event");
        if (l.family == 0) {
            ++t.matmul_launches;
            t.matmul_ms += ms;
            t.matmul_bytes += l.bytes;
        } else {
            ++t.attention_launches;
            t.attention_ms += ms;
            t.attention_bytes += l.bytes;
        }
        event_pool_.push_back(l.start);
        event_pool_.push_back(l.stop);
    }
    timed_.clear();
    return t;
}

void Qwen2Stage::free_scratch() {
    for (void * p : {static_cast<void *>(hidden_), static_cast<void *>(xf_), static_cast<void *>(q_),
                     static_cast<void *>(k_), static_cast<void *>(v_), static_cast<void *>(attn_),
                     static_cast<void *>(gate_), static_cast<void *>(up_), static_cast<void *>(q8_.qs),
                     static_cast<void *>(q8_.d), static_cast<void *>(q8_.bsums), static_cast<void *>(q8_.qs_f16),
                     static_cast<void *>(q8_.bsums_f16), static_cast<void *>(q8_.d_t),
                     static_cast<void *>(logits_), static_cast<void *>(tokens_dev_),
                     static_cast<void *>(error_flag_), meta_dev_, tc_workspace_}) {
        if (p != nullptr) cudaFree(p);
    }
    if (meta_host_ != nullptr) cudaFreeHost(meta_host_);
    hidden_ = xf_ = q_ = k_ = v_ = attn_ = gate_ = up_ = logits_ = nullptr;
    q8_ = jfb_q8k{};
    meta_dev_ = meta_host_ = nullptr;
    tokens_dev_ = error_flag_ = nullptr;
    tc_workspace_ = nullptr;
    tc_workspace_bytes_ = 0;
    cap_rows_ = cap_seqs_ = 0;
    scratch_bytes_ = 0;
}

void Qwen2Stage::ensure_attention_scratch(std::uint64_t bytes) {
    if (bytes <= attn_scratch_bytes_) return;
    // rare: only calls beyond the single-launch attention's limits get here
    cuda_check(cudaStreamSynchronize(m_.stream()), "synchronise before attention scratch growth");
    if (attn_scratch_ != nullptr) cudaFree(attn_scratch_);
    attn_scratch_ = nullptr;
    attn_scratch_bytes_ = 0;
    cuda_check(cudaMalloc(&attn_scratch_, bytes), "allocate native attention scratch");
    attn_scratch_bytes_ = bytes;
}

void Qwen2Stage::ensure_scratch(std::uint32_t rows, std::uint32_t seqs) {
    // Sizes depend only on the rows and sequences of a call, never on the
    // positions, so a decode loop reaches a steady state after its first
    // call: nothing is freed or allocated (no device-wide synchronisation)
    // while this stage's sends to a neighbour stage may be in flight.
    if (rows <= cap_rows_ && seqs <= cap_seqs_) return;
    cuda_check(cudaStreamSynchronize(m_.stream()), "synchronise before scratch growth");
    // grow by at least half again, so that slowly growing batches
    // reallocate a logarithmic number of times
    auto grow = [](std::uint32_t need, std::uint32_t have) {
        return need <= have ? have : std::max(need, have + have / 2);
    };
    const std::uint32_t R = grow(rows, cap_rows_), S = grow(seqs, cap_seqs_);
    free_scratch();
    const Qwen2HParams & hp = m_.hparams();
    const std::uint64_t h = hp.info.embedding_length, kvd = hp.kv_dim(), f = hp.feed_forward_length;
    const std::uint64_t wide = std::max(h, f);
    std::uint64_t total = 0;
    auto alloc = [&](auto ** p, std::uint64_t bytes) {
        bytes = std::max<std::uint64_t>(bytes, 256);
        cuda_check(cudaMalloc(reinterpret_cast<void **>(p), bytes), "allocate native stage scratch");
        total += bytes;
    };
    alloc(&hidden_, std::uint64_t(R) * h * 4);
    alloc(&xf_, std::uint64_t(R) * wide * 4);
    alloc(&q_, std::uint64_t(R) * h * 4);
    alloc(&k_, std::uint64_t(R) * kvd * 4);
    alloc(&v_, std::uint64_t(R) * kvd * 4);
    alloc(&attn_, std::uint64_t(R) * h * 4);
    alloc(&gate_, std::uint64_t(R) * f * 4);
    alloc(&up_, std::uint64_t(R) * f * 4);
    alloc(&q8_.qs, std::uint64_t(R) * wide);
    alloc(&q8_.d, std::uint64_t(R) * (wide / 256 + 1) * 4);
    alloc(&q8_.bsums, std::uint64_t(R) * (wide / 16 + 1) * 2);
    // the tensor-core operands every quantizer also writes: f16 codes and
    // partial sums, d transposed [blocks][d_stride]
    q8_.d_stride = (R + 3) / 4 * 4;
    alloc(&q8_.qs_f16, std::uint64_t(R) * wide * 2);
    alloc(&q8_.bsums_f16, std::uint64_t(R) * (wide / 16 + 1) * 2);
    alloc(&q8_.d_t, std::uint64_t(q8_.d_stride) * (wide / 256 + 1) * 4);
    if (m_.last_stage()) alloc(&logits_, std::uint64_t(S) * m_.vocabulary() * 4);
    alloc(&tokens_dev_, std::uint64_t(S) * 4);
    alloc(&error_flag_, 4);
    meta_bytes_ = align256(std::uint64_t(3 * R + S) * 4) + std::uint64_t(S) * sizeof(jfb_kv_slot) + 256;
    alloc(&meta_dev_, meta_bytes_);
    cuda_check(cudaMallocHost(&meta_host_, meta_bytes_), "allocate pinned staging");
    // stream-K workspace of the tensor-core matmul: the largest need of any
    // weight of this stage at R rows (S rows for the output head)
    auto tc_need = [](const jfb_weight & w, std::uint32_t n) -> std::uint64_t {
        return jfb_matmul_tc_supported(&w) ? jfb_matmul_tc_workspace_bytes(w.rows, w.cols, n) : 0;
    };
    std::uint64_t tc = 0;
    for (std::uint32_t li = 0; li < m_.layers(); ++li) {
        const LayerWeights & lw = m_.layer(li);
        for (const jfb_weight * x : {&lw.q, &lw.k, &lw.v, &lw.o, &lw.gate, &lw.up, &lw.down, &lw.qkv, &lw.qk, &lw.gate_up}) {
            if (x->type != 0) tc = std::max(tc, tc_need(*x, R));
        }
    }
    if (m_.last_stage()) tc = std::max(tc, tc_need(m_.output(), S));
    if (tc > 0) {
        alloc(&tc_workspace_, tc);
        tc_workspace_bytes_ = std::max<std::uint64_t>(tc, 256);
        cuda_check(cudaMemsetAsync(tc_workspace_, 0, tc_workspace_bytes_, m_.stream()), "clear matmul workspace");
    }
    if (tc_error_host_ == nullptr) {
        int * host = nullptr;
        cuda_check(cudaHostAlloc(reinterpret_cast<void **>(&host), sizeof(int), cudaHostAllocMapped),
                   "allocate matmul error word");
        *host = 0;
        tc_error_host_ = host;
        cuda_check(cudaHostGetDevicePointer(reinterpret_cast<void **>(&tc_error_dev_), host, 0),
                   "map matmul error word");
    }
    cap_rows_ = R;
    cap_seqs_ = S;
    scratch_bytes_ = total;
}

void Qwen2Stage::forward(std::span<const SequenceRows> seqs, const ForwardIo & io) {
    std::uint64_t total = 0;
    for (const SequenceRows & s : seqs) {
        if (s.rows == 0 || s.cache == nullptr || s.start + s.rows > s.cache->capacity()) {
            throw std::invalid_argument("native Qwen2 rows are outside session capacity");
        }
        total += s.rows;
    }
    if (total <= max_pass_rows_) {
        forward_pass(seqs, io);
        return;
    }
    // Chunked pass (a large batched prefill): every row's result is computed
    // exactly as in one pass, since a row depends only on the KV cache rows
    // before it, which earlier passes have appended. Sequences are packed
    // into passes of at most max_pass_rows_ rows; a longer sequence is cut
    // into pieces of max_pass_rows_ rows, each a pass of its own, and only its
    // last piece produces the sequence's output (the others send their
    // sampled token to a scratch word).
    struct Piece {
        std::uint32_t seq, start, rows;
        bool final;
    };
    std::vector<Piece> pieces;
    for (std::uint32_t i = 0; i < seqs.size(); ++i) {
        std::uint32_t done = 0;
        while (seqs[i].rows - done > max_pass_rows_) {
            pieces.push_back(Piece{i, seqs[i].start + done, max_pass_rows_, false});
            done += max_pass_rows_;
        }
        pieces.push_back(Piece{i, seqs[i].start + done, seqs[i].rows - done, true});
    }
    const std::uint64_t h = m_.hparams().info.embedding_length, V = m_.vocabulary();
    std::uint64_t row0 = 0;
    std::vector<SequenceRows> pass;
    for (std::size_t p = 0; p < pieces.size();) {
        pass.clear();
        std::uint64_t rows = 0;
        const std::size_t first = p;
        // a non-final piece is always a pass of its own
        do {
            pass.push_back(SequenceRows{seqs[pieces[p].seq].cache, pieces[p].start, pieces[p].rows});
            rows += pieces[p].rows;
            ++p;
        } while (p < pieces.size() && pieces[first].final && pieces[p].final &&
                 rows + pieces[p].rows <= max_pass_rows_);
        ForwardIo pio = io;
        pio.synchronize = false;
        if (io.tokens != nullptr) pio.tokens = io.tokens + row0;
        if (io.activations != nullptr) pio.activations = io.activations + row0 * h;
        if (io.activations_out != nullptr) pio.activations_out = io.activations_out + row0 * h;
        if (!pieces[first].final) {
            pio.tokens_out = nullptr;  // the final stage samples into its scratch word
            pio.logits_out = nullptr;
        } else {
            const std::uint32_t s0 = pieces[first].seq;
            if (io.tokens_out != nullptr) pio.tokens_out = io.tokens_out + s0;
            if (io.logits_out != nullptr) pio.logits_out = io.logits_out + std::uint64_t(s0) * V;
        }
        forward_pass(pass, pio);
        row0 += rows;
    }
    if (io.synchronize) {
        cuda_check(cudaStreamSynchronize(m_.stream()), "native Qwen2 stage computation failed");
        check_device_errors();
    }
}

void Qwen2Stage::forward_pass(std::span<const SequenceRows> seqs, const ForwardIo & io) {
    const Qwen2HParams & hp = m_.hparams();
    const std::uint32_t S = static_cast<std::uint32_t>(seqs.size());
    std::uint32_t R = 0, max_keys = 1;
    for (const SequenceRows & s : seqs) {
        if (s.rows == 0 || s.cache == nullptr || s.start + s.rows > s.cache->capacity()) {
            throw std::invalid_argument("native Qwen2 rows are outside session capacity");
        }
        R += s.rows;
        max_keys = std::max(max_keys, s.start + s.rows);
    }
    if (S == 0 || R == 0) return;
    ensure_scratch(R, S);
    if (jfb_attention_call_scratch_bytes(R, hp.head_count, hp.kv_head_count, hp.head_dim(), max_keys) > 0) {
        // beyond the single-launch attention's limits: scratch for the next
        // multiple of 1024 keys (within the sessions' capacity), so that a
        // decode loop grows it once per 1024 positions at most
        std::uint32_t cap = max_keys;
        for (const SequenceRows & s : seqs) cap = std::max(cap, s.cache->capacity());
        const std::uint32_t keys = std::min(cap, (max_keys + 1023u) / 1024u * 1024u);
        const std::uint64_t bytes = jfb_attention_scratch_bytes(R, hp.head_count, hp.head_dim(), keys);
        if (bytes == UINT64_MAX) throw std::invalid_argument("native Qwen2 attention span is too long");
        ensure_attention_scratch(bytes);
    }
    cudaStream_t st = m_.stream();
    // the previous call's metadata upload may still be queued: wait until the
    // GPU has consumed the pinned staging buffer before rewriting it
    if (meta_uploaded_ == nullptr) {
        cuda_check(cudaEventCreateWithFlags(&meta_uploaded_, cudaEventDisableTiming), "create staging event");
    } else {
        cuda_check(cudaEventSynchronize(meta_uploaded_), "wait for staging buffer");
    }
    const std::uint64_t h = hp.info.embedding_length, f = hp.feed_forward_length;

    // per-call metadata, one pinned upload: seq[R] pos[R] last_row[S] tokens[R] | slots[S]
    auto * seq_h = static_cast<std::int32_t *>(meta_host_);
    std::int32_t * pos_h = seq_h + R;
    std::int32_t * last_h = pos_h + R;
    std::int32_t * tok_h = last_h + S;
    const std::uint64_t slot_off = align256(std::uint64_t(3 * R + S) * 4);
    auto * slots_h = reinterpret_cast<jfb_kv_slot *>(static_cast<std::uint8_t *>(meta_host_) + slot_off);
    std::uint32_t row = 0;
    for (std::uint32_t s = 0; s < S; ++s) {
        slots_h[s] = seqs[s].cache->slot();
        for (std::uint32_t t = 0; t < seqs[s].rows; ++t, ++row) {
            seq_h[row] = std::int32_t(s);
            pos_h[row] = std::int32_t(seqs[s].start + t);
        }
        last_h[s] = std::int32_t(row - 1);
    }
    const bool host_tokens = m_.first_stage() && !io.inputs_on_device;
    if (host_tokens) std::memcpy(tok_h, io.tokens, std::size_t(R) * 4);
    const std::uint64_t upload = slot_off + std::uint64_t(S) * sizeof(jfb_kv_slot);
    if (upload > meta_bytes_) throw std::logic_error("native stage metadata overflow");
    cuda_check(cudaMemcpyAsync(meta_dev_, meta_host_, upload, cudaMemcpyHostToDevice, st), "upload stage metadata");
    cuda_check(cudaEventRecord(meta_uploaded_, st), "record staging event");
    const auto * seq_d = static_cast<const std::int32_t *>(meta_dev_);
    const std::int32_t * pos_d = seq_d + R;
    const std::int32_t * last_d = pos_d + R;
    const std::int32_t * tok_d = last_d + S;
    const auto * slots_d = reinterpret_cast<const jfb_kv_slot *>(static_cast<const std::uint8_t *>(meta_dev_) + slot_off);
    launches_ = 0;

    // input rows
    if (m_.first_stage()) {
        const std::int32_t * tokens = io.inputs_on_device ? io.tokens : tok_d;
        jfb_check(jfb_embed_rows(&m_.token_embd(), tokens, R, hidden_, error_flag_, st));
        ++launches_;
    } else if (io.inputs_on_device) {
        cuda_check(cudaMemcpyAsync(hidden_, io.activations, std::uint64_t(R) * h * 4, cudaMemcpyDeviceToDevice, st),
                   "copy stage activations");
    } else {
        cuda_check(cudaMemcpyAsync(hidden_, io.activations, std::uint64_t(R) * h * 4, cudaMemcpyHostToDevice, st),
                   "upload stage activations");
    }

    for (const TimedLaunch & t : timed_) {  // results of an uncollected earlier pass are dropped
        event_pool_.push_back(t.start);
        event_pool_.push_back(t.stop);
    }
    timed_.clear();
    auto timed = [&](int family, double bytes, auto && launch) {
        if (!timing_) {
            launch();
            return;
        }
        TimedLaunch t{family, bytes, take_event(), take_event()};
        cuda_check(cudaEventRecord(t.start, st), "record timing event");
        launch();
        cuda_check(cudaEventRecord(t.stop, st), "record timing event");
        timed_.push_back(t);
    };
    auto use_tc = [&](const jfb_weight & w, std::uint32_t n) {
        return w.type != 0 && matmul_path_ != 1 && tc_workspace_ != nullptr && jfb_matmul_tc_supported(&w) &&
               (matmul_path_ == 2 || n >= kTensorCoreMinRows);
    };
    // one tensor-core launch over a stacked weight, one output segment per member
    auto mm_fused = [&](const jfb_weight & w, std::uint32_t n, const jfb_matmul_segment * segs, std::uint32_t count,
                        double bytes) {
        timed(0, bytes, [&] {
            jfb_check(jfb_matmul_tc_segments(&w, &q8_, n, segs, count, tc_workspace_, tc_workspace_bytes_, tc_error_dev_,
                                             st));
        });
    };
    auto mm = [&](const jfb_weight & w, const float * xf, std::uint32_t n, std::uint32_t ep, const float * bias,
                  const float * residual, float * out) {
        const bool tc = use_tc(w, n);
        timed(0, matmul_bytes(w, n, ep), [&] {
            if (tc) {
                jfb_check(jfb_matmul_tc(&w, &q8_, n, ep, bias, residual, out, tc_workspace_, tc_workspace_bytes_,
                                        tc_error_dev_, st));
            } else {
                jfb_check(jfb_matmul(&w, &q8_, xf, n, ep, bias, residual, out, st));
            }
        });
    };
    double kv_rows = 0.0;  // keys read per layer, summed over rows
    for (const SequenceRows & s : seqs) {
        for (std::uint32_t t = 0; t < s.rows; ++t) kv_rows += double(s.start + t + 1);
    }
    const double attention_bytes = kv_rows * hp.kv_dim() * 2.0 * 2.0 + double(R) * h * 4.0 * 2.0;
    auto needs_q8 = [](const jfb_weight & w) { return w.type == JF_TENSOR_Q4_K || w.type == JF_TENSOR_Q6_K || w.type == JF_TENSOR_Q2_K; };
    for (std::uint32_t li = 0; li < m_.layers(); ++li) {
        const LayerWeights & w = m_.layer(li);
        const bool attn_q8 = needs_q8(w.q) || needs_q8(w.k) || needs_q8(w.v);
        const bool attn_f32 = !needs_q8(w.q) || !needs_q8(w.k) || !needs_q8(w.v);
        jfb_check(jfb_rmsnorm_quant(hidden_, nullptr, w.attn_norm, R, std::uint32_t(h), hp.rms_epsilon,
                                    attn_f32 ? xf_ : nullptr, attn_q8 ? &q8_ : nullptr, st));
        if (use_tc(w.qkv, R)) {
            const std::uint32_t qr = w.q.rows, kr = w.k.rows, vr = w.v.rows;
            const jfb_matmul_segment segs[3] = {{qr, JFB_EPILOGUE_BIAS, w.q_bias, nullptr, q_},
                                                {qr + kr, JFB_EPILOGUE_BIAS, w.k_bias, nullptr, k_},
                                                {qr + kr + vr, JFB_EPILOGUE_BIAS, w.v_bias, nullptr, v_}};
            mm_fused(w.qkv, R, segs, 3,
                     matmul_bytes(w.q, R, JFB_EPILOGUE_BIAS) + matmul_bytes(w.k, R, JFB_EPILOGUE_BIAS) +
                         matmul_bytes(w.v, R, JFB_EPILOGUE_BIAS));
            launches_ -= 2;
        } else if (use_tc(w.qk, R)) {
            const std::uint32_t qr = w.q.rows, kr = w.k.rows;
            const jfb_matmul_segment segs[2] = {{qr, JFB_EPILOGUE_BIAS, w.q_bias, nullptr, q_},
                                                {qr + kr, JFB_EPILOGUE_BIAS, w.k_bias, nullptr, k_}};
            mm_fused(w.qk, R, segs, 2, matmul_bytes(w.q, R, JFB_EPILOGUE_BIAS) + matmul_bytes(w.k, R, JFB_EPILOGUE_BIAS));
            mm(w.v, xf_, R, JFB_EPILOGUE_BIAS, w.v_bias, nullptr, v_);
            launches_ -= 1;
        } else {
            mm(w.q, xf_, R, JFB_EPILOGUE_BIAS, w.q_bias, nullptr, q_);
            mm(w.k, xf_, R, JFB_EPILOGUE_BIAS, w.k_bias, nullptr, k_);
            mm(w.v, xf_, R, JFB_EPILOGUE_BIAS, w.v_bias, nullptr, v_);
        }
        jfb_check(jfb_rope_kv_append(q_, k_, v_, R, seq_d, pos_d, hp.head_count, hp.kv_head_count, hp.head_dim(),
                                     hp.rope_dimension_count, m_.rope_table(), hp.info.context_length, slots_d, li, st));
        const bool o_q8 = needs_q8(w.o);
        timed(1, attention_bytes, [&] {
            jfb_check(jfb_attention(q_, R, seq_d, pos_d, hp.head_count, hp.kv_head_count, hp.head_dim(), max_keys,
                                    slots_d, li, attn_scratch_, attn_scratch_bytes_, attn_, o_q8 ? &q8_ : nullptr, st));
        });
        mm(w.o, attn_, R, JFB_EPILOGUE_RESIDUAL, nullptr, hidden_, hidden_);
        const bool ffn_q8 = needs_q8(w.gate) || needs_q8(w.up);
        const bool ffn_f32 = !needs_q8(w.gate) || !needs_q8(w.up);
        jfb_check(jfb_rmsnorm_quant(hidden_, nullptr, w.ffn_norm, R, std::uint32_t(h), hp.rms_epsilon,
                                    ffn_f32 ? xf_ : nullptr, ffn_q8 ? &q8_ : nullptr, st));
        if (use_tc(w.gate_up, R)) {
            const jfb_matmul_segment segs[2] = {{w.gate.rows, JFB_EPILOGUE_STORE, nullptr, nullptr, gate_},
                                                {w.gate.rows + w.up.rows, JFB_EPILOGUE_STORE, nullptr, nullptr, up_}};
            mm_fused(w.gate_up, R, segs, 2,
                     matmul_bytes(w.gate, R, JFB_EPILOGUE_STORE) + matmul_bytes(w.up, R, JFB_EPILOGUE_STORE));
            launches_ -= 1;
        } else {
            mm(w.gate, xf_, R, JFB_EPILOGUE_STORE, nullptr, nullptr, gate_);
            mm(w.up, xf_, R, JFB_EPILOGUE_STORE, nullptr, nullptr, up_);
        }
        const bool down_q8 = needs_q8(w.down);
        jfb_check(jfb_swiglu_quant(gate_, up_, R, std::uint32_t(f), down_q8 ? nullptr : xf_, down_q8 ? &q8_ : nullptr, st));
        mm(w.down, xf_, R, JFB_EPILOGUE_RESIDUAL, nullptr, hidden_, hidden_);
        launches_ += 13;
    }

    if (!m_.last_stage()) {
        if (io.activations_out != nullptr) {
            cuda_check(cudaMemcpyAsync(io.activations_out, hidden_, std::uint64_t(R) * h * 4,
                                       io.activations_out_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st),
                       "read stage activations");
        }
    } else {
        const jfb_weight & out = m_.output();
        const bool q8 = needs_q8(out);
        jfb_check(jfb_rmsnorm_quant(hidden_, last_d, m_.output_norm(), S, std::uint32_t(h), hp.rms_epsilon,
                                    q8 ? nullptr : xf_, q8 ? &q8_ : nullptr, st));
        mm(out, xf_, S, m_.output_bias() ? JFB_EPILOGUE_BIAS : JFB_EPILOGUE_STORE, m_.output_bias(), nullptr, logits_);
        std::int32_t * token_dst = io.tokens_out_on_device && io.tokens_out != nullptr ? io.tokens_out : tokens_dev_;
        jfb_check(jfb_argmax(logits_, S, m_.vocabulary(), token_dst, st));
        launches_ += 3;
        if (io.tokens_out != nullptr && !io.tokens_out_on_device) {
            cuda_check(cudaMemcpyAsync(io.tokens_out, tokens_dev_, std::uint64_t(S) * 4, cudaMemcpyDeviceToHost, st),
                       "read greedy tokens");
        }
        if (io.logits_out != nullptr) {
            cuda_check(cudaMemcpyAsync(io.logits_out, logits_, std::uint64_t(S) * m_.vocabulary() * 4,
                                       cudaMemcpyDeviceToHost, st),
                       "read logits");
        }
    }
    if (io.synchronize) {
        cuda_check(cudaStreamSynchronize(st), "native Qwen2 stage computation failed");
        check_device_errors();
    }
}

}  // namespace jfb::engine
