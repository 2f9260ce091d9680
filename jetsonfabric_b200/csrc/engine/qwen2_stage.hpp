// Device-resident Qwen2 stage: weight arena (the TensorStore of the
// reference), per-session KV caches and the batched stage forward pass.
#pragma once

#include "jetsonfabric/native_inference.hpp"
#include "jfb/jfb_kernels.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <span>
#include <unordered_map>
#include <string>
#include <vector>

namespace jfb::engine {

using jetsonfabric::native::ModelInfo;

// Qwen2 hyper-parameters (reference qwen2_metadata.hpp / Qwen2HParams).
struct Qwen2HParams {
    ModelInfo info;
    std::uint32_t feed_forward_length = 0;
    std::uint32_t head_count = 0;
    std::uint32_t kv_head_count = 0;
    std::uint32_t rope_dimension_count = 0;
    float rope_frequency_base = 0.0f;
    float rms_epsilon = 0.0f;

    std::uint32_t head_dim() const { return info.embedding_length / head_count; }
    std::uint32_t kv_dim() const { return head_dim() * kv_head_count; }
};

struct LayerWeights {
    jfb_weight q{}, k{}, v{}, o{}, gate{}, up{}, down{};
    // Q/K/V and gate/up stacked by rows when they share a K-quant type (type
    // 0 otherwise), or Q/K alone when only V differs; q, k, v, gate and up are
    // then row views into them
    jfb_weight qkv{}, qk{}, gate_up{};
    const float * attn_norm = nullptr;
    const float * q_bias = nullptr;
    const float * k_bias = nullptr;
    const float * v_bias = nullptr;
    const float * ffn_norm = nullptr;
};

class KvPool;

// Throws std::runtime_error with `what` and the CUDA error string.
void cuda_check(cudaError_t e, const char * what);
// Throws std::runtime_error for a failing jfb_status.
void jfb_check(const jfb_status & s);

class DeviceModel {
public:
    DeviceModel(const std::string & package_path, std::uint32_t layer_start, std::uint32_t layer_end);
    ~DeviceModel();
    DeviceModel(const DeviceModel &) = delete;
    DeviceModel & operator=(const DeviceModel &) = delete;

    const Qwen2HParams & hparams() const { return hp_; }
    bool first_stage() const { return layer_start_ == 0; }
    bool last_stage() const { return layer_end_ == hp_.info.layer_count; }
    std::uint32_t layer_start() const { return layer_start_; }
    std::uint32_t layer_end() const { return layer_end_; }
    std::uint32_t layers() const { return layer_end_ - layer_start_; }
    std::uint32_t vocabulary() const { return vocab_; }
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    const jfb_weight & token_embd() const { return token_embd_; }
    const jfb_weight & output() const { return output_; }
    const float * output_norm() const { return output_norm_; }
    const float * output_bias() const { return output_bias_; }
    const LayerWeights & layer(std::uint32_t i) const { return layer_weights_[i]; }
    // GGML rope cache (cos, sin) for positions [0, context_length), device
    const float * rope_table() const { return rope_table_; }
    // the stage's KV cache memory (shared with the caches it handed out)
    const std::shared_ptr<KvPool> & kv_pool() const { return kv_pool_; }

    const std::string & source_sha256() const { return source_sha256_; }
    const std::string & device_name() const { return device_name_; }
    std::uint64_t weight_bytes() const { return weight_bytes_; }
    std::uint64_t total_weight_bytes() const { return total_weight_bytes_; }
    std::uint64_t tensor_count() const { return tensor_count_; }
    std::uint64_t arena_bytes() const { return arena_bytes_; }

private:
    Qwen2HParams hp_;
    std::uint32_t layer_start_ = 0, layer_end_ = 0, vocab_ = 0;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    void * arena_ = nullptr;
    std::uint64_t arena_bytes_ = 0;
    float * rope_table_ = nullptr;
    std::shared_ptr<KvPool> kv_pool_;
    jfb_weight token_embd_{}, output_{};
    const float * output_norm_ = nullptr;
    const float * output_bias_ = nullptr;
    std::vector<LayerWeights> layer_weights_;
    std::string source_sha256_, device_name_;
    std::uint64_t weight_bytes_ = 0, total_weight_bytes_ = 0, tensor_count_ = 0;
};

// Device memory for the KV caches of one stage's sessions. The reference
// allocates one cache buffer per session (qwen2_architecture.cpp:1056-1092);
// here sessions take their caches from large chunks that the stage keeps until
// it is destroyed, and a closed session's cache goes back to a free list by
// size for the next session of that size. Opening or closing a session
// therefore never calls cudaFree, which would synchronise the whole device
// (and, in a pipeline, wait behind transfers that need a peer stage's
// progress). A new chunk is admitted only while the device keeps a margin of
// free memory; past that, a session that needs new memory is refused with the
// reference's allocation error.
class KvPool {
public:
    explicit KvPool(int device) : device_(device) {}
    ~KvPool();
    KvPool(const KvPool &) = delete;
    KvPool & operator=(const KvPool &) = delete;
    void * acquire(std::uint64_t bytes);
    void release(void * p, std::uint64_t bytes);
    std::uint64_t reserved_bytes() const;

private:
    int device_;
    mutable std::mutex mu_;
    std::vector<void *> chunks_;
    std::uint8_t * cursor_ = nullptr;
    std::uint64_t left_ = 0, reserved_ = 0;
    std::unordered_map<std::uint64_t, std::vector<void *>> free_;
};

// Per-session F16 KV cache: K and V, each [layers][capacity][kv_dim].
class KvCache {
public:
    KvCache(const DeviceModel & model, std::uint32_t capacity);
    ~KvCache();
    KvCache(const KvCache &) = delete;
    KvCache & operator=(const KvCache &) = delete;
    jfb_kv_slot slot() const { return jfb_kv_slot{k_, v_, capacity_, 0}; }
    std::uint32_t capacity() const { return capacity_; }
    std::uint64_t bytes() const { return bytes_; }

private:
    std::shared_ptr<KvPool> pool_;
    std::uint16_t * k_ = nullptr;
    std::uint16_t * v_ = nullptr;
    std::uint32_t capacity_ = 0;
    std::uint64_t bytes_ = 0;
    std::uint64_t block_ = 0;  // bytes taken from the pool (K and V together)
};

// One sequence's slice of a batched forward call: `rows` consecutive rows
// starting at absolute position `start`.
struct SequenceRows {
    const KvCache * cache = nullptr;
    std::uint32_t start = 0;
    std::uint32_t rows = 0;
};

// Where the inputs come from and where the outputs go.
struct ForwardIo {
    // inputs (exactly one): token ids of every row, or f32 activations [R][h]
    const std::int32_t * tokens = nullptr;
    const float * activations = nullptr;
    bool inputs_on_device = false;
    // outputs of a final stage: one greedy token per sequence (host or
    // device), optionally the last row's logits per sequence [S][V] (host)
    std::int32_t * tokens_out = nullptr;
    bool tokens_out_on_device = false;
    float * logits_out = nullptr;
    // output of an intermediate stage: activations [R][h] (host or device)
    float * activations_out = nullptr;
    bool activations_out_on_device = false;
    // synchronise the stream before returning (needed for host outputs)
    bool synchronize = true;
};

// Per-kernel-family device time and algorithmic bytes of the last forward
// call made with timing enabled (CUDA events around each launch).
struct KernelTiming {
    std::uint64_t matmul_launches = 0;
    double matmul_ms = 0.0;
    double matmul_bytes = 0.0;
    std::uint64_t attention_launches = 0;
    double attention_ms = 0.0;
    double attention_bytes = 0.0;
};

class Qwen2Stage {
public:
    explicit Qwen2Stage(DeviceModel & model);
    ~Qwen2Stage();
    Qwen2Stage(const Qwen2Stage &) = delete;
    Qwen2Stage & operator=(const Qwen2Stage &) = delete;

    // Runs the stage over the rows of every sequence (positions must already
    // be validated by the caller). Launches on model.stream().
    void forward(std::span<const SequenceRows> seqs, const ForwardIo & io);

    std::uint64_t scratch_bytes() const { return scratch_bytes_; }
    std::uint64_t kernel_launches() const { return launches_; }
    void set_timing(bool enabled) { timing_ = enabled; }
    // Throws std::runtime_error when a tensor-core matmul of an earlier
    // launch gave up on a pipeline wait; call after the stream is synchronised.
    void check_device_errors();
    // Waits for the timed launches of the last forward and sums them up.
    KernelTiming collect_timing();

private:
    void forward_pass(std::span<const SequenceRows> seqs, const ForwardIo & io);
    void ensure_scratch(std::uint32_t rows, std::uint32_t seqs);
    void ensure_attention_scratch(std::uint64_t bytes);
    void free_scratch();

    DeviceModel & m_;
    // scratch (device)
    float * hidden_ = nullptr;
    float * xf_ = nullptr;
    float * q_ = nullptr;
    float * k_ = nullptr;
    float * v_ = nullptr;
    float * attn_ = nullptr;
    float * gate_ = nullptr;
    float * up_ = nullptr;
    jfb_q8k q8_{};
    void * attn_scratch_ = nullptr;
    std::uint64_t attn_scratch_bytes_ = 0;
    float * logits_ = nullptr;
    std::int32_t * tokens_dev_ = nullptr;
    std::int32_t * error_flag_ = nullptr;
    // tensor-core matmul: stream-K workspace (zero-filled) and an error word
    // in host-mapped pinned memory, readable without a copy after a sync
    void * tc_workspace_ = nullptr;
    std::uint64_t tc_workspace_bytes_ = 0;
    volatile int * tc_error_host_ = nullptr;
    int * tc_error_dev_ = nullptr;
    int matmul_path_ = 0;  // 0 auto, 1 CUDA cores only, 2 tensor cores wherever supported
    // per-call metadata: seq[R], pos[R], last_row[S], tokens[R], slots[S]
    void * meta_dev_ = nullptr;
    void * meta_host_ = nullptr;
    std::uint64_t meta_bytes_ = 0;
    cudaEvent_t meta_uploaded_ = nullptr;  // the pinned staging buffer is free again
    std::uint32_t cap_rows_ = 0, cap_seqs_ = 0;
    std::uint32_t max_pass_rows_ = 65536;
    std::uint64_t scratch_bytes_ = 0;
    std::uint64_t launches_ = 0;
    // kernel timing
    struct TimedLaunch {
        int family;  // 0 matmul, 1 attention
        double bytes;
        cudaEvent_t start, stop;
    };
    bool timing_ = false;
    std::vector<TimedLaunch> timed_;
    std::vector<cudaEvent_t> event_pool_;
    cudaEvent_t take_event();
};

Qwen2HParams load_qwen2_hparams(std::span<const std::byte> gguf_metadata);

}  // namespace jfb::engine
