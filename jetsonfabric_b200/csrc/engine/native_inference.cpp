// NativeEngine / NativeSession on the B200 stage engine.
//
// Session rules follow the reference Qwen2Session
// (runtime/engines/native/src/qwen2_architecture.cpp:785-1134):
//   - prefill starts at position 0 and needs 1 <= tokens <= capacity (1037-1045);
//   - decode needs 0 < position < capacity (1050-1054) and advances by one;
//   - rollback removes 1..(position - prefill_position) decoded tokens (818-823);
//   - only the first stage takes tokens, later stages take f32 activations
//     [tokens, hidden] (869-947, 1029-1036); the last stage returns a greedy
//     token, earlier stages return activations.
// Engine entry points follow native_inference.cpp:119-251 (logits,
// forced_decode_logits, generate with TTFT = first call, ITL = mean of the
// rest).
#include "jetsonfabric/native_batch.hpp"
#include "jetsonfabric/native_inference.hpp"
#include "engine_internal.hpp"
#include "qwen2_stage.hpp"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <limits>
#include <mutex>
#include <stdexcept>
#include <unordered_set>

namespace jetsonfabric::native {

using jfb::engine::DeviceModel;
using jfb::engine::ForwardIo;
using jfb::engine::KvCache;
using jfb::engine::Qwen2Stage;
using jfb::engine::SequenceRows;

namespace {

double elapsed_ms(std::chrono::steady_clock::time_point start) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - start).count();
}

}  // namespace

class NativeEngine::Impl {
public:
    Impl(const std::string & path, const EngineOptions & options) {
        if (options.backend != Backend::Cuda) {
            throw std::invalid_argument("the B200 native engine requires the CUDA backend");
        }
        prefill_kernel = resolve(options.prefill_attention_kernel);
        decode_kernel = resolve(options.decode_attention_kernel);
        model = std::make_unique<DeviceModel>(path, options.layer_start, options.layer_end);
        stage = std::make_unique<Qwen2Stage>(*model);
        info = model->hparams().info;
        info.source_sha256 = model->source_sha256();
        info.compute_backend = "CUDA" + std::to_string(model->device());
        info.compute_device = model->device_name();
        info.vocabulary_size = model->vocabulary();
        info.weight_bytes = model->weight_bytes();
        info.total_weight_bytes = model->total_weight_bytes();
        info.tensor_count = model->tensor_count();
        info.resident_layer_start = model->layer_start();
        info.resident_layer_end = model->layer_end();
    }

    // The CUDA attention kernel serves both the unfused and the flash request
    // (resolve_attention_kernel, qwen2_architecture.cpp:1149-1165): Automatic
    // resolves to Flash as it does on the reference's CUDA backend.
    static AttentionKernel resolve(AttentionKernel requested) {
        return requested == AttentionKernel::Automatic ? AttentionKernel::Flash : requested;
    }

    void validate_tokens(std::span<const std::int32_t> tokens) const {
        for (const std::int32_t t : tokens) {
            if (t < 0 || static_cast<std::uint32_t>(t) >= info.vocabulary_size) {
                throw std::invalid_argument("native token ID is outside model vocabulary");
            }
        }
    }

    std::unique_ptr<DeviceModel> model;
    std::unique_ptr<Qwen2Stage> stage;
    std::unique_ptr<NativeSession> generation_session;
    ModelInfo info;
    AttentionKernel prefill_kernel = AttentionKernel::Flash;
    AttentionKernel decode_kernel = AttentionKernel::Flash;
    std::recursive_mutex mutex;
};

class NativeSession::Impl {
public:
    Impl(NativeEngine::Impl & engine_in, std::size_t capacity_in)
        : engine(engine_in), cache(*engine_in.model, static_cast<std::uint32_t>(capacity_in)), capacity(capacity_in) {}

    bool first() const { return engine.model->first_stage(); }
    bool last() const { return engine.model->last_stage(); }
    std::size_t hidden() const { return engine.info.embedding_length; }

    void require_full_model() const {
        if (!first() || !last()) throw std::logic_error("full-model native inference requires every model layer");
    }

    void validate_prefill_count(std::size_t n) const {
        if (position != 0 || n == 0 || n > capacity) {
            throw std::invalid_argument("native Qwen2 prefill is outside session capacity");
        }
    }

    void validate_decode() const {
        if (position == 0 || position >= capacity) {
            throw std::invalid_argument("native Qwen2 decode is outside session capacity");
        }
    }

    void validate_activation(const ActivationView & a) const {
        const std::size_t h = hidden();
        const std::size_t max = std::numeric_limits<std::size_t>::max();
        if (a.token_count == 0 || h == 0 || a.token_count > max / h || a.token_count * h > max / sizeof(float) ||
            a.bytes.size() != a.token_count * h * sizeof(float)) {
            throw std::invalid_argument("native stage activation shape is invalid");
        }
    }

    NativeEngine::Impl & engine;
    KvCache cache;
    std::size_t capacity;
    std::size_t position = 0;
    std::size_t prefill_position = 0;
};

NativeSession::NativeSession(std::unique_ptr<Impl> impl) : impl_(std::move(impl)) {}
NativeSession::~NativeSession() = default;
NativeSession::NativeSession(NativeSession &&) noexcept = default;
NativeSession & NativeSession::operator=(NativeSession &&) noexcept = default;

std::size_t NativeSession::capacity() const { return impl_->capacity; }
std::size_t NativeSession::position() const { return impl_->position; }

// Shared implementation of every single- and multi-session stage call.
struct BatchAccess {
    struct Item {
        NativeSession::Impl * s;
        std::span<const std::int32_t> tokens;
        ActivationView activation;
    };

    // Runs one batched pass; prefill == true for position-0 prompts.
    static std::vector<StageResult> run(NativeEngine::Impl & e, std::span<Item> items, bool prefill,
                                        std::vector<float> * logits = nullptr) {
        std::lock_guard lock(e.mutex);
        const bool first = e.model->first_stage(), last = e.model->last_stage();
        const std::size_t h = e.info.embedding_length;
        std::unordered_set<const NativeSession::Impl *> seen;
        std::vector<SequenceRows> seqs;
        std::vector<std::int32_t> tokens;
        std::vector<float> acts;
        std::size_t rows = 0;
        for (Item & it : items) {
            if (it.s == nullptr || &it.s->engine != &e) throw std::invalid_argument("native session belongs to another engine");
            if (!seen.insert(it.s).second) throw std::invalid_argument("native batch contains a session twice");
            std::size_t n;
            if (first) {
                if (!it.activation.empty()) throw std::invalid_argument("the first native stage does not accept activations");
                n = it.tokens.size();
                e.validate_tokens(it.tokens);
            } else {
                if (!it.tokens.empty()) throw std::invalid_argument("only the first native stage accepts tokens");
                it.s->validate_activation(it.activation);
                n = it.activation.token_count;
            }
            if (prefill) {
                it.s->validate_prefill_count(n);
            } else {
                if (n != 1) throw std::invalid_argument("native decode activation must contain one token row");
                it.s->validate_decode();
            }
            seqs.push_back(SequenceRows{&it.s->cache, static_cast<std::uint32_t>(it.s->position), static_cast<std::uint32_t>(n)});
            rows += n;
        }
        if (first) {
            tokens.reserve(rows);
            for (const Item & it : items) tokens.insert(tokens.end(), it.tokens.begin(), it.tokens.end());
        } else {
            acts.resize(rows * h);
            std::size_t off = 0;
            for (const Item & it : items) {
                std::memcpy(acts.data() + off, it.activation.bytes.data(), it.activation.bytes.size());
                off += it.activation.bytes.size() / sizeof(float);
            }
        }
        std::vector<StageResult> results(items.size());
        std::vector<std::int32_t> sampled(items.size(), -1);
        std::vector<float> out_acts;
        ForwardIo io;
        io.tokens = first ? tokens.data() : nullptr;
        io.activations = first ? nullptr : acts.data();
        if (last) {
            io.tokens_out = sampled.data();
            if (logits != nullptr) {
                logits->resize(items.size() * std::size_t(e.info.vocabulary_size));
                io.logits_out = logits->data();
            }
        } else {
            out_acts.resize(rows * h);
            io.activations_out = out_acts.data();
        }
        e.stage->forward(seqs, io);
        std::size_t off = 0;
        for (std::size_t i = 0; i < items.size(); ++i) {
            NativeSession::Impl & s = *items[i].s;
            const std::size_t n = seqs[i].rows;
            s.position += n;
            if (prefill) s.prefill_position = s.position;
            if (last) {
                results[i].sampled_token = sampled[i];
            } else {
                results[i].activation.token_count = n;
                results[i].activation.bytes.resize(n * h * sizeof(float));
                std::memcpy(results[i].activation.bytes.data(), out_acts.data() + off, n * h * sizeof(float));
            }
            off += n * h;
        }
        return results;
    }

    static StageResult single(NativeSession * session, std::span<const std::int32_t> tokens, ActivationView activation,
                              bool prefill, std::vector<float> * logits) {
        NativeSession::Impl * s = session->impl_.get();
        Item item{s, tokens, activation};
        return std::move(run(s->engine, std::span<Item>(&item, 1), prefill, logits).front());
    }

    // Device-resident pass of any stage (no host copies, no sync): the first
    // stage reads token ids, later stages f32 activations [rows][h]; the last
    // stage writes one greedy token per session, the others f32 activations.
    static void run_device(NativeEngine & engine, std::span<NativeSession * const> sessions, bool prefill,
                           const std::int32_t * tokens_device, const float * activations_device,
                           std::span<const std::uint32_t> counts, std::int32_t * tokens_out_device,
                           float * activations_out_device) {
        NativeEngine::Impl & e = *engine.impl_;
        std::lock_guard lock(e.mutex);
        const bool first = e.model->first_stage(), last = e.model->last_stage();
        if (first ? tokens_device == nullptr : activations_device == nullptr) {
            throw std::invalid_argument(first ? "only the first native stage accepts tokens"
                                              : "the first native stage does not accept activations");
        }
        if (last ? tokens_out_device == nullptr : activations_out_device == nullptr) {
            throw std::invalid_argument(last ? "the last native stage returns greedy tokens"
                                             : "an intermediate native stage returns activations");
        }
        if (prefill && counts.size() != sessions.size()) {
            throw std::invalid_argument("one prompt length per session is required");
        }
        std::unordered_set<const NativeSession::Impl *> seen;
        std::vector<SequenceRows> seqs;
        for (std::size_t i = 0; i < sessions.size(); ++i) {
            NativeSession::Impl * s = impl(sessions[i]);
            if (s == nullptr || &s->engine != &e) throw std::invalid_argument("native session belongs to another engine");
            if (!seen.insert(s).second) throw std::invalid_argument("native batch contains a session twice");
            const std::size_t n = prefill ? counts[i] : 1u;
            if (prefill) s->validate_prefill_count(n); else s->validate_decode();
            seqs.push_back(SequenceRows{&s->cache, static_cast<std::uint32_t>(s->position), static_cast<std::uint32_t>(n)});
        }
        if (seqs.empty()) return;
        ForwardIo io;
        io.tokens = first ? tokens_device : nullptr;
        io.activations = first ? nullptr : activations_device;
        io.inputs_on_device = true;
        io.tokens_out = last ? tokens_out_device : nullptr;
        io.tokens_out_on_device = true;
        io.activations_out = last ? nullptr : activations_out_device;
        io.activations_out_on_device = true;
        io.synchronize = false;
        e.stage->forward(seqs, io);
        for (std::size_t i = 0; i < sessions.size(); ++i) {
            NativeSession::Impl * s = impl(sessions[i]);
            s->position += seqs[i].rows;
            if (prefill) s->prefill_position = s->position;
        }
    }

    static NativeEngine::Impl & impl_of(const NativeEngine & e) { return *e.impl_; }
    static const NativeSession::Impl & impl_of(const NativeSession & s) { return *s.impl_; }

    static NativeSession::Impl * impl(NativeSession * s) { return s == nullptr ? nullptr : s->impl_.get(); }
    static NativeEngine::Impl & impl(NativeEngine & e) { return *e.impl_; }
};

namespace {

StageResult single(NativeSession * session, std::span<const std::int32_t> tokens, ActivationView activation,
                   bool prefill, std::vector<float> * logits = nullptr) {
    return BatchAccess::single(session, tokens, activation, prefill, logits);
}

}  // namespace

std::int32_t NativeSession::prefill_greedy(std::span<const std::int32_t> tokens) {
    impl_->require_full_model();
    return single(this, tokens, {}, true).sampled_token;
}

std::int32_t NativeSession::decode_greedy(std::int32_t token) {
    impl_->require_full_model();
    return single(this, std::span<const std::int32_t>(&token, 1), {}, false).sampled_token;
}

StageResult NativeSession::prefill_stage_tokens(std::span<const std::int32_t> tokens) {
    if (!impl_->first()) throw std::invalid_argument("only the first native stage accepts tokens");
    return single(this, tokens, {}, true);
}

StageResult NativeSession::prefill_stage_activations(ActivationView activation) {
    if (impl_->first()) throw std::invalid_argument("the first native stage does not accept activations");
    return single(this, {}, activation, true);
}

StageResult NativeSession::decode_stage_token(std::int32_t token) {
    if (!impl_->first()) throw std::invalid_argument("only the first native stage accepts decode tokens");
    return single(this, std::span<const std::int32_t>(&token, 1), {}, false);
}

StageResult NativeSession::decode_stage_activation(ActivationView activation) {
    if (impl_->first()) throw std::invalid_argument("the first native stage does not accept decode activations");
    if (activation.token_count != 1U) {
        impl_->validate_activation(activation);
        throw std::invalid_argument("native decode activation must contain one token row");
    }
    return single(this, {}, activation, false);
}

void NativeSession::rollback(std::size_t token_count) {
    std::lock_guard lock(impl_->engine.mutex);
    if (token_count == 0 || token_count > impl_->position - impl_->prefill_position) {
        throw std::invalid_argument("native Qwen2 rollback exceeds the decoded suffix");
    }
    impl_->position -= token_count;
}

// ---- engine -------------------------------------------------------------------

NativeEngine::NativeEngine(const std::string & package_path, Backend backend, int threads)
    : NativeEngine(package_path, EngineOptions{backend, AttentionKernel::Automatic, AttentionKernel::Automatic, threads, 0,
                                               std::numeric_limits<std::uint32_t>::max()}) {}

NativeEngine::NativeEngine(const std::string & package_path, EngineOptions options) {
    const auto start = std::chrono::steady_clock::now();
    impl_ = std::make_unique<Impl>(package_path, options);
    load_time_ms_ = elapsed_ms(start);
}

NativeEngine::~NativeEngine() = default;
NativeEngine::NativeEngine(NativeEngine &&) noexcept = default;
NativeEngine & NativeEngine::operator=(NativeEngine &&) noexcept = default;

const ModelInfo & NativeEngine::model_info() const { return impl_->info; }
AttentionKernel NativeEngine::prefill_attention_kernel() const { return impl_->prefill_kernel; }
AttentionKernel NativeEngine::decode_attention_kernel() const { return impl_->decode_kernel; }
double NativeEngine::load_time_ms() const { return load_time_ms_; }

std::unique_ptr<NativeSession> NativeEngine::create_session(std::size_t capacity) {
    if (capacity == 0 || capacity > impl_->info.context_length) {
        throw std::invalid_argument("native session capacity is outside model context");
    }
    std::lock_guard lock(impl_->mutex);
    return std::unique_ptr<NativeSession>(new NativeSession(std::make_unique<NativeSession::Impl>(*impl_, capacity)));
}

void NativeEngine::release_session() {
    std::lock_guard lock(impl_->mutex);
    impl_->generation_session.reset();
}

std::vector<float> NativeEngine::logits(std::span<const std::int32_t> tokens) {
    if (tokens.empty() || tokens.size() > impl_->info.context_length) {
        throw std::invalid_argument("native token sequence is outside model context");
    }
    impl_->validate_tokens(tokens);
    auto session = create_session(tokens.size());
    session->impl_->require_full_model();
    std::vector<float> out;
    single(session.get(), tokens, {}, true, &out);
    return out;
}

std::vector<std::vector<float>> NativeEngine::forced_decode_logits(std::span<const std::int32_t> prompt_tokens,
                                                                   std::span<const std::int32_t> forced_tokens) {
    if (prompt_tokens.empty() || prompt_tokens.size() + forced_tokens.size() > impl_->info.context_length) {
        throw std::invalid_argument("native logit trace is outside model context");
    }
    impl_->validate_tokens(prompt_tokens);
    impl_->validate_tokens(forced_tokens);
    auto session = create_session(prompt_tokens.size() + forced_tokens.size());
    session->impl_->require_full_model();
    std::vector<std::vector<float>> trace;
    trace.reserve(forced_tokens.size() + 1);
    std::vector<float> l;
    single(session.get(), prompt_tokens, {}, true, &l);
    trace.push_back(l);
    for (const std::int32_t t : forced_tokens) {
        single(session.get(), std::span<const std::int32_t>(&t, 1), {}, false, &l);
        trace.push_back(l);
    }
    return trace;
}

GenerationResult NativeEngine::generate(std::span<const std::int32_t> prompt_tokens, std::uint32_t max_tokens) {
    if (prompt_tokens.empty() || max_tokens == 0) {
        throw std::invalid_argument("native generation requires prompt and output tokens");
    }
    const std::size_t required = prompt_tokens.size() + max_tokens - 1U;
    if (required > impl_->info.context_length) throw std::invalid_argument("native generation exceeds model context");
    impl_->validate_tokens(prompt_tokens);
    std::lock_guard lock(impl_->mutex);
    bool reused = impl_->generation_session && impl_->generation_session->capacity() == required;
    if (!reused) impl_->generation_session = create_session(required);
    NativeSession & session = *impl_->generation_session;
    session.impl_->position = 0;
    session.impl_->prefill_position = 0;
    GenerationResult result;
    double total_ms = 0.0, decode_ms = 0.0;
    for (std::uint32_t i = 0; i < max_tokens; ++i) {
        const auto start = std::chrono::steady_clock::now();
        const std::int32_t token = i == 0 ? session.prefill_greedy(prompt_tokens)
                                          : session.decode_greedy(result.sampled_tokens.back());
        const double ms = elapsed_ms(start);
        if (i == 0) {
            result.time_to_first_token_ms = ms;
            result.prefill.compute_ms = ms;
        } else {
            decode_ms += ms;
        }
        total_ms += ms;
        result.sampled_tokens.push_back(token);
    }
    result.prefill.plan_reused = reused;
    result.prefill.attention_backend_verified = true;
    if (max_tokens > 1) {
        result.inter_token_latency_ms = decode_ms / double(max_tokens - 1);
        result.decode_tokens_per_second = 1000.0 / result.inter_token_latency_ms;
    }
    result.end_to_end_tokens_per_second = 1000.0 * double(max_tokens) / total_ms;
    result.buffers.kv_cache_bytes = session.impl_->cache.bytes();
    result.buffers.prefill_scratch_bytes = impl_->stage->scratch_bytes();
    result.buffers.decode_scratch_bytes = impl_->stage->scratch_bytes();
    result.buffers.prefill_host_input_bytes = prompt_tokens.size() * sizeof(std::int32_t);
    return result;
}

// ---- batch API --------------------------------------------------------------------

namespace {

std::vector<BatchAccess::Item> items_for(std::span<NativeSession * const> sessions) {
    std::vector<BatchAccess::Item> items;
    items.reserve(sessions.size());
    for (NativeSession * s : sessions) {
        if (s == nullptr) throw std::invalid_argument("native batch contains a null session");
        items.push_back(BatchAccess::Item{BatchAccess::impl(s), {}, {}});
    }
    return items;
}

}  // namespace

std::vector<StageResult> prefill_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                             std::span<const std::span<const std::int32_t>> prompts) {
    if (sessions.size() != prompts.size()) throw std::invalid_argument("one prompt per session is required");
    auto items = items_for(sessions);
    for (std::size_t i = 0; i < items.size(); ++i) items[i].tokens = prompts[i];
    if (items.empty()) return {};
    return BatchAccess::run(BatchAccess::impl(engine), items, true);
}

std::vector<StageResult> prefill_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                             std::span<const ActivationView> activations) {
    if (sessions.size() != activations.size()) throw std::invalid_argument("one activation block per session is required");
    auto items = items_for(sessions);
    for (std::size_t i = 0; i < items.size(); ++i) items[i].activation = activations[i];
    if (items.empty()) return {};
    return BatchAccess::run(BatchAccess::impl(engine), items, true);
}

std::vector<StageResult> decode_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                            std::span<const std::int32_t> tokens) {
    if (sessions.size() != tokens.size()) throw std::invalid_argument("one decode token per session is required");
    auto items = items_for(sessions);
    for (std::size_t i = 0; i < items.size(); ++i) items[i].tokens = tokens.subspan(i, 1);
    if (items.empty()) return {};
    return BatchAccess::run(BatchAccess::impl(engine), items, false);
}

std::vector<StageResult> decode_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                            std::span<const ActivationView> activations) {
    if (sessions.size() != activations.size()) throw std::invalid_argument("one activation row per session is required");
    auto items = items_for(sessions);
    for (std::size_t i = 0; i < items.size(); ++i) items[i].activation = activations[i];
    if (items.empty()) return {};
    return BatchAccess::run(BatchAccess::impl(engine), items, false);
}

namespace detail {

static void require_full_model_device(NativeEngine & engine) {
    const ModelInfo info = engine.model_info();
    if (info.resident_layer_start != 0 || info.resident_layer_end != info.layer_count) {
        throw std::logic_error("full-model native inference requires every model layer");
    }
}

void decode_batch_device(NativeEngine & engine, std::span<NativeSession * const> sessions,
                         const std::int32_t * tokens_device, std::int32_t * tokens_out_device) {
    require_full_model_device(engine);
    BatchAccess::run_device(engine, sessions, false, tokens_device, nullptr, {}, tokens_out_device, nullptr);
}

void prefill_batch_device(NativeEngine & engine, std::span<NativeSession * const> sessions,
                          const std::int32_t * tokens_device, std::span<const std::uint32_t> counts,
                          std::int32_t * tokens_out_device) {
    require_full_model_device(engine);
    if (counts.size() != sessions.size()) throw std::invalid_argument("one prompt length per session is required");
    BatchAccess::run_device(engine, sessions, true, tokens_device, nullptr, counts, tokens_out_device, nullptr);
}

void stage_batch_device(NativeEngine & engine, std::span<NativeSession * const> sessions, bool prefill,
                        std::span<const std::uint32_t> counts, const std::int32_t * tokens_device,
                        const float * activations_device, std::int32_t * tokens_out_device,
                        float * activations_out_device) {
    BatchAccess::run_device(engine, sessions, prefill, tokens_device, activations_device, counts, tokens_out_device,
                            activations_out_device);
}

void synchronize(NativeEngine & engine) {
    jfb::engine::cuda_check(cudaStreamSynchronize(BatchAccess::impl_of(engine).model->stream()),
                            "native Qwen2 stage computation failed");
    BatchAccess::impl_of(engine).stage->check_device_errors();
}

void * stream(NativeEngine & engine) { return BatchAccess::impl_of(engine).model->stream(); }

std::uint64_t last_launch_count(const NativeEngine & engine) { return BatchAccess::impl_of(engine).stage->kernel_launches(); }

std::uint64_t scratch_bytes(const NativeEngine & engine) { return BatchAccess::impl_of(engine).stage->scratch_bytes(); }

std::uint64_t kv_cache_bytes(const NativeSession & session) { return BatchAccess::impl_of(session).cache.bytes(); }

void reset(NativeSession & session) {
    auto * s = BatchAccess::impl(&session);
    std::lock_guard lock(s->engine.mutex);
    s->position = 0;
    s->prefill_position = 0;
}

void set_kernel_timing(NativeEngine & engine, bool enabled) {
    auto & e = BatchAccess::impl_of(engine);
    std::lock_guard lock(e.mutex);
    e.stage->set_timing(enabled);
}

void kernel_timing(NativeEngine & engine, std::uint64_t * mm_n, double * mm_ms, double * mm_bytes,
                   std::uint64_t * at_n, double * at_ms, double * at_bytes) {
    auto & e = BatchAccess::impl_of(engine);
    std::lock_guard lock(e.mutex);
    const jfb::engine::KernelTiming t = e.stage->collect_timing();
    *mm_n = t.matmul_launches;
    *mm_ms = t.matmul_ms;
    *mm_bytes = t.matmul_bytes;
    *at_n = t.attention_launches;
    *at_ms = t.attention_ms;
    *at_bytes = t.attention_bytes;
}

}  // namespace detail

const char * backend_name(Backend backend) { return backend == Backend::Cuda ? "cuda" : "cpu"; }

const char * attention_kernel_name(AttentionKernel kernel) {
    switch (kernel) {
    case AttentionKernel::Automatic: return "automatic";
    case AttentionKernel::Unfused: return "unfused";
    case AttentionKernel::Flash: return "flash";
    }
    return "unknown";
}

}  // namespace jetsonfabric::native
