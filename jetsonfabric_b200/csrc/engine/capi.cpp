// extern "C" wrappers of the engine (include/jfb/jfb_engine.h). Exceptions
// never cross the ABI: std::invalid_argument becomes
// JFB_STATUS_INVALID_ARGUMENT, std::bad_alloc JFB_STATUS_OUT_OF_MEMORY, any
// other exception JFB_STATUS_EXECUTION_FAILED, mirroring the reference stage
// executor's error mapping (runtime/adapters/native_stage_executor.cpp:129-139).
#include "jfb/jfb_engine.h"

#include "engine_internal.hpp"
#include "jetsonfabric/native_batch.hpp"
#include "jetsonfabric/native_inference.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <limits>
#include <memory>
#include <new>
#include <stdexcept>
#include <vector>

namespace native = jetsonfabric::native;

struct jfb_engine {
    std::unique_ptr<native::NativeEngine> engine;
    int device = 0;
};

struct jfb_session {
    jfb_engine * owner = nullptr;
    std::unique_ptr<native::NativeSession> session;
};

namespace {

jfb_status make(jfb_status_code code, const char * message) {
    jfb_status s;
    s.code = code;
    std::snprintf(s.message, sizeof(s.message), "%s", message);
    return s;
}

jfb_status ok() { return make(JFB_STATUS_OK, ""); }

template <typename F>
jfb_status guarded(F && body) {
    try {
        body();
        return ok();
    } catch (const std::invalid_argument & e) {
        return make(JFB_STATUS_INVALID_ARGUMENT, e.what());
    } catch (const std::bad_alloc &) {
        return make(JFB_STATUS_OUT_OF_MEMORY, "host allocation failed");
    } catch (const std::exception & e) {
        const char * what = e.what();
        const bool oom = std::strstr(what, "out of memory") != nullptr;
        return make(oom ? JFB_STATUS_OUT_OF_MEMORY : JFB_STATUS_EXECUTION_FAILED, what);
    } catch (...) {
        return make(JFB_STATUS_EXECUTION_FAILED, "unknown native engine failure");
    }
}

// Selects the engine's device for the duration of a call.
struct DeviceScope {
    int previous = -1;
    explicit DeviceScope(int device) {
        if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
        if (previous != device) cudaSetDevice(device);
    }
    ~DeviceScope() {
        if (previous >= 0) cudaSetDevice(previous);
    }
};

void copy_text(char * dst, std::size_t cap, const std::string & src) {
    std::snprintf(dst, cap, "%s", src.c_str());
}

std::uint32_t kernel_code(native::AttentionKernel k) {
    return k == native::AttentionKernel::Unfused ? 1u : k == native::AttentionKernel::Flash ? 2u : 0u;
}

native::AttentionKernel kernel_from(std::uint32_t code) {
    if (code > 2) throw std::invalid_argument("unknown attention kernel");
    return code == 1 ? native::AttentionKernel::Unfused
         : code == 2 ? native::AttentionKernel::Flash
                     : native::AttentionKernel::Automatic;
}

void write_stage_output(const native::StageResult & r, std::size_t hidden, jfb_stage_output * out, float * acts,
                        std::size_t capacity, std::size_t * offset) {
    if (r.has_sampled_token()) {
        if (out != nullptr) {
            out->sampled_token = r.sampled_token;
            out->activation_rows = 0;
        }
        return;
    }
    const std::size_t floats = r.activation.bytes.size() / sizeof(float);
    if (acts == nullptr || *offset + floats > capacity) {
        throw std::invalid_argument("activation output buffer is too small");
    }
    std::memcpy(acts + *offset, r.activation.bytes.data(), r.activation.bytes.size());
    *offset += floats;
    if (out != nullptr) {
        out->sampled_token = -1;
        out->activation_rows = static_cast<std::uint32_t>(floats / std::max<std::size_t>(hidden, 1));
    }
}

std::size_t hidden_of(const jfb_engine * e) { return e->engine->model_info().embedding_length; }

native::ActivationView view_of(const float * data, std::size_t rows, std::size_t hidden) {
    return native::ActivationView{
        std::span<const std::uint8_t>(reinterpret_cast<const std::uint8_t *>(data), rows * hidden * sizeof(float)), rows};
}

std::vector<native::NativeSession *> unwrap(jfb_engine * engine, jfb_session * const * sessions, std::size_t count) {
    if (count > 0 && sessions == nullptr) throw std::invalid_argument("sessions are required");
    std::vector<native::NativeSession *> out;
    out.reserve(count);
    for (std::size_t i = 0; i < count; ++i) {
        if (sessions[i] == nullptr || sessions[i]->owner != engine) {
            throw std::invalid_argument("native session belongs to another engine");
        }
        out.push_back(sessions[i]->session.get());
    }
    return out;
}

}  // namespace

extern "C" {

jfb_status jfb_engine_open(const char * package_path, const jfb_engine_options * options, jfb_engine ** engine) {
    if (package_path == nullptr || options == nullptr || engine == nullptr) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "package path, options and output are required");
    }
    *engine = nullptr;
    return guarded([&] {
        auto e = std::make_unique<jfb_engine>();
        int device = options->device;
        if (device < 0 && cudaGetDevice(&device) != cudaSuccess) throw std::runtime_error("no CUDA device is available");
        e->device = device;
        DeviceScope scope(device);
        native::EngineOptions o;
        if (options->backend > 1) throw std::invalid_argument("unknown compute backend");
        o.backend = options->backend == 1 ? native::Backend::Cuda : native::Backend::Cpu;
        o.prefill_attention_kernel = kernel_from(options->prefill_attention_kernel);
        o.decode_attention_kernel = kernel_from(options->decode_attention_kernel);
        o.threads = options->threads;
        o.layer_start = options->layer_start;
        o.layer_end = options->layer_end;
        e->engine = std::make_unique<native::NativeEngine>(package_path, o);
        *engine = e.release();
    });
}

void jfb_engine_close(jfb_engine * engine) {
    if (engine == nullptr) return;
    DeviceScope scope(engine->device);
    delete engine;
}

jfb_status jfb_engine_info(const jfb_engine * engine, jfb_model_info * info) {
    if (engine == nullptr || info == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "engine and output are required");
    return guarded([&] {
        const native::ModelInfo & m = engine->engine->model_info();
        std::memset(info, 0, sizeof(*info));
        copy_text(info->architecture, sizeof(info->architecture), m.architecture);
        copy_text(info->source_sha256, sizeof(info->source_sha256), m.source_sha256);
        copy_text(info->compute_backend, sizeof(info->compute_backend), m.compute_backend);
        copy_text(info->compute_device, sizeof(info->compute_device), m.compute_device);
        info->layer_count = m.layer_count;
        info->embedding_length = m.embedding_length;
        info->context_length = m.context_length;
        info->vocabulary_size = m.vocabulary_size;
        info->weight_bytes = m.weight_bytes;
        info->total_weight_bytes = m.total_weight_bytes;
        info->tensor_count = m.tensor_count;
        info->resident_layer_start = m.resident_layer_start;
        info->resident_layer_end = m.resident_layer_end;
        info->prefill_attention_kernel = kernel_code(engine->engine->prefill_attention_kernel());
        info->decode_attention_kernel = kernel_code(engine->engine->decode_attention_kernel());
        info->load_time_ms = engine->engine->load_time_ms();
    });
}

jfb_status jfb_session_open(jfb_engine * engine, size_t capacity, jfb_session ** session) {
    if (engine == nullptr || session == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "engine and output are required");
    *session = nullptr;
    return guarded([&] {
        DeviceScope scope(engine->device);
        auto s = std::make_unique<jfb_session>();
        s->owner = engine;
        s->session = engine->engine->create_session(capacity);
        *session = s.release();
    });
}

void jfb_session_close(jfb_session * session) {
    if (session == nullptr) return;
    DeviceScope scope(session->owner->device);
    delete session;
}

size_t jfb_session_capacity(const jfb_session * session) { return session ? session->session->capacity() : 0; }
size_t jfb_session_position(const jfb_session * session) { return session ? session->session->position() : 0; }

jfb_status jfb_session_prefill_tokens(jfb_session * session, const int32_t * tokens, size_t count,
                                      jfb_stage_output * out, float * activations_out, size_t activations_capacity) {
    if (session == nullptr || (tokens == nullptr && count > 0)) return make(JFB_STATUS_INVALID_ARGUMENT, "session and tokens are required");
    return guarded([&] {
        DeviceScope scope(session->owner->device);
        const auto r = session->session->prefill_stage_tokens(std::span<const std::int32_t>(tokens, count));
        std::size_t off = 0;
        write_stage_output(r, hidden_of(session->owner), out, activations_out, activations_capacity, &off);
    });
}

jfb_status jfb_session_prefill_activations(jfb_session * session, const float * activations, size_t rows,
                                           jfb_stage_output * out, float * activations_out,
                                           size_t activations_capacity) {
    if (session == nullptr || (activations == nullptr && rows > 0)) return make(JFB_STATUS_INVALID_ARGUMENT, "session and activations are required");
    return guarded([&] {
        DeviceScope scope(session->owner->device);
        const std::size_t h = hidden_of(session->owner);
        const auto r = session->session->prefill_stage_activations(view_of(activations, rows, h));
        std::size_t off = 0;
        write_stage_output(r, h, out, activations_out, activations_capacity, &off);
    });
}

jfb_status jfb_session_decode_token(jfb_session * session, int32_t token, jfb_stage_output * out,
                                    float * activations_out, size_t activations_capacity) {
    if (session == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "session is required");
    return guarded([&] {
        DeviceScope scope(session->owner->device);
        const auto r = session->session->decode_stage_token(token);
        std::size_t off = 0;
        write_stage_output(r, hidden_of(session->owner), out, activations_out, activations_capacity, &off);
    });
}

jfb_status jfb_session_decode_activation(jfb_session * session, const float * activation, jfb_stage_output * out,
                                         float * activations_out, size_t activations_capacity) {
    if (session == nullptr || activation == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "session and activation are required");
    return guarded([&] {
        DeviceScope scope(session->owner->device);
        const std::size_t h = hidden_of(session->owner);
        const auto r = session->session->decode_stage_activation(view_of(activation, 1, h));
        std::size_t off = 0;
        write_stage_output(r, h, out, activations_out, activations_capacity, &off);
    });
}

jfb_status jfb_session_prefill_greedy(jfb_session * session, const int32_t * tokens, size_t count, int32_t * token) {
    if (session == nullptr || token == nullptr || (tokens == nullptr && count > 0)) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "session, tokens and output are required");
    }
    return guarded([&] {
        DeviceScope scope(session->owner->device);
        *token = session->session->prefill_greedy(std::span<const std::int32_t>(tokens, count));
    });
}

jfb_status jfb_session_decode_greedy(jfb_session * session, int32_t token, int32_t * next) {
    if (session == nullptr || next == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "session and output are required");
    return guarded([&] {
        DeviceScope scope(session->owner->device);
        *next = session->session->decode_greedy(token);
    });
}

jfb_status jfb_session_reset(jfb_session * session) {
    if (session == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "session is required");
    return guarded([&] { native::detail::reset(*session->session); });
}

jfb_status jfb_session_rollback(jfb_session * session, size_t token_count) {
    if (session == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "session is required");
    return guarded([&] { session->session->rollback(token_count); });
}

jfb_status jfb_engine_logits(jfb_engine * engine, const int32_t * tokens, size_t count, float * logits_out,
                             size_t logits_capacity) {
    if (engine == nullptr || logits_out == nullptr || (tokens == nullptr && count > 0)) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine, tokens and output are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const std::vector<float> l = engine->engine->logits(std::span<const std::int32_t>(tokens, count));
        if (l.size() > logits_capacity) throw std::invalid_argument("logits output buffer is too small");
        std::memcpy(logits_out, l.data(), l.size() * sizeof(float));
    });
}

jfb_status jfb_engine_forced_decode_logits(jfb_engine * engine, const int32_t * prompt, size_t prompt_count,
                                           const int32_t * forced, size_t forced_count, float * trace_out,
                                           size_t trace_capacity) {
    if (engine == nullptr || trace_out == nullptr || (prompt == nullptr && prompt_count > 0) ||
        (forced == nullptr && forced_count > 0)) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine, tokens and output are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto trace = engine->engine->forced_decode_logits(std::span<const std::int32_t>(prompt, prompt_count),
                                                                std::span<const std::int32_t>(forced, forced_count));
        std::size_t off = 0;
        for (const auto & row : trace) {
            if (off + row.size() > trace_capacity) throw std::invalid_argument("logit trace buffer is too small");
            std::memcpy(trace_out + off, row.data(), row.size() * sizeof(float));
            off += row.size();
        }
    });
}

jfb_status jfb_engine_generate(jfb_engine * engine, const int32_t * prompt, size_t prompt_count, uint32_t max_tokens,
                               int32_t * tokens_out, jfb_generation_stats * stats) {
    if (engine == nullptr || tokens_out == nullptr || (prompt == nullptr && prompt_count > 0)) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine, prompt and output are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto r = engine->engine->generate(std::span<const std::int32_t>(prompt, prompt_count), max_tokens);
        std::copy(r.sampled_tokens.begin(), r.sampled_tokens.end(), tokens_out);
        if (stats != nullptr) {
            stats->time_to_first_token_ms = r.time_to_first_token_ms;
            stats->inter_token_latency_ms = r.inter_token_latency_ms;
            stats->decode_tokens_per_second = r.decode_tokens_per_second;
            stats->end_to_end_tokens_per_second = r.end_to_end_tokens_per_second;
            stats->kv_cache_bytes = r.buffers.kv_cache_bytes;
            stats->scratch_bytes = r.buffers.prefill_scratch_bytes;
        }
    });
}

void jfb_engine_release_session(jfb_engine * engine) {
    if (engine == nullptr) return;
    DeviceScope scope(engine->device);
    engine->engine->release_session();
}

static jfb_status batch_results(jfb_engine * engine, const std::vector<native::StageResult> & results,
                                int32_t * tokens_out, float * activations_out, size_t activations_capacity) {
    std::size_t off = 0;
    for (std::size_t i = 0; i < results.size(); ++i) {
        if (results[i].has_sampled_token()) {
            if (tokens_out == nullptr) throw std::invalid_argument("token output buffer is required");
            tokens_out[i] = results[i].sampled_token;
        } else {
            write_stage_output(results[i], hidden_of(engine), nullptr, activations_out, activations_capacity, &off);
            if (tokens_out != nullptr) tokens_out[i] = -1;
        }
    }
    return ok();
}

jfb_status jfb_engine_prefill_batch(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                    const int32_t * tokens, const uint32_t * token_counts, int32_t * tokens_out,
                                    float * activations_out, size_t activations_capacity) {
    if (engine == nullptr || tokens == nullptr || token_counts == nullptr) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine, tokens and counts are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto list = unwrap(engine, sessions, count);
        std::vector<std::span<const std::int32_t>> prompts;
        std::size_t off = 0;
        for (std::size_t i = 0; i < count; ++i) {
            prompts.emplace_back(tokens + off, token_counts[i]);
            off += token_counts[i];
        }
        const auto r = native::prefill_stage_batch(*engine->engine, list, prompts);
        batch_results(engine, r, tokens_out, activations_out, activations_capacity);
    });
}

jfb_status jfb_engine_prefill_batch_activations(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                                const float * activations, const uint32_t * row_counts,
                                                int32_t * tokens_out, float * activations_out,
                                                size_t activations_capacity) {
    if (engine == nullptr || activations == nullptr || row_counts == nullptr) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine, activations and counts are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto list = unwrap(engine, sessions, count);
        const std::size_t h = hidden_of(engine);
        std::vector<native::ActivationView> views;
        std::size_t off = 0;
        for (std::size_t i = 0; i < count; ++i) {
            views.push_back(view_of(activations + off * h, row_counts[i], h));
            off += row_counts[i];
        }
        const auto r = native::prefill_stage_batch(*engine->engine, list, views);
        batch_results(engine, r, tokens_out, activations_out, activations_capacity);
    });
}

jfb_status jfb_engine_decode_batch(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                   const int32_t * tokens, int32_t * tokens_out, float * activations_out,
                                   size_t activations_capacity) {
    if (engine == nullptr || tokens == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "engine and tokens are required");
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto list = unwrap(engine, sessions, count);
        const auto r = native::decode_stage_batch(*engine->engine, list, std::span<const std::int32_t>(tokens, count));
        batch_results(engine, r, tokens_out, activations_out, activations_capacity);
    });
}

jfb_status jfb_engine_decode_batch_activations(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                               const float * activations, int32_t * tokens_out,
                                               float * activations_out, size_t activations_capacity) {
    if (engine == nullptr || activations == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "engine and activations are required");
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto list = unwrap(engine, sessions, count);
        const std::size_t h = hidden_of(engine);
        std::vector<native::ActivationView> views;
        for (std::size_t i = 0; i < count; ++i) views.push_back(view_of(activations + i * h, 1, h));
        const auto r = native::decode_stage_batch(*engine->engine, list, views);
        batch_results(engine, r, tokens_out, activations_out, activations_capacity);
    });
}

jfb_status jfb_engine_decode_batch_device(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                          const int32_t * tokens_device, int32_t * tokens_out_device) {
    if (engine == nullptr || tokens_device == nullptr || tokens_out_device == nullptr) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine and device token buffers are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto list = unwrap(engine, sessions, count);
        native::detail::decode_batch_device(*engine->engine, list, tokens_device, tokens_out_device);
    });
}

jfb_status jfb_engine_stage_batch_device(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                         int prefill, const uint32_t * row_counts, const int32_t * tokens_device,
                                         const float * activations_device, int32_t * tokens_out_device,
                                         float * activations_out_device) {
    if (engine == nullptr || (prefill && row_counts == nullptr)) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine and, for prefill, row counts are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto list = unwrap(engine, sessions, count);
        native::detail::stage_batch_device(
            *engine->engine, list, prefill != 0,
            prefill ? std::span<const std::uint32_t>(row_counts, count) : std::span<const std::uint32_t>(),
            tokens_device, activations_device, tokens_out_device, activations_out_device);
    });
}

jfb_status jfb_engine_prefill_batch_device(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                           const int32_t * tokens_device, const uint32_t * token_counts,
                                           int32_t * tokens_out_device) {
    if (engine == nullptr || tokens_device == nullptr || token_counts == nullptr || tokens_out_device == nullptr) {
        return make(JFB_STATUS_INVALID_ARGUMENT, "engine, device tokens and counts are required");
    }
    return guarded([&] {
        DeviceScope scope(engine->device);
        const auto list = unwrap(engine, sessions, count);
        native::detail::prefill_batch_device(*engine->engine, list, tokens_device,
                                             std::span<const std::uint32_t>(token_counts, count), tokens_out_device);
    });
}

jfb_status jfb_engine_synchronize(jfb_engine * engine) {
    if (engine == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "engine is required");
    return guarded([&] {
        DeviceScope scope(engine->device);
        native::detail::synchronize(*engine->engine);
    });
}

jfb_status jfb_engine_set_kernel_timing(jfb_engine * engine, int enabled) {
    if (engine == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "engine is required");
    return guarded([&] { native::detail::set_kernel_timing(*engine->engine, enabled != 0); });
}

jfb_status jfb_engine_kernel_timing(jfb_engine * engine, jfb_kernel_timing * timing) {
    if (engine == nullptr || timing == nullptr) return make(JFB_STATUS_INVALID_ARGUMENT, "engine and output are required");
    return guarded([&] {
        DeviceScope scope(engine->device);
        native::detail::kernel_timing(*engine->engine, &timing->matmul_launches, &timing->matmul_ms,
                                      &timing->matmul_bytes, &timing->attention_launches, &timing->attention_ms,
                                      &timing->attention_bytes);
    });
}

void * jfb_engine_stream(jfb_engine * engine) {
    return engine == nullptr ? nullptr : native::detail::stream(*engine->engine);
}

uint64_t jfb_engine_last_launch_count(const jfb_engine * engine) {
    return engine == nullptr ? 0 : native::detail::last_launch_count(*engine->engine);
}

}  // extern "C"
