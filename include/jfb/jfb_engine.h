/*
 * C ABI of the native Qwen2 stage engine: the boundary an FFI caller (Python
 * ctypes here, a cgo stub in the Go node) binds instead of the C++ API.
 *
 * Each entry point wraps one member of the reference C++ API
 * (runtime/engines/native/include/jetsonfabric/native_inference.hpp) and is
 * cited below; errors come back as jfb_status with the exception mapping of
 * the reference stage executor (runtime/adapters/native_stage_executor.cpp:129-139):
 * std::invalid_argument -> JFB_STATUS_INVALID_ARGUMENT, any other failure ->
 * JFB_STATUS_EXECUTION_FAILED (or JFB_STATUS_CUDA_ERROR / OUT_OF_MEMORY).
 * Buffers are host memory unless a name ends in _device.
 *
 * Thread safety: calls on one engine (and its sessions) are serialised by an
 * engine-wide lock, like NativeStageExecutor's mutex (native_stage_executor.cpp:111).
 */
#ifndef JFB_ENGINE_H
#define JFB_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "jfb/jfb_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct jfb_engine jfb_engine;
typedef struct jfb_session jfb_session;

/* EngineOptions (native_inference.hpp:23-30) plus the CUDA device ordinal. */
typedef struct jfb_engine_options {
    uint32_t backend;                  /* 0 = cpu (rejected), 1 = cuda */
    uint32_t prefill_attention_kernel; /* 0 automatic, 1 unfused, 2 flash */
    uint32_t decode_attention_kernel;
    int32_t threads;
    uint32_t layer_start;
    uint32_t layer_end;                /* UINT32_MAX = through the last layer */
    int32_t device;                    /* CUDA device ordinal, -1 = current */
} jfb_engine_options;

/* ModelInfo (native_inference.hpp:32-46). */
typedef struct jfb_model_info {
    char architecture[32];
    char source_sha256[72];
    char compute_backend[32];
    char compute_device[128];
    uint32_t layer_count;
    uint32_t embedding_length;
    uint32_t context_length;
    uint32_t vocabulary_size;
    uint64_t weight_bytes;
    uint64_t total_weight_bytes;
    uint64_t tensor_count;
    uint32_t resident_layer_start;
    uint32_t resident_layer_end;
    uint32_t prefill_attention_kernel;
    uint32_t decode_attention_kernel;
    double load_time_ms;
} jfb_model_info;

/* GenerationResult timings (native_inference.hpp:89-97). */
typedef struct jfb_generation_stats {
    double time_to_first_token_ms;
    double inter_token_latency_ms;
    double decode_tokens_per_second;
    double end_to_end_tokens_per_second;
    uint64_t kv_cache_bytes;
    uint64_t scratch_bytes;
} jfb_generation_stats;

/* Stage output of one session: the greedy token (final stage) or f32
 * activations [rows, hidden] written to the caller's buffer. */
typedef struct jfb_stage_output {
    int32_t sampled_token;        /* -1 when the stage returns activations */
    uint32_t activation_rows;     /* rows written to activations */
} jfb_stage_output;

/* NativeEngine(package_path, EngineOptions) (native_inference.hpp:128-129). */
jfb_status jfb_engine_open(const char * package_path, const jfb_engine_options * options, jfb_engine ** engine);
void jfb_engine_close(jfb_engine * engine);
/* model_info(), prefill/decode_attention_kernel(), load_time_ms(). */
jfb_status jfb_engine_info(const jfb_engine * engine, jfb_model_info * info);

/* create_session(capacity) (native_inference.hpp:143). */
jfb_status jfb_session_open(jfb_engine * engine, size_t capacity, jfb_session ** session);
void jfb_session_close(jfb_session * session);
size_t jfb_session_capacity(const jfb_session * session);
size_t jfb_session_position(const jfb_session * session);

/* NativeSession::prefill_stage_tokens / prefill_stage_activations /
 * decode_stage_token / decode_stage_activation (native_inference.hpp:111-114).
 * activations_out must hold rows*hidden floats on intermediate stages. */
jfb_status jfb_session_prefill_tokens(jfb_session * session, const int32_t * tokens, size_t count,
                                      jfb_stage_output * out, float * activations_out, size_t activations_capacity);
jfb_status jfb_session_prefill_activations(jfb_session * session, const float * activations, size_t rows,
                                           jfb_stage_output * out, float * activations_out,
                                           size_t activations_capacity);
jfb_status jfb_session_decode_token(jfb_session * session, int32_t token, jfb_stage_output * out,
                                    float * activations_out, size_t activations_capacity);
jfb_status jfb_session_decode_activation(jfb_session * session, const float * activation, jfb_stage_output * out,
                                         float * activations_out, size_t activations_capacity);
/* NativeSession::prefill_greedy / decode_greedy (full model only). */
jfb_status jfb_session_prefill_greedy(jfb_session * session, const int32_t * tokens, size_t count, int32_t * token);
jfb_status jfb_session_decode_greedy(jfb_session * session, int32_t token, int32_t * next);
/* InferenceSession::reset (runtime/engines/native/src/model_architecture.hpp:33):
 * position back to 0 so the session's KV cache can serve a new prompt. */
jfb_status jfb_session_reset(jfb_session * session);
/* NativeSession::rollback (native_inference.hpp:115). */
jfb_status jfb_session_rollback(jfb_session * session, size_t token_count);

/* NativeEngine::logits (native_inference.hpp:145): logits_out holds vocabulary floats. */
jfb_status jfb_engine_logits(jfb_engine * engine, const int32_t * tokens, size_t count, float * logits_out,
                             size_t logits_capacity);
/* NativeEngine::forced_decode_logits (146-149): trace_out holds
 * (forced_count + 1) * vocabulary floats. */
jfb_status jfb_engine_forced_decode_logits(jfb_engine * engine, const int32_t * prompt, size_t prompt_count,
                                           const int32_t * forced, size_t forced_count, float * trace_out,
                                           size_t trace_capacity);
/* NativeEngine::generate (150-153): tokens_out holds max_tokens tokens. */
jfb_status jfb_engine_generate(jfb_engine * engine, const int32_t * prompt, size_t prompt_count, uint32_t max_tokens,
                               int32_t * tokens_out, jfb_generation_stats * stats);
/* NativeEngine::release_session (154). */
void jfb_engine_release_session(jfb_engine * engine);

/* Batched stage passes over several sessions of one engine (continuous
 * batching; the reference Executor::execute_batch contract,
 * runtime/inference/executor.hpp:20-29). Results in session order.
 * Prefill: tokens are the prompts concatenated, counts[i] their lengths;
 * activations likewise concatenated [sum rows, hidden]. */
jfb_status jfb_engine_prefill_batch(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                    const int32_t * tokens, const uint32_t * token_counts, int32_t * tokens_out,
                                    float * activations_out, size_t activations_capacity);
jfb_status jfb_engine_prefill_batch_activations(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                                const float * activations, const uint32_t * row_counts,
                                                int32_t * tokens_out, float * activations_out,
                                                size_t activations_capacity);
jfb_status jfb_engine_decode_batch(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                   const int32_t * tokens, int32_t * tokens_out, float * activations_out,
                                   size_t activations_capacity);
jfb_status jfb_engine_decode_batch_activations(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                               const float * activations, int32_t * tokens_out,
                                               float * activations_out, size_t activations_capacity);

/* Device-resident decode step for a full-model engine: the input tokens are
 * read from and the greedy tokens written to device memory, nothing is copied
 * to the host and the call returns without waiting for the GPU (use
 * jfb_engine_synchronize). Positions advance as for jfb_engine_decode_batch. */
jfb_status jfb_engine_decode_batch_device(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                          const int32_t * tokens_device, int32_t * tokens_out_device);
/* Device-resident prefill for a full-model engine (tokens_device holds the
 * concatenated prompts; token_counts is host memory). */
jfb_status jfb_engine_prefill_batch_device(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                           const int32_t * tokens_device, const uint32_t * token_counts,
                                           int32_t * tokens_out_device);
/* Device-resident pass of one pipeline stage over a batch of sessions. The
 * first stage reads token ids (tokens_device), later stages f32 activations
 * [rows][hidden] (activations_device); the last stage writes one greedy token
 * per session (tokens_out_device), the others f32 activations [rows][hidden]
 * (activations_out_device). All four are device memory. prefill selects the
 * prompt rows of each session (row_counts, host memory) or one decode row per
 * session. Nothing is copied to the host and the call returns without waiting
 * for the GPU. The engine counterpart of one Stagewire hop of the reference
 * pipeline (native_stage_executor.cpp:143-180 per session). */
jfb_status jfb_engine_stage_batch_device(jfb_engine * engine, jfb_session * const * sessions, size_t count,
                                         int prefill, const uint32_t * row_counts, const int32_t * tokens_device,
                                         const float * activations_device, int32_t * tokens_out_device,
                                         float * activations_out_device);
jfb_status jfb_engine_synchronize(jfb_engine * engine);

/* Device time and algorithmic bytes of the matmul and attention launches of
 * the engine's last pass, recorded with CUDA events on the engine stream when
 * timing is enabled (no counterpart in the reference; used for rooflines). */
typedef struct jfb_kernel_timing {
    uint64_t matmul_launches;
    double matmul_ms;
    double matmul_bytes;
    uint64_t attention_launches;
    double attention_ms;
    double attention_bytes;
} jfb_kernel_timing;
jfb_status jfb_engine_set_kernel_timing(jfb_engine * engine, int enabled);
jfb_status jfb_engine_kernel_timing(jfb_engine * engine, jfb_kernel_timing * timing);
/* The engine's CUDA stream (cudaStream_t) and the kernels its last pass launched. */
void * jfb_engine_stream(jfb_engine * engine);
uint64_t jfb_engine_last_launch_count(const jfb_engine * engine);

#ifdef __cplusplus
}
#endif

#endif
