// Multi-session (continuous-batching) entry points of the native engine.
//
// The reference native executor inherits the sequential execute_batch default
// (runtime/inference/executor.hpp:20-29) and its config rejects a decode batch
// size other than 1 for the native engine (runtime/worker/config.cpp:159-162).
// These functions run several sessions of one engine through a single batched
// stage pass, with the semantics of the llama.cpp stage adapter's batched
// decode (runtime/adapters/llama_cpp_stage_adapter.cpp:703-810): one step per
// session, duplicate sessions rejected. Results come back in input order.
#pragma once

#include "jetsonfabric/native_inference.hpp"

#include <cstdint>
#include <span>
#include <vector>

namespace jetsonfabric::native {

// First stage: one prompt per session (prefill at position 0).
std::vector<StageResult> prefill_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                             std::span<const std::span<const std::int32_t>> prompts);
// Later stages: one activation block per session.
std::vector<StageResult> prefill_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                             std::span<const ActivationView> activations);
// First stage: one decode token per session.
std::vector<StageResult> decode_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                            std::span<const std::int32_t> tokens);
// Later stages: one activation row per session.
std::vector<StageResult> decode_stage_batch(NativeEngine & engine, std::span<NativeSession * const> sessions,
                                            std::span<const ActivationView> activations);

}  // namespace jetsonfabric::native
