// Engine entry points that the C ABI needs but the reference C++ API has no
// member for: device-resident batched passes (used by the benchmark's
// device-timed loop) and engine introspection.
#pragma once

#include "jetsonfabric/native_inference.hpp"

#include <cstdint>
#include <span>

namespace jetsonfabric::native::detail {

// Decode one token for every session; tokens are read from and greedy tokens
// written to device memory; returns without synchronising.
void decode_batch_device(NativeEngine & engine, std::span<NativeSession * const> sessions,
                         const std::int32_t * tokens_device, std::int32_t * tokens_out_device);
// Prefill every session from concatenated device-resident prompts.
void prefill_batch_device(NativeEngine & engine, std::span<NativeSession * const> sessions,
                          const std::int32_t * tokens_device, std::span<const std::uint32_t> counts,
                          std::int32_t * tokens_out_device);
// Device-resident pass of any stage (tokens or activations in, tokens or
// activations out, all device memory); returns without synchronising.
void stage_batch_device(NativeEngine & engine, std::span<NativeSession * const> sessions, bool prefill,
                        std::span<const std::uint32_t> counts, const std::int32_t * tokens_device,
                        const float * activations_device, std::int32_t * tokens_out_device,
                        float * activations_out_device);
void synchronize(NativeEngine & engine);
void * stream(NativeEngine & engine);
std::uint64_t last_launch_count(const NativeEngine & engine);
std::uint64_t scratch_bytes(const NativeEngine & engine);
std::uint64_t kv_cache_bytes(const NativeSession & session);
void reset(NativeSession & session);
void set_kernel_timing(NativeEngine & engine, bool enabled);
// matmul launches, ms, bytes, attention launches, ms, bytes of the last pass
void kernel_timing(NativeEngine & engine, std::uint64_t * mm_n, double * mm_ms, double * mm_bytes,
                   std::uint64_t * at_n, double * at_ms, double * at_bytes);

}  // namespace jetsonfabric::native::detail
