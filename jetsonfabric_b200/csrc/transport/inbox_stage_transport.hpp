// In-box StageTransport for the reference runtime: stage operations between
// processes on one host as Stagewire v2 frames through the shared-memory
// frame channel of jfb/jfb_stagewire.h, registered beside the HTTP transports
// of runtime/transport/builtin_stage_transports.cpp.
//
// This file is written against the reference runtime's own headers
// (transport/stage_transport.hpp, transport/stage_transport_factory.hpp,
// pipeline_parallel/stage_worker.hpp, protocol/stage.hpp) and is compiled
// inside that tree; it links libjfb.so for the channel.
//
//   - InboxStageTransport::invoke keeps HTTPStageTransport::invoke's contract
//     (http_stage_transport.cpp:481-599): the request frame from
//     protocol::encode_stage_request_frame, the cluster token required and
//     sent with it, a JSON error body mapped to its status and code, the
//     response frame decoded with protocol::decode_stage_response, a
//     different acknowledged operation refused, a response error or a non-2xx
//     status returned as a stage error, and any failure on the way returned
//     as 502 runtime_stage_transport_failed. A stage is reached through its
//     `runtime_url`, which names the channel: "inbox://<channel>".
//   - InboxStageServer answers on one channel the way RuntimeService::run_stage
//     (engine/runtime_service.cpp:615-662) answers on the runtime's HTTP
//     port: operation and request decoded and validated, close/rollback/execute
//     dispatched to a pipeline_parallel::StageWorker, an error response frame
//     with the request's identity on failure, and the reference's 401
//     runtime_auth_failed body when the token does not match.
#pragma once

#include "jfb/jfb_stagewire.h"
#include "pipeline_parallel/stage_worker.hpp"
#include "transport/stage_transport.hpp"
#include "transport/stage_transport_factory.hpp"

#include <chrono>
#include <memory>
#include <stop_token>
#include <string>

namespace jetsonfabric::runtime::transport {

// Registration name, for Config::stage_transport.
inline constexpr const char * kInboxStageTransport = "inbox_frames_v1";
// runtime_url scheme of a stage served on this host.
inline constexpr const char * kInboxUrlScheme = "inbox://";

class InboxStageTransport final : public StageTransport {
public:
    explicit InboxStageTransport(std::string cluster_token,
                                 std::chrono::milliseconds timeout = std::chrono::minutes(5));
    ~InboxStageTransport() override;

    void shutdown() const override;
    pipeline_parallel::StageRunResult invoke(const protocol::GenerationStage & stage,
                                             const protocol::StageRequest & request,
                                             pipeline_parallel::StageOperation operation) const override;

private:
    class Impl;
    std::unique_ptr<Impl> impl_;
};

// Adds kInboxStageTransport to `factory`, built from Config::cluster_token.
void register_inbox_stage_transport(StageTransportFactory & factory);

class InboxStageServer {
public:
    // Creates channel `channel` (capacity 0: the largest Stagewire v2 frame).
    InboxStageServer(std::string channel, std::string cluster_token, const pipeline_parallel::StageWorker & worker,
                     std::uint64_t capacity = 0);
    ~InboxStageServer();
    InboxStageServer(const InboxStageServer &) = delete;
    InboxStageServer & operator=(const InboxStageServer &) = delete;

    // Answers one request if one arrives within `wait`; returns whether one did.
    bool serve_one(std::chrono::milliseconds wait);
    // Answers requests until `stop` is requested.
    void serve(std::stop_token stop);

private:
    std::string name_;
    std::string token_;
    const pipeline_parallel::StageWorker & worker_;
    jfb_frame_channel * channel_ = nullptr;
};

}  // namespace jetsonfabric::runtime::transport
