// In-box StageTransport and its server (see inbox_stage_transport.hpp).
#include "inbox_stage_transport.hpp"

#include "protocol/stage.hpp"
#include "protocol/stage_control.hpp"

#include <nlohmann/json.hpp>

#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <utility>

namespace jetsonfabric::runtime::transport {
namespace {

using pipeline_parallel::StageOperation;
using pipeline_parallel::StageRunResult;

// Request preamble: "JFTK", the token's length (u32, big-endian), the token.
// The frame follows it unchanged.
constexpr char kPreambleMagic[4] = {'J', 'F', 'T', 'K'};

std::string preamble(const std::string & token) {
    std::string out(kPreambleMagic, 4);
    const auto n = static_cast<std::uint32_t>(token.size());
    for (int shift = 24; shift >= 0; shift -= 8) out.push_back(static_cast<char>((n >> shift) & 0xffU));
    out += token;
    return out;
}

StageRunResult stage_error(std::string status, std::string code, std::string message) {
    StageRunResult result;
    result.status = std::move(status);
    result.error_code = std::move(code);
    result.error_message = std::move(message);
    return result;
}

std::string status_text(int code) {
    static const std::map<int, const char *> reasons = {
        {200, "OK"}, {400, "Bad Request"}, {401, "Unauthorized"}, {404, "Not Found"}, {409, "Conflict"},
        {413, "Payload Too Large"}, {429, "Too Many Requests"}, {499, "Client Closed Request"},
        {500, "Internal Server Error"}, {502, "Bad Gateway"}, {503, "Service Unavailable"}, {504, "Gateway Timeout"},
    };
    const auto it = reasons.find(code);
    return it == reasons.end() ? std::to_string(code) : std::to_string(code) + " " + it->second;
}

int status_code(const std::string & status) {
    try {
        return std::stoi(status);
    } catch (const std::exception &) {
        return 500;
    }
}

const char * operation_name(StageOperation op) {
    return op == StageOperation::CloseSession      ? protocol::kStageOperationCloseSession
           : op == StageOperation::RollbackSession ? protocol::kStageOperationRollbackSession
                                                   : protocol::kStageOperationExecute;
}

std::string channel_of(const std::string & url) {
    const std::string scheme = kInboxUrlScheme;
    if (url.compare(0, scheme.size(), scheme) != 0 || url.size() == scheme.size()) {
        throw std::invalid_argument("in-box stage runtime_url must be inbox://<channel>, got \"" + url + "\"");
    }
    return url.substr(scheme.size());
}

bool constant_time_equal(const std::string & left, const std::string & right) {
    const std::size_t n = std::max(left.size(), right.size());
    unsigned char diff = left.size() == right.size() ? 0 : 1;
    for (std::size_t i = 0; i < n; ++i) {
        const unsigned char a = i < left.size() ? static_cast<unsigned char>(left[i]) : 0;
        const unsigned char b = i < right.size() ? static_cast<unsigned char>(right[i]) : 0;
        diff |= a ^ b;
    }
    return diff == 0;
}

std::string json_error_body(const std::string & code, const std::string & message) {
    return "{\"error\":\"" + protocol::json_escape(code) + "\",\"message\":\"" + protocol::json_escape(message) +
           "\"}";
}

// The identity fields of an error response (RuntimeService::run_stage's
// error frame carries the request's identity, shape and bytes_in).
protocol::StageResponse error_response_for(const protocol::StageRequest & request) {
    protocol::StageResponse r;
    r.session_id = request.session_id;
    r.request_id = request.request_id;
    r.model_id = request.model_id;
    r.deployment_id = request.deployment_id;
    r.deployment_epoch = request.deployment_epoch;
    r.model_sha256 = request.model_sha256;
    r.phase = request.phase;
    r.decode_step = request.decode_step;
    r.stage_index = request.stage_index;
    r.stage_count = request.stage_count;
    r.node_name = request.node_name;
    r.layer_start = request.layer_start;
    r.layer_end = request.layer_end;
    r.payload_kind = request.payload_kind;
    r.encoding = request.encoding;
    r.dtype = request.dtype;
    r.shape = request.shape;
    r.byte_order = request.byte_order;
    r.layout = request.layout;
    r.bytes_in = static_cast<std::int64_t>(request.payload.size());
    return r;
}

void check(jfb_status st) {
    if (st.code != JFB_STATUS_OK) throw std::runtime_error(st.message);
}

}  // namespace

// ---- caller side ------------------------------------------------------------

class InboxStageTransport::Impl {
public:
    struct Connection {
        std::mutex mutex;
        jfb_frame_channel * channel = nullptr;
        ~Connection() { jfb_frame_channel_close(channel); }
    };

    Impl(std::string token, std::chrono::milliseconds timeout) : token_(std::move(token)), timeout_(timeout) {}

    const std::string & token() const { return token_; }
    std::uint32_t timeout_ms() const {
        const auto ms = timeout_.count();
        return ms <= 0 ? 0u : ms > 0x7fffffff ? 0x7fffffffu : static_cast<std::uint32_t>(ms);
    }

    std::shared_ptr<Connection> connection_for(const std::string & name) const {
        const std::lock_guard lock(mutex_);
        auto & slot = connections_[name];
        if (!slot) slot = std::make_shared<Connection>();
        return slot;
    }

    void shutdown() const {
        const std::lock_guard lock(mutex_);
        connections_.clear();
    }

private:
    std::string token_;
    std::chrono::milliseconds timeout_;
    mutable std::mutex mutex_;
    mutable std::map<std::string, std::shared_ptr<Connection>> connections_;
};

InboxStageTransport::InboxStageTransport(std::string cluster_token, std::chrono::milliseconds timeout)
    : impl_(std::make_unique<Impl>(std::move(cluster_token), timeout)) {}

InboxStageTransport::~InboxStageTransport() = default;

void InboxStageTransport::shutdown() const { impl_->shutdown(); }

StageRunResult InboxStageTransport::invoke(const protocol::GenerationStage & stage,
                                           const protocol::StageRequest & request, StageOperation operation) const {
    if (impl_->token().empty()) {
        return stage_error("503 Service Unavailable", "cluster_auth_unconfigured",
                           "runtime peer transport requires JETSONFABRIC_CLUSTER_TOKEN");
    }
    try {
        const auto call_start = std::chrono::steady_clock::now();
        std::string name;
        try {
            name = channel_of(stage.runtime_url);
        } catch (const std::invalid_argument & e) {
            return stage_error("400 Bad Request", "runtime_endpoint_unsupported", e.what());
        }
        const std::string op = operation_name(operation);
        const protocol::EncodedStageFrameView body = protocol::encode_stage_request_frame(request, op);
        const std::string head = preamble(impl_->token()) + body.prefix;

        const auto connection = impl_->connection_for(name);
        const std::lock_guard connection_lock(connection->mutex);
        if (connection->channel == nullptr) {
            check(jfb_frame_channel_open(name.c_str(), impl_->timeout_ms(), &connection->channel));
        }
        std::int32_t status = 0, is_frame = 0;
        const std::uint8_t * reply = nullptr;
        std::uint64_t reply_bytes = 0;
        const jfb_status st =
            jfb_frame_channel_call(connection->channel, head.data(), head.size(), body.payload.data(),
                                   body.payload.size(), impl_->timeout_ms(), &status, &is_frame, &reply, &reply_bytes);
        if (st.code != JFB_STATUS_OK) {
            // a closed or silent server: drop the handle so the next call reopens
            jfb_frame_channel_close(connection->channel);
            connection->channel = nullptr;
            throw std::runtime_error(st.message);
        }
        const std::string wire(reinterpret_cast<const char *>(reply), static_cast<std::size_t>(reply_bytes));
        if (!is_frame) {
            std::string code = "runtime_stage_failed";
            std::string message = wire;
            try {
                const nlohmann::json error = nlohmann::json::parse(wire);
                code = error.value("error", code);
                message = error.value("message", message);
            } catch (const nlohmann::json::exception &) {
            }
            return stage_error(status_text(status), code, message);
        }
        protocol::StageResponse decoded = protocol::decode_stage_response(wire);
        if (decoded.operation != op) {
            return stage_error("502 Bad Gateway", "runtime_stage_operation_mismatch",
                               "peer runtime acknowledged a different stage operation");
        }
        if (status < 200 || status >= 300 || !decoded.error.empty()) {
            return stage_error(status_text(status), decoded.error.empty() ? "runtime_stage_failed" : decoded.error,
                               decoded.message);
        }
        StageRunResult result;
        result.ok = true;
        result.status = status_text(status);
        result.response = std::move(decoded);
        result.remote_call_us =
            std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - call_start)
                .count();
        return result;
    } catch (const std::exception & error) {
        return stage_error("502 Bad Gateway", "runtime_stage_transport_failed", error.what());
    }
}

void register_inbox_stage_transport(StageTransportFactory & factory) {
    factory.register_transport(kInboxStageTransport, [](const Config & config) {
        return std::make_shared<InboxStageTransport>(config.cluster_token);
    });
}

// ---- server side --------------------------------------------------------------

InboxStageServer::InboxStageServer(std::string channel, std::string cluster_token,
                                   const pipeline_parallel::StageWorker & worker, std::uint64_t capacity)
    : name_(std::move(channel)), token_(std::move(cluster_token)), worker_(worker) {
    check(jfb_frame_channel_create(name_.c_str(), capacity, &channel_));
}

InboxStageServer::~InboxStageServer() { jfb_frame_channel_close(channel_); }

bool InboxStageServer::serve_one(std::chrono::milliseconds wait) {
    const std::uint8_t * frame = nullptr;
    std::uint64_t n = 0;
    const auto ms = static_cast<std::uint32_t>(std::max<std::int64_t>(0, std::min<std::int64_t>(wait.count(), 0x7fffffff)));
    const jfb_status st = jfb_frame_channel_receive(channel_, ms, &frame, &n);
    if (st.code == JFB_STATUS_TIMEOUT) return false;
    check(st);

    const auto reply_json = [&](int status, const std::string & code, const std::string & message) {
        const std::string body = json_error_body(code, message);
        check(jfb_frame_channel_reply(channel_, status, 0, body.data(), body.size(), nullptr, 0));
    };
    // a response the codec refuses to encode is answered as a 502 error body,
    // so the caller never waits for a reply that will not come
    const auto reply_frame = [&](int status, protocol::StageResponse response) {
        protocol::EncodedStageFrame out;
        try {
            out = protocol::encode_stage_response_frame(std::move(response));
        } catch (const std::exception & error) {
            reply_json(502, "invalid_stage_response", error.what());
            return;
        }
        check(jfb_frame_channel_reply(channel_, status, 1, out.prefix.data(), out.prefix.size(), out.payload.data(),
                                      out.payload.size()));
    };

    const char * bytes = reinterpret_cast<const char *>(frame);
    if (n < 8 || std::memcmp(bytes, kPreambleMagic, 4) != 0) {
        reply_json(400, "invalid_stage_request", "in-box stage request without its preamble");
        return true;
    }
    std::uint32_t token_bytes = 0;
    for (int i = 4; i < 8; ++i) token_bytes = (token_bytes << 8) | static_cast<unsigned char>(bytes[i]);
    if (token_bytes > n - 8) {
        reply_json(400, "invalid_stage_request", "in-box stage request preamble is truncated");
        return true;
    }
    if (!token_.empty() && !constant_time_equal(std::string(bytes + 8, token_bytes), token_)) {
        reply_json(401, "runtime_auth_failed", "runtime writes require the configured cluster token");
        return true;
    }
    const std::string body(bytes + 8 + token_bytes, static_cast<std::size_t>(n - 8 - token_bytes));

    std::string operation;
    protocol::StageRequest request;
    try {
        operation = protocol::decode_stage_operation(body);
        request = protocol::decode_stage_request(body);
        protocol::validate_stage_operation(operation, request.rollback_tokens);
    } catch (const std::exception & error) {
        reply_json(400, "invalid_stage_request", error.what());
        return true;
    }
    protocol::StageResponse failure = error_response_for(request);
    StageRunResult result;
    try {
        result = operation == protocol::kStageOperationCloseSession       ? worker_.close_session(request)
                 : operation == protocol::kStageOperationRollbackSession ? worker_.rollback_session(request)
                                                                          : worker_.run(std::move(request));
    } catch (const std::exception & error) {
        result = stage_error("502 Bad Gateway", "runtime_stage_failed", error.what());
    }
    if (!result.ok) {
        failure.operation = operation;
        failure.error = result.error_code;
        failure.message = result.error_message;
        reply_frame(status_code(result.status), std::move(failure));
        return true;
    }
    protocol::StageResponse response = std::move(result.response);
    response.operation = operation;
    reply_frame(200, std::move(response));
    return true;
}

void InboxStageServer::serve(std::stop_token stop) {
    while (!stop.stop_requested()) serve_one(std::chrono::milliseconds(100));
}

}  // namespace jetsonfabric::runtime::transport
