// Drives the in-box StageTransport with the reference runtime's own pieces
// (test infrastructure; built by oracle/ref_transport/build.py into
// oracle/_ref/ only where the reference sources are present).
//
// The generation loop is the reference's pipeline_parallel::GenerationRunner
// (runtime/pipeline_parallel/generation_runner.cpp), each stage answers
// through the reference's pipeline_parallel::StageWorker with the reference's
// F16 activation codec, and every frame is encoded and decoded by the
// reference's protocol/stage.cpp. Only the transport between them is this
// repository's (jetsonfabric_b200/csrc/transport/).
//
//   serve <channel> <token> <idle_ms> synthetic <index> <count> <start> <end>
//   serve <channel> <token> <idle_ms> native <package> <index> <count> <start> <end> <ctx>
//       answers on <channel> until no request arrives for idle_ms; the
//       synthetic executor is the reference's SyntheticActivationExecutor, the
//       native one the reference's NativeStageExecutor over libjfb.so (CUDA).
//   generate <token> <max_tokens> <prompt> <session> <channel:start:end>...
//       one GenerationRunner pass over the listed stages through the
//       transport, printed as one JSON line.
//   local <max_tokens> <prompt> <session> <start:end>...
//       the same pass with synthetic StageWorkers called in-process.
//   errors
//       the transport's refusal paths, in-process servers on threads.
//   golden
//       frames from the reference's Stagewire encoder, one hex JSON line each.
//   decode
//       hex frames on stdin through the reference's request decoder.
#include "activation/activation_codec_factory.hpp"
#include "adapters/native_stage_executor.hpp"
#include "inbox_stage_transport.hpp"
#include "pipeline_parallel/generation_runner.hpp"
#include "pipeline_parallel/synthetic_activation_executor.hpp"
#include "protocol/stage.hpp"
#include "protocol/stage_control.hpp"
#include "worker/config.hpp"

#include <charconv>
#include <chrono>
#include <cstdint>
#include <iostream>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <string_view>
#include <thread>
#include <vector>

namespace {

namespace rt = jetsonfabric::runtime;
namespace pp = jetsonfabric::runtime::pipeline_parallel;
namespace tr = jetsonfabric::runtime::transport;
namespace native = jetsonfabric::native;

constexpr const char * kModel = "jfb-transport-test";

// Prompts are decimal token ids separated by spaces; token t is spelled "<t>".
class IdTokens final : public rt::tokenization::Tokenizer {
public:
    std::vector<std::int32_t> tokenize(std::string_view text) const override {
        std::vector<std::int32_t> out;
        std::size_t i = 0;
        while (i < text.size()) {
            while (i < text.size() && text[i] == ' ') ++i;
            if (i == text.size()) break;
            std::int32_t v = 0;
            const auto r = std::from_chars(text.data() + i, text.data() + text.size(), v);
            if (r.ec != std::errc()) throw std::invalid_argument("id tokenizer: prompt must be decimal token ids");
            out.push_back(v);
            i = static_cast<std::size_t>(r.ptr - text.data());
        }
        if (out.empty()) throw std::invalid_argument("id tokenizer: empty prompt");
        return out;
    }
    std::string token_piece(std::int32_t token) const override { return "<" + std::to_string(token) + ">"; }
    bool is_end_token(std::int32_t) const override { return false; }
};

std::shared_ptr<const rt::activation::ActivationCodec> f16_codec() {
    return rt::activation::make_default_activation_codec_factory()->create_codec("f16");
}

std::vector<std::string> split(const std::string & s, char sep) {
    std::vector<std::string> out;
    std::stringstream in(s);
    std::string part;
    while (std::getline(in, part, sep)) out.push_back(part);
    return out;
}

std::string json_string(const std::string & s) { return "\"" + rt::protocol::json_escape(s) + "\""; }

void print_result(const pp::GenerationResult & r) {
    std::cout << "{\"ok\":" << (r.ok ? "true" : "false") << ",\"status\":" << json_string(r.status)
              << ",\"error_code\":" << json_string(r.error_code) << ",\"error_message\":" << json_string(r.error_message)
              << ",\"tokens\":[";
    for (std::size_t i = 0; i < r.sampled_tokens.size(); ++i) std::cout << (i ? "," : "") << r.sampled_tokens[i];
    std::cout << "],\"stage_calls\":" << r.stage_calls << ",\"remote_stage_calls\":" << r.remote_stage_calls
              << ",\"bytes_in\":" << r.bytes_in << ",\"bytes_out\":" << r.bytes_out << "}\n";
}

rt::protocol::GenerationRequest generation_request(const std::string & session, const std::string & prompt,
                                                    int max_tokens) {
    rt::protocol::GenerationRequest req;
    req.request_id = session + "-request";
    req.session_id = session;
    req.model_id = kModel;
    req.prompt = prompt;
    req.max_tokens = max_tokens;
    return req;
}

pp::GenerationResult run_generation(const pp::StageInvoker & invoke, const rt::protocol::GenerationRequest & req) {
    const pp::GenerationRunner runner(invoke);
    return runner.run(req, [](const pp::GenerationToken &) { return true; });
}

int serve(int argc, char ** argv) {
    if (argc < 6) throw std::invalid_argument("serve: missing arguments");
    const std::string channel = argv[2], token = argv[3];
    const auto idle = std::chrono::milliseconds(std::stoll(argv[4]));
    const std::string kind = argv[5];
    std::unique_ptr<rt::inference::Executor> executor;
    pp::StageAssignment a;
    int next = 6;
    if (kind == "synthetic") {
        if (argc != 10) throw std::invalid_argument("serve synthetic: <index> <count> <start> <end>");
        executor = std::make_unique<pp::SyntheticActivationExecutor>();
    } else if (kind == "native") {
        if (argc != 12) throw std::invalid_argument("serve native: <package> <index> <count> <start> <end> <ctx>");
        const std::string package = argv[6];
        next = 7;
        const auto start = static_cast<std::uint32_t>(std::stoul(argv[9])), end = static_cast<std::uint32_t>(std::stoul(argv[10]));
        auto engine = std::make_shared<native::NativeEngine>(
            package, native::EngineOptions{.backend = native::Backend::Cuda, .threads = 1, .layer_start = start,
                                           .layer_end = end});
        executor = std::make_unique<rt::adapters::NativeStageExecutor>(rt::adapters::NativeStageConfig{
            .engine = engine, .tokenizer = std::make_shared<IdTokens>(), .ctx_size = std::stoi(argv[11]),
            .position = {.index = std::stoi(argv[7]), .count = std::stoi(argv[8])},
            .layers = {.start = static_cast<int>(start), .end = static_cast<int>(end)}});
    } else {
        throw std::invalid_argument("serve: executor is synthetic or native");
    }
    a.stage_index = std::stoi(argv[next]);
    a.stage_count = std::stoi(argv[next + 1]);
    a.layer_start = std::stoi(argv[next + 2]);
    a.layer_end = std::stoi(argv[next + 3]);
    const pp::StageWorker worker("stage-" + std::to_string(a.stage_index), kModel, a, *executor, f16_codec());
    tr::InboxStageServer server(channel, token, worker);
    std::cout << "serving " << channel << std::endl;
    int served = 0;
    while (server.serve_one(idle)) ++served;
    std::cout << "served " << served << std::endl;
    return 0;
}

std::vector<rt::protocol::GenerationStage> stages_from(int argc, char ** argv, int first, bool with_channel) {
    std::vector<rt::protocol::GenerationStage> stages;
    const int count = argc - first;
    for (int i = first; i < argc; ++i) {
        const auto parts = split(argv[i], ':');
        if (parts.size() != (with_channel ? 3u : 2u)) throw std::invalid_argument("bad stage spec");
        rt::protocol::GenerationStage s;
        s.stage_index = i - first;
        s.stage_count = count;
        s.node_name = "stage-" + std::to_string(s.stage_index);
        s.node_id = s.node_name;
        s.runtime_url = with_channel ? std::string(tr::kInboxUrlScheme) + parts[0] : "";
        s.layer_start = std::stoi(parts[with_channel ? 1 : 0]);
        s.layer_end = std::stoi(parts[with_channel ? 2 : 1]);
        stages.push_back(s);
    }
    return stages;
}

std::shared_ptr<const tr::StageTransport> make_transport(const std::string & token) {
    tr::StageTransportFactory factory;
    tr::register_inbox_stage_transport(factory);
    if (!factory.supports(tr::kInboxStageTransport)) throw std::runtime_error("transport not registered");
    rt::Config config;
    config.stage_transport = tr::kInboxStageTransport;
    config.cluster_token = token;
    return factory.create_transport(config);
}

int generate(int argc, char ** argv) {
    if (argc < 7) throw std::invalid_argument("generate: <token> <max_tokens> <prompt> <session> <stages>...");
    const auto transport = make_transport(argv[2]);
    auto req = generation_request(argv[5], argv[4], std::stoi(argv[3]));
    req.stages = stages_from(argc, argv, 6, true);
    const pp::GenerationResult r = run_generation(
        [&](const rt::protocol::GenerationStage & st, const rt::protocol::StageRequest & rq, pp::StageOperation op) {
            return transport->invoke(st, rq, op);
        },
        req);
    transport->shutdown();
    print_result(r);
    return r.ok ? 0 : 3;
}

int local(int argc, char ** argv) {
    if (argc < 6) throw std::invalid_argument("local: <max_tokens> <prompt> <session> <stages>...");
    auto req = generation_request(argv[4], argv[3], std::stoi(argv[2]));
    req.stages = stages_from(argc, argv, 5, false);
    const pp::SyntheticActivationExecutor executor;
    std::vector<std::unique_ptr<pp::StageWorker>> workers;
    for (const auto & s : req.stages) {
        workers.push_back(std::make_unique<pp::StageWorker>(
            s.node_name, kModel,
            pp::StageAssignment{.stage_index = s.stage_index, .stage_count = s.stage_count,
                                .layer_start = s.layer_start, .layer_end = s.layer_end},
            executor, f16_codec()));
    }
    const pp::GenerationResult r = run_generation(
        [&](const rt::protocol::GenerationStage & st, const rt::protocol::StageRequest & rq, pp::StageOperation op) {
            const pp::StageWorker & w = *workers.at(static_cast<std::size_t>(st.stage_index));
            return op == pp::StageOperation::CloseSession      ? w.close_session(rq)
                   : op == pp::StageOperation::RollbackSession ? w.rollback_session(rq)
                                                               : w.run(rq);
        },
        req);
    print_result(r);
    return r.ok ? 0 : 3;
}

void expect(bool ok, const std::string & what) {
    if (!ok) throw std::runtime_error("errors: " + what);
}

void expect_error(const pp::StageRunResult & r, const std::string & status, const std::string & code,
                  const std::string & where) {
    expect(!r.ok && r.status == status && r.error_code == code,
           where + ": got " + r.status + " " + r.error_code + " (" + r.error_message + ")");
}

int errors() {
    const std::string token = "cluster-secret";
    const pp::SyntheticActivationExecutor executor;
    const pp::StageWorker worker("stage-0", kModel,
                                 pp::StageAssignment{.stage_index = 0, .stage_count = 2, .layer_start = 0,
                                                     .layer_end = 1},
                                 executor, f16_codec());
    const std::string name = "jfb-errors-" + std::to_string(::getpid());
    tr::InboxStageServer server(name, token, worker, 1 << 20);
    std::jthread serving([&](std::stop_token stop) { server.serve(stop); });

    rt::protocol::GenerationStage stage;
    stage.stage_index = 0;
    stage.stage_count = 2;
    stage.node_name = "stage-0";
    stage.runtime_url = std::string(tr::kInboxUrlScheme) + name;
    stage.layer_start = 0;
    stage.layer_end = 1;
    rt::protocol::StageRequest req;
    req.session_id = "s";
    req.request_id = "r";
    req.model_id = kModel;
    req.stage_index = 0;
    req.stage_count = 2;
    req.node_name = "stage-0";
    req.layer_start = 0;
    req.layer_end = 1;
    req.payload_kind = "text";
    req.encoding = "utf-8";
    const std::string prompt = "5 6 7";
    req.payload.assign(prompt.begin(), prompt.end());

    const tr::InboxStageTransport transport(token, std::chrono::milliseconds(2000));
    // a prefill through the channel: the first stage answers an activation
    const auto ok = transport.invoke(stage, req, pp::StageOperation::Execute);
    expect(ok.ok && ok.status == "200 OK" && ok.response.payload_kind == "activation" &&
               ok.response.operation == rt::protocol::kStageOperationExecute,
           "prefill through the channel: " + ok.error_code + " " + ok.error_message);
    // close acknowledged as close
    const auto closed = transport.invoke(stage, req, pp::StageOperation::CloseSession);
    expect(closed.ok && closed.response.operation == rt::protocol::kStageOperationCloseSession, "close_session");
    // the cluster token is required on both sides
    expect_error(tr::InboxStageTransport("", std::chrono::milliseconds(200)).invoke(stage, req,
                                                                                   pp::StageOperation::Execute),
                 "503 Service Unavailable", "cluster_auth_unconfigured", "empty token");
    expect_error(tr::InboxStageTransport("wrong", std::chrono::milliseconds(2000)).invoke(stage, req,
                                                                                         pp::StageOperation::Execute),
                 "401 Unauthorized", "runtime_auth_failed", "wrong token");
    // a stage that is not served in-box, and a channel without a server
    auto http_stage = stage;
    http_stage.runtime_url = "http://127.0.0.1:18080";
    expect_error(transport.invoke(http_stage, req, pp::StageOperation::Execute), "400 Bad Request",
                 "runtime_endpoint_unsupported", "http url");
    auto absent = stage;
    absent.runtime_url = std::string(tr::kInboxUrlScheme) + name + "-absent";
    expect_error(tr::InboxStageTransport(token, std::chrono::milliseconds(100)).invoke(absent, req,
                                                                                      pp::StageOperation::Execute),
                 "502 Bad Gateway", "runtime_stage_transport_failed", "no server");
    // the worker's own refusals travel back as a response frame with the error
    auto wrong_model = req;
    wrong_model.model_id = "another-model";
    expect_error(transport.invoke(stage, wrong_model, pp::StageOperation::Execute), "400 Bad Request",
                 "invalid_stage_request", "model mismatch");
    auto wrong_stage = req;
    wrong_stage.layer_end = 2;
    expect_error(transport.invoke(stage, wrong_stage, pp::StageOperation::Execute), "400 Bad Request",
                 "invalid_stage_request", "layer mismatch");
    // the encoder's own refusals (rollback without tokens) never reach the wire
    expect_error(transport.invoke(stage, req, pp::StageOperation::RollbackSession), "502 Bad Gateway",
                 "runtime_stage_transport_failed", "rollback without tokens");
    // a frame larger than the server's channel
    auto big = req;
    big.payload.assign(2 << 20, 'x');
    expect_error(transport.invoke(stage, big, pp::StageOperation::Execute), "502 Bad Gateway",
                 "runtime_stage_transport_failed", "oversized frame");
    // after all of that the channel still serves
    const auto again = transport.invoke(stage, req, pp::StageOperation::Execute);
    expect(again.ok, "channel usable after the refusals");
    serving.request_stop();
    serving.join();

    // a peer that acknowledges another operation
    const std::string raw = name + "-raw";
    jfb_frame_channel * ch = nullptr;
    if (jfb_frame_channel_create(raw.c_str(), 1 << 20, &ch).code != JFB_STATUS_OK) throw std::runtime_error("raw");
    std::jthread liar([&] {
        const std::uint8_t * f = nullptr;
        std::uint64_t n = 0;
        if (jfb_frame_channel_receive(ch, 5000, &f, &n).code != JFB_STATUS_OK) return;
        rt::protocol::StageResponse resp;
        resp.operation = rt::protocol::kStageOperationCloseSession;
        resp.session_id = "s";
        resp.request_id = "r";
        resp.model_id = kModel;
        resp.stage_count = 2;
        resp.layer_end = 1;
        const auto out = rt::protocol::encode_stage_response_frame(resp);
        jfb_frame_channel_reply(ch, 200, 1, out.prefix.data(), out.prefix.size(), out.payload.data(),
                                out.payload.size());
    });
    auto raw_stage = stage;
    raw_stage.runtime_url = std::string(tr::kInboxUrlScheme) + raw;
    expect_error(transport.invoke(raw_stage, req, pp::StageOperation::Execute), "502 Bad Gateway",
                 "runtime_stage_operation_mismatch", "operation mismatch");
    liar.join();
    jfb_frame_channel_close(ch);
    std::cout << "errors ok" << std::endl;
    return 0;
}

std::string hex(const std::string & bytes) {
    static const char digits[] = "0123456789abcdef";
    std::string out;
    out.reserve(bytes.size() * 2);
    for (const unsigned char c : bytes) {
        out.push_back(digits[c >> 4]);
        out.push_back(digits[c & 15]);
    }
    return out;
}

std::string unhex(const std::string & text) {
    if (text.size() % 2 != 0) throw std::invalid_argument("odd hex length");
    std::string out(text.size() / 2, '\0');
    for (std::size_t i = 0; i < out.size(); ++i) {
        out[i] = static_cast<char>(std::stoi(text.substr(2 * i, 2), nullptr, 16));
    }
    return out;
}

// Frames from the reference's own encoder (protocol/stage.cpp), one JSON line
// each: the golden vectors of the Stagewire codec tests.
int golden() {
    rt::protocol::StageRequest base;
    base.session_id = "session-7";
    base.request_id = "request-7-stage-1";
    base.model_id = "qwen2-7b";
    base.stage_index = 1;
    base.stage_count = 2;
    base.node_name = "stage-1";
    base.layer_start = 14;
    base.layer_end = 28;
    base.max_tokens = 256;
    const auto emit = [](const std::string & name, const std::string & op, const std::string & frame) {
        std::cout << "{\"name\":" << json_string(name) << ",\"operation\":" << json_string(op)
                  << ",\"frame\":\"" << hex(frame) << "\"}\n";
    };
    {
        auto r = base;
        r.stage_index = 0;
        r.layer_start = 0;
        r.layer_end = 14;
        r.payload_kind = "text";
        r.encoding = "utf-8";
        const std::string text = "151644 872 198";
        r.payload.assign(text.begin(), text.end());
        emit("text_prefill", "execute", rt::protocol::encode_stage_request(r, "execute"));
    }
    {
        auto r = base;
        r.payload_kind = "activation";
        r.encoding.clear();
        r.dtype = "f16";
        r.shape = {3, 8};
        r.byte_order = "little";
        r.layout = "row_major";
        for (int i = 0; i < 48; ++i) r.payload.push_back(static_cast<std::uint8_t>((i * 37 + 11) % 251));
        emit("activation_prefill", "execute", rt::protocol::encode_stage_request(r, "execute"));
        r.phase = "decode";
        r.decode_step = 5;
        r.shape = {1, 24};
        r.deployment_id = "deployment-a";
        r.deployment_epoch = 3;
        r.model_sha256 = std::string(64, 'a');
        emit("activation_decode_managed", "execute", rt::protocol::encode_stage_request(r, "execute"));
    }
    {
        auto r = base;
        r.stage_index = 0;
        r.layer_start = 0;
        r.layer_end = 14;
        r.phase = "decode";
        r.decode_step = 1;
        r.payload_kind = "sampled_token";
        r.encoding.clear();
        r.dtype = "u32";
        r.shape = {1};
        r.byte_order = "little";
        r.layout = "row_major";
        r.payload = {0x37, 0x12, 0x02, 0x00};
        emit("sampled_token_decode", "execute", rt::protocol::encode_stage_request(r, "execute"));
        auto rb = r;
        rb.payload_kind = "text";
        rb.encoding = "utf-8";
        rb.dtype.clear();
        rb.shape.clear();
        rb.byte_order.clear();
        rb.layout.clear();
        rb.payload.clear();
        rb.rollback_tokens = 2;
        emit("rollback", "rollback_session", rt::protocol::encode_stage_request(rb, "rollback_session"));
        rb.rollback_tokens = 0;
        emit("close", "close_session", rt::protocol::encode_stage_request(rb, "close_session"));
    }
    {
        rt::protocol::StageResponse r;
        r.operation = "execute";
        r.session_id = "session-7";
        r.request_id = "request-7-stage-1";
        r.model_id = "qwen2-7b";
        r.phase = "decode";
        r.decode_step = 4;
        r.stage_index = 1;
        r.stage_count = 2;
        r.node_name = "stage-1";
        r.layer_start = 14;
        r.layer_end = 28;
        r.payload_kind = "sampled_token";
        r.encoding.clear();
        r.dtype = "u32";
        r.shape = {1};
        r.byte_order = "little";
        r.layout = "row_major";
        r.payload = {0x2a, 0, 0, 0};
        r.bytes_in = 7168;
        r.bytes_out = 4;
        r.completion_tokens = 1;
        r.execution_us = 812;
        r.activation_decode_us = 9;
        r.stage_total_us = 850;
        r.message = "<42>";
        r.token_eog = {0};
        r.token_text_offsets = {0, 4};
        emit("response_sampled_token", "execute", rt::protocol::encode_stage_response(r));
        r.payload.clear();
        r.payload_kind = "text";
        r.encoding = "utf-8";
        r.dtype.clear();
        r.shape.clear();
        r.byte_order.clear();
        r.layout.clear();
        r.message = "session closed";
        r.token_eog.clear();
        r.token_text_offsets.clear();
        r.operation = "close_session";
        emit("response_close", "close_session", rt::protocol::encode_stage_response(r));
    }
    return 0;
}

// Decodes hex frames (one per input line) with the reference's request
// decoder; prints what it accepted or why it refused, one JSON line each.
int decode() {
    std::string line;
    while (std::getline(std::cin, line)) {
        if (line.empty()) continue;
        try {
            const std::string frame = unhex(line);
            const std::string op = rt::protocol::decode_stage_operation(frame);
            const rt::protocol::StageRequest r = rt::protocol::decode_stage_request(frame);
            rt::protocol::validate_stage_operation(op, r.rollback_tokens);
            std::cout << "{\"ok\":true,\"operation\":" << json_string(op) << ",\"session_id\":"
                      << json_string(r.session_id) << ",\"request_id\":" << json_string(r.request_id)
                      << ",\"phase\":" << json_string(r.phase) << ",\"decode_step\":" << r.decode_step
                      << ",\"stage_index\":" << r.stage_index << ",\"layer_start\":" << r.layer_start
                      << ",\"layer_end\":" << r.layer_end << ",\"payload_kind\":" << json_string(r.payload_kind)
                      << ",\"dtype\":" << json_string(r.dtype) << ",\"shape\":[";
            for (std::size_t i = 0; i < r.shape.size(); ++i) std::cout << (i ? "," : "") << r.shape[i];
            std::cout << "],\"payload_bytes\":" << r.payload_bytes << ",\"payload_crc32\":" << r.payload_crc32
                      << ",\"max_tokens\":" << r.max_tokens << "}\n";
        } catch (const std::exception & e) {
            std::cout << "{\"ok\":false,\"error\":" << json_string(e.what()) << "}\n";
        }
    }
    return 0;
}

}  // namespace

int main(int argc, char ** argv) {
    try {
        if (argc < 2) throw std::invalid_argument("usage: transport_replay serve|generate|local|errors ...");
        const std::string mode = argv[1];
        if (mode == "serve") return serve(argc, argv);
        if (mode == "generate") return generate(argc, argv);
        if (mode == "local") return local(argc, argv);
        if (mode == "errors") return errors();
        if (mode == "golden") return golden();
        if (mode == "decode") return decode();
        throw std::invalid_argument("unknown mode " + mode);
    } catch (const std::exception & e) {
        std::cerr << "transport replay: " << e.what() << std::endl;
        return 1;
    }
}
