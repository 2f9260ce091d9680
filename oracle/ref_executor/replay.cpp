// Replays the reference's NativeStageExecutor serving checks against this
// repository's engine: the reference executor (runtime/adapters/
// native_stage_executor.cpp, compiled unmodified except for the inserted
// execute_batch method) drives libjfb.so through the drop-in
// jetsonfabric/native_inference.hpp API on the CUDA backend.
//
// The sequence follows the reference's own test
// (runtime/adapters/native_stage_executor_test.cpp:85-235) on the reference's
// 2-layer F32 fixture package: direct session prefill/decode/rollback,
// executor prefill, duplicate prefill rejected, decode, rollback, close, the
// two-stage 0-1 / 1-2 split with its activation handoff, and an oversized
// activation shape rejected as invalid input. It then checks execute_batch:
// three sessions decoded in one batched engine pass, with an unknown session,
// a duplicate session and a wrong decode step rejected per input. Last, the
// reference's ContinuousBatchingExecutor coalesces three concurrent decode
// steps into one execute_batch call.
//
// Test infrastructure: built by oracle/ref_executor/build.py into
// oracle/_ref/ only when the reference sources are present.
#include "adapters/native_stage_executor.hpp"
#include "inference/token_payload.hpp"
#include "pipeline_parallel/continuous_batching_executor.hpp"

#include <atomic>
#include <thread>

#include <cstdint>
#include <iostream>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

namespace {

namespace native = jetsonfabric::native;
namespace inf = jetsonfabric::runtime::inference;
using jetsonfabric::runtime::adapters::NativeStageConfig;
using jetsonfabric::runtime::adapters::NativeStageExecutor;

// The fixture vocabulary: the text "fixture" is the single token 2, and the
// fixture model always answers 7, spelled "x".
class FixtureTokens final : public jetsonfabric::runtime::tokenization::Tokenizer {
public:
    std::vector<std::int32_t> tokenize(std::string_view text) const override {
        if (text != "fixture") throw std::invalid_argument("fixture tokenizer got unexpected text");
        return {2};
    }
    std::string token_piece(std::int32_t token) const override {
        if (token != 7) throw std::invalid_argument("fixture tokenizer got unexpected token");
        return "x";
    }
    bool is_end_token(std::int32_t) const override { return false; }
};

void check(bool ok, const std::string & what) {
    if (!ok) throw std::runtime_error(what);
}

inf::StageInput prefill_request(const std::string & session, int layers, int index, int count) {
    inf::StageInput in;
    in.session_id = session;
    in.request_id = session + "-request";
    in.model_id = "fixture";
    in.phase = inf::Phase::Prefill;
    in.decode_step = 0;
    in.position = inf::StagePosition{.index = index, .count = count};
    in.layers = inf::LayerRange{.start = index, .end = index + layers};
    in.payload.kind = inf::PayloadKind::Text;
    in.payload.encoding = "utf-8";
    const std::string text = "fixture";
    in.payload.bytes.assign(text.begin(), text.end());
    in.max_tokens = 2;
    return in;
}

inf::StageInput decode_request(inf::StageInput in, int step, inf::Payload payload) {
    in.phase = inf::Phase::Decode;
    in.decode_step = step;
    in.payload = std::move(payload);
    return in;
}

void check_token_seven(const inf::ExecutionResult & r, const std::string & where) {
    check(r.ok, where + ": " + r.error.code + " " + r.error.message);
    check(inf::decode_single_token(r.output.payload) == 7, where + ": sampled token is not 7");
    check(r.output.token_text == "x", where + ": token text is not \"x\"");
    check(r.output.completion_tokens == 1, where + ": completion token not counted");
}

std::shared_ptr<native::NativeEngine> engine(const std::string & path) {
    return std::make_shared<native::NativeEngine>(path, native::Backend::Cuda, 1);
}

std::shared_ptr<native::NativeEngine> engine(const std::string & path, std::uint32_t start, std::uint32_t end) {
    return std::make_shared<native::NativeEngine>(
        path, native::EngineOptions{.backend = native::Backend::Cuda, .threads = 1, .layer_start = start,
                                    .layer_end = end});
}

void single_stage(const std::string & path) {
    auto eng = engine(path);
    const int layers = int(eng->model_info().layer_count);
    auto direct = eng->create_session(2);
    const std::int32_t prompt[1] = {2};
    check(direct->prefill_greedy(prompt) == 7, "direct prefill token");
    check(direct->decode_greedy(7) == 7 && direct->position() == 2, "direct decode");
    direct->rollback(1);
    check(direct->position() == 1, "direct rollback position");

    NativeStageExecutor ex(NativeStageConfig{.engine = eng, .tokenizer = std::make_shared<FixtureTokens>(),
                                             .ctx_size = 16, .position = {.index = 0, .count = 1},
                                             .layers = {.start = 0, .end = layers}});
    const inf::StageInput pre = prefill_request("s", layers, 0, 1);
    const inf::ExecutionResult first = ex.execute(pre);
    check_token_seven(first, "executor prefill");
    check(first.output.prompt_tokens == 1 && first.output.prompt_token_ids == std::vector<std::uint32_t>{2},
          "prompt token accounting");
    check(ex.session_count() == 1, "session retained");
    const inf::ExecutionResult dup = ex.execute(pre);
    check(!dup.ok && dup.error.code == "duplicate_stage_session", "duplicate prefill rejected");
    const inf::StageInput dec = decode_request(pre, 1, inf::sampled_token_payload(7));
    check_token_seven(ex.execute(dec), "executor decode");
    ex.rollback_session("s", 1);
    check_token_seven(ex.execute(dec), "decode after rollback");
    ex.close_session("s");
    check(ex.session_count() == 0, "close releases the session");
    const inf::ExecutionResult gone = ex.execute(dec);
    check(!gone.ok && gone.error.code == "stage_session_not_found", "decode after close rejected");
}

void two_stages(const std::string & path) {
    auto a = engine(path, 0, 1);
    auto b = engine(path, 1, 2);
    check(a->model_info().resident_layer_end == 1 && b->model_info().resident_layer_start == 1, "stage ranges");
    check(a->model_info().weight_bytes < a->model_info().total_weight_bytes &&
              b->model_info().weight_bytes < b->model_info().total_weight_bytes,
          "stages hold part of the weights");
    auto tok = std::make_shared<FixtureTokens>();
    NativeStageExecutor first(NativeStageConfig{.engine = a, .tokenizer = tok, .ctx_size = 16,
                                                .position = {.index = 0, .count = 2}, .layers = {.start = 0, .end = 1}});
    NativeStageExecutor last(NativeStageConfig{.engine = b, .tokenizer = tok, .ctx_size = 16,
                                               .position = {.index = 1, .count = 2}, .layers = {.start = 1, .end = 2}});
    const inf::StageInput p0 = prefill_request("split", 1, 0, 2);
    const inf::ExecutionResult r0 = first.execute(p0);
    check(r0.ok && r0.output.payload.kind == inf::PayloadKind::Activation, "first stage returns an activation");
    inf::StageInput p1 = p0;
    p1.position = {.index = 1, .count = 2};
    p1.layers = {.start = 1, .end = 2};
    p1.payload = r0.output.payload;
    check_token_seven(last.execute(p1), "final stage prefill");

    inf::StageInput huge = p1;
    huge.session_id = "oversized";
    huge.payload.tensor.shape[0] = std::numeric_limits<std::int64_t>::max();
    huge.payload.bytes.clear();
    const inf::ExecutionResult rh = last.execute(huge);
    check(!rh.ok && rh.error.code == "invalid_native_stage_input", "oversized activation rejected");

    const inf::ExecutionResult d0 = first.execute(decode_request(p0, 1, inf::sampled_token_payload(7)));
    check(d0.ok && d0.output.payload.kind == inf::PayloadKind::Activation, "first stage decode activation");
    check_token_seven(last.execute(decode_request(p1, 1, d0.output.payload)), "final stage decode");
}

void batched(const std::string & path) {
    auto eng = engine(path);
    const int layers = int(eng->model_info().layer_count);
    NativeStageExecutor ex(NativeStageConfig{.engine = eng, .tokenizer = std::make_shared<FixtureTokens>(),
                                             .ctx_size = 16, .position = {.index = 0, .count = 1},
                                             .layers = {.start = 0, .end = layers}});
    const char * names[3] = {"b0", "b1", "b2"};
    std::vector<inf::StageInput> batch;
    for (const char * n : names) {
        const inf::StageInput pre = prefill_request(n, layers, 0, 1);
        check_token_seven(ex.execute(pre), std::string("batch prefill ") + n);
        batch.push_back(decode_request(pre, 1, inf::sampled_token_payload(7)));
    }
    std::vector<inf::StageInput> with_errors = batch;
    with_errors.push_back(batch[1]);  // the same session twice
    inf::StageInput unknown = batch[0];
    unknown.session_id = "nobody";
    with_errors.push_back(unknown);
    inf::StageInput wrong_step = batch[2];
    wrong_step.decode_step = 5;
    with_errors.insert(with_errors.begin(), wrong_step);
    const std::vector<inf::ExecutionResult> out = ex.execute_batch(with_errors);
    check(out.size() == with_errors.size(), "one result per input");
    check(!out[0].ok && out[0].error.code == "unexpected_decode_step", "wrong decode step rejected");
    for (int k = 1; k <= 3; ++k) check_token_seven(out[std::size_t(k)], "batched decode");
    check(!out[4].ok && out[4].error.code == "duplicate_batch_session", "duplicate batch session rejected");
    check(!out[5].ok && out[5].error.code == "stage_session_not_found", "unknown batch session rejected");
    // the batched step advanced each session once: the next step is 2
    for (inf::StageInput & in : batch) in.decode_step = 2;
    for (const inf::ExecutionResult & r : ex.execute_batch(batch)) check(!r.ok, "capacity 2 is exhausted after one decode");
}

// Forwards to the native executor and records the batches it is handed.
class CountingExecutor final : public inf::Executor {
public:
    explicit CountingExecutor(std::unique_ptr<NativeStageExecutor> inner) : inner_(std::move(inner)) {}
    inf::ExecutionResult execute(const inf::StageInput & in) const override { return inner_->execute(in); }
    std::vector<inf::ExecutionResult> execute_batch(const std::vector<inf::StageInput> & ins) const override {
        std::size_t seen = largest.load();
        while (ins.size() > seen && !largest.compare_exchange_weak(seen, ins.size())) {
        }
        return inner_->execute_batch(ins);
    }
    void close_session(const std::string & id) const override { inner_->close_session(id); }
    void rollback_session(const std::string & id, int n) const override { inner_->rollback_session(id, n); }
    mutable std::atomic<std::size_t> largest{0};

private:
    std::unique_ptr<NativeStageExecutor> inner_;
};

// The reference's ContinuousBatchingExecutor (continuous_batching_executor.cpp:
// 44-127) in front of the native executor, as the worker builds it once the
// decode_batch_size == 1 check is lifted: three sessions' decode steps sent
// concurrently are coalesced into one execute_batch call, which the native
// executor serves as one batched engine pass.
void continuous_batching(const std::string & path) {
    auto eng = engine(path);
    const int layers = int(eng->model_info().layer_count);
    auto native_ex = std::make_unique<NativeStageExecutor>(NativeStageConfig{
        .engine = eng, .tokenizer = std::make_shared<FixtureTokens>(), .ctx_size = 16,
        .position = {.index = 0, .count = 1}, .layers = {.start = 0, .end = layers}});
    auto counting = std::make_unique<CountingExecutor>(std::move(native_ex));
    CountingExecutor * probe = counting.get();
    using jetsonfabric::runtime::pipeline_parallel::ContinuousBatchingConfig;
    using jetsonfabric::runtime::pipeline_parallel::ContinuousBatchingExecutor;
    ContinuousBatchingExecutor cb(std::move(counting),
                                  ContinuousBatchingConfig{.max_batch_size = 3, .max_wait = std::chrono::seconds(2)});
    const char * names[3] = {"cb0", "cb1", "cb2"};
    std::vector<inf::StageInput> decodes;
    for (const char * n : names) {
        const inf::StageInput pre = prefill_request(n, layers, 0, 1);
        check_token_seven(cb.execute(pre), std::string("batching prefill ") + n);
        decodes.push_back(decode_request(pre, 1, inf::sampled_token_payload(7)));
    }
    std::vector<inf::ExecutionResult> results(decodes.size());
    {
        std::vector<std::jthread> callers;
        for (std::size_t i = 0; i < decodes.size(); ++i) {
            callers.emplace_back([&, i] { results[i] = cb.execute(decodes[i]); });
        }
    }
    for (const inf::ExecutionResult & r : results) check_token_seven(r, "coalesced decode");
    check(probe->largest.load() == decodes.size(), "the three decode steps reached the engine as one batch");
    for (const char * n : names) cb.close_session(n);
}

}  // namespace

int main(int argc, char ** argv) {
    try {
        if (argc != 2) throw std::invalid_argument("usage: native_executor_replay <fixture package>");
        single_stage(argv[1]);
        two_stages(argv[1]);
        batched(argv[1]);
        continuous_batching(argv[1]);
        std::cout << "replay ok\n";
        return 0;
    } catch (const std::exception & e) {
        std::cerr << "native executor replay: " << e.what() << '\n';
        return 1;
    }
}
