// Runs the reference worker's deployment-config validation
// (runtime/worker/config.cpp:142-188) on one native-engine configuration and
// prints "accepted" or "rejected: <reason>". Built twice by
// oracle/ref_executor/build.py: once from the reference's config.cpp as it
// is, once with its `decode_batch_size == 1` check for the native engine
// (config.cpp:159-162) taken out, the change that lets the worker put
// ContinuousBatchingExecutor in front of a native executor with execute_batch.
//
//   config_check <decode_batch_size> <parallel_sessions> <compute_backend>
//
// Test infrastructure: built into oracle/_ref/ only where the reference
// sources are present.
#include "worker/config.hpp"

#include <iostream>
#include <stdexcept>
#include <string>

int main(int argc, char ** argv) {
    if (argc != 4) {
        std::cerr << "usage: config_check <decode_batch_size> <parallel_sessions> <compute_backend>\n";
        return 2;
    }
    jetsonfabric::runtime::Config cfg;
    cfg.engine = "native";
    cfg.mode = jetsonfabric::runtime::ExecutionMode::PipelineParallel;
    cfg.decode_batch_size = std::stoi(argv[1]);
    cfg.parallel_sessions = std::stoi(argv[2]);
    cfg.http_workers = cfg.parallel_sessions;
    cfg.compute_backend = argv[3];
    cfg.model_path = "model.jfm";
    cfg.stage_assignment = {.stage_index = 0, .stage_count = 2, .layer_start = 0, .layer_end = 14};
    try {
        jetsonfabric::runtime::validate_deployment_config(cfg);
        std::cout << "accepted\n";
    } catch (const std::exception & e) {
        std::cout << "rejected: " << e.what() << "\n";
    }
    return 0;
}
