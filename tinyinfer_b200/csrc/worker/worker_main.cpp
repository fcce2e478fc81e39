// mpb200_worker: the reference worker (miniprefix/apps/worker.cpp) on the B200
// runner -- protocol v3 on stdin/stdout over an MPFX0001 model.
//   mpb200_worker MODEL b200 CONTEXT [BATCH TOKENS CHUNK BLOCK_TOKENS KV_BLOCKS PREFIX_BLOCKS
//                                     [MAX_SEQUENCES [DEVICE]]]
// Defaults as the reference's EngineConfig / KvCacheConfig. The batched engine
// needs device capacities: at most MAX_SEQUENCES live sequences (default
// BATCH + 8) and one forward of at most TOKENS tokens.
#include <iostream>
#include <memory>
#include <stdexcept>
#include <string>

#include "b200_runner.h"
#include "engine.h"
#include "mpfx.h"
#include "protocol.h"

using namespace miniprefix_b200;

int main(int argc, char** argv) {
    try {
        if (argc < 4 || argc > 12)
            throw std::invalid_argument(
                "usage: mpb200_worker MODEL b200 CONTEXT [BATCH TOKENS CHUNK BLOCK_TOKENS KV_BLOCKS PREFIX_BLOCKS "
                "[MAX_SEQUENCES [DEVICE]]]");
        const std::string backend = argv[2];
        if (backend != "b200") throw std::invalid_argument("backend unavailable in this build");
        const int context = std::stoi(argv[3]);
        EngineConfig config;
        config.context = context;
        if (argc > 4) config.max_batch_size = std::stoi(argv[4]);
        if (argc > 5) config.token_budget = std::stoi(argv[5]);
        if (argc > 6) config.prefill_chunk = std::stoi(argv[6]);
        KvCacheConfig kv;
        if (argc > 7) kv.block_tokens = std::stoi(argv[7]);
        if (argc > 8) kv.max_blocks = std::stoi(argv[8]);
        if (argc > 9) kv.prefix_cache_blocks = std::stoi(argv[9]);
        B200Options options;
        options.max_sequences = argc > 10 ? std::stoi(argv[10]) : config.max_batch_size + 8;
        options.max_step_sequences = options.max_sequences;
        options.max_step_tokens = std::max(config.token_budget, 1);
        options.device = argc > 11 ? std::stoi(argv[11]) : 0;
        const ModelConfig model = read_mpfx_config(argv[1]);
        auto runner = std::make_unique<B200Runner>(model, context, kv, options);
        read_mpfx(argv[1], [&](const MpfxTensor& t) { runner->set_weight(t.name, t.data, t.elements); });
        runner->finalize_weights();
        Engine engine(std::move(runner), config);
        protocol::ready(std::cout, model.vocabulary, model.eos, context, backend);
        return protocol::serve(engine, std::cin, std::cout);
    } catch (const std::exception& e) {
        std::cerr << e.what() << '\n';
        return 1;
    }
}
