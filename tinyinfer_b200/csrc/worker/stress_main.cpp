// mpb200_stress: long-running lifecycle stress of the batched engine on the B200
// runner, the reference's 8-request wave harness (miniprefix/benchmarks/stress.cpp)
// restated for this engine.
//   mpb200_stress MODEL b200 SECONDS MIN_WAVES
// Twelve prompt templates (lengths 8, 17, 33, 65; the first six share 8 leading
// tokens); their greedy 8-token continuations come first from a runner without a
// prefix cache (the same backend, one sequence at a time). Each wave submits 8
// requests: one cancelled while queued, one cancelled after the first step, one
// with an EOS equal to its first token, one that exceeds the KV pool, four that run
// to their length; every token must equal the no-cache stream. After each wave the
// runner must hold no sequence or table, only cache pages, within the pool bounds;
// every fifth wave clears the prefix cache. One JSON line per wave, then a summary.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <iomanip>
#include <iostream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>

#include "b200_runner.h"
#include "engine.h"
#include "mpfx.h"

using namespace miniprefix_b200;
using Clock = std::chrono::steady_clock;

namespace {

double ms_since(Clock::time_point t) { return std::chrono::duration<double, std::milli>(Clock::now() - t).count(); }

void require(bool ok, const char* what) {
    if (!ok) throw std::runtime_error(what);
}

std::unique_ptr<B200Runner> make_runner(const std::string& path, KvCacheConfig kv, int max_step_tokens) {
    const ModelConfig model = read_mpfx_config(path);
    B200Options o;
    o.max_sequences = 16;
    o.max_step_sequences = 16;
    o.max_step_tokens = max_step_tokens;
    auto r = std::make_unique<B200Runner>(model, 128, kv, o);
    read_mpfx(path, [&](const MpfxTensor& t) { r->set_weight(t.name, t.data, t.elements); });
    r->finalize_weights();
    return r;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        if (argc != 5) throw std::invalid_argument("usage: mpb200_stress MODEL b200 SECONDS MIN_WAVES");
        if (std::string(argv[2]) != "b200") throw std::invalid_argument("backend unavailable");
        const double seconds = std::stod(argv[3]);
        const int min_waves = std::stoi(argv[4]);
        require(std::isfinite(seconds) && seconds > 0 && min_waves > 0, "invalid run bounds");
        const std::string path = argv[1];
        const ModelConfig model = read_mpfx_config(path);

        std::vector<std::vector<TokenId>> prompts, expected;
        static const int kLengths[4] = {8, 17, 33, 65};
        for (int i = 0; i < 12; ++i) {
            const int length = kLengths[i % 4];
            std::vector<TokenId> p;
            for (int j = 0; j < length; ++j)
                p.push_back(1 + ((i < 6 && j < 8) ? j : (i * 37 + j * 13)) % (model.vocabulary - 1));
            prompts.push_back(p);
        }
        {
            auto plain = make_runner(path, {4, 128, 0}, 128);
            for (const auto& p : prompts) {
                plain->create("plain");
                std::vector<TokenId> input = p, stream;
                for (int j = 0; j < 8; ++j) {
                    const auto logits = plain->append("plain", input);
                    const TokenId t = TokenId(std::max_element(logits.begin(), logits.end()) - logits.begin());
                    stream.push_back(t);
                    input = {t};
                }
                plain->release("plain");
                expected.push_back(stream);
            }
        }

        auto runner = make_runner(path, {4, 24, 12}, 16);
        B200Runner* trace = runner.get();
        Engine engine(std::move(runner), EngineConfig{4, 16, 8, 128});
        const auto start = Clock::now();
        std::size_t total_requests = 0, total_tokens = 0;
        int wave = 0;
        std::cout << std::setprecision(12);
        while (ms_since(start) < seconds * 1000 || wave < min_waves) {
            const auto wave_start = Clock::now();
            const RunnerStats before = trace->stats();
            std::map<RequestId, int> templ, received, terminal;
            std::map<RequestId, FinishReason> reason;
            std::vector<RequestId> ids;
            std::size_t wave_tokens = 0, forward_tokens = 0, reused_tokens = 0;
            for (int i = 0; i < 8; ++i) {
                const RequestId id = std::to_string(wave * 8 + i);
                ids.push_back(id);
                const int k = (wave + i) % 12;
                templ[id] = k;
                Request r;
                r.id = id;
                r.prompt_token_ids = prompts[std::size_t(k)];
                r.generation.max_new_tokens = 8;
                if (i == 6) r.generation.eos_token_id = expected[std::size_t(k)][0];
                if (i == 7) {  // 97 tokens need 25 pages of 4: more than the 24-page pool
                    r.prompt_token_ids.assign(97, 1);
                    r.generation.max_new_tokens = 1;
                }
                engine.submit(std::move(r));
            }
            auto consume = [&] {
                for (const auto& e : engine.poll_events()) {
                    require(templ.count(e.request_id) != 0, "unknown event");
                    require(!terminal[e.request_id], "event after terminal");
                    if (e.token_id) {
                        int& n = received[e.request_id];
                        require(n < 8 && *e.token_id == expected[std::size_t(templ[e.request_id])][std::size_t(n)],
                                "token mismatch");
                        ++n;
                        ++wave_tokens;
                    }
                    if (e.finish_reason) {
                        ++terminal[e.request_id];
                        reason[e.request_id] = *e.finish_reason;
                    }
                }
            };
            engine.cancel(ids[5]);  // still queued
            consume();
            double step_ms = 0;
            int steps = 0;
            while (!engine.idle()) {
                require(++steps <= 256, "no bounded progress");
                const auto tick = Clock::now();
                engine.step();
                step_ms += ms_since(tick);
                const auto st = engine.last_step_stats();
                forward_tokens += st.prefill_tokens + st.decode_tokens;
                reused_tokens += st.prefix_reused_tokens;
                consume();
                if (steps == 1 && !terminal[ids[0]]) {  // after at least one step
                    engine.cancel(ids[0]);
                    consume();
                }
                require(!engine.failed(), "engine poisoned");
            }
            for (int i = 0; i < 8; ++i) {
                const RequestId& id = ids[std::size_t(i)];
                require(terminal[id] == 1, "missing or duplicate terminal event");
                const FinishReason want = i == 7 ? FinishReason::Error
                                          : i == 6 ? FinishReason::Eos
                                          : (i == 0 || i == 5) ? FinishReason::Cancelled
                                                               : FinishReason::Length;
                require(reason[id] == want, "wrong finish reason");
                if (want == FinishReason::Length) require(received[id] == 8, "short output");
                if (want == FinishReason::Eos) require(received[id] == 1, "EOS not early");
            }
            const RunnerStats after = trace->stats();
            require(after.forward_tokens - before.forward_tokens == forward_tokens &&
                        after.prefix_reused_tokens - before.prefix_reused_tokens == reused_tokens,
                    "step / runner accounting mismatch");
            require(after.live_sequences == 0 && after.block_table_device_bytes == 0, "sequence or table leak");
            require(after.kv_live_blocks == after.kv_cache_only_blocks && after.kv_cached_blocks == after.kv_cache_only_blocks,
                    "non-cache page leak");
            require(after.kv_live_blocks <= 12 && after.kv_peak_blocks <= 24, "pool / cache bound");
            require(after.weight_uploaded_bytes == before.weight_uploaded_bytes, "weights uploaded again");
            if (wave % 5 == 4) {
                trace->clear_prefix_cache();
                require(trace->stats().kv_live_blocks == 0, "clear leaked pages");
            }
            total_requests += 8;
            total_tokens += wave_tokens;
            std::cout << "{\"wave\":" << wave << ",\"elapsed_ms\":" << ms_since(start) << ",\"wall_ms\":"
                      << ms_since(wave_start) << ",\"step_ms\":" << step_ms << ",\"steps\":" << steps
                      << ",\"tokens\":" << wave_tokens << ",\"cached_pages\":" << after.kv_cached_blocks
                      << ",\"forward_tokens\":" << forward_tokens << ",\"reused_tokens\":" << reused_tokens
                      << ",\"evictions\":" << after.prefix_evictions - before.prefix_evictions
                      << ",\"flushes\":" << trace->flushes() << ",\"hazard_flushes\":" << trace->hazard_flushes()
                      << "}" << std::endl;
            ++wave;
        }
        engine.shutdown();
        const RunnerStats final_stats = trace->stats();
        require(final_stats.live_sequences == 0 && final_stats.kv_live_blocks == 0 &&
                    final_stats.block_table_device_bytes == 0,
                "final leak");
        std::cout << "{\"passed\":true,\"waves\":" << wave << ",\"requests\":" << total_requests
                  << ",\"tokens\":" << total_tokens << ",\"elapsed_ms\":" << ms_since(start) << "}" << std::endl;
        return 0;
    } catch (const std::exception& e) {
        std::cerr << e.what() << std::endl;
        return 1;
    }
}
