// The reference-side drop-in: miniprefix::make_cuda_runner backed by the B200
// runner.
//
// This file is compiled INSIDE a MiniPrefix build, against the reference's own
// headers (miniprefix/include/miniprefix/model.h:35-62), in place of
// miniprefix/src/backend/cuda/llama_runner.cu, and linked with libmpb200_host.so
// and libmpb200.so. Every ModelRunner virtual forwards to the host C ABI of this
// repository (include/miniprefix_b200_host.h); the host layer's error codes come
// back as the exception classes the reference's callers catch:
//   -1 std::invalid_argument, -2 std::logic_error, -3 miniprefix::KvCapacityError,
//   -4 std::runtime_error, -5 std::out_of_range, -6 std::runtime_error.
// Weights go tensor by tensor from the ModelWeights the caller loaded (same names
// and [in][out] orientation as MPFX0001); the device packs them at finalize.
//
// oracle/Makefile's `dropin` target builds the reference's own regression
// miniprefix/tests/cow_test.cpp, unmodified, with MINIPREFIX_ENABLE_CUDA against
// this file: its --cuda scenarios (fork, copy-on-write of shared partial tails,
// failed appends that roll back, partial prefix reuse, cost counters, publication
// snapshots) then run on the B200 runner through the reference's interface.
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "miniprefix/model.h"
#include "miniprefix_b200_host.h"

namespace miniprefix {
namespace {

[[noreturn]] void rethrow(long code) {
    const std::string message = mph_last_error();
    switch (code) {
        case -1: throw std::invalid_argument(message);
        case -2: throw std::logic_error(message);
        case -3: throw KvCapacityError(message);
        case -5: throw std::out_of_range(message);
        default: throw std::runtime_error(message);
    }
}

long checked(long rc) {
    if (rc < 0) rethrow(rc);
    return rc;
}

class B200ModelRunner final : public ModelRunner {
public:
    B200ModelRunner(const std::shared_ptr<ModelWeights>& weights, int context, KvCacheConfig kv)
        : config_(weights->config) {
        const ModelConfig& c = config_;
        mp_model_config m{};
        m.layers = c.layers;
        m.hidden = c.hidden;
        m.intermediate = c.intermediate;
        m.heads = c.heads;
        m.kv_heads = c.kv_heads;
        m.vocabulary = c.vocabulary;
        m.context = c.context;
        m.eos = c.eos;
        m.rms_epsilon = c.rms_epsilon;
        m.rope_theta = c.rope_theta;
        m.tied = c.tied ? 1 : 0;
        // Device capacities the reference runner does not have: one block-table
        // slot per page the pool can hold (a live sequence of any length fits),
        // and a forward as large as one append can be.
        const int sequences = std::max(8, std::min(kv.max_blocks, 4096));
        runner_ = mph_runner_new_b200(0, &m, context, kv.block_tokens, kv.max_blocks, kv.prefix_cache_blocks,
                                      sequences, std::max(context, 1), sequences);
        if (!runner_) throw std::invalid_argument(mph_last_error());
        try {
            for (const auto& [name, tensor] : weights->tensors)
                checked(mph_runner_set_weight(runner_, name.c_str(), tensor.data<float>(), std::size_t(tensor.numel())));
            checked(mph_runner_finalize(runner_));
        } catch (...) {
            mph_runner_free(runner_);
            throw;
        }
    }
    ~B200ModelRunner() override { mph_runner_free(runner_); }
    B200ModelRunner(const B200ModelRunner&) = delete;
    B200ModelRunner& operator=(const B200ModelRunner&) = delete;

    const ModelConfig& config() const override { return config_; }
    int context_limit() const override { return mph_runner_context_limit(runner_); }
    KvAdmission reserve_request(const RequestId& id, std::size_t tokens) override {
        return static_cast<KvAdmission>(checked(mph_runner_reserve(runner_, id.c_str(), tokens)));
    }
    void release_reservation(const RequestId& id) noexcept override {
        mph_runner_release_reservation(runner_, id.c_str());
    }
    void create(const RequestId& id) override { checked(mph_runner_create(runner_, id.c_str())); }
    void fork_sequence(const RequestId& source, const RequestId& target) override {
        checked(mph_runner_fork(runner_, source.c_str(), target.c_str()));
    }
    std::size_t reuse_prefix(const RequestId& id, const std::vector<TokenId>& prompt) override {
        const std::vector<int32_t> p(prompt.begin(), prompt.end());
        return std::size_t(checked(mph_runner_reuse_prefix(runner_, id.c_str(), p.data(), int32_t(p.size()))));
    }
    void cache_prefix(const RequestId& id) override { checked(mph_runner_cache_prefix(runner_, id.c_str())); }
    void clear_prefix_cache() override { checked(mph_runner_clear_prefix_cache(runner_)); }
    std::vector<float> append(const RequestId& id, const std::vector<TokenId>& tokens) override {
        const std::vector<int32_t> t(tokens.begin(), tokens.end());
        std::vector<float> logits(std::size_t(config_.vocabulary));
        checked(mph_runner_append(runner_, id.c_str(), t.data(), int32_t(t.size()), logits.data()));
        return logits;
    }
    void release(const RequestId& id) override { checked(mph_runner_release(runner_, id.c_str())); }
    void clear() override { checked(mph_runner_clear(runner_)); }
    RunnerStats stats() const override {
        std::size_t v[25] = {};
        mph_runner_stats(runner_, v);
        RunnerStats s;
        std::size_t* fields[] = {&s.live_sequences,        &s.live_kv_bytes,           &s.peak_kv_bytes,
                                 &s.forward_tokens,        &s.device_weight_bytes,     &s.weight_uploaded_bytes,
                                 &s.token_uploaded_bytes,  &s.kv_uploaded_bytes,       &s.logits_downloaded_bytes,
                                 &s.device_allocations,    &s.device_workspace_bytes,  &s.kv_block_tokens,
                                 &s.kv_total_blocks,       &s.kv_live_blocks,          &s.kv_peak_blocks,
                                 &s.kv_reserved_bytes,     &s.block_table_uploaded_bytes, &s.block_table_device_bytes,
                                 &s.prefix_cache_capacity, &s.kv_cached_blocks,        &s.kv_cache_only_blocks,
                                 &s.prefix_hits,           &s.prefix_misses,           &s.prefix_reused_tokens,
                                 &s.prefix_evictions};
        for (int i = 0; i < 25; ++i) *fields[i] = v[i];
        return s;
    }
    CostStats cost_stats() const override {
        std::uint64_t v[8] = {};
        mph_runner_cost_stats(runner_, v);
        CostStats c;
        c.lookup_calls = v[0];
        c.lookup_ns = v[1];
        c.publish_calls = v[2];
        c.publish_ns = v[3];
        c.cow_pages = v[4];
        c.cow_bytes = v[5];
        c.cow_copy_ns = v[6];
        c.cow_timed_copies = v[7];
        return c;
    }
    void set_cost_timing(bool enabled) override { mph_runner_set_cost_timing(runner_, enabled ? 1 : 0); }

private:
    ModelConfig config_;
    mph_runner* runner_ = nullptr;
};

}  // namespace

std::unique_ptr<ModelRunner> make_cuda_runner(std::shared_ptr<ModelWeights> weights, int context, KvCacheConfig kv) {
    return std::make_unique<B200ModelRunner>(weights, context, kv);
}

}  // namespace miniprefix
