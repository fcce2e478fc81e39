// ScriptedRunner: a device-free ModelRunner for testing host logic. It keeps the
// real KVManager (so every page, COW and prefix decision is the production one)
// but, instead of a model, each successful append of request `id` returns
// one-hot logits at the next token of that id's script (0 when exhausted), and
// an append that contains a poisoned token fails as a nonfinite forward would.
// It implements the staged-batch interface like B200Runner, so the Engine's
// batched step -- including the restore-and-replay of a failed step -- runs
// on a CPU and can be compared decision by decision with the reference engine.
#pragma once
#include <map>
#include <set>

#include "model_runner.h"

namespace miniprefix_b200 {

class ScriptedRunner final : public ModelRunner {
public:
    ScriptedRunner(int vocabulary, int context, int layers, int width, KvCacheConfig kv);
    void script(const RequestId& id, std::vector<TokenId> tokens);
    void poison(TokenId token) { poison_.insert(token); }
    std::vector<KVManager::TailCopyRegion> take_regions();

    const ModelConfig& config() const override { return config_; }
    int context_limit() const override { return kv_.context_limit(); }
    KvAdmission reserve_request(const RequestId& id, std::size_t n) override { return kv_.reserve_request(id, n); }
    void release_reservation(const RequestId& id) noexcept override { kv_.release_reservation(id); }
    void create(const RequestId& id) override { kv_.create(id); }
    void fork_sequence(const RequestId& s, const RequestId& t) override { kv_.fork_sequence(s, t); }
    std::size_t reuse_prefix(const RequestId& id, const std::vector<TokenId>& p) override {
        return kv_.reuse_prefix(id, p);
    }
    void cache_prefix(const RequestId& id) override { kv_.cache_prefix_deferred(id); }
    void clear_prefix_cache() override { kv_.clear_prefix_cache(); }
    std::vector<float> append(const RequestId& id, const std::vector<TokenId>& tokens) override;
    void release(const RequestId& id) override { kv_.release(id); }
    void clear() override { kv_.clear(); }
    RunnerStats stats() const override;
    CostStats cost_stats() const override { return kv_.cost_stats(); }
    std::size_t kv_block_tokens() const override { return std::size_t(kv_.config().block_tokens); }

    bool batched() const override { return true; }
    void begin_batch() override;
    std::size_t stage_append(const RequestId& id, const std::vector<TokenId>& tokens) override;
    void flush() override { kv_.settle_publishes(); }
    void restore_batch() override;
    void fail_append(const RequestId& id, const std::vector<TokenId>& tokens) override;
    void end_batch() override;
    void set_replay(bool) override {}

    const KVManager& kv() const { return kv_; }

private:
    bool poisoned(const std::vector<TokenId>& tokens) const;
    ModelConfig config_;
    KVManager kv_;
    std::map<RequestId, std::vector<TokenId>> script_;
    std::map<RequestId, std::size_t> cursor_;
    std::map<RequestId, std::size_t> saved_cursor_;
    std::vector<KVManager::TailCopyRegion> regions_;
    std::size_t saved_regions_ = 0;
    std::set<TokenId> poison_;
};

}  // namespace miniprefix_b200
