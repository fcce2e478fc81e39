#include "scripted_runner.h"

namespace miniprefix_b200 {

ScriptedRunner::ScriptedRunner(int vocabulary, int context, int layers, int width, KvCacheConfig kv)
    : kv_(kv, layers, width, context, vocabulary) {
    config_.vocabulary = vocabulary;
    config_.context = context;
    config_.layers = layers;
}

void ScriptedRunner::script(const RequestId& id, std::vector<TokenId> tokens) {
    script_[id] = std::move(tokens);
    cursor_[id] = 0;
}

std::vector<KVManager::TailCopyRegion> ScriptedRunner::take_regions() {
    auto r = std::move(regions_);
    regions_.clear();
    return r;
}

bool ScriptedRunner::poisoned(const std::vector<TokenId>& tokens) const {
    for (auto t : tokens)
        if (poison_.count(t)) return true;
    return false;
}

std::vector<float> ScriptedRunner::append(const RequestId& id, const std::vector<TokenId>& tokens) {
    auto tx = kv_.prepare_append(id, tokens);
    tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) { regions_.push_back(r); });
    std::vector<float> logits(std::size_t(config_.vocabulary), 0.0f);
    if (poisoned(tokens)) throw std::runtime_error("nonfinite logits");
    auto& list = script_[id];
    auto& at = cursor_[id];
    logits[std::size_t(at < list.size() ? list[at] : 0)] = 1.0f;
    tx.commit();
    ++at;
    return logits;
}

RunnerStats ScriptedRunner::stats() const {
    RunnerStats r;
    r.update_kv_stats(kv_.stats());
    return r;
}

void ScriptedRunner::begin_batch() {
    results_.clear();
    kv_.begin_checkpoint();
    saved_cursor_ = cursor_;
    saved_regions_ = regions_.size();
}

std::size_t ScriptedRunner::stage_append(const RequestId& id, const std::vector<TokenId>& tokens) {
    auto tx = kv_.prepare_append(id, tokens);
    tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) { regions_.push_back(r); });
    AppendResult result;
    result.finite = !poisoned(tokens);
    auto& list = script_[id];
    auto& at = cursor_[id];
    result.token = at < list.size() ? list[at] : 0;
    tx.commit();
    ++at;
    results_.push_back(result);
    return results_.size() - 1;
}

void ScriptedRunner::restore_batch() {
    kv_.restore_checkpoint();
    cursor_ = saved_cursor_;
    regions_.resize(saved_regions_);
    results_.clear();
}

void ScriptedRunner::fail_append(const RequestId& id, const std::vector<TokenId>& tokens) {
    auto tx = kv_.prepare_append(id, tokens);
    tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) { regions_.push_back(r); });
    throw std::runtime_error("nonfinite logits");
}

void ScriptedRunner::end_batch() {
    kv_.end_checkpoint();
    results_.clear();
}

}  // namespace miniprefix_b200
