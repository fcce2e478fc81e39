// Value contracts of the MiniPrefix host layer, mirroring the reference's public
// headers field by field so that a caller can switch without translation:
//   request.h (TokenId, RequestId, Request, GenerationEvent, FinishReason),
//   paged_kv.h:8-31 (KvCapacityError, KvAdmission, KvCacheConfig, PagedSequence),
//   model.h:9-34 (ModelConfig, RunnerStats: 25 size_t fields, layout frozen),
//   kv_manager.h:10-16 (KvStats), cost_stats.h:6-17 (CostStats, CostTimer),
//   engine.h:8-11 (EngineConfig, EngineStepStats), scheduler.h:6-8.
// (TinyInfer v0.3.0, paths under miniprefix/include/miniprefix/.)
#pragma once
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

namespace miniprefix_b200 {

using TokenId = std::int32_t;
using RequestId = std::string;

enum class FinishReason { Eos, Length, Cancelled, Error };

struct GenerationOptions {
    std::uint32_t max_new_tokens = 32;
    std::optional<TokenId> eos_token_id;
};

struct Request {
    RequestId id;
    std::vector<TokenId> prompt_token_ids;
    GenerationOptions generation;
};

struct GenerationEvent {
    RequestId request_id;
    std::optional<TokenId> token_id;
    std::optional<FinishReason> finish_reason;
    std::string error_message;
};

class KvCapacityError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

enum class KvAdmission { Ready, Wait, Impossible };

struct KvCacheConfig {
    int block_tokens = 16;
    int max_blocks = 128;
    int prefix_cache_blocks = 0;
};

// Complete pages are immutable; a shared partial tail is copied before writes.
struct PagedSequence {
    int used = 0;
    std::vector<int> blocks;
    std::vector<std::int32_t> tokens;
    // Lookup hint of the prefix cache: the index node of page i at this
    // sequence's last publish (validated before each use; never changes results).
    mutable std::vector<int> prefix_path;
};

struct ModelConfig {
    int layers = 0, hidden = 0, intermediate = 0, heads = 0, kv_heads = 0, vocabulary = 0, context = 0, eos = 0;
    float rms_epsilon = 0, rope_theta = 0;
    bool tied = true;
    int head_dimension() const { return hidden / heads; }
    int kv_width() const { return kv_heads * head_dimension(); }
    void validate() const;
};

struct KvStats {
    std::size_t live_sequences = 0, live_kv_bytes = 0, peak_kv_bytes = 0, forward_tokens = 0;
    std::size_t kv_block_tokens = 0, kv_total_blocks = 0, kv_live_blocks = 0, kv_peak_blocks = 0;
    std::size_t kv_reserved_bytes = 0;
    std::size_t prefix_cache_capacity = 0, kv_cached_blocks = 0, kv_cache_only_blocks = 0;
    std::size_t prefix_hits = 0, prefix_misses = 0, prefix_reused_tokens = 0, prefix_evictions = 0;
};

struct RunnerStats {
    std::size_t live_sequences = 0, live_kv_bytes = 0, peak_kv_bytes = 0, forward_tokens = 0;
    std::size_t device_weight_bytes = 0, weight_uploaded_bytes = 0, token_uploaded_bytes = 0;
    std::size_t kv_uploaded_bytes = 0, logits_downloaded_bytes = 0, device_allocations = 0;
    std::size_t device_workspace_bytes = 0;
    std::size_t kv_block_tokens = 0, kv_total_blocks = 0, kv_live_blocks = 0, kv_peak_blocks = 0;
    std::size_t kv_reserved_bytes = 0, block_table_uploaded_bytes = 0, block_table_device_bytes = 0;
    std::size_t prefix_cache_capacity = 0, kv_cached_blocks = 0, kv_cache_only_blocks = 0;
    std::size_t prefix_hits = 0, prefix_misses = 0, prefix_reused_tokens = 0, prefix_evictions = 0;
    // Copies the KV fields; device fields are untouched.
    void update_kv_stats(const KvStats& stats);
};
static_assert(sizeof(RunnerStats) == 25 * sizeof(std::size_t), "RunnerStats keeps 25 fields");
static_assert(sizeof(KvStats) == 16 * sizeof(std::size_t), "KvStats keeps 16 fields");

// Cumulative work counters; they survive release/clear. Durations are opt-in.
struct CostStats {
    std::uint64_t lookup_calls = 0, lookup_ns = 0, publish_calls = 0, publish_ns = 0;
    std::uint64_t cow_pages = 0, cow_bytes = 0, cow_copy_ns = 0, cow_timed_copies = 0;
};

class CostTimer {
    using Clock = std::chrono::steady_clock;
    std::uint64_t* total_;
    Clock::time_point start_;

public:
    CostTimer(bool enabled, std::uint64_t& total) : total_(enabled ? &total : nullptr) {
        if (total_) start_ = Clock::now();
    }
    ~CostTimer() {
        if (total_)
            *total_ += std::uint64_t(
                std::chrono::duration_cast<std::chrono::nanoseconds>(Clock::now() - start_).count());
    }
    CostTimer(const CostTimer&) = delete;
    CostTimer& operator=(const CostTimer&) = delete;
};

struct EngineConfig {
    int max_batch_size = 2, token_budget = 32, prefill_chunk = 16, context = 512;
};

struct EngineStepStats {
    std::size_t prefix_reused_tokens = 0, prefill_tokens = 0, decode_tokens = 0;
};

}  // namespace miniprefix_b200
