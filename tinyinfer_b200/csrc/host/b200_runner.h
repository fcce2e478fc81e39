// B200Runner: the ModelRunner that drives the sm_100a device layer
// (include/miniprefix_b200.h) -- the drop-in for the reference CudaRunner
// (miniprefix/src/backend/cuda/llama_runner.cu:51-186).
//
// Per-call semantics match CudaRunner: create() gives the sequence a device
// block table, append() performs prepare -> COW copy -> table upload -> forward
// -> logits download, throws "nonfinite CUDA logits" and rolls back on a
// nonfinite result, and commits otherwise; release/clear drop pages and tables.
// Beyond that, stage_append()/flush() let the Engine run all appends of a step as
// ONE device forward (see model_runner.h). The forward copies every COW source
// before writing any destination, then runs the layers; pending work is flushed
// early only where that order differs from sequential appends: a later append
// writes a page that a pending append's attention still reads (freed this step
// by that sequence and handed out again), copies a tail page that pending work
// writes, or belongs to a sequence that already has a pending append.
#pragma once
#include <map>
#include <unordered_map>
#include <memory>
#include <string>
#include <vector>

#include "miniprefix_b200.h"
#include "model_runner.h"

namespace miniprefix_b200 {

struct B200Options {
    int device = 0;
    int max_sequences = 256;      // live sequences (device block-table slots)
    int max_step_tokens = 4096;   // tokens of one device forward
    int max_step_sequences = 256; // appends of one device forward
    int timeout_ms = 600000;      // bounded wait of one forward
};

class B200Runner final : public ModelRunner {
public:
    B200Runner(const ModelConfig& config, int context, KvCacheConfig kv, B200Options options = {});
    ~B200Runner() override;
    B200Runner(const B200Runner&) = delete;
    B200Runner& operator=(const B200Runner&) = delete;

    // Weights (MPFX0001 names and [in, out] orientation); finalize before use.
    void set_weight(const std::string& name, const float* data, std::size_t elements);
    void finalize_weights();

    const ModelConfig& config() const override { return config_; }
    int context_limit() const override { return kv_.context_limit(); }
    KvAdmission reserve_request(const RequestId& id, std::size_t tokens) override { return kv_.reserve_request(id, tokens); }
    void release_reservation(const RequestId& id) noexcept override { kv_.release_reservation(id); }
    void create(const RequestId& id) override;
    void fork_sequence(const RequestId& source, const RequestId& target) override;
    std::size_t reuse_prefix(const RequestId& id, const std::vector<TokenId>& prompt) override;
    // inside a batch the publish runs while the batch's forward computes
    void cache_prefix(const RequestId& id) override { kv_.cache_prefix_deferred(id); }
    void clear_prefix_cache() override;
    std::vector<float> append(const RequestId& id, const std::vector<TokenId>& tokens) override;
    void release(const RequestId& id) override;
    void clear() override;
    RunnerStats stats() const override;
    CostStats cost_stats() const override;
    void set_cost_timing(bool enabled) override;
    std::size_t kv_block_tokens() const override { return std::size_t(kv_.config().block_tokens); }

    bool batched() const override { return true; }
    void begin_batch() override;
    std::size_t stage_append(const RequestId& id, const std::vector<TokenId>& tokens) override;
    void flush() override;
    void restore_batch() override;
    void fail_append(const RequestId& id, const std::vector<TokenId>& tokens) override;
    void end_batch() override;
    void set_replay(bool replay) override { replay_ = replay; }

    // Logits capture for parity checks of batched runs: while on, every flush also
    // downloads the logits of its staged appends (vocabulary floats each) and keeps
    // the latest ones per request (kept after the request is released, until
    // capture is switched off). Off by default; the hot path downloads greedy
    // tokens only.
    void set_logits_capture(bool on);
    // Copies the latest captured logits of `id` into `out`; false if there are none.
    bool captured_logits(const RequestId& id, std::vector<float>& out) const;

    // Introspection for tests and tools.
    const KVManager& kv() const { return kv_; }
    mp_context* device() const { return ctx_; }
    std::size_t flushes() const { return flushes_; }
    std::size_t hazard_flushes() const { return hazard_flushes_; }

private:
    int slot_of(const RequestId& id) const;
    void table_entries(int slot, const PagedSequence& sequence, std::vector<mp_table_entry>& out,
                       std::size_t from = 0);
    void free_slot(const RequestId& id);
    void mark_pending_reads(const RequestId& id);  // before a pending sequence drops its pages
    void drain() noexcept;  // best-effort completion of queued device work

    ModelConfig config_;
    KVManager kv_;
    B200Options options_;
    mp_context* ctx_ = nullptr;
    RunnerStats stats_;
    CostStats costs_;  // cow_* fields; lookup/publish come from the KV manager
    bool cost_timing_ = false;
    int table_stride_ = 0;

    std::unordered_map<RequestId, int> slots_;
    std::vector<int> free_slots_;
    std::vector<int> quarantine_;              // freed while device work may still read them
    std::vector<std::vector<int>> mirror_;     // device-known table of each slot
    std::vector<std::uint32_t> written_epoch_; // page -> epoch in which pending work writes it
    // page -> epoch in which it left a sequence whose pending append's attention
    // reads it (set when such a sequence is released or its table is replaced)
    std::vector<std::uint32_t> read_epoch_;
    std::vector<std::uint32_t> pending_epoch_; // slot -> epoch of its pending append

    // pending device work
    std::vector<mp_sequence_desc> descs_;
    std::vector<TokenId> tokens_;
    std::vector<mp_table_entry> entries_;
    std::vector<mp_tail_copy_region> regions_;
    std::vector<std::size_t> tickets_;
    std::vector<int32_t> out_tokens_, out_finite_;
    bool capture_ = false;
    std::vector<RequestId> pending_ids_;  // id of each pending append (capture only)
    std::vector<float> out_logits_;
    std::map<RequestId, std::vector<float>> captured_;
    std::uint32_t epoch_ = 1;
    bool replay_ = false;
    std::size_t flushes_ = 0, hazard_flushes_ = 0;

    // batch checkpoint of runner-side state
    struct Checkpoint {
        RunnerStats stats;
        CostStats costs;
        std::vector<std::pair<RequestId, int>> created;   // slots handed out in the window
        std::vector<std::pair<RequestId, int>> released;  // slots taken back in the window
    };
    std::unique_ptr<Checkpoint> checkpoint_;
};

}  // namespace miniprefix_b200
