// The runner surface the Engine drives: the reference ModelRunner
// (miniprefix/include/miniprefix/model.h:35-58), extended with a staged batch
// interface so that one step's appends run as ONE device forward.
//
// Batch contract (engine side):
//   begin_batch()                 checkpoint all host state
//   stage_append(id, tokens)      host bookkeeping of one append, as append()
//                                 does it, committed at once; the device work
//                                 joins the pending batch. Returns a ticket.
//   flush()                       run the pending device work, results by ticket
//   result(ticket)                greedy token and finiteness of that append
//   restore_batch()               return host state to the checkpoint
//   fail_append(id, tokens)       host effects of an append whose forward failed:
//                                 prepare, COW accounting, roll back, throw
//   end_batch()                   drop the checkpoint
#pragma once
#include <memory>

#include "kv_manager.h"

namespace miniprefix_b200 {

class ModelRunner {
public:
    virtual ~ModelRunner() = default;
    virtual const ModelConfig& config() const = 0;
    virtual int context_limit() const = 0;
    virtual KvAdmission reserve_request(const RequestId&, std::size_t) { return KvAdmission::Ready; }
    virtual void release_reservation(const RequestId&) noexcept {}
    virtual void create(const RequestId&) = 0;
    virtual void fork_sequence(const RequestId&, const RequestId&) { throw std::logic_error("fork unsupported"); }
    virtual std::size_t reuse_prefix(const RequestId&, const std::vector<TokenId>&) { return 0; }
    virtual void cache_prefix(const RequestId&) {}
    virtual void clear_prefix_cache() {}
    virtual std::vector<float> append(const RequestId&, const std::vector<TokenId>&) = 0;
    virtual void release(const RequestId&) = 0;
    virtual void clear() = 0;
    virtual RunnerStats stats() const = 0;
    virtual CostStats cost_stats() const { return {}; }
    virtual void set_cost_timing(bool) {}
    // Cheap accessor used by the engine where the reference reads stats().kv_block_tokens.
    virtual std::size_t kv_block_tokens() const { return stats().kv_block_tokens; }

    // ---- staged batches (see file comment). A runner without batch support
    // executes each staged append at once through append().
    struct AppendResult {
        TokenId token = 0;
        bool finite = true;
    };
    virtual bool batched() const { return false; }
    virtual void begin_batch() {}
    virtual std::size_t stage_append(const RequestId& id, const std::vector<TokenId>& tokens);
    virtual void flush() {}
    virtual AppendResult result(std::size_t ticket) const { return results_.at(ticket); }
    virtual void restore_batch() {}
    virtual void fail_append(const RequestId&, const std::vector<TokenId>&) {
        throw std::logic_error("fail_append requires a batched runner");
    }
    virtual void end_batch() { results_.clear(); }
    // While replaying a restored step, staged appends do host work only.
    virtual void set_replay(bool) {}

protected:
    std::vector<AppendResult> results_;
};

}  // namespace miniprefix_b200
