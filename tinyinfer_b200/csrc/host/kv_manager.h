// Sequence metadata, page references, reservations and prefix leases of one
// runner (host side). Payload, device tables and completion stay in the backend.
// Single-threaded API.
//
// Contract of the reference KVManager (miniprefix/include/miniprefix/kv_manager.h:18-96,
// miniprefix/src/kv/kv_manager.cpp), including every error class and message:
// logical reservations of 1+(max_tokens-1)/block_tokens pages without a sharing
// discount (:99-109), forks that share all pages (:115-130), prefix reuse with
// reservation checks (:131-145), and the Append transaction (:157-242): validate,
// reserve pages (evicting LRU cache leases while physically short, re-checking
// after every victim whether a shared partial tail still needs its copy-on-write
// page, :174-183), allocate the COW replacement, then commit or roll back.
//
// Batched steps: begin_checkpoint()/restore_checkpoint() bracket a window in
// which every mutation is recorded so that the exact state at the checkpoint can
// be restored (pages, references, free-list order, sequences, reservations,
// prefix index and counters).
//
// Inside a window a publish may wait (cache_prefix_deferred): queued publishes
// run in call order at settle_publishes(), and before any operation whose
// outcome they could change -- every public operation except an append that
// commutes with them (commutes_with_publishes), so every page, reference,
// free-list and index state matches the un-deferred order. A runner publishes
// the queue while its device forward runs.
#pragma once
#include <functional>
#include <map>
#include <unordered_map>
#include <memory>
#include <optional>

#include "prefix_cache.h"

namespace miniprefix_b200 {

class KVManager {
    struct State {
        PagedSequence sequence;
        bool appending = false;
        bool publish_queued = false;  // in pending_publishes_
        // journal entry of this sequence in the open checkpoint window (valid while
        // saved_window equals the window's number)
        std::uint64_t saved_window = 0;
        std::size_t saved_slot = 0;
    };

public:
    struct TailCopy {
        int source, destination, valid_tokens;
    };
    // Float-element offsets into ONE pool; rows are layers. Copy K and V alike.
    struct TailCopyRegion {
        std::size_t destination, source, pitch, width, rows;
    };

    class Append {
        friend class KVManager;
        KVManager* owner_;
        RequestId id_;
        State* state_;
        const std::vector<TokenId>* tokens_;  // the caller's tokens; they outlive the transaction
        std::size_t original_blocks_;
        std::optional<TailCopy> copy_;
        bool copied_ = false;
        Append(KVManager& owner, const RequestId& id, const std::vector<TokenId>& tokens);

    public:
        Append(const Append&) = delete;
        Append& operator=(const Append&) = delete;
        Append(Append&&) = delete;
        Append& operator=(Append&&) = delete;
        ~Append();
        const PagedSequence& sequence() const;
        std::size_t original_blocks() const { return original_blocks_; }
        const std::optional<TailCopy>& tail_copy() const { return copy_; }
        void copy_shared_tail(const std::function<void(std::size_t, std::size_t, std::size_t)>& copier);
        void copy_shared_tail_region(const std::function<void(const TailCopyRegion&)>& copier);
        void commit();
        void rollback() noexcept;
    };

    KVManager(KvCacheConfig config, int layers, int width, int context, int vocabulary);
    KVManager(const KVManager&) = delete;
    KVManager& operator=(const KVManager&) = delete;
    ~KVManager();

    const KvCacheConfig& config() const { return pool_.config(); }
    int context_limit() const { return context_; }
    std::size_t reserved_bytes() const { return pool_.reserved_bytes(); }
    std::size_t max_sequence_blocks() const;
    bool contains(const RequestId& id) const { return sequences_.count(id) != 0; }
    const PagedSequence& sequence(const RequestId& id) const { return sequences_.at(id).sequence; }
    std::size_t offset(const PagedSequence& sequence, int layer, int token) const {
        return pool_.offset(sequence, layer, token, layers_, width_);
    }
    KvAdmission reserve_request(const RequestId& id, std::size_t max_tokens);
    void release_reservation(const RequestId& id) noexcept;
    void create(const RequestId& id);
    void fork_sequence(const RequestId& source, const RequestId& target);
    std::size_t reuse_prefix(const RequestId& id, const std::vector<TokenId>& prompt);
    void cache_prefix(const RequestId& id);
    void cache_prefix_deferred(const RequestId& id);  // cache_prefix, queued inside a checkpoint window
    void settle_publishes();
    void clear_prefix_cache();
    Append prepare_append(const RequestId& id, const std::vector<TokenId>& tokens) {
        return Append(*this, id, tokens);
    }
    void reset_sequence(const RequestId& id);
    void release(const RequestId& id);
    void clear();
    KvStats stats() const;
    void set_cost_timing(bool enabled) { cost_timing_ = enabled; }
    CostStats cost_stats() const;
    const KvBlockPool& pool() const { return pool_; }
    bool freed_this_epoch(int block) const { return pool_.freed_this_epoch(block); }
    void next_epoch() { pool_.next_epoch(); }

    // ---- checkpoints for batched steps
    void begin_checkpoint();
    void restore_checkpoint();
    void end_checkpoint();

private:
    void require_idle() const;
    State& idle_state(const RequestId& id);
    void validate_tokens(const std::vector<TokenId>& tokens) const;
    std::size_t committed_blocks() const;
    void reserve_pages(const RequestId& id, PagedSequence& sequence, int end, bool& cow);
    // journal a sequence mutation; `known` is id's State when the caller has it
    void touch_sequence(const RequestId& id, bool dropping = false, State* known = nullptr);
    void touch_reservation(const RequestId& id);
    void publish(State& state);
    bool commutes_with_publishes(const State& state, std::size_t tokens) const;
    // Readers see the state after every queued publish (the queue is an
    // evaluation-order detail, not part of the observable state).
    void settle_for_read() const { const_cast<KVManager*>(this)->settle_publishes(); }

    int layers_, width_, context_, vocabulary_;
    KvBlockPool pool_;
    ExactPrefixCache prefix_;
    std::map<RequestId, State> sequences_;
    std::unordered_map<RequestId, std::size_t> reservations_;
    std::size_t reserved_pages_ = 0;  // sum of reservations_
    std::size_t forward_tokens_ = 0;
    bool append_active_ = false;
    bool cost_timing_ = false;
    CostStats costs_;
    // Queued publishes, in call order. A queued sequence is never erased: every
    // operation that can erase one settles or (restore) drops the queue first.
    std::vector<State*> pending_publishes_;
    std::vector<State*> settling_;  // the queue being applied (keeps its capacity)
    // the sequence of the last committed append (its id is the map key), so that
    // the publish that follows an append finds it without a lookup; cleared when
    // any sequence is erased
    State* last_append_ = nullptr;
    RequestId last_append_id_;

    // A sequence as it was at the checkpoint. Tokens only grow inside a window
    // unless the sequence is released, so only their count is kept until then.
    // A sequence's state at the checkpoint. Until it is dropped, an append can
    // only replace its last page (copy on write) and add pages after it, so the
    // page count and the last page restore it; a drop saves the full lists.
    struct SavedSequence {
        bool existed = false;
        int used = 0;
        std::size_t block_count = 0;
        int last_block = -1;
        std::optional<std::vector<int>> blocks;
        std::size_t token_count = 0;
        std::optional<std::vector<std::int32_t>> tokens;
    };
    struct Checkpoint {
        std::uint64_t window = 0;  // number of this checkpoint window
        std::vector<KvBlockPool::JournalEntry> pool_journal;
        std::size_t live = 0, peak = 0;
        // every sequence touched in the window, once, in first-touch order; a
        // sequence's entry is found through its State (saved_window / saved_slot)
        // or, while it has no State (created or dropped in the window), by id
        std::vector<std::pair<RequestId, SavedSequence>> sequences;
        std::unordered_map<RequestId, std::size_t> stateless;
        std::map<RequestId, std::optional<std::size_t>> reservations;  // nullopt: did not exist
        std::size_t reserved_pages = 0, forward_tokens = 0;
        CostStats costs;
        // empties the journals, keeping their storage for the next window
        void recycle() {
            pool_journal.clear();
            sequences.clear();
            stateless.clear();
            reservations.clear();
        }
    };
    std::unique_ptr<Checkpoint> checkpoint_;
    std::unique_ptr<Checkpoint> spare_checkpoint_;  // a closed window's storage, reused by the next
    void close_checkpoint();
    std::uint64_t windows_ = 0;  // checkpoint windows opened so far
};

}  // namespace miniprefix_b200
