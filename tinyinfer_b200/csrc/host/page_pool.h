// Physical page ownership of the paged KV pools (host side).
//
// Same contract as the reference KvBlockPool (miniprefix/include/miniprefix/
// paged_kv.h:25-51, miniprefix/src/kv/paged_kv.cpp): a LIFO free list whose first
// hand-outs are pages 0, 1, 2, ... and to whose back freed pages return, per-page
// reference counts, live/peak counters, atomic multi-page reservation, and the
// element offset of (page, layer, slot) in [block][layer][slot][width] storage.
// Page ids are therefore identical to the reference's for any operation sequence.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include "types.h"

namespace miniprefix_b200 {

class KvBlockPool {
public:
    KvBlockPool(KvCacheConfig config, int layers, int width);

    const KvCacheConfig& config() const { return config_; }
    std::size_t block_elements() const { return block_elements_; }
    std::size_t block_bytes() const { return block_elements_ * sizeof(float) * 2; }
    std::size_t reserved_bytes() const { return block_bytes() * std::size_t(config_.max_blocks); }
    std::size_t live_blocks() const { return live_; }
    std::size_t peak_blocks() const { return peak_; }
    std::size_t free_blocks() const { return free_.size(); }
    // Throws std::out_of_range for a page outside the pool.
    std::size_t references(int block) const { return refs_.at(std::size_t(block)); }
    // Prefix-cache leases per page (index nodes holding it; each is also one of the
    // page's references), kept beside the references so that the number of
    // cache-only pages -- leased, and every reference a lease -- is exact at all times.
    std::size_t leases(int block) const { return leases_[std::size_t(block)]; }
    void add_lease(int block, int delta) noexcept;
    std::size_t cache_only_blocks() const { return cache_only_; }

    int allocate();
    void retain(int block);
    void unref(int block) noexcept;
    // Grows `sequence.blocks` to cover `end` tokens; all-or-nothing.
    void reserve(PagedSequence& sequence, int end);
    void rollback(PagedSequence& sequence, std::size_t original_blocks) noexcept;
    void release(PagedSequence& sequence) noexcept;
    std::size_t offset(const PagedSequence& sequence, int layer, int token, int layers, int width) const;

    // Undo journal support (used by the batched engine to restore the exact pool
    // state of a failed step). When a journal is attached every mutation records
    // an inverse operation.
    struct JournalEntry {
        enum Kind : std::uint8_t { Popped, Pushed, RefUp, RefDown } kind;
        int block;
    };
    void attach_journal(std::vector<JournalEntry>* journal) { journal_ = journal; }
    // Free epochs: a page freed since the last next_epoch() call may still be read
    // by device work queued before it was freed (used by batched runners).
    bool freed_this_epoch(int block) const { return freed_epoch_[std::size_t(block)] == epoch_; }
    void next_epoch() { ++epoch_; }
    void undo(const std::vector<JournalEntry>& journal, std::size_t mark, std::size_t live, std::size_t peak) noexcept;

private:
    void record(JournalEntry::Kind kind, int block) {
        if (journal_) journal_->push_back({kind, block});
    }
    bool cache_only(std::size_t block) const { return leases_[block] && refs_[block] == leases_[block]; }
    void set_refs(std::size_t block, std::uint32_t refs) noexcept;  // every reference count write
    KvCacheConfig config_;
    std::size_t block_elements_ = 0;
    std::vector<int> free_;  // back() is handed out next
    std::vector<std::uint32_t> refs_;
    std::vector<std::uint32_t> leases_;
    std::size_t cache_only_ = 0;
    std::size_t live_ = 0, peak_ = 0;
    std::vector<JournalEntry>* journal_ = nullptr;
    std::vector<std::uint32_t> freed_epoch_;
    std::uint32_t epoch_ = 1;
};

}  // namespace miniprefix_b200
