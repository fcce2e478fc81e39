#include "page_pool.h"

#include <algorithm>
#include <limits>

namespace miniprefix_b200 {

KvBlockPool::KvBlockPool(KvCacheConfig config, int layers, int width) : config_(config) {
    if (config.block_tokens < 1 || config.max_blocks < 1 || layers < 1 || width < 1 || config.prefix_cache_blocks < 0 ||
        config.prefix_cache_blocks > config.max_blocks)
        throw std::invalid_argument("invalid paged KV configuration");
    // Both pools together must stay addressable in bytes.
    const std::size_t limit = std::numeric_limits<std::size_t>::max() / sizeof(float) / 2;
    std::size_t total = std::size_t(layers);
    for (int factor : {config.block_tokens, width, config.max_blocks}) {
        if (total > limit / std::size_t(factor)) throw std::invalid_argument("paged KV size overflow");
        total *= std::size_t(factor);
    }
    block_elements_ = total / std::size_t(config.max_blocks);
    refs_.assign(std::size_t(config.max_blocks), 0);
    leases_.assign(std::size_t(config.max_blocks), 0);
    freed_epoch_.assign(std::size_t(config.max_blocks), 0);
    free_.resize(std::size_t(config.max_blocks));
    // Descending, so that pages 0, 1, 2, ... are handed out first.
    for (int i = 0; i < config.max_blocks; ++i) free_[std::size_t(i)] = config.max_blocks - 1 - i;
}

void KvBlockPool::set_refs(std::size_t block, std::uint32_t refs) noexcept {
    const bool before = cache_only(block);
    refs_[block] = refs;
    cache_only_ = cache_only_ + std::size_t(cache_only(block)) - std::size_t(before);
}

void KvBlockPool::add_lease(int block, int delta) noexcept {
    const std::size_t b = std::size_t(block);
    const bool before = cache_only(b);
    leases_[b] = std::uint32_t(int(leases_[b]) + delta);
    cache_only_ = cache_only_ + std::size_t(cache_only(b)) - std::size_t(before);
}

int KvBlockPool::allocate() {
    if (free_.empty()) throw KvCapacityError("paged KV block pool exhausted");
    const int block = free_.back();
    free_.pop_back();
    set_refs(std::size_t(block), 1);
    ++live_;
    peak_ = std::max(peak_, live_);
    record(JournalEntry::Popped, block);
    return block;
}

void KvBlockPool::retain(int block) {
    set_refs(std::size_t(block), refs_.at(std::size_t(block)) + 1);
    record(JournalEntry::RefUp, block);
}

void KvBlockPool::unref(int block) noexcept {
    set_refs(std::size_t(block), refs_[std::size_t(block)] - 1);
    if (refs_[std::size_t(block)] == 0) {
        free_.push_back(block);
        --live_;
        freed_epoch_[std::size_t(block)] = epoch_;
        record(JournalEntry::Pushed, block);
    } else {
        record(JournalEntry::RefDown, block);
    }
}

void KvBlockPool::reserve(PagedSequence& sequence, int end) {
    if (end < sequence.used) throw std::invalid_argument("paged KV cannot truncate through reserve");
    const int bt = config_.block_tokens;
    const std::size_t needed = std::size_t(end / bt + (end % bt != 0));
    if (needed <= sequence.blocks.size()) return;
    if (needed - sequence.blocks.size() > free_.size()) throw KvCapacityError("paged KV block pool exhausted");
    if (sequence.blocks.capacity() < needed) sequence.blocks.reserve(std::max(needed, 2 * sequence.blocks.capacity()));
    while (sequence.blocks.size() < needed) {
        const int block = free_.back();
        free_.pop_back();
        set_refs(std::size_t(block), 1);
        ++live_;
        sequence.blocks.push_back(block);
        record(JournalEntry::Popped, block);
    }
    peak_ = std::max(peak_, live_);
}

void KvBlockPool::rollback(PagedSequence& sequence, std::size_t original_blocks) noexcept {
    while (sequence.blocks.size() > original_blocks) {
        unref(sequence.blocks.back());
        sequence.blocks.pop_back();
    }
}

void KvBlockPool::release(PagedSequence& sequence) noexcept {
    rollback(sequence, 0);
    sequence.used = 0;
    sequence.tokens.clear();
}

std::size_t KvBlockPool::offset(const PagedSequence& sequence, int layer, int token, int layers, int width) const {
    const int bt = config_.block_tokens;
    const std::size_t page = std::size_t(sequence.blocks.at(std::size_t(token / bt)));
    return ((page * std::size_t(layers) + std::size_t(layer)) * std::size_t(bt) + std::size_t(token % bt)) *
           std::size_t(width);
}

void KvBlockPool::undo(const std::vector<JournalEntry>& journal, std::size_t mark, std::size_t live,
                       std::size_t peak) noexcept {
    for (std::size_t i = journal.size(); i-- > mark;) {
        const auto& e = journal[i];
        const std::size_t b = std::size_t(e.block);
        switch (e.kind) {
            case JournalEntry::Popped:  // was free with 0 references, at the back
                set_refs(b, 0);
                free_.push_back(e.block);
                break;
            case JournalEntry::Pushed:  // was live with 1 reference
                free_.pop_back();
                set_refs(b, 1);
                break;
            case JournalEntry::RefUp: set_refs(b, refs_[b] - 1); break;
            case JournalEntry::RefDown: set_refs(b, refs_[b] + 1); break;
        }
    }
    live_ = live;
    peak_ = peak;
}

}  // namespace miniprefix_b200
