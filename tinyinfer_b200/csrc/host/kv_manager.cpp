#include "kv_manager.h"

#include <algorithm>

namespace miniprefix_b200 {

namespace {
// Pages a request of `tokens` tokens may hold: its last token's page index + 1.
std::size_t pages_for(std::size_t tokens, int block_tokens) { return (tokens - 1) / std::size_t(block_tokens) + 1; }
// Whether `pages` more fit beside `committed` of `total` (never underflows).
bool fits(std::size_t committed, std::size_t pages, std::size_t total) {
    return committed <= total && pages <= total - committed;
}
}  // namespace

KVManager::KVManager(KvCacheConfig config, int layers, int width, int context, int vocabulary)
    : layers_(layers), width_(width), context_(context), vocabulary_(vocabulary), pool_(config, layers, width),
      prefix_(pool_) {
    const bool usable = context >= 1 && vocabulary >= 1;
    if (!usable) throw std::invalid_argument("invalid KV manager context/vocabulary");
}

KVManager::~KVManager() {
    checkpoint_.reset();
    pool_.attach_journal(nullptr);
    for (auto& item : sequences_) pool_.release(item.second.sequence);
    prefix_.clear();
}

std::size_t KVManager::max_sequence_blocks() const {
    const int bt = config().block_tokens;
    return std::size_t(context_ / bt + (context_ % bt != 0));
}

void KVManager::require_idle() const {
    if (append_active_) throw std::logic_error("KV append transaction is active");
}

KVManager::State& KVManager::idle_state(const RequestId& id) {
    require_idle();
    auto& state = sequences_.at(id);
    if (state.appending) throw std::logic_error("sequence has an active KV append");
    return state;
}

void KVManager::validate_tokens(const std::vector<TokenId>& tokens) const {
    const auto outside = [this](TokenId t) { return t < 0 || t >= vocabulary_; };
    if (std::any_of(tokens.begin(), tokens.end(), outside)) throw std::invalid_argument("invalid token");
}

// Pages held logically: every reservation, plus the pages of sequences that
// have no reservation (kv_manager.cpp:93-98).
std::size_t KVManager::committed_blocks() const {
    std::size_t count = reserved_pages_;
    for (const auto& [id, state] : sequences_)
        if (!reservations_.count(id)) count += state.sequence.blocks.size();
    return count;
}

void KVManager::touch_sequence(const RequestId& id, bool dropping, State* known) {
    if (!checkpoint_) return;
    auto& cp = *checkpoint_;
    State* state = known;
    if (!state) {
        auto it = sequences_.find(id);
        state = it != sequences_.end() ? &it->second : nullptr;
    }
    std::size_t slot;
    if (state && state->saved_window == cp.window) {
        slot = state->saved_slot;
    } else if (const auto known = cp.stateless.find(id); known != cp.stateless.end()) {
        slot = known->second;
    } else {
        SavedSequence saved;
        if (state) {
            const auto& s = state->sequence;
            saved.existed = true;
            saved.used = s.used;
            saved.block_count = s.blocks.size();
            saved.last_block = s.blocks.empty() ? -1 : s.blocks.back();
            saved.token_count = s.tokens.size();
        }
        slot = cp.sequences.size();
        cp.sequences.emplace_back(id, std::move(saved));
        if (!state) cp.stateless.emplace(id, slot);
    }
    if (state) {
        state->saved_window = cp.window;
        state->saved_slot = slot;
    }
    auto& saved = cp.sequences[slot].second;
    if (dropping) {
        // the State may be erased next: keep the entry reachable by id
        cp.stateless.emplace(id, slot);
        if (saved.existed && !saved.tokens) {
            const auto& s = sequences_.at(id).sequence;
            saved.tokens.emplace(s.tokens.begin(), s.tokens.begin() + std::ptrdiff_t(std::min(saved.token_count, s.tokens.size())));
            saved.blocks.emplace(s.blocks.begin(), s.blocks.begin() + std::ptrdiff_t(saved.block_count));
            if (saved.block_count) saved.blocks->back() = saved.last_block;
        }
    }
}

void KVManager::touch_reservation(const RequestId& id) {
    if (!checkpoint_ || checkpoint_->reservations.count(id)) return;
    auto it = reservations_.find(id);
    checkpoint_->reservations.emplace(id, it == reservations_.end() ? std::nullopt
                                                                    : std::optional<std::size_t>(it->second));
}

KvAdmission KVManager::reserve_request(const RequestId& id, std::size_t max_tokens) {
    settle_publishes();
    require_idle();
    const bool known = contains(id) || reservations_.count(id) != 0;
    if (known) throw std::invalid_argument("duplicate KV reservation");
    const bool in_context = max_tokens >= 1 && max_tokens <= std::size_t(context_);
    if (!in_context) throw std::invalid_argument("invalid KV reservation context");
    // no discount for pages another sequence already shares (kv_manager.cpp:46-51)
    const std::size_t need = pages_for(max_tokens, config().block_tokens);
    const std::size_t pool = std::size_t(config().max_blocks);
    if (need > pool) return KvAdmission::Impossible;
    if (!fits(committed_blocks(), need, pool)) return KvAdmission::Wait;
    touch_reservation(id);
    reservations_[id] = need;
    reserved_pages_ += need;
    return KvAdmission::Ready;
}

void KVManager::release_reservation(const RequestId& id) noexcept {
    auto it = reservations_.find(id);
    if (it == reservations_.end()) return;
    try {
        touch_reservation(id);
    } catch (...) {
    }
    reserved_pages_ -= it->second;
    reservations_.erase(it);
}

void KVManager::create(const RequestId& id) {
    settle_publishes();
    require_idle();
    if (sequences_.count(id)) throw std::invalid_argument("sequence already exists");
    touch_sequence(id);
    sequences_.emplace(id, State{});
}

void KVManager::fork_sequence(const RequestId& source, const RequestId& target) {
    settle_publishes();
    require_idle();
    const PagedSequence& from = sequences_.at(source).sequence;
    PagedSequence& into = idle_state(target).sequence;
    const bool empty_target = into.used == 0 && into.blocks.empty() && into.tokens.empty();
    if (source == target || !empty_target) throw std::invalid_argument("fork requires a distinct empty target");
    // The target takes every page of the source: within its reservation if it has
    // one, else within the pool's unreserved capacity.
    const std::size_t pages = from.blocks.size();
    if (const auto r = reservations_.find(target); r != reservations_.end()) {
        if (pages > r->second) throw KvCapacityError("fork exceeds KV reservation");
    } else if (!fits(committed_blocks(), pages, std::size_t(config().max_blocks))) {
        throw KvCapacityError("fork exceeds unreserved KV capacity");
    }
    PagedSequence shared = from;  // the host metadata is copied before any lease is taken
    touch_sequence(target);
    for (const int block : shared.blocks) pool_.retain(block);
    into = std::move(shared);
}

std::size_t KVManager::reuse_prefix(const RequestId& id, const std::vector<TokenId>& prompt) {
    settle_publishes();
    if (prompt.empty() || prompt.size() > std::size_t(context_)) throw std::invalid_argument("invalid prefix context");
    for (auto t : prompt)
        if (t < 0 || t >= vocabulary_) throw std::invalid_argument("invalid prefix token");
    auto& sequence = idle_state(id).sequence;
    ++costs_.lookup_calls;
    CostTimer timer(cost_timing_, costs_.lookup_ns);
    touch_sequence(id);
    const std::size_t count = std::size_t(prefix_.reuse(sequence, prompt));
    const auto reservation = reservations_.find(id);
    if (reservation != reservations_.end() && sequence.blocks.size() > reservation->second) {
        pool_.release(sequence);
        throw KvCapacityError("request exceeds KV reservation");
    }
    if (!reservations_.empty() && committed_blocks() > std::size_t(config().max_blocks)) {
        pool_.release(sequence);
        throw KvCapacityError("KV capacity reserved by active requests");
    }
    return count;
}

void KVManager::publish(State& state) {
    ++costs_.publish_calls;
    CostTimer timer(cost_timing_, costs_.publish_ns);
    prefix_.publish(state.sequence);
}

void KVManager::cache_prefix(const RequestId& id) {
    settle_publishes();
    publish(idle_state(id));
}

void KVManager::cache_prefix_deferred(const RequestId& id) {
    if (!checkpoint_) return cache_prefix(id);
    require_idle();
    State& state = last_append_ && last_append_id_ == id ? *last_append_ : idle_state(id);
    // a publish that would fail fails here, where the caller made it
    if (state.publish_queued || state.sequence.tokens.size() != std::size_t(state.sequence.used))
        return cache_prefix(id);
    state.publish_queued = true;
    pending_publishes_.push_back(&state);
}

void KVManager::settle_publishes() {
    // (not inside an append transaction: the queue waits for its end)
    if (pending_publishes_.empty() || append_active_) return;
    settling_.swap(pending_publishes_);
    struct Drop {  // a failure drops the rest, as it would end the step
        std::vector<State*>& v;
        ~Drop() { v.clear(); }
    } drop{settling_};
    for (State* s : settling_) s->publish_queued = false;
    for (State* s : settling_) publish(*s);
}

// A queued publish changes the prefix index, leases (page references) and LRU
// order, and frees a page only by evicting the last lease of a cache-only page.
// So an append commutes with the queue when it copies no page (its partial last
// page has no other holder), and any pages it takes from the free list come
// without an eviction while no page is cache-only (the queue then frees none).
bool KVManager::commutes_with_publishes(const State& state, std::size_t tokens) const {
    const auto& sequence = state.sequence;
    const std::size_t bt = std::size_t(config().block_tokens);
    const std::size_t end = std::size_t(sequence.used) + tokens;
    if (state.publish_queued) return false;
    if (sequence.used % int(bt) && pool_.references(sequence.blocks.back()) != 1) return false;  // may copy
    const std::size_t count = (end + bt - 1) / bt;
    if (count <= sequence.blocks.size()) return true;
    return pool_.cache_only_blocks() == 0 && pool_.free_blocks() >= count - sequence.blocks.size();
}

CostStats KVManager::cost_stats() const {
    settle_for_read();
    return costs_;
}

void KVManager::clear_prefix_cache() {
    settle_publishes();
    require_idle();
    for (const auto& item : sequences_)
        if (item.second.appending) throw std::logic_error("cannot clear prefix cache during KV append");
    prefix_.clear();
}

void KVManager::reserve_pages(const RequestId& id, PagedSequence& sequence, int end, bool& cow) {
    const int bt = config().block_tokens;
    const std::size_t count = std::size_t(end / bt + (end % bt != 0));
    const std::size_t required = count > sequence.blocks.size() ? count - sequence.blocks.size() : 0;
    if (!reservations_.empty()) {
        const auto found = reservations_.find(id);
        if (found != reservations_.end()) {
            if (count > found->second) throw KvCapacityError("request exceeds KV reservation");
        } else {
            const std::size_t committed = committed_blocks(), total = std::size_t(config().max_blocks);
            if (committed > total || required > total - committed)
                throw KvCapacityError("KV capacity reserved by active requests");
        }
    }
    // Evict LRU cache leases while physically short; a victim may have been the
    // only other holder of the shared tail, which then needs no copy.
    while (pool_.free_blocks() < required + std::size_t(cow) && prefix_.evict_one())
        if (cow && pool_.references(sequence.blocks.back()) == 1) cow = false;
    if (cow && pool_.free_blocks() < required + 1) throw KvCapacityError("paged KV block pool exhausted");
    pool_.reserve(sequence, end);
}

KVManager::Append::Append(KVManager& owner, const RequestId& id, const std::vector<TokenId>& tokens)
    : owner_(&owner), id_(id), state_(&owner.idle_state(id)), tokens_(&tokens),
      original_blocks_(state_->sequence.blocks.size()) {
    auto& sequence = state_->sequence;
    if (!owner.pending_publishes_.empty() && !owner.commutes_with_publishes(*state_, tokens.size()))
        owner.settle_publishes();
    if (tokens.empty() || tokens.size() > std::size_t(owner.context_ - sequence.used))
        throw std::invalid_argument("context overflow/empty input");
    owner.validate_tokens(tokens);
    owner.touch_sequence(id, false, state_);
    // room for the commit up front (commit must not allocate); grow geometrically,
    // an exact reserve would copy the whole history on every decode append
    const std::size_t need = std::size_t(sequence.used) + tokens.size();
    if (sequence.tokens.capacity() < need) sequence.tokens.reserve(std::max(need, 2 * sequence.tokens.capacity()));
    const int valid = sequence.used % owner.config().block_tokens;
    bool cow = valid && owner.pool_.references(sequence.blocks.back()) > 1;
    owner.reserve_pages(id, sequence, sequence.used + int(tokens.size()), cow);
    if (cow) {
        const int old = sequence.blocks[original_blocks_ - 1];
        const int replacement = owner.pool_.allocate();
        copy_ = TailCopy{old, replacement, valid};
        sequence.blocks[original_blocks_ - 1] = replacement;
    }
    state_->appending = true;
    owner.append_active_ = true;
}

KVManager::Append::~Append() { rollback(); }

const PagedSequence& KVManager::Append::sequence() const {
    if (!owner_) throw std::logic_error("KV append already finished");
    return state_->sequence;
}

void KVManager::Append::copy_shared_tail(const std::function<void(std::size_t, std::size_t, std::size_t)>& copier) {
    copy_shared_tail_region([&](const TailCopyRegion& r) {
        for (std::size_t row = 0; row < r.rows; ++row)
            copier(r.destination + row * r.pitch, r.source + row * r.pitch, r.width);
    });
}

void KVManager::Append::copy_shared_tail_region(const std::function<void(const TailCopyRegion&)>& copier) {
    if (!owner_) throw std::logic_error("KV append already finished");
    if (!copy_) return;
    copied_ = false;
    const std::size_t pitch = std::size_t(owner_->config().block_tokens) * std::size_t(owner_->width_);
    const std::size_t rows = std::size_t(owner_->layers_);
    copier({std::size_t(copy_->destination) * rows * pitch, std::size_t(copy_->source) * rows * pitch, pitch,
            std::size_t(copy_->valid_tokens) * std::size_t(owner_->width_), rows});
    copied_ = true;
}

void KVManager::Append::commit() {
    if (!owner_) throw std::logic_error("KV append already finished");
    if (copy_ && !copied_) throw std::logic_error("shared tail payload was not copied");
    auto& sequence = state_->sequence;
    sequence.tokens.insert(sequence.tokens.end(), tokens_->begin(), tokens_->end());
    sequence.used += int(tokens_->size());
    owner_->forward_tokens_ += tokens_->size();
    if (copy_) owner_->pool_.unref(copy_->source);
    state_->appending = false;
    owner_->append_active_ = false;
    owner_->last_append_ = state_;
    owner_->last_append_id_ = id_;
    owner_ = nullptr;
}

void KVManager::Append::rollback() noexcept {
    if (!owner_) return;
    owner_->pool_.rollback(state_->sequence, original_blocks_);
    if (copy_) {
        state_->sequence.blocks[original_blocks_ - 1] = copy_->source;
        owner_->pool_.unref(copy_->destination);
    }
    state_->appending = false;
    owner_->append_active_ = false;
    owner_ = nullptr;
}

void KVManager::reset_sequence(const RequestId& id) {
    settle_publishes();
    auto& state = idle_state(id);
    touch_sequence(id, true);
    pool_.release(state.sequence);
}

void KVManager::release(const RequestId& id) {
    settle_publishes();
    require_idle();
    auto it = sequences_.find(id);
    if (it == sequences_.end()) throw std::invalid_argument("unknown sequence");
    if (it->second.appending) throw std::logic_error("cannot release sequence during KV append");
    touch_sequence(id, true);
    touch_reservation(id);
    pool_.release(it->second.sequence);
    last_append_ = nullptr;
    sequences_.erase(it);
    auto r = reservations_.find(id);
    if (r != reservations_.end()) {
        reserved_pages_ -= r->second;
        reservations_.erase(r);
    }
}

void KVManager::clear() {
    settle_publishes();
    require_idle();
    for (const auto& item : sequences_)
        if (item.second.appending) throw std::logic_error("cannot clear sequences during KV append");
    for (auto& item : sequences_) {
        touch_sequence(item.first, true);
        pool_.release(item.second.sequence);
    }
    last_append_ = nullptr;
    sequences_.clear();
    prefix_.clear();
    for (const auto& r : reservations_) touch_reservation(r.first);
    reservations_.clear();
    reserved_pages_ = 0;
}

KvStats KVManager::stats() const {
    settle_for_read();
    KvStats r;
    r.live_sequences = sequences_.size();
    r.forward_tokens = forward_tokens_;
    r.kv_block_tokens = std::size_t(config().block_tokens);
    r.kv_total_blocks = std::size_t(config().max_blocks);
    r.kv_live_blocks = pool_.live_blocks();
    r.kv_peak_blocks = pool_.peak_blocks();
    r.kv_reserved_bytes = pool_.reserved_bytes();
    r.live_kv_bytes = pool_.live_blocks() * pool_.block_bytes();
    r.peak_kv_bytes = pool_.peak_blocks() * pool_.block_bytes();
    r.prefix_cache_capacity = std::size_t(config().prefix_cache_blocks);
    r.kv_cached_blocks = prefix_.size();
    r.kv_cache_only_blocks = prefix_.cache_only_blocks();
    r.prefix_hits = prefix_.hits();
    r.prefix_misses = prefix_.misses();
    r.prefix_reused_tokens = prefix_.reused_tokens();
    r.prefix_evictions = prefix_.evictions();
    return r;
}

void KVManager::begin_checkpoint() {
    settle_publishes();
    require_idle();
    checkpoint_ = spare_checkpoint_ ? std::move(spare_checkpoint_) : std::make_unique<Checkpoint>();
    checkpoint_->window = ++windows_;
    checkpoint_->live = pool_.live_blocks();
    checkpoint_->peak = pool_.peak_blocks();
    prefix_.begin_journal();
    checkpoint_->reserved_pages = reserved_pages_;
    checkpoint_->forward_tokens = forward_tokens_;
    checkpoint_->costs = costs_;
    pool_.attach_journal(&checkpoint_->pool_journal);
}

void KVManager::restore_checkpoint() {
    if (!checkpoint_) throw std::logic_error("no KV checkpoint");
    for (State* s : pending_publishes_) s->publish_queued = false;
    pending_publishes_.clear();  // never applied: nothing of them to undo
    auto& cp = *checkpoint_;
    last_append_ = nullptr;
    pool_.attach_journal(nullptr);
    pool_.undo(cp.pool_journal, 0, cp.live, cp.peak);
    prefix_.rollback_journal();
    for (auto& [id, saved] : cp.sequences) {
        if (!saved.existed) {
            sequences_.erase(id);
            continue;
        }
        auto& state = sequences_[id];
        state.appending = false;
        state.sequence.used = saved.used;
        if (saved.blocks) {
            state.sequence.blocks = std::move(*saved.blocks);
        } else {
            state.sequence.blocks.resize(saved.block_count);
            if (saved.block_count) state.sequence.blocks.back() = saved.last_block;
        }
        if (saved.tokens) state.sequence.tokens = std::move(*saved.tokens);
        else state.sequence.tokens.resize(saved.token_count);
    }
    for (auto& [id, pages] : cp.reservations) {
        if (pages) reservations_[id] = *pages;
        else reservations_.erase(id);
    }
    reserved_pages_ = cp.reserved_pages;
    forward_tokens_ = cp.forward_tokens;
    costs_ = cp.costs;
    append_active_ = false;
    close_checkpoint();
}

void KVManager::close_checkpoint() {
    if (!checkpoint_) return;
    checkpoint_->recycle();
    spare_checkpoint_ = std::move(checkpoint_);
}

void KVManager::end_checkpoint() {
    settle_publishes();
    pool_.attach_journal(nullptr);
    prefix_.end_journal();
    close_checkpoint();
}

}  // namespace miniprefix_b200
