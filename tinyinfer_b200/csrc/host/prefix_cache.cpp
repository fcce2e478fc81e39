#include "prefix_cache.h"

#include <algorithm>
#include <iterator>

namespace miniprefix_b200 {

ExactPrefixCache::ExactPrefixCache(KvBlockPool& pool) : pool_(pool) {
    s_.nodes.emplace_back();
}

ExactPrefixCache::~ExactPrefixCache() { clear(); }

std::size_t ExactPrefixCache::cache_only_blocks() const { return pool_.cache_only_blocks(); }

void ExactPrefixCache::lease_add(int page, int delta) {
    log(Op::Lease, page, delta);
    pool_.add_lease(page, delta);
}

int ExactPrefixCache::new_node(int parent, View edge) {
    int id;
    const bool spare = !s_.spare.empty();
    if (spare) {
        id = s_.spare.back();
        s_.spare.pop_back();
    } else {
        id = int(s_.nodes.size());
        s_.nodes.emplace_back();
    }
    log(Op::NewNode, id, parent, spare ? 1 : 0);
    Node& n = s_.nodes[std::size_t(id)];
    n.parent = parent;
    n.edge.assign(edge.p, edge.p + edge.n);
    n.block = -1;
    n.stamp = 0;
    n.prev = n.next = -1;
    n.children.clear();
    n.leased.clear();
    s_.nodes[std::size_t(parent)].children.insert(view(n.edge), id);
    ++s_.live_nodes;
    s_.key_tokens += edge.n;
    return id;
}

// The stamp a node had when the undo window opened is all a rollback needs, so
// it is journaled at the node's first stamp change in the window only.
void ExactPrefixCache::log_stamp(Node& n, int id) {
    if (journaling_ && n.logged != window_) {
        log(Op::Stamp, id, 0, n.stamp);
        n.logged = window_;
    }
}

void ExactPrefixCache::touch(int id) {
    Node& n = s_.nodes[std::size_t(id)];
    log_stamp(n, id);
    if (s_.lru_last != id) {
        if (n.stamp) {  // unlink; a listed node that is not the tail has a successor
            if (n.prev >= 0) s_.nodes[std::size_t(n.prev)].next = n.next;
            else s_.lru_first = n.next;
            s_.nodes[std::size_t(n.next)].prev = n.prev;
        }
        n.prev = s_.lru_last;
        n.next = -1;
        if (s_.lru_last >= 0) s_.nodes[std::size_t(s_.lru_last)].next = id;
        else s_.lru_first = id;
        s_.lru_last = id;
    }
    n.stamp = ++s_.clock;
}

void ExactPrefixCache::unstamp(int id) noexcept {
    Node& n = s_.nodes[std::size_t(id)];
    log_stamp(n, id);
    if (n.stamp) {
        if (n.prev >= 0) s_.nodes[std::size_t(n.prev)].next = n.next;
        else s_.lru_first = n.next;
        if (n.next >= 0) s_.nodes[std::size_t(n.next)].prev = n.prev;
        else s_.lru_last = n.prev;
    }
    n.prev = n.next = -1;
    n.stamp = 0;
}

// Links every leased node (stamp != 0) in stamp order. Used after a rollback has
// restored the stamps; `relink_` was reserved for all nodes when the window opened
// and a rollback never leaves more nodes than that.
void ExactPrefixCache::relink_lru() noexcept {
    relink_.clear();
    for (std::size_t id = 1; id < s_.nodes.size(); ++id)
        if (s_.nodes[id].stamp) relink_.emplace_back(s_.nodes[id].stamp, int(id));
    std::sort(relink_.begin(), relink_.end());
    s_.lru_first = s_.lru_last = -1;
    for (const auto& [stamp, id] : relink_) {
        Node& n = s_.nodes[std::size_t(id)];
        n.prev = s_.lru_last;
        n.next = -1;
        if (s_.lru_last >= 0) s_.nodes[std::size_t(s_.lru_last)].next = id;
        else s_.lru_first = id;
        s_.lru_last = id;
    }
}

// Erase empty structural leaves from `id` upward, never the root or `keep`.
void ExactPrefixCache::prune(int id, int keep) noexcept {
    while (id > 0 && id != keep) {
        Node& n = s_.nodes[std::size_t(id)];
        if (n.block >= 0 || !n.children.empty()) break;
        const int parent = n.parent;
        s_.key_tokens -= n.edge.size();
        s_.nodes[std::size_t(parent)].children.erase(view(n.edge));
        if (journaling_) {
            log(Op::Prune, id, parent);
            pruned_edges_.push_back(std::move(n.edge));
        }
        n.edge.clear();
        n.parent = -1;
        --s_.live_nodes;
        s_.spare.push_back(id);
        id = parent;
    }
}

void ExactPrefixCache::drop(int id, int keep) noexcept {
    Node& n = s_.nodes[std::size_t(id)];
    s_.nodes[std::size_t(n.parent)].leased.erase(view(n.edge));
    log(Op::LeasedDrop, n.parent, id);
    const int block = n.block;
    lease_add(block, -1);
    unstamp(id);
    pool_.unref(block);
    log(Op::Block, id, block);
    n.block = -1;
    --s_.cached;
    prune(id, keep);
}

bool ExactPrefixCache::evict_one() {
    const int victim = lru_front();
    if (victim < 0) return false;
    drop(victim, -1);
    ++s_.evictions;
    return true;
}

void ExactPrefixCache::clear() noexcept {
    // Lexicographic pre-order of the leased nodes, collected before any pruning;
    // pruning only ever removes nodes that precede the current one in this order.
    std::vector<int> order, stack{0};
    while (!stack.empty()) {
        const int id = stack.back();
        stack.pop_back();
        if (id > 0 && s_.nodes[std::size_t(id)].block >= 0) order.push_back(id);
        const auto& ch = s_.nodes[std::size_t(id)].children.items();
        for (auto it = ch.rbegin(); it != ch.rend(); ++it) stack.push_back(it->id);
    }
    for (int id : order) drop(id, -1);
}

int ExactPrefixCache::reuse(PagedSequence& sequence, const std::vector<std::int32_t>& prompt) {
    if (sequence.used || !sequence.blocks.empty() || !sequence.tokens.empty())
        throw std::invalid_argument("prefix reuse requires an empty sequence");
    if (!pool_.config().prefix_cache_blocks) return 0;
    const std::size_t bt = std::size_t(pool_.config().block_tokens);
    const std::size_t limit = prompt.empty() ? 0 : prompt.size() - 1;
    std::vector<int> pages;
    int parent = 0;
    std::size_t count = 0;
    while (count < limit) {
        const std::size_t length = std::min(bt, limit - count);
        const std::int32_t* q = prompt.data() + count;
        const auto& leased = s_.nodes[std::size_t(parent)].leased.items();
        const std::size_t next = s_.nodes[std::size_t(parent)].leased.lower_bound(View{q, length});
        int best = -1;
        std::size_t matched = 0;
        auto consider = [&](int id) {
            const auto& e = s_.nodes[std::size_t(id)].edge;
            std::size_t n = 0;
            while (n < length && n < e.size() && e[n] == q[n]) ++n;
            if (n > matched) {
                matched = n;
                best = id;
            }
        };
        if (next < leased.size()) consider(leased[next].id);
        if (next > 0) consider(leased[next - 1].id);
        if (!matched) break;
        pages.push_back(s_.nodes[std::size_t(best)].block);
        touch(best);
        count += matched;
        if (matched != bt) break;
        parent = best;
    }
    for (int page : pages) pool_.retain(page);
    sequence.blocks = std::move(pages);
    sequence.tokens.assign(prompt.begin(), prompt.begin() + std::ptrdiff_t(count));
    sequence.used = int(count);
    if (count) {
        ++s_.hits;
        s_.reused += count;
    } else {
        ++s_.misses;
    }
    return sequence.used;
}

void ExactPrefixCache::publish(const PagedSequence& sequence) {
    if (sequence.tokens.size() != std::size_t(sequence.used))
        throw std::logic_error("invalid committed KV token history");
    const std::size_t bt = std::size_t(pool_.config().block_tokens);
    const std::size_t used = std::size_t(sequence.used);
    const std::size_t capacity = std::size_t(pool_.config().prefix_cache_blocks);
    const std::size_t count = std::min(sequence.blocks.size(), std::min((used + bt - 1) / bt, capacity));
    auto& path = sequence.prefix_path;
    if (path.size() > count) path.resize(count);
    int parent = 0;
    for (std::size_t i = 0; i < count; ++i) {
        const View key{sequence.tokens.data() + i * bt, std::min(bt, used - i * bt)};
        int id = -1;
        if (i < path.size()) {
            // the hinted node is the child of `parent` under `key` iff it is live
            // under that parent with that edge (edges are unique among siblings)
            const int h = path[i];
            if (h > 0 && std::size_t(h) < s_.nodes.size()) {
                const Node& n = s_.nodes[std::size_t(h)];
                if (n.parent == parent && n.edge.size() == key.n && std::equal(key.p, key.p + key.n, n.edge.begin()))
                    id = h;
            }
        }
        if (id < 0) {
            id = s_.nodes[std::size_t(parent)].children.find(key);
            if (id < 0) id = new_node(parent, key);
        }
        if (s_.nodes[std::size_t(id)].block >= 0) {
            touch(id);
        } else {
            const int page = sequence.blocks[i];
            s_.nodes[std::size_t(parent)].leased.insert(view(s_.nodes[std::size_t(id)].edge), id);
            log(Op::LeasedAdd, parent, id);
            try {
                pool_.retain(page);
            } catch (...) {
                s_.nodes[std::size_t(parent)].leased.erase(view(s_.nodes[std::size_t(id)].edge));
                log(Op::LeasedDrop, parent, id);
                prune(id, -1);
                throw;
            }
            if (s_.cached == capacity) {
                drop(lru_front(), id);
                ++s_.evictions;
            }
            lease_add(page, +1);
            log(Op::Block, id, s_.nodes[std::size_t(id)].block);
            s_.nodes[std::size_t(id)].block = page;
            touch(id);
            ++s_.cached;
        }
        if (i < path.size()) path[i] = id;
        else path.push_back(id);
        parent = id;
    }
}

void ExactPrefixCache::begin_journal() {
    journal_.clear();
    pruned_edges_.clear();
    relink_.reserve(s_.nodes.size());
    saved_.counters = s_;
    saved_.clock = s_.clock;
    ++window_;
    journaling_ = true;
}

void ExactPrefixCache::end_journal() noexcept {
    journaling_ = false;
    journal_.clear();
    pruned_edges_.clear();
}

void ExactPrefixCache::rollback_journal() noexcept {
    journaling_ = false;
    for (auto e = journal_.rbegin(); e != journal_.rend(); ++e) {
        switch (e->op) {
        case Op::NewNode: {
            Node& n = s_.nodes[std::size_t(e->a)];
            s_.nodes[std::size_t(e->b)].children.erase(view(n.edge));
            n.edge.clear();
            n.parent = -1;
            n.block = -1;
            n.stamp = 0;
            n.children.clear();
            n.leased.clear();
            if (e->v) s_.spare.push_back(e->a);
            else s_.nodes.pop_back();
            break;
        }
        case Op::Prune: {
            s_.spare.pop_back();
            Node& n = s_.nodes[std::size_t(e->a)];
            n.edge = std::move(pruned_edges_.back());
            pruned_edges_.pop_back();
            n.parent = e->b;
            s_.nodes[std::size_t(e->b)].children.insert(view(n.edge), e->a);
            break;
        }
        case Op::LeasedAdd:
            s_.nodes[std::size_t(e->a)].leased.erase(view(s_.nodes[std::size_t(e->b)].edge));
            break;
        case Op::LeasedDrop:
            s_.nodes[std::size_t(e->a)].leased.insert(view(s_.nodes[std::size_t(e->b)].edge), e->b);
            break;
        case Op::Stamp:
            s_.nodes[std::size_t(e->a)].stamp = e->v;
            break;
        case Op::Block:
            s_.nodes[std::size_t(e->a)].block = e->b;
            break;
        case Op::Lease: {
            pool_.add_lease(e->a, -e->b);
            break;
        }
        }
    }
    static_cast<Counters&>(s_) = saved_.counters;
    s_.clock = saved_.clock;
    relink_lru();
    journal_.clear();
    pruned_edges_.clear();
}

}  // namespace miniprefix_b200
