#include "prefix_cache.h"

#include <algorithm>
#include <iterator>

namespace miniprefix_b200 {

ExactPrefixCache::ExactPrefixCache(KvBlockPool& pool) : pool_(pool) { s_.nodes.emplace_back(); }

ExactPrefixCache::~ExactPrefixCache() { clear(); }

std::size_t ExactPrefixCache::cache_only_blocks() const {
    std::size_t count = 0;
    for (const auto& [block, leases] : s_.leases)
        if (leases && pool_.references(block) == leases) ++count;
    return count;
}

int ExactPrefixCache::new_node(int parent, View edge) {
    int id;
    if (!s_.spare.empty()) {
        id = s_.spare.back();
        s_.spare.pop_back();
    } else {
        id = int(s_.nodes.size());
        s_.nodes.emplace_back();
    }
    Node& n = s_.nodes[std::size_t(id)];
    n.parent = parent;
    n.edge.assign(edge.p, edge.p + edge.n);
    n.block = -1;
    n.older = n.newer = -1;
    n.children.clear();
    n.leased.clear();
    s_.nodes[std::size_t(parent)].children.emplace(n.edge, id);
    ++s_.live_nodes;
    s_.key_tokens += edge.n;
    return id;
}

void ExactPrefixCache::lru_unlink(int id) noexcept {
    Node& n = s_.nodes[std::size_t(id)];
    if (n.older >= 0) s_.nodes[std::size_t(n.older)].newer = n.newer;
    else s_.oldest = n.newer;
    if (n.newer >= 0) s_.nodes[std::size_t(n.newer)].older = n.older;
    else s_.newest = n.older;
    n.older = n.newer = -1;
}

void ExactPrefixCache::lru_append(int id) noexcept {
    Node& n = s_.nodes[std::size_t(id)];
    n.older = s_.newest;
    n.newer = -1;
    if (s_.newest >= 0) s_.nodes[std::size_t(s_.newest)].newer = id;
    else s_.oldest = id;
    s_.newest = id;
}

void ExactPrefixCache::touch(int id) noexcept {
    lru_unlink(id);
    lru_append(id);
}

// Erase empty structural leaves from `id` upward, never the root or `keep`.
void ExactPrefixCache::prune(int id, int keep) noexcept {
    while (id > 0 && id != keep) {
        Node& n = s_.nodes[std::size_t(id)];
        if (n.block >= 0 || !n.children.empty()) break;
        const int parent = n.parent;
        s_.key_tokens -= n.edge.size();
        s_.nodes[std::size_t(parent)].children.erase(n.edge);
        n.edge.clear();
        n.parent = -1;
        --s_.live_nodes;
        s_.spare.push_back(id);
        id = parent;
    }
}

void ExactPrefixCache::drop(int id, int keep) noexcept {
    Node& n = s_.nodes[std::size_t(id)];
    s_.nodes[std::size_t(n.parent)].leased.erase(n.edge);
    const int block = n.block;
    auto lease = s_.leases.find(block);
    if (--lease->second == 0) s_.leases.erase(lease);
    lru_unlink(id);
    pool_.unref(block);
    n.block = -1;
    --s_.cached;
    prune(id, keep);
}

bool ExactPrefixCache::evict_one() {
    if (s_.oldest < 0) return false;
    drop(s_.oldest, -1);
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
        const auto& ch = s_.nodes[std::size_t(id)].children;
        for (auto it = ch.rbegin(); it != ch.rend(); ++it) stack.push_back(it->second);
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
        const Children& leased = s_.nodes[std::size_t(parent)].leased;
        const auto next = leased.lower_bound(View{q, length});
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
        if (next != leased.end()) consider(next->second);
        if (next != leased.begin()) consider(std::prev(next)->second);
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
    int parent = 0;
    for (std::size_t i = 0; i < count; ++i) {
        const View key{sequence.tokens.data() + i * bt, std::min(bt, used - i * bt)};
        int id;
        {
            const auto& ch = s_.nodes[std::size_t(parent)].children;
            const auto it = ch.find(key);
            id = it != ch.end() ? it->second : new_node(parent, key);
        }
        if (s_.nodes[std::size_t(id)].block >= 0) {
            touch(id);
        } else {
            const int page = sequence.blocks[i];
            s_.nodes[std::size_t(parent)].leased.emplace(s_.nodes[std::size_t(id)].edge, id);
            try {
                pool_.retain(page);
            } catch (...) {
                s_.nodes[std::size_t(parent)].leased.erase(s_.nodes[std::size_t(id)].edge);
                prune(id, -1);
                throw;
            }
            if (s_.cached == capacity) {
                drop(s_.oldest, id);
                ++s_.evictions;
            }
            ++s_.leases[page];
            s_.nodes[std::size_t(id)].block = page;
            lru_append(id);
            ++s_.cached;
        }
        parent = id;
    }
}

ExactPrefixCache::Snapshot ExactPrefixCache::snapshot() const { return s_; }

void ExactPrefixCache::restore(const Snapshot& snapshot) { s_ = snapshot; }

}  // namespace miniprefix_b200
