// Exact prefix cache over paged KV: a trie of page-sized token edges whose
// paths spell the whole causal history, with page leases in LRU order.
//
// Observable behaviour is that of the reference ExactPrefixCache
// (miniprefix/include/miniprefix/prefix_cache.h, miniprefix/src/kv/prefix_cache.cpp):
//  * reuse(): walk from the root; at each level look up the prompt's next
//    (<= block_tokens) tokens among the LEASED children, compare the
//    lexicographic lower_bound neighbour and its predecessor, take the longer
//    common prefix (the lower_bound one on ties, :129-133), touch it in LRU order,
//    stop at a partial match; the result is capped at prompt.size()-1 (:116) and
//    nothing happens when the cache capacity is 0 (:114).
//  * publish(): for each of min(pages, ceil(used/bt), capacity) pages find or
//    create the edge node (structural nodes included), touch a leased node or
//    lease the sequence's page, evicting the LRU lease first when at capacity
//    (:144-198). A page outside the pool throws std::out_of_range and leaves no node.
//  * evict_one(): drop the LRU lease and prune empty leaves upward.
//  * clear(): drop every lease in lexicographic pre-order (:104-110), which fixes
//    the order pages return to the pool's free list.
// Internals differ: nodes live in an arena addressed by index, keys are owned
// token vectors, and the whole index is a value, so it can be snapshotted and
// restored (used to roll back a failed batched step exactly).
#pragma once
#include <cstdint>
#include <deque>
#include <map>
#include <unordered_map>
#include <vector>

#include "page_pool.h"

namespace miniprefix_b200 {

class ExactPrefixCache {
public:
    explicit ExactPrefixCache(KvBlockPool& pool);
    ExactPrefixCache(const ExactPrefixCache&) = delete;
    ExactPrefixCache& operator=(const ExactPrefixCache&) = delete;
    ~ExactPrefixCache();

    std::size_t size() const { return s_.cached; }
    std::size_t index_nodes() const { return s_.live_nodes; }
    std::size_t key_token_bytes() const { return s_.key_tokens * sizeof(std::int32_t); }
    std::size_t hits() const { return s_.hits; }
    std::size_t misses() const { return s_.misses; }
    std::size_t reused_tokens() const { return s_.reused; }
    std::size_t evictions() const { return s_.evictions; }
    std::size_t cache_only_blocks() const;

    void clear() noexcept;
    int reuse(PagedSequence& sequence, const std::vector<std::int32_t>& prompt);
    void publish(const PagedSequence& sequence);
    bool evict_one();

    // Opaque copy of the whole index (pool state is journaled separately).
    struct Snapshot;
    Snapshot snapshot() const;
    void restore(const Snapshot& snapshot);

private:
    struct EdgeLess {
        using is_transparent = void;
        struct View {
            const std::int32_t* p;
            std::size_t n;
        };
        static View view(const std::vector<std::int32_t>& v) { return {v.data(), v.size()}; }
        static View view(const View& v) { return v; }
        template <class A, class B>
        bool operator()(const A& a, const B& b) const {
            const View x = view(a), y = view(b);
            return std::lexicographical_compare(x.p, x.p + x.n, y.p, y.p + y.n);
        }
    };
    using View = EdgeLess::View;
    using Children = std::map<std::vector<std::int32_t>, int, EdgeLess>;
    struct Node {
        int parent = -1;
        std::vector<std::int32_t> edge;
        int block = -1;
        int older = -1, newer = -1;  // LRU links among leased nodes
        Children children;           // every child
        Children leased;             // children holding a lease (lookup set of reuse)
    };

public:
    struct Snapshot {
        std::deque<Node> nodes;
        std::vector<int> spare;
        int oldest = -1, newest = -1;
        std::size_t cached = 0, live_nodes = 0, key_tokens = 0;
        std::unordered_map<int, std::uint32_t> leases;
        std::size_t hits = 0, misses = 0, reused = 0, evictions = 0;
    };

private:
    int new_node(int parent, View edge);
    void lru_unlink(int n) noexcept;
    void lru_append(int n) noexcept;
    void touch(int n) noexcept;
    void prune(int n, int keep) noexcept;
    void drop(int n, int keep) noexcept;

    KvBlockPool& pool_;
    Snapshot s_;  // the live index (nodes[0] is the root)
};

}  // namespace miniprefix_b200
