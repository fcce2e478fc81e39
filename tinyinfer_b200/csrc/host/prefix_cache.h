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
// token vectors, every mutation can be recorded in an undo journal (used to roll
// back a failed batched step exactly, at a cost proportional to the step's own
// changes), leases are kept in LRU order on an intrusive doubly-linked list
// (touch = move to the tail, eviction = the head), and publish() first tries the
// node path the same sequence reached at its previous publish (each hinted node
// is checked against its parent and edge before use, so a stale hint only costs
// the ordinary lookup).
#pragma once
#include <algorithm>
#include <cstdint>
#include <type_traits>
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

    // Undo journal of the index (pool state is journaled separately): between
    // begin_journal() and end_journal(), rollback_journal() returns the index to
    // its state at begin_journal().
    void begin_journal();
    void rollback_journal() noexcept;
    void end_journal() noexcept;

private:
    struct View {
        const std::int32_t* p;
        std::size_t n;
    };
    static View view(const std::vector<std::int32_t>& v) { return {v.data(), v.size()}; }
    static bool less(View a, View b) { return std::lexicographical_compare(a.p, a.p + a.n, b.p, b.p + b.n); }
    // Children of a node in lexicographic order of their edges: a sorted vector of
    // (edge view, node). A view points into the child's own edge buffer, which
    // stays put while the child is listed (moving a Node moves the buffer as a
    // whole); nodes have few children, so lookups and inserts stay cheap.
    class Children {
    public:
        struct Item {
            View key;
            int id;
        };
        bool empty() const { return items_.empty(); }
        void clear() { items_.clear(); }
        const std::vector<Item>& items() const { return items_; }
        std::size_t lower_bound(View k) const {
            return std::size_t(std::lower_bound(items_.begin(), items_.end(), k,
                                                [](const Item& a, View b) { return less(a.key, b); }) -
                               items_.begin());
        }
        int find(View k) const {
            const std::size_t i = lower_bound(k);
            return i < items_.size() && !less(k, items_[i].key) ? items_[i].id : -1;
        }
        void insert(View k, int id) { items_.insert(items_.begin() + std::ptrdiff_t(lower_bound(k)), Item{k, id}); }
        void erase(View k) {
            const std::size_t i = lower_bound(k);
            if (i < items_.size() && !less(k, items_[i].key)) items_.erase(items_.begin() + std::ptrdiff_t(i));
        }

    private:
        std::vector<Item> items_;
    };
    struct Node {
        int parent = -1;
        std::vector<std::int32_t> edge;
        int block = -1;
        std::uint64_t stamp = 0;  // LRU time of the last touch; 0 while not leased
        std::uint64_t logged = 0; // undo window that already journaled the stamp
        int prev = -1, next = -1; // LRU list neighbours while leased
        Children children;        // every child
        Children leased;          // children holding a lease (lookup set of reuse)
    };
    // Children views stay valid across reallocation of the node arena only if
    // nodes move (never copy) their edge buffers.
    static_assert(std::is_nothrow_move_constructible<Node>::value, "nodes must move their edges");

    struct Counters {
        std::size_t cached = 0, live_nodes = 0, key_tokens = 0;
        std::size_t hits = 0, misses = 0, reused = 0, evictions = 0;
    };
    // LRU order is the order of the nodes' stamps: every leased node is on the
    // list from `lru_first` (least recently used) to `lru_last`, and a touch takes
    // the next clock value and moves the node to the tail, so list order and stamp
    // order agree.
    struct State : Counters {
        std::vector<Node> nodes;
        std::vector<int> spare;
        int lru_first = -1, lru_last = -1;
        std::uint64_t clock = 0;
    };
    // Journal entries: each records what its inverse needs.
    enum class Op : std::uint8_t {
        NewNode,     // a = node, b = parent, v = 1 when taken from the spare list
        Prune,       // a = node, b = parent; the edge moves to pruned_edges_
        LeasedAdd,   // a = parent, b = node
        LeasedDrop,  // a = parent, b = node
        Stamp,       // a = node, v = stamp before the window (logged once per window)
        Block,       // a = node, b = previous block
        Lease,       // a = page, b = +1 / -1
    };
    struct Entry {
        Op op;
        int a, b;
        std::uint64_t v;
    };
    void log(Op op, int a, int b = 0, std::uint64_t v = 0) {
        if (journaling_) journal_.push_back({op, a, b, v});
    }
    void lease_add(int page, int delta);

    int new_node(int parent, View edge);
    void log_stamp(Node& n, int id);
    void touch(int n);            // becomes the most recently used lease
    void unstamp(int n) noexcept; // leaves the LRU order
    int lru_front() const noexcept { return s_.lru_first; }
    void relink_lru() noexcept;   // rebuilds the list from the stamps
    void prune(int n, int keep) noexcept;
    void drop(int n, int keep) noexcept;

    KvBlockPool& pool_;
    State s_;  // the live index (nodes[0] is the root)
    bool journaling_ = false;
    std::uint64_t window_ = 0;  // id of the current undo window (ids never repeat)
    std::vector<Entry> journal_;
    std::vector<std::vector<std::int32_t>> pruned_edges_;
    std::vector<std::pair<std::uint64_t, int>> relink_;  // rollback scratch, reserved per window
    struct Window {
        Counters counters;
        std::uint64_t clock = 0;
    } saved_;
};

}  // namespace miniprefix_b200
