// C shim over the reference MiniPrefix CPU engine -- TEST INFRASTRUCTURE ONLY.
//
// Built by oracle/Makefile from the reference's own sources (TinyInfer v0.3.0,
// compiled in place, objects and the shared library written to oracle/_ref/).
// It lets the Python tests and bench.py's reference arm drive the UNMODIFIED
// reference classes through plain C calls:
//   - CpuRunner (miniprefix/src/backend/cpu/llama_runner.cpp) with in-memory weights,
//   - KVManager (miniprefix/src/kv/kv_manager.cpp) directly,
//   - Engine (miniprefix/src/engine/engine.cpp) over either the CpuRunner or a
//     scripted runner that keeps the real KVManager but returns one-hot logits
//     (used to replay a GPU run's token stream through the reference bookkeeping).
// Nothing here is product code; tinyinfer_b200 never links it.
//
// Error convention shared with the product host library (include/miniprefix_b200_host.h):
//   >= 0 success; -1 std::invalid_argument; -2 std::logic_error; -3 KvCapacityError;
//   -4 other std::runtime_error; -5 std::out_of_range; -6 anything else.
#include <algorithm>
#include <sstream>

#include "protocol/session.h"
#include "miniprefix/engine.h"
#include "miniprefix/kv_manager.h"
#include "miniprefix/model.h"
#include "miniprefix/prefix_cache.h"
#include <cstring>
#include <map>
#include <set>
#include <memory>
#include <string>
#include <vector>

using namespace miniprefix;

namespace {
thread_local std::string g_error;

template <class F> int guarded(F&& body) {
    try {
        return body();
    } catch (const KvCapacityError& e) {
        g_error = e.what();
        return -3;
    } catch (const std::invalid_argument& e) {
        g_error = e.what();
        return -1;
    } catch (const std::out_of_range& e) {
        g_error = e.what();
        return -5;
    } catch (const std::logic_error& e) {
        g_error = e.what();
        return -2;
    } catch (const std::runtime_error& e) {
        g_error = e.what();
        return -4;
    } catch (...) {
        g_error = "unknown exception";
        return -6;
    }
}

// Runner that owns a real KVManager and returns scripted one-hot logits. Each
// completed append of request `id` returns logits whose first maximum is the
// next scripted token for that id (token 0 once the script is exhausted).
class ScriptedRunner final : public ModelRunner {
public:
    ModelConfig config_;
    KVManager kv_;
    std::map<RequestId, std::vector<TokenId>> script_;
    std::map<RequestId, std::size_t> cursor_;
    std::vector<KVManager::TailCopyRegion> regions_;
    std::set<TokenId> poison_;
    RunnerStats stats_;
    ScriptedRunner(int vocabulary, int context, int layers, int width, KvCacheConfig kv)
        : kv_(kv, layers, width, context, vocabulary) {
        config_.vocabulary = vocabulary;
        config_.context = context;
        config_.layers = layers;
    }
    const ModelConfig& config() const override { return config_; }
    int context_limit() const override { return kv_.context_limit(); }
    KvAdmission reserve_request(const RequestId& id, std::size_t n) override { return kv_.reserve_request(id, n); }
    void release_reservation(const RequestId& id) noexcept override { kv_.release_reservation(id); }
    void create(const RequestId& id) override { kv_.create(id); }
    void fork_sequence(const RequestId& s, const RequestId& t) override { kv_.fork_sequence(s, t); }
    std::size_t reuse_prefix(const RequestId& id, const std::vector<TokenId>& p) override {
        return kv_.reuse_prefix(id, p);
    }
    void cache_prefix(const RequestId& id) override { kv_.cache_prefix(id); }
    void clear_prefix_cache() override { kv_.clear_prefix_cache(); }
    std::vector<float> append(const RequestId& id, const std::vector<TokenId>& tokens) override {
        auto tx = kv_.prepare_append(id, tokens);
        tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) { regions_.push_back(r); });
        std::vector<float> logits(config_.vocabulary, 0.0f);
        for (auto t : tokens)
            if (poison_.count(t)) throw std::runtime_error("nonfinite logits");
        auto& list = script_[id];
        auto& at = cursor_[id];
        const TokenId next = at < list.size() ? list[at] : 0;
        logits[next] = 1.0f;
        tx.commit();
        ++at;
        return logits;
    }
    void release(const RequestId& id) override { kv_.release(id); }
    void clear() override { kv_.clear(); }
    RunnerStats stats() const override {
        auto r = stats_;
        r.update_kv_stats(kv_.stats());
        return r;
    }
    CostStats cost_stats() const override { return kv_.cost_stats(); }
};

struct CacheHandle {
    KvBlockPool pool;
    ExactPrefixCache cache;
    std::map<std::string, PagedSequence> sequences;
    CacheHandle(KvCacheConfig c, int layers, int width) : pool(c, layers, width), cache(pool) {}
    ~CacheHandle() {
        for (auto& s : sequences) pool.release(s.second);
        cache.clear();
    }
};

struct RunnerHandle {
    std::unique_ptr<ModelRunner> owned;
    ModelRunner* runner = nullptr;
    ScriptedRunner* scripted = nullptr;
};

struct EngineHandle {
    std::unique_ptr<Engine> engine;
    ScriptedRunner* scripted = nullptr;
};

void stats_out(const RunnerStats& s, std::size_t* out) {
    static_assert(sizeof(RunnerStats) == 25 * sizeof(std::size_t), "25-field layout");
    std::memcpy(out, &s, sizeof(RunnerStats));
}
void kv_stats_out(const KvStats& s, std::size_t* out) {
    static_assert(sizeof(KvStats) == 16 * sizeof(std::size_t), "16-field layout");
    std::memcpy(out, &s, sizeof(KvStats));
}
std::vector<TokenId> tokens_of(const int* p, int n) { return std::vector<TokenId>(p, p + (n > 0 ? n : 0)); }
int sequence_out(const PagedSequence& s, int* used, int* blocks, int capacity) {
    *used = s.used;
    const int n = static_cast<int>(s.blocks.size());
    for (int i = 0; i < n && i < capacity; ++i) blocks[i] = s.blocks[i];
    return n;
}
}  // namespace

extern "C" {
const char* ref_last_error() { return g_error.c_str(); }

// ---------------------------------------------------------------- weights
void* ref_weights_new(int layers, int hidden, int intermediate, int heads, int kv_heads, int vocabulary,
                      int context, int eos, float eps, float theta, int tied) {
    auto* w = new std::shared_ptr<ModelWeights>(std::make_shared<ModelWeights>());
    auto& c = (*w)->config;
    c.layers = layers; c.hidden = hidden; c.intermediate = intermediate; c.heads = heads;
    c.kv_heads = kv_heads; c.vocabulary = vocabulary; c.context = context; c.eos = eos;
    c.rms_epsilon = eps; c.rope_theta = theta; c.tied = tied != 0;
    if (guarded([&] { c.validate(); return 0; }) < 0) { delete w; return nullptr; }
    return w;
}
int ref_weights_put(void* handle, const char* name, const float* data, int rank, const long* dims) {
    return guarded([&] {
        auto& w = *static_cast<std::shared_ptr<ModelWeights>*>(handle);
        tinyinfer::Shape shape(dims, dims + rank);
        tinyinfer::Tensor t(shape);
        std::memcpy(t.data<float>(), data, t.numel() * sizeof(float));
        w->tensors.erase(name);
        w->tensors.emplace(name, std::move(t));
        return 0;
    });
}
void ref_weights_free(void* handle) { delete static_cast<std::shared_ptr<ModelWeights>*>(handle); }
// The reference's own MPFX0001 loader (ModelWeights::load, model.cpp:20-56): NULL
// and ref_last_error() on failure.
void* ref_weights_load(const char* path) {
    std::shared_ptr<ModelWeights> loaded;
    if (guarded([&] { loaded = ModelWeights::load(path); return 0; }) < 0) return nullptr;
    return new std::shared_ptr<ModelWeights>(std::move(loaded));
}
// layers, hidden, intermediate, heads, kv_heads, vocabulary, context, eos, tied;
// eps and theta through `f`.
int ref_weights_config(void* handle, int* out, float* f) {
    const auto& c = (*static_cast<std::shared_ptr<ModelWeights>*>(handle))->config;
    const int v[9] = {c.layers, c.hidden, c.intermediate, c.heads, c.kv_heads, c.vocabulary, c.context, c.eos,
                      c.tied ? 1 : 0};
    std::memcpy(out, v, sizeof(v));
    f[0] = c.rms_epsilon;
    f[1] = c.rope_theta;
    return 0;
}
// Copies tensor `name` (count floats); returns its element count, -1 if absent.
long ref_weights_tensor(void* handle, const char* name, float* out, long count) {
    const auto& w = *static_cast<std::shared_ptr<ModelWeights>*>(handle);
    const auto it = w->tensors.find(name);
    if (it == w->tensors.end()) return -1;
    const long n = static_cast<long>(it->second.numel());
    std::memcpy(out, it->second.data<float>(), std::size_t(std::min(n, count)) * sizeof(float));
    return n;
}
long ref_weights_count(void* handle) { return long((*static_cast<std::shared_ptr<ModelWeights>*>(handle))->tensors.size()); }

// ---------------------------------------------------------------- runners
void* ref_cpu_runner_new(void* weights, int context, int block_tokens, int max_blocks, int prefix_blocks) {
    auto* h = new RunnerHandle;
    if (guarded([&] {
            h->owned = make_cpu_runner(*static_cast<std::shared_ptr<ModelWeights>*>(weights), context,
                                       KvCacheConfig{block_tokens, max_blocks, prefix_blocks});
            h->runner = h->owned.get();
            return 0;
        }) < 0) {
        delete h;
        return nullptr;
    }
    return h;
}
void* ref_scripted_runner_new(int vocabulary, int context, int layers, int width, int block_tokens,
                              int max_blocks, int prefix_blocks) {
    auto* h = new RunnerHandle;
    if (guarded([&] {
            auto r = std::make_unique<ScriptedRunner>(vocabulary, context, layers, width,
                                                      KvCacheConfig{block_tokens, max_blocks, prefix_blocks});
            h->scripted = r.get();
            h->runner = r.get();
            h->owned = std::move(r);
            return 0;
        }) < 0) {
        delete h;
        return nullptr;
    }
    return h;
}
int ref_scripted_set(void* handle, const char* id, const int* tokens, int count) {
    auto* h = static_cast<RunnerHandle*>(handle);
    if (!h->scripted) return -2;
    h->scripted->script_[id] = tokens_of(tokens, count);
    h->scripted->cursor_[id] = 0;
    return 0;
}
int ref_scripted_poison(void* handle, int token) {
    auto* h = static_cast<RunnerHandle*>(handle);
    if (!h->scripted) return -2;
    h->scripted->poison_.insert(token);
    return 0;
}
// Copies the recorded COW regions (5 size_t each) and clears the record.
long ref_scripted_regions(void* handle, std::size_t* out, long capacity) {
    auto* h = static_cast<RunnerHandle*>(handle);
    if (!h->scripted) return -2;
    const long n = static_cast<long>(h->scripted->regions_.size());
    for (long i = 0; i < n && i < capacity; ++i) {
        const auto& r = h->scripted->regions_[i];
        out[5 * i] = r.destination; out[5 * i + 1] = r.source; out[5 * i + 2] = r.pitch;
        out[5 * i + 3] = r.width; out[5 * i + 4] = r.rows;
    }
    h->scripted->regions_.clear();
    return n;
}
int ref_scripted_sequence(void* handle, const char* id, int* used, int* blocks, int capacity) {
    auto* h = static_cast<RunnerHandle*>(handle);
    if (!h->scripted) return -2;
    return guarded([&] { return sequence_out(h->scripted->kv_.sequence(id), used, blocks, capacity); });
}
void ref_runner_free(void* handle) { delete static_cast<RunnerHandle*>(handle); }

#define RUNNER (static_cast<RunnerHandle*>(handle)->runner)
int ref_runner_reserve(void* handle, const char* id, std::size_t tokens) {
    return guarded([&] { return static_cast<int>(RUNNER->reserve_request(id, tokens)); });
}
int ref_runner_release_reservation(void* handle, const char* id) {
    RUNNER->release_reservation(id);
    return 0;
}
int ref_runner_create(void* handle, const char* id) { return guarded([&] { RUNNER->create(id); return 0; }); }
int ref_runner_fork(void* handle, const char* source, const char* target) {
    return guarded([&] { RUNNER->fork_sequence(source, target); return 0; });
}
long ref_runner_reuse_prefix(void* handle, const char* id, const int* prompt, int n) {
    long result = 0;
    const int rc = guarded([&] { result = static_cast<long>(RUNNER->reuse_prefix(id, tokens_of(prompt, n))); return 0; });
    return rc < 0 ? rc : result;
}
int ref_runner_cache_prefix(void* handle, const char* id) { return guarded([&] { RUNNER->cache_prefix(id); return 0; }); }
int ref_runner_clear_prefix_cache(void* handle) { return guarded([&] { RUNNER->clear_prefix_cache(); return 0; }); }
int ref_runner_append(void* handle, const char* id, const int* tokens, int n, float* logits) {
    return guarded([&] {
        auto out = RUNNER->append(id, tokens_of(tokens, n));
        if (logits) std::memcpy(logits, out.data(), out.size() * sizeof(float));
        return static_cast<int>(out.size());
    });
}
int ref_runner_release(void* handle, const char* id) { return guarded([&] { RUNNER->release(id); return 0; }); }
int ref_runner_clear(void* handle) { return guarded([&] { RUNNER->clear(); return 0; }); }
int ref_runner_stats(void* handle, std::size_t* out) { stats_out(RUNNER->stats(), out); return 0; }
int ref_runner_cost_stats(void* handle, std::uint64_t* out) {
    const auto c = RUNNER->cost_stats();
    const std::uint64_t v[8] = {c.lookup_calls, c.lookup_ns, c.publish_calls, c.publish_ns,
                                c.cow_pages, c.cow_bytes, c.cow_copy_ns, c.cow_timed_copies};
    std::memcpy(out, v, sizeof(v));
    return 0;
}
int ref_runner_set_cost_timing(void* handle, int enabled) { RUNNER->set_cost_timing(enabled != 0); return 0; }
int ref_runner_context_limit(void* handle) { return RUNNER->context_limit(); }
#undef RUNNER

// ---------------------------------------------------------------- pool + prefix cache
void* ref_cache_new(int block_tokens, int max_blocks, int prefix_blocks, int layers, int width) {
    CacheHandle* h = nullptr;
    if (guarded([&] {
            h = new CacheHandle(KvCacheConfig{block_tokens, max_blocks, prefix_blocks}, layers, width);
            return 0;
        }) < 0)
        return nullptr;
    return h;
}
void ref_cache_free(void* h) { delete static_cast<CacheHandle*>(h); }
#define CH (static_cast<CacheHandle*>(h))
int ref_cache_append(void* h, const char* seq, const int* tokens, int count) {
    return guarded([&] {
        auto& s = CH->sequences[seq];
        CH->pool.reserve(s, s.used + count);
        s.tokens.insert(s.tokens.end(), tokens, tokens + count);
        s.used += count;
        return 0;
    });
}
int ref_cache_publish(void* h, const char* seq) { return guarded([&] { CH->cache.publish(CH->sequences[seq]); return 0; }); }
long ref_cache_reuse(void* h, const char* seq, const int* prompt, int count) {
    long r = 0;
    const int rc = guarded([&] { r = CH->cache.reuse(CH->sequences[seq], tokens_of(prompt, count)); return 0; });
    return rc < 0 ? rc : r;
}
int ref_cache_release(void* h, const char* seq) { return guarded([&] { CH->pool.release(CH->sequences[seq]); return 0; }); }
int ref_cache_evict_one(void* h) { return guarded([&] { return CH->cache.evict_one() ? 1 : 0; }); }
int ref_cache_clear(void* h) { CH->cache.clear(); return 0; }
int ref_cache_stats(void* h, std::uint64_t* out) {
    const std::uint64_t v[11] = {CH->cache.size(), CH->cache.index_nodes(), CH->cache.key_token_bytes(),
                                 CH->cache.hits(), CH->cache.misses(), CH->cache.reused_tokens(),
                                 CH->cache.evictions(), CH->cache.cache_only_blocks(), CH->pool.live_blocks(),
                                 CH->pool.peak_blocks(), CH->pool.free_blocks()};
    std::memcpy(out, v, sizeof(v));
    return 0;
}
int ref_cache_references(void* h, std::uint64_t* out, int count) {
    return guarded([&] { for (int i = 0; i < count; ++i) out[i] = CH->pool.references(i); return 0; });
}
int ref_cache_define(void* h, const char* seq, int used, const int* tokens, int token_count, const int* blocks,
                     int block_count) {
    return guarded([&] {
        auto& s = CH->sequences[seq];
        s.used = used;
        s.tokens.assign(tokens, tokens + token_count);
        s.blocks.assign(blocks, blocks + block_count);
        return 0;
    });
}
int ref_cache_sequence(void* h, const char* seq, int* used, int* blocks, int capacity, int* tokens, int token_capacity) {
    return guarded([&] {
        const auto& s = CH->sequences.at(seq);
        for (int i = 0; i < int(s.tokens.size()) && i < token_capacity; ++i) tokens[i] = s.tokens[i];
        return sequence_out(s, used, blocks, capacity);
    });
}
#undef CH

// ---------------------------------------------------------------- KVManager
void* ref_kv_new(int block_tokens, int max_blocks, int prefix_blocks, int layers, int width, int context,
                 int vocabulary) {
    KVManager* m = nullptr;
    if (guarded([&] {
            m = new KVManager(KvCacheConfig{block_tokens, max_blocks, prefix_blocks}, layers, width, context,
                              vocabulary);
            return 0;
        }) < 0)
        return nullptr;
    return m;
}
void ref_kv_free(void* m) { delete static_cast<KVManager*>(m); }
#define KV (static_cast<KVManager*>(m))
int ref_kv_reserve(void* m, const char* id, std::size_t tokens) {
    return guarded([&] { return static_cast<int>(KV->reserve_request(id, tokens)); });
}
int ref_kv_release_reservation(void* m, const char* id) { KV->release_reservation(id); return 0; }
int ref_kv_create(void* m, const char* id) { return guarded([&] { KV->create(id); return 0; }); }
int ref_kv_fork(void* m, const char* s, const char* t) { return guarded([&] { KV->fork_sequence(s, t); return 0; }); }
long ref_kv_reuse_prefix(void* m, const char* id, const int* prompt, int n) {
    long result = 0;
    const int rc = guarded([&] { result = static_cast<long>(KV->reuse_prefix(id, tokens_of(prompt, n))); return 0; });
    return rc < 0 ? rc : result;
}
int ref_kv_cache_prefix(void* m, const char* id) { return guarded([&] { KV->cache_prefix(id); return 0; }); }
int ref_kv_clear_prefix_cache(void* m) { return guarded([&] { KV->clear_prefix_cache(); return 0; }); }
// One Append transaction. mode 0: commit after copying; 1: roll back; 2: copier
// throws (commit must then fail, transaction rolls back). tail[0..2] receives
// {source, destination, valid} or {-1,-1,-1}; region[0..4] the merged region.
int ref_kv_append(void* m, const char* id, const int* tokens, int n, int mode, long* tail, std::size_t* region) {
    return guarded([&] {
        tail[0] = tail[1] = tail[2] = -1;
        auto tx = KV->prepare_append(id, tokens_of(tokens, n));
        if (tx.tail_copy()) {
            tail[0] = tx.tail_copy()->source; tail[1] = tx.tail_copy()->destination; tail[2] = tx.tail_copy()->valid_tokens;
        }
        if (mode == 2) {
            try {
                tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion&) { throw std::runtime_error("copy"); });
            } catch (const std::runtime_error&) {
            }
            bool rejected = false;
            try { tx.commit(); } catch (const std::logic_error&) { rejected = true; }
            if (tx.tail_copy() && !rejected) throw std::logic_error("commit accepted an uncopied tail");
            tx.rollback();
            return 0;
        }
        tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) {
            region[0] = r.destination; region[1] = r.source; region[2] = r.pitch; region[3] = r.width; region[4] = r.rows;
        });
        if (mode == 0) tx.commit();
        else tx.rollback();
        return 0;
    });
}
int ref_kv_reset_sequence(void* m, const char* id) { return guarded([&] { KV->reset_sequence(id); return 0; }); }
int ref_kv_release(void* m, const char* id) { return guarded([&] { KV->release(id); return 0; }); }
int ref_kv_clear(void* m) { return guarded([&] { KV->clear(); return 0; }); }
int ref_kv_stats(void* m, std::size_t* out) { kv_stats_out(KV->stats(), out); return 0; }
int ref_kv_sequence(void* m, const char* id, int* used, int* blocks, int capacity) {
    return guarded([&] { return sequence_out(KV->sequence(id), used, blocks, capacity); });
}
long ref_kv_offset(void* m, const char* id, int layer, int token) {
    long r = 0;
    const int rc = guarded([&] { r = static_cast<long>(KV->offset(KV->sequence(id), layer, token)); return 0; });
    return rc < 0 ? rc : r;
}
#undef KV

// ---------------------------------------------------------------- Engine
// Takes ownership of the runner handle's runner.
// The reference's worker protocol (apps/protocol/session.cpp) over an engine.
long ref_protocol_serve(void* engine, const char* input, char* out, long capacity) {
    auto* h = static_cast<EngineHandle*>(engine);
    std::istringstream in(input);
    std::ostringstream os;
    miniprefix::protocol::serve(*h->engine, in, os);
    const std::string s = os.str();
    if (out && capacity > 0) {
        const std::size_t n = std::min(s.size(), std::size_t(capacity - 1));
        std::memcpy(out, s.data(), n);
        out[n] = '\0';
    }
    return long(s.size());
}

void* ref_engine_new(void* runner, int max_batch, int budget, int chunk, int context) {
    auto* rh = static_cast<RunnerHandle*>(runner);
    auto* h = new EngineHandle;
    if (guarded([&] {
            h->scripted = rh->scripted;
            h->engine = std::make_unique<Engine>(std::move(rh->owned), EngineConfig{max_batch, budget, chunk, context});
            rh->runner = nullptr;  // owned by the engine now; script/poison stay usable
            return 0;
        }) < 0) {
        delete h;
        return nullptr;
    }
    return h;
}
void ref_engine_free(void* e) { delete static_cast<EngineHandle*>(e); }
#define ENG (static_cast<EngineHandle*>(e)->engine)
int ref_engine_submit(void* e, const char* id, const int* prompt, int n, unsigned max_new, int eos) {
    return guarded([&] {
        Request r;
        r.id = id;
        r.prompt_token_ids = tokens_of(prompt, n);
        r.generation.max_new_tokens = max_new;
        if (eos >= 0) r.generation.eos_token_id = eos;
        ENG->submit(std::move(r));
        return 0;
    });
}
int ref_engine_step(void* e) { return guarded([&] { return ENG->step() ? 1 : 0; }); }
// Events as text lines "id\ttoken\treason\terror\n" (token/reason -1 when absent;
// reason 0 Eos, 1 Length, 2 Cancelled, 3 Error). Returns bytes needed.
long ref_engine_poll(void* e, char* buffer, long capacity) {
    std::string text;
    for (const auto& ev : ENG->poll_events()) {
        text += ev.request_id + "\t" + std::to_string(ev.token_id ? *ev.token_id : -1) + "\t" +
                std::to_string(ev.finish_reason ? static_cast<int>(*ev.finish_reason) : -1) + "\t" + ev.error_message + "\n";
    }
    const long n = static_cast<long>(text.size());
    if (buffer && capacity > 0) {
        const long c = n < capacity - 1 ? n : capacity - 1;
        std::memcpy(buffer, text.data(), c);
        buffer[c] = 0;
    }
    return n;
}
int ref_engine_cancel(void* e, const char* id) { return guarded([&] { ENG->cancel(id); return 0; }); }
int ref_engine_shutdown(void* e) { return guarded([&] { ENG->shutdown(); return 0; }); }
int ref_engine_idle(void* e) { return ENG->idle() ? 1 : 0; }
int ref_engine_failed(void* e) { return ENG->failed() ? 1 : 0; }
int ref_engine_step_stats(void* e, std::size_t* out) {
    const auto& s = ENG->last_step_stats();
    out[0] = s.prefix_reused_tokens; out[1] = s.prefill_tokens; out[2] = s.decode_tokens;
    return 0;
}
int ref_engine_runner_stats(void* e, std::size_t* out) { stats_out(ENG->runner().stats(), out); return 0; }
int ref_engine_cost_stats(void* e, std::uint64_t* out) {
    const auto c = ENG->runner().cost_stats();
    const std::uint64_t v[8] = {c.lookup_calls, c.lookup_ns, c.publish_calls, c.publish_ns,
                                c.cow_pages, c.cow_bytes, c.cow_copy_ns, c.cow_timed_copies};
    std::memcpy(out, v, sizeof(v));
    return 0;
}
int ref_engine_sequence(void* e, const char* id, int* used, int* blocks, int capacity) {
    auto* h = static_cast<EngineHandle*>(e);
    if (!h->scripted) return -2;
    return guarded([&] { return sequence_out(h->scripted->kv_.sequence(id), used, blocks, capacity); });
}
int ref_engine_script(void* e, const char* id, const int* tokens, int count) {
    auto* h = static_cast<EngineHandle*>(e);
    if (!h->scripted) return -2;
    h->scripted->script_[id] = tokens_of(tokens, count);
    h->scripted->cursor_[id] = 0;
    return 0;
}
long ref_engine_regions(void* e, std::size_t* out, long capacity) {
    auto* h = static_cast<EngineHandle*>(e);
    if (!h->scripted) return -2;
    RunnerHandle tmp;
    tmp.scripted = h->scripted;
    return ref_scripted_regions(&tmp, out, capacity);
}
#undef ENG
}
