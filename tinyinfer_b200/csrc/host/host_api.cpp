// C ABI of the host layer (include/miniprefix_b200_host.h).
#include <cstring>
#include <map>
#include <memory>
#include <string>

#include "b200_runner.h"
#include "engine.h"
#include "miniprefix_b200_host.h"
#include "mpfx.h"
#include "protocol.h"

#include <sstream>
#include "scripted_runner.h"

using namespace miniprefix_b200;

namespace {

thread_local std::string g_error;

template <class F>
long guarded(F&& body) {
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

std::vector<TokenId> tokens_of(const int32_t* p, int32_t n) { return std::vector<TokenId>(p, p + (n > 0 ? n : 0)); }

int sequence_out(const PagedSequence& s, int32_t* used, int32_t* blocks, int32_t capacity) {
    *used = s.used;
    const int n = int(s.blocks.size());
    for (int i = 0; i < n && i < capacity; ++i) blocks[i] = s.blocks[std::size_t(i)];
    return n;
}

void runner_stats_out(const RunnerStats& s, size_t* out) { std::memcpy(out, &s, sizeof(RunnerStats)); }

void cost_out(const CostStats& c, uint64_t* out) {
    const uint64_t v[8] = {c.lookup_calls, c.lookup_ns, c.publish_calls, c.publish_ns,
                           c.cow_pages,    c.cow_bytes, c.cow_copy_ns,   c.cow_timed_copies};
    std::memcpy(out, v, sizeof(v));
}

}  // namespace

struct mph_cache {
    KvBlockPool pool;
    ExactPrefixCache cache;
    std::map<std::string, PagedSequence> sequences;
    // an open undo window (mph_cache_journal)
    std::vector<KvBlockPool::JournalEntry> journal;
    std::size_t live = 0, peak = 0;
    std::map<std::string, PagedSequence> saved;
    bool journaling = false;
    mph_cache(KvCacheConfig c, int layers, int width) : pool(c, layers, width), cache(pool) {}
    ~mph_cache() {
        for (auto& s : sequences) pool.release(s.second);
        cache.clear();
    }
};

struct mph_kv {
    KVManager kv;
    mph_kv(KvCacheConfig c, int layers, int width, int context, int vocabulary) : kv(c, layers, width, context, vocabulary) {}
};

struct mph_runner {
    std::unique_ptr<ModelRunner> owned;
    ModelRunner* runner = nullptr;
    B200Runner* b200 = nullptr;
    ScriptedRunner* scripted = nullptr;
};

struct mph_engine {
    std::unique_ptr<Engine> engine;
    B200Runner* b200 = nullptr;
    ScriptedRunner* scripted = nullptr;
    std::map<std::string, int32_t> index;
};

extern "C" {

const char* mph_last_error(void) { return g_error.c_str(); }

// ------------------------------------------------------------------ cache
mph_cache* mph_cache_new(int32_t block_tokens, int32_t max_blocks, int32_t prefix_blocks, int32_t layers,
                         int32_t width) {
    mph_cache* c = nullptr;
    if (guarded([&] {
            c = new mph_cache(KvCacheConfig{block_tokens, max_blocks, prefix_blocks}, layers, width);
            return 0L;
        }) < 0)
        return nullptr;
    return c;
}
void mph_cache_free(mph_cache* c) { delete c; }
int mph_cache_append(mph_cache* c, const char* seq, const int32_t* tokens, int32_t count) {
    return int(guarded([&] {
        auto& s = c->sequences[seq];
        c->pool.reserve(s, s.used + count);
        s.tokens.insert(s.tokens.end(), tokens, tokens + count);
        s.used += count;
        return 0L;
    }));
}
int mph_cache_publish(mph_cache* c, const char* seq) {
    return int(guarded([&] {
        c->cache.publish(c->sequences[seq]);
        return 0L;
    }));
}
long mph_cache_reuse(mph_cache* c, const char* seq, const int32_t* prompt, int32_t count) {
    return guarded([&] { return long(c->cache.reuse(c->sequences[seq], tokens_of(prompt, count))); });
}
int mph_cache_release(mph_cache* c, const char* seq) {
    return int(guarded([&] {
        c->pool.release(c->sequences[seq]);
        return 0L;
    }));
}
int mph_cache_evict_one(mph_cache* c) {
    return int(guarded([&] { return c->cache.evict_one() ? 1L : 0L; }));
}
int mph_cache_clear(mph_cache* c) {
    c->cache.clear();
    return 0;
}
int mph_cache_journal(mph_cache* c, int32_t op) {
    return int(guarded([&] {
        if (op == 0) {
            if (c->journaling) throw std::logic_error("undo window already open");
            c->journal.clear();
            c->live = c->pool.live_blocks();
            c->peak = c->pool.peak_blocks();
            c->saved = c->sequences;
            c->pool.attach_journal(&c->journal);
            c->cache.begin_journal();
            c->journaling = true;
        } else if (op == 1 || op == 2) {
            if (!c->journaling) throw std::logic_error("no undo window");
            c->pool.attach_journal(nullptr);
            if (op == 1) {
                c->pool.undo(c->journal, 0, c->live, c->peak);
                c->cache.rollback_journal();
                c->sequences = std::move(c->saved);
            } else {
                c->cache.end_journal();
            }
            c->saved.clear();
            c->journaling = false;
        } else {
            throw std::invalid_argument("unknown journal operation");
        }
        return 0L;
    }));
}
int mph_cache_stats(mph_cache* c, uint64_t* out) {
    const uint64_t v[11] = {c->cache.size(),          c->cache.index_nodes(), c->cache.key_token_bytes(),
                            c->cache.hits(),          c->cache.misses(),      c->cache.reused_tokens(),
                            c->cache.evictions(),     c->cache.cache_only_blocks(), c->pool.live_blocks(),
                            c->pool.peak_blocks(),    c->pool.free_blocks()};
    std::memcpy(out, v, sizeof(v));
    return 0;
}
int mph_cache_references(mph_cache* c, uint64_t* out, int32_t count) {
    return int(guarded([&] {
        for (int i = 0; i < count; ++i) out[i] = c->pool.references(i);
        return 0L;
    }));
}
int mph_cache_define(mph_cache* c, const char* seq, int32_t used, const int32_t* tokens, int32_t token_count,
                     const int32_t* blocks, int32_t block_count) {
    return int(guarded([&] {
        auto& s = c->sequences[seq];
        s.used = used;
        s.tokens.assign(tokens, tokens + token_count);
        s.blocks.assign(blocks, blocks + block_count);
        return 0L;
    }));
}
int mph_cache_sequence(mph_cache* c, const char* seq, int32_t* used, int32_t* blocks, int32_t capacity,
                       int32_t* tokens, int32_t token_capacity) {
    return int(guarded([&] {
        const auto& s = c->sequences.at(seq);
        for (int i = 0; i < int(s.tokens.size()) && i < token_capacity; ++i) tokens[i] = s.tokens[std::size_t(i)];
        return long(sequence_out(s, used, blocks, capacity));
    }));
}

// ------------------------------------------------------------------ KV manager
mph_kv* mph_kv_new(int32_t block_tokens, int32_t max_blocks, int32_t prefix_blocks, int32_t layers, int32_t width,
                   int32_t context, int32_t vocabulary) {
    mph_kv* m = nullptr;
    if (guarded([&] {
            m = new mph_kv(KvCacheConfig{block_tokens, max_blocks, prefix_blocks}, layers, width, context, vocabulary);
            return 0L;
        }) < 0)
        return nullptr;
    return m;
}
void mph_kv_free(mph_kv* m) { delete m; }
int mph_kv_reserve(mph_kv* m, const char* id, size_t max_tokens) {
    return int(guarded([&] { return long(m->kv.reserve_request(id, max_tokens)); }));
}
int mph_kv_release_reservation(mph_kv* m, const char* id) {
    m->kv.release_reservation(id);
    return 0;
}
int mph_kv_create(mph_kv* m, const char* id) {
    return int(guarded([&] {
        m->kv.create(id);
        return 0L;
    }));
}
int mph_kv_fork(mph_kv* m, const char* source, const char* target) {
    return int(guarded([&] {
        m->kv.fork_sequence(source, target);
        return 0L;
    }));
}
long mph_kv_reuse_prefix(mph_kv* m, const char* id, const int32_t* prompt, int32_t count) {
    return guarded([&] { return long(m->kv.reuse_prefix(id, tokens_of(prompt, count))); });
}
int mph_kv_cache_prefix(mph_kv* m, const char* id) {
    return int(guarded([&] {
        m->kv.cache_prefix(id);
        return 0L;
    }));
}
int mph_kv_clear_prefix_cache(mph_kv* m) {
    return int(guarded([&] {
        m->kv.clear_prefix_cache();
        return 0L;
    }));
}
int mph_kv_append(mph_kv* m, const char* id, const int32_t* tokens, int32_t count, int32_t mode, long* tail,
                  size_t* region) {
    return int(guarded([&] {
        tail[0] = tail[1] = tail[2] = -1;
        const auto input = tokens_of(tokens, count);  // outlives the transaction
        auto tx = m->kv.prepare_append(id, input);
        if (tx.tail_copy()) {
            tail[0] = tx.tail_copy()->source;
            tail[1] = tx.tail_copy()->destination;
            tail[2] = tx.tail_copy()->valid_tokens;
        }
        if (mode == 2) {
            try {
                tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion&) { throw std::runtime_error("copy"); });
            } catch (const std::runtime_error&) {
            }
            bool refused = false;
            try {
                tx.commit();
            } catch (const std::logic_error&) {
                refused = true;
            }
            if (tx.tail_copy() && !refused) throw std::logic_error("commit accepted an uncopied tail");
            tx.rollback();
            return 0L;
        }
        tx.copy_shared_tail_region([&](const KVManager::TailCopyRegion& r) {
            region[0] = r.destination;
            region[1] = r.source;
            region[2] = r.pitch;
            region[3] = r.width;
            region[4] = r.rows;
        });
        if (mode == 0) tx.commit();
        else tx.rollback();
        return 0L;
    }));
}
int mph_kv_reset_sequence(mph_kv* m, const char* id) {
    return int(guarded([&] {
        m->kv.reset_sequence(id);
        return 0L;
    }));
}
int mph_kv_release(mph_kv* m, const char* id) {
    return int(guarded([&] {
        m->kv.release(id);
        return 0L;
    }));
}
int mph_kv_clear(mph_kv* m) {
    return int(guarded([&] {
        m->kv.clear();
        return 0L;
    }));
}
int mph_kv_stats(mph_kv* m, size_t* out) {
    const KvStats s = m->kv.stats();
    std::memcpy(out, &s, sizeof(KvStats));
    return 0;
}
int mph_kv_sequence(mph_kv* m, const char* id, int32_t* used, int32_t* blocks, int32_t capacity) {
    return int(guarded([&] { return long(sequence_out(m->kv.sequence(id), used, blocks, capacity)); }));
}
long mph_kv_offset(mph_kv* m, const char* id, int32_t layer, int32_t token) {
    return guarded([&] { return long(m->kv.offset(m->kv.sequence(id), layer, token)); });
}

// ------------------------------------------------------------------ runners
mph_runner* mph_runner_new_b200(int32_t device, const mp_model_config* model, int32_t context, int32_t block_tokens,
                                int32_t max_blocks, int32_t prefix_blocks, int32_t max_sequences,
                                int32_t max_step_tokens, int32_t max_step_sequences) {
    auto* h = new mph_runner;
    if (guarded([&] {
            ModelConfig c;
            c.layers = model->layers;
            c.hidden = model->hidden;
            c.intermediate = model->intermediate;
            c.heads = model->heads;
            c.kv_heads = model->kv_heads;
            c.vocabulary = model->vocabulary;
            c.context = model->context;
            c.eos = model->eos;
            c.rms_epsilon = model->rms_epsilon;
            c.rope_theta = model->rope_theta;
            c.tied = model->tied != 0;
            c.validate();
            B200Options o;
            o.device = device;
            o.max_sequences = max_sequences;
            o.max_step_tokens = max_step_tokens;
            o.max_step_sequences = max_step_sequences;
            auto r = std::make_unique<B200Runner>(c, context, KvCacheConfig{block_tokens, max_blocks, prefix_blocks}, o);
            h->b200 = r.get();
            h->runner = r.get();
            h->owned = std::move(r);
            return 0L;
        }) < 0) {
        delete h;
        return nullptr;
    }
    return h;
}
namespace {
mp_model_config to_c(const ModelConfig& c) {
    mp_model_config m{};
    m.layers = c.layers;
    m.hidden = c.hidden;
    m.intermediate = c.intermediate;
    m.heads = c.heads;
    m.kv_heads = c.kv_heads;
    m.vocabulary = c.vocabulary;
    m.context = c.context;
    m.eos = c.eos;
    m.rms_epsilon = c.rms_epsilon;
    m.rope_theta = c.rope_theta;
    m.tied = c.tied ? 1 : 0;
    return m;
}
}  // namespace

mph_runner* mph_runner_new_b200_file(int32_t device, const char* path, int32_t context, int32_t block_tokens,
                                     int32_t max_blocks, int32_t prefix_blocks, int32_t max_sequences,
                                     int32_t max_step_tokens, int32_t max_step_sequences) {
    auto* h = new mph_runner;
    if (guarded([&] {
            if (!path) throw std::invalid_argument("null model path");
            const ModelConfig c = read_mpfx_config(path);
            B200Options o;
            o.device = device;
            o.max_sequences = max_sequences;
            o.max_step_tokens = max_step_tokens;
            o.max_step_sequences = max_step_sequences;
            auto r = std::make_unique<B200Runner>(c, context, KvCacheConfig{block_tokens, max_blocks, prefix_blocks}, o);
            read_mpfx(path, [&](const MpfxTensor& t) { r->set_weight(t.name, t.data, t.elements); });
            r->finalize_weights();
            h->b200 = r.get();
            h->runner = r.get();
            h->owned = std::move(r);
            return 0L;
        }) < 0) {
        delete h;
        return nullptr;
    }
    return h;
}

long mph_engine_serve(mph_engine* e, const char* input, char* out, long capacity) {
    return guarded([&] {
        if (!e || !input) throw std::invalid_argument("null argument");
        std::istringstream in(input);
        std::ostringstream os;
        protocol::serve(*e->engine, in, os);
        const std::string s = os.str();
        if (out && capacity > 0) {
            const std::size_t n = std::min(s.size(), std::size_t(capacity - 1));
            std::memcpy(out, s.data(), n);
            out[n] = '\0';
        }
        return long(s.size());
    });
}

int mph_mpfx_config(const char* path, mp_model_config* out) {
    return int(guarded([&] {
        if (!path || !out) throw std::invalid_argument("null argument");
        *out = to_c(read_mpfx_config(path));
        return 0L;
    }));
}

int mph_mpfx_read(const char* path, mp_model_config* out, mph_tensor_sink sink, void* user) {
    return int(guarded([&] {
        if (!path || !out || !sink) throw std::invalid_argument("null argument");
        *out = to_c(read_mpfx(path, [&](const MpfxTensor& t) {
            if (sink(t.name.c_str(), t.data, uint64_t(t.elements), user) != 0)
                throw std::runtime_error("tensor sink stopped the read");
        }));
        return 0L;
    }));
}

int mph_runner_set_weight(mph_runner* r, const char* name, const float* data, size_t elements) {
    return int(guarded([&] {
        if (!r->b200) throw std::logic_error("not a B200 runner");
        r->b200->set_weight(name, data, elements);
        return 0L;
    }));
}
int mph_runner_finalize(mph_runner* r) {
    return int(guarded([&] {
        if (!r->b200) throw std::logic_error("not a B200 runner");
        r->b200->finalize_weights();
        return 0L;
    }));
}
mph_runner* mph_runner_new_scripted(int32_t vocabulary, int32_t context, int32_t layers, int32_t width,
                                    int32_t block_tokens, int32_t max_blocks, int32_t prefix_blocks) {
    auto* h = new mph_runner;
    if (guarded([&] {
            auto r = std::make_unique<ScriptedRunner>(vocabulary, context, layers, width,
                                                      KvCacheConfig{block_tokens, max_blocks, prefix_blocks});
            h->scripted = r.get();
            h->runner = r.get();
            h->owned = std::move(r);
            return 0L;
        }) < 0) {
        delete h;
        return nullptr;
    }
    return h;
}
int mph_runner_script(mph_runner* r, const char* id, const int32_t* tokens, int32_t count) {
    if (!r->scripted) return -2;
    r->scripted->script(id, tokens_of(tokens, count));
    return 0;
}
int mph_runner_poison(mph_runner* r, int32_t token) {
    if (!r->scripted) return -2;
    r->scripted->poison(token);
    return 0;
}
void mph_runner_free(mph_runner* r) { delete r; }

#define RUNNER (r->runner)
int mph_runner_reserve(mph_runner* r, const char* id, size_t tokens) {
    return int(guarded([&] { return long(RUNNER->reserve_request(id, tokens)); }));
}
int mph_runner_release_reservation(mph_runner* r, const char* id) {
    RUNNER->release_reservation(id);
    return 0;
}
int mph_runner_create(mph_runner* r, const char* id) {
    return int(guarded([&] {
        RUNNER->create(id);
        return 0L;
    }));
}
int mph_runner_fork(mph_runner* r, const char* source, const char* target) {
    return int(guarded([&] {
        RUNNER->fork_sequence(source, target);
        return 0L;
    }));
}
long mph_runner_reuse_prefix(mph_runner* r, const char* id, const int32_t* prompt, int32_t count) {
    return guarded([&] { return long(RUNNER->reuse_prefix(id, tokens_of(prompt, count))); });
}
int mph_runner_cache_prefix(mph_runner* r, const char* id) {
    return int(guarded([&] {
        RUNNER->cache_prefix(id);
        return 0L;
    }));
}
int mph_runner_clear_prefix_cache(mph_runner* r) {
    return int(guarded([&] {
        RUNNER->clear_prefix_cache();
        return 0L;
    }));
}
int mph_runner_append(mph_runner* r, const char* id, const int32_t* tokens, int32_t count, float* logits) {
    return int(guarded([&] {
        const auto out = RUNNER->append(id, tokens_of(tokens, count));
        if (logits) std::memcpy(logits, out.data(), out.size() * sizeof(float));
        return long(out.size());
    }));
}
int mph_runner_release(mph_runner* r, const char* id) {
    return int(guarded([&] {
        RUNNER->release(id);
        return 0L;
    }));
}
int mph_runner_clear(mph_runner* r) {
    return int(guarded([&] {
        RUNNER->clear();
        return 0L;
    }));
}
int mph_runner_stats(mph_runner* r, size_t* out) {
    runner_stats_out(RUNNER->stats(), out);
    return 0;
}
int mph_runner_cost_stats(mph_runner* r, uint64_t* out) {
    cost_out(RUNNER->cost_stats(), out);
    return 0;
}
int mph_runner_set_cost_timing(mph_runner* r, int32_t enabled) {
    RUNNER->set_cost_timing(enabled != 0);
    return 0;
}
int mph_runner_context_limit(mph_runner* r) { return RUNNER->context_limit(); }
int mph_runner_sequence(mph_runner* r, const char* id, int32_t* used, int32_t* blocks, int32_t capacity) {
    return int(guarded([&] {
        if (r->b200) return long(sequence_out(r->b200->kv().sequence(id), used, blocks, capacity));
        if (r->scripted) return long(sequence_out(r->scripted->kv().sequence(id), used, blocks, capacity));
        throw std::logic_error("runner without a visible KV manager");
    }));
}
long mph_runner_regions(mph_runner* r, size_t* out, long capacity) {
    if (!r->scripted) return -2;
    const auto regions = r->scripted->take_regions();
    const long n = long(regions.size());
    for (long i = 0; i < n && i < capacity; ++i) {
        const auto& g = regions[std::size_t(i)];
        out[5 * i] = g.destination;
        out[5 * i + 1] = g.source;
        out[5 * i + 2] = g.pitch;
        out[5 * i + 3] = g.width;
        out[5 * i + 4] = g.rows;
    }
    return n;
}
#undef RUNNER

// ------------------------------------------------------------------ engine
mph_engine* mph_engine_new(mph_runner* runner, int32_t max_batch, int32_t token_budget, int32_t prefill_chunk,
                           int32_t context) {
    auto* h = new mph_engine;
    if (guarded([&] {
            h->b200 = runner->b200;
            h->scripted = runner->scripted;
            h->engine = std::make_unique<Engine>(std::move(runner->owned),
                                                 EngineConfig{max_batch, token_budget, prefill_chunk, context});
            return 0L;
        }) < 0) {
        delete h;
        return nullptr;
    }
    return h;
}
void mph_engine_free(mph_engine* e) { delete e; }
int mph_engine_submit(mph_engine* e, const char* id, const int32_t* prompt, int32_t count, uint32_t max_new_tokens,
                      int32_t eos) {
    return int(guarded([&] {
        Request r;
        r.id = id;
        r.prompt_token_ids = tokens_of(prompt, count);
        r.generation.max_new_tokens = max_new_tokens;
        if (eos >= 0) r.generation.eos_token_id = eos;
        e->engine->submit(std::move(r));
        e->index.emplace(id, int32_t(e->index.size()));
        return 0L;
    }));
}
int mph_engine_step(mph_engine* e) {
    return int(guarded([&] { return e->engine->step() ? 1L : 0L; }));
}
long mph_engine_poll(mph_engine* e, char* buffer, long capacity) {
    std::string text;
    for (const auto& ev : e->engine->poll_events())
        text += ev.request_id + "\t" + std::to_string(ev.token_id ? *ev.token_id : -1) + "\t" +
                std::to_string(ev.finish_reason ? int(*ev.finish_reason) : -1) + "\t" + ev.error_message + "\n";
    const long n = long(text.size());
    if (buffer && capacity > 0) {
        const long c = n < capacity - 1 ? n : capacity - 1;
        std::memcpy(buffer, text.data(), std::size_t(c));
        buffer[c] = 0;
    }
    return n;
}
long mph_engine_poll_compact(mph_engine* e, int32_t* request, int32_t* token, int32_t* reason, long capacity) {
    const auto events = e->engine->poll_events();
    long i = 0;
    for (const auto& ev : events) {
        if (i < capacity) {
            auto it = e->index.find(ev.request_id);
            request[i] = it == e->index.end() ? -1 : it->second;
            token[i] = ev.token_id ? *ev.token_id : -1;
            reason[i] = ev.finish_reason ? int32_t(*ev.finish_reason) : -1;
        }
        ++i;
    }
    return long(events.size());
}
int mph_engine_cancel(mph_engine* e, const char* id) {
    return int(guarded([&] {
        e->engine->cancel(id);
        return 0L;
    }));
}
int mph_engine_shutdown(mph_engine* e) {
    return int(guarded([&] {
        e->engine->shutdown();
        return 0L;
    }));
}
int mph_engine_idle(mph_engine* e) { return e->engine->idle() ? 1 : 0; }
int mph_engine_failed(mph_engine* e) { return e->engine->failed() ? 1 : 0; }
int mph_engine_step_stats(mph_engine* e, size_t* out) {
    const auto& s = e->engine->last_step_stats();
    out[0] = s.prefix_reused_tokens;
    out[1] = s.prefill_tokens;
    out[2] = s.decode_tokens;
    return 0;
}
int mph_engine_runner_stats(mph_engine* e, size_t* out) {
    runner_stats_out(e->engine->runner().stats(), out);
    return 0;
}
int mph_engine_cost_stats(mph_engine* e, uint64_t* out) {
    cost_out(e->engine->runner().cost_stats(), out);
    return 0;
}
int mph_engine_sequence(mph_engine* e, const char* id, int32_t* used, int32_t* blocks, int32_t capacity) {
    return int(guarded([&] {
        if (e->b200) return long(sequence_out(e->b200->kv().sequence(id), used, blocks, capacity));
        if (e->scripted) return long(sequence_out(e->scripted->kv().sequence(id), used, blocks, capacity));
        throw std::logic_error("runner without a visible KV manager");
    }));
}
int mph_engine_flushes(mph_engine* e, size_t* flushes, size_t* hazard_flushes) {
    *flushes = e->b200 ? e->b200->flushes() : 0;
    *hazard_flushes = e->b200 ? e->b200->hazard_flushes() : 0;
    return 0;
}

mp_context* mph_engine_device(mph_engine* e) { return e->b200 ? e->b200->device() : nullptr; }

int mph_engine_capture_logits(mph_engine* e, int32_t on) {
    return int(guarded([&]() -> long {
        if (!e->b200) throw std::logic_error("logits capture needs a B200 runner");
        e->b200->set_logits_capture(on != 0);
        return 0;
    }));
}

long mph_engine_logits(mph_engine* e, const char* id, float* out, long capacity) {
    if (!e->b200) return -2;
    std::vector<float> logits;
    if (!e->b200->captured_logits(id, logits)) return -1;
    const long n = long(logits.size());
    if (out) std::copy(logits.begin(), logits.begin() + std::min(n, capacity), out);
    return n;
}

}  // extern "C"
