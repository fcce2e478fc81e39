/*
 * miniprefix_b200_host.h -- C ABI of the host layer: page pool + exact prefix
 * cache, KV manager, B200 runner and engine (libmpb200_host.so).
 *
 * Each handle wraps one C++ object of the host layer, whose contract is the
 * reference MiniPrefix one (TinyInfer v0.3.0):
 *   mph_cache_*  KvBlockPool + ExactPrefixCache   (miniprefix/include/miniprefix/paged_kv.h:25-51,
 *                                                   prefix_cache.h:9-34)
 *   mph_kv_*     KVManager and its Append          (miniprefix/include/miniprefix/kv_manager.h:20-96)
 *   mph_runner_* ModelRunner: the B200 runner, or a device-free scripted runner
 *                for host-logic tests              (miniprefix/include/miniprefix/model.h:35-62)
 *   mph_engine_* Engine                            (miniprefix/include/miniprefix/engine.h:12-36)
 * Request ids are NUL-terminated strings; token arrays are int32.
 *
 * Return codes: >= 0 success (some calls return a count); the C++ exception a
 * reference call would throw maps to -1 std::invalid_argument, -2 std::logic_error,
 * -3 KvCapacityError, -4 other std::runtime_error, -5 std::out_of_range, -6 other.
 * mph_last_error() returns the exception message of the last failure on this thread.
 */
#ifndef MINIPREFIX_B200_HOST_H
#define MINIPREFIX_B200_HOST_H

#include <stddef.h>
#include <stdint.h>

#include "miniprefix_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mph_cache mph_cache;
typedef struct mph_kv mph_kv;
typedef struct mph_runner mph_runner;
typedef struct mph_engine mph_engine;

const char* mph_last_error(void);

/* ---- page pool + prefix cache over named test sequences
 * (the operations miniprefix/tests/prefix_cache_test.cpp drives). */
mph_cache* mph_cache_new(int32_t block_tokens, int32_t max_blocks, int32_t prefix_blocks, int32_t layers,
                         int32_t width);
void mph_cache_free(mph_cache* c);
int mph_cache_append(mph_cache* c, const char* seq, const int32_t* tokens, int32_t count); /* reserve + commit */
int mph_cache_publish(mph_cache* c, const char* seq);
long mph_cache_reuse(mph_cache* c, const char* seq, const int32_t* prompt, int32_t count);
int mph_cache_release(mph_cache* c, const char* seq);
int mph_cache_evict_one(mph_cache* c); /* 1 evicted, 0 nothing to evict */
/* Undo window over pool, index and sequences (the batched engine's step
 * checkpoint): op 0 opens it, 1 rolls everything back to the opening state, 2
 * keeps the changes and closes it. */
int mph_cache_journal(mph_cache* c, int32_t op);
int mph_cache_clear(mph_cache* c);
/* size, index_nodes, key_token_bytes, hits, misses, reused_tokens, evictions,
 * cache_only_blocks, live_blocks, peak_blocks, free_blocks */
int mph_cache_stats(mph_cache* c, uint64_t* out11);
int mph_cache_references(mph_cache* c, uint64_t* out, int32_t count);
/* Sets a named sequence's fields verbatim, without page accounting (tests build
 * malformed sequences this way, as miniprefix/tests/prefix_cache_test.cpp:81 does). */
int mph_cache_define(mph_cache* c, const char* seq, int32_t used, const int32_t* tokens, int32_t token_count,
                     const int32_t* blocks, int32_t block_count);
int mph_cache_sequence(mph_cache* c, const char* seq, int32_t* used, int32_t* blocks, int32_t capacity,
                       int32_t* tokens, int32_t token_capacity);

/* ---- KV manager */
mph_kv* mph_kv_new(int32_t block_tokens, int32_t max_blocks, int32_t prefix_blocks, int32_t layers, int32_t width,
                   int32_t context, int32_t vocabulary);
void mph_kv_free(mph_kv* m);
int mph_kv_reserve(mph_kv* m, const char* id, size_t max_tokens); /* 0 Ready, 1 Wait, 2 Impossible */
int mph_kv_release_reservation(mph_kv* m, const char* id);
int mph_kv_create(mph_kv* m, const char* id);
int mph_kv_fork(mph_kv* m, const char* source, const char* target);
long mph_kv_reuse_prefix(mph_kv* m, const char* id, const int32_t* prompt, int32_t count);
int mph_kv_cache_prefix(mph_kv* m, const char* id);
int mph_kv_clear_prefix_cache(mph_kv* m);
/* One Append transaction. mode 0: copy and commit; 1: roll back; 2: the copier
 * throws, commit must be refused, then roll back. tail3 = {source, destination,
 * valid} or -1s; region5 = the merged TailCopyRegion when one was copied. */
int mph_kv_append(mph_kv* m, const char* id, const int32_t* tokens, int32_t count, int32_t mode, long* tail3,
                  size_t* region5);
int mph_kv_reset_sequence(mph_kv* m, const char* id);
int mph_kv_release(mph_kv* m, const char* id);
int mph_kv_clear(mph_kv* m);
int mph_kv_stats(mph_kv* m, size_t* out16); /* KvStats field order */
int mph_kv_sequence(mph_kv* m, const char* id, int32_t* used, int32_t* blocks, int32_t capacity);
long mph_kv_offset(mph_kv* m, const char* id, int32_t layer, int32_t token);

/* ---- runners */
/* The B200 runner: model config, per-sequence context limit, KvCacheConfig, and
 * device capacities. Weights follow with mph_runner_set_weight + finalize. */
mph_runner* mph_runner_new_b200(int32_t device, const mp_model_config* model, int32_t context, int32_t block_tokens,
                                int32_t max_blocks, int32_t prefix_blocks, int32_t max_sequences,
                                int32_t max_step_tokens, int32_t max_step_sequences);
int mph_runner_set_weight(mph_runner* r, const char* name, const float* data, size_t elements);
int mph_runner_finalize(mph_runner* r);
/* The B200 runner built from an MPFX0001 model file: what make_cuda_runner(
 * ModelWeights::load(path), context, kv) does in the reference (model.h:59-62,
 * model.cpp:20-56). The file's config and every tensor are checked as the
 * reference loader checks them (same messages); tensors stream to the device one
 * at a time and the weights are finalized. NULL on failure (mph_last_error). */
mph_runner* mph_runner_new_b200_file(int32_t device, const char* path, int32_t context, int32_t block_tokens,
                                     int32_t max_blocks, int32_t prefix_blocks, int32_t max_sequences,
                                     int32_t max_step_tokens, int32_t max_step_sequences);
/* MPFX0001 reading without a device: the config alone, or the config and every
 * tensor (in file order) through `sink`, which returns 0 to continue. Errors as
 * the reference loader's (mph_last_error), -1 invalid argument, -4 format. */
typedef int (*mph_tensor_sink)(const char* name, const float* data, uint64_t elements, void* user);
/* Worker protocol v3 (miniprefix/apps/protocol/session.cpp) over the engine: serves the
 * newline-separated commands of `input` until QUIT or their end and writes the
 * response lines into `out` (NUL-terminated, at most capacity - 1 bytes).
 * Returns the full response length. The mpb200_worker executable serves the same
 * protocol on stdin/stdout. */
long mph_engine_serve(mph_engine* e, const char* input, char* out, long capacity);
int mph_mpfx_config(const char* path, mp_model_config* out);
int mph_mpfx_read(const char* path, mp_model_config* out, mph_tensor_sink sink, void* user);
/* Device-free runner with the real KV manager and scripted one-hot logits. */
mph_runner* mph_runner_new_scripted(int32_t vocabulary, int32_t context, int32_t layers, int32_t width,
                                    int32_t block_tokens, int32_t max_blocks, int32_t prefix_blocks);
int mph_runner_script(mph_runner* r, const char* id, const int32_t* tokens, int32_t count);
int mph_runner_poison(mph_runner* r, int32_t token);
void mph_runner_free(mph_runner* r);
int mph_runner_reserve(mph_runner* r, const char* id, size_t tokens);
int mph_runner_release_reservation(mph_runner* r, const char* id);
int mph_runner_create(mph_runner* r, const char* id);
int mph_runner_fork(mph_runner* r, const char* source, const char* target);
long mph_runner_reuse_prefix(mph_runner* r, const char* id, const int32_t* prompt, int32_t count);
int mph_runner_cache_prefix(mph_runner* r, const char* id);
int mph_runner_clear_prefix_cache(mph_runner* r);
/* Returns the vocabulary size; logits may be NULL. */
int mph_runner_append(mph_runner* r, const char* id, const int32_t* tokens, int32_t count, float* logits);
int mph_runner_release(mph_runner* r, const char* id);
int mph_runner_clear(mph_runner* r);
int mph_runner_stats(mph_runner* r, size_t* out25);  /* RunnerStats field order */
int mph_runner_cost_stats(mph_runner* r, uint64_t* out8); /* CostStats field order */
int mph_runner_set_cost_timing(mph_runner* r, int32_t enabled);
int mph_runner_context_limit(mph_runner* r);
int mph_runner_sequence(mph_runner* r, const char* id, int32_t* used, int32_t* blocks, int32_t capacity);
/* Scripted runner: recorded COW regions (5 size_t each), cleared on read. */
long mph_runner_regions(mph_runner* r, size_t* out, long capacity);

/* ---- engine (takes ownership of the runner; the runner handle becomes a view) */
mph_engine* mph_engine_new(mph_runner* runner, int32_t max_batch, int32_t token_budget, int32_t prefill_chunk,
                           int32_t context);
void mph_engine_free(mph_engine* e);
int mph_engine_submit(mph_engine* e, const char* id, const int32_t* prompt, int32_t count, uint32_t max_new_tokens,
                      int32_t eos /* < 0: none */);
int mph_engine_step(mph_engine* e); /* 1 progressed, 0 not */
/* Drains events as text lines "id\ttoken\treason\terror\n" (token/reason -1 when
 * absent; reason 0 Eos, 1 Length, 2 Cancelled, 3 Error). Returns the byte count. */
long mph_engine_poll(mph_engine* e, char* buffer, long capacity);
/* Drains events as arrays: per event request index (order of submission),
 * token (-1 none) and reason (-1 none). Returns the event count. Messages are
 * dropped; use mph_engine_poll for them. */
long mph_engine_poll_compact(mph_engine* e, int32_t* request, int32_t* token, int32_t* reason, long capacity);
int mph_engine_cancel(mph_engine* e, const char* id);
int mph_engine_shutdown(mph_engine* e);
int mph_engine_idle(mph_engine* e);
int mph_engine_failed(mph_engine* e);
int mph_engine_step_stats(mph_engine* e, size_t* out3); /* reused, prefill, decode tokens */
int mph_engine_runner_stats(mph_engine* e, size_t* out25);
int mph_engine_cost_stats(mph_engine* e, uint64_t* out8);
int mph_engine_sequence(mph_engine* e, const char* id, int32_t* used, int32_t* blocks, int32_t capacity);
/* Device forwards launched by the B200 runner so far, and how many of them were
 * split off early to keep a reused page's old readers ahead of its new writer. */
int mph_engine_flushes(mph_engine* e, size_t* flushes, size_t* hazard_flushes);
/* The device context of the engine's B200 runner (NULL for other runners), for
 * timing and counters through include/miniprefix_b200.h. */
mp_context* mph_engine_device(mph_engine* e);
/* Parity checks of batched runs (no counterpart in the reference, whose append()
 * returns every request's logits): while capture is on, each device forward of
 * the engine's B200 runner also downloads the logits of its appends, and
 * mph_engine_logits copies the latest ones of request `id` (at most `capacity`
 * floats) and returns the vocabulary size, or -1 when none were captured, -2
 * when the runner is not a B200 runner. Switching capture off drops them. */
int mph_engine_capture_logits(mph_engine* e, int32_t on);
long mph_engine_logits(mph_engine* e, const char* id, float* out, long capacity);

#ifdef __cplusplus
}
#endif
#endif
