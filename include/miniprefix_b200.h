/*
 * miniprefix_b200.h -- C ABI of the B200 (sm_100a) MiniPrefix forward over paged KV.
 *
 * This is the drop-in boundary for the device half of TinyInfer MiniPrefix's
 * CudaRunner (TinyInfer v0.3.0, miniprefix/src/backend/cuda/llama_runner.cu). The
 * reference's host bookkeeping (KVManager, ExactPrefixCache, Engine) keeps owning
 * metadata; it calls these functions where CudaRunner called cudaMalloc, cuBLAS,
 * its seven kernels and cudaMemcpy*. Plain C types only; every pointer is
 * caller-owned unless stated. One context per GPU, single-threaded per context
 * (the reference's ModelRunner contract, miniprefix/include/miniprefix/kv_manager.h:18-19).
 *
 * Return codes: MP_OK or one of MP_ERR_*; mp_last_error() gives the message of
 * the last failure on the calling thread.
 */
#ifndef MINIPREFIX_B200_H
#define MINIPREFIX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MP_OK 0
#define MP_ERR_INVALID 1     /* rejected argument; no state changed */
#define MP_ERR_CUDA 2        /* CUDA runtime failure */
#define MP_ERR_NONFINITE 3   /* a logit of the step was NaN/Inf */
#define MP_ERR_BOUNDS 4      /* device bounds check tripped (page id, token, region) */
#define MP_ERR_TIMEOUT 5     /* bounded wait expired (host sync or in-kernel copy wait) */
#define MP_ERR_NOMEM 6       /* device allocation failed */
#define MP_ERR_UNSUPPORTED 7 /* model geometry outside the specialised kernels */

typedef struct mp_context mp_context;

/* Mirrors miniprefix::ModelConfig (miniprefix/include/miniprefix/model.h:9-16). */
typedef struct {
    int32_t layers, hidden, intermediate, heads, kv_heads, vocabulary, context, eos;
    float rms_epsilon, rope_theta;
    int32_t tied;
} mp_model_config;

/* Paged KV pool and step capacities. block_tokens / max_blocks are
 * KvCacheConfig's (miniprefix/include/miniprefix/paged_kv.h:13-17); each of the K
 * and V pools holds max_blocks * layers * block_tokens * kv_width floats. On the
 * device a pool is layer-major, [layer][block][slot][kv_width], so that one layer's
 * pages share a compact address range; every pool offset this API takes (COW
 * regions, mp_kv_read / mp_kv_write) is an offset in the reference layout
 * [block][layer][slot][kv_width] (paged_kv.h:25-27) and is translated. */
typedef struct {
    int32_t block_tokens;
    int32_t max_blocks;
    int32_t max_sequences;      /* device block-table slots */
    int32_t table_stride;       /* entries per slot: >= ceil(context / block_tokens) */
    int32_t max_step_tokens;    /* most tokens one forward may carry (sum over sequences) */
    int32_t max_step_sequences; /* most sequences one forward may carry */
} mp_runtime_config;

/* One sequence of a forward: `count` new tokens appended at positions
 * start .. start+count-1 of the sequence whose block table lives in `slot`. The
 * table must already map every page that covers start+count tokens. */
typedef struct {
    int32_t slot, start, count;
} mp_sequence_desc;

/* One block-table entry: tables[slot][index] = block. */
typedef struct {
    int32_t slot, index, block;
} mp_table_entry;

/* KVManager::TailCopyRegion (miniprefix/include/miniprefix/kv_manager.h:38): float
 * element offsets into ONE pool; the copy is applied to both the K and V pools. */
typedef struct {
    uint64_t destination, source, pitch, width, rows;
} mp_tail_copy_region;

const char* mp_last_error(void);

/* Replaces CudaRunner's constructor (llama_runner.cu:78-87): selects `device`,
 * creates the stream, allocates weights, both pools (zeroed), tables and the
 * step workspace. */
int mp_create(int device, const mp_model_config* model, const mp_runtime_config* runtime, mp_context** out);
void mp_destroy(mp_context* ctx);

/* Replaces upload_parameter (llama_runner.cu:72-76): one MPFX0001 tensor by name,
 * [in, out] orientation as stored by the reference (miniprefix/src/model/model.cpp:28-38).
 * The tied head is read from the embedding; no transposed copy is made (:84). */
int mp_set_weight(mp_context* ctx, const char* name, const float* host, size_t elements);
/* Checks every tensor arrived and packs the device copies. Required before forward. */
int mp_finalize_weights(mp_context* ctx);

/* Replaces the incremental block-table upload (llama_runner.cu:139-143, :113):
 * entries [first, first+count) of `slot` := blocks. Queued on the context stream. */
int mp_table_write(mp_context* ctx, int32_t slot, int32_t first, const int32_t* blocks, int32_t count);

/* Replaces the COW cudaMemcpy2DAsync pair (llama_runner.cu:130-137), batched:
 * every region copies rows x width floats at pitch in both pools. */
int mp_cow_copy(mp_context* ctx, const mp_tail_copy_region* regions, int32_t count);

/* Replaces the append body (llama_runner.cu:128-170) for a BATCH of sequences:
 * uploads tokens, descriptors, block-table entries and COW regions in one copy,
 * applies the table entries, performs the COW copies (all layers, both pools,
 * before any layer runs), runs the 30-layer forward, and downloads per
 * sequence the greedy token (first index of the maximum, engine.cpp:99), a
 * finiteness flag (:94-95) and, when out_logits is not NULL, the full last-row
 * logits (sequences x vocabulary floats, the reference's append() result).
 * Blocks until the step completed or timeout_ms elapsed (MP_ERR_TIMEOUT).
 * Returns MP_ERR_NONFINITE when any sequence had a nonfinite logit (outputs are
 * still written) and MP_ERR_BOUNDS when a device bounds check tripped. */
int mp_forward(mp_context* ctx, const mp_sequence_desc* sequences, int32_t count, const int32_t* tokens,
               const mp_table_entry* entries, int32_t entry_count, const mp_tail_copy_region* regions,
               int32_t region_count, int32_t* out_tokens, int32_t* out_finite, float* out_logits,
               int32_t timeout_ms);

/* The same step split in three, for callers that keep inputs resident and time
 * the device work alone: prepare uploads, launch only enqueues kernels that read
 * device memory, collect downloads and waits. */
int mp_forward_prepare(mp_context* ctx, const mp_sequence_desc* sequences, int32_t count, const int32_t* tokens,
                       const mp_table_entry* entries, int32_t entry_count, const mp_tail_copy_region* regions,
                       int32_t region_count);
int mp_forward_launch(mp_context* ctx);
int mp_forward_collect(mp_context* ctx, int32_t* out_tokens, int32_t* out_finite, float* out_logits,
                       int32_t timeout_ms);

/* Failure-path tests (no counterpart in the reference, whose kernels have no
 * bounded waits): the next forward's first GEMM launch gets a producer that issues
 * no copies and waits bounded at `wait_us` microseconds (1 us .. 1 s). Its waits run
 * out, the kernel records the timeout bit, releases its tensor memory and returns,
 * and that forward reports MP_ERR_TIMEOUT (its outputs and the K/V rows it should
 * have written are garbage). The context stays usable: later forwards are normal. */
int mp_inject_wait_timeout(mp_context* ctx, int32_t wait_us);
/* Waits for all queued work with a bounded host wait (event polling). */
int mp_sync(mp_context* ctx, int32_t timeout_ms);

/* Device pointers of the K and V pools (layer-major, see mp_runtime_config) and
 * their element count (tests, tools). */
int mp_kv_pools(mp_context* ctx, float** keys, float** values, uint64_t* elements);
/* Synchronous host copies of pool payload (0 = K pool, 1 = V pool), element
 * offsets in the reference layout; for tests and tools that inspect or seed pages. */
int mp_kv_read(mp_context* ctx, int32_t pool, uint64_t offset, uint64_t count, float* host);
int mp_kv_write(mp_context* ctx, int32_t pool, uint64_t offset, uint64_t count, const float* host);
/* The context stream as a cudaStream_t (void* here to keep the ABI CUDA-free). */
void* mp_stream(mp_context* ctx);

/* Device event timing on the context stream: mp_timer_mark records a mark;
 * mp_timer_elapsed gives milliseconds between the last two marks. */
int mp_timer_mark(mp_context* ctx);
int mp_timer_elapsed(mp_context* ctx, float* milliseconds);
/* When enabled, forward launches bracket every attention launch with events;
 * mp_profile_read returns the summed attention milliseconds and launch count
 * since the last read (and resets them). */
int mp_profile_enable(mp_context* ctx, int32_t enabled);
/* No counterpart in the reference. Shared-prefix decode attention: decode rows
 * whose block tables start with the same physical pages (prefix reuse, forks)
 * form a group when at least min_rows rows share at least min_tokens tokens of
 * full pages, and a tensor-core kernel reads the group's shared pages once for
 * all its rows. min_rows 0 (the default) turns it off: every row then reads its
 * whole context, and the shared pages, read by many rows, stay in L2 -- measured
 * faster on B200 for every workload tried (1K-7K shared tokens x 256 rows, and
 * prefix-tree serving). */
int mp_set_shared_prefix(mp_context* ctx, int32_t min_rows, int32_t min_tokens);
int mp_profile_read(mp_context* ctx, float* attention_ms, int32_t* attention_launches, double* attention_bytes);
/* The same profiling (no counterpart in the reference) for the projection GEMMs:
 * the summed milliseconds and count of the intervals between one layer's attention
 * and the next layer's (each: O, gate/up and down of a layer plus the next layer's
 * QKV), and of the LM head GEMM; reset on read. */
int mp_profile_read_gemm(mp_context* ctx, float* layer_gemm_ms, int32_t* intervals, float* head_ms, int32_t* heads);
/* Cumulative counters of collected forwards: device time from the first to the
 * last kernel of each forward (CUDA events on the context stream), kernels
 * launched, and bytes moved host->device / device->host by the forwards;
 * shared_prefix_rows counts decode rows whose leading pages were served by the
 * shared-prefix kernel (once per forward), shared_prefix_tokens the tokens those
 * rows did not read themselves. host_prepare_ms, host_launch_ms and host_wait_ms
 * are host wall time spent in mp_forward_prepare (validation, attention plan,
 * metadata upload), mp_forward_launch (enqueueing the kernels) and waiting for
 * completion in mp_forward_collect. */
typedef struct {
    uint64_t forwards;
    double forward_ms;
    uint64_t kernel_launches;
    uint64_t h2d_bytes, d2h_bytes;
    uint64_t shared_prefix_rows, shared_prefix_tokens;
    double host_prepare_ms, host_launch_ms, host_wait_ms;
} mp_counters;
int mp_read_counters(mp_context* ctx, mp_counters* out, int32_t reset);

/* Device time of the COW copies of the last collected forward that had any
 * (milliseconds; 0 when it had none). Recorded only while cost timing is on. */
int mp_cow_timing(mp_context* ctx, int32_t enabled);
int mp_cow_elapsed(mp_context* ctx, float* milliseconds);

/* C = A . B^T (a [m][k], b [n][k], c [m][n] row-major, device buffers) through the
 * split-precision FP16 tcgen05 GEMM of the forward (each operand as FP16 halves,
 * three products per useful one; Store epilogue, with the forward's split-K
 * choice: shapes with few output tiles run as K slices summed in slice order);
 * n a multiple of 64, k of 32. Allocates its own scratch and synchronises
 * `stream`: a test/tool entry, not the hot path. */
int mp_gemm_f32(const float* a, const float* b, float* c, int32_t m, int32_t n, int32_t k, void* stream);

/* The paged-attention decode OPERATOR alone (one query row per sequence), on
 * caller device buffers: q [count][9*64] roped queries, pools in the reference
 * layout with `layers` layers, tables [count][table_stride] (device), out
 * [count][9*64]. `lengths` is a HOST array (tokens to attend per sequence);
 * pages_per_split 0 cuts the sequences' pages, concatenated, into one equal run
 * per CTA of a single wave (3 per SM); > 0 cuts each sequence into slices of
 * that many pages, pulled longest first by the wave. Runs on `stream`
 * (cudaStream_t, NULL = legacy default) and does not synchronise. Uses an
 * internal scratch buffer that grows on demand. */
int mp_paged_attention_decode(const float* q, const float* keys, const float* values, int32_t layers, int32_t layer,
                              int32_t block_tokens, int32_t max_blocks, const int32_t* tables, int32_t table_stride,
                              const int32_t* lengths, int32_t count, float* out, int32_t pages_per_split, void* stream);
/* No counterpart in the reference. The same decode operator for callers that
 * cannot allocate device memory -- e.g. a host embedding this library in another
 * runtime that owns all GPU memory or fixes its budget up front, or a path where
 * cudaMalloc/cudaFree must not run because they synchronise the device. It calls
 * no allocator: its scratch is one file-scope __device__ array of about 5 MB held
 * by every GPU that loads the library. At most 512 sequences and 2048 slices per
 * call (pages_per_split 0: equal runs per CTA, which always fit); larger requests return
 * MP_ERR_INVALID. All calls on a device share that array: calls whose device work
 * overlaps race. The first call on a device, with that device current, looks up
 * the array's address; make it before any stream capture. `device_error`
 * (optional, caller-owned device word, zeroed by the caller) receives the kernel's
 * error bits (1 = page id out of range, 2 = copy wait expired); when it is NULL the
 * bits go to a word inside the fixed array, which mp_paged_attention_status reads
 * and clears (before the next call on the device, which clears it again). */
int mp_paged_attention_decode_noalloc(const float* q, const float* keys, const float* values, int32_t layers,
                                      int32_t layer, int32_t block_tokens, int32_t max_blocks, const int32_t* tables,
                                      int32_t table_stride, const int32_t* lengths, int32_t count, float* out,
                                      int32_t pages_per_split, void* stream, uint32_t* device_error);
/* Synchronises `stream`, then reads and clears the decode operators' device error
 * words on the current device (mp_paged_attention_decode's, and the word that
 * mp_paged_attention_decode_noalloc fills when given no device_error): MP_OK,
 * MP_ERR_BOUNDS (a page id outside [0, max_blocks)) or MP_ERR_TIMEOUT (an in-kernel
 * copy wait expired; the allocating operator's arrival counters are reset). */
/* The paged-attention PREFILL operator alone: causal attention of chunks of
 * query rows (miniprefix/src/backend/cuda/llama_runner.cu:33-48 for rows past the
 * first; the CPU runner's loop miniprefix/src/backend/cpu/llama_runner.cpp:85-93).
 * Sequence i appends seq_counts[i] rows at positions seq_starts[i] ..
 * seq_starts[i] + seq_counts[i] - 1; its rows are consecutive in q and out
 * ([rows][9*64], sequences in order) and its K/V rows up to the last position are
 * already in the pools. Row r attends to the sequence's tokens 0 .. its position.
 * seq_starts / seq_counts are HOST arrays; tables [count][table_stride] (device).
 * Runs the tensor-core prefill kernel on `stream` without synchronising; shares
 * the decode operator's internal scratch (errors: mp_paged_attention_status). */
int mp_paged_attention_prefill(const float* q, const float* keys, const float* values, int32_t layers,
                               int32_t layer, int32_t block_tokens, int32_t max_blocks, const int32_t* tables,
                               int32_t table_stride, const int32_t* seq_starts, const int32_t* seq_counts,
                               int32_t count, float* out, void* stream);
int mp_paged_attention_status(void* stream);

#ifdef __cplusplus
}
#endif
#endif
