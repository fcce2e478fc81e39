// Host-visible launch interfaces of the sm_100a kernels (internal to the library;
// the public boundary is include/miniprefix_b200.h).
#pragma once
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace mpb {

// Attention geometry the kernels are specialised for (SmolLM2-135M shape):
// 9 query heads share 3 KV heads of dimension 64 (GQA group 3).
constexpr int kHeads = 9;
constexpr int kKvHeads = 3;
constexpr int kHeadDim = 64;
constexpr int kGroup = kHeads / kKvHeads;
constexpr int kKvWidth = kKvHeads * kHeadDim;  // 192 floats per token per pool
constexpr int kQWidth = kHeads * kHeadDim;     // 576

// Page addressing in a K or V pool of `block_tokens`-slot pages (kKvWidth floats
// per slot). The page of (block, layer) starts at
//   pool_page(block, page_stride, layer_offset) * block_tokens * kKvWidth
// floats. Two layouts use it:
//  * the reference's [block][layer][slot][192] (caller pools of the operator entry
//    points): page_stride = layers, layer_offset = layer;
//  * layer-major [layer][block][slot][192] (the forward context's own pools, so one
//    layer's pages share a compact address range): page_stride = 1,
//    layer_offset = layer * max_blocks.
__host__ __device__ __forceinline__ size_t pool_page(int block, int page_stride, int64_t layer_offset) {
    return size_t(block) * size_t(page_stride) + size_t(layer_offset);
}

// Device error word bits (read back by the host after each step).
enum : unsigned {
    kErrBounds = 1u,    // a block-table entry or index fell outside its buffer
    kErrTimeout = 2u,   // a bounded wait on a copy gave up
};


// One CTA of paged attention: query row `row`, context pages [page_begin, page_end).
// Slices of a row are contiguous in the work list, in page order.
struct AttnWork {
    int32_t row;
    int32_t page_begin;
    int32_t page_end;
    int32_t split;
};

struct AttnParams {
    const float* q;  // roped queries, [rows][q_stride], 9 heads x 64 per row
    int q_stride;
    const float* keys;    // K pool, pages addressed by pool_page(block, page_stride, layer_offset)
    const float* values;  // V pool, same layout
    int page_stride, block_tokens, max_blocks;
    int64_t layer_offset;
    const int32_t* tables;  // [slots][table_stride] physical page ids
    int table_stride;
    const int32_t* row_slot;    // table slot of each query row
    const int32_t* row_len;     // causal context length of each query row
    const int32_t* row_splits;  // slices of each row
    const int32_t* row_work0;   // first work index of each row
    const int32_t* row_x0;      // first shared-prefix partial slot of each row
    const int32_t* row_nx;      // shared-prefix partial slots of each row (0: none)
    const AttnWork* work;
    int work_count;
    const int32_t* order;  // optional processing order of the work items (longest first)
    unsigned* sched;       // optional [2] zeroed counters: persistent CTAs pull work items
    // optional static schedule ([cta_count + 1]): CTA c processes work items
    // [cta_items[c], cta_items[c + 1]) in order (order and sched unused)
    const int32_t* cta_items;
    int cta_count;
    float* partial;      // [slots][9][66] slice results: work items first, then shared-prefix slots
    unsigned* counters;  // [rows][3 kv heads] zero between launches
    float* out;          // [rows][out_stride] FP32 output (when out_hi is null)
    __half* out_hi;      // optional: the output as the O projection's FP16 operand
    __half* out_lo;      // halves (split_f16), same layout; `out` is then unused
    int out_stride;
    unsigned* error;
    // Static schedule only: the schedule arrays, the tables and every page token
    // below row_len - kPrefillMinRows were written before the previous kernel
    // started (host upload, table patch, COW copies, earlier layers), so the
    // producer may read them, and fill its ring, before the programmatic wait.
    // Tokens at or past that bound may be the rows' appends by the preceding
    // QKV epilogue (a decode row's sequence appends fewer than kPrefillMinRows).
    int early_copies;
};

// Shared-prefix decode attention (attention_shared.cu). Decode rows whose block
// tables start with the same physical pages form a group; the group's shared
// tokens are read once per launch for all its rows. One CTA per (group, kv head,
// block of kPrefixQueries (row, head) query vectors, token chunk of whole
// kPrefixSubChunk-token sub-chunks) writes (max, sum, unnormalised output)
// partials that the decode kernel's split merge combines with the rows' own slices.
constexpr int kPrefixQueries = 128;
constexpr int kPrefixSubChunk = 64;
struct PrefixWork {
    int32_t group;
    int32_t kv_head;
    int32_t q_begin;    // first query vector (row_in_group * 3 + head_in_group)
    int32_t q_count;    // 1..kPrefixQueries
    int32_t tok_begin;  // shared tokens [tok_begin, tok_end) of this chunk
    int32_t tok_end;
    int32_t chunk;      // partial slot offset within each row's shared-prefix slots
    int32_t pad;
};
struct PrefixParams {
    const float* q;
    int q_stride;
    const float* keys;
    const float* values;
    int page_stride, block_tokens, max_blocks;
    int64_t layer_offset;  // pool_page()
    const int32_t* tables;
    int table_stride;
    const int32_t* group_rows;  // batch rows of every group, concatenated
    const int32_t* group_row0;  // [groups + 1] offsets into group_rows
    const int32_t* group_slot;  // [groups] table slot whose table maps the shared pages
    const int32_t* row_x0;      // first shared-prefix partial slot of each row
    const PrefixWork* work;
    int work_count;
    float* partial;
    unsigned* error;
};
cudaError_t launch_prefix_attention(const PrefixParams& p, cudaStream_t stream);
cudaError_t configure_prefix_attention();

// Chunked prefill: one CTA per (64-row query tile of one sequence, kv head).
struct PrefillWork {
    int32_t row0;      // batch row of the tile's first query
    int32_t rows;      // valid rows in the tile (1..kPrefillTileRows)
    int32_t position;  // sequence position of the first row
    int32_t slot;      // block-table slot of the sequence
    int32_t kv_head;
    int32_t pad[3];
};

struct PrefillParams {
    const float* q;
    int q_stride;
    const float* keys;
    const float* values;
    int page_stride, block_tokens, max_blocks;
    int64_t layer_offset;  // pool_page()
    const int32_t* tables;
    int table_stride;
    const PrefillWork* work;
    int work_count;
    float* out;
    __half* out_hi;  // optional FP16 operand halves, as in AttnParams
    __half* out_lo;
    int out_stride;
    unsigned* error;
};

// Sequences appending at least this many rows in one forward take the tiled
// prefill kernel; shorter appends (decode) take the split-K decode kernel per row.
constexpr int kPrefillMinRows = 8;
// query rows per prefill CTA: rows x 3 heads of a kv group fill the 128 rows of
// the tensor-core tile
constexpr int kPrefillTileRows = 42;

cudaError_t configure_prefill_attention();
cudaError_t launch_prefill_attention(const PrefillParams& p, cudaStream_t stream);
// Slice length (pages) of the split-K decode work list when the caller leaves it
// open: about two waves of the 148 SMs x 3 resident CTAs over all rows' tokens,
// never below 64 tokens per slice, rounded to whole 16-token stages.
inline int auto_pages_per_split(long long total_tokens, int block_tokens) {
    const long long target = 148LL * 3 * 2;
    long long slice = (total_tokens + target - 1) / target;
    if (slice < 64) slice = 64;
    slice = (slice + 15) / 16 * 16;
    const long long pages = slice / block_tokens;
    return int(pages < 1 ? 1 : pages);
}

#ifndef MPB_ATTN_CTAS_PER_SM
#define MPB_ATTN_CTAS_PER_SM 3
#endif
constexpr int kAttnCtasPerSm = MPB_ATTN_CTAS_PER_SM;  // resident decode-attention CTAs per SM
constexpr int kAttnPersistentCtas = 148 * kAttnCtasPerSm;  // one wave of the decode kernel
// Static decode schedule for the operator entry points: the rows' pages,
// concatenated in row order, cut into one equal run per CTA (min(persistent
// CTAs, total pages) runs; a run may end one row and start the next). A row's
// part of a run is one work item. Calls emit(row, page_begin, page_end, k) per
// item in order (k = the item's index within its row) and cta_start(c, items)
// when run c begins at item index `items` (c = 1 .. runs, the last one being
// the total). Returns the number of runs (CTAs).
template <class PagesOf, class Emit, class CtaStart>
inline int plan_static_runs(int rows, PagesOf pages_of, Emit emit, CtaStart cta_start) {
    long long total = 0;
    for (int r = 0; r < rows; ++r) total += pages_of(r);
    const long long runs = total < kAttnPersistentCtas ? (total > 0 ? total : 1) : kAttnPersistentCtas;
    auto run_end = [&](long long c) { return (c + 1) * total / runs; };
    long long pos = 0;
    int run = 0, items = 0;
    for (int r = 0; r < rows; ++r) {
        const int pages = pages_of(r);
        int k = 0;
        if (pages <= 0) {
            emit(r, 0, 0, k++);
            ++items;
        }
        for (int pg = 0; pg < pages;) {
            while (pos >= run_end(run)) cta_start(++run, items);
            const int n = int(std::min<long long>(pages - pg, run_end(run) - pos));
            emit(r, pg, pg + n, k++);
            ++items;
            pg += n;
            pos += n;
        }
    }
    while (run < runs) cta_start(++run, items);
    return int(runs);
}

cudaError_t configure_attention();
// Message returned by mp_last_error() on this thread.
void set_last_error(const char* message);
cudaError_t launch_paged_attention(const AttnParams& p, cudaStream_t stream);
// Reads and clears (on `stream`, synchronising it) the error word that
// mp_paged_attention_decode_noalloc writes for callers that pass no device_error;
// *bits = 0 when no such call has run on the current device. Allocates nothing.
cudaError_t noalloc_take_error(cudaStream_t stream, unsigned* bits);

// ---------------------------------------------------------------- GEMM
// C[M][N] (op) A[M][K] * B[N][K]^T, B stored K-contiguous ("nn.Linear" layout).
enum class Epilogue : int {
    Store = 0,   // C = acc
    AddTo = 1,   // C = C + acc  (residual add)
    SwiGLU = 2,  // gate/up column pairs -> silu(gate) * up as FP16 hi/lo halves
    Rope = 3,    // QKV projection (64-wide tiles = heads): RoPE on q and k, q to the
                 // attention input, k and v into the rows' page slots (TcGemmParams::rope)
};

// Epilogue::Rope: the rope_append step of the forward done by the QKV GEMM. Output
// columns are 9 q heads, 3 k heads, 3 v heads of 64; tile n0 / 64 is one head. Row
// r's position is row_pos[r]; its K/V slot is page tables[row_slot[r]][pos / bt],
// slot pos % bt of layer `layer`. Rotation x0' = x0 cos - x1 sin, x1' = x1 cos + x0
// sin of dims (d, d + 32) with host tables cos/sin[pos][d], each product rounded.
struct RopeEpilogue {
    const int32_t* row_pos;
    const int32_t* row_slot;
    const float* cos;
    const float* sin;
    int max_position;
    float* q;
    int q_stride;
    float* keys;
    float* values;
    const int32_t* tables;
    int table_stride;
    int page_stride, block_tokens, max_blocks;
    int64_t layer_offset;  // pool_page()
};

// GEMM operands in split precision. Every FP32 operand value x travels as two FP16
// halves (split_f16, common.cuh): hi = fp16(x) rounded to nearest and
// lo = fp16((x - hi) * 2^11), so x = hi + lo * 2^-11 within about 2^-23 |x|. The
// tensor-core GEMM forms the three products A_hi.B_hi + 2^-11 (A_hi.B_lo + A_lo.B_hi)
// (the dropped A_lo.B_lo term is below 2^-22 relative). |x| must stay below 65504,
// the FP16 range; a larger operand becomes infinite and the forward's logits then
// come out nonfinite, which the step reports as an error.
constexpr float kSplitLoScale = 2048.0f;
constexpr float kSplitLoUnscale = 1.0f / 2048.0f;

// Tensor-core split-precision GEMM (tc_gemm.cu). A and B come as FP16 hi/lo halves
// through 2-D TMA tensor maps (fp16, rows x K, 128-byte swizzle, boxes of 64 x 128
// rows for A and 64 x bn rows for B, bn = 64, 128 or 256); B's rows start at b_row0
// (stacked per-layer weights). Epilogues: Store / AddTo into c; SwiGLU expects B's
// rows in 32-row gate/up blocks (rows 64b..64b+31 gate, 64b+32..64b+63 up) and
// writes silu(gate) * up for output columns 32b..32b+31 as hi/lo halves (out_hi,
// out_lo). Small-M problems split K over a thread-block cluster of up to 8 CTAs
// per output tile, reduced in slice order through distributed shared memory
// (deterministic).
constexpr int kTcBN = 64;
struct TcGemmMaps {
    const struct CUtensorMap_st* a_hi;
    const struct CUtensorMap_st* a_lo;
    const struct CUtensorMap_st* b_hi;
    const struct CUtensorMap_st* b_lo;
};
struct TcGemmParams {
    int m, n, k;
    int bn;  // B tile rows (the B maps' box): 64, 128 or 256 (0: 64)
    int b_row0;
    float* c;
    int ldc;
    __half* out_hi;
    __half* out_lo;
    int ld_out;
    unsigned* error;
    RopeEpilogue rope;  // Epilogue::Rope only
    // RMSNorm folded into the GEMMs around it (hidden = N of the producer = K of the
    // consumer, a multiple of 64):
    //  * AddTo with norm_w: besides c, writes the FP16 halves of c[row] * norm_w
    //    (the next GEMM's A operand) into out_hi / out_lo (ld_out) and the sum of
    //    squares of each 64-column group of c[row] into ssq_out[row][n0 / 64];
    //  * Rope / SwiGLU with ssq_in: scales row r of the product by
    //    1 / sqrt(sum_g ssq_in[r][g] / k + eps) (groups in order) before the epilogue.
    const float* norm_w;
    float* ssq_out;
    const float* ssq_in;
    float eps;
    // Bound of each mbarrier wait in ns (0: kWaitNanoseconds), and the failure-path
    // test switch: with `stall` set the producer issues no copies, so every wait
    // runs out after wait_ns, the kernel records kErrTimeout and returns (no copy
    // is in flight, the tensor memory is released).
    uint64_t wait_ns;
    int stall;
    // The residual rows (AddTo) and the Rope destinations' metadata and block
    // tables were written at least two kernels earlier, so they may be gathered
    // before the programmatic wait (the forward's layer sequence guarantees it).
    int early_rows;
};
constexpr int kSsqGroup = 64;  // columns per partial sum of squares
cudaError_t configure_tc_gemm();
// K must be a multiple of 8 (16-byte rows for the tensor maps); a partial last
// 64-wide K block is zero-filled by the TMA engine.
cudaError_t launch_tc_gemm(const TcGemmMaps& maps, const TcGemmParams& p, Epilogue e, cudaStream_t stream);
// FP16 hi/lo operand halves of x (split_f16), elementwise.
cudaError_t launch_split(const float* x, __half* hi, __half* lo, size_t n, cudaStream_t stream);

// ---------------------------------------------------------------- fused small ops
// x[r][:] = embed[tokens[r]][:]; rmsnorm(x[r]) * w written as FP16 hi/lo halves, or
// with ssq (norm folded into the next GEMM): x[r] * w as halves and the sums of
// squares of x[r]'s 64-column groups into ssq[r][hidden / 64].
cudaError_t launch_embed_rmsnorm(const int32_t* tokens, const float* embed, int vocabulary, const float* norm_w,
                                 float eps, float* x, __half* normed_hi, __half* normed_lo, int rows, int hidden,
                                 float* ssq, unsigned* error, cudaStream_t stream);
// rmsnorm(x[rows ? rows[i] : i]) * w as FP16 hi/lo halves into out_hi/out_lo[i] for i < count.
cudaError_t launch_rmsnorm(const float* x, const int32_t* rows, const float* norm_w, float eps, __half* out_hi,
                           __half* out_lo, int count, int hidden, cudaStream_t stream);
// Greedy token (first index of the maximum) and finiteness of each logits row.
cudaError_t launch_argmax(const float* logits, int rows, int vocabulary, int32_t* tokens, int32_t* finite,
                          cudaStream_t stream);
// COW regions {destination, source, pitch, width, rows} in float elements, applied to both pools.
struct CowRegion {
    uint64_t destination, source, pitch, width, rows;
};
// COW copies of `count` regions, both pools, all rows. kCowDirect copies source
// to destination; a two-phase step first gathers every source into `scratch`
// (kCowGather: region i's rows at scratch_offset[i], keys in the first
// scratch_elements floats, values in the next) and then scatters it
// (kCowScatter), so that every source is read before any destination is written.
enum CowMode : int { kCowDirect = 0, kCowGather = 1, kCowScatter = 2 };
// Region offsets are reference-layout element offsets ([block][layer][slot][192],
// as KVManager's tail-copy regions carry them). A pool in that layout is addressed
// directly (layers = 0); a layer-major pool ([layer][block][slot][192]) through
// layer_major_offset().
struct PoolGeometry {
    uint64_t page_elements;  // block_tokens * kKvWidth
    uint64_t layers;         // 0: the pool is in the reference layout
    uint64_t max_blocks;
};
__host__ __device__ __forceinline__ uint64_t layer_major_offset(const PoolGeometry& g, uint64_t e) {
    const uint64_t page = e / g.page_elements, within = e - page * g.page_elements;
    const uint64_t block = page / g.layers, layer = page - block * g.layers;
    return (layer * g.max_blocks + block) * g.page_elements + within;
}
cudaError_t launch_cow_copy(const CowRegion* regions, int count, int max_rows, float* keys, float* values,
                            uint64_t pool_elements, const PoolGeometry& geometry, unsigned* error,
                            cudaStream_t stream, CowMode mode = kCowDirect, const uint64_t* scratch_offset = nullptr,
                            float* scratch = nullptr, uint64_t scratch_elements = 0);
// tables[index[i]] = value[i]
cudaError_t launch_table_patch(const int32_t* pairs, int count, int32_t* tables, int64_t table_elements,
                               unsigned* error, cudaStream_t stream);

}  // namespace mpb
