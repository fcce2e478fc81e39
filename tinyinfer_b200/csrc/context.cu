// C ABI of the device layer (include/miniprefix_b200.h): context, weights, pools,
// block tables, COW, the batched forward and the paged-attention operator.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "kernels.h"
#include "miniprefix_b200.h"

namespace {

thread_local std::string g_error;

struct Failure {
    int code;
    std::string message;
};

void fail(int code, const std::string& message) { throw Failure{code, message}; }

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(e == cudaErrorMemoryAllocation ? MP_ERR_NOMEM : MP_ERR_CUDA,
                               std::string(what) + ": " + cudaGetErrorString(e));
}

template <class F>
int guarded(F&& body) {
    try {
        body();
        return MP_OK;
    } catch (const Failure& f) {
        g_error = f.message;
        return f.code;
    } catch (const std::bad_alloc&) {
        g_error = "host allocation failed";
        return MP_ERR_NOMEM;
    } catch (const std::exception& e) {
        g_error = e.what();
        return MP_ERR_INVALID;
    }
}

template <class T>
T* device_alloc(size_t count, const char* what) {
    void* p = nullptr;
    if (count == 0) count = 1;
    cuda_check(cudaMalloc(&p, count * sizeof(T)), what);
    return static_cast<T*>(p);
}

template <class T>
T* host_alloc(size_t count, const char* what) {
    void* p = nullptr;
    if (count == 0) count = 1;
    cuda_check(cudaMallocHost(&p, count * sizeof(T)), what);
    return static_cast<T*>(p);
}

// Work decomposition of paged attention.
//  * Decode rows (sequences appending fewer than kPrefillMinRows rows): with
//    pages_per_split 0 the rows' pages, concatenated, are cut into one equal run
//    per CTA of the decode kernel's single wave (mpb::plan_static_runs); else each
//    row's pages are cut into slices of `pages_per_split` pages, pulled longest
//    first.
//  * Shared prefixes (only when enabled with mp_set_shared_prefix): decode rows
//    whose block tables begin with the same physical pages (prefix reuse, forks)
//    form a group when at least `group_min_rows` rows share at least
//    `group_min_tokens` tokens of full pages. The group's shared tokens become
//    prefix work (attention_shared.cu, one CTA per kv head x 128 query vectors x
//    chunk) and each row's slices start after them. A page that holds a row's
//    newest token is never shared (it was just written), so only pages before it
//    count. Off by default: every row reading the shared pages itself, which
//    then stay in L2, measured faster on B200.
//  * Prefill sequences: one work item per (64-row tile, kv head).
struct AttnPlan {
    std::vector<int32_t> splits, work0, x0, nx;
    std::vector<mpb::AttnWork> work;
    std::vector<int32_t> order;  // decode work items, longest first (persistent schedule)
    std::vector<int32_t> cta_items;  // static schedule: CTA c runs items [cta_items[c], cta_items[c + 1])
    std::vector<mpb::PrefillWork> prefill;
    std::vector<mpb::PrefixWork> prefix;
    std::vector<int32_t> group_rows, group_row0, group_slot;
    int extra_slots = 0;
    double bytes = 0;          // algorithmic bytes of one layer's attention (shared tokens once per group)
    double logical_bytes = 0;  // the same with every row reading its whole context
};

constexpr int kGroupMinTokensFloor = 16;  // smallest shared span worth a group
constexpr int kPrefixMaxChunks = 64;
constexpr double kPrefixTargetCtas = 148.0;  // one wave (one CTA per SM)

// tables: host mirror of the device block tables ([slots][table_stride]).
// group_min_rows 0: no shared-prefix groups.
void plan_attention(const mp_sequence_desc* seqs, int count, int block_tokens, int table_stride,
                    const std::vector<int32_t>& tables, int pages_per_split, size_t extra_capacity,
                    size_t prefix_capacity, int group_min_rows, int group_min_tokens, AttnPlan& plan) {
    group_min_tokens = std::max(group_min_tokens, kGroupMinTokensFloor);
    int rows = 0;
    for (int i = 0; i < count; ++i) rows += seqs[i].count;
    plan.splits.assign(rows, 0);
    plan.work0.assign(rows, 0);
    plan.x0.assign(rows, 0);
    plan.nx.assign(rows, 0);
    plan.work.clear();
    plan.prefill.clear();
    plan.prefix.clear();
    plan.group_rows.clear();
    plan.group_row0.assign(1, 0);
    plan.group_slot.clear();
    plan.extra_slots = 0;
    plan.bytes = 0;
    plan.logical_bytes = 0;
    const double kv_token_bytes = 2.0 * mpb::kKvWidth * sizeof(float);

    // decode rows: (row, slot, len)
    struct DecodeRow {
        int row, slot, len;
    };
    std::vector<DecodeRow> decode;
    {
        int row = 0;
        for (int i = 0; i < count; ++i) {
            const auto& s = seqs[i];
            if (s.count < mpb::kPrefillMinRows)
                for (int j = 0; j < s.count; ++j) decode.push_back({row + j, s.slot, s.start + j + 1});
            row += s.count;
        }
    }
    // shared-prefix groups: bucket rows by their first page, then the longest
    // common run of page ids within the bucket
    std::vector<int> shared_pages(rows, 0);
    {
        std::vector<std::pair<int32_t, int>> keyed;  // (first page, index into decode)
        for (int i = 0; i < int(decode.size()); ++i) {
            const int full = (decode[i].len - 1) / block_tokens;
            if (group_min_rows > 0 && full * block_tokens >= group_min_tokens)
                keyed.push_back({tables[size_t(decode[i].slot) * table_stride], i});
        }
        std::stable_sort(keyed.begin(), keyed.end(),
                         [](const auto& a, const auto& b) { return a.first < b.first; });
        // candidates: (first, last) index into keyed, shared full pages
        struct Candidate {
            size_t b, e;
            int pages;
        };
        std::vector<Candidate> candidates;
        for (size_t b = 0; b < keyed.size();) {
            size_t e = b;
            while (e < keyed.size() && keyed[e].first == keyed[b].first) ++e;
            if (int(e - b) >= group_min_rows && keyed[b].first >= 0) {
                const DecodeRow& ref = decode[keyed[b].second];
                const int32_t* rt = tables.data() + size_t(ref.slot) * table_stride;
                int lcp = (ref.len - 1) / block_tokens;
                for (size_t k = b + 1; k < e && lcp > 0; ++k) {
                    const DecodeRow& d = decode[keyed[k].second];
                    lcp = std::min(lcp, (d.len - 1) / block_tokens);
                    const int32_t* t = tables.data() + size_t(d.slot) * table_stride;
                    for (int i = 1; i < lcp; ++i)
                        if (t[i] != rt[i]) {
                            lcp = i;
                            break;
                        }
                }
                if (lcp * block_tokens >= group_min_tokens) candidates.push_back({b, e, lcp});
            }
            b = e;
        }
        // One chunk length for the step: the groups' (tokens x query blocks x kv
        // heads) spread over about kPrefixTargetCtas CTAs, in whole sub-chunks.
        double work = 0;
        for (const auto& g : candidates) {
            const int qblocks = (int(g.e - g.b) * mpb::kGroup + mpb::kPrefixQueries - 1) / mpb::kPrefixQueries;
            work += double(g.pages) * block_tokens * qblocks * mpb::kKvHeads;
        }
        const int sub = mpb::kPrefixSubChunk;
        const int step_chunk = std::max(sub, int(std::ceil(work / kPrefixTargetCtas / sub)) * sub);
        for (const auto& g : candidates) {
            const int n = int(g.e - g.b);
            const DecodeRow& ref = decode[keyed[g.b].second];
            const int shared = g.pages * block_tokens;
            int chunk_tokens = std::max(step_chunk, (shared + kPrefixMaxChunks - 1) / kPrefixMaxChunks);
            chunk_tokens = (chunk_tokens + sub - 1) / sub * sub;
            const int chunks = (shared + chunk_tokens - 1) / chunk_tokens;
            const int qvecs = n * mpb::kGroup;
            const int qblocks = (qvecs + mpb::kPrefixQueries - 1) / mpb::kPrefixQueries;
            const size_t works = size_t(mpb::kKvHeads) * qblocks * chunks;
            if (size_t(plan.extra_slots) + size_t(n) * chunks > extra_capacity ||
                plan.prefix.size() + works > prefix_capacity)
                continue;
            const int gi = int(plan.group_slot.size());
            plan.group_slot.push_back(ref.slot);
            for (size_t k = g.b; k < g.e; ++k) {
                const DecodeRow& d = decode[keyed[k].second];
                plan.group_rows.push_back(d.row);
                shared_pages[d.row] = g.pages;
                plan.nx[d.row] = chunks;
                plan.x0[d.row] = plan.extra_slots;  // made absolute below
                plan.extra_slots += chunks;
            }
            plan.group_row0.push_back(int(plan.group_rows.size()));
            for (int kh = 0; kh < mpb::kKvHeads; ++kh)
                for (int ch = 0; ch < chunks; ++ch)
                    for (int qb = 0; qb < qblocks; ++qb) {
                        const int q0 = qb * mpb::kPrefixQueries;
                        plan.prefix.push_back({gi, kh, q0, std::min(mpb::kPrefixQueries, qvecs - q0),
                                               ch * chunk_tokens, std::min(shared, (ch + 1) * chunk_tokens), ch, 0});
                    }
            plan.bytes += double(shared) * kv_token_bytes;
        }
    }
    long long decode_tokens = 0;
    for (const auto& d : decode) decode_tokens += d.len - shared_pages[d.row] * block_tokens;
    const int pps = pages_per_split > 0 ? pages_per_split : mpb::auto_pages_per_split(decode_tokens, block_tokens);
    const bool runs = pages_per_split <= 0;
    struct OwnPages {
        int row, first, pages;
    };
    std::vector<OwnPages> own;  // decode rows of a static schedule, in row order
    plan.cta_items.clear();
    int row = 0;
    for (int i = 0; i < count; ++i) {
        const auto& s = seqs[i];
        if (s.count >= mpb::kPrefillMinRows) {
            for (int t = 0; t * mpb::kPrefillTileRows < s.count; ++t) {
                const int rows_in = std::min(mpb::kPrefillTileRows, s.count - t * mpb::kPrefillTileRows);
                for (int kh = 0; kh < mpb::kKvHeads; ++kh)
                    plan.prefill.push_back({row + t * mpb::kPrefillTileRows, rows_in,
                                            s.start + t * mpb::kPrefillTileRows, s.slot, kh, {0, 0, 0}});
            }
            // The context of the whole chunk is read once per row tile.
            const int tiles = (s.count + mpb::kPrefillTileRows - 1) / mpb::kPrefillTileRows;
            double b = 0;
            for (int t = 0; t < tiles; ++t) {
                const int last = s.start + std::min(s.count, (t + 1) * mpb::kPrefillTileRows);
                b += double(last) * kv_token_bytes;
            }
            b += double(s.count) * 2.0 * mpb::kQWidth * sizeof(float);
            plan.bytes += b;
            plan.logical_bytes += b;
            row += s.count;
            continue;
        }
        for (int j = 0; j < s.count; ++j, ++row) {
            const int len = s.start + j + 1;
            const int pages = (len + block_tokens - 1) / block_tokens;
            const int first = shared_pages[row];
            if (runs) {
                own.push_back({row, first, pages});
            } else {
                const int n = std::max(1, (pages - first + pps - 1) / pps);
                plan.splits[row] = n;
                plan.work0[row] = int(plan.work.size());
                for (int k = 0; k < n; ++k)
                    plan.work.push_back({row, first + k * pps, std::min(pages, first + (k + 1) * pps), k});
            }
            // K and V rows, the query row and output row, the table entries.
            const double own = 2.0 * mpb::kQWidth * sizeof(float) + double(pages) * sizeof(int32_t);
            plan.bytes += double(len - first * block_tokens) * kv_token_bytes + own;
            plan.logical_bytes += double(len) * kv_token_bytes + own;
        }
    }
    if (runs && !own.empty()) {
        plan.cta_items.push_back(0);
        mpb::plan_static_runs(
            int(own.size()), [&](int i) { return own[i].pages - own[i].first; },
            [&](int i, int b, int e, int k) {
                const int row = own[i].row;
                if (k == 0) plan.work0[row] = int(plan.work.size());
                plan.splits[row] = k + 1;
                plan.work.push_back({row, own[i].first + b, own[i].first + e, k});
            },
            [&](int, int items) { plan.cta_items.push_back(items); });
    }
    // prefill tiles with the longest context first: the CTAs with the most work
    // start in the first wave
    std::stable_sort(plan.prefill.begin(), plan.prefill.end(), [](const mpb::PrefillWork& a, const mpb::PrefillWork& b) {
        return a.position + a.rows > b.position + b.rows;
    });
    // shared-prefix slots follow the decode work items in the partial array
    for (int r = 0; r < rows; ++r)
        if (plan.nx[r]) plan.x0[r] += int(plan.work.size());
    // longest slices first: the persistent decode CTAs then finish together
    std::vector<int32_t> tokens(plan.work.size());
    {
        std::vector<int32_t> row_len(rows, 0);
        int r = 0;
        for (int i = 0; i < count; ++i)
            for (int j = 0; j < seqs[i].count; ++j, ++r) row_len[r] = seqs[i].start + j + 1;
        for (size_t w = 0; w < plan.work.size(); ++w) {
            const auto& it = plan.work[w];
            tokens[w] = std::min(it.page_end * block_tokens, row_len[it.row]) - it.page_begin * block_tokens;
        }
    }
    plan.order.resize(plan.work.size());
    for (size_t w = 0; w < plan.order.size(); ++w) plan.order[w] = int32_t(w);
    if (!plan.cta_items.empty()) return;  // static schedule: no pull order
    std::stable_sort(plan.order.begin(), plan.order.end(),
                     [&](int32_t a, int32_t b) { return tokens[a] > tokens[b]; });
}

}  // namespace

namespace mpb {
void set_last_error(const char* message) { g_error = message; }
}  // namespace mpb

struct mp_context {
    int device = 0;
    mp_model_config model{};
    mp_runtime_config rt{};
    int dim = 64, kvw = 192, qkvw = 960;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr, idle = nullptr, mark[2] = {nullptr, nullptr};
    int mark_count = 0;
    // weights: the embedding in FP32 (row gather), every GEMM operand packed [N][K]
    // (K contiguous) as FP16 hi/lo halves (split_f16); per-layer matrices stacked by layer
    float *embed = nullptr, *final_norm = nullptr, *in_norm = nullptr, *post_norm = nullptr;
    struct Split {
        __half* hi = nullptr;
        __half* lo = nullptr;
    };
    // gate and up are fused: rows 64b..64b+31 of wgu hold gate rows 32b..32b+31 and
    // rows 64b+32..64b+63 the matching up rows, so a 64-row GEMM tile carries both
    // halves of 32 SwiGLU outputs.
    Split wqkv, wo, wgu, wdown, head;
    std::set<std::string> received;
    bool finalized = false;
    // pools and tables. Each pool is layer-major, [layer][block][slot][192]: the pages
    // one layer's attention reads share a compact address range (a [block][layer]
    // pool spreads them at a stride of `layers` pages, which measured ~10% slower
    // streaming). The API speaks reference-layout offsets ([block][layer][slot][192]:
    // COW regions, mp_kv_read / mp_kv_write), translated by layer_major_offset().
    float *keys = nullptr, *values = nullptr;
    uint64_t pool_elements = 0;
    int32_t* tables = nullptr;
    // host mirror of the device block tables (shared-prefix grouping reads it)
    std::vector<int32_t> h_tables;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    // workspace (GEMM inputs as hi/lo halves)
    float *x = nullptr, *q = nullptr, *logits = nullptr, *partial = nullptr;
    float* ssq = nullptr;  // [rows][hidden / 64] sums of squares of x (folded RMSNorm)
    Split xn, attn, h, xl;
    // TMA tensor maps of every GEMM operand
    struct alignas(64) Maps {
        CUtensorMap xn_hi, xn_lo, attn_hi, attn_lo, h_hi, h_lo, xl_hi, xl_lo;
        CUtensorMap wqkv_hi, wqkv_lo, wo_hi, wo_lo, wgu_hi, wgu_lo, wdown_hi, wdown_lo, head_hi, head_lo;
    };
    Maps maps;
    unsigned *counters = nullptr, *error = nullptr, *attn_sched = nullptr;
    int32_t *meta = nullptr, *out_tokens = nullptr, *out_finite = nullptr, *cow = nullptr, *patch = nullptr;
    size_t meta_capacity = 0, work_capacity = 0;
    // pinned host staging
    int32_t* h_meta = nullptr;
    int32_t *h_tokens = nullptr, *h_finite = nullptr;
    unsigned* h_error = nullptr;
    int32_t* h_patch = nullptr;
    size_t patch_capacity = 0;
    uint64_t* h_cow = nullptr;
    size_t cow_capacity = 0;
    // two-phase COW: sources gathered here (keys, then values) before any
    // destination is written, when a destination overlaps a source of the step
    float* cow_scratch = nullptr;
    size_t cow_scratch_capacity = 0;  // floats per pool
    uint64_t cow_scratch_elements = 0;
    bool cow_two_phase = false;
    // current step
    int rows = 0, seqs = 0, work_count = 0, prefill_count = 0, prefix_count = 0, entry_count = 0, region_count = 0,
        region_rows = 0;
    size_t extra_capacity = 0, prefix_capacity = 0;
    uint64_t step_prefix_rows = 0, step_prefix_tokens = 0;
    size_t off_entries = 0, off_regions = 0, off_scratch = 0, entry_capacity = 0, region_capacity = 0;
    bool cow_timing = false, cow_timed = false;
    cudaEvent_t cow_events[2] = {nullptr, nullptr};
    cudaEvent_t fwd_events[2] = {nullptr, nullptr};
    mp_counters counters_total{};
    uint64_t step_launches = 0, step_h2d = 0, step_d2h = 0;
    float cow_ms = 0.f;
    size_t off_tokens = 0, off_pos = 0, off_slot = 0, off_len = 0, off_splits = 0, off_work0 = 0, off_last = 0,
           off_work = 0, off_prefill = 0, off_x0 = 0, off_nx = 0, off_group_rows = 0, off_group_row0 = 0,
           off_group_slot = 0, off_prefix = 0, off_order = 0, off_cta = 0;
    int cta_count = 0;  // static decode-attention schedule of the step (0: none)
    size_t prefill_capacity = 0;
    bool prepared = false;
    // host waits of staging reuse and pool copies (bounded, MP_ERR_TIMEOUT)
    int host_wait_ms = 600000;
    // failure-path tests (mp_inject_wait_timeout): the next forward's first GEMM
    // issues no copies and bounds its waits at this many microseconds
    int stall_next_us = 0;
    AttnPlan plan;
    // attention profiling
    bool profile = false;
    int group_min_rows = 0, group_min_tokens = 128;  // shared-prefix path (mp_set_shared_prefix)
    std::vector<cudaEvent_t> prof_events;
    int prof_used = 0;
    float prof_ms = 0.f;
    int prof_launches = 0;
    double prof_bytes = 0;
    // projection GEMMs: the interval from one layer's attention end to the next
    // layer's attention start is that layer's O, gate/up and down GEMMs plus the
    // next layer's QKV GEMM; the LM head is bracketed by its own pair of events
    float prof_gemm_ms = 0.f, prof_head_ms = 0.f;
    int prof_gemm_intervals = 0, prof_heads = 0;
    cudaEvent_t head_events[2] = {nullptr, nullptr};
};

namespace {

size_t max_work(const mp_runtime_config& rt) { return size_t(rt.max_step_tokens) + 2048; }

// Tile width (B rows per CTA tile) of the fused gate/up projection: 64 (more tiles,
// three stages, usually no K split at decode sizes) or 128 (half the activation
// re-reads, two stages, split K).
#ifndef MPB_GATE_UP_BN
#define MPB_GATE_UP_BN 64
#endif
constexpr int kGateUpBN = MPB_GATE_UP_BN;  // 2 x intermediate is a multiple of 128 (intermediate % 64 == 0)
int head_tile_n(int vocabulary) { return vocabulary % 256 == 0 ? 256 : (vocabulary % 128 == 0 ? 128 : 64); }
int gemm_tile_n(int n) {
    if (n >= 8192) return head_tile_n(n);
    if (n % kGateUpBN == 0 && n >= 2048) return kGateUpBN;
    return mpb::kTcBN;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q{};
        void* p = nullptr;
        cuda_check(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q),
                   "locate cuTensorMapEncodeTiled");
        if (q != cudaDriverEntryPointSuccess || !p) fail(MP_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D fp16 map over a row-major [rows][cols] buffer (cols a multiple of 8), boxes of
// 64 columns (one 128-byte swizzled row) x box_rows rows; columns past `cols` read
// as zeros.
void encode_map(CUtensorMap* map, const __half* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * sizeof(__half)};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims,
                                            strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(MP_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
}

// FP16 hi/lo halves on the host, the rule of the device split_f16: hi = x rounded
// to FP16, lo = (x - hi) * 2^11 rounded to FP16.
void split_host(const float* x, __half* hi, __half* lo, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        hi[i] = __float2half_rn(x[i]);
        lo[i] = __float2half_rn((x[i] - __half2float(hi[i])) * mpb::kSplitLoScale);
    }
}

void free_context(mp_context* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    // queued work must end before its buffers are freed: poll, bounded by the
    // context's host wait limit (after that the buffers are freed regardless)
    if (c->stream) {
        const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(c->host_wait_ms);
        while (cudaStreamQuery(c->stream) == cudaErrorNotReady && std::chrono::steady_clock::now() < deadline)
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    for (void* p : {(void*)c->embed, (void*)c->final_norm, (void*)c->in_norm, (void*)c->post_norm, (void*)c->keys,
                    (void*)c->values, (void*)c->tables, (void*)c->rope_cos, (void*)c->rope_sin, (void*)c->x,
                    (void*)c->q, (void*)c->logits, (void*)c->ssq,
                    (void*)c->partial,
                    (void*)c->counters, (void*)c->attn_sched, (void*)c->error, (void*)c->meta, (void*)c->out_tokens, (void*)c->out_finite,
                    (void*)c->cow, (void*)c->patch, (void*)c->cow_scratch})
        if (p) cudaFree(p);
    for (auto* s : {&c->wqkv, &c->wo, &c->wgu, &c->wdown, &c->head, &c->xn, &c->attn, &c->h, &c->xl}) {
        if (s->hi) cudaFree(s->hi);
        if (s->lo) cudaFree(s->lo);
    }
    for (void* p : {(void*)c->h_meta, (void*)c->h_tokens, (void*)c->h_finite, (void*)c->h_error, (void*)c->h_patch,
                    (void*)c->h_cow})
        if (p) cudaFreeHost(p);
    for (auto e : c->prof_events) cudaEventDestroy(e);
    for (auto e : c->head_events)
        if (e) cudaEventDestroy(e);
    for (auto e : c->cow_events)
        if (e) cudaEventDestroy(e);
    for (auto e : c->fwd_events)
        if (e) cudaEventDestroy(e);
    if (c->done) cudaEventDestroy(c->done);
    if (c->idle) cudaEventDestroy(c->idle);
    for (auto e : c->mark)
        if (e) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

// Adds the wall time of its scope to `sink` (milliseconds).
struct HostTimer {
    double& sink;
    std::chrono::steady_clock::time_point start = std::chrono::steady_clock::now();
    explicit HostTimer(double& s) : sink(s) {}
    ~HostTimer() {
        sink += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - start).count();
    }
};

// Polls `e` until it completes or `timeout_ms` elapses. For the first 50 ms the
// thread only yields between polls, so a forward's completion (a few ms) is seen
// within microseconds; a sleep would stretch each poll to the kernel's timer
// slack (tens of microseconds). Longer waits sleep 100 us between polls.
void wait_event(cudaEvent_t e, int timeout_ms) {
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t s = cudaEventQuery(e);
        if (s == cudaSuccess) return;
        if (s != cudaErrorNotReady) cuda_check(s, "step completion");
        const auto waited = std::chrono::steady_clock::now() - start;
        if (timeout_ms >= 0 && waited > std::chrono::milliseconds(timeout_ms))
            fail(MP_ERR_TIMEOUT, "device work did not complete within the timeout");
        if (waited < std::chrono::milliseconds(50)) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// Bounded wait until everything queued on the context's stream has completed
// (staging buffers about to be refilled, pool copies ordered after the forward).
void wait_stream(mp_context* c, const char* what) {
    cuda_check(cudaEventRecord(c->idle, c->stream), what);
    wait_event(c->idle, c->host_wait_ms);
}

// The layer-major pools as seen from reference-layout offsets.
mpb::PoolGeometry pool_geometry(const mp_context* c) {
    return {uint64_t(c->rt.block_tokens) * uint64_t(c->kvw), uint64_t(c->model.layers), uint64_t(c->rt.max_blocks)};
}

void validate_geometry(const mp_model_config& m, const mp_runtime_config& r) {
    const bool valid = m.layers >= 1 && m.layers <= 128 && m.hidden >= 2 && m.hidden <= 8192 && m.intermediate >= 1 &&
                       m.intermediate <= 65536 && m.heads >= 1 && m.kv_heads >= 1 && m.hidden % m.heads == 0 &&
                       m.heads % m.kv_heads == 0 && (m.hidden / m.heads) % 2 == 0 && m.hidden / m.heads <= 256 &&
                       m.vocabulary >= 2 && m.vocabulary <= 262144 && m.context >= 1 && m.context <= 131072 &&
                       m.eos >= 0 && m.eos < m.vocabulary && std::isfinite(m.rms_epsilon) && m.rms_epsilon > 0 &&
                       std::isfinite(m.rope_theta) && m.rope_theta > 1;
    if (!valid) fail(MP_ERR_INVALID, "unsupported/invalid Llama configuration");
    if (m.heads != mpb::kHeads || m.kv_heads != mpb::kKvHeads || m.hidden != mpb::kQWidth)
        fail(MP_ERR_UNSUPPORTED, "kernels are specialised for 9 query heads, 3 kv heads, head_dim 64");
    if (m.intermediate % 64 || m.vocabulary % 64)
        fail(MP_ERR_UNSUPPORTED, "intermediate and vocabulary must be multiples of 64");
    if (r.block_tokens < 1 || r.max_blocks < 1 || r.max_sequences < 1 || r.max_step_tokens < 1 ||
        r.max_step_sequences < 1 || r.max_step_sequences > r.max_step_tokens || r.table_stride < 1 ||
        int64_t(r.table_stride) * r.block_tokens < m.context)
        fail(MP_ERR_INVALID, "invalid runtime configuration");
}

struct WeightSlot {
    float* base;     // fp32 destination (embedding, norms) or nullptr
    __half* hi;      // FP16 halves destination of a GEMM operand slice, or nullptr
    __half* lo;
    int rows_n;      // N of the packed [N][K] matrix slice
    int k;           // K
    bool transpose;  // MPFX [K][N] -> packed [N][K]
    size_t elements;
    int interleave;  // 0: packed row n at n; 1/2: gate/up row n at 64*(n/32) + 32*(interleave-1) + n%32
};

// Resolve an MPFX0001 tensor name to its packed destination.
WeightSlot resolve(mp_context* c, const std::string& name) {
    const auto& m = c->model;
    const int H = m.hidden, I = m.intermediate, kvw = c->kvw, V = m.vocabulary;
    if (name == "model.embed_tokens.weight")
        return {c->embed, m.tied ? c->head.hi : nullptr, m.tied ? c->head.lo : nullptr, V, H, false, size_t(V) * H, 0};
    if (name == "model.norm.weight") return {c->final_norm, nullptr, nullptr, 1, H, false, size_t(H), 0};
    if (name == "lm_head.weight") {
        if (m.tied) fail(MP_ERR_INVALID, "tied model has no lm_head.weight");
        return {nullptr, c->head.hi, c->head.lo, V, H, true, size_t(V) * H, 0};
    }
    const std::string prefix = "model.layers.";
    if (name.compare(0, prefix.size(), prefix) != 0) fail(MP_ERR_INVALID, "unknown tensor: " + name);
    size_t dot = name.find('.', prefix.size());
    if (dot == std::string::npos) fail(MP_ERR_INVALID, "unknown tensor: " + name);
    int layer = -1;
    try {
        layer = std::stoi(name.substr(prefix.size(), dot - prefix.size()));
    } catch (...) {
        fail(MP_ERR_INVALID, "unknown tensor: " + name);
    }
    if (layer < 0 || layer >= m.layers) fail(MP_ERR_INVALID, "unknown tensor: " + name);
    const std::string s = name.substr(dot + 1);
    const size_t L = size_t(layer);
    if (s == "input_layernorm.weight") return {c->in_norm + L * H, nullptr, nullptr, 1, H, false, size_t(H), 0};
    if (s == "post_attention_layernorm.weight")
        return {c->post_norm + L * H, nullptr, nullptr, 1, H, false, size_t(H), 0};
    auto slice = [](const mp_context::Split& s, size_t offset) {
        return std::pair<__half*, __half*>(s.hi + offset, s.lo + offset);
    };
    const size_t qkv = L * size_t(c->qkvw) * H;
    if (s == "self_attn.q_proj.weight") {
        auto p = slice(c->wqkv, qkv);
        return {nullptr, p.first, p.second, H, H, true, size_t(H) * H, 0};
    }
    if (s == "self_attn.k_proj.weight") {
        auto p = slice(c->wqkv, qkv + size_t(H) * H);
        return {nullptr, p.first, p.second, kvw, H, true, size_t(H) * kvw, 0};
    }
    if (s == "self_attn.v_proj.weight") {
        auto p = slice(c->wqkv, qkv + size_t(H + kvw) * H);
        return {nullptr, p.first, p.second, kvw, H, true, size_t(H) * kvw, 0};
    }
    if (s == "self_attn.o_proj.weight") {
        auto p = slice(c->wo, L * size_t(H) * H);
        return {nullptr, p.first, p.second, H, H, true, size_t(H) * H, 0};
    }
    if (s == "mlp.gate_proj.weight") {
        auto p = slice(c->wgu, L * size_t(2 * I) * H);
        return {nullptr, p.first, p.second, I, H, true, size_t(H) * I, 1};
    }
    if (s == "mlp.up_proj.weight") {
        auto p = slice(c->wgu, L * size_t(2 * I) * H);
        return {nullptr, p.first, p.second, I, H, true, size_t(H) * I, 2};
    }
    if (s == "mlp.down_proj.weight") {
        auto p = slice(c->wdown, L * size_t(H) * I);
        return {nullptr, p.first, p.second, H, I, true, size_t(I) * H, 0};
    }
    fail(MP_ERR_INVALID, "unknown tensor: " + name);
    return {nullptr, nullptr, nullptr, 0, 0, false, 0, 0};
}

size_t expected_tensors(const mp_model_config& m) { return size_t(m.layers) * 9 + 2 + (m.tied ? 0 : 1); }

void ensure_patch(mp_context* c, size_t pairs) {
    if (pairs <= c->patch_capacity) return;
    wait_stream(c, "patch staging reuse");
    if (c->h_patch) cudaFreeHost(c->h_patch);
    if (c->patch) cudaFree(c->patch);
    c->h_patch = nullptr;
    c->patch = nullptr;
    c->patch_capacity = 0;
    c->h_patch = host_alloc<int32_t>(2 * pairs, "table patch staging");
    c->patch = device_alloc<int32_t>(2 * pairs, "table patch buffer");
    c->patch_capacity = pairs;
}

void record_attention_event(mp_context* c) {
    if (size_t(c->prof_used) == c->prof_events.size()) {
        cudaEvent_t e;
        cuda_check(cudaEventCreate(&e), "profile event");
        c->prof_events.push_back(e);
    }
    cuda_check(cudaEventRecord(c->prof_events[c->prof_used++], c->stream), "profile event record");
}

void harvest_profile(mp_context* c) {
    for (int i = 0; i + 1 < c->prof_used; i += 2) {
        float ms = 0.f;
        cuda_check(cudaEventElapsedTime(&ms, c->prof_events[i], c->prof_events[i + 1]), "profile elapsed");
        c->prof_ms += ms;
        c->prof_launches += 1;
        if (i + 2 < c->prof_used) {
            cuda_check(cudaEventElapsedTime(&ms, c->prof_events[i + 1], c->prof_events[i + 2]), "profile elapsed");
            c->prof_gemm_ms += ms;
            c->prof_gemm_intervals += 1;
        }
    }
    c->prof_used = 0;
    if (c->head_events[0]) {
        float ms = 0.f;
        cuda_check(cudaEventElapsedTime(&ms, c->head_events[0], c->head_events[1]), "profile elapsed");
        c->prof_head_ms += ms;
        c->prof_heads += 1;
    }
}

}  // namespace

extern "C" {

const char* mp_last_error(void) { return g_error.c_str(); }

int mp_create(int device, const mp_model_config* model, const mp_runtime_config* runtime, mp_context** out) {
    if (!model || !runtime || !out) {
        g_error = "null argument";
        return MP_ERR_INVALID;
    }
    *out = nullptr;
    mp_context* c = new (std::nothrow) mp_context;
    if (!c) return MP_ERR_NOMEM;
    const int rc = guarded([&] {
        validate_geometry(*model, *runtime);
        c->device = device;
        c->model = *model;
        c->rt = *runtime;
        const auto& m = c->model;
        const auto& r = c->rt;
        c->dim = m.hidden / m.heads;
        c->kvw = m.kv_heads * c->dim;
        c->qkvw = m.hidden + 2 * c->kvw;
        cuda_check(cudaSetDevice(device), "select device");
        cuda_check(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "create stream");
        cuda_check(cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming), "create event");
        cuda_check(cudaEventCreateWithFlags(&c->idle, cudaEventDisableTiming), "create event");
        for (auto& e : c->mark) cuda_check(cudaEventCreate(&e), "create timer event");
        cuda_check(mpb::configure_attention(), "configure attention kernel");
        cuda_check(mpb::configure_prefix_attention(), "configure shared-prefix attention kernel");
        cuda_check(mpb::configure_prefill_attention(), "configure prefill attention kernel");
        const size_t H = m.hidden, I = m.intermediate, L = m.layers, V = m.vocabulary;
        cuda_check(mpb::configure_tc_gemm(), "configure tensor-core GEMM");
        auto split = [](mp_context::Split& s, size_t n, const char* what) {
            s.hi = device_alloc<__half>(n, what);
            s.lo = device_alloc<__half>(n, what);
        };
        c->embed = device_alloc<float>(V * H, "embedding");
        c->final_norm = device_alloc<float>(H, "final norm");
        c->in_norm = device_alloc<float>(L * H, "input norms");
        c->post_norm = device_alloc<float>(L * H, "post-attention norms");
        split(c->head, V * H, "lm head");
        split(c->wqkv, L * c->qkvw * H, "qkv projections");
        split(c->wo, L * H * H, "o projections");
        split(c->wgu, L * 2 * I * H, "gate/up projections");
        split(c->wdown, L * H * I, "down projections");
        c->pool_elements = uint64_t(r.max_blocks) * L * r.block_tokens * c->kvw;
        c->keys = device_alloc<float>(c->pool_elements, "K pool");
        c->values = device_alloc<float>(c->pool_elements, "V pool");
        cuda_check(cudaMemsetAsync(c->keys, 0, c->pool_elements * sizeof(float), c->stream), "zero K pool");
        cuda_check(cudaMemsetAsync(c->values, 0, c->pool_elements * sizeof(float), c->stream), "zero V pool");
        const size_t table_elements = size_t(r.max_sequences) * r.table_stride;
        c->tables = device_alloc<int32_t>(table_elements, "block tables");
        cuda_check(cudaMemsetAsync(c->tables, 0xff, table_elements * sizeof(int32_t), c->stream), "clear tables");
        c->h_tables.assign(table_elements, -1);
        // RoPE tables, computed exactly as the CPU runner computes each angle
        // (miniprefix/src/backend/cpu/llama_runner.cpp:19-20).
        {
            const int half = c->dim / 2;
            std::vector<float> cs(size_t(m.context) * half), sn(size_t(m.context) * half);
            for (int p = 0; p < m.context; ++p)
                for (int d = 0; d < half; ++d) {
                    const float angle = float(p) / std::pow(m.rope_theta, float(2 * d) / float(c->dim));
                    cs[size_t(p) * half + d] = std::cos(angle);
                    sn[size_t(p) * half + d] = std::sin(angle);
                }
            c->rope_cos = device_alloc<float>(cs.size(), "rope cos");
            c->rope_sin = device_alloc<float>(sn.size(), "rope sin");
            cuda_check(cudaMemcpy(c->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "upload rope cos");
            cuda_check(cudaMemcpy(c->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "upload rope sin");
        }
        // Row capacities rounded up to whole 128-row GEMM tiles: every TMA box of an
        // activation operand then lies inside its allocation.
        const size_t T = (size_t(r.max_step_tokens) + 127) / 128 * 128;
        const size_t S = (size_t(r.max_step_sequences) + 127) / 128 * 128;
        c->x = device_alloc<float>(T * H, "residual stream");
        split(c->xn, T * H, "normed activations");
        c->ssq = device_alloc<float>(T * (H / mpb::kSsqGroup), "row sums of squares");
        c->q = device_alloc<float>(T * H, "roped queries");
        split(c->attn, T * H, "attention output");
        split(c->h, T * I, "mlp activations");
        split(c->xl, S * H, "last-row activations");
        c->logits = device_alloc<float>(S * V, "logits");
        // TMA maps: activations in 128-row boxes (the A tile), weights in boxes of their
        // GEMM's tile width (64; 128 gate/up; up to 256 LM head).
        auto& mp = c->maps;
        encode_map(&mp.xn_hi, c->xn.hi, T, H, 128);
        encode_map(&mp.xn_lo, c->xn.lo, T, H, 128);
        encode_map(&mp.attn_hi, c->attn.hi, T, H, 128);
        encode_map(&mp.attn_lo, c->attn.lo, T, H, 128);
        encode_map(&mp.h_hi, c->h.hi, T, I, 128);
        encode_map(&mp.h_lo, c->h.lo, T, I, 128);
        encode_map(&mp.xl_hi, c->xl.hi, S, H, 128);
        encode_map(&mp.xl_lo, c->xl.lo, S, H, 128);
        const uint32_t bn = mpb::kTcBN;
        encode_map(&mp.wqkv_hi, c->wqkv.hi, L * c->qkvw, H, bn);
        encode_map(&mp.wqkv_lo, c->wqkv.lo, L * c->qkvw, H, bn);
        encode_map(&mp.wo_hi, c->wo.hi, L * H, H, bn);
        encode_map(&mp.wo_lo, c->wo.lo, L * H, H, bn);
        encode_map(&mp.wgu_hi, c->wgu.hi, L * 2 * I, H, kGateUpBN);
        encode_map(&mp.wgu_lo, c->wgu.lo, L * 2 * I, H, kGateUpBN);
        encode_map(&mp.wdown_hi, c->wdown.hi, L * H, I, bn);
        encode_map(&mp.wdown_lo, c->wdown.lo, L * H, I, bn);
        encode_map(&mp.head_hi, c->head.hi, V, H, uint32_t(head_tile_n(int(V))));
        encode_map(&mp.head_lo, c->head.lo, V, H, uint32_t(head_tile_n(int(V))));
        c->work_capacity = max_work(r);
        // shared-prefix slots (rows x chunks) and prefix work items of one step
        c->extra_capacity = 8192;
        c->prefix_capacity = 8192;
        c->partial = device_alloc<float>((c->work_capacity + c->extra_capacity) * mpb::kHeads * (mpb::kHeadDim + 2),
                                         "attention partials");
        // one arrival counter per (row, kv head)
        c->counters = device_alloc<unsigned>(T * mpb::kKvHeads, "attention counters");
        cuda_check(cudaMemsetAsync(c->counters, 0, T * mpb::kKvHeads * sizeof(unsigned), c->stream), "zero counters");
        c->attn_sched = device_alloc<unsigned>(2, "attention schedule");
        cuda_check(cudaMemsetAsync(c->attn_sched, 0, 2 * sizeof(unsigned), c->stream), "zero schedule");
        c->error = device_alloc<unsigned>(1, "error word");
        cuda_check(cudaMemsetAsync(c->error, 0, sizeof(unsigned), c->stream), "zero error word");
        c->prefill_capacity = (T / mpb::kPrefillTileRows + S) * mpb::kKvHeads;
        c->entry_capacity = S * size_t(r.table_stride);
        c->region_capacity = S;
        c->meta_capacity = 6 * T + S + 4 * c->work_capacity + 8 * c->prefill_capacity + 2 * c->entry_capacity +
                           12 * c->region_capacity + 2 + 4 * T + 2 + 8 * c->prefix_capacity + c->work_capacity +
                           mpb::kAttnPersistentCtas + 1;
        for (auto& e : c->cow_events) cuda_check(cudaEventCreate(&e), "create cow timing event");
        for (auto& e : c->fwd_events) cuda_check(cudaEventCreate(&e), "create forward timing event");
        c->meta = device_alloc<int32_t>(c->meta_capacity, "step metadata");
        c->h_meta = host_alloc<int32_t>(c->meta_capacity, "step metadata staging");
        c->out_tokens = device_alloc<int32_t>(S, "greedy tokens");
        c->out_finite = device_alloc<int32_t>(S, "finite flags");
        c->h_tokens = host_alloc<int32_t>(S, "token staging");
        c->h_finite = host_alloc<int32_t>(S, "finite staging");
        c->h_error = host_alloc<unsigned>(1, "error staging");
        wait_stream(c, "context initialisation");
    });
    if (rc != MP_OK) {
        free_context(c);
        return rc;
    }
    *out = c;
    return MP_OK;
}

void mp_destroy(mp_context* c) { free_context(c); }

int mp_set_weight(mp_context* c, const char* name, const float* host, size_t elements) {
    return guarded([&] {
        if (!c || !name || !host) fail(MP_ERR_INVALID, "null argument");
        cuda_check(cudaSetDevice(c->device), "select device");
        const WeightSlot slot = resolve(c, name);
        if (elements != slot.elements) fail(MP_ERR_INVALID, std::string("tensor shape mismatch: ") + name);
        if (slot.base) cuda_check(cudaMemcpy(slot.base, host, elements * 4, cudaMemcpyHostToDevice), "upload weight");
        if (slot.hi) {
            // MPFX stores [K][N] ([in][out]); the GEMM reads [N][K] as FP16 halves.
            std::vector<float> t;
            const float* packed = host;
            if (slot.transpose) {
                const int N = slot.rows_n, K = slot.k;
                t.resize(elements);
                for (int k = 0; k < K; ++k)
                    for (int n = 0; n < N; ++n) t[size_t(n) * K + k] = host[size_t(k) * N + n];
                packed = t.data();
            }
            std::vector<__half> hi(elements), lo(elements);
            split_host(packed, hi.data(), lo.data(), elements);
            if (!slot.interleave) {
                cuda_check(cudaMemcpy(slot.hi, hi.data(), elements * 2, cudaMemcpyHostToDevice), "upload weight");
                cuda_check(cudaMemcpy(slot.lo, lo.data(), elements * 2, cudaMemcpyHostToDevice), "upload weight");
            } else {
                // gate/up rows go to alternating 32-row blocks of the fused matrix
                const size_t K = size_t(slot.k), block = 32 * K;
                const size_t half = size_t(slot.interleave - 1) * block;
                for (int b = 0; b < slot.rows_n / 32; ++b) {
                    const size_t dst = size_t(b) * 2 * block + half, src = size_t(b) * block;
                    cuda_check(cudaMemcpy(slot.hi + dst, hi.data() + src, block * 2, cudaMemcpyHostToDevice),
                               "upload weight");
                    cuda_check(cudaMemcpy(slot.lo + dst, lo.data() + src, block * 2, cudaMemcpyHostToDevice),
                               "upload weight");
                }
            }
        }
        c->received.insert(name);
        c->finalized = false;
    });
}

int mp_finalize_weights(mp_context* c) {
    return guarded([&] {
        if (!c) fail(MP_ERR_INVALID, "null context");
        if (c->received.size() != expected_tensors(c->model)) fail(MP_ERR_INVALID, "model tensor count mismatch");
        c->finalized = true;
    });
}

int mp_table_write(mp_context* c, int32_t slot, int32_t first, const int32_t* blocks, int32_t count) {
    return guarded([&] {
        if (!c || (count > 0 && !blocks)) fail(MP_ERR_INVALID, "null argument");
        if (slot < 0 || slot >= c->rt.max_sequences || first < 0 || count < 0 ||
            int64_t(first) + count > c->rt.table_stride)
            fail(MP_ERR_INVALID, "block table write out of range");
        if (count == 0) return;
        for (int i = 0; i < count; ++i)
            if (blocks[i] < 0 || blocks[i] >= c->rt.max_blocks) fail(MP_ERR_INVALID, "invalid physical page id");
        cuda_check(cudaSetDevice(c->device), "select device");
        ensure_patch(c, size_t(count));
        // The staging buffer may still feed the previous patch: wait for it.
        wait_stream(c, "table staging reuse");
        for (int i = 0; i < count; ++i) {
            c->h_patch[2 * i] = slot * c->rt.table_stride + first + i;
            c->h_patch[2 * i + 1] = blocks[i];
            c->h_tables[size_t(slot) * c->rt.table_stride + first + i] = blocks[i];
        }
        cuda_check(cudaMemcpyAsync(c->patch, c->h_patch, size_t(count) * 8, cudaMemcpyHostToDevice, c->stream),
                   "upload block table entries");
        cuda_check(mpb::launch_table_patch(c->patch, count, c->tables,
                                           int64_t(c->rt.max_sequences) * c->rt.table_stride, c->error, c->stream),
                   "table patch launch");
    });
}

int mp_cow_copy(mp_context* c, const mp_tail_copy_region* regions, int32_t count) {
    return guarded([&] {
        if (!c || (count > 0 && !regions)) fail(MP_ERR_INVALID, "null argument");
        if (count <= 0) return;
        uint64_t max_rows = 0;
        for (int i = 0; i < count; ++i) {
            const auto& r = regions[i];
            if (r.width % 4 || r.destination % 4 || r.source % 4 || r.pitch % 4 || r.width > r.pitch ||
                r.destination + (r.rows ? (r.rows - 1) * r.pitch + r.width : 0) > c->pool_elements ||
                r.source + (r.rows ? (r.rows - 1) * r.pitch + r.width : 0) > c->pool_elements)
                fail(MP_ERR_INVALID, "COW region outside the pools");
            max_rows = std::max(max_rows, r.rows);
        }
        cuda_check(cudaSetDevice(c->device), "select device");
        if (size_t(count) > c->cow_capacity) {
            wait_stream(c, "cow staging reuse");
            if (c->h_cow) cudaFreeHost(c->h_cow);
            if (c->cow) cudaFree(c->cow);
            c->h_cow = nullptr;
            c->cow = nullptr;
            c->cow_capacity = 0;
            c->h_cow = host_alloc<uint64_t>(size_t(count) * 5, "cow staging");
            c->cow = device_alloc<int32_t>(size_t(count) * 10, "cow regions");
            c->cow_capacity = count;
        }
        wait_stream(c, "cow staging reuse");
        std::memcpy(c->h_cow, regions, size_t(count) * sizeof(mp_tail_copy_region));
        cuda_check(cudaMemcpyAsync(c->cow, c->h_cow, size_t(count) * sizeof(mp_tail_copy_region),
                                   cudaMemcpyHostToDevice, c->stream),
                   "upload cow regions");
        cuda_check(mpb::launch_cow_copy(reinterpret_cast<const mpb::CowRegion*>(c->cow), count, int(max_rows), c->keys,
                                        c->values, c->pool_elements, pool_geometry(c), c->error, c->stream),
                   "cow launch");
    });
}

int mp_forward_prepare(mp_context* c, const mp_sequence_desc* seqs, int32_t count, const int32_t* tokens,
                       const mp_table_entry* entries, int32_t entry_count, const mp_tail_copy_region* regions,
                       int32_t region_count) {
    return guarded([&] {
        if (!c || !seqs || !tokens || (entry_count > 0 && !entries) || (region_count > 0 && !regions))
            fail(MP_ERR_INVALID, "null argument");
        HostTimer host_time(c->counters_total.host_prepare_ms);
        if (entry_count < 0 || size_t(entry_count) > c->entry_capacity) fail(MP_ERR_INVALID, "too many table entries");
        if (region_count < 0 || size_t(region_count) > c->region_capacity) fail(MP_ERR_INVALID, "too many COW regions");
        for (int i = 0; i < entry_count; ++i) {
            const auto& e = entries[i];
            if (e.slot < 0 || e.slot >= c->rt.max_sequences || e.index < 0 || e.index >= c->rt.table_stride ||
                e.block < 0 || e.block >= c->rt.max_blocks)
                fail(MP_ERR_INVALID, "invalid block table entry");
        }
        int region_rows = 0;
        uint64_t region_elements = 0;  // rows x width summed over the regions (per pool)
        for (int i = 0; i < region_count; ++i) {
            const auto& r = regions[i];
            if (r.width % 4 || r.destination % 4 || r.source % 4 || r.pitch % 4 || r.width > r.pitch ||
                r.destination + (r.rows ? (r.rows - 1) * r.pitch + r.width : 0) > c->pool_elements ||
                r.source + (r.rows ? (r.rows - 1) * r.pitch + r.width : 0) > c->pool_elements)
                fail(MP_ERR_INVALID, "COW region outside the pools");
            region_rows = std::max(region_rows, int(r.rows));
            region_elements += r.rows * r.width;
        }
        // Regions apply as if every source were read before any destination is
        // written: a destination span that overlaps some region's source span
        // (a page freed and handed out again within the step) makes the copy
        // two-phase through the gather scratch.
        bool two_phase = false;
        if (region_count > 1) {
            auto span_end = [](const mp_tail_copy_region& r, uint64_t start) {
                return start + (r.rows ? (r.rows - 1) * r.pitch + r.width : 0);
            };
            std::vector<std::pair<uint64_t, uint64_t>> sources(static_cast<size_t>(region_count));
            for (int i = 0; i < region_count; ++i)
                sources[size_t(i)] = {regions[i].source, span_end(regions[i], regions[i].source)};
            std::sort(sources.begin(), sources.end());
            std::vector<uint64_t> reach(sources.size());  // max end over sources[0..i]
            for (size_t i = 0; i < sources.size(); ++i)
                reach[i] = std::max(sources[i].second, i ? reach[i - 1] : 0);
            for (int i = 0; i < region_count && !two_phase; ++i) {
                const uint64_t d0 = regions[i].destination, d1 = span_end(regions[i], d0);
                // sources starting before d1; overlap when one of them ends after d0
                const size_t n = size_t(std::lower_bound(sources.begin(), sources.end(), std::make_pair(d1, uint64_t(0))) -
                                        sources.begin());
                two_phase = n > 0 && reach[n - 1] > d0;
            }
        }
        if (!c->finalized) fail(MP_ERR_INVALID, "weights not finalized");
        const auto& r = c->rt;
        if (count < 1 || count > r.max_step_sequences) fail(MP_ERR_INVALID, "invalid sequence count");
        int64_t total = 0;
        for (int i = 0; i < count; ++i) {
            const auto& s = seqs[i];
            if (s.slot < 0 || s.slot >= r.max_sequences || s.start < 0 || s.count < 1 ||
                int64_t(s.start) + s.count > c->model.context ||
                int64_t(s.start) + s.count > int64_t(r.table_stride) * r.block_tokens)
                fail(MP_ERR_INVALID, "invalid sequence descriptor");
            total += s.count;
        }
        if (total > r.max_step_tokens) fail(MP_ERR_INVALID, "step exceeds max_step_tokens");
        const int T = int(total);
        for (int i = 0; i < T; ++i)
            if (tokens[i] < 0 || tokens[i] >= c->model.vocabulary) fail(MP_ERR_INVALID, "invalid token");
        // the device applies this step's table entries first; so does the mirror
        // (restored below if the step is rejected before it is queued)
        std::vector<std::pair<size_t, int32_t>> mirror_undo;
        mirror_undo.reserve(size_t(entry_count));
        for (int i = 0; i < entry_count; ++i) {
            const size_t at = size_t(entries[i].slot) * r.table_stride + entries[i].index;
            mirror_undo.push_back({at, c->h_tables[at]});
            c->h_tables[at] = entries[i].block;
        }
        struct MirrorGuard {
            std::vector<int32_t>& tables;
            std::vector<std::pair<size_t, int32_t>>& undo;
            bool keep = false;
            ~MirrorGuard() {
                if (!keep)
                    for (auto it = undo.rbegin(); it != undo.rend(); ++it) tables[it->first] = it->second;
            }
        } mirror_guard{c->h_tables, mirror_undo};
        plan_attention(seqs, count, r.block_tokens, r.table_stride, c->h_tables, 0, c->extra_capacity,
                       c->prefix_capacity, c->group_min_rows, c->group_min_tokens, c->plan);
        const size_t W = c->plan.work.size(), P = c->plan.prefill.size(), X = c->plan.prefix.size();
        const size_t G = c->plan.group_slot.size();
        if (W > c->work_capacity) fail(MP_ERR_INVALID, "attention work list exceeds capacity");
        if (P > c->prefill_capacity) fail(MP_ERR_INVALID, "prefill work list exceeds capacity");
        // layout: tokens | pos | slot | len | splits | work0 | last | work
        cuda_check(cudaSetDevice(c->device), "select device");
        wait_stream(c, "metadata staging reuse");
        int32_t* h = c->h_meta;
        c->off_tokens = 0;
        c->off_pos = c->off_tokens + T;
        c->off_slot = c->off_pos + T;
        c->off_len = c->off_slot + T;
        c->off_splits = c->off_len + T;
        c->off_work0 = c->off_splits + T;
        c->off_last = c->off_work0 + T;
        c->off_work = c->off_last + count;
        c->off_prefill = c->off_work + 4 * W;
        c->off_x0 = c->off_prefill + 8 * P;
        c->off_nx = c->off_x0 + T;
        c->off_group_rows = c->off_nx + T;
        c->off_group_row0 = c->off_group_rows + c->plan.group_rows.size();
        c->off_group_slot = c->off_group_row0 + G + 1;
        c->off_prefix = c->off_group_slot + G;
        c->off_order = c->off_prefix + 8 * X;
        c->off_cta = c->off_order + W;
        c->off_entries = c->off_cta + c->plan.cta_items.size();
        c->off_regions = (c->off_entries + 2 * size_t(entry_count) + 1) & ~size_t(1);  // 8-byte aligned
        c->off_scratch = c->off_regions + 10 * size_t(region_count);                   // uint64 per region
        std::memcpy(h + c->off_tokens, tokens, size_t(T) * 4);
        int row = 0;
        for (int i = 0; i < count; ++i) {
            for (int j = 0; j < seqs[i].count; ++j, ++row) {
                h[c->off_pos + row] = seqs[i].start + j;
                h[c->off_slot + row] = seqs[i].slot;
                h[c->off_len + row] = seqs[i].start + j + 1;
            }
            h[c->off_last + i] = row - 1;
        }
        std::memcpy(h + c->off_splits, c->plan.splits.data(), size_t(T) * 4);
        std::memcpy(h + c->off_work0, c->plan.work0.data(), size_t(T) * 4);
        std::memcpy(h + c->off_work, c->plan.work.data(), W * sizeof(mpb::AttnWork));
        std::memcpy(h + c->off_prefill, c->plan.prefill.data(), P * sizeof(mpb::PrefillWork));
        std::memcpy(h + c->off_x0, c->plan.x0.data(), size_t(T) * 4);
        std::memcpy(h + c->off_nx, c->plan.nx.data(), size_t(T) * 4);
        std::memcpy(h + c->off_group_rows, c->plan.group_rows.data(), c->plan.group_rows.size() * 4);
        std::memcpy(h + c->off_group_row0, c->plan.group_row0.data(), (G + 1) * 4);
        std::memcpy(h + c->off_group_slot, c->plan.group_slot.data(), G * 4);
        std::memcpy(h + c->off_prefix, c->plan.prefix.data(), X * sizeof(mpb::PrefixWork));
        std::memcpy(h + c->off_order, c->plan.order.data(), W * 4);
        std::memcpy(h + c->off_cta, c->plan.cta_items.data(), c->plan.cta_items.size() * 4);
        for (int i = 0; i < entry_count; ++i) {
            h[c->off_entries + 2 * i] = entries[i].slot * c->rt.table_stride + entries[i].index;
            h[c->off_entries + 2 * i + 1] = entries[i].block;
        }
        if (region_count)
            std::memcpy(h + c->off_regions, regions, size_t(region_count) * sizeof(mp_tail_copy_region));
        if (two_phase) {
            if (region_elements > c->cow_scratch_capacity) {
                if (c->cow_scratch) cudaFree(c->cow_scratch);
                c->cow_scratch = nullptr;
                c->cow_scratch_capacity = 0;
                c->cow_scratch = device_alloc<float>(2 * size_t(region_elements), "COW gather scratch");
                c->cow_scratch_capacity = region_elements;
            }
            uint64_t at = 0;
            for (int i = 0; i < region_count; ++i) {
                std::memcpy(h + c->off_scratch + 2 * size_t(i), &at, sizeof(at));
                at += regions[i].rows * regions[i].width;
            }
        }
        const size_t bytes = (c->off_scratch + (two_phase ? 2 * size_t(region_count) : 0)) * 4;
        cuda_check(cudaMemcpyAsync(c->meta, h, bytes, cudaMemcpyHostToDevice, c->stream), "upload step metadata");
        c->step_h2d = bytes;
        c->rows = T;
        c->seqs = count;
        c->work_count = int(W);
        c->cta_count = c->plan.cta_items.empty() ? 0 : int(c->plan.cta_items.size()) - 1;
        c->prefill_count = int(P);
        c->prefix_count = int(X);
        c->step_prefix_rows = c->plan.group_rows.size();
        c->step_prefix_tokens = 0;
        for (int g = 0; g < int(G); ++g) {
            const auto& pl = c->plan;
            const int n = pl.group_row0[g + 1] - pl.group_row0[g];
            int tokens = 0;
            for (size_t w = 0; w < pl.prefix.size(); ++w)
                if (pl.prefix[w].group == g && pl.prefix[w].kv_head == 0 && pl.prefix[w].q_begin == 0)
                    tokens += pl.prefix[w].tok_end - pl.prefix[w].tok_begin;
            c->step_prefix_tokens += uint64_t(n) * tokens;
        }
        c->entry_count = entry_count;
        c->region_count = region_count;
        c->region_rows = region_rows;
        c->cow_two_phase = two_phase;
        c->cow_scratch_elements = region_elements;
        c->prepared = true;
        mirror_guard.keep = true;
    });
}

int mp_forward_launch(mp_context* c) {
    return guarded([&] {
        if (!c || !c->prepared) fail(MP_ERR_INVALID, "no prepared step");
        HostTimer host_time(c->counters_total.host_launch_ms);
        cuda_check(cudaSetDevice(c->device), "select device");
        const auto& m = c->model;
        const auto& r = c->rt;
        const int T = c->rows, S = c->seqs, H = m.hidden, I = m.intermediate;
        cudaStream_t st = c->stream;
        const int32_t* meta = c->meta;
        cuda_check(cudaMemsetAsync(c->error, 0, sizeof(unsigned), st), "reset error word");
        cuda_check(cudaEventRecord(c->fwd_events[0], st), "forward timing");
        // kernels of this forward: embed; per layer qkv (with rope/append), o, gate/up,
        // down (+1 per attention kind present); final norm, head, argmax; table
        // patch / COW if any
        c->step_launches = uint64_t(c->entry_count > 0) +
                           uint64_t(c->region_count > 0 && c->region_rows > 0) * (c->cow_two_phase ? 2 : 1) + 1 +
                           uint64_t(m.layers) * (4 + uint64_t(c->prefill_count > 0) + uint64_t(c->work_count > 0) +
                                                 uint64_t(c->prefix_count > 0)) +
                           3;
        cuda_check(mpb::launch_table_patch(meta + c->off_entries, c->entry_count, c->tables,
                                           int64_t(r.max_sequences) * r.table_stride, c->error, st),
                   "table patch launch");
        c->cow_timed = c->cow_timing && c->region_count > 0;
        if (c->cow_timed) cuda_check(cudaEventRecord(c->cow_events[0], st), "cow timing");
        const auto* regions = reinterpret_cast<const mpb::CowRegion*>(meta + c->off_regions);
        if (c->cow_two_phase) {
            const auto* at = reinterpret_cast<const uint64_t*>(meta + c->off_scratch);
            cuda_check(mpb::launch_cow_copy(regions, c->region_count, c->region_rows, c->keys, c->values,
                                            c->pool_elements, pool_geometry(c), c->error, st, mpb::kCowGather, at, c->cow_scratch,
                                            c->cow_scratch_elements),
                       "cow gather launch");
            cuda_check(mpb::launch_cow_copy(regions, c->region_count, c->region_rows, c->keys, c->values,
                                            c->pool_elements, pool_geometry(c), c->error, st, mpb::kCowScatter, at, c->cow_scratch,
                                            c->cow_scratch_elements),
                       "cow scatter launch");
        } else {
            cuda_check(mpb::launch_cow_copy(regions, c->region_count, c->region_rows, c->keys, c->values,
                                            c->pool_elements, pool_geometry(c), c->error, st),
                       "cow launch");
        }
        if (c->cow_timed) cuda_check(cudaEventRecord(c->cow_events[1], st), "cow timing");
        // RMSNorm before the QKV and gate/up projections is folded into the GEMMs: the
        // producer of x (embedding, O and down epilogues) writes x * w as the next
        // A operand and per-64-column sums of squares; the consumer scales its rows
        cuda_check(mpb::launch_embed_rmsnorm(meta + c->off_tokens, c->embed, m.vocabulary, c->in_norm, m.rms_epsilon,
                                             c->x, c->xn.hi, c->xn.lo, T, H, c->ssq, c->error, st),
                   "embed launch");
        const auto& mp = c->maps;
        // the QKV projection's epilogue applies RoPE and appends K/V to the pages
        mpb::RopeEpilogue rope{};
        rope.row_pos = meta + c->off_pos;
        rope.row_slot = meta + c->off_slot;
        rope.cos = c->rope_cos;
        rope.sin = c->rope_sin;
        rope.max_position = m.context;
        rope.q = c->q;
        rope.q_stride = H;
        rope.keys = c->keys;
        rope.values = c->values;
        rope.tables = c->tables;
        rope.table_stride = r.table_stride;
        rope.page_stride = 1;  // layer-major pools
        rope.block_tokens = r.block_tokens;
        rope.max_blocks = r.max_blocks;
        auto gemm = [&](const CUtensorMap& a_hi, const CUtensorMap& a_lo, const CUtensorMap& b_hi,
                        const CUtensorMap& b_lo, int rows, int n, int k, int b_row0, float* out, int ldc,
                        mpb::Epilogue e, const char* what, int bn = mpb::kTcBN, const float* norm_next = nullptr,
                        bool scale_rows = false) {
            mpb::TcGemmParams g{};
            g.m = rows;
            g.n = n;
            g.k = k;
            g.bn = bn;
            g.b_row0 = b_row0;
            g.c = out;
            g.ldc = ldc;
            g.rope = rope;
            g.out_hi = c->h.hi;
            g.out_lo = c->h.lo;
            g.ld_out = I;
            g.error = c->error;
            // x (the residual) is written only by the embedding, O and down launches,
            // each at least two launches before its next reader; the Rope metadata and
            // tables by the step's upload and table patch
            g.early_rows = 1;
            if (norm_next) {  // producer of the next GEMM's normalised input
                g.norm_w = norm_next;
                g.out_hi = c->xn.hi;
                g.out_lo = c->xn.lo;
                g.ld_out = H;
                g.ssq_out = c->ssq;
            }
            if (scale_rows) {  // consumer: rows scaled by 1 / rms
                g.ssq_in = c->ssq;
                g.eps = m.rms_epsilon;
            }
            if (c->stall_next_us > 0) {  // mp_inject_wait_timeout: this launch's waits run out
                g.stall = 1;
                g.wait_ns = uint64_t(c->stall_next_us) * 1000u;
                c->stall_next_us = 0;
            }
            cuda_check(mpb::launch_tc_gemm({&a_hi, &a_lo, &b_hi, &b_lo}, g, e, st), what);
        };
        mpb::AttnParams ap{};
        ap.q = c->q;
        ap.q_stride = H;
        ap.keys = c->keys;
        ap.values = c->values;
        ap.page_stride = 1;  // layer-major pools
        ap.block_tokens = r.block_tokens;
        ap.max_blocks = r.max_blocks;
        ap.tables = c->tables;
        ap.table_stride = r.table_stride;
        ap.row_slot = meta + c->off_slot;
        ap.row_len = meta + c->off_len;
        ap.row_splits = meta + c->off_splits;
        ap.row_work0 = meta + c->off_work0;
        ap.row_x0 = meta + c->off_x0;
        ap.row_nx = meta + c->off_nx;
        ap.order = meta + c->off_order;
        ap.sched = c->attn_sched;
        ap.cta_items = c->cta_count ? meta + c->off_cta : nullptr;
        ap.cta_count = c->cta_count;
        ap.work = reinterpret_cast<const mpb::AttnWork*>(meta + c->off_work);
        ap.work_count = c->work_count;
        ap.partial = c->partial;
        ap.counters = c->counters;
        ap.out = nullptr;
        ap.out_hi = c->attn.hi;
        ap.out_lo = c->attn.lo;
        ap.out_stride = H;
        ap.error = c->error;
        ap.early_copies = 1;  // the step's uploads and COW copies precede every layer
        mpb::PrefixParams xp{};
        xp.q = c->q;
        xp.q_stride = H;
        xp.keys = c->keys;
        xp.values = c->values;
        xp.page_stride = 1;  // layer-major pools
        xp.block_tokens = r.block_tokens;
        xp.max_blocks = r.max_blocks;
        xp.tables = c->tables;
        xp.table_stride = r.table_stride;
        xp.group_rows = meta + c->off_group_rows;
        xp.group_row0 = meta + c->off_group_row0;
        xp.group_slot = meta + c->off_group_slot;
        xp.row_x0 = meta + c->off_x0;
        xp.work = reinterpret_cast<const mpb::PrefixWork*>(meta + c->off_prefix);
        xp.work_count = c->prefix_count;
        xp.partial = c->partial;
        xp.error = c->error;
        mpb::PrefillParams pp{};
        pp.q = c->q;
        pp.q_stride = H;
        pp.keys = c->keys;
        pp.values = c->values;
        pp.page_stride = 1;  // layer-major pools
        pp.block_tokens = r.block_tokens;
        pp.max_blocks = r.max_blocks;
        pp.tables = c->tables;
        pp.table_stride = r.table_stride;
        pp.work = reinterpret_cast<const mpb::PrefillWork*>(meta + c->off_prefill);
        pp.work_count = c->prefill_count;
        pp.out = nullptr;
        pp.out_hi = c->attn.hi;
        pp.out_lo = c->attn.lo;
        pp.out_stride = H;
        pp.error = c->error;
        for (int l = 0; l < m.layers; ++l) {
            const size_t L = size_t(l);
            const int64_t layer_offset = int64_t(l) * r.max_blocks;  // pool_page(): layer-major pools
            rope.layer_offset = layer_offset;
            gemm(mp.xn_hi, mp.xn_lo, mp.wqkv_hi, mp.wqkv_lo, T, c->qkvw, H, l * c->qkvw, nullptr, 0,
                 mpb::Epilogue::Rope, "qkv gemm", mpb::kTcBN, nullptr, true);
            ap.layer_offset = layer_offset;
            pp.layer_offset = layer_offset;
            xp.layer_offset = layer_offset;
            if (c->profile) record_attention_event(c);
            cuda_check(mpb::launch_prefill_attention(pp, st), "prefill attention launch");
            cuda_check(mpb::launch_prefix_attention(xp, st), "shared-prefix attention launch");
            cuda_check(mpb::launch_paged_attention(ap, st), "attention launch");
            if (c->profile) record_attention_event(c);
            gemm(mp.attn_hi, mp.attn_lo, mp.wo_hi, mp.wo_lo, T, H, H, l * H, c->x, H, mpb::Epilogue::AddTo, "o gemm",
                 mpb::kTcBN, c->post_norm + L * H);
            gemm(mp.xn_hi, mp.xn_lo, mp.wgu_hi, mp.wgu_lo, T, 2 * I, H, l * 2 * I, nullptr, I, mpb::Epilogue::SwiGLU,
                 "gate/up gemm", kGateUpBN, nullptr, true);
            gemm(mp.h_hi, mp.h_lo, mp.wdown_hi, mp.wdown_lo, T, H, I, l * H, c->x, H, mpb::Epilogue::AddTo,
                 "down gemm", mpb::kTcBN, l + 1 < m.layers ? c->in_norm + (L + 1) * H : nullptr);
        }
        cuda_check(mpb::launch_rmsnorm(c->x, meta + c->off_last, c->final_norm, m.rms_epsilon, c->xl.hi, c->xl.lo, S,
                                       H, st),
                   "final norm launch");
        if (c->profile) {
            for (auto& e : c->head_events)
                if (!e) cuda_check(cudaEventCreate(&e), "profile event");
            cuda_check(cudaEventRecord(c->head_events[0], st), "profile event record");
        }
        gemm(mp.xl_hi, mp.xl_lo, mp.head_hi, mp.head_lo, S, m.vocabulary, H, 0, c->logits, m.vocabulary,
             mpb::Epilogue::Store, "lm head gemm", head_tile_n(m.vocabulary));
        if (c->profile) cuda_check(cudaEventRecord(c->head_events[1], st), "profile event record");
        cuda_check(mpb::launch_argmax(c->logits, S, m.vocabulary, c->out_tokens, c->out_finite, st), "argmax launch");
        cuda_check(cudaEventRecord(c->fwd_events[1], st), "forward timing");
        if (c->profile) c->prof_bytes += c->plan.bytes * m.layers;
    });
}

int mp_forward_collect(mp_context* c, int32_t* out_tokens, int32_t* out_finite, float* out_logits,
                       int32_t timeout_ms) {
    int finite_all = 1;
    int rc = guarded([&] {
        if (!c || !c->prepared) fail(MP_ERR_INVALID, "no prepared step");
        cuda_check(cudaSetDevice(c->device), "select device");
        const int S = c->seqs;
        cudaStream_t st = c->stream;
        cuda_check(cudaMemcpyAsync(c->h_tokens, c->out_tokens, size_t(S) * 4, cudaMemcpyDeviceToHost, st),
                   "download tokens");
        cuda_check(cudaMemcpyAsync(c->h_finite, c->out_finite, size_t(S) * 4, cudaMemcpyDeviceToHost, st),
                   "download finite flags");
        cuda_check(cudaMemcpyAsync(c->h_error, c->error, sizeof(unsigned), cudaMemcpyDeviceToHost, st),
                   "download error word");
        if (out_logits)
            cuda_check(cudaMemcpyAsync(out_logits, c->logits, size_t(S) * c->model.vocabulary * 4,
                                       cudaMemcpyDeviceToHost, st),
                       "download logits");
        cuda_check(cudaEventRecord(c->done, st), "record completion");
        {
            HostTimer host_time(c->counters_total.host_wait_ms);
            wait_event(c->done, timeout_ms);
        }
        if (c->profile) harvest_profile(c);
        {
            float ms = 0.f;
            cuda_check(cudaEventElapsedTime(&ms, c->fwd_events[0], c->fwd_events[1]), "forward elapsed");
            c->counters_total.forwards += 1;
            c->counters_total.forward_ms += ms;
            c->counters_total.kernel_launches += c->step_launches;
            c->counters_total.h2d_bytes += c->step_h2d;
            c->counters_total.shared_prefix_rows += c->step_prefix_rows;
            c->counters_total.shared_prefix_tokens += c->step_prefix_tokens;
            c->counters_total.d2h_bytes += size_t(S) * 8 + sizeof(unsigned) +
                                           (out_logits ? size_t(S) * c->model.vocabulary * 4 : 0);
        }
        if (c->cow_timed) {
            cuda_check(cudaEventElapsedTime(&c->cow_ms, c->cow_events[0], c->cow_events[1]), "cow elapsed");
            c->cow_timed = false;
        }
        if (out_tokens) std::memcpy(out_tokens, c->h_tokens, size_t(S) * 4);
        if (out_finite) std::memcpy(out_finite, c->h_finite, size_t(S) * 4);
        for (int i = 0; i < S; ++i) finite_all &= c->h_finite[i] != 0;
        c->prepared = false;
        const unsigned err = *c->h_error;
        if (err & mpb::kErrTimeout) {
            // an attention CTA that gave up never counted its slice in
            cuda_check(cudaMemsetAsync(c->counters, 0, size_t(c->rt.max_step_tokens) * mpb::kKvHeads * sizeof(unsigned),
                                       c->stream),
                       "reset attention counters");
            cuda_check(cudaMemsetAsync(c->attn_sched, 0, 2 * sizeof(unsigned), c->stream), "reset schedule");
            fail(MP_ERR_TIMEOUT, "an in-kernel copy wait expired");
        }
        if (err & mpb::kErrBounds) fail(MP_ERR_BOUNDS, "device bounds check failed (page id, token or region)");
    });
    if (rc == MP_OK && !finite_all) {
        g_error = "nonfinite logits";
        rc = MP_ERR_NONFINITE;
    }
    return rc;
}

int mp_forward(mp_context* c, const mp_sequence_desc* seqs, int32_t count, const int32_t* tokens,
               const mp_table_entry* entries, int32_t entry_count, const mp_tail_copy_region* regions,
               int32_t region_count, int32_t* out_tokens, int32_t* out_finite, float* out_logits,
               int32_t timeout_ms) {
    int rc = mp_forward_prepare(c, seqs, count, tokens, entries, entry_count, regions, region_count);
    if (rc != MP_OK) return rc;
    rc = mp_forward_launch(c);
    if (rc != MP_OK) {
        if (c && c->stream) {
            const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(c->host_wait_ms);
            while (cudaStreamQuery(c->stream) == cudaErrorNotReady && std::chrono::steady_clock::now() < deadline)
                std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
        if (c) c->prepared = false;
        return rc;
    }
    return mp_forward_collect(c, out_tokens, out_finite, out_logits, timeout_ms);
}

int mp_inject_wait_timeout(mp_context* c, int32_t wait_us) {
    return guarded([&] {
        if (!c || wait_us < 1 || wait_us > 1000000) fail(MP_ERR_INVALID, "wait limit must be 1 us .. 1 s");
        c->stall_next_us = wait_us;
    });
}

int mp_sync(mp_context* c, int32_t timeout_ms) {
    return guarded([&] {
        if (!c) fail(MP_ERR_INVALID, "null context");
        cuda_check(cudaSetDevice(c->device), "select device");
        cuda_check(cudaEventRecord(c->done, c->stream), "record completion");
        wait_event(c->done, timeout_ms);
        cuda_check(cudaMemcpy(c->h_error, c->error, sizeof(unsigned), cudaMemcpyDeviceToHost), "read error word");
        const unsigned err = *c->h_error;
        if (err) {
            cuda_check(cudaMemsetAsync(c->error, 0, sizeof(unsigned), c->stream), "reset error word");
            if (err & mpb::kErrTimeout) fail(MP_ERR_TIMEOUT, "an in-kernel copy wait expired");
            fail(MP_ERR_BOUNDS, "device bounds check failed (page id, token or region)");
        }
    });
}

int mp_kv_pools(mp_context* c, float** keys, float** values, uint64_t* elements) {
    if (!c) return MP_ERR_INVALID;
    if (keys) *keys = c->keys;
    if (values) *values = c->values;
    if (elements) *elements = c->pool_elements;
    return MP_OK;
}

// Host copies of the reference-layout element range [offset, offset + count): the
// range is cut at page boundaries of the reference layout, and each run of whole
// blocks moves as one strided copy per layer.
static int kv_copy(mp_context* c, int32_t pool, uint64_t offset, uint64_t count, void* host, bool to_device) {
    return guarded([&] {
        if (!c || !host || (pool != 0 && pool != 1)) fail(MP_ERR_INVALID, "invalid argument");
        if (offset > c->pool_elements || count > c->pool_elements - offset) fail(MP_ERR_INVALID, "range outside the pool");
        cuda_check(cudaSetDevice(c->device), "select device");
        wait_stream(c, "pool copy ordering");
        float* base = pool == 0 ? c->keys : c->values;
        float* h = static_cast<float*>(host);
        const mpb::PoolGeometry g = pool_geometry(c);
        const uint64_t page = g.page_elements, block = page * g.layers;
        auto piece = [&](uint64_t e, uint64_t n) {  // n floats inside one reference page
            float* d = base + mpb::layer_major_offset(g, e);
            float* hp = h + (e - offset);
            cuda_check(to_device ? cudaMemcpy(d, hp, n * 4, cudaMemcpyHostToDevice)
                                 : cudaMemcpy(hp, d, n * 4, cudaMemcpyDeviceToHost),
                       "pool copy");
        };
        uint64_t e = offset;
        const uint64_t end = offset + count;
        while (e < end && (e % block != 0 || end - e < block)) {  // head: pieces up to a block boundary
            const uint64_t n = std::min(end - e, page - e % page);
            piece(e, n);
            e += n;
        }
        if (e < end) {  // whole blocks [b0, b1): one 2D copy per layer
            const uint64_t b0 = e / block, b1 = b0 + (end - e) / block;
            for (uint64_t l = 0; l < g.layers; ++l) {
                float* d = base + (l * g.max_blocks + b0) * page;
                float* hp = h + (b0 * block + l * page - offset);
                cuda_check(to_device ? cudaMemcpy2D(d, page * 4, hp, block * 4, page * 4, b1 - b0,
                                                    cudaMemcpyHostToDevice)
                                     : cudaMemcpy2D(hp, block * 4, d, page * 4, page * 4, b1 - b0,
                                                    cudaMemcpyDeviceToHost),
                           "pool copy");
            }
            e = b1 * block;
            while (e < end) {  // tail
                const uint64_t n = std::min(end - e, page - e % page);
                piece(e, n);
                e += n;
            }
        }
    });
}

int mp_kv_read(mp_context* c, int32_t pool, uint64_t offset, uint64_t count, float* host) {
    return kv_copy(c, pool, offset, count, host, false);
}

int mp_kv_write(mp_context* c, int32_t pool, uint64_t offset, uint64_t count, const float* host) {
    return kv_copy(c, pool, offset, count, const_cast<float*>(host), true);
}

void* mp_stream(mp_context* c) { return c ? static_cast<void*>(c->stream) : nullptr; }

int mp_timer_mark(mp_context* c) {
    return guarded([&] {
        if (!c) fail(MP_ERR_INVALID, "null context");
        cuda_check(cudaEventRecord(c->mark[c->mark_count & 1], c->stream), "timer mark");
        ++c->mark_count;
    });
}

int mp_timer_elapsed(mp_context* c, float* ms) {
    return guarded([&] {
        if (!c || !ms || c->mark_count < 2) fail(MP_ERR_INVALID, "need two timer marks");
        cudaEvent_t a = c->mark[(c->mark_count - 2) & 1], b = c->mark[(c->mark_count - 1) & 1];
        cuda_check(cudaEventSynchronize(b), "timer wait");
        cuda_check(cudaEventElapsedTime(ms, a, b), "timer elapsed");
    });
}

int mp_read_counters(mp_context* c, mp_counters* out, int32_t reset) {
    if (!c || !out) return MP_ERR_INVALID;
    *out = c->counters_total;
    if (reset) c->counters_total = mp_counters{};
    return MP_OK;
}

int mp_cow_timing(mp_context* c, int32_t enabled) {
    if (!c) return MP_ERR_INVALID;
    c->cow_timing = enabled != 0;
    return MP_OK;
}

int mp_cow_elapsed(mp_context* c, float* ms) {
    if (!c || !ms) return MP_ERR_INVALID;
    *ms = c->cow_ms;
    c->cow_ms = 0.f;
    return MP_OK;
}

int mp_set_shared_prefix(mp_context* c, int32_t min_rows, int32_t min_tokens) {
    if (!c || min_rows < 0 || min_tokens < 0) return MP_ERR_INVALID;
    c->group_min_rows = min_rows;
    c->group_min_tokens = min_tokens;
    return MP_OK;
}

int mp_profile_enable(mp_context* c, int32_t enabled) {
    if (!c) return MP_ERR_INVALID;
    c->profile = enabled != 0;
    return MP_OK;
}

int mp_profile_read(mp_context* c, float* attention_ms, int32_t* launches, double* bytes) {
    if (!c) return MP_ERR_INVALID;
    if (attention_ms) *attention_ms = c->prof_ms;
    if (launches) *launches = c->prof_launches;
    if (bytes) *bytes = c->prof_bytes;
    c->prof_ms = 0.f;
    c->prof_launches = 0;
    c->prof_bytes = 0;
    return MP_OK;
}

int mp_profile_read_gemm(mp_context* c, float* layer_gemm_ms, int32_t* intervals, float* head_ms, int32_t* heads) {
    if (!c) return MP_ERR_INVALID;
    if (layer_gemm_ms) *layer_gemm_ms = c->prof_gemm_ms;
    if (intervals) *intervals = c->prof_gemm_intervals;
    if (head_ms) *head_ms = c->prof_head_ms;
    if (heads) *heads = c->prof_heads;
    c->prof_gemm_ms = c->prof_head_ms = 0.f;
    c->prof_gemm_intervals = c->prof_heads = 0;
    return MP_OK;
}

// C = A . B^T through the split-precision tensor-core GEMM on caller device buffers
// (a [m][k], b [n][k], c [m][n], row-major). Allocates and frees its own hi/lo
// scratch and synchronises `stream`; meant for tests and tools, not for the hot path.
int mp_gemm_f32(const float* a, const float* b, float* out, int32_t m, int32_t n, int32_t k, void* stream_ptr) {
    std::vector<void*> scratch;
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    const int rc = guarded([&] {
        if (!a || !b || !out || m < 1 || n < 1 || k < 1) fail(MP_ERR_INVALID, "invalid argument");
        if (n % mpb::kTcBN || k % 32) fail(MP_ERR_INVALID, "n must be a multiple of 64 and k of 32");
        cuda_check(mpb::configure_tc_gemm(), "configure tensor-core GEMM");
        const size_t rows_a = (size_t(m) + 127) / 128 * 128, rows_b = size_t(n);
        auto alloc = [&](size_t count) {
            __half* p = device_alloc<__half>(count, "gemm scratch");
            scratch.push_back(p);
            cuda_check(cudaMemsetAsync(p, 0, count * sizeof(__half), st), "clear gemm scratch");
            return p;
        };
        __half *ah = alloc(rows_a * k), *al = alloc(rows_a * k), *bh = alloc(rows_b * k), *bl = alloc(rows_b * k);
        cuda_check(mpb::launch_split(a, ah, al, size_t(m) * k, st), "split a");
        cuda_check(mpb::launch_split(b, bh, bl, size_t(n) * k, st), "split b");
        struct alignas(64) M4 {
            CUtensorMap ah, al, bh, bl;
        };
        auto maps = std::make_unique<M4>();
        encode_map(&maps->ah, ah, rows_a, k, 128);
        encode_map(&maps->al, al, rows_a, k, 128);
        // the forward's tile width for this N: 256 for the LM head, 128 for gate/up, else 64
        const int bn = gemm_tile_n(n);
        encode_map(&maps->bh, bh, rows_b, k, uint32_t(bn));
        encode_map(&maps->bl, bl, rows_b, k, uint32_t(bn));
        unsigned* err = device_alloc<unsigned>(1, "gemm error word");
        scratch.push_back(err);
        cuda_check(cudaMemsetAsync(err, 0, 4, st), "clear error word");
        mpb::TcGemmParams g{};
        g.m = m;
        g.n = n;
        g.k = k;
        g.bn = bn;
        g.c = out;
        g.ldc = n;
        g.error = err;
        cuda_check(mpb::launch_tc_gemm({&maps->ah, &maps->al, &maps->bh, &maps->bl}, g, mpb::Epilogue::Store, st),
                   "gemm launch");
        unsigned herr = 0;
        cuda_check(cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, st), "read error word");
        cudaEvent_t done = nullptr;
        cuda_check(cudaEventCreateWithFlags(&done, cudaEventDisableTiming), "create event");
        const cudaError_t recorded = cudaEventRecord(done, st);
        try {
            cuda_check(recorded, "gemm completion");
            wait_event(done, 600000);
        } catch (...) {
            cudaEventDestroy(done);
            throw;
        }
        cudaEventDestroy(done);
        if (herr) fail(MP_ERR_TIMEOUT, "tensor-core GEMM wait expired");
    });
    for (void* p : scratch) cudaFree(p);
    return rc;
}

}  // extern "C"
