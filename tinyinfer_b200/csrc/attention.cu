// Paged attention over the MiniPrefix K/V page pools (sm_100a), decode rows.
//
// Replaces the reference's attention_kernel (miniprefix/src/backend/cuda/
// llama_runner.cu:33-48: one block per (row, q head), one token per iteration,
// eight __syncthreads per token, each K/V row fetched once per q head) and
// computes the CPU runner's attention (miniprefix/src/backend/cpu/
// llama_runner.cpp:85-93): causal GQA, kv head = h / 3, scale 1/sqrt(64), softmax.
//
// Work: a row's context is cut into slices [page_begin, page_end) (work items).
// Rows with several slices, or with shared-prefix partials written earlier on the
// stream by attention_shared.cu, are merged per (row, kv head) by the last slice
// to finish (an arrival counter per (row, kv head)), so one launch produces the
// final output.
//
// CTA = 4 warps, warp-specialised, no block-wide barrier in the steady state:
//  * warp 3 (producer) walks its work items -- one; or a fixed run of items (a
//    static schedule that gives every CTA an equal share of the pages); or items
//    pulled from a shared counter in the given order (persistent, one wave) --
//    and for every 16-token stage writes a stage descriptor (item, row, first
//    token, valid tokens, first/last flags) and moves the stage's K and V runs
//    (contiguous inside a page: [slot][192] floats of one layer) into a ring of 3
//    shared-memory stages with the bulk-copy engine (cp.async.bulk), completing
//    on the stage's `full` mbarrier. It refills a stage once the three consumers
//    released it (`empty` mbarrier, count 3).
//  * warps 0..2 (consumers) each own one kv head and its 3 query heads. Lane =
//    (token t of 8, quarter c of the 64 dims); two passes cover 16 tokens. A lane
//    keeps its 3 heads' 16 query values (rotated by t so a 128-bit phase spans all
//    banks) in registers. Scores are reduced over the quarters by shuffles, the
//    online softmax over the 16 tokens by shuffles, probabilities go through a
//    per-warp scratch row, and P.V accumulates dims (2 lane, 2 lane + 1) of 3 heads.
//  * Each consumer finishes a slice on its own: direct output for a single-slice
//    row, else its partial (max, sum, unnormalised output) and the merge when it
//    is the last arrival for (row, its kv head).
//  * Arithmetic: packed FP32 FMAs (fma.rn.f32x2) for Q.K (even / odd dims) and
//    P.V (dims 2 lane / 2 lane + 1); softmax weights as exp2 of scores scaled by
//    log2(e) / 8, so maxima in partials are base-2 quantities.
// Every wait is bounded (common.cuh); a timeout sets the error word and the warp
// stops. Tokens past the row length are masked by select (never by multiplying).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace mpb {
namespace {

#ifndef MPB_ATTN_STAGE_TOKENS
#define MPB_ATTN_STAGE_TOKENS 16
#endif
#ifndef MPB_ATTN_STAGES
#define MPB_ATTN_STAGES 3
#endif
constexpr int kStageTokens = MPB_ATTN_STAGE_TOKENS;  // a multiple of 8
constexpr int kStages = MPB_ATTN_STAGES;
constexpr int kPasses = kStageTokens / 8;            // 8 tokens per consumer pass
static_assert(kStageTokens % 8 == 0 && kPasses >= 1, "stage = whole consumer passes");
// Query of a consumer's current row: in registers (48 per lane), or, with
// MPB_ATTN_Q_SMEM, in a per-warp shared-memory slot read once per pass (frees the
// registers for more resident CTAs per SM).
#ifndef MPB_ATTN_Q_SMEM
#define MPB_ATTN_Q_SMEM 0
#endif
constexpr bool kQInSmem = MPB_ATTN_Q_SMEM != 0;
constexpr int kConsumers = kKvHeads;                   // 3 consumer warps
constexpr int kThreads = (kConsumers + 1) * 32;        // + producer warp
constexpr int kStageFloats = kStageTokens * kKvWidth;  // per pool

struct StageDesc {
    int32_t work;     // work item index, -1: no more work
    int32_t row;
    int32_t token;    // first context token of the stage
    int32_t n_valid;  // tokens of the stage inside the row (0..16)
    int32_t flags;    // kFirst: first stage of its item; kLast: last
    int32_t pad[3];
};
constexpr int kFirst = 1, kLast = 2;

constexpr size_t kAttnSmem = size_t(kStages) * 2 * kStageFloats * sizeof(float) +         // K/V stages
                             size_t(kConsumers) * kGroup * kStageTokens * sizeof(float) +  // probabilities
                             size_t(kConsumers) * kGroup * kHeadDim * sizeof(float) +      // queries
                             kStages * sizeof(StageDesc) + 2 * kStages * sizeof(uint64_t) + 16;

// Output elements: plain FP32, or the O projection's FP16 hi/lo halves when the
// caller asked for them. write_out2 writes elements i and i + 1 (i even).
__device__ __forceinline__ void write_out(const AttnParams& p, size_t i, float v) {
    if (p.out_hi) {
        __half h, l;
        split_f16(v, h, l);
        p.out_hi[i] = h;
        p.out_lo[i] = l;
    } else {
        p.out[i] = v;
    }
}
__device__ __forceinline__ void write_out2(const AttnParams& p, size_t i, float v0, float v1) {
    if (p.out_hi) {
        store_split2(p.out_hi + i, p.out_lo + i, v0, v1);
    } else {  // caller buffers of the operator entry points: 4-byte alignment only
        p.out[i] = v0;
        p.out[i + 1] = v1;
    }
}

// Producer: copy context tokens [a, b) into stage buffers kdst/vdst; the whole
// warp calls it. Lane L moves the run inside page a/bt + L. Page ids come from the
// warp's window of staged table entries (lane i holds page win0 + i) when they
// fall inside it, else from the table.
__device__ __forceinline__ void issue_stage(const AttnParams& p, const int32_t* table, int win0, int window, int a,
                                            int b, float* kdst, float* vdst, uint64_t* bar, int lane) {
    const int bt = p.block_tokens;
    const int first_page = a / bt;
    const int run_begin = max(a, (first_page + lane) * bt);
    const int run_end = min(b, (first_page + lane + 1) * bt);
    const int page = first_page + lane;
    const int rel = page - win0;
    const int staged = __shfl_sync(0xffffffffu, window, rel & 31);
    if (lane == 0) mbar_arrive_expect_tx(bar, uint32_t(b - a) * 2u * kKvWidth * sizeof(float));
    __syncwarp();
    if (run_begin < run_end) {
        int block = rel >= 0 && rel < 32 ? staged : (page < p.table_stride ? table[page] : -1);
        if (block < 0 || block >= p.max_blocks) {
            raise_error(p.error, kErrBounds);
            block = 0;  // stay in bounds; the error word fails the step
        }
        const size_t src = (pool_page(block, p.page_stride, p.layer_offset) * bt + (run_begin - page * bt)) * kKvWidth;
        const uint32_t bytes = uint32_t(run_end - run_begin) * kKvWidth * sizeof(float);
        bulk_copy_g2s(kdst + (run_begin - a) * kKvWidth, p.keys + src, bytes, bar);
        bulk_copy_g2s(vdst + (run_begin - a) * kKvWidth, p.values + src, bytes, bar);
    }
}

__device__ void producer(const AttnParams& p, float* stages, StageDesc* desc, uint64_t* full, uint64_t* empty,
                         bool persistent, unsigned* failed, int lane) {
    uint32_t g = 0;  // stages issued so far
    const bool fixed = p.cta_items != nullptr;
    // With early copies the schedule is read, and the first ring fill of stages
    // below row_len - kPrefillMinRows is issued, before the programmatic wait.
    bool waited = false;
    auto enter = [&] {
        if (!waited) {
            pdl_enter();
            waited = true;
        }
    };
    if (!(fixed && p.early_copies)) enter();
    int item = fixed ? p.cta_items[blockIdx.x] : int(blockIdx.x);
    const int item_end = fixed ? p.cta_items[blockIdx.x + 1] : p.work_count;
    // a stage's previous use must have been released by the 3 consumers
    auto acquire = [&](int buf) -> bool {
        if (g < uint32_t(kStages)) return true;
        return mbar_wait_bounded(&empty[buf], ((g / kStages) - 1) & 1);
    };
    while (true) {
        if (item >= item_end) {
            enter();
            // no more work: a descriptor without copies releases the consumers
            const int buf = g % kStages;
            if (!acquire(buf)) {
                if (lane == 0) atomicOr(failed, 1u);
                return;
            }
            if (lane == 0) {
                desc[buf].work = -1;
                mbar_arrive_expect_tx(&full[buf], 0);
            }
            return;
        }
        const int wi = !fixed && p.order ? p.order[item] : item;
        int next = 0;
        if (fixed) next = item + 1;
        else if (lane == 0) next = persistent ? int(gridDim.x + atomicAdd(&p.sched[0], 1u)) : p.work_count;
        next = __shfl_sync(0xffffffffu, next, 0);
        const AttnWork w = p.work[wi];
        const int row = w.row;
        const int len = p.row_len[row];
        const int32_t* table = p.tables + size_t(p.row_slot[row]) * p.table_stride;
        const int tok_begin = w.page_begin * p.block_tokens;
        const int tok_end = min(w.page_end * p.block_tokens, len);
        const int n_stages = max(1, (tok_end - tok_begin + kStageTokens - 1) / kStageTokens);
        // table entries of the slice's first 32 pages, one per lane, loaded once;
        // the window moves on when a stage starts past it
        int win0 = w.page_begin;
        auto load_window = [&](int first) {
            const int pg = first + lane;
            return pg < w.page_end && pg < p.table_stride ? table[pg] : -1;
        };
        int window = load_window(win0);
        for (int i = 0; i < n_stages; ++i) {
            const int b = g % kStages;
            {
                const int first_page = (tok_begin + i * kStageTokens) / p.block_tokens;
                if (first_page + (kStageTokens + p.block_tokens - 1) / p.block_tokens >= win0 + 32) {
                    win0 = first_page;
                    window = load_window(win0);
                }
            }
            const int a = tok_begin + i * kStageTokens;
            const int e = min(a + kStageTokens, tok_end);
            if (g >= uint32_t(kStages) || e + kPrefillMinRows > len) enter();
            if (!acquire(b)) {
                if (lane == 0) atomicOr(failed, 1u);
                return;
            }
            if (lane == 0) {
                desc[b].work = wi;
                desc[b].row = row;
                desc[b].token = a;
                desc[b].n_valid = max(0, e - a);
                desc[b].flags = (i == 0 ? kFirst : 0) | (i == n_stages - 1 ? kLast : 0);
            }
            __syncwarp();
            // buffers last read by the consumers (generic proxy) are now refilled by
            // the bulk-copy engine (async proxy)
            fence_proxy_async_shared();
            if (e > a) {
                issue_stage(p, table, win0, window, a, e, stages + 2 * b * kStageFloats,
                            stages + (2 * b + 1) * kStageFloats, &full[b], lane);
            } else if (lane == 0) {
                mbar_arrive_expect_tx(&full[b], 0);  // an empty slice still reports
            }
            ++g;
        }
        item = next;
    }
}

__device__ void consumer(const AttnParams& p, const float* stages, const StageDesc* desc, uint64_t* full,
                         uint64_t* empty, float* probs, float* qs, unsigned* failed, int kh, int lane) {
    const int t = lane >> 2, c = lane & 3;
    float4 qr[kGroup][4];
    // softmax state of head c (lanes with c == 3 carry an unused copy)
    float m_run = -INFINITY, l_run = 0.f, acc[kGroup][2];
#pragma unroll
    for (int hh = 0; hh < kGroup; ++hh) {
        acc[hh][0] = acc[hh][1] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) qr[hh][j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    uint32_t g = 0;
    while (true) {
        const int buf = g % kStages;
        if (!mbar_wait_bounded(&full[buf], (g / kStages) & 1)) {
            if (lane == 0) atomicOr(failed, 1u);
            return;
        }
        const StageDesc d = desc[buf];
        if (d.work < 0) return;
        if (d.flags & kFirst) {
            const float* qrow = p.q + size_t(d.row) * p.q_stride + kh * kGroup * kHeadDim;
            if constexpr (kQInSmem) {
                // the row's 3 x 64 query values into this warp's slot (48 float4)
                for (int i = lane; i < kGroup * kHeadDim / 4; i += 32)
                    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(qrow)[i];
                __syncwarp();
            }
#pragma unroll
            for (int hh = 0; hh < kGroup; ++hh) {
                if constexpr (!kQInSmem) {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        qr[hh][j] = *reinterpret_cast<const float4*>(qrow + hh * kHeadDim + c * 16 + 4 * ((j + t) & 3));
                }
                acc[hh][0] = acc[hh][1] = 0.f;
            }
            m_run = -INFINITY;
            l_run = 0.f;
        }
        const float* kst = stages + 2 * buf * kStageFloats + kh * kHeadDim + c * 16;
        const float* vst = stages + (2 * buf + 1) * kStageFloats + kh * kHeadDim + 2 * lane;
        const bool full_stage = d.n_valid == kStageTokens;
        // Q.K partial sums of tokens t + 8 ps over this lane's quarter of the dims,
        // for the 3 heads (even / odd dims in the two halves of a packed FMA)
        float x[kPasses][4];
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps) {
            const float* krow = kst + (t + 8 * ps) * kKvWidth;
            float pe[kGroup] = {0.f, 0.f, 0.f}, po[kGroup] = {0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 kv = *reinterpret_cast<const float4*>(krow + 4 * ((j + t) & 3));
#pragma unroll
                for (int hh = 0; hh < kGroup; ++hh) {
                    const float4 qv = kQInSmem ? *reinterpret_cast<const float4*>(qs + hh * kHeadDim + c * 16 +
                                                                                  4 * ((j + t) & 3))
                                               : qr[hh][j];
                    fma2(pe[hh], po[hh], qv.x, qv.y, kv.x, kv.y);
                    fma2(pe[hh], po[hh], qv.z, qv.w, kv.z, kv.w);
                }
            }
#pragma unroll
            for (int hh = 0; hh < kGroup; ++hh) x[ps][hh] = pe[hh] + po[hh];
            x[ps][3] = 0.f;
        }
        // Reduce-scatter over the 4 quarter lanes of a token: lane c ends with the
        // full score of head c (c = 3: an unused fourth slot). Pairs xor 1 first,
        // then xor 2, so each sum is ((q0 + q1) + (q2 + q3)) in quarter order.
        const bool odd = c & 1, high = c & 2;
        float s[kPasses];
#pragma unroll
        for (int ps = 0; ps < kPasses; ++ps) {
            // lanes with even c keep heads {0, 2}, odd c heads {1, 3}
            const float k0 = odd ? x[ps][1] : x[ps][0], k1 = odd ? x[ps][3] : x[ps][2];
            const float g0 = odd ? x[ps][0] : x[ps][1], g1 = odd ? x[ps][2] : x[ps][3];
            const float y0 = k0 + __shfl_xor_sync(0xffffffffu, g0, 1);
            const float y1 = k1 + __shfl_xor_sync(0xffffffffu, g1, 1);
            // c < 2 keep the first of the pair (head 0 or 1), c >= 2 the second (head 2 or 3)
            const float keep = high ? y1 : y0, give = high ? y0 : y1;
            const float part = keep + __shfl_xor_sync(0xffffffffu, give, 2);
            const bool valid = full_stage || t + 8 * ps < d.n_valid;
            s[ps] = valid ? part * (0.125f * kLog2e) : -INFINITY;  // base-2 units
        }
        // online softmax of head c over the stage's tokens (lanes differ in t across bits 2..4)
        float alpha;
        {
            float mx = s[0];
#pragma unroll
            for (int ps = 1; ps < kPasses; ++ps) mx = fmaxf(mx, s[ps]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float m_new = fmaxf(m_run, mx);
            const float ms = m_new == -INFINITY ? 0.f : m_new;  // no valid token yet: all terms stay 0
            alpha = exp2f(m_run - ms);
            float pw[kPasses];
            float sum = 0.f;
#pragma unroll
            for (int ps = 0; ps < kPasses; ++ps) {
                pw[ps] = exp2f(s[ps] - ms);
                sum += pw[ps];
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            sum += __shfl_xor_sync(0xffffffffu, sum, 8);
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            l_run = l_run * alpha + sum;
            m_run = m_new;
            if (c < kGroup) {
#pragma unroll
                for (int ps = 0; ps < kPasses; ++ps) probs[c * kStageTokens + t + 8 * ps] = pw[ps];
            }
        }
        // every lane rescales its dims of all 3 heads: head hh's factor from lane hh
#pragma unroll
        for (int hh = 0; hh < kGroup; ++hh) {
            const float a = __shfl_sync(0xffffffffu, alpha, hh);
            acc[hh][0] *= a;
            acc[hh][1] *= a;
        }
        __syncwarp();
        // P.V: dims (2 lane, 2 lane + 1) of this kv head, one packed FMA per head and token
#pragma unroll
        for (int q4 = 0; q4 < kStageTokens / 4; ++q4) {
            float4 pr[kGroup];
#pragma unroll
            for (int hh = 0; hh < kGroup; ++hh)
                pr[hh] = *reinterpret_cast<const float4*>(probs + hh * kStageTokens + 4 * q4);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int tt = 4 * q4 + u;
                const float2 vv = *reinterpret_cast<const float2*>(vst + tt * kKvWidth);
                float v0 = vv.x, v1 = vv.y;
                if (!full_stage && tt >= d.n_valid) v0 = v1 = 0.f;
#pragma unroll
                for (int hh = 0; hh < kGroup; ++hh) {
                    const float pv = u == 0 ? pr[hh].x : (u == 1 ? pr[hh].y : (u == 2 ? pr[hh].z : pr[hh].w));
                    fma2(acc[hh][0], acc[hh][1], pv, pv, v0, v1);
                }
            }
        }
        __syncwarp();  // every lane is done with the stage and the scratch row
        if (lane == 0) mbar_arrive(&empty[buf]);
        ++g;
        if (!(d.flags & kLast)) continue;

        // ---- slice finished: output, or partial + merge for (row, kv head)
        const int row = d.row;
        const int splits = p.row_splits[row];
        const int nx = p.row_nx ? p.row_nx[row] : 0;
        if (splits == 1 && nx == 0) {
#pragma unroll
            for (int hh = 0; hh < kGroup; ++hh) {
                const float l = __shfl_sync(0xffffffffu, l_run, hh);
                const size_t o = size_t(row) * p.out_stride + (kh * kGroup + hh) * kHeadDim;
                write_out2(p, o + 2 * lane, acc[hh][0] / l, acc[hh][1] / l);
            }
            continue;
        }
#pragma unroll
        for (int hh = 0; hh < kGroup; ++hh) {
            float* part = p.partial + (size_t(d.work) * kHeads + kh * kGroup + hh) * (kHeadDim + 2);
            part[2 + 2 * lane] = acc[hh][0];
            part[3 + 2 * lane] = acc[hh][1];
        }
        if (lane < kGroup) {  // lane hh (t = 0, c = hh) holds head hh's max and sum
            float* part = p.partial + (size_t(d.work) * kHeads + kh * kGroup + lane) * (kHeadDim + 2);
            part[0] = m_run;
            part[1] = l_run;
        }
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        unsigned* counter = p.counters + size_t(row) * kKvHeads + kh;
        if (lane == 0) prev = atomicAdd(counter, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != unsigned(splits - 1)) continue;
        __threadfence();
        // last slice of (row, kv head): merge the shared-prefix slots, then all
        // slices, in that fixed order. The loads of a batch of slots are issued
        // together (the sums still run slot by slot, in order), so the merge costs a
        // few round trips to L2 rather than one per slot, head and value.
        const int w0 = p.row_work0[row];
        const int x0 = nx ? p.row_x0[row] : 0;
        const int ns = nx + splits;
        auto slot_part = [&](int k, int hh) {
            const int sl = k < nx ? x0 + k : w0 + (k - nx);
            return p.partial + (size_t(sl) * kHeads + kh * kGroup + hh) * (kHeadDim + 2);
        };
        float mx[kGroup] = {-INFINITY, -INFINITY, -INFINITY};
        for (int k0 = 0; k0 < ns; k0 += 8) {
            float mv[8][kGroup];
#pragma unroll
            for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int hh = 0; hh < kGroup; ++hh) mv[u][hh] = k0 + u < ns ? __ldcg(slot_part(k0 + u, hh)) : -INFINITY;
#pragma unroll
            for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int hh = 0; hh < kGroup; ++hh) mx[hh] = fmaxf(mx[hh], mv[u][hh]);
        }
        float n0[kGroup] = {0.f, 0.f, 0.f}, n1[kGroup] = {0.f, 0.f, 0.f}, den[kGroup] = {0.f, 0.f, 0.f};
        for (int k0 = 0; k0 < ns; k0 += 4) {
            float mv[4][kGroup], lv[4][kGroup], d0[4][kGroup], d1[4][kGroup];
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int hh = 0; hh < kGroup; ++hh) {
                    if (k0 + u < ns) {
                        const float* part = slot_part(k0 + u, hh);
                        mv[u][hh] = __ldcg(part);
                        lv[u][hh] = __ldcg(part + 1);
                        d0[u][hh] = __ldcg(part + 2 + lane);
                        d1[u][hh] = __ldcg(part + 2 + lane + 32);
                    }
                }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (k0 + u < ns) {
#pragma unroll
                    for (int hh = 0; hh < kGroup; ++hh) {
                        const float sc = exp2f(mv[u][hh] - mx[hh]);  // maxima are in base-2 units
                        den[hh] = fmaf(lv[u][hh], sc, den[hh]);
                        n0[hh] = fmaf(d0[u][hh], sc, n0[hh]);
                        n1[hh] = fmaf(d1[u][hh], sc, n1[hh]);
                    }
                }
        }
#pragma unroll
        for (int hh = 0; hh < kGroup; ++hh) {
            const size_t o = size_t(row) * p.out_stride + (kh * kGroup + hh) * kHeadDim;
            write_out(p, o + lane, n0[hh] / den[hh]);
            write_out(p, o + lane + 32, n1[hh] / den[hh]);
        }
        if (lane == 0) *counter = 0u;  // ready for the next launch
    }
}

__global__ void __launch_bounds__(kThreads, kAttnCtasPerSm) paged_attention_kernel(const AttnParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float* stages = reinterpret_cast<float*>(smem_raw);
    float* probs = stages + 2 * kStages * kStageFloats;  // [3 consumers][3][16]
    float* qsm = probs + kConsumers * kGroup * kStageTokens;  // [3 consumers][3][64] (kQInSmem)
    StageDesc* desc = reinterpret_cast<StageDesc*>(qsm + kConsumers * kGroup * kHeadDim);
    uint64_t* full = reinterpret_cast<uint64_t*>(desc + kStages);
    uint64_t* empty = full + kStages;
    unsigned* failed = reinterpret_cast<unsigned*>(empty + kStages);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumers);
        }
        *failed = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const bool persistent = p.sched != nullptr && p.cta_items == nullptr;
    // Only shared memory is touched above. The consumers read the queries (the
    // preceding QKV epilogue's output) and so wait for the previous kernel first;
    // the producer waits before its first copy that may not be read early.
    if (warp == kConsumers) {
        producer(p, stages, desc, full, empty, persistent, failed, lane);
    } else {
        pdl_enter();
        consumer(p, stages, desc, full, empty, probs + warp * kGroup * kStageTokens, qsm + warp * kGroup * kHeadDim,
                 failed, warp, lane);
    }
    __syncthreads();
    if (tid == 0 && *failed) raise_error(p.error, kErrTimeout);
    if (persistent && tid == 0 && atomicAdd(&p.sched[1], 1u) == gridDim.x - 1) {
        // the last CTA to leave resets the schedule for the next launch
        p.sched[0] = 0u;
        p.sched[1] = 0u;
    }
}

}  // namespace

cudaError_t configure_attention() {
    return cudaFuncSetAttribute(paged_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmem));
}

cudaError_t launch_paged_attention(const AttnParams& p, cudaStream_t stream) {
    if (p.work_count <= 0) return cudaSuccess;
    // static schedule: one CTA per segment; persistent: one wave of 3 CTAs per SM
    // pulls the work items; else one CTA per item
    const int grid = p.cta_items ? p.cta_count : (p.sched ? std::min(p.work_count, kAttnPersistentCtas) : p.work_count);
    if (grid <= 0) return cudaSuccess;
    return launch_pdl(paged_attention_kernel, dim3(grid), dim3(kThreads), kAttnSmem, stream, p);
}

}  // namespace mpb
