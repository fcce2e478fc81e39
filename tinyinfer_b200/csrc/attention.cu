// Paged attention over the MiniPrefix K/V page pools (sm_100a).
//
// Replaces the reference's attention_kernel (miniprefix/src/backend/cuda/
// llama_runner.cu:33-48: one block per (row, q head), one token per iteration,
// eight __syncthreads per token, each K/V row fetched once per q head) and
// computes the CPU runner's attention (miniprefix/src/backend/cpu/
// llama_runner.cpp:85-93): causal GQA, kv head = h / 3, scale 1/sqrt(64), softmax.
//
// Design (one query row, all 9 heads, per CTA; split-K over pages):
//  * A CTA owns one slice [page_begin, page_end) of one query row's context. A row
//    with more than one slice, or with shared-prefix partials computed earlier on
//    the stream by attention_shared.cu, is merged by the last slice to finish
//    (arrival counter per row), so one launch produces the final output.
//  * K and V of 16 consecutive tokens form one stage. Runs of tokens that are
//    contiguous inside a page (a page is [slot][192] floats for one layer) are
//    moved by the bulk-copy engine (cp.async.bulk) into shared memory and
//    complete on a per-stage mbarrier, so 2 stages stay in flight while one is
//    consumed. Each K/V byte is read from HBM once for all 3 q heads of its group.
//    192 threads and ~75 KB of shared memory let 3 CTAs share an SM.
//  * Scores: 48 (token, kv head) pairs x 4 lanes; each lane keeps its 3 heads'
//    16 query values in registers and dots one 64-byte quarter of the key row,
//    quarters rotated by pair parity so the 8 lanes of a 128-bit phase hit
//    distinct banks. Softmax: 16 lanes per head, online (running max / sum).
//    P.V: one (kv head, dim) column per thread, 3 heads.
//  * Tokens past the row length are masked by select (never by multiplying), so
//    stale or uninitialised shared memory cannot leak NaN into the result.
#include "common.cuh"
#include "kernels.h"

namespace mpb {
namespace {

constexpr int kStageTokens = 16;
constexpr int kThreads = 192;  // 48 (token, kv head) pairs x 4 lanes; 192 (kv head, dim) columns
constexpr int kStages = 3;
constexpr int kStageFloats = kStageTokens * kKvWidth;  // per pool
constexpr size_t kAttnSmem = size_t(kStages) * 2 * kStageFloats * sizeof(float) +
                             2 * kHeads * kStageTokens * sizeof(float) + 4 * kHeads * sizeof(float) +
                             kStages * sizeof(uint64_t) + 16;

struct Shared {
    float* stages;  // stage i: K at stages + 2*i*kStageFloats, V right after
    float* scores;  // [9][16]
    float* probs;   // [9][16]
    float* alpha;   // [9]
    float* m;       // [9]
    float* l;       // [9]
    int* flag;      // [1] error / last-arriver broadcast
    uint64_t* bar;  // [kStages]
};

// Output element: plain FP32, or TF32 hi/lo halves when the caller asked for them.
__device__ __forceinline__ void write_out(const AttnParams& p, size_t i, float v) {
    if (p.out_lo) {
        float h, l;
        split_tf32(v, h, l);
        p.out[i] = h;
        p.out_lo[i] = l;
    } else {
        p.out[i] = v;
    }
}

// Issue the copies for context tokens [a, b) into stage buffers (warp 0 only).
__device__ __forceinline__ void issue_stage(const AttnParams& p, const int32_t* table, int a, int b, float* kdst,
                                            float* vdst, uint64_t* bar, int lane) {
    const int bt = p.block_tokens;
    const int first_page = a / bt;
    const int run_begin = max(a, (first_page + lane) * bt);
    const int run_end = min(b, (first_page + lane + 1) * bt);
    if (lane == 0) mbar_arrive_expect_tx(bar, uint32_t(b - a) * 2u * kKvWidth * sizeof(float));
    __syncwarp();
    if (run_begin < run_end) {
        const int page = first_page + lane;
        int block = page < p.table_stride ? table[page] : -1;
        if (block < 0 || block >= p.max_blocks) {
            raise_error(p.error, kErrBounds);
            block = 0;  // stay in bounds; the error word fails the step
        }
        const size_t src = ((size_t(block) * p.layers + p.layer) * bt + (run_begin - page * bt)) * kKvWidth;
        const uint32_t bytes = uint32_t(run_end - run_begin) * kKvWidth * sizeof(float);
        bulk_copy_g2s(kdst + (run_begin - a) * kKvWidth, p.keys + src, bytes, bar);
        bulk_copy_g2s(vdst + (run_begin - a) * kKvWidth, p.values + src, bytes, bar);
    }
}

__global__ void __launch_bounds__(kThreads, 3) paged_attention_kernel(const AttnParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Shared s;
    {
        float* f = reinterpret_cast<float*>(smem_raw);
        s.stages = f;
        f += 2 * kStages * kStageFloats;
        s.scores = f; f += kHeads * kStageTokens;
        s.probs = f; f += kHeads * kStageTokens;
        s.alpha = f; f += kHeads;
        s.m = f; f += kHeads;
        s.l = f; f += kHeads;
        s.flag = reinterpret_cast<int*>(f); f += kHeads;
        s.bar = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(f) + 7) & ~uintptr_t(7));
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const AttnWork w = p.work[blockIdx.x];
    const int row = w.row;
    const int len = p.row_len[row];
    const int32_t* table = p.tables + size_t(p.row_slot[row]) * p.table_stride;
    const int tok_begin = w.page_begin * p.block_tokens;
    const int tok_end = min(w.page_end * p.block_tokens, len);
    const int n_stages = tok_end > tok_begin ? (tok_end - tok_begin + kStageTokens - 1) / kStageTokens : 0;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&s.bar[i], 1);
        s.flag[0] = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (warp == 0)
        for (int i = 0; i < kStages && i < n_stages; ++i) {
            const int a = tok_begin + i * kStageTokens;
            issue_stage(p, table, a, min(a + kStageTokens, tok_end), s.stages + 2 * i * kStageFloats,
                        s.stages + (2 * i + 1) * kStageFloats, &s.bar[i], lane);
        }

    // Score identity: pair = (token st, kv head skh), 4 lanes per pair; each lane
    // holds its kv group's 3 heads x 16 query values (4 of the 16 float4 chunks of
    // a 64-dim row, rotated by pair parity so a 128-bit phase hits distinct banks).
    const int pair = tid >> 2, sub = tid & 3;
    const int st = pair / kKvHeads, skh = pair % kKvHeads, rot = pair & 1;
    float4 qr[kGroup][4];
    {
        const float* qrow = p.q + size_t(row) * p.q_stride;
#pragma unroll
        for (int hh = 0; hh < kGroup; ++hh)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int chunk = sub + 4 * ((j + rot) & 3);
                qr[hh][j] = *reinterpret_cast<const float4*>(qrow + (skh * kGroup + hh) * kHeadDim + 4 * chunk);
            }
    }
    // Softmax identity: 16 lanes per head (two heads per warp, warps 0..4).
    const int shead = warp * 2 + (lane >> 4), stok = lane & 15;
    // P.V identity: one (kv head, dim) column per thread, 3 heads.
    const int pkh = tid / kHeadDim;
    float acc[kGroup] = {0.f, 0.f, 0.f};
    float m_run = -INFINITY, l_run = 0.f;  // of head `shead`

    for (int i = 0; i < n_stages; ++i) {
        const int stage = i % kStages;
        const int a = tok_begin + i * kStageTokens;
        const int n_valid = min(kStageTokens, tok_end - a);
        if (!mbar_wait_bounded(&s.bar[stage], (i / kStages) & 1)) s.flag[0] = 1;
        {
            const float* krow = s.stages + 2 * stage * kStageFloats + st * kKvWidth + skh * kHeadDim;
            float part[kGroup] = {0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int chunk = sub + 4 * ((j + rot) & 3);
                const float4 kv = *reinterpret_cast<const float4*>(krow + 4 * chunk);
#pragma unroll
                for (int hh = 0; hh < kGroup; ++hh) {
                    part[hh] = fmaf(qr[hh][j].x, kv.x, part[hh]);
                    part[hh] = fmaf(qr[hh][j].y, kv.y, part[hh]);
                    part[hh] = fmaf(qr[hh][j].z, kv.z, part[hh]);
                    part[hh] = fmaf(qr[hh][j].w, kv.w, part[hh]);
                }
            }
#pragma unroll
            for (int hh = 0; hh < kGroup; ++hh) {
                part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], 1);
                part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], 2);
            }
            if (sub < kGroup) {
                const float sc = sub == 0 ? part[0] : (sub == 1 ? part[1] : part[2]);
                s.scores[(skh * kGroup + sub) * kStageTokens + st] = st < n_valid ? sc * 0.125f : -INFINITY;
            }
        }
        __syncthreads();
        if (s.flag[0]) break;
        if (warp < 5) {
            // all 32 lanes take part in the shuffles; heads >= 9 use a dummy row
            const bool live = shead < kHeads;
            const float sc = live ? s.scores[shead * kStageTokens + stok] : -INFINITY;
            float mx = sc;
#pragma unroll
            for (int o = 8; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_new = fmaxf(m_run, mx);
            const float alpha = live ? expf(m_run - m_new) : 0.f;
            const float pr = live ? expf(sc - m_new) : 0.f;
            float sum = pr;
#pragma unroll
            for (int o = 8; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (live) {
                l_run = l_run * alpha + sum;
                m_run = m_new;
                s.probs[shead * kStageTokens + stok] = pr;
                if (stok == 0) s.alpha[shead] = alpha;
            }
        }
        __syncthreads();
        {
            const float* vbase = s.stages + (2 * stage + 1) * kStageFloats + tid;
            const float* pb = s.probs + (pkh * kGroup) * kStageTokens;
#pragma unroll
            for (int hh = 0; hh < kGroup; ++hh) acc[hh] *= s.alpha[pkh * kGroup + hh];
#pragma unroll
            for (int t = 0; t < kStageTokens; ++t) {
                const float v = t < n_valid ? vbase[t * kKvWidth] : 0.f;
#pragma unroll
                for (int hh = 0; hh < kGroup; ++hh) acc[hh] = fmaf(pb[hh * kStageTokens + t], v, acc[hh]);
            }
        }
        __syncthreads();
        if (warp == 0 && i + kStages < n_stages) {
            fence_proxy_async_shared();
            const int a2 = tok_begin + (i + kStages) * kStageTokens;
            issue_stage(p, table, a2, min(a2 + kStageTokens, tok_end), s.stages + 2 * stage * kStageFloats,
                        s.stages + (2 * stage + 1) * kStageFloats, &s.bar[stage], lane);
        }
    }
    if (s.flag[0]) {
        if (tid == 0) raise_error(p.error, kErrTimeout);
        return;
    }
    if (warp < 5 && stok == 0 && shead < kHeads) {
        s.m[shead] = m_run;
        s.l[shead] = l_run;
    }
    __syncthreads();
    const int splits = p.row_splits[row];
    // shared-prefix partials of this row (written by the prefix kernel earlier on
    // the same stream) join the merge as extra slots
    const int nx = p.row_nx ? p.row_nx[row] : 0;
    const bool direct = splits == 1 && nx == 0;
    {
        const int d = tid % kHeadDim;
#pragma unroll
        for (int hh = 0; hh < kGroup; ++hh) {
            const int h = pkh * kGroup + hh;
            if (direct) {
                write_out(p, size_t(row) * p.out_stride + h * kHeadDim + d, acc[hh] / s.l[h]);
            } else {
                float* part = p.partial + (size_t(blockIdx.x) * kHeads + h) * (kHeadDim + 2);
                part[2 + d] = acc[hh];
                if (d == 0) {
                    part[0] = s.m[h];
                    part[1] = s.l[h];
                }
            }
        }
    }
    if (direct) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(&p.counters[row], 1u);
        s.flag[0] = prev == unsigned(splits - 1) ? 2 : 0;
    }
    __syncthreads();
    if (s.flag[0] != 2) return;
    __threadfence();
    // Last slice of this row: merge the shared-prefix slots, then all slices'
    // (m, l, acc), in that fixed order.
    const int w0 = p.row_work0[row];
    const int x0 = nx ? p.row_x0[row] : 0;
    auto slot = [&](int k) { return k < nx ? x0 + k : w0 + (k - nx); };
    for (int o = tid; o < kHeads * kHeadDim; o += kThreads) {
        const int h = o / kHeadDim, d = o % kHeadDim;
        float mx = -INFINITY;
        for (int k = 0; k < nx + splits; ++k)
            mx = fmaxf(mx, __ldcg(p.partial + (size_t(slot(k)) * kHeads + h) * (kHeadDim + 2)));
        float num = 0.f, den = 0.f;
        for (int k = 0; k < nx + splits; ++k) {
            const float* part = p.partial + (size_t(slot(k)) * kHeads + h) * (kHeadDim + 2);
            const float sc = expf(__ldcg(part) - mx);
            den = fmaf(__ldcg(part + 1), sc, den);
            num = fmaf(__ldcg(part + 2 + d), sc, num);
        }
        write_out(p, size_t(row) * p.out_stride + o, num / den);
    }
    if (tid == 0) p.counters[row] = 0u;  // ready for the next launch
}

}  // namespace

cudaError_t configure_attention() {
    return cudaFuncSetAttribute(paged_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmem));
}

cudaError_t launch_paged_attention(const AttnParams& p, cudaStream_t stream) {
    if (p.work_count <= 0) return cudaSuccess;
    paged_attention_kernel<<<p.work_count, kThreads, kAttnSmem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mpb
