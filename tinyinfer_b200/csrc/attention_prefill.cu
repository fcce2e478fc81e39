// Chunked-prefill paged attention on the tensor cores (sm_100a): many query rows
// of one sequence against its paged context.
//
// Computes the causal GQA attention of the CPU runner
// (miniprefix/src/backend/cpu/llama_runner.cpp:85-93: scores q.k / sqrt(64) over
// the tokens at or before the row's position, softmax, weighted sum of V; kv head
// = head / 3) for a chunk of rows appended at positions start .. start + count - 1,
// sharing every K/V sub-chunk among the 42 rows x 3 heads of one kv group instead
// of re-reading the context per row and head as the reference kernel does
// (miniprefix/src/backend/cuda/llama_runner.cu:33-48).
//
// CTA = (tile of up to 42 query rows, kv head), 4 warps. Query vector v (UMMA row,
// TMEM lane, and the thread that owns it) is row v / 3, head kh * 3 + v % 3;
// vectors 126, 127 and those of rows past the tile are padding. The query block is
// split once into TF32 hi / lo halves as a K-major 128-byte-swizzled UMMA tile.
// Per 64-token sub-chunk i of the context [0, start_of_tile + rows):
//  * S_i = Q K_i^T as 3xTF32 tcgen05.mma (M=128, N=64) into tensor memory:
//    Q_lo K_hi + Q_hi K_lo + Q_hi K_hi per 8-dim step (FP32-level products from TF32
//    tensor cores; the dropped lo.lo term is below 2^-20 relative);
//  * thread = query vector: tcgen05.ld of its 64 scores, the causal mask (token <=
//    the row's position), exact softmax over the sub-chunk in registers (base 2,
//    log2(e) folded into the 1/8 scale), probabilities written as hi / lo A tiles;
//  * O_i = P_i V_i the same way (K = the 64 tokens);
//  * thread = query vector: tcgen05.ld of its 64 outputs, folded into a running
//    (max, sum, output) in registers -- online softmax across sub-chunks; a
//    sub-chunk that masks all of a vector's tokens leaves its state unchanged.
// Pipeline: one thread issues P_i V_i and S_{i+1} back to back (two MMA barriers,
// S and O in separate tensor-memory columns). While the tensor core runs them,
// the threads fold O_i and split sub-chunk i+1's V rows into the V^T tiles (free
// once P_i V_i is done); sub-chunk i+1's K rows were split into the K tiles (free
// once S_i is done) before the issue. The raw K / V rows of sub-chunk i+2 are
// gathered through the block table by 16-byte cp.async once i+1's are split.
// The output (running output / sum) goes out as TF32 hi / lo halves, the O
// projection's A operand. All MMA waits are bounded mbarrier waits; a timeout sets
// the error word and the CTA still releases its tensor memory.
#include "attn_tc.cuh"

namespace mpb {
namespace {

using namespace attn_tc;
constexpr int kThreads = 128;
constexpr int kRows = kPrefillTileRows;  // query rows per CTA
static_assert(kRows * kGroup <= kQ, "a tile's query vectors fit the UMMA M of 128");

__global__ void __launch_bounds__(kThreads, 1) prefill_attention_kernel(const PrefillParams p) {
    pdl_enter();  // before any global memory access
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *qhi = sm + kOffQhi, *qlo = sm + kOffQlo, *phi = sm + kOffPhi, *plo = sm + kOffPlo;
    unsigned char *khi = sm + kOffKhi, *klo = sm + kOffKlo;
    unsigned char *vhi = sm + kOffVhi, *vlo = sm + kOffVlo;
    float* raw_k = reinterpret_cast<float*>(sm + kOffRawK);
    float* raw_v = reinterpret_cast<float*>(sm + kOffRawV);
    int* blk = reinterpret_cast<int*>(sm + kOffBlk);
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + kOffBar);  // S_i complete
    uint64_t* bar_o = bar_s + 1;                                     // P_i V_i complete
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar_o + 1);
    int* failed = reinterpret_cast<int*>(tmem_holder + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    const PrefillWork w = p.work[blockIdx.x];
    const int kh = w.kv_head;
    const int rows = w.rows;          // valid query rows of the tile (1..42)
    const int pos0 = w.position;      // position of the tile's first row
    const int len = pos0 + rows;      // context of the tile's last row
    const int subs = (len + kT - 1) / kT;
    const int32_t* table = p.tables + size_t(w.slot) * p.table_stride;
    auto block_of = [&](int token) {
        return attn_tc::token_block(table, p.table_stride, p.block_tokens, p.max_blocks, token, p.error);
    };
    auto valid_in = [&](int sub) { return min(kT, len - sub * kT); };  // tokens of sub-chunk `sub`
    auto gather = [&](int sub) {
        gather_raw(p.keys, p.values, p.page_stride, p.layer_offset, p.block_tokens, blk, sub * kT, valid_in(sub), kh, raw_k,
                   raw_v, tid, kThreads);
    };

    if (warp == 0) tmem_alloc(tmem_holder, kTmemCols);
    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        *failed = 0;
        fence_barrier_init();
    }
    // sub-chunk 0's gathers first, then the query block while they fly
    if (tid < kT) blk[tid] = tid < len ? block_of(tid) : 0;
    __syncthreads();
    gather(0);
    int next_blk = 0;  // physical block of this thread's token in the next sub-chunk to gather
    if (tid < kT && kT + tid < len) next_blk = block_of(kT + tid);
    {
        // query vector v -> tile row v: 16 float4 per vector; all loads first
        constexpr int kPer = kQ * 16 / kThreads;
        float4 v[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = tid + u * kThreads;
            const int qv = i >> 4, c4 = i & 15;
            v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (qv < rows * kGroup) {
                const int head = kh * kGroup + qv % kGroup;
                v[u] = *reinterpret_cast<const float4*>(p.q + size_t(w.row0 + qv / kGroup) * p.q_stride +
                                                        head * kHeadDim + c4 * 4);
            }
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = tid + u * kThreads;
            const int qv = i >> 4, c4 = i & 15;
            store_split4(qhi + (c4 >> 3) * kQTile, qlo + (c4 >> 3) * kQTile, sw128_offset(qv, c4 & 7), v[u]);
        }
    }
    // prologue: sub-chunk 0's tiles and S_0, then sub-chunk 1's gathers
    cp_async_wait_all();
    __syncthreads();  // sub-chunk 0's raw rows are in shared memory
    split_kv(raw_k, raw_v, valid_in(0), khi, klo, vhi, vlo, tid, kThreads);
    fence_proxy_async_shared();  // generic-proxy tile writes -> tensor-core reads
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tmem_s = tmem, tmem_o = tmem + kT;
    constexpr uint32_t idesc = umma_idesc_tf32<kQ, kT>();
    if (tid == 0) {
        issue_3xtf32(tmem_s, qhi, qlo, kQTile, khi, klo, kKTile, idesc);
        mma_commit(bar_s);
    }
    if (subs > 1) {
        if (tid < kT) blk[tid] = next_blk;
        __syncthreads();
        gather(1);
        next_blk = 0;
        if (tid < kT && 2 * kT + tid < len) next_blk = block_of(2 * kT + tid);
    }

    const int qv = warp * 32 + (tid & 31);  // this thread's query vector = TMEM lane
    const bool live = qv < rows * kGroup;
    const int my_pos = pos0 + qv / kGroup;  // keys at positions <= my_pos are visible
    const uint32_t lane_base = uint32_t(warp * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f, o_run[kHeadDim];
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) o_run[d] = 0.f;
    uint32_t phase_s = 0, phase_o = 0;
    bool ok = true;

    for (int i = 0; i < subs; ++i) {
        const int t0 = i * kT;
        const bool more = i + 1 < subs;
        if (!mbar_wait_bounded(bar_s, phase_s)) *failed = 1;
        phase_s ^= 1;
        tmem_fence_after();
        // scores in base-2 units; the causal mask keeps tokens t0 + j <= my_pos
        // (the TMEM load is warp-collective: every lane executes it)
        float s[kT];
        tmem_row64(tmem_s + lane_base, s);
        const int visible = live ? min(valid_in(i), my_pos - t0 + 1) : 0;  // tokens j < visible
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < kT; ++j) {
            s[j] = j < visible ? s[j] * (0.125f * kLog2e) : -INFINITY;
            mx = fmaxf(mx, s[j]);
        }
        float sum = 0.f;
        const float base = visible > 0 ? mx : 0.f;  // all masked: every weight 0
#pragma unroll
        for (int j = 0; j < kT; ++j) {
            s[j] = j < visible ? exp2f(s[j] - base) : 0.f;
            sum += s[j];
        }
        // P_i as the A operand (rows = query vectors, K = tokens); P_{i-1} V_{i-1}
        // completed in the previous iteration
#pragma unroll
        for (int c4 = 0; c4 < kT / 4; ++c4)
            store_split4(phi + (c4 >> 3) * kQTile, plo + (c4 >> 3) * kQTile, sw128_offset(qv, c4 & 7),
                         make_float4(s[4 * c4], s[4 * c4 + 1], s[4 * c4 + 2], s[4 * c4 + 3]));
        if (more) cp_async_wait_all();  // sub-chunk i+1's raw rows (this thread's copies)
        tmem_fence_before();
        __syncthreads();  // S_i read by every thread; the raw rows of i+1 landed
        if (*failed) {
            ok = false;
            break;
        }
        if (more) split_k(raw_k, valid_in(i + 1), khi, klo, tid, kThreads);  // K tiles: S_i is done
        fence_proxy_async_shared();
        __syncthreads();  // P_i and K_{i+1} tiles complete
        tmem_fence_after();
        if (tid == 0) {
            issue_3xtf32(tmem_o, phi, plo, kQTile, vhi, vlo, kKTile, idesc);
            mma_commit(bar_o);
            if (more) {
                issue_3xtf32(tmem_s, qhi, qlo, kQTile, khi, klo, kKTile, idesc);
                mma_commit(bar_s);
            }
        }
        if (!mbar_wait_bounded(bar_o, phase_o)) *failed = 1;
        phase_o ^= 1;
        tmem_fence_after();
        float o[kT];
        tmem_row64(tmem_o + lane_base, o);  // warp-collective: every lane
        if (visible > 0) {
            // fold this sub-chunk into the running (max, sum, output)
            const float m_new = fmaxf(m_run, mx);
            const float a_old = exp2f(m_run - m_new), a_new = exp2f(mx - m_new);  // m_run = -inf: a_old = 0
            l_run = l_run * a_old + sum * a_new;
            m_run = m_new;
#pragma unroll
            for (int d = 0; d < kHeadDim; ++d) o_run[d] = fmaf(o_run[d], a_old, o[d] * a_new);
        }
        if (more) split_v(raw_v, valid_in(i + 1), vhi, vlo, tid, kThreads);  // V^T tiles: P_i V_i is done
        tmem_fence_before();
        __syncthreads();  // O_i read; the staging buffer is free; V_{i+1} written
        if (*failed) {
            ok = false;
            break;
        }
        if (i + 2 < subs) {
            if (tid < kT) blk[tid] = next_blk;
            __syncthreads();
            gather(i + 2);
            next_blk = 0;
            if (tid < kT && (i + 3) * kT + tid < len) next_blk = block_of((i + 3) * kT + tid);
        }
    }
    cp_async_wait_all();  // nothing may still land in shared memory after the CTA ends

    if (ok && live) {
        const int r = qv / kGroup, head = kh * kGroup + qv % kGroup;
        const size_t at = size_t(w.row0 + r) * p.out_stride + head * kHeadDim;
        const float inv = 1.0f / l_run;
#pragma unroll
        for (int c4 = 0; c4 < kHeadDim / 4; ++c4) {
            const float4 val = make_float4(o_run[4 * c4] * inv, o_run[4 * c4 + 1] * inv, o_run[4 * c4 + 2] * inv,
                                           o_run[4 * c4 + 3] * inv);
            if (p.out_hi) {
                store_split4(p.out_hi + at + 4 * c4, p.out_lo + at + 4 * c4, val);
            } else {
                *reinterpret_cast<float4*>(p.out + at + 4 * c4) = val;
            }
        }
    }
    if (!ok && tid == 0) raise_error(p.error, kErrTimeout);
    tmem_fence_before();
    __syncthreads();
    if (warp == 0) {
        tmem_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

cudaError_t configure_prefill_attention() {
    return cudaFuncSetAttribute(prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem));
}

cudaError_t launch_prefill_attention(const PrefillParams& p, cudaStream_t stream) {
    if (p.work_count <= 0) return cudaSuccess;
    return launch_pdl(prefill_attention_kernel, dim3(p.work_count), dim3(kThreads), kSmem, stream, p);
}

}  // namespace mpb
