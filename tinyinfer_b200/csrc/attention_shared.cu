// Shared-prefix decode attention on the tensor cores (sm_100a): the pages that a
// group of decode rows share are read once per launch for the whole group.
//
// Decode attention is bandwidth-bound when every row streams its whole context
// (miniprefix/src/backend/cuda/llama_runner.cu:33-48 reads it once per row and
// head). Rows that reuse a cached prefix (miniprefix/src/kv/prefix_cache.cpp) map
// the same physical pages at the start of their block tables, so the host groups
// such rows and this kernel computes their attention over the shared tokens as a
// dense problem per (group, kv head): Q[rows x 3 heads][64] against
// K/V[shared tokens][64] -- softmax(Q K^T / 8) V as the CPU runner computes it
// (miniprefix/src/backend/cpu/llama_runner.cpp:85-93), restricted to those tokens.
// Each CTA writes, per query vector, the maximum, the sum of exponentials and the
// unnormalised output of its token chunk -- the decode kernel's partial format
// (base-2 units) -- and the decode kernel's merge combines them with the rows'
// own pages (attention.cu).
//
// CTA = (group, kv head, 128 query vectors, token chunk), 4 warps. The query block
// is split once into TF32 hi / lo halves and written as K-major 128-byte-swizzled
// UMMA tiles. Per 64-token sub-chunk:
//  * the raw K and V rows were gathered through the group's block table by 16-byte
//    cp.async into a staging buffer while the previous sub-chunk computed; all
//    threads split them into hi / lo K (64 tokens x 64 dims) and V^T (64 dims x 64
//    tokens) tiles, then start the next sub-chunk's gathers;
//  * one thread issues S = Q K^T as 3xTF32 tcgen05.mma (M=128, N=64: Q_lo K_hi +
//    Q_hi K_lo + Q_hi K_hi per 8-dim step) into tensor memory;
//  * thread = query row: tcgen05.ld of its 64 scores, exact softmax over the
//    sub-chunk in registers (no shuffles), probabilities written as hi/lo A tiles;
//  * one thread issues O = P V the same way (K = the 64 tokens);
//  * thread = query row: tcgen05.ld of its 64 outputs, folded into a running
//    (max, sum, output) in registers -- online softmax across sub-chunks.
// All MMA waits are bounded mbarrier waits; a timeout sets the error word.
#include "attn_tc.cuh"

namespace mpb {
namespace {

using namespace attn_tc;
constexpr int kPQ = kPrefixQueries;  // 128 query vectors = UMMA M
static_assert(kPQ == attn_tc::kQ, "query block of the tensor-core attention tiles");
constexpr int kPT = attn_tc::kT;     // tokens per sub-chunk
constexpr int kPThreads = 128;
constexpr size_t kPrefixSmem = attn_tc::kSmem;

// Query block: qv = row_in_group * 3 + head_in_group -> tile row, hi/lo halves.
// All 16 loads of a thread are issued before any is split and stored.
__device__ __forceinline__ void load_queries(const PrefixParams& p, const PrefixWork& w, const int32_t* rows,
                                             unsigned char* qhi, unsigned char* qlo, int tid) {
    constexpr int kPer = kPQ * 16 / kPThreads;  // 16
    float4 v[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int i = tid + u * kPThreads;
        const int qi = i >> 4, c4 = i & 15;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < w.q_count) {
            const int qv = w.q_begin + qi;
            const int row = rows[qv / kGroup];
            const int head = w.kv_head * kGroup + qv % kGroup;
            v[u] = *reinterpret_cast<const float4*>(p.q + size_t(row) * p.q_stride + head * kHeadDim + c4 * 4);
        }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int i = tid + u * kPThreads;
        const int qi = i >> 4, c4 = i & 15;
        store_split4(qhi + (c4 >> 3) * kQTile, qlo + (c4 >> 3) * kQTile, sw128_offset(qi, c4 & 7), v[u]);
    }
}

// Physical block of shared token `token`, bounds-checked.
__device__ __forceinline__ int token_block(const PrefixParams& p, const int32_t* table, int token) {
    return attn_tc::token_block(table, p.table_stride, p.block_tokens, p.max_blocks, token, p.error);
}

__global__ void __launch_bounds__(kPThreads, 1) prefix_attention_kernel(const PrefixParams p) {
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
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 1);
    int* failed = reinterpret_cast<int*>(tmem_holder + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    const PrefixWork w = p.work[blockIdx.x];
    const int32_t* rows = p.group_rows + p.group_row0[w.group];
    const int32_t* table = p.tables + size_t(p.group_slot[w.group]) * p.table_stride;
    const int kh = w.kv_head;

    if (warp == 0) tmem_alloc(tmem_holder, kTmemCols);
    if (tid == 0) {
        mbar_init(bar, 1);
        *failed = 0;
        fence_barrier_init();
    }
    // sub-chunk 0's gathers first, then the query block while they fly
    if (tid < kPT) blk[tid] = w.tok_begin + tid < w.tok_end ? token_block(p, table, w.tok_begin + tid) : 0;
    __syncthreads();
    gather_raw(p.keys, p.values, p.page_stride, p.layer_offset, p.block_tokens, blk, w.tok_begin,
               min(kPT, w.tok_end - w.tok_begin), kh, raw_k, raw_v, tid, kPThreads);
    // physical block of this thread's token in the next sub-chunk, fetched early
    int next_blk = 0;
    if (tid < kPT && w.tok_begin + kPT + tid < w.tok_end) next_blk = token_block(p, table, w.tok_begin + kPT + tid);
    load_queries(p, w, rows, qhi, qlo, tid);
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tmem_s = tmem, tmem_o = tmem + kPT;
    constexpr uint32_t idesc = umma_idesc_tf32<kPQ, kPT>();

    const int qrow = warp * 32 + (tid & 31);  // TMEM lane = query row of this thread
    const uint32_t lane_base = uint32_t(warp * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f, o_run[kHeadDim];
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) o_run[d] = 0.f;
    uint32_t phase = 0;
    bool ok = true;

    for (int t0 = w.tok_begin; t0 < w.tok_end; t0 += kPT) {
        const int n_valid = min(kPT, w.tok_end - t0);
        cp_async_wait_all();
        __syncthreads();  // this sub-chunk's raw rows are in shared memory
        // split into hi / lo K rows (token-major) and V^T (dim-major); tokens past
        // the sub-chunk are zero
        split_kv(raw_k, raw_v, n_valid, khi, klo, vhi, vlo, tid, kPThreads);
        fence_proxy_async_shared();  // generic-proxy tile writes -> tensor-core reads
        tmem_fence_before();
        __syncthreads();  // split tiles complete; the staging buffer is free
        tmem_fence_after();
        if (tid == 0) {
            issue_3xtf32(tmem_s, qhi, qlo, kQTile, khi, klo, kKTile, idesc);
            mma_commit(bar);
        }
        // the next sub-chunk's gathers overlap this one's products
        const int t1 = t0 + kPT;
        if (t1 < w.tok_end) {
            if (tid < kPT) blk[tid] = next_blk;
            __syncthreads();
            gather_raw(p.keys, p.values, p.page_stride, p.layer_offset, p.block_tokens, blk, t1, min(kPT, w.tok_end - t1), kh,
                       raw_k, raw_v, tid, kPThreads);
            next_blk = 0;
            if (tid < kPT && t1 + kPT + tid < w.tok_end) next_blk = token_block(p, table, t1 + kPT + tid);
        }
        if (!mbar_wait_bounded(bar, phase)) *failed = 1;
        phase ^= 1;
        __syncthreads();
        if (*failed) {
            ok = false;
            break;
        }
        tmem_fence_after();
        // scores of this thread's query row, base-2 units; exact softmax over the sub-chunk
        float s[kPT];
        {
            uint32_t r[32];
            tmem_load32(tmem_s + lane_base, r);
#pragma unroll
            for (int j = 0; j < 32; ++j) s[j] = __uint_as_float(r[j]);
            tmem_load32(tmem_s + lane_base + 32, r);
#pragma unroll
            for (int j = 0; j < 32; ++j) s[32 + j] = __uint_as_float(r[j]);
        }
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < kPT; ++j) {
            s[j] = j < n_valid ? s[j] * (0.125f * kLog2e) : -INFINITY;
            mx = fmaxf(mx, s[j]);
        }
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < kPT; ++j) {
            s[j] = exp2f(s[j] - mx);
            sum += s[j];
        }
        // P as the A operand (rows = query vectors, K = tokens)
#pragma unroll
        for (int c4 = 0; c4 < kPT / 4; ++c4)
            store_split4(phi + (c4 >> 3) * kQTile, plo + (c4 >> 3) * kQTile, sw128_offset(qrow, c4 & 7),
                         make_float4(s[4 * c4], s[4 * c4 + 1], s[4 * c4 + 2], s[4 * c4 + 3]));
        fence_proxy_async_shared();
        tmem_fence_before();
        __syncthreads();
        tmem_fence_after();
        if (tid == 0) {
            issue_3xtf32(tmem_o, phi, plo, kQTile, vhi, vlo, kKTile, idesc);
            mma_commit(bar);
        }
        if (!mbar_wait_bounded(bar, phase)) *failed = 1;
        phase ^= 1;
        __syncthreads();
        if (*failed) {
            ok = false;
            break;
        }
        tmem_fence_after();
        // fold this sub-chunk into the running (max, sum, output)
        {
            const float m_new = fmaxf(m_run, mx);
            const float a_old = exp2f(m_run - m_new), a_new = exp2f(mx - m_new);
            l_run = l_run * a_old + sum * a_new;
            m_run = m_new;
            uint32_t r[32];
            tmem_load32(tmem_o + lane_base, r);
#pragma unroll
            for (int j = 0; j < 32; ++j) o_run[j] = fmaf(o_run[j], a_old, __uint_as_float(r[j]) * a_new);
            tmem_load32(tmem_o + lane_base + 32, r);
#pragma unroll
            for (int j = 0; j < 32; ++j) o_run[32 + j] = fmaf(o_run[32 + j], a_old, __uint_as_float(r[j]) * a_new);
        }
        tmem_fence_before();
    }
    cp_async_wait_all();  // nothing may still land in shared memory after the CTA ends

    if (ok && qrow < w.q_count) {
        const int qv = w.q_begin + qrow;
        const int row = rows[qv / kGroup];
        const int head = kh * kGroup + qv % kGroup;
        float* part = p.partial + (size_t(p.row_x0[row] + w.chunk) * kHeads + head) * (kHeadDim + 2);
        part[0] = m_run;
        part[1] = l_run;
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) part[2 + d] = o_run[d];
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

cudaError_t configure_prefix_attention() {
    return cudaFuncSetAttribute(prefix_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kPrefixSmem));
}

cudaError_t launch_prefix_attention(const PrefixParams& p, cudaStream_t stream) {
    if (p.work_count <= 0) return cudaSuccess;
    return launch_pdl(prefix_attention_kernel, dim3(p.work_count), dim3(kPThreads), kPrefixSmem, stream, p);
}

}  // namespace mpb
