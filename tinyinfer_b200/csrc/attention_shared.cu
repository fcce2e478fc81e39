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
// CTA = (group, kv head, 128 query vectors, token chunk), 4 warps. Per 64-token
// sub-chunk:
//  * all threads gather K and V rows through the group's block table, split them
//    into TF32 hi / lo halves and write K (64 tokens x 64 dims) and V^T (64 dims x
//    64 tokens) as K-major 128-byte-swizzled UMMA tiles (the query block is
//    written the same way);
//  * one thread issues S = Q K^T as 3xTF32 tcgen05.mma (M=128, N=64: Q_lo K_hi +
//    Q_hi K_lo + Q_hi K_hi per 8-dim step) into tensor memory;
//  * thread = query row: tcgen05.ld of its 64 scores, exact softmax over the
//    sub-chunk in registers (no shuffles), probabilities written as hi/lo A tiles;
//  * one thread issues O = P V the same way (K = the 64 tokens);
//  * thread = query row: tcgen05.ld of its 64 outputs, folded into a running
//    (max, sum, output) in registers -- online softmax across sub-chunks.
// All MMA waits are bounded mbarrier waits; a timeout sets the error word.
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace mpb {
namespace {

constexpr int kPQ = kPrefixQueries;  // 128 query vectors = UMMA M
constexpr int kPT = 64;              // tokens per sub-chunk = UMMA N of S, K of P.V
constexpr int kPThreads = 128;
constexpr int kQTile = kPQ * 32 * 4;   // one 32-element K block of a 128-row tile (16 KB)
constexpr int kKTile = kPT * 32 * 4;   // one K block of a 64-row tile (8 KB)
// shared memory (1024-aligned tiles): Q/P hi, Q/P lo (2 K blocks each), K hi, K lo,
// V^T hi, V^T lo (2 K blocks each), then the barrier and the TMEM address
constexpr int kOffQhi = 0, kOffQlo = 2 * kQTile;
constexpr int kOffKhi = 4 * kQTile, kOffKlo = kOffKhi + 2 * kKTile;
constexpr int kOffVhi = kOffKlo + 2 * kKTile, kOffVlo = kOffVhi + 2 * kKTile;
constexpr int kOffBlk = kOffVlo + 2 * kKTile;  // [64] physical blocks of the sub-chunk's tokens
constexpr int kOffBar = kOffBlk + kPT * 4;
constexpr size_t kPrefixSmem = size_t(kOffBar) + 64 + 1024 /*alignment slack*/;
constexpr uint32_t kTmemCols = 128;  // S: columns 0..63, O: 64..127

__device__ __forceinline__ void store_split4(unsigned char* hi_tile, unsigned char* lo_tile, uint32_t off,
                                             float4 v) {
    float4 h, l;
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
    *reinterpret_cast<float4*>(hi_tile + off) = h;
    *reinterpret_cast<float4*>(lo_tile + off) = l;
}

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

// Float offset of the K/V row of token t0 + t (kv head kh) in either pool, from the
// sub-chunk's staged physical block ids (blk[t]).
__device__ __forceinline__ size_t kv_offset(const PrefixParams& p, const int* blk, int t0, int t, int kh) {
    const int token = t0 + t;
    return ((size_t(blk[t]) * p.layers + p.layer) * p.block_tokens + token % p.block_tokens) * kKvWidth +
           kh * kHeadDim;
}

// 3xTF32 product over 2 K blocks of 32: D = A_lo B_hi + A_hi B_lo + A_hi B_hi.
__device__ __forceinline__ void issue_3xtf32(uint32_t tmem_d, const unsigned char* a_hi, const unsigned char* a_lo,
                                             int a_block_bytes, const unsigned char* b_hi, const unsigned char* b_lo,
                                             int b_block_bytes, uint32_t idesc) {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
        const uint64_t ah = smem_desc(a_hi + kb * a_block_bytes), al = smem_desc(a_lo + kb * a_block_bytes);
        const uint64_t bh = smem_desc(b_hi + kb * b_block_bytes), bl = smem_desc(b_lo + kb * b_block_bytes);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint64_t step = uint64_t(j * 32) >> 4;  // 8 tf32 = 32 bytes along the swizzled row
            mma_tf32(tmem_d, al + step, bh + step, idesc, (kb | j) != 0);
            mma_tf32(tmem_d, ah + step, bl + step, idesc, 1);
            mma_tf32(tmem_d, ah + step, bh + step, idesc, 1);
        }
    }
}

__global__ void __launch_bounds__(kPThreads, 1) prefix_attention_kernel(const PrefixParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *qhi = sm + kOffQhi, *qlo = sm + kOffQlo;
    unsigned char *khi = sm + kOffKhi, *klo = sm + kOffKlo;
    unsigned char *vhi = sm + kOffVhi, *vlo = sm + kOffVlo;
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
        // physical block of each token of the sub-chunk, looked up once
        if (tid < kPT) {
            int block = 0;
            if (tid < n_valid) {
                const int page = (t0 + tid) / p.block_tokens;
                block = page < p.table_stride ? table[page] : -1;
                if (block < 0 || block >= p.max_blocks) {
                    raise_error(p.error, kErrBounds);
                    block = 0;  // stay in bounds; the error word fails the step
                }
            }
            blk[tid] = block;
        }
        __syncthreads();
        // K rows (token-major) and V^T (dim-major), hi / lo; tokens past the chunk are
        // zero. Every load of a thread is issued before any store. K: consecutive
        // threads walk one token's dims (coalesced); V: consecutive threads walk
        // tokens, so a warp's transposed stores (one dim row, 32 tokens) hit 32
        // distinct banks.
        {
            constexpr int kPer = kPT * 16 / kPThreads;  // 8
            float4 kv[kPer], vv[kPer];
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int i = tid + u * kPThreads;
                const int tk = i >> 4, ck = i & 15;
                const int tv = i & (kPT - 1), cv = i / kPT;
                kv[u] = tk < n_valid ? *reinterpret_cast<const float4*>(p.keys + kv_offset(p, blk, t0, tk, kh) + ck * 4)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                vv[u] = tv < n_valid
                            ? *reinterpret_cast<const float4*>(p.values + kv_offset(p, blk, t0, tv, kh) + cv * 4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int i = tid + u * kPThreads;
                const int tk = i >> 4, ck = i & 15;
                store_split4(khi + (ck >> 3) * kKTile, klo + (ck >> 3) * kKTile, sw128_offset(tk, ck & 7), kv[u]);
                const int tv = i & (kPT - 1), cv = i / kPT;
                const float ve[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int d = 4 * cv + e;  // V^T row; column = token tv (K block tv / 32)
                    const uint32_t off = sw128_offset(d, (tv & 31) >> 2) + uint32_t(tv & 3) * 4;
                    float h, l;
                    split_tf32(ve[e], h, l);
                    *reinterpret_cast<float*>(vhi + (tv >> 5) * kKTile + off) = h;
                    *reinterpret_cast<float*>(vlo + (tv >> 5) * kKTile + off) = l;
                }
            }
        }
        fence_proxy_async_shared();  // generic-proxy tile writes -> tensor-core reads
        tmem_fence_before();
        __syncthreads();
        tmem_fence_after();
        if (tid == 0) {
            issue_3xtf32(tmem_s, qhi, qlo, kQTile, khi, klo, kKTile, idesc);
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
        // P as the A operand (rows = query vectors, K = tokens), written over the
        // query tiles now that S is complete; they are reloaded for a next sub-chunk
#pragma unroll
        for (int c4 = 0; c4 < kPT / 4; ++c4)
            store_split4(qhi + (c4 >> 3) * kQTile, qlo + (c4 >> 3) * kQTile, sw128_offset(qrow, c4 & 7),
                         make_float4(s[4 * c4], s[4 * c4 + 1], s[4 * c4 + 2], s[4 * c4 + 3]));
        fence_proxy_async_shared();
        tmem_fence_before();
        __syncthreads();
        tmem_fence_after();
        if (tid == 0) {
            issue_3xtf32(tmem_o, qhi, qlo, kQTile, vhi, vlo, kKTile, idesc);
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
        if (t0 + kPT < w.tok_end) {
            // the next sub-chunk needs the query tiles again (they hold P now)
            tmem_fence_before();
            __syncthreads();
            load_queries(p, w, rows, qhi, qlo, tid);
        }
    }

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
    prefix_attention_kernel<<<p.work_count, kPThreads, kPrefixSmem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mpb
