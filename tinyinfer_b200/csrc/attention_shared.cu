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
// shared memory (1024-aligned tiles): Q hi / lo and P hi / lo (2 K blocks each),
// K hi / lo and V^T hi / lo (2 K blocks each), the raw K and V staging rows
// ([64 tokens][64 floats]; V's 16-byte chunks XOR-swizzled by token so the
// transposing reads spread over the banks), the physical blocks of the staged
// tokens, then the barrier and the TMEM address
constexpr int kOffQhi = 0, kOffQlo = 2 * kQTile;
constexpr int kOffPhi = 4 * kQTile, kOffPlo = 6 * kQTile;
constexpr int kOffKhi = 8 * kQTile, kOffKlo = kOffKhi + 2 * kKTile;
constexpr int kOffVhi = kOffKlo + 2 * kKTile, kOffVlo = kOffVhi + 2 * kKTile;
constexpr int kOffRawK = kOffVlo + 2 * kKTile, kOffRawV = kOffRawK + kPT * kHeadDim * 4;
constexpr int kOffBlk = kOffRawV + kPT * kHeadDim * 4;
constexpr int kOffBar = kOffBlk + kPT * 4;
constexpr size_t kPrefixSmem = size_t(kOffBar) + 64 + 1024 /*alignment slack*/;
static_assert(kPrefixSmem <= 232448, "shared memory of the prefix kernel");
constexpr uint32_t kTmemCols = 128;  // S: columns 0..63, O: 64..127

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

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

// Physical block of shared token `token`, bounds-checked.
__device__ __forceinline__ int token_block(const PrefixParams& p, const int32_t* table, int token) {
    const int page = token / p.block_tokens;
    int block = page < p.table_stride ? table[page] : -1;
    if (block < 0 || block >= p.max_blocks) {
        raise_error(p.error, kErrBounds);
        block = 0;  // stay in bounds; the error word fails the step
    }
    return block;
}

// Start the gathers of the raw K / V rows of tokens [t0, t0 + n) into staging
// (blk holds their physical blocks); rows past n are not fetched.
__device__ __forceinline__ void gather_raw(const PrefixParams& p, const int* blk, int t0, int n, int kh, float* raw_k,
                                           float* raw_v, int tid) {
    for (int i = tid; i < kPT * 16; i += kPThreads) {
        const int t = i >> 4, c4 = i & 15;
        if (t >= n) continue;
        const size_t off = kv_offset(p, blk, t0, t, kh) + c4 * 4;
        cp_async16(raw_k + t * kHeadDim + c4 * 4, p.keys + off);
        cp_async16(raw_v + t * kHeadDim + ((c4 ^ (t & 15)) * 4), p.values + off);
    }
    cp_async_commit();
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
    gather_raw(p, blk, w.tok_begin, min(kPT, w.tok_end - w.tok_begin), kh, raw_k, raw_v, tid);
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
        for (int i = tid; i < kPT * 16; i += kPThreads) {
            const int t = i >> 4, c4 = i & 15;
            const float4 kv = t < n_valid ? *reinterpret_cast<const float4*>(raw_k + t * kHeadDim + c4 * 4)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
            store_split4(khi + (c4 >> 3) * kKTile, klo + (c4 >> 3) * kKTile, sw128_offset(t, c4 & 7), kv);
        }
        for (int i = tid; i < kPT * 16; i += kPThreads) {
            const int t = i & (kPT - 1), c4 = i / kPT;  // consecutive threads: consecutive tokens
            const float4 vv = t < n_valid ? *reinterpret_cast<const float4*>(raw_v + t * kHeadDim + ((c4 ^ (t & 15)) * 4))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
            const float ve[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int d = 4 * c4 + e;  // V^T row; column = token t (K block t / 32)
                const uint32_t off = sw128_offset(d, (t & 31) >> 2) + uint32_t(t & 3) * 4;
                float h, l;
                split_tf32(ve[e], h, l);
                *reinterpret_cast<float*>(vhi + (t >> 5) * kKTile + off) = h;
                *reinterpret_cast<float*>(vlo + (t >> 5) * kKTile + off) = l;
            }
        }
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
            gather_raw(p, blk, t1, min(kPT, w.tok_end - t1), kh, raw_k, raw_v, tid);
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
