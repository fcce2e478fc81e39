// Chunked-prefill paged attention (sm_100a): many query rows of one sequence.
//
// Computes the same causal GQA attention as the CPU runner
// (miniprefix/src/backend/cpu/llama_runner.cpp:85-93) for a chunk of `count` rows
// appended at positions start..start+count-1, but shares every K/V tile among
// 64 query rows x 3 heads of one KV group instead of re-reading the context per
// row and head as the reference kernel does (miniprefix/src/backend/cuda/
// llama_runner.cu:33-48).
//
// CTA = (64-row query tile, kv head). Per 32-token context tile:
//   S[192][32] = Q K^T (each thread a 6 x 4 block), masked causally and by length;
//   online softmax per query vector (one thread per vector, running max / sum);
//   O[192][64] = O * alpha + P V (each thread a 6 x 8 block).
// K/V rows are gathered through the block table with 16-byte cp.async into a
// double-buffered tile; rows past the sequence end are zero-filled so stale
// shared memory cannot reach the result.
#include "common.cuh"
#include "kernels.h"

namespace mpb {
namespace {

constexpr int kQRows = kPrefillTileRows;   // query rows per CTA
constexpr int kQVec = kQRows * kGroup;     // 192 query vectors (row, head of the group)
constexpr int kKT = 32;                    // context tokens per tile
constexpr int kThreads = 256;
constexpr int kQStride = kHeadDim + 1;     // 65: conflict-free column reads
constexpr int kKVStride = kHeadDim + 4;    // 68: 16-byte aligned rows for cp.async
constexpr int kSStride = kKT + 1;          // 33
constexpr size_t kPrefillSmem =
    (size_t(kQVec) * kQStride + 2 * 2 * kKT * kKVStride + size_t(kQVec) * kSStride + kQVec) * sizeof(float);

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Stage context tokens [t0, t0 + 32) of kv head kh into K/V tile buffers.
__device__ __forceinline__ void load_tile(const PrefillParams& p, const int32_t* table, int len, int kh, int t0,
                                          float* kt, float* vt, int tid) {
    // 32 tokens x 16 float4 per pool; 256 threads -> 2 float4 of K and 2 of V each.
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int idx = tid + it * kThreads;  // 0..511
        const int tok = idx >> 4, c4 = idx & 15;
        const int t = t0 + tok;
        float* kd = kt + tok * kKVStride + c4 * 4;
        float* vd = vt + tok * kKVStride + c4 * 4;
        if (t < len) {
            const int page = t / p.block_tokens;
            int block = page < p.table_stride ? table[page] : -1;
            if (block < 0 || block >= p.max_blocks) {
                raise_error(p.error, kErrBounds);
                block = 0;
            }
            const size_t off = ((size_t(block) * p.layers + p.layer) * p.block_tokens + (t - page * p.block_tokens)) *
                                   kKvWidth + kh * kHeadDim + c4 * 4;
            cp_async16(kd, p.keys + off);
            cp_async16(vd, p.values + off);
        } else {
            *reinterpret_cast<float4*>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(kThreads, 2) prefill_attention_kernel(const PrefillParams p) {
    pdl_enter();  // before any global memory access
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                                  // [192][65]
    float* Ks = Qs + kQVec * kQStride;               // [2][32][68]
    float* Vs = Ks + 2 * kKT * kKVStride;            // [2][32][68]
    float* Ss = Vs + 2 * kKT * kKVStride;            // [192][33]
    float* alpha_s = Ss + kQVec * kSStride;          // [192]

    const PrefillWork w = p.work[blockIdx.x];
    const int kh = w.kv_head;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rows = w.rows;                     // valid query rows in this tile (<= 64)
    const int pos0 = w.position;                 // position of the first query row
    const int len = pos0 + rows;                 // context needed by the last row
    const int32_t* table = p.tables + size_t(w.slot) * p.table_stride;

    // Q tile: vector v = r * 3 + hh holds row (row0 + r), head kh*3 + hh.
    for (int i = tid; i < kQVec * kHeadDim; i += kThreads) {
        const int v = i / kHeadDim, d = i % kHeadDim;
        const int r = v / kGroup, hh = v % kGroup;
        Qs[v * kQStride + d] =
            r < rows ? p.q[size_t(w.row0 + r) * p.q_stride + (kh * kGroup + hh) * kHeadDim + d] : 0.f;
    }
    const int n_tiles = (len + kKT - 1) / kKT;
    load_tile(p, table, len, kh, 0, Ks, Vs, tid);

    // identities
    const int sq = lane, sk = warp;          // scores: vectors sq + 32 i (i < 6), keys sk + 8 j (j < 4)
    const int oq = lane, od = warp * 8;      // output: vectors oq + 32 i, dims od .. od + 7
    float m_run = -INFINITY, l_run = 0.f;    // softmax state of vector `tid` (tid < 192)
    float acc[6][8];
#pragma unroll
    for (int i = 0; i < 6; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    for (int tile = 0; tile < n_tiles; ++tile) {
        const int buf = tile & 1;
        cp_async_wait_all();
        __syncthreads();  // tile `tile` landed; previous tile fully consumed
        if (tile + 1 < n_tiles)
            load_tile(p, table, len, kh, (tile + 1) * kKT, Ks + (buf ^ 1) * kKT * kKVStride,
                      Vs + (buf ^ 1) * kKT * kKVStride, tid);
        const float* K = Ks + buf * kKT * kKVStride;
        const float* V = Vs + buf * kKT * kKVStride;
        const int t0 = tile * kKT;
        // S = Q K^T / 8 with causal mask
        {
            float s[6][4];
#pragma unroll
            for (int i = 0; i < 6; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 8
            for (int d = 0; d < kHeadDim; ++d) {
                float qv[6], kv[4];
#pragma unroll
                for (int i = 0; i < 6; ++i) qv[i] = Qs[(sq + 32 * i) * kQStride + d];
#pragma unroll
                for (int j = 0; j < 4; ++j) kv[j] = K[(sk + 8 * j) * kKVStride + d];
#pragma unroll
                for (int i = 0; i < 6; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
            }
#pragma unroll
            for (int i = 0; i < 6; ++i) {
                const int v = sq + 32 * i;
                const int qpos = pos0 + v / kGroup;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int key = sk + 8 * j;
                    Ss[v * kSStride + key] = (t0 + key <= qpos) ? s[i][j] * 0.125f : -INFINITY;
                }
            }
        }
        __syncthreads();
        // online softmax, one thread per query vector
        if (tid < kQVec) {
            float* srow = Ss + tid * kSStride;
            float mx = m_run;
#pragma unroll
            for (int k = 0; k < kKT; ++k) mx = fmaxf(mx, srow[k]);
            // Rows past `rows` see only masked keys beyond their position; keep them finite.
            const float m_new = mx;
            const float alpha = m_new == -INFINITY ? 1.f : expf(m_run - m_new);
            float sum = 0.f;
#pragma unroll
            for (int k = 0; k < kKT; ++k) {
                const float e = m_new == -INFINITY ? 0.f : expf(srow[k] - m_new);
                srow[k] = e;
                sum += e;
            }
            l_run = l_run * alpha + sum;
            m_run = m_new;
            alpha_s[tid] = alpha;
        }
        __syncthreads();
        // O = O * alpha + P V
        {
            float al[6];
#pragma unroll
            for (int i = 0; i < 6; ++i) al[i] = alpha_s[oq + 32 * i];
#pragma unroll
            for (int i = 0; i < 6; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] *= al[i];
#pragma unroll 4
            for (int k = 0; k < kKT; ++k) {
                const float4 v0 = *reinterpret_cast<const float4*>(V + k * kKVStride + od);
                const float4 v1 = *reinterpret_cast<const float4*>(V + k * kKVStride + od + 4);
                const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int i = 0; i < 6; ++i) {
                    const float pr = Ss[(oq + 32 * i) * kSStride + k];
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(pr, vv[j], acc[i][j]);
                }
            }
        }
    }
    __syncthreads();
    if (tid < kQVec) alpha_s[tid] = l_run;  // reuse as the final denominators
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        const int v = oq + 32 * i;
        const int r = v / kGroup, hh = v % kGroup;
        if (r >= rows) continue;
        const float den = alpha_s[v];
        const size_t at = size_t(w.row0 + r) * p.out_stride + (kh * kGroup + hh) * kHeadDim + od;
        float val[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) val[j] = acc[i][j] / den;
        if (p.out_lo) {
            float hi[8], lo[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) split_tf32(val[j], hi[j], lo[j]);
            *reinterpret_cast<float4*>(p.out + at) = make_float4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<float4*>(p.out + at + 4) = make_float4(hi[4], hi[5], hi[6], hi[7]);
            *reinterpret_cast<float4*>(p.out_lo + at) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<float4*>(p.out_lo + at + 4) = make_float4(lo[4], lo[5], lo[6], lo[7]);
        } else {
            *reinterpret_cast<float4*>(p.out + at) = make_float4(val[0], val[1], val[2], val[3]);
            *reinterpret_cast<float4*>(p.out + at + 4) = make_float4(val[4], val[5], val[6], val[7]);
        }
    }
}

}  // namespace

cudaError_t configure_prefill_attention() {
    return cudaFuncSetAttribute(prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kPrefillSmem));
}

cudaError_t launch_prefill_attention(const PrefillParams& p, cudaStream_t stream) {
    if (p.work_count <= 0) return cudaSuccess;
    return launch_pdl(prefill_attention_kernel, dim3(p.work_count), dim3(kThreads), kPrefillSmem, stream, p);
}

}  // namespace mpb
