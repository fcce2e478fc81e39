// Shared-prefix decode attention (sm_100a): the pages that a group of decode rows
// share are read once per launch for the whole group.
//
// Decode attention is bandwidth-bound when every row streams its whole context
// (miniprefix/src/backend/cuda/llama_runner.cu:33-48 reads it once per row and
// head). Rows that reuse a cached prefix (miniprefix/src/kv/prefix_cache.cpp) map
// the same physical pages at the start of their block tables, so the host groups
// such rows and this kernel computes their attention over the shared tokens as a
// small dense problem per (group, kv head): Q[rows x 3 heads][64] against
// K/V[shared tokens][64], i.e. the same causal-free softmax(QK^T / 8) V the CPU
// runner computes (miniprefix/src/backend/cpu/llama_runner.cpp:85-93) restricted
// to those tokens. Each CTA produces, per query vector, the running maximum, the
// sum of exponentials and the unnormalised output of its token chunk -- the same
// partial format as the split-K decode kernel -- and the decode kernel's last
// slice merges them with the rows' own pages (attention.cu).
//
// CTA = (group, kv head, 64 query vectors, token chunk), 128 threads. Per 32-token
// tile (double-buffered 16-byte cp.async gathers through the group's table):
//   S[64][32] = Q K^T / 8: thread (query qi = tid/2, tokens sub + 2k) 16 scores;
//   online softmax per query vector (2 lanes per vector, shuffles);
//   O[64][64] = O * alpha + P V: thread (qi, dims sub*4 + 8k) 32 outputs.
// All FP32 FMA. Tokens past the chunk end are masked by select, never by
// multiplying, so stale shared memory cannot reach the result.
#include "common.cuh"
#include "kernels.h"

namespace mpb {
namespace {

constexpr int kPQ = kPrefixQueries;  // 64 query vectors per CTA
constexpr int kPT = 32;              // tokens per tile
constexpr int kPThreads = 128;
constexpr int kRowStride = kHeadDim + 4;  // 68 floats: 16-byte aligned rows
constexpr int kPStride = kPT + 1;         // 33
constexpr size_t kPrefixSmem =
    (size_t(kPQ) * kRowStride + 2 * 2 * kPT * kRowStride + size_t(kPQ) * kPStride) * sizeof(float);

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Gather tokens [t0, min(t0 + 32, t1)) of kv head kh into a K/V tile pair;
// rows past t1 are zero-filled. 32 tokens x 16 float4 x 2 pools = 8 per thread.
__device__ __forceinline__ void load_tile(const PrefixParams& p, const int32_t* table, int kh, int t0, int t1,
                                          float* kt, float* vt, int tid) {
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int idx = tid + it * kPThreads;  // 0..511
        const int tok = idx >> 4, c4 = idx & 15;
        const int t = t0 + tok;
        float* kd = kt + tok * kRowStride + c4 * 4;
        float* vd = vt + tok * kRowStride + c4 * 4;
        if (t < t1) {
            const int page = t / p.block_tokens;
            int block = page < p.table_stride ? table[page] : -1;
            if (block < 0 || block >= p.max_blocks) {
                raise_error(p.error, kErrBounds);
                block = 0;  // stay in bounds; the error word fails the step
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

__global__ void __launch_bounds__(kPThreads, 3) prefix_attention_kernel(const PrefixParams p) {
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                            // [64][68]
    float* Kt = Qs + kPQ * kRowStride;         // [2][32][68]
    float* Vt = Kt + 2 * kPT * kRowStride;     // [2][32][68]
    float* Ps = Vt + 2 * kPT * kRowStride;     // [64][33]

    const int tid = threadIdx.x;
    const PrefixWork w = p.work[blockIdx.x];
    const int32_t* rows = p.group_rows + p.group_row0[w.group];
    const int32_t* table = p.tables + size_t(p.group_slot[w.group]) * p.table_stride;
    const int kh = w.kv_head;

    // Query vectors: qv = row_in_group * 3 + head_in_group, 64 x 16 float4.
#pragma unroll
    for (int it = 0; it < 8; ++it) {
        const int idx = tid + it * kPThreads;  // 0..1023
        const int qi = idx >> 4, c4 = idx & 15;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < w.q_count) {
            const int qv = w.q_begin + qi;
            const int row = rows[qv / kGroup];
            const int head = kh * kGroup + qv % kGroup;
            v = *reinterpret_cast<const float4*>(p.q + size_t(row) * p.q_stride + head * kHeadDim + c4 * 4);
        }
        *reinterpret_cast<float4*>(Qs + qi * kRowStride + c4 * 4) = v;
    }
    const int n_tiles = (w.tok_end - w.tok_begin + kPT - 1) / kPT;
    load_tile(p, table, kh, w.tok_begin, w.tok_end, Kt, Vt, tid);

    const int qi = tid >> 1, sub = tid & 1;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    for (int i = 0; i < n_tiles; ++i) {
        const int buf = i & 1;
        const int t0 = w.tok_begin + i * kPT;
        const int n_valid = min(kPT, w.tok_end - t0);
        if (i + 1 < n_tiles) {
            load_tile(p, table, kh, t0 + kPT, w.tok_end, Kt + (buf ^ 1) * kPT * kRowStride,
                      Vt + (buf ^ 1) * kPT * kRowStride, tid);
            cp_async_wait_one();
        } else {
            cp_async_wait_all();
        }
        __syncthreads();
        const float* kt = Kt + buf * kPT * kRowStride;
        const float* vt = Vt + buf * kPT * kRowStride;

        // scores of tokens sub + 2k
        float s[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) s[k] = 0.f;
        const float* qrow = Qs + qi * kRowStride;
#pragma unroll 4
        for (int d4 = 0; d4 < kHeadDim / 4; ++d4) {
            const float4 qv = *reinterpret_cast<const float4*>(qrow + 4 * d4);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float4 kv = *reinterpret_cast<const float4*>(kt + (sub + 2 * k) * kRowStride + 4 * d4);
                s[k] = fmaf(qv.x, kv.x, s[k]);
                s[k] = fmaf(qv.y, kv.y, s[k]);
                s[k] = fmaf(qv.z, kv.z, s[k]);
                s[k] = fmaf(qv.w, kv.w, s[k]);
            }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            s[k] = sub + 2 * k < n_valid ? s[k] * 0.125f : -INFINITY;
            mx = fmaxf(mx, s[k]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = expf(m_run - m_new);
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float pr = expf(s[k] - m_new);
            sum += pr;
            Ps[qi * kPStride + sub + 2 * k] = pr;
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        l_run = l_run * alpha + sum;
        m_run = m_new;
#pragma unroll
        for (int i2 = 0; i2 < 32; ++i2) acc[i2] *= alpha;
        __syncwarp();  // the two lanes of a query vector read each other's probabilities

        // O += P V over the tile: dims sub*4 + 8k
        const float* prow = Ps + qi * kPStride;
#pragma unroll 4
        for (int j = 0; j < kPT; ++j) {
            const float pr = prow[j];
            const float* vrow = vt + j * kRowStride + sub * 4;
            const bool valid = j < n_valid;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                float4 v = *reinterpret_cast<const float4*>(vrow + 8 * k);
                if (!valid) v = make_float4(0.f, 0.f, 0.f, 0.f);
                acc[4 * k] = fmaf(pr, v.x, acc[4 * k]);
                acc[4 * k + 1] = fmaf(pr, v.y, acc[4 * k + 1]);
                acc[4 * k + 2] = fmaf(pr, v.z, acc[4 * k + 2]);
                acc[4 * k + 3] = fmaf(pr, v.w, acc[4 * k + 3]);
            }
        }
        __syncthreads();  // the tile buffer is refilled next iteration
    }

    if (qi >= w.q_count) return;
    const int qv = w.q_begin + qi;
    const int row = rows[qv / kGroup];
    const int head = kh * kGroup + qv % kGroup;
    float* part = p.partial + (size_t(p.row_x0[row] + w.chunk) * kHeads + head) * (kHeadDim + 2);
    // partial records are 66 floats: 8-byte aligned, so scalar stores
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e) part[2 + sub * 4 + 8 * k + e] = acc[4 * k + e];
    if (sub == 0) {
        part[0] = m_run;
        part[1] = l_run;
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
