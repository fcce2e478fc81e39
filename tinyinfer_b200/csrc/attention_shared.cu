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
//   S[64][32] = Q K^T / 8: thread (queries qp and qp + 32, tokens sub + 4k) 16 scores,
//     2 query and 8 key float4 loads per 64 FMA;
//   online softmax per query vector (4 lanes per vector, shuffles);
//   O[64][64] = O * alpha + P V: thread (both queries, dims sub*4 + 16k) 32 outputs.
// All FP32 FMA; softmax weights are exp2 of scores scaled by log2(e) / 8, so the
// partials' maxima are base-2 quantities like the decode kernel's. Tokens past
// the chunk end are masked by select, never by multiplying, so stale shared
// memory cannot reach the result.
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

    // Thread = (query pair qp / qp + 32, token / dim quarter sub).
    const int qp = tid >> 2, sub = tid & 3;
    float acc[2][16];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[a][i] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

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

        // S: queries qp, qp + 32 x tokens sub + 4k
        float s[2][8];
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int k = 0; k < 8; ++k) s[a][k] = 0.f;
        const float* q0 = Qs + qp * kRowStride;
        const float* q1 = Qs + (qp + 32) * kRowStride;
#pragma unroll 2
        for (int d4 = 0; d4 < kHeadDim / 4; ++d4) {
            const float4 qa = *reinterpret_cast<const float4*>(q0 + 4 * d4);
            const float4 qb = *reinterpret_cast<const float4*>(q1 + 4 * d4);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 kv = *reinterpret_cast<const float4*>(kt + (sub + 4 * k) * kRowStride + 4 * d4);
                s[0][k] = fmaf(qa.x, kv.x, s[0][k]);
                s[0][k] = fmaf(qa.y, kv.y, s[0][k]);
                s[0][k] = fmaf(qa.z, kv.z, s[0][k]);
                s[0][k] = fmaf(qa.w, kv.w, s[0][k]);
                s[1][k] = fmaf(qb.x, kv.x, s[1][k]);
                s[1][k] = fmaf(qb.y, kv.y, s[1][k]);
                s[1][k] = fmaf(qb.z, kv.z, s[1][k]);
                s[1][k] = fmaf(qb.w, kv.w, s[1][k]);
            }
        }
        // online softmax; the 4 lanes of a query pair hold its 32 scores
#pragma unroll
        for (int a = 0; a < 2; ++a) {
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                s[a][k] = sub + 4 * k < n_valid ? s[a][k] * (0.125f * kLog2e) : -INFINITY;
                mx = fmaxf(mx, s[a][k]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_new = fmaxf(m_run[a], mx);
            const float alpha = exp2f(m_run[a] - m_new);
            float sum = 0.f;
            float* prow = Ps + (qp + 32 * a) * kPStride + sub;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float pr = exp2f(s[a][k] - m_new);
                sum += pr;
                prow[4 * k] = pr;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            l_run[a] = l_run[a] * alpha + sum;
            m_run[a] = m_new;
#pragma unroll
            for (int i2 = 0; i2 < 16; ++i2) acc[a][i2] *= alpha;
        }
        __syncwarp();  // the 4 lanes of a query pair read each other's probabilities

        // O += P V: dims sub*4 + 16k of both queries
        const float* p0 = Ps + qp * kPStride;
        const float* p1 = Ps + (qp + 32) * kPStride;
#pragma unroll 4
        for (int j = 0; j < kPT; ++j) {
            const float pa = p0[j], pb = p1[j];
            const float* vrow = vt + j * kRowStride + sub * 4;
            const bool valid = j < n_valid;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float4 v = *reinterpret_cast<const float4*>(vrow + 16 * k);
                if (!valid) v = make_float4(0.f, 0.f, 0.f, 0.f);
                acc[0][4 * k] = fmaf(pa, v.x, acc[0][4 * k]);
                acc[0][4 * k + 1] = fmaf(pa, v.y, acc[0][4 * k + 1]);
                acc[0][4 * k + 2] = fmaf(pa, v.z, acc[0][4 * k + 2]);
                acc[0][4 * k + 3] = fmaf(pa, v.w, acc[0][4 * k + 3]);
                acc[1][4 * k] = fmaf(pb, v.x, acc[1][4 * k]);
                acc[1][4 * k + 1] = fmaf(pb, v.y, acc[1][4 * k + 1]);
                acc[1][4 * k + 2] = fmaf(pb, v.z, acc[1][4 * k + 2]);
                acc[1][4 * k + 3] = fmaf(pb, v.w, acc[1][4 * k + 3]);
            }
        }
        __syncthreads();  // the tile buffer is refilled next iteration
    }

#pragma unroll
    for (int a = 0; a < 2; ++a) {
        const int qi = qp + 32 * a;
        if (qi >= w.q_count) continue;
        const int qv = w.q_begin + qi;
        const int row = rows[qv / kGroup];
        const int head = kh * kGroup + qv % kGroup;
        float* part = p.partial + (size_t(p.row_x0[row] + w.chunk) * kHeads + head) * (kHeadDim + 2);
        // partial records are 66 floats: 8-byte aligned, so scalar stores
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int e = 0; e < 4; ++e) part[2 + sub * 4 + 16 * k + e] = acc[a][4 * k + e];
        if (sub == 0) {
            part[0] = m_run[a];
            part[1] = l_run[a];
        }
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
