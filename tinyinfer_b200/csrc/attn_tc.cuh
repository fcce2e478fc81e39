// Building blocks of the tensor-core attention kernels (sm_100a): softmax(Q K^T)
// V over 64-token sub-chunks of a paged context as 3xTF32 tcgen05 MMAs with
// M = 128 query vectors.
//
// Tiles in shared memory are K-major, 128-byte swizzled UMMA operands (umma.cuh),
// each as TF32 hi / lo halves: Q and P are 128 rows x 2 K blocks of 32, K is 64
// tokens x 2 K blocks (the 64 head dims), V^T is 64 dims x 2 K blocks (the 64
// tokens). Raw K and V rows are gathered through the block table with 16-byte
// cp.async into a staging buffer (V's 16-byte chunks XOR-swizzled by token so
// that the transposing reads spread over the banks), then split into the tiles.
#pragma once
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace mpb {
namespace attn_tc {

constexpr int kQ = 128;                 // query vectors per CTA = UMMA M
constexpr int kT = 64;                  // tokens per sub-chunk = UMMA N of S, K of P.V
constexpr int kQTile = kQ * 32 * 4;     // one 32-element K block of a 128-row tile (16 KB)
constexpr int kKTile = kT * 32 * 4;     // one K block of a 64-row tile (8 KB)
// shared memory layout (1024-aligned tiles): Q hi / lo and P hi / lo (2 K blocks
// each), K hi / lo and V^T hi / lo (2 K blocks each), the raw K and V staging
// rows ([64 tokens][64 floats]), the physical blocks of the staged tokens, then
// the MMA barriers, the TMEM address and a failure flag
constexpr int kOffQhi = 0, kOffQlo = 2 * kQTile;
constexpr int kOffPhi = 4 * kQTile, kOffPlo = 6 * kQTile;
constexpr int kOffKhi = 8 * kQTile, kOffKlo = kOffKhi + 2 * kKTile;
constexpr int kOffVhi = kOffKlo + 2 * kKTile, kOffVlo = kOffVhi + 2 * kKTile;
constexpr int kOffRawK = kOffVlo + 2 * kKTile, kOffRawV = kOffRawK + kT * kHeadDim * 4;
constexpr int kOffBlk = kOffRawV + kT * kHeadDim * 4;
constexpr int kOffBar = kOffBlk + kT * 4;
constexpr size_t kSmem = size_t(kOffBar) + 64 + 1024 /*alignment slack*/;  // barriers etc. in the 64 bytes
static_assert(kSmem <= 232448, "shared memory of a tensor-core attention CTA");
constexpr uint32_t kTmemCols = 128;  // S: columns 0..63, O: 64..127

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Splits v into TF32 halves and stores them at byte offset `off` of two tiles.
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

// Physical block of context token `token` through `table`, bounds-checked (an
// out-of-range entry reads block 0 and sets the bounds bit, which fails the step).
__device__ __forceinline__ int token_block(const int32_t* table, int table_stride, int block_tokens, int max_blocks,
                                           int token, unsigned* error) {
    const int page = token / block_tokens;
    int block = page < table_stride ? table[page] : -1;
    if (block < 0 || block >= max_blocks) {
        raise_error(error, kErrBounds);
        block = 0;
    }
    return block;
}

// Starts the gathers of the raw K / V rows (kv head kh; pages addressed by
// pool_page(block, page_stride, layer_offset)) of tokens t0 .. t0 + n - 1 into
// staging; blk[t] holds token t0 + t's physical block. Rows past n are not fetched.
__device__ __forceinline__ void gather_raw(const float* keys, const float* values, int page_stride,
                                           int64_t layer_offset,
                                           int block_tokens, const int* blk, int t0, int n, int kh, float* raw_k,
                                           float* raw_v, int tid, int threads) {
    for (int i = tid; i < kT * 16; i += threads) {
        const int t = i >> 4, c4 = i & 15;
        if (t >= n) continue;
        const int token = t0 + t;
        const size_t off = (pool_page(blk[t], page_stride, layer_offset) * block_tokens + token % block_tokens) * kKvWidth +
                           kh * kHeadDim + c4 * 4;
        cp_async16(raw_k + t * kHeadDim + c4 * 4, keys + off);
        cp_async16(raw_v + t * kHeadDim + ((c4 ^ (t & 15)) * 4), values + off);
    }
    cp_async_commit();
}

// Splits the staged K rows into the hi / lo K tiles (token-major); tokens at or
// past n_valid become zero.
__device__ __forceinline__ void split_k(const float* raw_k, int n_valid, unsigned char* khi, unsigned char* klo,
                                        int tid, int threads) {
    for (int i = tid; i < kT * 16; i += threads) {
        const int t = i >> 4, c4 = i & 15;
        const float4 kv = t < n_valid ? *reinterpret_cast<const float4*>(raw_k + t * kHeadDim + c4 * 4)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        store_split4(khi + (c4 >> 3) * kKTile, klo + (c4 >> 3) * kKTile, sw128_offset(t, c4 & 7), kv);
    }
}

// Splits the staged V rows into the hi / lo V^T tiles (dim-major); tokens at or
// past n_valid become zero.
__device__ __forceinline__ void split_v(const float* raw_v, int n_valid, unsigned char* vhi, unsigned char* vlo,
                                        int tid, int threads) {
    for (int i = tid; i < kT * 16; i += threads) {
        const int t = i & (kT - 1), c4 = i / kT;  // consecutive threads: consecutive tokens
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
}

__device__ __forceinline__ void split_kv(const float* raw_k, const float* raw_v, int n_valid, unsigned char* khi,
                                         unsigned char* klo, unsigned char* vhi, unsigned char* vlo, int tid,
                                         int threads) {
    split_k(raw_k, n_valid, khi, klo, tid, threads);
    split_v(raw_v, n_valid, vhi, vlo, tid, threads);
}

// The 64 fp32 columns [col, col + 64) of this thread's TMEM lane.
__device__ __forceinline__ void tmem_row64(uint32_t taddr, float (&out)[kT]) {
    uint32_t r[32];
    tmem_load32(taddr, r);
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j] = __uint_as_float(r[j]);
    tmem_load32(taddr + 32, r);
#pragma unroll
    for (int j = 0; j < 32; ++j) out[32 + j] = __uint_as_float(r[j]);
}

}  // namespace attn_tc
}  // namespace mpb
