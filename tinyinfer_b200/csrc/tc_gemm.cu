// Tensor-core FP32 GEMM for sm_100a: 3xTF32 on tcgen05 with TMEM accumulators.
//
// C[M][N] (op)= A[M][K] . B[N][K]^T for the projections of the forward (fused QKV,
// O, gate, up, down, LM head) -- the reference runs them as pedantic FP32 cuBLAS
// SGEMMs (miniprefix/src/backend/cuda/llama_runner.cu:69-71).
//
// FP32 accuracy from TF32 tensor cores (the published split-precision method,
// e.g. Ootomo & Yokota 2022): every operand x is stored as hi + lo with
// hi = x with its 13 low mantissa bits cleared (exact in TF32) and lo = x - hi
// (exact in FP32); C = A_lo.B_hi + A_hi.B_lo + A_hi.B_hi, accumulated in FP32 in
// tensor memory. The dropped A_lo.B_lo term and TF32 truncation of lo are below
// 2^-20 relative per product. Weights are split once at upload; the kernels that
// produce GEMM inputs (RMSNorm, attention, SwiGLU) write hi/lo pairs directly.
//
// A CTA computes the K-slice blockIdx.z (of gridDim.z) of a 128 x BN tile with 4 warps:
//  * warp 0 / one lane: TMA producer. Per 32-element K block it loads the four
//    operand tiles (A_hi, A_lo, B_hi, B_lo; 128-byte swizzled rows, one CTA per load)
//    into a stage and signals the stage's full mbarrier by transaction count;
//  * warp 1 / one lane: MMA issuer. Per K block 4 K-steps x 3 tcgen05.mma
//    (kind::tf32, M=128, N=BN, K=8) into one TMEM accumulator; tcgen05.commit
//    releases the stage to the producer, and after the last block signals the
//    accumulator barrier;
//  * all 4 warps: epilogue. Each warp reads its 32 TMEM lanes (= tile rows) with
//    tcgen05.ld.32x32b and applies the fused epilogue -- directly when the tile
//    has one K slice, else after the last slice to finish has summed every
//    slice's partial tile in slice order (deterministic split-K for the small-M
//    decode GEMMs, which otherwise leave most SMs idle).
// Every mbarrier wait is bounded; a timeout sets the error word and the CTA still
// releases its tensor memory before returning.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace mpb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;  // fp32 elements per K block = one 128-byte swizzle row
constexpr int kThreads = 128;

template <int BN>
struct TcConfig {
    static constexpr int kStages = BN <= 64 ? 4 : (BN <= 128 ? 3 : 2);
    static constexpr int kATile = kBM * kBK * 4;  // bytes
    static constexpr int kBTile = BN * kBK * 4;
    static constexpr int kStage = 2 * kATile + 2 * kBTile;
    static constexpr int kSmem = kStages * kStage + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr int kTmemCols = BN < 32 ? 32 : BN;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// K-major, 128-byte swizzle UMMA shared-memory descriptor: start address >> 4,
// LBO (ignored for swizzled K-major) 1, SBO = 1024 B between 8-row groups,
// version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc(const void* tile) {
    const uint64_t addr = smem_u32(tile);
    uint64_t d = (addr >> 4) & 0x3FFFull;
    d |= uint64_t(1) << 16;
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Instruction descriptor: D f32 (1 @ bit 4), A/B tf32 (2 @ bits 7, 10), both
// K-major, N >> 3 @ bit 17, M >> 4 @ bit 24.
template <int BN>
__host__ __device__ constexpr uint32_t instr_desc() {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The fused epilogue for one output row of the tile: v[0..BN) are columns n0.. .
//  Store  : c[row][n0 + j] = v[j]
//  AddTo  : c[row][n0 + j] += v[j]                     (residual add)
//  SwiGLU : the tile holds gate columns (v[0..BN/2)) and the matching up columns
//           (v[BN/2..BN)) of output columns n0/2 .. n0/2 + BN/2; writes
//           h = silu(gate) * up as TF32 hi/lo halves (the down projection's input).
template <int BN, Epilogue E>
__device__ __forceinline__ void epilogue(const TcGemmParams& p, int row, int n0, const float* v) {
    if (E == Epilogue::Store) {
        float4* dst = reinterpret_cast<float4*>(p.c + size_t(row) * p.ldc + n0);
#pragma unroll
        for (int i = 0; i < BN / 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else if (E == Epilogue::AddTo) {
        float4* dst = reinterpret_cast<float4*>(p.c + size_t(row) * p.ldc + n0);
#pragma unroll
        for (int i = 0; i < BN / 4; ++i) {
            const float4 x = dst[i];
            dst[i] = make_float4(__fadd_rn(x.x, v[4 * i]), __fadd_rn(x.y, v[4 * i + 1]), __fadd_rn(x.z, v[4 * i + 2]),
                                 __fadd_rn(x.w, v[4 * i + 3]));
        }
    } else {
        constexpr int H = BN / 2;
        const size_t at = size_t(row) * p.ld_out + n0 / 2;
#pragma unroll
        for (int i = 0; i < H / 4; ++i) {
            float hv[4], lv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float g = v[4 * i + e], u = v[H + 4 * i + e];
                const float o = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                split_tf32(o, hv[e], lv[e]);
            }
            reinterpret_cast<float4*>(p.out_hi + at)[i] = make_float4(hv[0], hv[1], hv[2], hv[3]);
            reinterpret_cast<float4*>(p.out_lo + at)[i] = make_float4(lv[0], lv[1], lv[2], lv[3]);
        }
    }
}

template <int BN, Epilogue E>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
                   const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo,
                   const TcGemmParams p) {
    using Cfg = TcConfig<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStage);
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accum + 1);
    int* failed = reinterpret_cast<int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
    // K blocks of this CTA's split: [kb_begin, kb_end)
    const int kb_total = p.k / kBK, splits = gridDim.z;
    const int kb_per = (kb_total + splits - 1) / splits;
    const int kb_begin = blockIdx.z * kb_per, kb_end = min(kb_total, kb_begin + kb_per);
    const int kblocks = kb_end - kb_begin;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(uint32_t(Cfg::kTmemCols))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        *failed = 0;
        fence_barrier_init();
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0 && lane == 0) {
        // TMA producer
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % S;
            if (kb >= S && !mbar_wait_bounded(&empty[s], ((kb / S) - 1) & 1)) {
                *failed = 1;
                break;
            }
            unsigned char* st = smem + s * Cfg::kStage;
            mbar_arrive_expect_tx(&full[s], Cfg::kStage);
            const int kx = (kb_begin + kb) * kBK;
            tma_load_2d(st, &a_hi, kx, m0, &full[s]);
            tma_load_2d(st + Cfg::kATile, &a_lo, kx, m0, &full[s]);
            tma_load_2d(st + 2 * Cfg::kATile, &b_hi, kx, p.b_row0 + n0, &full[s]);
            tma_load_2d(st + 2 * Cfg::kATile + Cfg::kBTile, &b_lo, kx, p.b_row0 + n0, &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        constexpr uint32_t idesc = instr_desc<BN>();
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % S;
            if (!mbar_wait_bounded(&full[s], (kb / S) & 1)) {
                *failed = 1;
                ok = false;
                break;
            }
            tmem_fence_after();
            unsigned char* st = smem + s * Cfg::kStage;
            const uint64_t dah = smem_desc(st), dal = smem_desc(st + Cfg::kATile);
            const uint64_t dbh = smem_desc(st + 2 * Cfg::kATile), dbl = smem_desc(st + 2 * Cfg::kATile + Cfg::kBTile);
#pragma unroll
            for (int j = 0; j < kBK / 8; ++j) {
                const uint64_t step = uint64_t(j * 32) >> 4;  // 8 tf32 = 32 bytes along the swizzled row
                mma_tf32(tmem, dal + step, dbh + step, idesc, (kb | j) != 0);
                mma_tf32(tmem, dah + step, dbl + step, idesc, 1);
                mma_tf32(tmem, dah + step, dbh + step, idesc, 1);
            }
            mma_commit(&empty[s]);
        }
        if (ok) mma_commit(accum);
    }
    __syncwarp();
    // Epilogue: all 4 warps; warp w owns TMEM lanes / tile rows 32w .. 32w+31.
    // The outcome is made CTA-uniform before any branch that holds a barrier.
    if (!mbar_wait_bounded(accum, 0)) *failed = 1;
    __syncthreads();
    const bool ok = *failed == 0;
    __syncthreads();
    const int row_in_tile = warp * 32 + lane;
    const int row = m0 + row_in_tile;
    if (!ok) {
        if (threadIdx.x == 0) raise_error(p.error, kErrTimeout);
    } else if (splits == 1) {
        tmem_fence_after();
        uint32_t r[BN];
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32)
            tmem_load32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c0), *reinterpret_cast<uint32_t(*)[32]>(&r[c0]));
        if (row < p.m) epilogue<BN, E>(p, row, n0, reinterpret_cast<const float*>(r));
    } else {
        // Deterministic split-K: park this slice's partial tile, and let the last
        // slice to arrive sum all partials in slice order before the epilogue.
        tmem_fence_after();
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        float* part = p.workspace + (size_t(tile) * splits + blockIdx.z) * (kBM * BN) + size_t(row_in_tile) * BN;
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
            uint32_t r[32];
            tmem_load32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c0), r);
#pragma unroll
            for (int v = 0; v < 8; ++v)
                __stcg(reinterpret_cast<float4*>(part + c0) + v,
                       make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3])));
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) *failed = atomicAdd(&p.counters[tile], 1u) == unsigned(splits - 1) ? 2 : 0;
        __syncthreads();
        if (*failed == 2) {
            __threadfence();
            float acc[BN];
#pragma unroll
            for (int j = 0; j < BN; ++j) acc[j] = 0.f;
            for (int s = 0; s < splits; ++s) {
                const float4* src = reinterpret_cast<const float4*>(
                    p.workspace + (size_t(tile) * splits + s) * (kBM * BN) + size_t(row_in_tile) * BN);
#pragma unroll
                for (int v = 0; v < BN / 4; ++v) {
                    const float4 x = __ldcg(src + v);
                    acc[4 * v] += x.x;
                    acc[4 * v + 1] += x.y;
                    acc[4 * v + 2] += x.z;
                    acc[4 * v + 3] += x.w;
                }
            }
            if (row < p.m) epilogue<BN, E>(p, row, n0, acc);
            if (threadIdx.x == 0) p.counters[tile] = 0u;  // ready for the next launch
        }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 0) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(uint32_t(Cfg::kTmemCols))
                     : "memory");
    }
}

template <int BN, Epilogue E>
cudaError_t launch_bn(const TcGemmMaps& maps, const TcGemmParams& p, cudaStream_t stream) {
    using Cfg = TcConfig<BN>;
    static_assert(Cfg::kSmem <= 232448, "stage buffers exceed shared memory");
    const int tiles = (p.n / BN) * ((p.m + kBM - 1) / kBM);
    const int kb = p.k / kBK;
    // K slices: fill about one wave of the 148 SMs, at least 2 K blocks per slice,
    // within the workspace the caller provides.
    int splits = 1;
    if (p.workspace && p.counters) {
        splits = std::max(1, std::min(148 / std::max(tiles, 1), kb / 2));
        while (splits > 1 && size_t(tiles) * splits * kBM * BN > p.workspace_floats) --splits;
        if (tiles > p.counter_count) splits = 1;
        // equalise: no empty trailing slice
        while (splits > 1 && (splits - 1) * ((kb + splits - 1) / splits) >= kb) --splits;
    }
    const dim3 grid(p.n / BN, (p.m + kBM - 1) / kBM, splits);
    tc_gemm_kernel<BN, E><<<grid, kThreads, Cfg::kSmem, stream>>>(*maps.a_hi, *maps.a_lo, *maps.b_hi, *maps.b_lo, p);
    return cudaGetLastError();
}

template <int BN>
cudaError_t configure_bn() {
    using Cfg = TcConfig<BN>;
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, Epilogue::Store>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_gemm_kernel<BN, Epilogue::AddTo>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_gemm_kernel<BN, Epilogue::SwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    return e;
}

// hi/lo split of a whole buffer (weights at upload, test inputs).
__global__ void split_kernel(const float* x, float* hi, float* lo, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        split_tf32(x[i], hi[i], lo[i]);
}

}  // namespace

cudaError_t configure_tc_gemm() { return configure_bn<kTcBN>(); }

cudaError_t launch_tc_gemm(const TcGemmMaps& maps, const TcGemmParams& p, Epilogue e, cudaStream_t stream) {
    if (p.m <= 0) return cudaSuccess;
    if (p.n % kTcBN || p.k % kBK) return cudaErrorInvalidValue;
    switch (e) {
        case Epilogue::Store: return launch_bn<kTcBN, Epilogue::Store>(maps, p, stream);
        case Epilogue::AddTo: return launch_bn<kTcBN, Epilogue::AddTo>(maps, p, stream);
        case Epilogue::SwiGLU: return launch_bn<kTcBN, Epilogue::SwiGLU>(maps, p, stream);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_split(const float* x, float* hi, float* lo, size_t n, cudaStream_t stream) {
    if (!n) return cudaSuccess;
    split_kernel<<<1184, 256, 0, stream>>>(x, hi, lo, n);
    return cudaGetLastError();
}

}  // namespace mpb
