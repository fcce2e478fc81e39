// Tensor-core FP32 GEMM for sm_100a: split-precision FP16 products on tcgen05 with
// TMEM accumulators.
//
// C[M][N] (op)= A[M][K] . B[N][K]^T for the projections of the forward (fused QKV,
// O, gate, up, down, LM head) -- the reference runs them as pedantic FP32 cuBLAS
// SGEMMs (miniprefix/src/backend/cuda/llama_runner.cu:69-71).
//
// FP32 accuracy from 16-bit tensor cores (the published split-precision method,
// Ootomo & Yokota 2022, in its FP16 form): every operand x is stored as two FP16
// halves, hi = fp16(x) and lo = fp16((x - hi) * 2^11) (kernels.h), and
// C = A_hi.B_hi + 2^-11 (A_hi.B_lo + A_lo.B_hi). The FP16 products are exact in the
// tensor core's FP32 accumulation; the two sums are kept in separate TMEM
// accumulators (the main product and the scaled cross terms) and combined as
// main + 2^-11 cross with one fused multiply-add. The dropped A_lo.B_lo term and
// the rounding of lo are below 2^-22 relative per product. The kind::f16 pipe runs
// at twice the TF32 rate and the halves take 4 bytes per value instead of 8, so a
// K block moves half the operand bytes of the same product in TF32 halves.
// Weights are split once at upload; the kernels that produce GEMM inputs
// (RMSNorm, attention, SwiGLU, the residual epilogues) write the halves directly.
//
// A CTA computes the K-slice blockIdx.z (of gridDim.z) of a 128 x BN tile with 4 warps:
//  * warp 0 / one lane: TMA producer. Per 64-element K block it loads the four
//    operand tiles (A_hi, A_lo, B_hi, B_lo; 128-byte swizzled rows, one CTA per load)
//    into a stage and signals the stage's full mbarrier by transaction count;
//  * warp 1 / one lane: MMA issuer. Per K block 4 K-steps x 3 tcgen05.mma
//    (kind::f16, M=128, N=BN, K=16) into the two TMEM accumulators; tcgen05.commit
//    releases the stage to the producer, and after the last block signals the
//    accumulator barrier;
//  * warps 2-3, meanwhile: gather the epilogue's per-row inputs that need global
//    reads (RMSNorm row scales, RoPE destinations) into shared memory;
//  * all 4 warps: the K slices of one output tile form a thread-block cluster
//    (cluster dims 1 x 1 x slices) and each CTA owns a contiguous share of the
//    tile's rows. As soon as its own accumulators are final, each thread reads its
//    TMEM lane (= tile row) with tcgen05.ld.32x32b, combines the two sums, and
//    writes the row into a staging copy of the tile in the (now idle) stage ring;
//    one thread then sends each owner CTA its rows with one bulk shared-to-shared
//    copy (cp.async.bulk.shared::cluster, this slice's block in the owner's
//    receive area), completing bytes on the owner's receive mbarrier. The owner
//    waits on that barrier alone -- no cluster-wide barrier separates the MMAs
//    from the push -- then sums its rows over the slices' blocks in slice order
//    (deterministic split-K for the small-M decode GEMMs, no global round trip and
//    no remote loads) and applies the fused epilogue with coalesced row-contiguous
//    stores. Two split cluster barriers remain off the critical path: one whose
//    arrival follows the barrier set-up at the start and whose wait precedes the
//    first copy, and one whose arrival follows the copies and whose wait precedes
//    the exit.
// Every mbarrier wait is bounded; a timeout sets the error word, and the CTA still
// passes both cluster barriers and releases its tensor memory.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace mpb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // fp16 elements per K block = one 128-byte swizzle row
constexpr int kThreads = 128;
constexpr int kMaxSlices = 8;  // portable cluster size

template <int BN>
struct TcConfig {
    // Tiles up to 128 wide may split K: their slices push partial rows into a
    // receive area of its own, so a slice can push while its owner still runs MMAs
    // out of the stage ring. The 256-wide LM-head tiles never split K and reuse the
    // idle ring for their rows.
    static constexpr bool kOwnRecv = BN <= 128;
    static constexpr int kStages = BN <= 64 ? 3 : 2;
    static constexpr int kATile = kBM * kBK * 2;  // bytes
    static constexpr int kBTile = BN * kBK * 2;
    static constexpr int kStage = 2 * kATile + 2 * kBTile;
    static constexpr int kTileStride = BN + 4;  // floats per received accumulator row (bank spread)
    // receive area: `slices` partial row blocks of ceil(128 / slices) rows each
    static constexpr int kRecvBytes = (kBM + kMaxSlices) * kTileStride * 4;
    static constexpr int kRing = kStages * kStage;
    static constexpr int kData = kOwnRecv ? kRing + kRecvBytes : (kRing > kRecvBytes ? kRing : kRecvBytes);
    static constexpr int kSmem = kData + 1024 /*align*/ + 256 /*barriers*/;
    // two accumulators of BN columns: A_hi.B_hi, then the cross terms
    static constexpr int kTmemCols = 2 * BN;
};
// AddTo at 64-wide tiles (the O and down projections) fetches its rows of the
// residual and the norm weights into shared memory while the MMAs run: a residual
// read issued only in the epilogue waited several microseconds for the data.
template <int BN, Epilogue E>
__host__ __device__ constexpr bool prefetch_residual() { return E == Epilogue::AddTo && BN == 64; }
template <int BN>
constexpr int kResidStride = BN + 4;  // floats per prefetched residual row (bank spread)
template <int BN, Epilogue E>
__host__ __device__ constexpr int resid_bytes() { return prefetch_residual<BN, E>() ? (kBM * kResidStride<BN> + BN) * 4 : 0; }
template <int BN, Epilogue E>
constexpr int dynamic_smem() { return TcConfig<BN>::kSmem + resid_bytes<BN, E>(); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Rows [slice_row0(r), slice_row0(r + 1)) of a tile are reduced and stored by
// cluster rank r.
__host__ __device__ constexpr int slice_row0(int rank, int slices) { return rank * kBM / slices; }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Split cluster barrier: every thread of every CTA of the cluster arrives, then
// waits for all arrivals of that phase.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
// Arrival that orders no memory: the exit barrier only keeps a CTA alive while a
// slice may still push into it (the pushed bytes are tracked by its mbarrier).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Address of the same shared-memory offset in cluster CTA `rank` (its own included).
__device__ __forceinline__ uint32_t map_cluster(const void* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    return remote;
}

// Bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory to a
// cluster CTA's shared memory at `dst`, completing its bytes on that CTA's
// mbarrier at `bar` (dst and bar: shared::cluster addresses of the same CTA).
__device__ __forceinline__ void bulk_copy_s2c(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst),
                 "r"(smem_u32(src)), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk copy of this thread has read its source.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// g / (1 + exp(-g)) * u (miniprefix/src/backend/cpu/llama_runner.cpp:97). The
// reciprocal of d = 1 + exp(-g) >= 1 is the hardware approximation refined by one
// Newton step, r' = r + r (1 - d r), within about 1 ulp of 1 / d; it has no
// per-element branch (unlike the IEEE-rounded division and reciprocal), so the
// compiler interleaves a round's independent outputs. d = inf (g < -88) gives 0.
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float d = __fadd_rn(1.0f, expf(-g));
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
    r = fmaf(r, fmaf(-d, r, 1.0f), r);
    r = isinf(d) ? 0.0f : r;
    return __fmul_rn(__fmul_rn(g, r), u);
}

// Fused epilogue over rows [r0, r1) of the tile, columns in parallel (coalesced).
// Each output float4 is the sum over the cluster's slices, in slice order, of the
// partial tiles the slices pushed into this CTA's receive area (`recv`, one block
// of `slice_floats` per slice, local row = row - r0). Per-row inputs that need
// global reads (RMSNorm row scales, RoPE destinations and positions) were
// gathered into shared memory by epilogue_rows_prepare while the MMAs ran.
//  Store  : c[row][n0 + j] = acc
//  AddTo  : c[row][n0 + j] += acc                        (residual add)
//  SwiGLU : per 64-column group g of the tile, columns 0..31 are gate and 32..63 up
//           of output columns (n0 + 64 g) / 2 + 0..31; writes h = silu(gate) * up as
//           FP16 hi/lo halves (the down projection's input).
//  Rope   : the tile is one head of the QKV projection; dims (d, d + 32) rotate
//           together (q and k heads) as the CPU runner does (a' = a cos - b sin,
//           b' = b cos + a sin, products rounded separately; miniprefix/src/backend/
//           cpu/llama_runner.cpp:17-22, cos/sin from host tables filled with its libm
//           calls) and go to the attention input (q) or the row's page slot (k, v,
//           paged_kv.cpp:53-56 offsets), see RopeEpilogue.
template <Epilogue E>
__host__ __device__ constexpr int epilogue_unroll() { return E == Epilogue::SwiGLU || E == Epilogue::Rope ? 2 : 4; }

// Physical page of position `pos` of table slot `slot` (-1 past the table or the
// context).
__device__ __forceinline__ int rope_block(const TcGemmParams& p, int slot, int pos) {
    const RopeEpilogue& r = p.rope;
    const int page = pos / r.block_tokens;
    if (page < r.table_stride && pos < r.max_position) return r.tables[size_t(slot) * r.table_stride + page];
    return -1;
}

// Destination of head `head` (0..14) of batch row `grow` at position `pos` in page
// `block` for the Rope epilogue: the q row, or the K/V page slot (nullptr and an
// error bit when the row's page is outside its table or the pool).
__device__ __forceinline__ float* rope_destination(const TcGemmParams& p, int head, int grow, int pos, int block) {
    const RopeEpilogue& r = p.rope;
    if (head < kHeads) return r.q + size_t(grow) * r.q_stride + head * kHeadDim;
    if (block < 0 || block >= r.max_blocks) {
        raise_error(p.error, kErrBounds);
        return nullptr;
    }
    const size_t off = (pool_page(block, r.page_stride, r.layer_offset) * r.block_tokens + pos % r.block_tokens) * kKvWidth;
    const int kvh = (head - kHeads) % kKvHeads;
    return (head < kHeads + kKvHeads ? r.keys : r.values) + off + kvh * kHeadDim;
}

// Per-row epilogue inputs of rows [r0, r1), indexed by row - r0.
struct RowInputs {
    float* scale;  // RMSNorm 1 / rms (SwiGLU, Rope with ssq_in)
    float** dst;   // Rope: destination of the tile's head
    int* pos;      // Rope: cos / sin table row
    float* resid;  // AddTo (prefetch_residual): rows [r0, r1) of c's tile, kResidStride apart
    float* norm;   // AddTo (prefetch_residual): the tile's BN norm weights
};

// Gathers RowInputs with `threads` threads (thread index t); runs beside the MMAs.
// `parts`: kRowsSettled gathers what was written at least two kernels earlier (the
// residual rows and norm weights, the Rope destinations), kRowsFresh what the
// preceding kernel writes (the row scales' sums of squares).
constexpr int kRowsSettled = 1, kRowsFresh = 2;
template <int BN, Epilogue E>
__device__ __forceinline__ void epilogue_rows_prepare(const TcGemmParams& p, const RowInputs& in, int m0, int n0,
                                                      int r0, int r1, int t, int threads, int parts) {
    constexpr bool kPairs = E == Epilogue::SwiGLU || E == Epilogue::Rope;
    if (prefetch_residual<BN, E>() && (parts & kRowsSettled)) {
        // 16-byte copies, not waited for here: the threads wait just before the epilogue
        constexpr int kChunks = BN / 4;
        for (int i = t; i < (r1 - r0) * kChunks; i += threads) {
            const int lr = i / kChunks, c = i % kChunks;
            if (m0 + r0 + lr < p.m)
                cp_async16(in.resid + lr * kResidStride<BN> + 4 * c,
                           p.c + size_t(m0 + r0 + lr) * p.ldc + n0 + 4 * c);
        }
        if (p.norm_w != nullptr)
            for (int c = t; c < kChunks; c += threads) cp_async16(in.norm + 4 * c, p.norm_w + n0 + 4 * c);
        cp_async_commit();
    }
    // Two rows per thread and pass; every global load of a pass is requested before
    // any of them is used, so a pass costs one round trip (two for Rope's table
    // entries) instead of one per value -- these gathers run beside the MMAs and
    // must not outlast them.
    if (kPairs && p.ssq_in != nullptr && (parts & kRowsFresh)) {
        // this CTA's rows' 1 / rms from the producer's per-64-column sums of
        // squares, summed in group order
        const int groups = p.k / kSsqGroup;
        constexpr int kMaxGroups = 16;
        for (int base = r0 + t; base < r1; base += 2 * threads) {
            if (groups <= kMaxGroups) {
                float v[2][kMaxGroups];
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const int r = base + b * threads;
                    const bool live = r < r1 && m0 + r < p.m;
#pragma unroll
                    for (int g = 0; g < kMaxGroups; ++g)
                        v[b][g] = live && g < groups ? p.ssq_in[size_t(m0 + r) * groups + g] : 0.f;
                }
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const int r = base + b * threads;
                    if (r >= r1) continue;
                    float ss = 0.f;
#pragma unroll
                    for (int g = 0; g < kMaxGroups; ++g)
                        if (g < groups) ss = __fadd_rn(ss, v[b][g]);
                    in.scale[r - r0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(p.k)), p.eps)));
                }
            } else {
                for (int b = 0; b < 2; ++b) {
                    const int r = base + b * threads;
                    if (r >= r1) continue;
                    float ss = 0.f;
                    if (m0 + r < p.m)
                        for (int g = 0; g < groups; ++g) ss = __fadd_rn(ss, p.ssq_in[size_t(m0 + r) * groups + g]);
                    in.scale[r - r0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(p.k)), p.eps)));
                }
            }
        }
    }
    if constexpr (E == Epilogue::Rope) {
        if (parts & kRowsSettled) {
            const int head = n0 / 64;
            const bool kv = head >= kHeads;
            for (int base = r0 + t; base < r1; base += 2 * threads) {
                bool live[2];
                int pos[2], slot[2], block[2];
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const int r = base + b * threads;
                    live[b] = r < r1 && m0 + r < p.m;
                    pos[b] = live[b] ? p.rope.row_pos[m0 + r] : 0;
                    slot[b] = live[b] && kv ? p.rope.row_slot[m0 + r] : 0;
                }
#pragma unroll
                for (int b = 0; b < 2; ++b) block[b] = live[b] && kv ? rope_block(p, slot[b], pos[b]) : -1;
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const int r = base + b * threads;
                    if (r >= r1) continue;
                    in.dst[r - r0] = live[b] ? rope_destination(p, head, m0 + r, pos[b], block[b]) : nullptr;
                    in.pos[r - r0] = live[b] && head < kHeads + kKvHeads ? min(pos[b], p.rope.max_position - 1) : 0;
                }
            }
        }
    }
}

template <int BN, Epilogue E>
__device__ __forceinline__ void epilogue_rows(const TcGemmParams& p, const float* recv, int slice_floats,
                                              const RowInputs& in, int m0, int n0, int r0, int r1, int slices) {
    using Cfg = TcConfig<BN>;
    constexpr bool kSwiGLU = E == Epilogue::SwiGLU;
    constexpr bool kRope = E == Epilogue::Rope;
    constexpr bool kPairs = kSwiGLU || kRope;  // columns (c, c + 32) of each 64-column group together
    constexpr int kUnroll = epilogue_unroll<E>();
    // items per row: float4 of the tile (Store/AddTo) or of the first halves (SwiGLU gate, Rope dims 0..31)
    constexpr int kItems = kPairs ? (BN / 64) * 8 : BN / 4;
    constexpr int kLoads = kPairs ? 2 : 1;
    const int head = n0 / 64;  // Rope: the tile's head
    const int total = (r1 - r0) * kItems;
    const bool scaled = kPairs && p.ssq_in != nullptr;
    const bool produce = E == Epilogue::AddTo && p.norm_w != nullptr;
    // warp-uniform trip count (the producer's half-warp shuffles need every lane)
    for (int base = threadIdx.x; base - int(threadIdx.x & 31) < total; base += kThreads * kUnroll) {
        int off[kUnroll];
        bool live[kUnroll];
        float4* dst[kUnroll];
        float4 resid[kUnroll], wn[kUnroll];
        float4 rc[kUnroll], rs[kUnroll];  // Rope: cos / sin of the item's dims
        // global loads of the round first, so that their latencies overlap
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int i = base + u * kThreads;
            const int lr = i < total ? i / kItems : 0, it = i % kItems;
            live[u] = i < total && m0 + r0 + lr < p.m;
            off[u] = lr * Cfg::kTileStride + (kPairs ? 64 * (it / 8) + 4 * (it % 8) : 4 * it);
            dst[u] = nullptr;
            if (kRope) {
                if (live[u]) {
                    float* d = in.dst[lr];
                    dst[u] = d ? reinterpret_cast<float4*>(d + 4 * it) : nullptr;
                    if (head < kHeads + kKvHeads) {
                        const int pc = in.pos[lr];
                        rc[u] = *reinterpret_cast<const float4*>(p.rope.cos + size_t(pc) * 32 + 4 * it);
                        rs[u] = *reinterpret_cast<const float4*>(p.rope.sin + size_t(pc) * 32 + 4 * it);
                    }
                }
            } else if (!kSwiGLU) {
                dst[u] = reinterpret_cast<float4*>(p.c + size_t(m0 + r0 + lr) * p.ldc + n0 + 4 * it);
                if (E == Epilogue::AddTo && live[u]) {
                    if constexpr (prefetch_residual<BN, E>()) {
                        resid[u] = *reinterpret_cast<const float4*>(in.resid + lr * kResidStride<BN> + 4 * it);
                        if (produce) wn[u] = *reinterpret_cast<const float4*>(in.norm + 4 * it);
                    } else {
                        resid[u] = *dst[u];
                        if (produce) wn[u] = *reinterpret_cast<const float4*>(p.norm_w + n0 + 4 * it);
                    }
                }
            }
        }
        float4 acc[kUnroll][kLoads];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
#pragma unroll
            for (int h = 0; h < kLoads; ++h) {
                const float* at = recv + off[u] + 32 * h;
                acc[u][h] = *reinterpret_cast<const float4*>(at);
                for (int k = 1; k < slices; ++k) {
                    const float4 v = *reinterpret_cast<const float4*>(at + k * slice_floats);
                    acc[u][h].x += v.x;
                    acc[u][h].y += v.y;
                    acc[u][h].z += v.z;
                    acc[u][h].w += v.w;
                }
            }
        if (scaled) {
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int i = base + u * kThreads;
                const float sc = in.scale[i < total ? i / kItems : 0];
#pragma unroll
                for (int h = 0; h < kLoads; ++h)
                    acc[u][h] = make_float4(__fmul_rn(acc[u][h].x, sc), __fmul_rn(acc[u][h].y, sc),
                                            __fmul_rn(acc[u][h].z, sc), __fmul_rn(acc[u][h].w, sc));
            }
        }
        float sq[kUnroll];     // producer: sum of squares of the item's 4 new values
        float4 sum[kUnroll];   // AddTo: residual + product
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            sq[u] = 0.f;
            if (!live[u]) continue;
            const int i = base + u * kThreads;
            const int row = r0 + i / kItems, it = i % kItems;
            if (kRope) {
                if (!dst[u]) continue;
                float4 a = acc[u][0], b = acc[u][kLoads - 1];
                if (head < kHeads + kKvHeads) {
                    const float4 cs = rc[u], sn = rs[u];
                    const float4 x0 = a, x1 = b;
                    a = make_float4(__fsub_rn(__fmul_rn(x0.x, cs.x), __fmul_rn(x1.x, sn.x)),
                                    __fsub_rn(__fmul_rn(x0.y, cs.y), __fmul_rn(x1.y, sn.y)),
                                    __fsub_rn(__fmul_rn(x0.z, cs.z), __fmul_rn(x1.z, sn.z)),
                                    __fsub_rn(__fmul_rn(x0.w, cs.w), __fmul_rn(x1.w, sn.w)));
                    b = make_float4(__fadd_rn(__fmul_rn(x1.x, cs.x), __fmul_rn(x0.x, sn.x)),
                                    __fadd_rn(__fmul_rn(x1.y, cs.y), __fmul_rn(x0.y, sn.y)),
                                    __fadd_rn(__fmul_rn(x1.z, cs.z), __fmul_rn(x0.z, sn.z)),
                                    __fadd_rn(__fmul_rn(x1.w, cs.w), __fmul_rn(x0.w, sn.w)));
                }
                dst[u][0] = a;
                dst[u][8] = b;  // dims + 32
            } else if (kSwiGLU) {
                const float4 gt = acc[u][0], up = acc[u][kLoads - 1];
                const float o[4] = {silu_mul(gt.x, up.x), silu_mul(gt.y, up.y), silu_mul(gt.z, up.z),
                                    silu_mul(gt.w, up.w)};
                const size_t at = size_t(m0 + row) * p.ld_out + (n0 + 64 * (it / 8)) / 2 + 4 * (it % 8);
                store_split4(p.out_hi + at, p.out_lo + at, make_float4(o[0], o[1], o[2], o[3]));
            } else {
                const float4 a = acc[u][0];
                if (E == Epilogue::Store) {
                    *dst[u] = a;
                } else {
                    const float4 x = resid[u];
                    const float4 y = make_float4(__fadd_rn(x.x, a.x), __fadd_rn(x.y, a.y), __fadd_rn(x.z, a.z),
                                                 __fadd_rn(x.w, a.w));
                    sum[u] = y;
                    if (produce) {
                        float q = __fmul_rn(y.x, y.x);
                        q = fmaf(y.y, y.y, q);
                        q = fmaf(y.z, y.z, q);
                        sq[u] = fmaf(y.w, y.w, q);
                    }
                }
            }
        }
        if (produce) {
            // 16 consecutive items (lanes) of a row cover one 64-column group: reduce
            // over the half warp (a fixed tree) and let its first lane write the sum
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                float q = sq[u];
                q += __shfl_xor_sync(0xffffffffu, q, 1);
                q += __shfl_xor_sync(0xffffffffu, q, 2);
                q += __shfl_xor_sync(0xffffffffu, q, 4);
                q += __shfl_xor_sync(0xffffffffu, q, 8);
                const int i = base + u * kThreads;
                const int row = r0 + i / kItems, it = i % kItems;
                if (live[u] && it % 16 == 0) p.ssq_out[size_t(m0 + row) * (p.n / kSsqGroup) + (n0 + 4 * it) / kSsqGroup] = q;
            }
        }
        // AddTo: the residual sums (and, producing, the next GEMM's A operand y * norm
        // weight as FP16 halves) are stored after the row sums of squares are reduced
        if (E == Epilogue::AddTo) {
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                if (!live[u]) continue;
                const float4 y = sum[u];
                *dst[u] = y;
                if (produce) {
                    const int i = base + u * kThreads;
                    const int row = r0 + i / kItems, it = i % kItems;
                    const float4 w = wn[u];
                    const size_t at = size_t(m0 + row) * p.ld_out + n0 + 4 * it;
                    store_split4(p.out_hi + at, p.out_lo + at,
                                 make_float4(__fmul_rn(y.x, w.x), __fmul_rn(y.y, w.y), __fmul_rn(y.z, w.z),
                                             __fmul_rn(y.w, w.w)));
                }
            }
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
    float* recv = reinterpret_cast<float*>(smem + (Cfg::kOwnRecv ? Cfg::kRing : 0));
    // split K: the tile's combined rows are staged in the stage ring (idle once the
    // accumulators are final) for the bulk copies to their owners
    float* stage_rows = reinterpret_cast<float*>(smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kData);
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint64_t* recv_bar = accum + 1;  // the slices' partial rows of this CTA's share have landed
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(recv_bar + 1);
    int* failed = reinterpret_cast<int*>(tmem_holder + 1);
    float* resid_rows = reinterpret_cast<float*>(smem + Cfg::kData + 256);  // resid_bytes<BN, E>()

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
    // K blocks of this CTA's split: [kb_begin, kb_end)
    const int kb_total = (p.k + kBK - 1) / kBK, splits = gridDim.z;
    const int kb_per = (kb_total + splits - 1) / splits;
    const int kb_begin = blockIdx.z * kb_per, kb_end = min(kb_total, kb_begin + kb_per);
    const int kblocks = kb_end - kb_begin;
    // this CTA reduces and stores tile rows [r0, r1)
    const int rank = splits > 1 ? int(cluster_rank()) : 0;
    const int r0 = slice_row0(rank, splits), r1 = slice_row0(rank + 1, splits);
    __shared__ float row_scale[kBM];
    __shared__ float* row_dst[kBM];
    __shared__ int row_pos[kBM];
    const RowInputs rows{row_scale, row_dst, row_pos, resid_rows, resid_rows + kBM * kResidStride<BN>};

    if (warp == 0) tmem_alloc(tmem_holder, uint32_t(Cfg::kTmemCols));
    if (threadIdx.x == 32) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        mbar_init(recv_bar, 1);
        // every slice (this one included) sends (r1 - r0) rows of kTileStride floats
        if (splits > 1) mbar_arrive_expect_tx(recv_bar, uint32_t(splits * (r1 - r0) * Cfg::kTileStride) * 4u);
        *failed = 0;
        fence_barrier_init();
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    // phase 1: this CTA's barriers are initialised (waited before the first push)
    if (splits > 1) cluster_arrive();
    const uint32_t tmem = *tmem_holder;

    // The weights (B) never depend on an earlier kernel: the first stages' weight
    // tiles are requested before waiting for the predecessor (programmatic
    // dependent launch), the activations (A) only after.
    const uint64_t wait_ns = p.wait_ns ? p.wait_ns : kWaitNanoseconds;
    const int pre = p.stall ? 0 : min(S, kblocks);
    if (warp == 0 && lane == 0) {
        for (int kb = 0; kb < pre; ++kb) {
            unsigned char* st = smem + kb * Cfg::kStage;
            mbar_arrive_expect_tx(&full[kb], Cfg::kStage);
            const int kx = (kb_begin + kb) * kBK;
            tma_load_2d(st + 2 * Cfg::kATile, &b_hi, kx, p.b_row0 + n0, &full[kb]);
            tma_load_2d(st + 2 * Cfg::kATile + Cfg::kBTile, &b_lo, kx, p.b_row0 + n0, &full[kb]);
        }
    } else if (warp >= 2 && p.early_rows) {
        epilogue_rows_prepare<BN, E>(p, rows, m0, n0, r0, r1, int(threadIdx.x) - 64, kThreads - 64, kRowsSettled);
    }
    pdl_enter();
    if (warp == 0 && lane == 0) {
        // TMA producer
        for (int kb = 0; kb < (p.stall ? 0 : kblocks); ++kb) {
            const int s = kb % S;
            if (kb >= S && !mbar_wait_bounded(&empty[s], ((kb / S) - 1) & 1, wait_ns)) {
                *failed = 1;
                break;
            }
            unsigned char* st = smem + s * Cfg::kStage;
            const int kx = (kb_begin + kb) * kBK;
            if (kb >= pre) {
                mbar_arrive_expect_tx(&full[s], Cfg::kStage);
                tma_load_2d(st + 2 * Cfg::kATile, &b_hi, kx, p.b_row0 + n0, &full[s]);
                tma_load_2d(st + 2 * Cfg::kATile + Cfg::kBTile, &b_lo, kx, p.b_row0 + n0, &full[s]);
            }
            tma_load_2d(st, &a_hi, kx, m0, &full[s]);
            tma_load_2d(st + Cfg::kATile, &a_lo, kx, m0, &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: main = A_hi.B_hi in columns [0, BN), cross = A_lo.B_hi +
        // A_hi.B_lo in columns [BN, 2 BN)
        constexpr uint32_t idesc = umma_idesc_f16<kBM, BN>();
        const uint32_t d_main = tmem, d_cross = tmem + uint32_t(BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % S;
            if (!mbar_wait_bounded(&full[s], (kb / S) & 1, wait_ns)) {
                *failed = 1;
                ok = false;
                break;
            }
            tmem_fence_after();
            unsigned char* st = smem + s * Cfg::kStage;
            const uint64_t dah = smem_desc(st), dal = smem_desc(st + Cfg::kATile);
            const uint64_t dbh = smem_desc(st + 2 * Cfg::kATile), dbl = smem_desc(st + 2 * Cfg::kATile + Cfg::kBTile);
#pragma unroll
            for (int j = 0; j < kBK / 16; ++j) {
                const uint64_t step = uint64_t(j * 32) >> 4;  // 16 fp16 = 32 bytes along the swizzled row
                const uint32_t acc = (kb | j) != 0;
                mma_f16(d_cross, dal + step, dbh + step, idesc, acc);
                mma_f16(d_cross, dah + step, dbl + step, idesc, 1);
                mma_f16(d_main, dah + step, dbh + step, idesc, acc);
            }
            mma_commit(&empty[s]);
        }
        if (ok) mma_commit(accum);
    } else if (warp >= 2) {
        // idle until the accumulator is ready: gather the epilogue's row inputs
        epilogue_rows_prepare<BN, E>(p, rows, m0, n0, r0, r1, int(threadIdx.x) - 64, kThreads - 64,
                                     p.early_rows ? kRowsFresh : kRowsSettled | kRowsFresh);
    }
    __syncwarp();
    // Epilogue. The outcome is made CTA-uniform before anything that holds a barrier.
    if (!mbar_wait_bounded(accum, 0, wait_ns)) *failed = 1;
    __syncthreads();
    bool ok = *failed == 0;
    const int rows_max = (kBM + splits - 1) / splits;
    const int slice_floats = rows_max * Cfg::kTileStride;
    // phase 1: every CTA of the cluster can receive
    if (splits > 1) cluster_wait();
    if (ok) {
        // each thread moves its TMEM lane (= tile row), main + 2^-11 cross: unsplit
        // straight into the receive area; split, into a staging copy of the tile in
        // the idle stage ring, from which one bulk copy per owner CTA sends that
        // owner's rows as this slice's block there
        tmem_fence_after();
        const int row = warp * 32 + lane;
        float* slot = (splits > 1 ? stage_rows : recv) + row * Cfg::kTileStride;
        const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
            uint32_t hm[32], hc[32];
            tmem_load32(lane_base + uint32_t(c0), hm);
            tmem_load32(lane_base + uint32_t(BN + c0), hc);
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                float f[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    f[e] = fmaf(__uint_as_float(hc[4 * v + e]), kSplitLoUnscale, __uint_as_float(hm[4 * v + e]));
                *reinterpret_cast<float4*>(slot + c0 + 4 * v) = make_float4(f[0], f[1], f[2], f[3]);
            }
        }
        // the staged rows are read by the bulk-copy engine (async proxy)
        if (splits > 1) fence_proxy_async_shared();
    } else if (threadIdx.x == 0) {
        raise_error(p.error, kErrTimeout);
    }
    tmem_fence_before();
    // tensor memory reads are done (and, unsplit, the tile rows and row inputs are visible)
    __syncthreads();
    if (warp == 0) {
        tmem_fence_after();
        tmem_dealloc(tmem, uint32_t(Cfg::kTmemCols));
    }
    if (splits > 1) {
        if (ok && threadIdx.x == 0) {
            // owner j's rows [slice_row0(j), slice_row0(j + 1)) are contiguous in the
            // staging copy, at the stride of the receive area
            for (int j = 0; j < splits; ++j) {
                const int a = slice_row0(j, splits), b = slice_row0(j + 1, splits);
                bulk_copy_s2c(map_cluster(recv + rank * slice_floats, uint32_t(j)), stage_rows + a * Cfg::kTileStride,
                              uint32_t((b - a) * Cfg::kTileStride) * 4u, map_cluster(recv_bar, uint32_t(j)));
            }
            bulk_commit();
        }
        // phase 2: this CTA's copies are issued (waited before the exit, so no CTA
        // leaves while a slice may still copy into it)
        cluster_arrive_relaxed();
        // every slice's block of this CTA's rows has landed
        const bool got = mbar_wait_bounded(recv_bar, 0, wait_ns);
        const bool all = __syncthreads_and(got) != 0;
        if (ok && !all) {
            if (threadIdx.x == 0) raise_error(p.error, kErrTimeout);
            ok = false;
        }
    }
    if constexpr (prefetch_residual<BN, E>()) {
        // the residual rows that warps 2-3 requested are in shared memory
        if (warp >= 2) cp_async_commit_wait_all();
        __syncthreads();
    }
    if (ok) epilogue_rows<BN, E>(p, recv, slice_floats, rows, m0, n0, r0, r1, splits);
    if (splits > 1) {
        if (threadIdx.x == 0) bulk_wait_read_all();  // the staging copy is read before the CTA ends
        cluster_wait();
    }
}

// Clusters of each size (index = slices) that the device holds at once, per tile
// width (a cluster lives inside one GPC, so this is below 148 / slices).
int g_active_clusters[3][kMaxSlices + 1];

constexpr int bn_index(int bn) { return bn == 64 ? 0 : (bn == 128 ? 1 : 2); }

template <int BN, Epilogue E>
cudaError_t launch_bn(const TcGemmMaps& maps, const TcGemmParams& p, cudaStream_t stream) {
    using Cfg = TcConfig<BN>;
    static_assert(dynamic_smem<BN, E>() + 2048 /*static*/ <= 232448, "stage buffers exceed shared memory");
    static_assert(!Cfg::kOwnRecv || Cfg::kRing >= kBM * Cfg::kTileStride * 4, "split-K staging exceeds the ring");
    const int tiles = (p.n / BN) * ((p.m + kBM - 1) / kBM);
    const int kb = (p.k + kBK - 1) / kBK;
    // K slices (tiles with their own receive area only): as many as keep every
    // tile's cluster resident in one wave, at most one portable cluster, no empty
    // slice
    int splits = Cfg::kOwnRecv ? std::max(1, std::min(kMaxSlices, kb)) : 1;
    while (splits > 1 && tiles > g_active_clusters[bn_index(BN)][splits]) --splits;
    while (splits > 1 && (splits - 1) * ((kb + splits - 1) / splits) >= kb) --splits;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.n / BN, (p.m + kBM - 1) / kBM, splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = dynamic_smem<BN, E>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = unsigned(splits);
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, E>, *maps.a_hi, *maps.a_lo, *maps.b_hi, *maps.b_lo, p);
}

template <int BN>
cudaError_t configure_bn() {
    using Cfg = TcConfig<BN>;
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, Epilogue::Store>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_gemm_kernel<BN, Epilogue::AddTo>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 dynamic_smem<BN, Epilogue::AddTo>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_gemm_kernel<BN, Epilogue::SwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
    if constexpr (BN == 64)
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(tc_gemm_kernel<BN, Epilogue::Rope>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cfg::kSmem);
    // resident clusters of 1..8 CTAs (same resources for every epilogue)
    for (int s = 1; s <= kMaxSlices && e == cudaSuccess; ++s) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(1, 1, s);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = Cfg::kSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = unsigned(s);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<BN, Epilogue::Store>, &cfg);
        g_active_clusters[bn_index(BN)][s] = n;
    }
    return e;
}

// hi/lo split of a whole buffer (test inputs).
__global__ void split_kernel(const float* x, __half* hi, __half* lo, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        split_f16(x[i], hi[i], lo[i]);
}

}  // namespace

cudaError_t configure_tc_gemm() {
    cudaError_t e = configure_bn<64>();
    if (e == cudaSuccess) e = configure_bn<128>();
    if (e == cudaSuccess) e = configure_bn<256>();
    return e;
}

template <int BN>
cudaError_t launch_e(const TcGemmMaps& maps, const TcGemmParams& p, Epilogue e, cudaStream_t stream) {
    if (p.n % BN) return cudaErrorInvalidValue;
    switch (e) {
        case Epilogue::Store: return launch_bn<BN, Epilogue::Store>(maps, p, stream);
        case Epilogue::AddTo: return launch_bn<BN, Epilogue::AddTo>(maps, p, stream);
        case Epilogue::SwiGLU: return launch_bn<BN, Epilogue::SwiGLU>(maps, p, stream);
        case Epilogue::Rope:
            if constexpr (BN == 64) {
                if (p.n != (kHeads + 2 * kKvHeads) * kHeadDim) return cudaErrorInvalidValue;
                return launch_bn<BN, Epilogue::Rope>(maps, p, stream);
            }
            return cudaErrorInvalidValue;
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_tc_gemm(const TcGemmMaps& maps, const TcGemmParams& p, Epilogue e, cudaStream_t stream) {
    if (p.m <= 0) return cudaSuccess;
    if (p.k <= 0 || p.k % 8) return cudaErrorInvalidValue;
    switch (p.bn == 0 ? 64 : p.bn) {
        case 64: return launch_e<64>(maps, p, e, stream);
        case 128: return launch_e<128>(maps, p, e, stream);
        case 256: return launch_e<256>(maps, p, e, stream);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_split(const float* x, __half* hi, __half* lo, size_t n, cudaStream_t stream) {
    if (!n) return cudaSuccess;
    split_kernel<<<1184, 256, 0, stream>>>(x, hi, lo, n);
    return cudaGetLastError();
}

}  // namespace mpb
