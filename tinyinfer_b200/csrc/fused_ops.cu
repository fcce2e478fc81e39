// Bandwidth-bound fused ops of the forward (sm_100a).
//
//  embed_rmsnorm : reference embedding_kernel + first rms_kernel
//                  (miniprefix/src/backend/cuda/llama_runner.cu:15-22, launches :146,148)
//  rmsnorm       : rms_kernel (:17-22); final norm only on each sequence's last row (:166)
//  (rope_kernel x2 + append_kernel, :23-32, run in the QKV GEMM's epilogue: tc_gemm.cu)
//  argmax        : greedy sampling of Engine::step (miniprefix/src/engine/engine.cpp:99)
//                  + the nonfinite check (:94-95; runner :173), on device
//  cow_copy      : the 2 cudaMemcpy2DAsync of a COW tail region (:130-137)
//  table_patch   : block-table delta upload (:139-143) applied as (index, value) pairs
#include "common.cuh"
#include "kernels.h"

namespace mpb {
namespace {

// One warp per row. Sum of squares by per-lane partials and a butterfly; the
// normalisation order matches the CPU runner: (x * scale) * w
// (miniprefix/src/backend/cpu/llama_runner.cpp:10-16).
__device__ __forceinline__ void rms_row(const float* x, const float* w, float eps, __half* out_hi, __half* out_lo,
                                        int hidden, int lane) {
    float sum = 0.f;
    for (int d = lane * 4; d < hidden; d += 128) {
        const float4 v = *reinterpret_cast<const float4*>(x + d);
        sum = fmaf(v.x, v.x, sum);
        sum = fmaf(v.y, v.y, sum);
        sum = fmaf(v.z, v.z, sum);
        sum = fmaf(v.w, v.w, sum);
    }
    sum = warp_sum(sum);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, float(hidden)), eps)));
    for (int d = lane * 4; d < hidden; d += 128) {
        const float4 v = *reinterpret_cast<const float4*>(x + d);
        const float4 g = *reinterpret_cast<const float4*>(w + d);
        store_split4(out_hi + d, out_lo + d,
                     make_float4(__fmul_rn(__fmul_rn(v.x, scale), g.x), __fmul_rn(__fmul_rn(v.y, scale), g.y),
                                 __fmul_rn(__fmul_rn(v.z, scale), g.z), __fmul_rn(__fmul_rn(v.w, scale), g.w)));
    }
}

// With ssq (the first layer's norm folded into its QKV GEMM): writes x * w as
// FP16 halves and the sum of squares of each 64-column group of x, reduced the
// way the GEMM epilogue reduces it (4 values per lane, then a half-warp tree);
// hidden a multiple of 64. Without: the normalised row, as rms_row.
__global__ void embed_rmsnorm_kernel(const int32_t* tokens, const float* embed, int vocabulary, const float* w,
                                     float eps, float* x, __half* normed_hi, __half* normed_lo, int rows,
                                     int hidden, float* ssq, unsigned* error) {
    pdl_enter();  // before any global memory access
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (row >= rows) return;
    int tok = tokens[row];
    if (tok < 0 || tok >= vocabulary) {
        if (lane == 0) raise_error(error, kErrBounds);
        tok = 0;
    }
    const float* src = embed + size_t(tok) * hidden;
    float* xr = x + size_t(row) * hidden;
    if (ssq) {
        for (int d0 = 0; d0 < hidden; d0 += 128) {
            const int d = d0 + lane * 4;
            float q = 0.f;
            if (d < hidden) {
                const float4 v = *reinterpret_cast<const float4*>(src + d);
                const float4 g = *reinterpret_cast<const float4*>(w + d);
                *reinterpret_cast<float4*>(xr + d) = v;
                store_split4(normed_hi + size_t(row) * hidden + d, normed_lo + size_t(row) * hidden + d,
                             make_float4(__fmul_rn(v.x, g.x), __fmul_rn(v.y, g.y), __fmul_rn(v.z, g.z),
                                         __fmul_rn(v.w, g.w)));
                q = __fmul_rn(v.x, v.x);
                q = fmaf(v.y, v.y, q);
                q = fmaf(v.z, v.z, q);
                q = fmaf(v.w, v.w, q);
            }
            q += __shfl_xor_sync(0xffffffffu, q, 1);
            q += __shfl_xor_sync(0xffffffffu, q, 2);
            q += __shfl_xor_sync(0xffffffffu, q, 4);
            q += __shfl_xor_sync(0xffffffffu, q, 8);
            if ((lane & 15) == 0 && d < hidden) ssq[size_t(row) * (hidden / 64) + d / 64] = q;
        }
        return;
    }
    for (int d = lane * 4; d < hidden; d += 128)
        *reinterpret_cast<float4*>(xr + d) = *reinterpret_cast<const float4*>(src + d);
    __syncwarp();
    rms_row(xr, w, eps, normed_hi + size_t(row) * hidden, normed_lo + size_t(row) * hidden, hidden, lane);
}

__global__ void rmsnorm_kernel(const float* x, const int32_t* rows, const float* w, float eps, __half* out_hi,
                               __half* out_lo, int count, int hidden) {
    pdl_enter();  // before any global memory access
    const int i = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (i >= count) return;
    const int r = rows ? rows[i] : i;
    rms_row(x + size_t(r) * hidden, w, eps, out_hi + size_t(i) * hidden, out_lo + size_t(i) * hidden, hidden, lane);
}

// One CTA of 1024 threads per logits row. First maximum wins (std::max_element):
// candidates compare by value, then by lower index.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* logits, int vocabulary, int32_t* tokens,
                                                      int32_t* finite) {
    pdl_enter();  // before any global memory access
    const int row = blockIdx.x, t = threadIdx.x;
    const float* x = logits + size_t(row) * vocabulary;
    float best = -INFINITY;
    int index = vocabulary;
    bool ok = true;
    for (int i = t; i < vocabulary; i += 1024) {
        const float v = x[i];
        ok &= isfinite(v);
        if (v > best || (index == vocabulary && !(v < best))) {
            best = v;
            index = i;
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int sok[32];
    const int lane = t & 31, warp = t >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, index, o);
        if (ov > best || (ov == best && oi < index)) {
            best = ov;
            index = oi;
        }
    }
    const int all_ok = __all_sync(0xffffffffu, ok);
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = index;
        sok[warp] = all_ok;
    }
    __syncthreads();
    if (warp == 0) {
        best = sv[lane];
        index = si[lane];
        ok = sok[lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, index, o);
            if (ov > best || (ov == best && oi < index)) {
                best = ov;
                index = oi;
            }
        }
        const int fin = __all_sync(0xffffffffu, ok);
        if (lane == 0) {
            tokens[row] = index < vocabulary ? index : 0;
            finite[row] = fin;
        }
    }
}

// grid (count, max_rows): one CTA per (region, layer row), float4 copies of
// `width` floats in both pools (or between the pools and the gather scratch).
// Offsets are validated against the pool and scratch sizes. With a layer-major
// pool a row is copied in pieces that stay inside one page of the reference
// layout, each piece's pool offsets translated (a tail-copy row is one piece).
__global__ void cow_copy_kernel(const CowRegion* regions, float* keys, float* values, uint64_t pool_elements,
                                PoolGeometry g, unsigned* error, int mode, const uint64_t* scratch_offset,
                                float* scratch, uint64_t scratch_elements) {
    pdl_enter();  // before any global memory access
    const CowRegion r = regions[blockIdx.x];
    const uint64_t row = blockIdx.y;
    if (row >= r.rows) return;
    const uint64_t dst = r.destination + row * r.pitch, src = r.source + row * r.pitch;
    const uint64_t at = mode == kCowDirect ? 0 : scratch_offset[blockIdx.x] + row * r.width;
    bool ok = !((r.width | dst | src | at) & 3) && !(g.page_elements & 3) && g.page_elements > 0;
    if (mode != kCowScatter) ok = ok && src + r.width <= pool_elements;
    if (mode != kCowGather) ok = ok && dst + r.width <= pool_elements;
    if (mode != kCowDirect) ok = ok && at + r.width <= scratch_elements && !(scratch_elements & 3);
    if (!ok) {
        if (threadIdx.x == 0) raise_error(error, kErrBounds);
        return;
    }
    const bool pool_src = mode != kCowScatter, pool_dst = mode != kCowGather;
    auto place = [&](uint64_t e) { return g.layers ? layer_major_offset(g, e) : e; };
    for (uint64_t pos = 0; pos < r.width;) {
        uint64_t n = r.width - pos;  // floats in this piece (a multiple of 4)
        if (g.layers) {
            if (pool_src) n = min(n, g.page_elements - (src + pos) % g.page_elements);
            if (pool_dst) n = min(n, g.page_elements - (dst + pos) % g.page_elements);
        }
        const float4 *ks, *vs;
        float4 *kd, *vd;
        if (pool_src) {
            const uint64_t o = place(src + pos);
            ks = reinterpret_cast<const float4*>(keys + o);
            vs = reinterpret_cast<const float4*>(values + o);
        } else {
            ks = reinterpret_cast<const float4*>(scratch + at + pos);
            vs = reinterpret_cast<const float4*>(scratch + scratch_elements + at + pos);
        }
        if (pool_dst) {
            const uint64_t o = place(dst + pos);
            kd = reinterpret_cast<float4*>(keys + o);
            vd = reinterpret_cast<float4*>(values + o);
        } else {
            kd = reinterpret_cast<float4*>(scratch + at + pos);
            vd = reinterpret_cast<float4*>(scratch + scratch_elements + at + pos);
        }
        for (uint64_t i = threadIdx.x; i < n / 4; i += blockDim.x) {
            kd[i] = ks[i];
            vd[i] = vs[i];
        }
        pos += n;
    }
}

__global__ void table_patch_kernel(const int32_t* pairs, int count, int32_t* tables, int64_t elements,
                                   unsigned* error) {
    pdl_enter();  // before any global memory access
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const int64_t index = pairs[2 * i];
    if (index < 0 || index >= elements) {
        raise_error(error, kErrBounds);
        return;
    }
    tables[index] = pairs[2 * i + 1];
}

}  // namespace

cudaError_t launch_embed_rmsnorm(const int32_t* tokens, const float* embed, int vocabulary, const float* norm_w,
                                 float eps, float* x, __half* normed_hi, __half* normed_lo, int rows, int hidden,
                                 float* ssq, unsigned* error, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    if (ssq && hidden % 64) return cudaErrorInvalidValue;
    return launch_pdl(embed_rmsnorm_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream, tokens, embed, vocabulary,
                      norm_w, eps, x, normed_hi, normed_lo, rows, hidden, ssq, error);
}

cudaError_t launch_rmsnorm(const float* x, const int32_t* rows, const float* norm_w, float eps, __half* out_hi,
                           __half* out_lo, int count, int hidden, cudaStream_t stream) {
    if (count <= 0) return cudaSuccess;
    return launch_pdl(rmsnorm_kernel, dim3((count + 7) / 8), dim3(256), 0, stream, x, rows, norm_w, eps, out_hi, out_lo,
                      count, hidden);
}

cudaError_t launch_argmax(const float* logits, int rows, int vocabulary, int32_t* tokens, int32_t* finite,
                          cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(argmax_kernel, dim3(rows), dim3(1024), 0, stream, logits, vocabulary, tokens, finite);
}

cudaError_t launch_cow_copy(const CowRegion* regions, int count, int max_rows, float* keys, float* values,
                            uint64_t pool_elements, const PoolGeometry& geometry, unsigned* error,
                            cudaStream_t stream, CowMode mode, const uint64_t* scratch_offset, float* scratch,
                            uint64_t scratch_elements) {
    if (count <= 0 || max_rows <= 0) return cudaSuccess;
    if (mode != kCowDirect && (!scratch_offset || !scratch)) return cudaErrorInvalidValue;
    if (geometry.layers && (geometry.page_elements == 0 || geometry.max_blocks == 0 ||
                            geometry.page_elements * geometry.layers * geometry.max_blocks != pool_elements))
        return cudaErrorInvalidValue;
    return launch_pdl(cow_copy_kernel, dim3(count, max_rows), dim3(256), 0, stream, regions, keys, values,
                      pool_elements, geometry, error, int(mode), scratch_offset, scratch, scratch_elements);
}

cudaError_t launch_table_patch(const int32_t* pairs, int count, int32_t* tables, int64_t table_elements,
                               unsigned* error, cudaStream_t stream) {
    if (count <= 0) return cudaSuccess;
    return launch_pdl(table_patch_kernel, dim3((count + 255) / 256), dim3(256), 0, stream, pairs, count, tables,
                      table_elements, error);
}

}  // namespace mpb
