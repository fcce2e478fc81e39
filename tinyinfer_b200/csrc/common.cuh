// Shared device helpers for the sm_100a kernels: bulk-copy (TMA engine) staging
// through mbarriers with bounded waits, warp reductions, and the device error word.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace mpb {

// Bounds of an mbarrier wait: at most kWaitNanoseconds of wall time (read from
// %globaltimer) and at most kWaitLimit polls, whichever comes first.
constexpr uint64_t kWaitNanoseconds = 2000000000ull;
constexpr uint32_t kWaitLimit = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait. Returns false (and the caller must record kErrTimeout) when the
// phase did not complete within `limit_ns` of wall time (default
// kWaitNanoseconds) or kWaitLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitNanoseconds) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && global_ns() - start > limit_ns) return false;
    }
    return false;
}

// One bulk global->shared copy completing on `bar`. dst, src 16-byte aligned;
// bytes a positive multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Packed FP32: (a0, a1) = (b0 * c0 + a0, b1 * c1 + a1), each an IEEE fused
// multiply-add (fma.rn.f32x2, sm_100).
__device__ __forceinline__ void fma2(float& a0, float& a1, float b0, float b1, float c0, float c1) {
    asm("{\n\t.reg .b64 pa, pb, pc;\n\t"
        "mov.b64 pa, {%2, %3};\n\t"
        "mov.b64 pb, {%4, %5};\n\t"
        "mov.b64 pc, {%0, %1};\n\t"
        "fma.rn.f32x2 pc, pa, pb, pc;\n\t"
        "mov.b64 {%0, %1}, pc;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// log2(e): softmax weights are evaluated as exp2 of scores pre-scaled by it
// (exp(x) = 2^(x log2 e)); running maxima are kept in the same base-2 units.
constexpr float kLog2e = 1.4426950408889634f;

// TF32 hi/lo split: hi keeps sign, exponent and the 10 leading mantissa bits
// (exact in TF32), lo = x - hi is exact in FP32.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    lo = __fsub_rn(x, hi);
}

// FP16 operand halves of the tensor-core GEMMs: hi = x rounded to FP16, lo = the
// remainder x - hi (exact in FP32) scaled by 2^11 and rounded to FP16, so that
// x = hi + lo * 2^-11 within about 2^-23 |x| (kernels.h, kSplitLoScale).
__device__ __forceinline__ void split_f16(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(__fmul_rn(__fsub_rn(x, __half2float(hi)), kSplitLoScale));
}

__device__ __forceinline__ uint32_t pack_half2(__half a, __half b) {
    return uint32_t(__half_as_ushort(a)) | (uint32_t(__half_as_ushort(b)) << 16);
}

// Halves of 4 consecutive values at hi[0..3] / lo[0..3] (8-byte aligned).
__device__ __forceinline__ void store_split4(__half* hi, __half* lo, float4 v) {
    __half h[4], l[4];
    split_f16(v.x, h[0], l[0]);
    split_f16(v.y, h[1], l[1]);
    split_f16(v.z, h[2], l[2]);
    split_f16(v.w, h[3], l[3]);
    *reinterpret_cast<uint2*>(hi) = make_uint2(pack_half2(h[0], h[1]), pack_half2(h[2], h[3]));
    *reinterpret_cast<uint2*>(lo) = make_uint2(pack_half2(l[0], l[1]), pack_half2(l[2], l[3]));
}

// Halves of 2 consecutive values (4-byte aligned).
__device__ __forceinline__ void store_split2(__half* hi, __half* lo, float a, float b) {
    __half h0, l0, h1, l1;
    split_f16(a, h0, l0);
    split_f16(b, h1, l1);
    *reinterpret_cast<uint32_t*>(hi) = pack_half2(h0, h1);
    *reinterpret_cast<uint32_t*>(lo) = pack_half2(l0, l1);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void raise_error(unsigned* error, unsigned bits) {
    if (error) atomicOr(error, bits);
}

// Programmatic dependent launch. Kernels of the forward are launched with
// programmatic stream serialisation: a kernel may start while its predecessor
// finishes, runs only work that touches no memory of earlier kernels, then waits
// (pdl_wait) until the predecessor completed and its writes are visible. Once
// past the wait a kernel lets its own successor launch (pdl_trigger), so at most
// two kernels of the chain overlap. Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
    pdl_wait();
    pdl_trigger();
}

// Host: launch `kernel` with programmatic stream serialisation.
template <class... Params, class... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

}  // namespace mpb
