// q38_common.cuh -- device helpers shared by the q38attn kernels (sm_100a).
//
// Arithmetic convention: the library is compiled with -fmad=false, so every
// a*b+c written in source stays a separate multiply and add, as in the Rust
// reference (which never contracts). Fused multiply-adds appear only where the
// reference calls f32::mul_add, written explicitly as fmaf / ffma2.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "q38_internal.h"

namespace q38 {

// ---------------------------------------------------------------------------
// Device error flags (bits OR-ed into q38_state::d_err, read by
// q38_state_errors). No kernel traps: a failed check records a bit and the
// kernel skips the work it guards.
// ---------------------------------------------------------------------------
constexpr int kDevErrPosition = 1;   // a position outside [0, context_length)
constexpr int kDevErrTimeout = 2;    // a bounded wait gave up
constexpr int kDevErrShape = 4;      // a launch-shape invariant failed
constexpr int kDevErrRange = 8;      // a V value outside the f16 range of the prefill's P V operand

// Bounded waits give up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;

__device__ __forceinline__ void set_error(int *err, int bit) {
    if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, non-tensor form: contiguous global ranges).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the barrier phase with the given parity to complete, for at most
// limit_ns nanoseconds. Returns false on timeout; the caller records the
// error and abandons the work.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// The same with the library's limit, kWaitTimeoutNs.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    return mbar_wait_ns(bar, parity, kWaitTimeoutNs);
}

// Global -> shared bulk copy completing on `bar` (bytes: multiple of 16,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_load(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Packed f32x2 arithmetic (sm_100a FFMA2): two independent correctly-rounded
// fused multiply-adds per instruction.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(r)
        : "l"(*reinterpret_cast<uint64_t *>(&a)), "l"(*reinterpret_cast<uint64_t *>(&b)),
          "l"(*reinterpret_cast<uint64_t *>(&c)));
    return *reinterpret_cast<float2 *>(&r);
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(*reinterpret_cast<uint64_t *>(&a)), "l"(*reinterpret_cast<uint64_t *>(&b)));
    return *reinterpret_cast<float2 *>(&r);
}

// bf16x2 (one 32-bit word) -> two floats, exactly.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
    float2 r;
    r.x = __uint_as_float(w << 16);
    r.y = __uint_as_float(w & 0xffff0000u);
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

// Block-wide f64 sum for blockDim.x a multiple of 32 (<= 1024). `scratch`
// holds >= 32 doubles. Every thread receives the total.
__device__ __forceinline__ double block_sum_f64(double v, double *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    v = warp_sum_f64(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < warps; ++w) t += scratch[w];
    return t;
}

// The reference's scalar nonlinearities (src/model/ops.rs:500-516), using the
// full-precision CUDA expf/logf (never the fast-math intrinsics).
__device__ __forceinline__ float sigmoidf_ref(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_ref(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplusf_ref(float x) {
    return x > 20.0f ? x : logf(1.0f + expf(x));
}

// rms_scale (ops.rs:476-483) given the f64 sum of squares of n values.
__device__ __forceinline__ float rms_scale_from_sum(double sum, int n, float eps) {
    const float mean = static_cast<float>(sum / static_cast<double>(n));
    return 1.0f / sqrtf(mean + eps);
}

// Two floats -> bf16x2 (round to nearest even), lo in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

template <typename T>
struct KvTraits;
template <>
struct KvTraits<float> {
    static __device__ __forceinline__ float store(float x) { return x; }
};
template <>
struct KvTraits<__nv_bfloat16> {
    static __device__ __forceinline__ __nv_bfloat16 store(float x) { return __float2bfloat16_rn(x); }
};

}  // namespace q38
