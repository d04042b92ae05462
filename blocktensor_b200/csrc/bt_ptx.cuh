// bt_ptx.cuh -- thin wrappers over the PTX the kernels need: mbarriers,
// 1-D bulk (TMA) copies, named barriers, %globaltimer and the s8 tensor-core
// MMA.  No multicast form of any copy is used anywhere.
#pragma once

#include "bt_common.cuh"

namespace bt {

constexpr uint32_t kWaitNs = 2000000000u;  // every bounded wait gives up after 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase with parity `parity`; false (and *err set) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitNs) {
            if (err) atomicExch(err, 1u);
            return false;
        }
    }
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`
// (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of a global range into L2 (no shared memory, no completion).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Barrier among the first 256 threads of the CTA (named barrier 1).
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// D = A(16x32 s8, row) * B(32x8 s8, col) + 0, 32-bit integer accumulation.
__device__ __forceinline__ void mma_s8_16832(const uint4& a, const uint2& b, int& d0, int& d1, int& d2, int& d3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(0));
}

// Exact int -> float for |v| < 2^22 with two full-rate ops.
__device__ __forceinline__ float small_i2f(int v) {
    return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

}  // namespace bt
