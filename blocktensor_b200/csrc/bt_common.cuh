// bt_common.cuh -- shared device helpers and host error plumbing for the
// sm_100a BlockTensor backend.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <string>

#include "../../include/bt_cuda.h"

namespace bt {

// ---------------------------------------------------------------- host errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
extern std::atomic<uint64_t> g_launches;
// When set, launch helpers configure kernel attributes but launch nothing
// (used once before stream capture, so no attribute call happens while capturing).
extern thread_local bool g_dry_run;

#define BT_CUDA_CHECK(expr)                                                            \
    do {                                                                               \
        cudaError_t _e = (expr);                                                       \
        if (_e != cudaSuccess) {                                                       \
            return ::bt::fail(_e == cudaErrorMemoryAllocation ? BT_ERR_OUT_OF_MEMORY   \
                                                              : BT_ERR_CUDA,           \
                              std::string(#expr) + ": " + cudaGetErrorString(_e));     \
        }                                                                              \
    } while (0)

#define BT_CHECK_ARG(cond, msg)                                      \
    do {                                                             \
        if (!(cond)) return ::bt::fail(BT_ERR_INVALID_ARGUMENT, msg); \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Launch with programmatic dependent launch (PDL) allowed: the kernel may
// start while the previous kernel on the stream drains; it must call
// pdl_wait() before touching anything the previous kernel writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (g_dry_run) return cudaSuccess;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- device helpers

// Wait until the grid this launch depends on has completed and its writes are
// visible (no-op when launched without the PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel on the stream to be scheduled early.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// 16-byte streaming load of weights: read-only path, no L1 allocation,
// 256-byte L2 prefetch.  Weights are read once per token.
__device__ __forceinline__ int4 ld_stream_v4(const void* p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float ld_stream_f32(const float* p) {
    float r;
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(r) : "l"(p));
    return r;
}

// Exact int8 -> fp32 of byte k of a word: build the float 2^23 + (b + 128)
// with a byte permute and subtract 2^23 + 128.  Exact for every byte value.
__device__ __forceinline__ float i8_to_f32(uint32_t w_xor80, int k) {
    uint32_t u = __byte_perm(w_xor80, 0x4B000000u, 0x7540u + (uint32_t)k);
    return __fsub_rn(__uint_as_float(u), 8388736.0f);
}

// Dot product of 16 int8 weights (one 16-byte chunk) with 16 fp32 x values,
// accumulated left to right in fp32.
__device__ __forceinline__ float dot16(int4 w, const float4* x) {
    const uint32_t a = (uint32_t)w.x ^ 0x80808080u, b = (uint32_t)w.y ^ 0x80808080u;
    const uint32_t c = (uint32_t)w.z ^ 0x80808080u, d = (uint32_t)w.w ^ 0x80808080u;
    const float4 x0 = x[0], x1 = x[1], x2 = x[2], x3 = x[3];
    float s = i8_to_f32(a, 0) * x0.x;
    s = fmaf(i8_to_f32(a, 1), x0.y, s);
    s = fmaf(i8_to_f32(a, 2), x0.z, s);
    s = fmaf(i8_to_f32(a, 3), x0.w, s);
    s = fmaf(i8_to_f32(b, 0), x1.x, s);
    s = fmaf(i8_to_f32(b, 1), x1.y, s);
    s = fmaf(i8_to_f32(b, 2), x1.z, s);
    s = fmaf(i8_to_f32(b, 3), x1.w, s);
    s = fmaf(i8_to_f32(c, 0), x2.x, s);
    s = fmaf(i8_to_f32(c, 1), x2.y, s);
    s = fmaf(i8_to_f32(c, 2), x2.z, s);
    s = fmaf(i8_to_f32(c, 3), x2.w, s);
    s = fmaf(i8_to_f32(d, 0), x3.x, s);
    s = fmaf(i8_to_f32(d, 1), x3.y, s);
    s = fmaf(i8_to_f32(d, 2), x3.z, s);
    s = fmaf(i8_to_f32(d, 3), x3.w, s);
    return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Argmax with the reference's tie rule (std::max_element: the first maximum
// wins, NaN never replaces the current best).
__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
    return (bv < v) || (v == bv && i < bi);
}

__device__ __forceinline__ void warp_argmax(float& v, uint32_t& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, v, o);
        uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
}

// Block-wide sum for blockDim.x <= 1024; `red` needs 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.0f;
    if (warp == 0) t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = (threadIdx.x < nw) ? red[threadIdx.x] : -INFINITY;
    if (warp == 0) t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    return red[0];
}

// KV element conversions.
template <typename T> struct KVConv;
template <> struct KVConv<float> {
    __device__ static float load(const float* p) { return *p; }
    __device__ static float to_f(float v) { return v; }
    __device__ static float from_f(float v) { return v; }
};
template <> struct KVConv<__half> {
    __device__ static float to_f(__half v) { return __half2float(v); }
    __device__ static __half from_f(float v) { return __float2half_rn(v); }
};

// Where the K (or V) row of (sequence, KV head, position) of one layer lives, in
// elements from that layer's base pointer.
//   contiguous (table null): every sequence owns [L][KVH][max_seq][hd], so
//     row = seq * seq_stride + (h * max_seq + pos) * hd, the layer's offset in the base;
//   paged: a pool of pages of 2^page_shift positions, a page holding every layer's
//     [KVH][2^page_shift][hd] rows; table[seq * max_pages + pos >> page_shift] names
//     the page of a position, so row = page * page_stride + (h 2^page_shift +
//     pos mod 2^page_shift) * hd, the layer's offset inside a page in the base.
// Callers bound pos by max_seq (positions a sequence may hold) before asking.
struct KVMap {
    const uint32_t* table = nullptr;
    size_t seq_stride = 0;
    size_t page_stride = 0;
    uint32_t max_seq = 0;
    uint32_t max_pages = 0;
    uint32_t page_shift = 0;
    uint32_t hd = 0;
    __host__ __device__ __forceinline__ bool paged() const { return table != nullptr; }
    __device__ __forceinline__ size_t row(uint32_t seq, uint32_t h, uint32_t pos) const {
        if (!table) return (size_t)seq * seq_stride + ((size_t)h * max_seq + pos) * hd;
        const uint32_t pg = __ldg(table + (size_t)seq * max_pages + (pos >> page_shift));
        const uint32_t in_page = pos & ((1u << page_shift) - 1u);
        return (size_t)pg * page_stride + ((size_t)h * (1u << page_shift) + in_page) * hd;
    }
};

// The contiguous map of one sequence's cache [KVH][max_seq][hd] (sequence index 0).
inline KVMap kv_map_flat(uint32_t max_seq, uint32_t hd) {
    KVMap m;
    m.max_seq = max_seq;
    m.hd = hd;
    return m;
}

// Cache element loaded through L2 (rows may have been written by another SM in the same kernel).
__device__ __forceinline__ float ldcg_kv(const float* p) { return __ldcg(p); }
__device__ __forceinline__ __half ldcg_kv(const __half* p) {
    return __ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(p)));
}

}  // namespace bt
