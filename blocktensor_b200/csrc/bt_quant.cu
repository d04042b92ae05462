// bt_quant.cu -- Q8_0 quantize / dequantize / repack and the seeded synthetic
// generators, as sm_100a kernels.
//
// Q8_0 follows quantization/quant_types.cpp:8-48 of the reference bit for bit:
// amax = max |x| over a 32-block, scale = amax / 127 (IEEE division),
// inv = 1 / scale (or 0), q = clamp(int(round_half_away(x * inv)), -128, 127).
#include "bt_common.cuh"
#include "bt_internal.h"

#include <mutex>

namespace bt {

std::atomic<uint64_t> g_launches{0};
thread_local bool g_dry_run = false;

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
    set_error(msg);
    return code;
}

// x86-64 cvttss2si semantics of static_cast<int>(float), which the reference
// relies on (NaN / out-of-range -> INT_MIN, then clamped to -128).
__device__ __forceinline__ int to_int_trunc(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT_MIN;
    return __float2int_rz(v);
}

// One warp per 32-element block.  Lane i owns element i.
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float* __restrict__ src,
                                                            uint8_t* __restrict__ dst,
                                                            uint64_t n_blocks) {
    const uint64_t b = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    const float x = src[b * 32 + lane];
    // std::max(amax, std::abs(x)) skips NaN; fmaxf(0, NaN) = 0 does the same.
    float amax = fmaxf(0.0f, fabsf(x));
    amax = warp_max(amax);
    const float scale = amax / 127.0f;
    const float inv = (scale != 0.0f) ? (1.0f / scale) : 0.0f;
    int q = to_int_trunc(roundf(__fmul_rn(x, inv)));
    q = q < -128 ? -128 : (q > 127 ? 127 : q);
    // gather 4 bytes per lane 0..7 and store 4-byte words (blocks are 4-byte aligned)
    uint32_t byte = (uint32_t)(q & 0xFF);
    uint32_t b0 = __shfl_sync(0xffffffffu, byte, (lane * 4 + 0) & 31);
    uint32_t b1 = __shfl_sync(0xffffffffu, byte, (lane * 4 + 1) & 31);
    uint32_t b2 = __shfl_sync(0xffffffffu, byte, (lane * 4 + 2) & 31);
    uint32_t b3 = __shfl_sync(0xffffffffu, byte, (lane * 4 + 3) & 31);
    uint8_t* blk = dst + b * 36;
    if (lane == 0) *reinterpret_cast<float*>(blk) = scale;
    if (lane < 8) *reinterpret_cast<uint32_t*>(blk + 4 + lane * 4) = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
}

__global__ void dequantize_q8_0_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t* blk = src + (i >> 5) * 36;
    const float scale = *reinterpret_cast<const float*>(blk);
    const int8_t q = (int8_t)blk[4 + (i & 31)];
    dst[i] = __fmul_rn(__int2float_rn(q), scale);
}


// One thread per 32-block: 36-byte block -> 32 int8 (two 16-byte stores) + one scale.
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ blocks, int8_t* __restrict__ qs,
                                   float* __restrict__ scales, uint32_t M, uint32_t K, RowMap map) {
    const uint64_t nb = (uint64_t)M * (K / 32);
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nb) return;
    const uint32_t bpr = K / 32;
    const uint32_t r = (uint32_t)(i / bpr), b = (uint32_t)(i % bpr);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(blocks + i * 36);
    const uint32_t dr = map_row(r, map);
    scales[(uint64_t)dr * bpr + b] = __uint_as_float(w[0]);
    int4* out = reinterpret_cast<int4*>(qs + (uint64_t)dr * K + (uint64_t)b * 32);
    out[0] = make_int4((int)w[1], (int)w[2], (int)w[3], (int)w[4]);
    out[1] = make_int4((int)w[5], (int)w[6], (int)w[7], (int)w[8]);
}

// One thread per (row, 32-block) of a 36-byte-block matrix -> the 4608-byte
// tile layout of the tensor-core GEMV: destination row dr lands in row tile
// dr/128, row rl = dr%128 of tile (dr/128, b); its 32 int8 go to the UMMA
// K-major canonical layout (bytes 0-15 to offset (rl/8)*256 + (rl%8)*16, bytes
// 16-31 to that + 128) and its scale to float rl after the 4096 weight bytes.
// Padding rows stay zero.  The source rows hold src_bpr blocks, of which
// blocks cb0 .. cb0 + K/32 - 1 are packed (a column slice, for tensor
// parallelism; src_bpr = K/32 and cb0 = 0 pack whole rows).
__global__ void pack_units_kernel(const uint8_t* __restrict__ blocks, uint8_t* __restrict__ units, uint32_t M,
                                  uint32_t K, RowMap map, uint32_t src_bpr, uint32_t cb0) {
    const uint64_t nb = (uint64_t)M * (K / 32);
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nb) return;
    const uint32_t bpr = K / 32;
    const uint32_t r = (uint32_t)(i / bpr), b = (uint32_t)(i % bpr);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(blocks + ((uint64_t)r * src_bpr + cb0 + b) * 36);
    const uint32_t dr = map_row(r, map);
    const uint32_t rl = dr % 128;
    uint8_t* tile = units + ((uint64_t)(dr / 128) * bpr + b) * 4608;
    reinterpret_cast<uint32_t*>(tile + 4096)[rl] = w[0];
    uint8_t* q = tile + (rl / 8) * 256 + (rl % 8) * 16;
    *reinterpret_cast<uint4*>(q) = make_uint4(w[1], w[2], w[3], w[4]);
    *reinterpret_cast<uint4*>(q + 128) = make_uint4(w[5], w[6], w[7], w[8]);
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Approximately normal: (sum of four 16-bit uniforms - 131070) * k, exactly as
// the CPU oracle computes it (integer sum, exact int->float, one rounded multiply).
__global__ void gen_normal_kernel(uint64_t base, uint64_t offset, uint64_t n, float k, float* __restrict__ out) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t h = splitmix64(base + offset + i);
        const int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) +
                          (int32_t)((h >> 32) & 0xFFFF) + (int32_t)(h >> 48);
        out[i] = __fmul_rn(__int2float_rn(s - 131070), k);
    }
}

__global__ void fill_kernel(float* out, uint64_t n, float v) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = v;
}

uint64_t splitmix64_host(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t stream_base_host(uint64_t seed, uint64_t stream) {
    return splitmix64_host(splitmix64_host(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}

float normal_k(float sigma) { return (float)((double)sigma / 37837.22712838299); }

static unsigned grid_for(uint64_t n, unsigned block, unsigned cap = 148u * 64u) {
    uint64_t g = (n + block - 1) / block;
    if (g > cap) g = cap;
    if (g == 0) g = 1;
    return (unsigned)g;
}

cudaError_t launch_quantize_q8_0(const float* src, void* dst, uint64_t n_blocks, cudaStream_t s) {
    if (n_blocks == 0) return cudaSuccess;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    quantize_q8_0_kernel<<<(unsigned)((n_blocks + 7) / 8), 256, 0, s>>>(src, (uint8_t*)dst, n_blocks);
    return cudaGetLastError();
}

cudaError_t launch_dequantize_q8_0(const void* src, float* dst, uint64_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    dequantize_q8_0_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_repack_q8_0(const void* blocks, int8_t* qs, float* scales, uint32_t M, uint32_t K,
                               RowMap map, cudaStream_t s) {
    const uint64_t nb = (uint64_t)M * (K / 32);
    if (nb == 0) return cudaSuccess;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    repack_q8_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>((const uint8_t*)blocks, qs, scales, M, K, map);
    return cudaGetLastError();
}

cudaError_t launch_pack_units(const void* blocks, uint8_t* units, uint32_t M, uint32_t K, RowMap map,
                              cudaStream_t s, uint32_t src_bpr, uint32_t cb0) {
    const uint64_t nb = (uint64_t)M * (K / 32);
    if (nb == 0) return cudaSuccess;
    if (src_bpr == 0) src_bpr = K / 32;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    pack_units_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>((const uint8_t*)blocks, units, M, K, map,
                                                                     src_bpr, cb0);
    return cudaGetLastError();
}

cudaError_t launch_gen_normal(uint64_t seed, uint64_t stream_id, uint64_t offset, uint64_t n, float k,
                              float* out, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    gen_normal_kernel<<<grid_for(n, 256), 256, 0, s>>>(stream_base_host(seed, stream_id), offset, n, k, out);
    return cudaGetLastError();
}

cudaError_t launch_fill(float* out, uint64_t n, float v, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(out, n, v);
    return cudaGetLastError();
}

}  // namespace bt

using namespace bt;

extern "C" {

int bt_cuda_abi_version(void) { return BT_ABI_VERSION; }
const char* bt_cuda_last_error(void) { return t_last_error.c_str(); }
uint64_t bt_cuda_launch_count(void) { return g_launches.load(); }

int bt_cuda_quantize_q8_0(const float* src, void* dst_blocks, uint64_t n, void* stream) {
    if (n % 32 != 0) return fail(BT_ERR_INVALID_ARGUMENT, "quantize_q8_0: num_elements must be a multiple of block size");
    BT_CHECK_ARG(n == 0 || (src && dst_blocks), "quantize_q8_0: null buffer");
    BT_CHECK_ARG(((uintptr_t)dst_blocks & 3) == 0, "quantize_q8_0: dst must be 4-byte aligned");
    BT_CUDA_CHECK(launch_quantize_q8_0(src, dst_blocks, n / 32, as_stream(stream)));
    return BT_OK;
}

int bt_cuda_dequantize_q8_0(const void* src_blocks, float* dst, uint64_t n, void* stream) {
    BT_CHECK_ARG(n % 32 == 0, "dequantize_q8_0: num_elements must be a multiple of block size");
    BT_CHECK_ARG(n == 0 || (src_blocks && dst), "dequantize_q8_0: null buffer");
    BT_CHECK_ARG(((uintptr_t)src_blocks & 3) == 0, "dequantize_q8_0: src must be 4-byte aligned");
    BT_CUDA_CHECK(launch_dequantize_q8_0(src_blocks, dst, n, as_stream(stream)));
    return BT_OK;
}

int bt_cuda_pack_q8_units(const void* W_blocks, void* units, uint32_t M, uint32_t K, void* stream) {
    BT_CHECK_ARG(K % 32 == 0, "pack_q8_units: K must be a multiple of 32");
    BT_CHECK_ARG(W_blocks && units, "pack_q8_units: null buffer");
    BT_CHECK_ARG(((uintptr_t)W_blocks & 3) == 0 && ((uintptr_t)units & 15) == 0,
                 "pack_q8_units: misaligned buffer (blocks 4 B, units 16 B)");
    BT_CUDA_CHECK(cudaMemsetAsync(units, 0, unit_bytes(M, K), as_stream(stream)));
    BT_CUDA_CHECK(launch_pack_units(W_blocks, static_cast<uint8_t*>(units), M, K, RowMap{0, 0, 0, 0, 0},
                                    as_stream(stream)));
    return BT_OK;
}

int bt_cuda_repack_q8_0(const void* W_blocks, int8_t* qs, float* scales, uint32_t M, uint32_t K, void* stream) {
    BT_CHECK_ARG(K % 32 == 0, "repack_q8_0: K must be a multiple of 32");
    BT_CHECK_ARG(W_blocks && qs && scales, "repack_q8_0: null buffer");
    BT_CHECK_ARG(((uintptr_t)W_blocks & 3) == 0 && ((uintptr_t)qs & 15) == 0 && ((uintptr_t)scales & 3) == 0,
                 "repack_q8_0: misaligned buffer (blocks 4 B, qs 16 B, scales 4 B)");
    BT_CUDA_CHECK(launch_repack_q8_0(W_blocks, qs, scales, M, K, RowMap{0, 0, 0, 0, 0}, as_stream(stream)));
    return BT_OK;
}

}  // extern "C"
