// bt_q4.cu -- Q4_0 (4-bit) blocks on the device: quantize, dequantize, matvec,
// and the repack of Q4_0 matrices into the engine's tile layout.
//
// BlockQ4_0 (quantization/quant_types.hpp:17-20) is 20 bytes: an fp32 scale and
// 16 bytes holding 32 4-bit codes, element 2i in the low nibble of byte i and
// element 2i+1 in the high nibble, each code q + 8 for q in [-8, 7].
// quantize_q4_0 (quant_types.cpp:50-79): amax = max |x| (NaN skipped),
// scale = amax / 7, inv = 1 / scale (or 0), code = clamp(int(round_half_away(x
// inv)) + 8, 0, 15); dequantize (:81-99): (code - 8) * scale; matvec_q4_0
// (:123-147): y[r] = sum_b scale * sum_i (code_i - 8) x_i in fp32.
//
// The engine reads Q4_0 matrices by repacking them into its int8 tiles
// (value code - 8, the block's scale): exactly the int8 weights a Q8_0 matrix
// with the same values and scales has, so every decode path runs unchanged on
// them and computes (code - 8) * scale * x as the reference does.
#include "bt_common.cuh"
#include "bt_internal.h"

namespace bt {

__device__ __forceinline__ int q4_to_int_trunc(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT_MIN;  // x86 cvttss2si
    return __float2int_rz(v);
}

// One warp per 32-element block; lane i owns element i.
__global__ void __launch_bounds__(256) quantize_q4_0_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                            uint64_t n_blocks) {
    const uint64_t b = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    const float x = src[b * 32 + lane];
    float amax = warp_max(fmaxf(0.0f, fabsf(x)));
    const float scale = amax / 7.0f;
    const float inv = (scale != 0.0f) ? (1.0f / scale) : 0.0f;
    int q = q4_to_int_trunc(roundf(__fmul_rn(x, inv)));
    q = (q == INT_MIN) ? q : q + 8;
    q = q < 0 ? 0 : (q > 15 ? 15 : q);
    // byte i = code(2i) | code(2i+1) << 4, gathered into four 32-bit words on lanes 0-3
    const uint32_t hi = __shfl_down_sync(0xffffffffu, (uint32_t)q, 1);
    const uint32_t byte = ((uint32_t)q & 15u) | ((hi & 15u) << 4);  // valid on even lanes
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t v = __shfl_sync(0xffffffffu, byte, (lane * 8 + 2 * k) & 31);
        w |= v << (8 * k);
    }
    uint8_t* blk = dst + b * 20;
    if (lane == 0) *reinterpret_cast<float*>(blk) = scale;
    if (lane < 4) *reinterpret_cast<uint32_t*>(blk + 4 + 4 * lane) = w;
}

__global__ void dequantize_q4_0_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t* blk = src + (i >> 5) * 20;
    const float scale = *reinterpret_cast<const float*>(blk);
    const uint32_t e = (uint32_t)(i & 31);
    const uint8_t packed = blk[4 + (e >> 1)];
    const int q = (int)((e & 1) ? (packed >> 4) : (packed & 15)) - 8;
    dst[i] = __fmul_rn(__int2float_rn(q), scale);
}

// One warp per row, lanes over the row's blocks, fp32 accumulation.
__global__ void __launch_bounds__(256) matvec_q4_0_kernel(const uint8_t* __restrict__ W, const float* __restrict__ X,
                                                          float* __restrict__ Y, uint32_t M, uint32_t N) {
    const uint32_t row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const uint32_t bpr = N / 32;
    float acc = 0.0f;
    for (uint32_t b = lane; b < bpr; b += 32) {
        const uint32_t* blk = reinterpret_cast<const uint32_t*>(W + ((size_t)row * bpr + b) * 20);
        const float scale = __uint_as_float(__ldg(blk));
        const float4* xb = reinterpret_cast<const float4*>(X + (size_t)b * 32);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t w = __ldg(blk + 1 + j);  // bytes 4j .. 4j+3 = elements 8j .. 8j+7
            const float4 x0 = __ldg(xb + 2 * j), x1 = __ldg(xb + 2 * j + 1);
            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t byte = (w >> (8 * k)) & 255u;
                const float q0 = (float)((int)(byte & 15u) - 8), q1 = (float)((int)(byte >> 4) - 8);
                s = __fadd_rn(s, __fadd_rn(__fmul_rn(q0, xs[2 * k]), __fmul_rn(q1, xs[2 * k + 1])));
            }
        }
        acc = fmaf(s, scale, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) Y[row] = acc;
}

// One thread per (row, 32-block) of a Q4_0 matrix -> the 4608-byte int8 tiles
// (layout of pack_units_kernel, bt_quant.cu), value code - 8.
__global__ void pack_units_q4_kernel(const uint8_t* __restrict__ blocks, uint8_t* __restrict__ units, uint32_t M,
                                     uint32_t K, RowMap map, uint32_t src_bpr, uint32_t cb0) {
    const uint64_t nb = (uint64_t)M * (K / 32);
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nb) return;
    const uint32_t bpr = K / 32;
    const uint32_t r = (uint32_t)(i / bpr), b = (uint32_t)(i % bpr);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(blocks + ((uint64_t)r * src_bpr + cb0 + b) * 20);
    const uint32_t dr = map_row(r, map);
    const uint32_t rl = dr % 128;
    uint8_t* tile = units + ((uint64_t)(dr / 128) * bpr + b) * 4608;
    reinterpret_cast<uint32_t*>(tile + 4096)[rl] = w[0];
    uint32_t out[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t p = w[1 + j];  // elements 8j .. 8j+7
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t byte = (p >> (8 * k)) & 255u;
            const uint32_t e0 = (uint32_t)((int)(byte & 15u) - 8) & 255u, e1 = (uint32_t)((int)(byte >> 4) - 8) & 255u;
            if (k < 2) lo |= (e0 | (e1 << 8)) << (16 * k);
            else hi |= (e0 | (e1 << 8)) << (16 * (k - 2));
        }
        out[2 * j] = lo;
        out[2 * j + 1] = hi;
    }
    uint8_t* q = tile + (rl / 8) * 256 + (rl % 8) * 16;
    *reinterpret_cast<uint4*>(q) = make_uint4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<uint4*>(q + 128) = make_uint4(out[4], out[5], out[6], out[7]);
}

cudaError_t launch_pack_units_q4(const void* blocks, uint8_t* units, uint32_t M, uint32_t K, RowMap map,
                                 cudaStream_t s, uint32_t src_bpr, uint32_t cb0) {
    const uint64_t nb = (uint64_t)M * (K / 32);
    if (nb == 0) return cudaSuccess;
    if (src_bpr == 0) src_bpr = K / 32;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    pack_units_q4_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>((const uint8_t*)blocks, units, M, K, map,
                                                                        src_bpr, cb0);
    return cudaGetLastError();
}

}  // namespace bt

using namespace bt;

extern "C" {

int bt_cuda_quantize_q4_0(const float* src, void* dst_blocks, uint64_t n, void* stream) {
    if (n % 32 != 0) return fail(BT_ERR_INVALID_ARGUMENT, "quantize_q4_0: num_elements must be a multiple of block size");
    BT_CHECK_ARG(n == 0 || (src && dst_blocks), "quantize_q4_0: null buffer");
    if (n == 0) return BT_OK;
    const uint64_t nb = n / 32;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    quantize_q4_0_kernel<<<(unsigned)((nb + 7) / 8), 256, 0, as_stream(stream)>>>(src, (uint8_t*)dst_blocks, nb);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_dequantize_q4_0(const void* src_blocks, float* dst, uint64_t n, void* stream) {
    BT_CHECK_ARG(n % 32 == 0, "dequantize_q4_0: num_elements must be a multiple of block size");
    BT_CHECK_ARG(n == 0 || (src_blocks && dst), "dequantize_q4_0: null buffer");
    if (n == 0) return BT_OK;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    dequantize_q4_0_kernel<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>((const uint8_t*)src_blocks,
                                                                                       dst, n);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_matvec_q4_0(const void* W_blocks, const float* X, float* Y, uint32_t M, uint32_t N, void* stream) {
    BT_CHECK_ARG(N % 32 == 0, "matvec_q4_0: N must be a multiple of 32");
    BT_CHECK_ARG(W_blocks && X && Y, "matvec_q4_0: null buffer");
    BT_CHECK_ARG(((uintptr_t)W_blocks & 3) == 0 && ((uintptr_t)X & 15) == 0,
                 "matvec_q4_0: W must be 4-byte and X 16-byte aligned");
    if (M == 0) return BT_OK;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    matvec_q4_0_kernel<<<(M + 7) / 8, 256, 0, as_stream(stream)>>>((const uint8_t*)W_blocks, X, Y, M, N);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

}  // extern "C"
