// bt_internal.h -- host-side declarations shared between the .cu files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace bt {

// Row permutation applied while repacking a matrix into the device layout.
struct RowMap {
    int mode;          // 0 identity, 1 RoPE pair interleave within heads, 2 stride-2 interleave
    uint32_t hd;       // head_dim for mode 1
    uint32_t parity;   // 0/1 for mode 2
    uint32_t src_off;  // row index of the first source row (slab offset)
    uint32_t dst_off;  // added to the mapped row
};

#ifdef __CUDACC__
// Destination row of source row `local` of a repacked matrix.
__device__ __forceinline__ uint32_t map_row(uint32_t local, RowMap m) {
    const uint32_t r = local + m.src_off;
    uint32_t d = r;
    if (m.mode == 1) {
        const uint32_t h = r / m.hd, i = r % m.hd, half = m.hd / 2;
        d = h * m.hd + (i < half ? 2 * i : 2 * (i - half) + 1);
    } else if (m.mode == 2) {
        d = 2 * r + m.parity;
    }
    return d + m.dst_off;
}
#endif

// Launchers (stream-ordered, no synchronisation).  Return cudaError_t of the launch.
cudaError_t launch_quantize_q8_0(const float* src, void* dst, uint64_t n_blocks, cudaStream_t s);
cudaError_t launch_dequantize_q8_0(const void* src, float* dst, uint64_t n, cudaStream_t s);
cudaError_t launch_repack_q8_0(const void* blocks, int8_t* qs, float* scales, uint32_t M, uint32_t K,
                               RowMap map, cudaStream_t s);
// 36-byte blocks -> 576-byte mma units (rows padded to 16; the caller zeroes padding).
// src_bpr: blocks per source row (0: K/32); cb0: first packed block of each source row.
cudaError_t launch_pack_units(const void* blocks, uint8_t* units, uint32_t M, uint32_t K, RowMap map,
                              cudaStream_t s, uint32_t src_bpr = 0, uint32_t cb0 = 0);
// The same from 20-byte Q4_0 blocks (values code - 8, bt_q4.cu).
cudaError_t launch_pack_units_q4(const void* blocks, uint8_t* units, uint32_t M, uint32_t K, RowMap map,
                                 cudaStream_t s, uint32_t src_bpr = 0, uint32_t cb0 = 0);
inline uint64_t unit_bytes(uint32_t M, uint32_t K) { return (uint64_t)((M + 127) / 128) * (K / 32) * 4608; }
cudaError_t launch_gen_normal(uint64_t seed, uint64_t stream_id, uint64_t offset, uint64_t n, float k,
                              float* out, cudaStream_t s);
cudaError_t launch_fill(float* out, uint64_t n, float v, cudaStream_t s);

// Standalone tensor-core GEMV: waits for the call on stream s and turns its
// bounded-wait flag into BT_ERR_DEVICE_TIMEOUT (clearing flag and tickets).
int gemv_check_timeout(uint32_t* flag, uint32_t* tickets, size_t ticket_bytes, cudaStream_t s);
// Sets the no-alloc GEMV's bounded-wait flag on `device` (host-side fault injection for tests).
int noalloc_inject_timeout(int device);

// The multi-token tensor-core GEMM (bt_prefill.cu): token image of X [T][K] into the
// workspace ws (gemm_units_scratch bytes: the image, then split-K partial sums), then
// Y [T][M] = X W^T.
cudaError_t gemm_units_launch(const void* units, const float* X, float* Y, uint32_t M, uint32_t K, uint32_t T,
                              uint8_t* ws, uint32_t* err, uint32_t nsm, cudaStream_t s);
size_t gemm_units_scratch(uint32_t K, uint32_t T, uint32_t nsm);

// Same formula as the CPU oracle (oracle/bt_oracle.c bto_normal_k).
float normal_k(float sigma);
uint64_t splitmix64_host(uint64_t z);
uint64_t stream_base_host(uint64_t seed, uint64_t stream);

}  // namespace bt
