// bt_prims.cu -- standalone device versions of the reference's CPU kernels
// (kernels/cpu_ref.hpp, sampler.hpp, quant_types.cpp matvec) and the batched
// int8 GEMV.  The decode engine uses the fused kernels of bt_gemv.cuh and
// bt_engine.cu; these entry points serve the pipeline-by-name dispatch of the
// backend (the shader names of transformer_engine.cpp:56-64) and the
// kernel-level parity tests.
#include "bt_common.cuh"
#include "bt_gemv.cuh"
#include "bt_gemv_mma.cuh"
#include "bt_internal.h"

#include <mutex>

namespace bt {

// Per-device workspace of the standalone tensor-core GEMV: partial sums of
// row groups cut between two CTAs ([num_sms][32] floats), their tickets
// ([num_sms], zero between launches) and the bounded-wait error flag.
constexpr uint32_t kWsTickets = 8192;  // row tiles: M <= 1048576

struct GemvWorkspace {
    float* part = nullptr;       // [num_sms][2][128] partial sums of split row tiles
    uint32_t* ticket = nullptr;  // kWsTickets tickets followed by the error flag
    uint32_t nsm = 0;
};

static std::mutex g_ws_mutex;
static GemvWorkspace g_ws[64];

static int gemv_workspace(int dev, GemvWorkspace** out) {
    if (dev < 0 || dev >= 64) return fail(BT_ERR_INVALID_ARGUMENT, "gemv workspace: device index out of range");
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    GemvWorkspace& w = g_ws[dev];
    if (!w.part) {
        int nsm = 0;
        BT_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
        float* part = nullptr;
        uint32_t* ticket = nullptr;
        BT_CUDA_CHECK(cudaMalloc(&part, sizeof(float) * 2 * kTileRows * nsm));
        cudaError_t e = cudaMalloc(&ticket, sizeof(uint32_t) * (kWsTickets + 1));
        if (e == cudaSuccess) e = cudaMemset(ticket, 0, sizeof(uint32_t) * (kWsTickets + 1));
        if (e != cudaSuccess) {
            cudaFree(part);
            if (ticket) cudaFree(ticket);
            return fail(BT_ERR_CUDA, std::string("gemv workspace: ") + cudaGetErrorString(e));
        }
        w.part = part;
        w.ticket = ticket;
        w.nsm = (uint32_t)nsm;
    }
    *out = &w;
    return BT_OK;
}

// After a standalone tensor-core GEMV on stream s: waits for it and reads its
// bounded-wait flag.  A set flag means a wait inside the kernel gave up after
// its 2 s limit, so y is not valid; the flag and the arrival tickets (which an
// interrupted call may leave mid-count) are then cleared for the next call and
// BT_ERR_DEVICE_TIMEOUT is returned.
int gemv_check_timeout(uint32_t* flag, uint32_t* tickets, size_t ticket_bytes, cudaStream_t s) {
    uint32_t h = 0;
    BT_CUDA_CHECK(cudaStreamSynchronize(s));
    BT_CUDA_CHECK(cudaMemcpy(&h, flag, sizeof(h), cudaMemcpyDeviceToHost));
    if (h == 0) return BT_OK;
    BT_CUDA_CHECK(cudaMemsetAsync(tickets, 0, ticket_bytes, s));
    BT_CUDA_CHECK(cudaMemsetAsync(flag, 0, sizeof(uint32_t), s));
    BT_CUDA_CHECK(cudaStreamSynchronize(s));
    return fail(BT_ERR_DEVICE_TIMEOUT, "gemv_q8_units: a device wait timed out; the output is not valid");
}

// cpu_ref::rmsnorm (cpu_ref.hpp:11-28): one CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ in, const float* __restrict__ w,
                                                      float* __restrict__ out, uint32_t dim, float eps) {
    __shared__ float red[32];
    const float* x = in + (size_t)blockIdx.x * dim;
    float* o = out + (size_t)blockIdx.x * dim;
    float ss = 0.0f;
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) ss = fmaf(x[d], x[d], ss);
    ss = block_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) o[d] = __fmul_rn(__fmul_rn(x[d], inv), w[d]);
}

// cpu_ref::rope (cpu_ref.hpp:30-53): one thread per rotation pair; the base is a parameter.
__global__ void rope_kernel(const float* __restrict__ in, float* __restrict__ out, uint32_t seq, uint32_t heads,
                            uint32_t hd, uint32_t pos0, float theta) {
    const uint32_t half = hd / 2;
    const uint64_t n = (uint64_t)seq * heads * half;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t p = (uint32_t)(i % half);
    const uint64_t sh = i / half;  // s * heads + h
    const uint32_t s = (uint32_t)(sh / heads);
    const float freq = __fdiv_rn(1.0f, powf(theta, __fdiv_rn((float)(2 * p), (float)hd)));
    const float val = __fmul_rn((float)(s + pos0), freq);
    const float c = cosf(val), sn = sinf(val);
    const float* ih = in + sh * hd;
    float* oh = out + sh * hd;
    const float x1 = ih[p], x2 = ih[p + half];
    oh[p] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    oh[p + half] = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, c));
}

// cpu_ref::softmax (cpu_ref.hpp:55-72): one CTA per row.
__global__ void __launch_bounds__(256) softmax_kernel(const float* __restrict__ in, float* __restrict__ out,
                                                      uint32_t dim) {
    __shared__ float red[32];
    const float* x = in + (size_t)blockIdx.x * dim;
    float* o = out + (size_t)blockIdx.x * dim;
    float m = -INFINITY;
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) m = fmaxf(m, x[d]);
    m = block_max(m, red);
    float s = 0.0f;
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) {
        const float e = expf(x[d] - m);
        o[d] = e;
        s += e;
    }
    s = block_sum(s, red);
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) o[d] = __fdiv_rn(o[d], s);
}

// cpu_ref::silu (cpu_ref.hpp:74-79)
__global__ void silu_kernel(const float* __restrict__ in, float* __restrict__ out, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float x = in[i];
        out[i] = __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
    }
}

// sampling::sample_greedy (sampler.hpp:11-13): one CTA, first maximum wins.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, uint32_t n, uint32_t* out) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
        if (bi == 0xFFFFFFFFu || better(x[i], i, bv, bi)) { bv = x[i]; bi = i; }
    warp_argmax(bv, bi);
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = sv[0];
        uint32_t ix = si[0];
        for (uint32_t w = 1; w < blockDim.x / 32; ++w)
            if (si[w] != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || better(sv[w], si[w], v, ix))) { v = sv[w]; ix = si[w]; }
        *out = ix == 0xFFFFFFFFu ? 0 : ix;
    }
}

// quantization::matvec_q8_0 on the reference's 36-byte blocks
// (quant_types.cpp:101-121): one warp per row, lanes over blocks, block dot
// accumulated in element order then scaled, as the reference does.
__global__ void __launch_bounds__(256) matvec_aos_kernel(const uint8_t* __restrict__ W, const float* __restrict__ X,
                                                         float* __restrict__ Y, uint32_t M, uint32_t N) {
    const uint32_t row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const uint32_t bpr = N / 32;
    float acc = 0.0f;
    for (uint32_t b = lane; b < bpr; b += 32) {
        const uint32_t* blk = reinterpret_cast<const uint32_t*>(W + ((size_t)row * bpr + b) * 36);
        const float scale = __uint_as_float(__ldg(blk));
        const float4* xb = reinterpret_cast<const float4*>(X + (size_t)b * 32);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t w = __ldg(blk + 1 + j) ^ 0x80808080u;
            const float4 xv = __ldg(xb + j);
            s = fmaf(i8_to_f32(w, 0), xv.x, s);
            s = fmaf(i8_to_f32(w, 1), xv.y, s);
            s = fmaf(i8_to_f32(w, 2), xv.z, s);
            s = fmaf(i8_to_f32(w, 3), xv.w, s);
        }
        acc = fmaf(s, scale, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) Y[row] = acc;
}

// Batched GEMV, B > 1: 8 rows per CTA (one warp each), x staged in shared
// memory in K tiles of at most 64 KB; each 16-byte weight chunk is converted
// once and used for all B right-hand sides.
template <int B>
__global__ void __launch_bounds__(256) gemv_batch_kernel(const int8_t* __restrict__ qs, const float* __restrict__ sc,
                                                         const float* __restrict__ X, float* __restrict__ Y,
                                                         uint32_t M, uint32_t K, uint32_t nb) {
    constexpr uint32_t KT = 16384 / B;  // floats per batch row per tile (64 KB total)
    extern __shared__ float4 smem4[];
    float* xs = reinterpret_cast<float*>(smem4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * 8 + warp;
    const bool ok = row < M;
    const int8_t* wrow = qs + (size_t)(ok ? row : 0) * K;
    const float* srow = sc + (size_t)(ok ? row : 0) * (K / 32);
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.0f;
    for (uint32_t k0 = 0; k0 < K; k0 += KT) {
        const uint32_t kt = min(KT, K - k0);
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < nb * kt / 4; i += blockDim.x) {
            const uint32_t b = i / (kt / 4), j = i % (kt / 4);
            reinterpret_cast<float4*>(xs)[b * (KT / 4) + j] = reinterpret_cast<const float4*>(X + (size_t)b * K + k0)[j];
        }
        __syncthreads();
        if (!ok) continue;
        for (uint32_t c = lane; c < kt / 16; c += 32) {
            const int4 w = ld_stream_v4(wrow + k0 + (size_t)c * 16);
            const float s = ld_stream_f32(srow + ((k0 / 16 + c) >> 1));
            float f[16];
            const uint32_t ww[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u,
                                    (uint32_t)w.z ^ 0x80808080u, (uint32_t)w.w ^ 0x80808080u};
#pragma unroll
            for (int j = 0; j < 16; ++j) f[j] = i8_to_f32(ww[j >> 2], j & 3);
#pragma unroll
            for (int b = 0; b < B; ++b) {
                if ((uint32_t)b >= nb) break;
                const float4* xv = reinterpret_cast<const float4*>(xs + b * KT + c * 16);
                float d = 0.0f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 v = xv[q];
                    d = fmaf(f[4 * q + 0], v.x, d);
                    d = fmaf(f[4 * q + 1], v.y, d);
                    d = fmaf(f[4 * q + 2], v.z, d);
                    d = fmaf(f[4 * q + 3], v.w, d);
                }
                acc[b] = fmaf(d, s, acc[b]);
            }
        }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
        const float v = warp_sum(acc[b]);
        if (ok && lane == 0 && (uint32_t)b < nb) Y[(size_t)b * M + row] = v;
    }
}

template <int B>
static cudaError_t launch_gemv_batch(const int8_t* qs, const float* sc, const float* X, float* Y, uint32_t M,
                                     uint32_t K, uint32_t nb, cudaStream_t s) {
    auto kern = gemv_batch_kernel<B>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    kern<<<(M + 7) / 8, 256, 64 * 1024, s>>>(qs, sc, X, Y, M, K, nb);
    return cudaGetLastError();
}

}  // namespace bt

using namespace bt;

extern "C" {

int bt_cuda_device_info(int device, char* name, uint64_t* total_bytes, uint32_t* max_threads_per_block,
                        uint32_t* max_shared_bytes) {
    cudaDeviceProp p;
    BT_CUDA_CHECK(cudaGetDeviceProperties(&p, device));
    if (name) {
        snprintf(name, 256, "%s", p.name);
    }
    if (total_bytes) *total_bytes = p.totalGlobalMem;
    if (max_threads_per_block) *max_threads_per_block = (uint32_t)p.maxThreadsPerBlock;
    if (max_shared_bytes) *max_shared_bytes = (uint32_t)p.sharedMemPerBlockOptin;
    return BT_OK;
}

int bt_cuda_alloc(int device, uint64_t bytes, void** ptr) {
    BT_CHECK_ARG(ptr, "alloc: null output");
    BT_CUDA_CHECK(cudaSetDevice(device));
    void* p = nullptr;
    BT_CUDA_CHECK(cudaMalloc(&p, bytes ? bytes : 16));
    cudaError_t e = cudaMemset(p, 0, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(BT_ERR_CUDA, cudaGetErrorString(e));
    }
    *ptr = p;
    return BT_OK;
}

int bt_cuda_free(int device, void* ptr) {
    if (!ptr) return BT_OK;
    BT_CUDA_CHECK(cudaSetDevice(device));
    BT_CUDA_CHECK(cudaFree(ptr));
    return BT_OK;
}

int bt_cuda_copy_h2d(int device, void* dst, const void* src, uint64_t bytes) {
    BT_CHECK_ARG(bytes == 0 || (dst && src), "copy_h2d: null buffer");
    BT_CUDA_CHECK(cudaSetDevice(device));
    BT_CUDA_CHECK(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return BT_OK;
}

int bt_cuda_copy_d2h(int device, void* dst, const void* src, uint64_t bytes) {
    BT_CHECK_ARG(bytes == 0 || (dst && src), "copy_d2h: null buffer");
    BT_CUDA_CHECK(cudaSetDevice(device));
    BT_CUDA_CHECK(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return BT_OK;
}

int bt_cuda_synchronize(int device) {
    BT_CUDA_CHECK(cudaSetDevice(device));
    BT_CUDA_CHECK(cudaDeviceSynchronize());
    return BT_OK;
}

int bt_cuda_rmsnorm(const float* in, const float* w, float* out, uint32_t rows, uint32_t dim, float eps,
                    void* stream) {
    BT_CHECK_ARG(in && w && out, "rmsnorm: null buffer");
    if (rows == 0 || dim == 0) return BT_OK;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    rmsnorm_kernel<<<rows, 256, 0, as_stream(stream)>>>(in, w, out, dim, eps);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_rope(const float* in, float* out, uint32_t seq, uint32_t heads, uint32_t head_dim, uint32_t pos,
                 float theta, void* stream) {
    BT_CHECK_ARG(in && out, "rope: null buffer");
    BT_CHECK_ARG(head_dim % 2 == 0, "rope: head_dim must be even");
    const uint64_t n = (uint64_t)seq * heads * (head_dim / 2);
    if (n == 0) return BT_OK;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(in, out, seq, heads, head_dim, pos, theta);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_softmax(const float* in, float* out, uint32_t rows, uint32_t dim, void* stream) {
    BT_CHECK_ARG(in && out, "softmax: null buffer");
    if (rows == 0 || dim == 0) return BT_OK;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    softmax_kernel<<<rows, 256, 0, as_stream(stream)>>>(in, out, dim);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_silu(const float* in, float* out, uint32_t n, void* stream) {
    BT_CHECK_ARG(in && out, "silu: null buffer");
    if (n == 0) return BT_OK;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    silu_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(in, out, n);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_argmax(const float* logits, uint32_t n, uint32_t* out, void* stream) {
    BT_CHECK_ARG(logits && out, "argmax: null buffer");
    BT_CHECK_ARG(n > 0, "argmax: empty input");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    argmax_kernel<<<1, 1024, 0, as_stream(stream)>>>(logits, n, out);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_matvec_q8_0(const void* W_blocks, const float* X, float* Y, uint32_t M, uint32_t N, void* stream) {
    BT_CHECK_ARG(N % 32 == 0, "matvec_q8_0: N must be a multiple of 32");
    BT_CHECK_ARG(W_blocks && X && Y, "matvec_q8_0: null buffer");
    BT_CHECK_ARG(((uintptr_t)W_blocks & 3) == 0 && ((uintptr_t)X & 15) == 0,
                 "matvec_q8_0: W must be 4-byte and X 16-byte aligned");
    if (M == 0) return BT_OK;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    matvec_aos_kernel<<<(M + 7) / 8, 256, 0, as_stream(stream)>>>((const uint8_t*)W_blocks, X, Y, M, N);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}

int bt_cuda_gemv_q8_units(const void* units, const float* x, float* y, uint32_t M, uint32_t K, void* stream) {
    BT_CHECK_ARG(K % 32 == 0 && K > 0, "gemv_q8_units: K must be a positive multiple of 32");
    BT_CHECK_ARG(K <= kGemvMaxK, "gemv_q8_units: K above 48384 not supported");
    BT_CHECK_ARG(units && x && y, "gemv_q8_units: null buffer");
    BT_CHECK_ARG(((uintptr_t)units & 15) == 0 && ((uintptr_t)x & 15) == 0,
                 "gemv_q8_units: units and x must be 16-byte aligned");
    BT_CHECK_ARG(M <= kWsTickets * kTileRows, "gemv_q8_units: M above 1048576 rows not supported");
    if (M == 0) return BT_OK;
    int dev = 0;
    BT_CUDA_CHECK(cudaGetDevice(&dev));
    GemvWorkspace* ws = nullptr;
    int rc = gemv_workspace(dev, &ws);
    if (rc != BT_OK) return rc;
    const UnitW w{static_cast<const uint8_t*>(units), M, unit_rows(M), K};
    cudaStream_t s = as_stream(stream);
    BT_CUDA_CHECK(launch_gemv_mma(w, MProCopy{x}, SEpiStore{y}, SplitScratch{ws->part, ws->ticket},
                                  ws->ticket + kWsTickets, ws->nsm, s, false));
    return gemv_check_timeout(ws->ticket + kWsTickets, ws->ticket, sizeof(uint32_t) * kWsTickets, s);
}

int bt_cuda_gemv_bench(int kind, const void* w, const float* X, float* Y, uint32_t M, uint32_t K, uint32_t B,
                       uint32_t n_copies, uint64_t copy_stride, uint32_t iters, void* stream, float* us_per_call) {
    BT_CHECK_ARG(w && X && Y && us_per_call, "gemv_bench: null argument");
    BT_CHECK_ARG(K % 32 == 0 && K > 0 && K <= kGemvMaxK && M > 0, "gemv_bench: bad shape");
    BT_CHECK_ARG(n_copies >= 1 && iters >= 1 && B >= 1, "gemv_bench: bad count");
    BT_CHECK_ARG(kind != 0 || B == 1, "gemv_bench: the tile-layout GEMV takes one vector");
    BT_CHECK_ARG(kind != 2 || B <= 16, "gemv_bench: the split-layout GEMV takes at most 16 vectors");
    BT_CHECK_ARG(kind >= 0 && kind <= 2, "gemv_bench: kind must be 0, 1 or 2");
    BT_CHECK_ARG(M <= kWsTickets * kTileRows, "gemv_bench: M too large");
    cudaStream_t s = as_stream(stream);
    int dev = 0;
    BT_CUDA_CHECK(cudaGetDevice(&dev));
    GemvWorkspace* ws = nullptr;
    int rc = gemv_workspace(dev, &ws);
    if (rc != BT_OK) return rc;
    uint8_t* img = nullptr;
    if (kind == 1) BT_CUDA_CHECK(cudaMallocAsync(reinterpret_cast<void**>(&img), gemm_units_scratch(K, B, ws->nsm), s));
    cudaEvent_t e0, e1;
    BT_CUDA_CHECK(cudaEventCreate(&e0));
    BT_CUDA_CHECK(cudaEventCreate(&e1));
    auto one = [&](uint32_t i) -> cudaError_t {
        const uint8_t* wi = static_cast<const uint8_t*>(w) + (uint64_t)(i % n_copies) * copy_stride;
        if (kind == 0)
            return launch_gemv_mma(UnitW{wi, M, unit_rows(M), K}, MProCopy{X}, SEpiStore{Y},
                                   SplitScratch{ws->part, ws->ticket}, ws->ticket + kWsTickets, ws->nsm, s, false);
        if (kind == 1) return gemm_units_launch(wi, X, Y, M, K, B, img, ws->ticket + kWsTickets, ws->nsm, s);
        const int8_t* qs = reinterpret_cast<const int8_t*>(wi);
        const float* sc = reinterpret_cast<const float*>(wi + (uint64_t)M * K);
        if (B == 1) return launch_gemv(GemvW{qs, sc, M, K}, ProCopy{X}, EpiStore{Y}, s, false);
        if (B == 2) return launch_gemv_batch<2>(qs, sc, X, Y, M, K, B, s);
        if (B <= 4) return launch_gemv_batch<4>(qs, sc, X, Y, M, K, B, s);
        if (B <= 8) return launch_gemv_batch<8>(qs, sc, X, Y, M, K, B, s);
        return launch_gemv_batch<16>(qs, sc, X, Y, M, K, B, s);
    };
    cudaError_t ce = cudaSuccess;
    for (uint32_t i = 0; i < 3 && ce == cudaSuccess; ++i) ce = one(i);  // warm-up
    if (ce == cudaSuccess) ce = cudaEventRecord(e0, s);
    for (uint32_t i = 0; i < iters && ce == cudaSuccess; ++i) ce = one(i);
    if (ce == cudaSuccess) ce = cudaEventRecord(e1, s);
    if (ce == cudaSuccess) ce = cudaEventSynchronize(e1);
    float ms = 0.0f;
    if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, e0, e1);
    if (img) cudaFreeAsync(img, s);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (ce != cudaSuccess) return fail(BT_ERR_CUDA, std::string("gemv_bench: ") + cudaGetErrorString(ce));
    *us_per_call = ms * 1000.0f / (float)iters;
    return gemv_check_timeout(ws->ticket + kWsTickets, ws->ticket, sizeof(uint32_t) * kWsTickets, s);
}

int bt_cuda_gemv_inject_timeout(int device, int noalloc) {
    int prev = 0;
    BT_CUDA_CHECK(cudaGetDevice(&prev));
    BT_CUDA_CHECK(cudaSetDevice(device));
    int rc = BT_OK;
    if (noalloc) {
        rc = noalloc_inject_timeout(device);
    } else {
        GemvWorkspace* ws = nullptr;
        rc = gemv_workspace(device, &ws);
        const uint32_t one = 1;
        if (rc == BT_OK) {
            const cudaError_t ce = cudaMemcpy(ws->ticket + kWsTickets, &one, sizeof(one), cudaMemcpyHostToDevice);
            if (ce != cudaSuccess) rc = fail(BT_ERR_CUDA, std::string("gemv_inject_timeout: ") + cudaGetErrorString(ce));
        }
    }
    cudaSetDevice(prev);
    return rc;
}

int bt_cuda_gemv_q8(const int8_t* qs, const float* scales, const float* X, float* Y, uint32_t M, uint32_t K,
                    uint32_t B, void* stream) {
    BT_CHECK_ARG(K % 32 == 0, "gemv_q8: K must be a multiple of 32");
    BT_CHECK_ARG(qs && scales && X && Y, "gemv_q8: null buffer");
    BT_CHECK_ARG(((uintptr_t)qs & 15) == 0 && ((uintptr_t)X & 15) == 0 && ((uintptr_t)scales & 3) == 0,
                 "gemv_q8: qs and X must be 16-byte aligned");
    BT_CHECK_ARG(B >= 1 && B <= 16, "gemv_q8: batch must be in [1, 16]");
    BT_CHECK_ARG(K <= 48 * 1024, "gemv_q8: K above 49152 not supported");
    if (M == 0) return BT_OK;
    cudaStream_t s = as_stream(stream);
    cudaError_t e;
    if (B == 1) e = launch_gemv(GemvW{qs, scales, M, K}, ProCopy{X}, EpiStore{Y}, s, false);
    else if (B == 2) e = launch_gemv_batch<2>(qs, scales, X, Y, M, K, B, s);
    else if (B <= 4) e = launch_gemv_batch<4>(qs, scales, X, Y, M, K, B, s);
    else if (B <= 8) e = launch_gemv_batch<8>(qs, scales, X, Y, M, K, B, s);
    else e = launch_gemv_batch<16>(qs, scales, X, Y, M, K, B, s);
    BT_CUDA_CHECK(e);
    return BT_OK;
}

}  // extern "C"
