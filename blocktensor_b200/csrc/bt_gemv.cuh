// bt_gemv.cuh -- the int8-weight GEMV at the core of every decode projection.
//
// y[m] = sum_k W[m][k] * x[k], W as qs[M][K] int8 + scales[M][K/32] fp32
// (the reference's Q8_0 blocks, quantization/quant_types.hpp:12-15, repacked).
// Arithmetic per row follows quantization/quant_types.cpp:101-121: products of
// the exact int8 value and fp32 x accumulated in fp32, scaled per block.
// The summation order differs (16-element partial sums scaled per half block,
// then a warp tree), which is the documented fp32 tolerance.
//
// Kernel shape (B = 1 decode):
//   * 256 threads = 8 warps, ROWS rows per CTA, WPR warps per row (K split
//     across the warps of a row), 16-byte chunks strided so that each warp
//     instruction reads 512 contiguous bytes of one row.
//   * Before griddepcontrol.wait the CTA already issues the loads of its first
//     CH chunks per lane (weights never depend on the previous kernel), so with
//     programmatic dependent launch the weight stream of kernel N+1 overlaps the
//     tail of kernel N.
//   * A prologue functor stages the input vector in shared memory (plain copy,
//     or RMSNorm fused: the CTA recomputes sum(x^2) of the whole vector).
//   * An epilogue functor consumes the ROWS results (store, residual add,
//     RoPE + KV append, SwiGLU, logits + argmax).
#pragma once

#include "bt_common.cuh"

namespace bt {

constexpr int kGemvThreads = 256;
constexpr int kGemvCH = 8;  // 16-byte chunks per lane per round

struct GemvW {
    const int8_t* qs;
    const float* sc;
    uint32_t M, K;
};

// Device-resident decode state of one sequence.
struct DevState {
    uint32_t pos;          // position of the token processed by the current step
    uint32_t cur_token;    // token consumed by the current step
    uint32_t n_fixed;      // tok_hist[0..n_fixed) are given (prompt); later entries are argmax
    uint32_t last_argmax;  // greedy token of the last finished step
    uint32_t error;
    uint32_t pad[3];
};

// ---------------------------------------------------------------- prologues

// xs[k] = src[k]
struct ProCopy {
    const float* src;
    __device__ void stage(float* xs, float* red, uint32_t K) const {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* x4 = reinterpret_cast<float4*>(xs);
        for (uint32_t i = threadIdx.x; i < K / 4; i += blockDim.x) x4[i] = s4[i];
        __syncthreads();
    }
};

// xs = rmsnorm(src) * w  (kernels/cpu_ref.hpp:11-28).  When `embed` is set the
// source row is embed[state->cur_token] (transformer_engine.cpp:233-238) and
// CTA 0 also writes it to x_out (the residual stream).
struct ProNorm {
    const float* src;
    const float* w;
    float eps;
    const float* embed;
    const DevState* st;
    float* x_out;
    __device__ void stage(float* xs, float* red, uint32_t K) const {
        const float* s = src;
        if (embed) s = embed + (size_t)st->cur_token * K;
        const float4* s4 = reinterpret_cast<const float4*>(s);
        float4* x4 = reinterpret_cast<float4*>(xs);
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < K / 4; i += blockDim.x) {
            const float4 v = s4[i];
            x4[i] = v;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
            if (embed && blockIdx.x == 0) reinterpret_cast<float4*>(x_out)[i] = v;
        }
        ss = block_sum(ss, red);
        const float mean = __fdiv_rn(ss, (float)K);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        const float4* w4 = reinterpret_cast<const float4*>(w);
        for (uint32_t i = threadIdx.x; i < K / 4; i += blockDim.x) {
            float4 v = x4[i];
            const float4 g = w4[i];
            v.x = __fmul_rn(__fmul_rn(v.x, inv), g.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), g.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), g.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), g.w);
            x4[i] = v;
        }
        __syncthreads();
    }
};

// ---------------------------------------------------------------- epilogues
// finish() runs on every thread after the ROWS results are in y[0..ROWS).

struct EpiStore {
    static constexpr bool kPairs = false;
    float* y;
    template <int ROWS>
    __device__ void finish(const float* yr, uint32_t row0, uint32_t M) const {
        if (threadIdx.x < ROWS && row0 + threadIdx.x < M) y[row0 + threadIdx.x] = yr[threadIdx.x];
    }
};

// x[m] += y[m] (transformer_engine.cpp:191-195, 222-225); optional per-layer tap.
struct EpiResidual {
    static constexpr bool kPairs = false;
    float* x;
    float* tap;
    template <int ROWS>
    __device__ void finish(const float* yr, uint32_t row0, uint32_t M) const {
        if (threadIdx.x < ROWS && row0 + threadIdx.x < M) {
            const uint32_t r = row0 + threadIdx.x;
            const float v = __fadd_rn(x[r], yr[threadIdx.x]);
            x[r] = v;
            if (tap) tap[r] = v;
        }
    }
};

// Rows come in (gate, up) pairs: act[j] = silu(gate) * up
// (cpu_ref.hpp:74-79 and transformer_engine.cpp:212-215).
struct EpiSwiGLU {
    static constexpr bool kPairs = true;  // needs ROWS >= 2
    float* act;
    template <int ROWS>
    __device__ void finish(const float* yr, uint32_t row0, uint32_t M) const {
        if (threadIdx.x < ROWS / 2 && row0 + 2 * threadIdx.x + 1 < M) {
            const float g = yr[2 * threadIdx.x], u = yr[2 * threadIdx.x + 1];
            const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            act[(row0 >> 1) + threadIdx.x] = __fmul_rn(s, u);
        }
    }
};

// Fused q/k/v: rows [0,D) are q, [D,D+KVD) k, [D+KVD, D+2KVD) v.  q and k rows
// are stored as RoPE pairs (i, i+hd/2) of one head next to each other, so each
// pair is rotated here (cpu_ref.hpp:30-53 with the host-computed cos/sin of
// the reference formula) and k, v are appended to the cache at `pos`
// (runtime/src/kv_cache.cpp:17-27).  Cache layout: [kv_head][max_seq][hd].
template <typename KVT>
struct EpiQKV {
    static constexpr bool kPairs = true;  // needs ROWS >= 2
    float* q;
    KVT* kc;
    KVT* vc;
    const float2* rope;  // [max_seq][hd/2] (cos, sin)
    const DevState* st;
    uint32_t D, KVD, hd, max_seq;
    template <int ROWS>
    __device__ void finish(const float* yr, uint32_t row0, uint32_t M) const {
        if (threadIdx.x >= ROWS / 2) return;
        const uint32_t r = row0 + 2 * threadIdx.x;
        if (r >= M) return;
        const float a = yr[2 * threadIdx.x], b = yr[2 * threadIdx.x + 1];
        const uint32_t pos = st->pos;
        if (pos >= max_seq) return;
        if (r < D + KVD) {
            const bool isq = r < D;
            const uint32_t local = isq ? r : r - D;
            const uint32_t h = local / hd, j = (local % hd) >> 1, half = hd >> 1;
            const float2 cs = rope[(size_t)pos * half + j];
            const float o1 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
            const float o2 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
            if (isq) {
                q[h * hd + j] = o1;
                q[h * hd + j + half] = o2;
            } else {
                KVT* dst = kc + ((size_t)h * max_seq + pos) * hd;
                dst[j] = KVConv<KVT>::from_f(o1);
                dst[j + half] = KVConv<KVT>::from_f(o2);
            }
        } else {
            const uint32_t local = r - D - KVD;
            const uint32_t h = local / hd, d = local % hd;
            KVT* dst = vc + ((size_t)h * max_seq + pos) * hd;
            dst[d] = KVConv<KVT>::from_f(a);
            dst[d + 1] = KVConv<KVT>::from_f(b);
        }
    }
};

// Logits + greedy argmax (transformer_engine.cpp:244-250, sampler.hpp:11-13).
// Each CTA writes its logits and its local argmax; the last CTA to finish
// (atomic ticket) reduces the partials, advances the sequence state and
// resets the ticket.
struct EpiLogits {
    static constexpr bool kPairs = false;
    float* logits;
    float* part_val;
    uint32_t* part_idx;
    uint32_t* ticket;
    DevState* st;
    uint32_t* tok_hist;  // [max_seq + 1]
    uint32_t max_seq;
    // persistent step kernel: the last CTA also counts the step in st->pad[0] and
    // the engine's step launches in ticket[1] (the tag of its split partials)
    bool bump_epoch = false;
    // tensor parallelism: this rank's vocab rows start at v0; with tp_world > 1 the last CTA trades
    // its best (value, index) with the other ranks through the argmax slots of their exchange
    // buffers (xch[q] + xch_off: [tp_world][2] tagged words) and every rank takes the same token
    uint32_t v0 = 0, tp_rank = 0, tp_world = 1, tag = 0;
    uint64_t* const* xch = nullptr;
    size_t xch_off = 0;
    template <int ROWS>
    __device__ void finish(const float* yr, uint32_t row0, uint32_t M) const {
        __shared__ bool s_last;
        __shared__ float s_bv[32];
        __shared__ uint32_t s_bi[32];
        if (threadIdx.x < ROWS && row0 + threadIdx.x < M) logits[row0 + threadIdx.x] = yr[threadIdx.x];
        if (threadIdx.x == 0) {
            float bv = yr[0];
            uint32_t bi = row0;
            for (int i = 1; i < ROWS; ++i)
                if (row0 + i < M && better(yr[i], row0 + i, bv, bi)) { bv = yr[i]; bi = row0 + i; }
            part_val[blockIdx.x] = bv;
            part_idx[blockIdx.x] = bi;
            __threadfence();
            const uint32_t prev = atomicAdd(ticket, 1u);
            s_last = (prev == gridDim.x - 1);
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t i = threadIdx.x; i < gridDim.x; i += blockDim.x) {
            const float v = __ldcg(part_val + i);
            const uint32_t ix = __ldcg(part_idx + i);
            if (bi == 0xFFFFFFFFu || better(v, ix, bv, bi)) { bv = v; bi = ix; }
        }
        // lanes that saw nothing carry index 0xFFFFFFFF and -inf: never better than a real entry
        warp_argmax(bv, bi);
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        if (lane == 0) { s_bv[warp] = bv; s_bi[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = s_bv[0];
            uint32_t ix = s_bi[0];
            for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
                if (s_bi[w] != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || better(s_bv[w], s_bi[w], v, ix))) {
                    v = s_bv[w];
                    ix = s_bi[w];
                }
            if (ix == 0xFFFFFFFFu) ix = 0;
            const uint32_t pos = st->pos;
            const uint32_t next = (pos + 1 < st->n_fixed) ? tok_hist[pos + 1] : ix;
            if (pos < max_seq) tok_hist[pos + 1] = next;
            st->last_argmax = ix;
            st->cur_token = next;
            st->pos = pos + 1;
            *ticket = 0;
        }
    }
};

// ---------------------------------------------------------------- kernel

template <int ROWS, int WPR, class Pro, class Epi>
__global__ void __launch_bounds__(kGemvThreads)
gemv_q8_kernel(GemvW g, Pro pro, Epi epi) {
    static_assert(ROWS * WPR == kGemvThreads / 32, "8 warps per CTA");
    extern __shared__ float4 smem_x4[];
    float* xs = reinterpret_cast<float*>(smem_x4);
    __shared__ float red[32];
    __shared__ float part[ROWS][WPR];
    __shared__ float yr[ROWS];

    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rl = warp / WPR, ks = warp % WPR;
    const uint32_t row0 = blockIdx.x * ROWS;
    const uint32_t row = row0 + rl;
    const bool row_ok = row < g.M;
    const uint32_t NC = g.K >> 4;
    constexpr uint32_t stride = 32u * WPR;
    const uint32_t c0 = (uint32_t)ks * 32u + (uint32_t)lane;
    const int8_t* wrow = g.qs + (size_t)(row_ok ? row : 0) * g.K;
    const float* srow = g.sc + (size_t)(row_ok ? row : 0) * (g.K >> 5);

    int4 w[kGemvCH];
    float s[kGemvCH];
#pragma unroll
    for (int i = 0; i < kGemvCH; ++i) {
        const uint32_t c = c0 + (uint32_t)i * stride;
        w[i] = make_int4(0, 0, 0, 0);
        s[i] = 0.0f;
        if (row_ok && c < NC) {
            w[i] = ld_stream_v4(wrow + (size_t)c * 16);
            s[i] = ld_stream_f32(srow + (c >> 1));
        }
    }

    pdl_wait();
    pro.stage(xs, red, g.K);

    float acc = 0.0f;
    uint32_t base = c0;
    while (true) {
#pragma unroll
        for (int i = 0; i < kGemvCH; ++i) {
            const uint32_t c = base + (uint32_t)i * stride;
            if (row_ok && c < NC)
                acc = fmaf(dot16(w[i], reinterpret_cast<const float4*>(xs + (size_t)c * 16)), s[i], acc);
        }
        base += kGemvCH * stride;
        if (base >= NC) break;
#pragma unroll
        for (int i = 0; i < kGemvCH; ++i) {
            const uint32_t c = base + (uint32_t)i * stride;
            if (row_ok && c < NC) {
                w[i] = ld_stream_v4(wrow + (size_t)c * 16);
                s[i] = ld_stream_f32(srow + (c >> 1));
            }
        }
    }
    acc = warp_sum(acc);
    if (WPR == 1) {
        if (lane == 0) yr[rl] = acc;
    } else {
        if (lane == 0) part[rl][ks] = acc;
        __syncthreads();
        if (threadIdx.x < ROWS) {
            float v = 0.0f;
#pragma unroll
            for (int k = 0; k < WPR; ++k) v += part[threadIdx.x][k];
            yr[threadIdx.x] = v;
        }
    }
    __syncthreads();
    epi.template finish<ROWS>(yr, row0, g.M);
}

// WPR for a reduction length K: enough warps per row that one round of
// kGemvCH chunks per lane covers most of the row.
inline int gemv_wpr(uint32_t K, int max_wpr = 8) {
    const uint32_t nc = K / 16;
    int w = 1;
    while (w < max_wpr && nc > (uint32_t)(32 * kGemvCH * w)) w *= 2;
    return w;
}

template <int WPR, class Pro, class Epi>
cudaError_t launch_gemv_wpr(const GemvW& g, const Pro& pro, const Epi& epi, cudaStream_t s, bool pdl) {
    constexpr int ROWS = 8 / WPR;
    auto kern = gemv_q8_kernel<ROWS, WPR, Pro, Epi>;
    const size_t smem = (size_t)g.K * sizeof(float);
    static bool attr_set[64] = {};  // per instantiation and device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const unsigned grid = (g.M + ROWS - 1) / ROWS;
    return launch_pdl(kern, dim3(grid), dim3(kGemvThreads), smem, s, pdl, g, pro, epi);
}

template <class Pro, class Epi>
cudaError_t launch_gemv(const GemvW& g, const Pro& pro, const Epi& epi, cudaStream_t s, bool pdl,
                        int max_wpr = 8) {
    switch (gemv_wpr(g.K, max_wpr)) {
        case 1: return launch_gemv_wpr<1>(g, pro, epi, s, pdl);
        case 2: return launch_gemv_wpr<2>(g, pro, epi, s, pdl);
        case 4: return launch_gemv_wpr<4>(g, pro, epi, s, pdl);
        default:
            if constexpr (Epi::kPairs) return cudaErrorInvalidValue;  // pair epilogues need ROWS >= 2
            else return launch_gemv_wpr<8>(g, pro, epi, s, pdl);
    }
}

}  // namespace bt
