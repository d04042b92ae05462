// bt_gemv_stream.cuh -- persistent, bulk-copy-fed int8 GEMV for batch-1 decode.
//
// Same arithmetic contract as bt_gemv.cuh (exact int8 x fp32 products, fp32
// accumulation, fp32 per-32 scales; quant_types.cpp:101-121), different
// machine mapping, built for HBM streaming on B200:
//
//   * one CTA per SM (grid = #SMs), 9 warps: warp 8 is the producer, warps 0-7
//     consume.  A CTA owns a contiguous range of row tiles; a tile is T rows,
//     whose int8 rows and fp32 scales are two contiguous HBM ranges.
//   * the producer streams tiles into an NS-stage shared-memory ring with
//     cp.async.bulk (TMA engine, no multicast) completing on mbarriers.  It
//     never waits on the previous kernel, so under programmatic dependent
//     launch the ring of kernel N+1 fills while kernel N drains (<= ~110 KB of
//     shared memory and <= 113 registers keep two CTAs co-resident per SM).
//   * consumers wait for the previous kernel (griddepcontrol.wait), stage the
//     input vector once per CTA (plain or RMSNorm-fused), keep their slice of
//     x in registers, and split each row's K range over WK warps; WG = 8/WK
//     warp groups split the rows of a tile.  int8 -> fp32 is exact (byte
//     permute into 2^23+u, subtract) and the products accumulate with packed
//     fp32x2 FMAs.  Per tile: warp transpose-reduce, cross-warp reduce in
//     shared memory, then the epilogue of the tile's rows.
//   * every mbarrier wait is bounded (2 s of %globaltimer); on expiry the
//     kernel sets *err and leaves, after the producer has waited (bounded) for
//     its copies in flight.
#pragma once

#include "bt_common.cuh"
#include "bt_gemv.cuh"

namespace bt {

constexpr int kStreamConsumers = 8;                       // consumer warps
constexpr int kStreamThreads = (kStreamConsumers + 1) * 32;  // + producer warp
constexpr uint32_t kWaitNs = 2000000000u;                 // bounded waits: 2 s

// ---------------------------------------------------------------- PTX helpers

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

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ float consumer_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    consumer_sync();
    if (lane == 0) red[warp] = v;
    consumer_sync();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kStreamConsumers; ++w) t += red[w];
    return t;
}

// ---------------------------------------------------------------- packed fp32x2

__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// 2^23 + 128 + b for byte k of a two's-complement word (exact), as raw float bits
__device__ __forceinline__ float i8_raw(uint32_t w_xor80, int k) {
    return __uint_as_float(__byte_perm(w_xor80, 0x4B000000u, 0x7540u + (uint32_t)k));
}

// sum_{j<16} q_j * x_j for one 16-byte chunk; x as 8 packed pairs.
__device__ __forceinline__ float dot16_f2(uint4 w, const uint64_t* x2) {
    const uint64_t bias = f2_pack(-8388736.0f, -8388736.0f);
    const uint32_t ww[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
    uint64_t acc = f2_pack(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t word = ww[k >> 1];
        const int b = (k & 1) * 2;
        const uint64_t q = f2_add(f2_pack(i8_raw(word, b), i8_raw(word, b + 1)), bias);
        acc = f2_fma(q, x2[k], acc);
    }
    const float2 r = f2_unpack(acc);
    return r.x + r.y;
}

// ---------------------------------------------------------------- prologues (consumer threads only)

struct SProCopy {
    const float* src;
    __device__ void stage(float* xs, float* red, uint32_t K) const {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* x4 = reinterpret_cast<float4*>(xs);
        for (uint32_t i = threadIdx.x; i < K / 4; i += 256) x4[i] = s4[i];
        consumer_sync();
    }
};

// RMSNorm (kernels/cpu_ref.hpp:11-28) fused: the CTA recomputes sum(x^2).
struct SProNorm {
    const float* src;
    const float* w;
    float eps;
    const float* embed;   // when set: source = embed[st->cur_token], CTA 0 also writes x_out
    const DevState* st;
    float* x_out;
    __device__ void stage(float* xs, float* red, uint32_t K) const {
        const float* s = embed ? embed + (size_t)st->cur_token * K : src;
        const float4* s4 = reinterpret_cast<const float4*>(s);
        float4* x4 = reinterpret_cast<float4*>(xs);
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < K / 4; i += 256) {
            const float4 v = s4[i];
            x4[i] = v;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
            if (embed && blockIdx.x == 0) reinterpret_cast<float4*>(x_out)[i] = v;
        }
        ss = consumer_sum(ss, red);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
        const float4* w4 = reinterpret_cast<const float4*>(w);
        for (uint32_t i = threadIdx.x; i < K / 4; i += 256) {
            float4 v = x4[i];
            const float4 g = w4[i];
            v.x = __fmul_rn(__fmul_rn(v.x, inv), g.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), g.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), g.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), g.w);
            x4[i] = v;
        }
        consumer_sync();
    }
};

// ---------------------------------------------------------------- epilogues
// tile(): consumer threads after the tile's row sums are reducible through rs(r).
// end():  consumer threads after the last tile of the CTA.

struct StreamState {
    float bv;     // running argmax value (logits epilogue)
    uint32_t bi;  // running argmax index, 0xFFFFFFFF = none
};

struct SEpiStore {
    float* y;
    using State = StreamState;
    template <class F>
    __device__ void tile(State&, uint32_t row0, uint32_t T, uint32_t M, F rs) const {
        if (threadIdx.x < T && row0 + threadIdx.x < M) y[row0 + threadIdx.x] = rs(threadIdx.x);
    }
    __device__ void end(State&) const {}
};

struct SEpiResidual {
    float* x;
    float* tap;
    using State = StreamState;
    template <class F>
    __device__ void tile(State&, uint32_t row0, uint32_t T, uint32_t M, F rs) const {
        if (threadIdx.x < T && row0 + threadIdx.x < M) {
            const uint32_t r = row0 + threadIdx.x;
            const float v = __fadd_rn(x[r], rs(threadIdx.x));
            x[r] = v;
            if (tap) tap[r] = v;
        }
    }
    __device__ void end(State&) const {}
};

struct SEpiSwiGLU {
    float* act;
    using State = StreamState;
    template <class F>
    __device__ void tile(State&, uint32_t row0, uint32_t T, uint32_t M, F rs) const {
        const uint32_t p = threadIdx.x;
        if (p < T / 2 && row0 + 2 * p + 1 < M) {
            const float g = rs(2 * p), u = rs(2 * p + 1);
            const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            act[(row0 >> 1) + p] = __fmul_rn(s, u);
        }
    }
    __device__ void end(State&) const {}
};

template <typename KVT>
struct SEpiQKV {
    EpiQKV<KVT> e;
    using State = StreamState;
    template <class F>
    __device__ void tile(State&, uint32_t row0, uint32_t T, uint32_t M, F rs) const {
        const uint32_t p = threadIdx.x;
        if (p >= T / 2) return;
        const uint32_t r = row0 + 2 * p;
        if (r >= M) return;
        const float a = rs(2 * p), b = rs(2 * p + 1);
        const uint32_t pos = e.st->pos;
        if (pos >= e.max_seq) return;
        if (r < e.D + e.KVD) {
            const bool isq = r < e.D;
            const uint32_t local = isq ? r : r - e.D;
            const uint32_t h = local / e.hd, j = (local % e.hd) >> 1, half = e.hd >> 1;
            const float2 cs = e.rope[(size_t)pos * half + j];
            const float o1 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
            const float o2 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
            if (isq) {
                e.q[h * e.hd + j] = o1;
                e.q[h * e.hd + j + half] = o2;
            } else {
                KVT* dst = e.kc + ((size_t)h * e.max_seq + pos) * e.hd;
                dst[j] = KVConv<KVT>::from_f(o1);
                dst[j + half] = KVConv<KVT>::from_f(o2);
            }
        } else {
            const uint32_t local = r - e.D - e.KVD;
            const uint32_t h = local / e.hd, d = local % e.hd;
            KVT* dst = e.vc + ((size_t)h * e.max_seq + pos) * e.hd;
            dst[d] = KVConv<KVT>::from_f(a);
            dst[d + 1] = KVConv<KVT>::from_f(b);
        }
    }
    __device__ void end(State&) const {}
};

// Logits + greedy argmax with the last-CTA reduction of EpiLogits.
struct SEpiLogits {
    EpiLogits e;
    using State = StreamState;
    template <class F>
    __device__ void tile(State& s, uint32_t row0, uint32_t T, uint32_t M, F rs) const {
        if (threadIdx.x < T && row0 + threadIdx.x < M) e.logits[row0 + threadIdx.x] = rs(threadIdx.x);
        if (threadIdx.x == 0) {
            for (uint32_t t = 0; t < T && row0 + t < M; ++t) {
                const float v = rs(t);
                if (s.bi == 0xFFFFFFFFu || better(v, row0 + t, s.bv, s.bi)) { s.bv = v; s.bi = row0 + t; }
            }
        }
    }
    __device__ void end(State& s) const {
        __shared__ bool s_last;
        __shared__ float s_v[kStreamConsumers];
        __shared__ uint32_t s_i[kStreamConsumers];
        if (threadIdx.x == 0) {
            e.part_val[blockIdx.x] = s.bv;
            e.part_idx[blockIdx.x] = s.bi;
            __threadfence();
            s_last = (atomicAdd(e.ticket, 1u) == gridDim.x - 1);
        }
        consumer_sync();
        if (!s_last) return;
        __threadfence();
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t i = threadIdx.x; i < gridDim.x; i += 256) {
            const float v = __ldcg(e.part_val + i);
            const uint32_t ix = __ldcg(e.part_idx + i);
            if (ix != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || better(v, ix, bv, bi))) { bv = v; bi = ix; }
        }
        warp_argmax(bv, bi);
        if ((threadIdx.x & 31) == 0) { s_v[threadIdx.x >> 5] = bv; s_i[threadIdx.x >> 5] = bi; }
        consumer_sync();
        if (threadIdx.x == 0) {
            float v = s_v[0];
            uint32_t ix = s_i[0];
            for (int w = 1; w < kStreamConsumers; ++w)
                if (s_i[w] != 0xFFFFFFFFu && (ix == 0xFFFFFFFFu || better(s_v[w], s_i[w], v, ix))) {
                    v = s_v[w];
                    ix = s_i[w];
                }
            if (ix == 0xFFFFFFFFu) ix = 0;
            DevState* st = e.st;
            const uint32_t pos = st->pos;
            const uint32_t next = (pos + 1 < st->n_fixed) ? e.tok_hist[pos + 1] : ix;
            if (pos < e.max_seq) e.tok_hist[pos + 1] = next;
            st->last_argmax = ix;
            st->cur_token = next;
            st->pos = pos + 1;
            *e.ticket = 0;
        }
    }
};

// ---------------------------------------------------------------- kernel

struct StreamShape {
    uint32_t T;            // rows per tile (= RPW * WG)
    uint32_t WK;           // warps splitting K (1, 2, 4, 8)
    uint32_t NS;           // ring stages
    uint32_t stage_bytes;  // bytes per stage slot (multiple of 128)
    uint32_t ntiles;       // tiles in the matrix
};

// CPL: 16-byte chunks per lane per row; RPW: rows per warp per tile.
template <int CPL, int RPW, class Pro, class Epi>
__global__ void __launch_bounds__(kStreamThreads, 2)
gemv_stream_kernel(GemvW g, StreamShape sh, Pro pro, Epi epi, uint32_t* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[2 * 16];
    __shared__ float red[2][kStreamConsumers][RPW];
    __shared__ float red32[32];

    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t K = g.K, T = sh.T, NS = sh.NS;
    const uint32_t t_begin = (uint32_t)(((uint64_t)sh.ntiles * blockIdx.x) / gridDim.x);
    const uint32_t t_end = (uint32_t)(((uint64_t)sh.ntiles * (blockIdx.x + 1)) / gridDim.x);
    const uint32_t nt = t_end - t_begin;
    uint64_t* full = bars;
    uint64_t* empty = bars + 16;
    uint8_t* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + (size_t)NS * sh.stage_bytes);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStreamConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kStreamConsumers) {
        // ---------------- producer: weights never depend on the previous kernel
        if (lane == 0) {
            const uint32_t wbytes = T * K, sbytes = T * (K / 8);
            uint32_t issued = 0;
            for (uint32_t j = 0; j < nt; ++j) {
                const uint32_t s = j % NS, k = j / NS;
                if (j >= NS && !mbar_wait(&empty[s], (k - 1) & 1, err)) break;
                const size_t row0 = (size_t)(t_begin + j) * T;
                uint8_t* dst = ring + (size_t)s * sh.stage_bytes;
                mbar_expect_tx(&full[s], wbytes + sbytes);
                bulk_g2s(dst, g.qs + row0 * K, wbytes, &full[s]);
                bulk_g2s(dst + wbytes, g.sc + row0 * (K / 32), sbytes, &full[s]);
                issued = j + 1;
            }
            // copies still in flight must land before the CTA may exit
            const uint32_t first = issued > NS ? issued - NS : 0;
            for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, nullptr);
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();
    pro.stage(xs, red32, K);

    const uint32_t WK = sh.WK;
    const uint32_t grp = (uint32_t)warp / WK, kw = (uint32_t)warp % WK;
    const uint32_t NC = K / 16;
    uint64_t xr[CPL][8];
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const uint32_t c = kw * 32 + lane + i * 32 * WK;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float2 v = c < NC ? reinterpret_cast<const float2*>(xs)[c * 8 + k] : make_float2(0.0f, 0.0f);
            xr[i][k] = f2_pack(v.x, v.y);
        }
    }
    StreamState est{-INFINITY, 0xFFFFFFFFu};

    // After a failed (timed-out) wait a consumer stops waiting but keeps every
    // barrier of the loop, so the CTA cannot hang; the error flag is set.
    bool ok = true;
    for (uint32_t j = 0; j < nt; ++j) {
        const uint32_t s = j % NS, k = j / NS;
        if (ok) ok = mbar_wait(&full[s], k & 1, err);
        const uint8_t* stq = ring + (size_t)s * sh.stage_bytes;
        const float* sts = reinterpret_cast<const float*>(stq + (size_t)T * K);
        float acc[RPW];
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            acc[q] = 0.0f;
            const uint32_t r = grp * RPW + q;  // row within the tile
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const uint32_t c = kw * 32 + lane + i * 32 * WK;
                if (c < NC) {
                    const uint4 w = *reinterpret_cast<const uint4*>(stq + (size_t)r * K + c * 16);
                    const float sc = sts[r * (K / 32) + (c >> 1)];
                    acc[q] = fmaf(dot16_f2(w, xr[i]), sc, acc[q]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // warp reduction of the RPW row partials
#pragma unroll
        for (int q = 0; q < RPW; ++q) acc[q] = warp_sum(acc[q]);
        const int buf = j & 1;
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < RPW; ++q) red[buf][warp][q] = acc[q];
        }
        consumer_sync();
        const uint32_t row0 = (t_begin + j) * T;
        auto rs = [&](uint32_t t) {
            const uint32_t gg = t / RPW, q = t % RPW;
            float v = 0.0f;
            for (uint32_t w2 = 0; w2 < WK; ++w2) v += red[buf][gg * WK + w2][q];
            return v;
        };
        epi.tile(est, row0, T, g.M, rs);
    }
    epi.end(est);
}

// Shared memory per CTA: ring + staged input vector.
inline size_t stream_smem(const StreamShape& sh, uint32_t K) {
    return (size_t)sh.NS * sh.stage_bytes + (size_t)K * sizeof(float);
}

// Picks the stream shape for an [M x K] matrix, or returns false when the
// matrix does not fit its constraints (the caller falls back to gemv_q8_kernel).
inline bool stream_plan(uint32_t M, uint32_t K, bool pairs, uint32_t nsm, StreamShape& sh, int& cpl, int& rpw) {
    if (K % 32 || M == 0) return false;
    const uint32_t NC = K / 16;
    uint32_t WK = 1;
    while (WK < 8 && NC > 32 * WK) WK *= 2;
    cpl = (int)((NC + 32 * WK - 1) / (32 * WK));
    if (cpl > 4) return false;
    const uint32_t WG = 8 / WK;
    // rows per tile T = rpw * WG: the largest rpw in {8,4,2,1} with about 16 KB of
    // int8 per stage, an even T for pair epilogues, a 16-byte multiple of scale
    // bytes per tile (bulk-copy rule), and M a multiple of T
    rpw = 0;
    for (int r = 8; r >= 1; r /= 2) {
        const uint32_t T = (uint32_t)r * WG;
        if (T * K > 24576 && r > 1) continue;
        if (pairs && (T % 2)) continue;
        if ((T * (K / 8)) % 16) continue;
        if (M % T) continue;
        rpw = r;
        break;
    }
    if (rpw == 0) return false;
    const uint32_t T = (uint32_t)rpw * WG;
    sh.T = T;
    sh.WK = WK;
    sh.ntiles = M / T;
    const uint32_t raw = T * K + T * (K / 8);
    sh.stage_bytes = (raw + 127) / 128 * 128;
    const uint32_t ring = 73728;  // 72 KB ring: with the staged vector <= ~110 KB, two CTAs per SM
    uint32_t ns = ring / sh.stage_bytes;
    if (ns < 2) ns = 2;
    if (ns > 16) ns = 16;
    sh.NS = ns;
    (void)nsm;
    return stream_smem(sh, K) <= 110 * 1024;
}

template <int CPL, int RPW, class Pro, class Epi>
cudaError_t launch_stream_t(const GemvW& g, const StreamShape& sh, const Pro& pro, const Epi& epi, uint32_t* err,
                            uint32_t nsm, cudaStream_t s, bool pdl) {
    auto kern = gemv_stream_kernel<CPL, RPW, Pro, Epi>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const uint32_t grid = sh.ntiles < nsm ? sh.ntiles : nsm;
    return launch_pdl(kern, dim3(grid), dim3(kStreamThreads), stream_smem(sh, g.K), s, pdl, g, sh, pro, epi, err);
}

template <int CPL, class Pro, class Epi>
cudaError_t launch_stream_c(const GemvW& g, const StreamShape& sh, int rpw, const Pro& pro, const Epi& epi,
                            uint32_t* err, uint32_t nsm, cudaStream_t s, bool pdl) {
    switch (rpw) {
        case 1: return launch_stream_t<CPL, 1>(g, sh, pro, epi, err, nsm, s, pdl);
        case 2: return launch_stream_t<CPL, 2>(g, sh, pro, epi, err, nsm, s, pdl);
        case 4: return launch_stream_t<CPL, 4>(g, sh, pro, epi, err, nsm, s, pdl);
        default: return launch_stream_t<CPL, 8>(g, sh, pro, epi, err, nsm, s, pdl);
    }
}

// Streams when the shape allows, otherwise runs the register-prefetch kernel.
template <class SPro, class SEpi, class Pro, class Epi>
cudaError_t launch_gemv_best(const GemvW& g, const SPro& spro, const SEpi& sepi, const Pro& pro, const Epi& epi,
                             bool pairs, uint32_t* err, uint32_t nsm, cudaStream_t s, bool pdl, bool allow_stream) {
    StreamShape sh;
    int cpl = 0, rpw = 0;
    if (allow_stream && stream_plan(g.M, g.K, pairs, nsm, sh, cpl, rpw)) {
        switch (cpl) {
            case 1: return launch_stream_c<1>(g, sh, rpw, spro, sepi, err, nsm, s, pdl);
            case 2: return launch_stream_c<2>(g, sh, rpw, spro, sepi, err, nsm, s, pdl);
            case 3: return launch_stream_c<3>(g, sh, rpw, spro, sepi, err, nsm, s, pdl);
            default: return launch_stream_c<4>(g, sh, rpw, spro, sepi, err, nsm, s, pdl);
        }
    }
    return launch_gemv(g, pro, epi, s, pdl, pairs ? 4 : 8);
}

}  // namespace bt
