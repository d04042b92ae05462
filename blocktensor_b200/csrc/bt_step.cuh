// bt_step.cuh -- one decode step (TransformerEngine::forward_single_token,
// runtime/src/transformer_engine.cpp:228-251) as one persistent kernel.
//
// One CTA per SM, launched cooperatively so that all CTAs are resident.  The
// step is a sequence of phases: for every layer qkv GEMV, attention, o-proj
// GEMV, gate/up GEMV, down GEMV (execute_layer, :114-226), then the head GEMV
// with the greedy argmax.  Every phase needs the whole output of the one
// before it, so phases are separated by grid-wide counters in device memory:
// a CTA adds 1 to cnt[p] (release, gpu scope) when all of its writes of phase
// p are done, and a CTA starts phase p+1 once cnt[p] reaches G * (epoch + 1)
// (acquire poll, bounded), epoch being the sequence's step count.
//
// The weights never depend on earlier phases, so the producer warp streams the
// CTA's tiles of every GEMV of the step back to back through one shared-memory
// ring, without waiting at phase boundaries: while the consumers wait for a
// phase counter, build the next input's digits or run attention, the ring
// keeps filling.  The GEMV arithmetic, layout, warp roles and stream-K merge
// are those of bt_gemv_mma.cuh; attention runs on the consumer warps between
// the qkv and o-proj GEMVs.
//
// Activations written inside the kernel are read with ld.global.cg (L2), never
// through L1, where another SM's earlier line could be stale.
#pragma once

#include "bt_common.cuh"
#include "bt_gemv.cuh"
#include "bt_gemv_mma.cuh"
#include "bt_ptx.cuh"

namespace bt {

struct StepMat {
    const uint8_t* units;
    uint32_t M, Mp, K;
};

struct StepLayer {
    StepMat qkv, o, gu, d;
    const float* attn_norm;
    const float* ffn_norm;
};

struct StepArgs {
    const StepLayer* layers;  // [L], device memory
    StepMat head;
    const float* embed;
    const float* out_norm;
    float* x;
    float* q;
    float* attn;
    float* act;
    float* logits;
    float* taps;              // [L][D] or null
    void* kc;                 // [L][KVH][max_seq][hd]
    void* vc;
    const float2* rope;       // [max_seq][hd/2]
    DevState* st;
    uint32_t* tok_hist;
    float* split_part;        // [G][2][128]
    uint32_t* split_ticket;   // [row tiles of the tallest matrix]
    float* am_val;            // [G]
    uint32_t* am_idx;
    uint32_t* am_ticket;
    float* att_part;          // [KVH][GQ][S][hd + 2]
    uint32_t* att_ticket;     // [KVH]
    uint32_t* cnt;            // [5 L + 1] phase counters
    uint32_t L, D, KVD, hd, KVH, GQ, max_seq, S_att;
    float eps, scale;
    uint32_t NS, xstride, tmem_cols, scratch_off;
};

enum : uint32_t { kPhQKV = 0, kPhAttn = 1, kPhO = 2, kPhGU = 3, kPhDown = 4, kPhHead = 5 };

__device__ __forceinline__ uint32_t phase_kind(uint32_t p, uint32_t L) { return p == 5 * L ? kPhHead : p % 5; }

__device__ __forceinline__ StepMat phase_mat(const StepArgs& a, uint32_t p) {
    const uint32_t k = phase_kind(p, a.L);
    if (k == kPhHead) return a.head;
    const StepLayer& l = a.layers[p / 5];
    return k == kPhQKV ? l.qkv : k == kPhO ? l.o : k == kPhGU ? l.gu : l.d;
}

// Tile range of CTA c in the stream-K split of matrix m over Gm = min(G, U)
// CTAs (every CTA of the split owns at least one tile; CTAs c >= Gm own none).
struct Geo {
    uint32_t NB, U, Gm, u0, u1, g_first, g_last, nstages;
};

__device__ __forceinline__ Geo phase_geo(const StepMat& m, uint32_t c, uint32_t G) {
    Geo r;
    r.NB = m.K / kTileK;
    r.U = (m.Mp / kTileRows) * r.NB;
    r.Gm = r.U < G ? r.U : G;
    if (c >= r.Gm) {
        r.u0 = r.u1 = 0;
        r.g_first = 1;
        r.g_last = 0;
        r.nstages = 0;
        return r;
    }
    r.u0 = (uint32_t)(((uint64_t)r.U * c) / r.Gm);
    r.u1 = (uint32_t)(((uint64_t)r.U * (c + 1)) / r.Gm);
    r.g_first = r.u0 / r.NB;
    r.g_last = (r.u1 - 1) / r.NB;
    r.nstages = (r.u1 - r.u0 + kStageTiles - 1) / kStageTiles;
    return r;
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Atomic add with acquire and release semantics at gpu scope; returns the old value.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Add with release semantics at gpu scope (no result).
__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Prologue of any GEMV of the step: RMSNorm with weight w (kernels/cpu_ref.hpp:11-28)
// or, when w is null, a plain copy; the element loads are step_x / step_p below.
// With `embed` the source is the embedding row of the current token and CTA 0
// also writes it to x_out.  Activations are read through L2.
struct MProStep {
    const float* src;
    const float* w;
    float eps;
    const float* embed;
    const DevState* st;
    float* x_out;
    __device__ const float* base(uint32_t K) const { return embed ? embed + (size_t)st->cur_token * K : src; }
    __device__ float factor(float ss, uint32_t K) const {
        return w ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps))) : 1.0f;
    }
};

// Digits of the input of a GEMV phase (build_digits of bt_gemv_mma.cuh).  The
// norm weights do not depend on earlier phases: step_prefetch_w pulls them
// into L2 before the phase barrier, so after it the weight and activation
// loads of step_build_digits share one round trip to L2.
constexpr int kStepR = 6;  // items (8 elements) per digit thread held in registers: K <= 13824

__device__ __forceinline__ void step_prefetch_w(const float* w, uint32_t K, uint32_t tid) {
    if (!w) return;
    for (uint32_t off = tid * 32; off < K; off += kDigitThreads * 32)  // one 128-byte line per thread
        asm volatile("prefetch.global.L2 [%0];" ::"l"(w + off));
}

__device__ __forceinline__ float4 step_x(const MProStep& pro, const float* s, uint32_t k) {
    return pro.embed ? *reinterpret_cast<const float4*>(s + k) : ldcg4(s + k);
}

__device__ __forceinline__ float4 step_p(const MProStep& pro, const float4& v, const float4& g, uint32_t k, float& ss,
                                         float& mx) {
    if (!pro.w) {
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        return v;
    }
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
    if (pro.embed && blockIdx.x == 0) *reinterpret_cast<float4*>(pro.x_out + k) = v;
    const float4 p = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(p.x), fabsf(p.y)), fmaxf(fabsf(p.z), fabsf(p.w))));
    return p;
}

__device__ int step_build_digits(const MProStep& pro, uint32_t K, uint8_t* xb, uint32_t xstride, float* red,
                                 uint32_t tid, bool& bad) {
    const float* s = pro.base(K);
    const uint32_t items = K >> 3;
    float ss = 0.0f, mx = 0.0f;
    float4 pa[kStepR], pb[kStepR];
    const float4 one = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
#pragma unroll
    for (int i = 0; i < kStepR; ++i) {
        const uint32_t idx = tid + kDigitThreads * i;
        if (idx < items) {
            const uint32_t k = (idx >> 2) * 32 + (idx & 3) * 4;
            const float4 xa = step_x(pro, s, k), xc = step_x(pro, s, k + 16);
            const float4 ga = pro.w ? *reinterpret_cast<const float4*>(pro.w + k) : one;
            const float4 gb = pro.w ? *reinterpret_cast<const float4*>(pro.w + k + 16) : one;
            pa[i] = step_p(pro, xa, ga, k, ss, mx);
            pb[i] = step_p(pro, xc, gb, k + 16, ss, mx);
        }
    }
    for (uint32_t idx = tid + kDigitThreads * kStepR; idx < items; idx += kDigitThreads) {
        const uint32_t k = (idx >> 2) * 32 + (idx & 3) * 4;
        const float4 ga = pro.w ? *reinterpret_cast<const float4*>(pro.w + k) : one;
        const float4 gb = pro.w ? *reinterpret_cast<const float4*>(pro.w + k + 16) : one;
        step_p(pro, step_x(pro, s, k), ga, k, ss, mx);
        step_p(pro, step_x(pro, s, k + 16), gb, k + 16, ss, mx);
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    const uint32_t lane = tid & 31, w = tid >> 5;
    if (lane == 0) { red[w] = ss; red[kDigitWarps + w] = mx; }
    digit_sync();
    float tss = 0.0f, tmx = 0.0f;
#pragma unroll
    for (int i = 0; i < kDigitWarps; ++i) { tss += red[i]; tmx = fmaxf(tmx, red[kDigitWarps + i]); }
    const float f = pro.factor(tss, K);
    const float m = tmx * f;
    int e = 0;
    bad = !isfinite(m);
    if (m > 0.0f && !bad) {
        int ex;
        frexpf(m, &ex);
        e = 21 - ex;
    }
    const float c1 = ldexpf(1.0f, e / 2), c2 = ldexpf(f, e - e / 2);
#pragma unroll
    for (int i = 0; i < kStepR; ++i) {
        const uint32_t idx = tid + kDigitThreads * i;
        if (idx < items) pack_item(xb, xstride, idx, pa[i], pb[i], c1, c2);
    }
    for (uint32_t idx = tid + kDigitThreads * kStepR; idx < items; idx += kDigitThreads) {
        const uint32_t k = (idx >> 2) * 32 + (idx & 3) * 4;
        float d0 = 0.0f, d1 = 0.0f;
        const float4 ga = pro.w ? *reinterpret_cast<const float4*>(pro.w + k) : one;
        const float4 gb = pro.w ? *reinterpret_cast<const float4*>(pro.w + k + 16) : one;
        const float4 pa2 = step_p(pro, step_x(pro, s, k), ga, k, d0, d1);
        const float4 pb2 = step_p(pro, step_x(pro, s, k + 16), gb, k + 16, d0, d1);
        pack_item(xb, xstride, idx, pa2, pb2, c1, c2);
    }
    fence_proxy_async();
    digit_sync();
    return e;
}

// Waits (one thread) until cnt reaches target; bounded, and no wait at all
// once an earlier wait of the step has timed out (*err set).
__device__ __forceinline__ void wait_count(const uint32_t* cnt, uint32_t target, uint32_t* err) {
    if ((int32_t)(ld_acquire_gpu(cnt) - target) >= 0) return;
    const uint64_t t0 = global_ns();
    while ((int32_t)(ld_acquire_gpu(cnt) - target) < 0) {
        if (*reinterpret_cast<volatile uint32_t*>(err)) return;
        if (global_ns() - t0 > kWaitNs) {
            atomicExch(err, 1u);
            return;
        }
    }
}

// ---------------------------------------------------------------- attention phase
// Items (kv head, split) are dealt to the CTAs round robin; the 9 consumer
// warps of a CTA take the item's keys round robin in batches (2 to 8 keys,
// up to 64 bytes of K and V per lane, all loads of a batch in flight at once), with an online softmax per query head (lane i
// holds head dims NV*i .. NV*i+NV-1), merge in shared memory, write the CTA's
// partial (max m, sum l, o = sum e^(s-m) v), and the last CTA of a KV head
// (ticket) merges the splits into attn (:148-184).

// One lane's NV consecutive cache elements as 32-bit words, loaded through L2.
template <int NV, typename KVT>
struct RowWords {
    static constexpr int W = (int)(NV * sizeof(KVT) / 4);
    uint32_t w[W];
    __device__ __forceinline__ void load(const KVT* p) {
        if constexpr (W == 1) {
            w[0] = __ldcg(reinterpret_cast<const unsigned int*>(p));
        } else if constexpr (W == 2) {
            const uint2 v = __ldcg(reinterpret_cast<const uint2*>(p));
            w[0] = v.x; w[1] = v.y;
        } else {
#pragma unroll
            for (int h = 0; h < W / 4; ++h) {
                const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p) + h);
                w[4 * h] = v.x; w[4 * h + 1] = v.y; w[4 * h + 2] = v.z; w[4 * h + 3] = v.w;
            }
        }
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < W; ++i) w[i] = 0u;
    }
    __device__ __forceinline__ float at(int i) const {
        if constexpr (sizeof(KVT) == 2) {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[i >> 1]);
            return (i & 1) ? __high2float(h) : __low2float(h);
        } else {
            return __uint_as_float(w[i]);
        }
    }
};

template <int NV, int GQM, typename KVT>
__device__ void attn_phase(const StepArgs& a, uint32_t l, uint8_t* scratch, uint32_t tid) {
    // GQM: query heads per KV head held in registers; B: keys per batch and warp
    constexpr int BW = 16 / RowWords<NV, KVT>::W;
    constexpr int B = BW > 8 ? 8 : (BW < 2 ? 2 : BW);
    const uint32_t lane = tid & 31, w = tid >> 5, G = gridDim.x;
    const uint32_t HD = a.hd, GQ = a.GQ, S = a.S_att;
    const uint32_t pos = a.st->pos;
    const uint32_t c = min(pos + 1, a.max_seq);
    const size_t layer_off = (size_t)l * a.KVH * a.max_seq * HD;
    const KVT* kl = reinterpret_cast<const KVT*>(a.kc) + layer_off;
    const KVT* vl = reinterpret_cast<const KVT*>(a.vc) + layer_off;
    float* wm = reinterpret_cast<float*>(scratch);  // [9][GQ][HD + 2]
    __shared__ uint32_t s_last;
    const uint32_t pstride = HD + 2;
    const uint32_t d0 = lane * NV;
    const bool active = d0 < HD;
    for (uint32_t it = blockIdx.x; it < a.KVH * S; it += G) {
        const uint32_t kvh = it / S, sidx = it % S;
        const uint32_t Lk = (c + S - 1) / S;
        const uint32_t t0 = sidx * Lk, t1 = min(c, t0 + Lk);
        float qv[GQM][NV], o[GQM][NV], m[GQM], ls[GQM];
#pragma unroll
        for (int g = 0; g < GQM; ++g) {
            m[g] = -INFINITY;
            ls[g] = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                o[g][i] = 0.0f;
                qv[g][i] = ((uint32_t)g < GQ && active) ? __ldcg(a.q + (size_t)(kvh * GQ + g) * HD + d0 + i) : 0.0f;
            }
        }
        const KVT* kb = kl + (size_t)kvh * a.max_seq * HD + d0;
        const KVT* vb = vl + (size_t)kvh * a.max_seq * HD + d0;
        for (uint32_t base = t0 + w; base < t1; base += B * kDigitWarps) {
            RowWords<NV, KVT> kr[B], vr[B];
#pragma unroll
            for (int j = 0; j < B; ++j) {
                const uint32_t t = base + j * kDigitWarps;
                if (t < t1 && active) {
                    kr[j].load(kb + (size_t)t * HD);
                    vr[j].load(vb + (size_t)t * HD);
                } else {
                    kr[j].zero();
                    vr[j].zero();
                }
            }
#pragma unroll
            for (int g = 0; g < GQM; ++g) {
                if ((uint32_t)g >= GQ) break;
                float sc[B];
                float mb = -INFINITY;
#pragma unroll
                for (int j = 0; j < B; ++j) {
                    float p = 0.0f;
#pragma unroll
                    for (int i = 0; i < NV; ++i) p = fmaf(qv[g][i], kr[j].at(i), p);
                    p = warp_sum(p);
                    sc[j] = base + j * kDigitWarps < t1 ? __fmul_rn(p, a.scale) : -INFINITY;
                    mb = fmaxf(mb, sc[j]);
                }
                const float mn = fmaxf(m[g], mb);
                const float alpha = expf(m[g] - mn);
                float lsum = ls[g] * alpha;
                float acc[NV];
#pragma unroll
                for (int i = 0; i < NV; ++i) acc[i] = o[g][i] * alpha;
#pragma unroll
                for (int j = 0; j < B; ++j) {
                    const float e = expf(sc[j] - mn);  // 0 for keys past t1
                    lsum += e;
#pragma unroll
                    for (int i = 0; i < NV; ++i) acc[i] = fmaf(e, vr[j].at(i), acc[i]);
                }
                ls[g] = lsum;
                m[g] = mn;
#pragma unroll
                for (int i = 0; i < NV; ++i) o[g][i] = acc[i];
            }
        }
        // warp partials -> shared memory
        for (uint32_t g = 0; g < GQ && g < (uint32_t)GQM; ++g) {
            float* p = wm + ((size_t)w * GQ + g) * pstride;
            if (lane == 0) { p[0] = m[g]; p[1] = ls[g]; }
#pragma unroll
            for (int i = 0; i < NV; ++i)
                if (active) p[2 + d0 + i] = o[g][i];
        }
        digit_sync();
        // CTA partial of this split
        float* pg = a.att_part + (size_t)kvh * GQ * S * pstride;
        for (uint32_t e = tid; e < GQ * HD; e += kDigitThreads) {
            const uint32_t g = e / HD, d = e % HD;
            float M = -INFINITY;
            for (uint32_t ww = 0; ww < kDigitWarps; ++ww) {
                const float* p = wm + ((size_t)ww * GQ + g) * pstride;
                if (p[1] > 0.0f) M = fmaxf(M, p[0]);
            }
            float lsum = 0.0f, acc = 0.0f;
            for (uint32_t ww = 0; ww < kDigitWarps; ++ww) {
                const float* p = wm + ((size_t)ww * GQ + g) * pstride;
                if (p[1] > 0.0f) {
                    const float f = expf(p[0] - M);
                    lsum = fmaf(p[1], f, lsum);
                    acc = fmaf(p[2 + d], f, acc);
                }
            }
            float* dst = pg + ((size_t)g * S + sidx) * pstride;
            dst[2 + d] = acc;
            if (d == 0) { dst[0] = M; dst[1] = lsum; }
        }
        __threadfence();
        digit_sync();
        if (tid == 0) s_last = atomicAdd(a.att_ticket + kvh, 1u) == S - 1 ? 1u : 0u;
        digit_sync();
        if (s_last) {
            __threadfence();
            for (uint32_t e = tid; e < GQ * HD; e += kDigitThreads) {
                const uint32_t g = e / HD, d = e % HD;
                const float* pb = pg + (size_t)g * S * pstride;
                float M = -INFINITY;
                for (uint32_t s = 0; s < S; ++s)
                    if (__ldcg(pb + s * pstride + 1) > 0.0f) M = fmaxf(M, __ldcg(pb + s * pstride));
                float lsum = 0.0f, acc = 0.0f;
                for (uint32_t s = 0; s < S; ++s) {
                    const float ll = __ldcg(pb + s * pstride + 1);
                    if (ll > 0.0f) {
                        const float f = expf(__ldcg(pb + s * pstride) - M);
                        lsum = fmaf(ll, f, lsum);
                        acc = fmaf(__ldcg(pb + s * pstride + 2 + d), f, acc);
                    }
                }
                a.attn[(size_t)(kvh * GQ + g) * HD + d] = __fdiv_rn(acc, lsum);
            }
            if (tid == 0) a.att_ticket[kvh] = 0;
        }
        digit_sync();  // shared memory reused by the next item
    }
}

// Bulk L2 prefetch of the K and V rows the CTA's attention items of layer l
// will read (rows before `pos` already exist; the row at `pos` is written by
// this step's qkv phase, in L2 by then).  Issued by one thread at the start of
// the qkv phase, so that attention finds its rows in L2.
template <typename KVT>
__device__ void prefetch_attn_rows(const StepArgs& a, uint32_t l) {
    const uint32_t row_bytes = a.hd * (uint32_t)sizeof(KVT);
    if (row_bytes % 16) return;
    const uint32_t c = min(a.st->pos + 1, a.max_seq), S = a.S_att;
    const uint32_t Lk = (c + S - 1) / S;
    const size_t layer_off = (size_t)l * a.KVH * a.max_seq * a.hd;
    for (uint32_t it = blockIdx.x; it < a.KVH * S; it += gridDim.x) {
        const uint32_t kvh = it / S, sidx = it % S;
        const uint32_t t0 = sidx * Lk, t1 = min(c, t0 + Lk);
        if (t1 <= t0) continue;
        const size_t off = (layer_off + ((size_t)kvh * a.max_seq + t0) * a.hd) * sizeof(KVT);
        const uint64_t bytes = (uint64_t)(t1 - t0) * row_bytes;
        for (int kv = 0; kv < 2; ++kv) {
            const uint8_t* base = static_cast<const uint8_t*>(kv ? a.vc : a.kc) + off;
            for (uint64_t o = 0; o < bytes; o += 32768) {
                const uint32_t n = (uint32_t)((bytes - o) < 32768 ? (bytes - o) : 32768);
                bulk_prefetch_l2(base + o, n);
            }
        }
    }
}

// ---------------------------------------------------------------- the step kernel

template <int NV, int GQM, typename KVT>
__global__ void __launch_bounds__(kMmaThreads, 1) decode_step_kernel(StepArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMmaMaxRing], empty[kMmaMaxRing], mma_done[kMmaMaxRing];
    __shared__ __align__(8) uint64_t red_full[kRedSlots], red_free[kRedSlots];
    __shared__ float red[kRedSlots][kTileRows];
    __shared__ float fin[kTileRows];
    __shared__ float redd[2 * kDigitWarps];
    __shared__ uint32_t s_tmem;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x, NS = a.NS;
    const uint32_t P = 5 * a.L + 1;
    uint32_t* err = &a.st->error;
    uint8_t* ring = smem;
    uint8_t* xb = smem + a.scratch_off;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kAccWarps);
            mbar_init(&mma_done[s], kStageTiles);
        }
        for (int r = 0; r < kRedSlots; ++r) {
            mbar_init(&red_full[r], kAccWarps);
            mbar_init(&red_free[r], 1);
        }
        fence_mbar_init();
    }
    if (warp == kMmaWarp0) {
        tmem_alloc(&s_tmem, a.tmem_cols);
        tmem_relinquish();
    }
    tcgen05_fence_before();
    __syncthreads();
    tcgen05_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == kProducerWarp) {
        // ---------------- producer: every GEMV of the step, back to back
        if (lane == 0) {
            uint32_t issued = 0, s = 0, ph = 0;
            bool ok = true;
            for (uint32_t p = 0; p < P && ok; ++p) {
                if (phase_kind(p, a.L) == kPhAttn) continue;
                const StepMat mt = phase_mat(a, p);
                const Geo gm = phase_geo(mt, c, G);
                for (uint32_t j = 0; j < gm.nstages; ++j) {
                    if (issued >= NS && !(ok = mbar_wait(&empty[s], ph ^ 1, err))) break;
                    const uint32_t ub = gm.u0 + j * kStageTiles;
                    const uint32_t n = min(kStageTiles, gm.u1 - ub);
                    mbar_expect_tx(&full[s], n * kTileBytes);
                    bulk_g2s(ring + (size_t)s * kStageBytes, mt.units + (size_t)ub * kTileBytes, n * kTileBytes,
                             &full[s]);
                    ++issued;
                    if (++s == NS) { s = 0; ph ^= 1; }
                }
            }
            const uint32_t first = issued > NS ? issued - NS : 0;
            for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, nullptr);
        }
        return;
    }

    // ---------------- consumers (warps 1-9)
    const uint32_t tid = threadIdx.x - 32;
    const uint32_t epoch = a.st->pad[0];
    const uint32_t target = G * (epoch + 1);
    bool ok = true;
    // per-role pipeline state, carried across phases
    uint32_t rs = 0, rph = 0;              // ring slot (issuers, accumulators)
    uint32_t qs = 0, qph = 0, qn = 0;      // reduction slot (accumulators, finisher) and slots used
    StreamState est{-INFINITY, 0xFFFFFFFFu};
    for (uint32_t p = 0; p < P; ++p) {
        const uint32_t kind = phase_kind(p, a.L);
        const uint32_t l = p / 5;
        const StepLayer* ly = kind == kPhHead ? nullptr : a.layers + l;
        MProStep pro{a.x, nullptr, a.eps, nullptr, a.st, a.x};
        if (kind == kPhQKV) {
            pro.w = ly->attn_norm;
            if (l == 0) pro.embed = a.embed;
        } else if (kind == kPhO) {
            pro.src = a.attn;
        } else if (kind == kPhGU) {
            pro.w = ly->ffn_norm;
        } else if (kind == kPhDown) {
            pro.src = a.act;
        } else if (kind == kPhHead) {
            pro.w = a.out_norm;
        }
        const StepMat mt = phase_mat(a, p);
        step_prefetch_w(kind == kPhAttn ? nullptr : pro.w, mt.K, tid);  // before the barrier
        if (p > 0) {
            if (tid == 0) wait_count(a.cnt + (p - 1), target, err);  // acquire
            digit_sync();
        }
        if (kind == kPhQKV && tid == 32 * 8) prefetch_attn_rows<KVT>(a, l);  // the finisher warp, before its first group
        if (kind == kPhAttn) {
            attn_phase<NV, GQM, KVT>(a, l, xb, tid);
            if (tid == 0) {
                __threadfence();
                atomicAdd(a.cnt + p, 1u);
            }
            continue;
        }
        const Geo gm = phase_geo(mt, c, G);
        bool bad = false;
        const int e = step_build_digits(pro, mt.K, xb, a.xstride, redd, tid, bad);

        if (warp < kAccWarp0) {
            // ---------------- MMA issue
            const uint32_t t = warp - kMmaWarp0;
            if (lane == 0) {
                uint32_t b = (gm.u0 + t) % gm.NB;
                const uint64_t a0 = umma_desc(smem_u32(ring + t * kTileBytes), 128, 256);
                const uint64_t b0 = umma_desc(smem_u32(xb), a.xstride, 128);
                const uint32_t d0 = tmem + t * kTileCols;
                uint32_t s = rs, ph = rph;
                for (uint32_t j = 0; j < gm.nstages; ++j) {
                    if (ok) ok = mbar_wait(&full[s], ph, err);
                    tcgen05_fence_after();
                    if (ok && t < min(kStageTiles, gm.u1 - (gm.u0 + j * kStageTiles)))
                        umma_s8(d0 + s * (kStageTiles * kTileCols), a0 + ((s * kStageBytes) >> 4), b0 + b * 3,
                                kIdescS8, 0);
                    umma_commit(&mma_done[s]);
                    if (++s == NS) { s = 0; ph ^= 1; }
                    b += kStageTiles;
                    while (b >= gm.NB) b -= gm.NB;
                }
            }
            // every issuer lane tracks the ring position
            for (uint32_t j = 0; j < gm.nstages; ++j)
                if (++rs == NS) { rs = 0; rph ^= 1; }
            __syncwarp();
            continue;
        }

        if (warp == kFinWarp) {
            // ---------------- finisher
            const bool resid = kind == kPhO || kind == kPhDown;
            for (uint32_t g = gm.g_first; g <= gm.g_last; ++g) {
                const uint32_t row0 = g * kTileRows;
                float xv[4];  // residual input, loaded before the merge wait
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    xv[i] = (resid && row0 + lane + 32 * i < mt.M) ? __ldcg(a.x + row0 + lane + 32 * i) : 0.0f;
                if (ok) ok = mbar_wait(&red_full[qs], qph, err);
                float v[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    v[i] = bad ? __int_as_float(0x7fc00000) : ldexpf(red[qs][lane + 32 * i], -e);
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_free[qs]);
                if (++qs == kRedSlots) { qs = 0; qph ^= 1; }
                const uint32_t c_lo = split_cta((uint64_t)g * gm.NB, gm.U, gm.Gm);
                const uint32_t c_hi = split_cta((uint64_t)(g + 1) * gm.NB - 1, gm.U, gm.Gm);
                if (c_lo != c_hi) {
                    const uint32_t side = g == gm.g_first ? 0 : 1;
                    float* part = a.split_part + ((size_t)c * 2 + side) * kTileRows;
#pragma unroll
                    for (int i = 0; i < 4; ++i) part[lane + 32 * i] = v[i];
                    __syncwarp();
                    uint32_t last = 0;  // release our partial, acquire the others' (last arriver)
                    if (lane == 0) last = atom_add_acq_rel_gpu(a.split_ticket + g, 1u) == c_hi - c_lo;
                    last = __shfl_sync(0xffffffffu, last, 0);
                    if (!last) continue;
#pragma unroll
                    for (int i = 0; i < 4; ++i) v[i] = 0.0f;
                    for (uint32_t cb = c_lo; cb <= c_hi; cb += 8) {  // 8 CTAs' partials in flight, summed in CTA order
                        float pv[8][4];
#pragma unroll
                        for (uint32_t u = 0; u < 8; ++u) {
                            const uint32_t cc = cb + u;
                            if (cc > c_hi) break;
                            const uint32_t first_cc = (uint32_t)(((uint64_t)gm.U * cc) / gm.Gm) / gm.NB;
                            const float* pc = a.split_part + ((size_t)cc * 2 + (g == first_cc ? 0 : 1)) * kTileRows;
#pragma unroll
                            for (int i = 0; i < 4; ++i) pv[u][i] = __ldcg(pc + lane + 32 * i);
                        }
#pragma unroll
                        for (uint32_t u = 0; u < 8; ++u) {
                            if (cb + u > c_hi) break;
#pragma unroll
                            for (int i = 0; i < 4; ++i) v[i] += pv[u][i];
                        }
                    }
                    if (lane == 0) a.split_ticket[g] = 0;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) fin[lane + 32 * i] = v[i];
                __syncwarp();
                auto rsf = [&](uint32_t t) { return fin[t]; };
                if (resid) {
                    // x += y (transformer_engine.cpp:191-195, 222-225), optional per-layer tap
                    float* tap = (kind == kPhDown && a.taps) ? a.taps + (size_t)l * a.D : nullptr;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t r = row0 + lane + 32 * i;
                        if (r >= mt.M) continue;
                        const float xn = __fadd_rn(xv[i], v[i]);
                        a.x[r] = xn;
                        if (tap) tap[r] = xn;
                    }
                } else if (kind == kPhQKV) {
                    EpiQKV<KVT> q{a.q,
                                  reinterpret_cast<KVT*>(a.kc) + (size_t)l * a.KVH * a.max_seq * a.hd,
                                  reinterpret_cast<KVT*>(a.vc) + (size_t)l * a.KVH * a.max_seq * a.hd,
                                  a.rope, a.st, a.D, a.KVD, a.hd, a.max_seq};
                    SEpiQKV<KVT>{q}.tile(est, row0, kTileRows, mt.M, lane, rsf);
                } else if (kind == kPhGU) {
                    SEpiSwiGLU{a.act}.tile(est, row0, kTileRows, mt.M, lane, rsf);
                } else {
                    EpiLogits lg{a.logits, a.am_val, a.am_idx, a.am_ticket, a.st, a.tok_hist, a.max_seq};
                    SEpiLogits{lg}.tile(est, row0, kTileRows, mt.M, lane, rsf);
                }
                __syncwarp();
            }
            if (kind == kPhHead) {
                EpiLogits lg{a.logits, a.am_val, a.am_idx, a.am_ticket, a.st, a.tok_hist, a.max_seq, true};
                SEpiLogits{lg}.end(est, lane);  // the last CTA advances the sequence (and its step count)
            } else if (lane == 0) {
                red_add_release_gpu(a.cnt + p, 1u);  // the warp's writes are ordered by the __syncwarp above
            }
            __syncwarp();
            continue;
        }

        // ---------------- accumulators
        {
            const uint32_t qd = warp & 3;
            const uint32_t row = 32 * qd + lane;
            const uint32_t taddr = tmem + ((32 * qd) << 16);
            float acc = 0.0f;
            uint32_t cur_g = gm.g_first;
            auto flush = [&]() {
                if (qn >= kRedSlots && ok) ok = mbar_wait(&red_free[qs], qph ^ 1, err);
                red[qs][row] = acc;
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_full[qs]);
                acc = 0.0f;
                ++qn;
                if (++qs == kRedSlots) { qs = 0; qph ^= 1; }
                ++cur_g;
            };
            uint32_t g = gm.u0 / gm.NB, b = gm.u0 - g * gm.NB;
            for (uint32_t j = 0; j < gm.nstages; ++j) {
                if (ok) ok = mbar_wait(&mma_done[rs], rph, err);
                tcgen05_fence_after();
                uint32_t d[32];
                tmem_ld32(taddr + rs * (kStageTiles * kTileCols), d);
                const uint32_t n = min(kStageTiles, gm.u1 - (gm.u0 + j * kStageTiles));
                const uint8_t* st = ring + (size_t)rs * kStageBytes + kTileQBytes + row * 4;
                float sc[kStageTiles];
#pragma unroll
                for (uint32_t t = 0; t < kStageTiles; ++t)
                    sc[t] = t < n ? *reinterpret_cast<const float*>(st + t * kTileBytes) : 0.0f;
                tmem_wait_ld();
                tcgen05_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[rs]);
                if (++rs == NS) { rs = 0; rph ^= 1; }
#pragma unroll
                for (uint32_t t = 0; t < kStageTiles; ++t) {
                    if (t < n) {
                        while (cur_g < g) flush();
                        const uint32_t* dt = d + kTileCols * t;
                        const float y = fmaf(fmaf(small_i2f((int)dt[0]), 256.0f, small_i2f((int)dt[1])), 256.0f,
                                             small_i2f((int)dt[2]));
                        acc = fmaf(sc[t], y, acc);
                    }
                    if (++b == gm.NB) { b = 0; ++g; }
                }
            }
            while (cur_g <= gm.g_last) flush();
        }
    }

    // ---------------- release the tensor memory (issuers and accumulators)
    if (warp < kFinWarp) {
        tcgen05_fence_before();
        tmem_sync();
        if (warp == kMmaWarp0) {
            tcgen05_fence_after();
            tmem_dealloc(tmem, a.tmem_cols);
        }
    }
}

}  // namespace bt
