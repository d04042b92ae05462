// bt_attn_mma.cuh -- decode attention of the query heads that share one KV head
// (grouped-query attention) on the tensor cores.
//
// The reference scores every key with every query head, s = q.k / sqrt(hd),
// softmaxes over the keys and sums p v (runtime/src/transformer_engine.cpp:
// 148-184, kernels/cpu_ref.hpp:55-72), all in fp32.  With G query heads per KV
// head the work of a block of 16 keys is two small matrix products, S = K Q^T
// (16 keys x hd x G heads) and O += P V (G heads x 16 keys x hd), so one warp
// issues them as mma.sync m16n8k8 (tf32 in, fp32 accumulate), the G <= 8 heads
// as the N dimension:
//   S^T = K Q^T : A = 16 key rows x 8 dims, B = Q^T (8 dims x 8 heads);
//   O^T += V^T P^T : A = 16 dims x 8 keys of V^T, B = P^T (8 keys x 8 heads).
// Accuracy: an fp16 cache element is exact in tf32 (11 significant bits); q and
// p are split into two tf32 terms, x = hi + lo with |x - hi - lo| <= 2^-22 |x|,
// and both terms are multiplied (fp32 caches split K and V too: hi.hi + hi.lo +
// lo.hi), so every product carries about the error of an fp32 multiply and the
// sums accumulate in fp32 like the CUDA-core kernels.
//
// Fragment layouts (PTX ISA, m16n8k8 tf32): lane = 4 g + c; A a0 (g, c), a1
// (g + 8, c), a2 (g, c + 4), a3 (g + 8, c + 4); B b0 (k c, n g), b1 (k c + 4,
// n g); C c0 (g, 2c), c1 (g, 2c + 1), c2 (g + 8, 2c), c3 (g + 8, 2c + 1).
// The order of the contracted dimension is free, so each lane's share of it is
// made contiguous: in S, lane c holds dims [c hd/4, (c + 1) hd/4) of its key
// rows and of q (k-step j takes dims c hd/4 + 2j and + 2j + 1); in O, the M
// index of tile mt, row g (g + 8) is dim g hd/8 + 2 mt (+ 1), so lane g loads
// dims [g hd/8, (g + 1) hd/8) of its V rows.  Every load is one contiguous run
// of a row, and a warp reads whole rows.
#pragma once

#include "bt_common.cuh"

namespace bt {

__device__ __forceinline__ uint32_t tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// x = hi + lo in tf32 (lo carries the next 11 bits).
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = tf32_rna(x);
    lo = tf32_rna(__fsub_rn(x, __uint_as_float(hi)));
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// N consecutive cache elements of one row as tf32 terms: fp16 is one exact
// term, fp32 two (hi, lo).
template <typename KVT, int N>
struct RowTf32;

template <int N>
struct RowTf32<__half, N> {
    static constexpr bool kTwo = false;
    uint32_t w[N / 2];  // the row's halves as loaded, two per word; converted when used
    __device__ __forceinline__ void load(const __half* p) {
        static_assert(N % 8 == 0, "16-byte loads");
#pragma unroll
        for (int i = 0; i < N / 8; ++i) {
            const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p) + i);
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
    }
    // the same from shared memory (rows staged by bulk copies)
    __device__ __forceinline__ void load_s(const __half* p) {
#pragma unroll
        for (int i = 0; i < N / 8; ++i) {
            const uint4 v = reinterpret_cast<const uint4*>(p)[i];
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < N / 2; ++i) w[i] = 0u;
    }
    // element i as tf32 (exact: 11 significant bits)
    __device__ __forceinline__ uint32_t hi(int i) const {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i >> 1]);
        return __float_as_uint((i & 1) ? __high2float(h) : __low2float(h));
    }
    __device__ __forceinline__ uint32_t lo(int) const { return 0u; }
};

template <int N>
struct RowTf32<float, N> {
    static constexpr bool kTwo = true;
    float w[N];  // split into hi + lo when used
    __device__ __forceinline__ void load(const float* p) {
        static_assert(N % 4 == 0, "16-byte loads");
#pragma unroll
        for (int i = 0; i < N / 4; ++i) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(p) + i);
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < N; ++i) w[i] = 0.0f;
    }
    __device__ __forceinline__ uint32_t hi(int i) const { return tf32_rna(w[i]); }
    __device__ __forceinline__ uint32_t lo(int i) const {
        return tf32_rna(__fsub_rn(w[i], __uint_as_float(tf32_rna(w[i]))));
    }
};

// One warp's share of the attention of up to 8 query heads over keys of one KV
// head: online softmax state of heads 2c and 2c + 1 (m: running max, l: this
// lane's part of the sum of e^(s - m)) and its part of O.  The B fragments of q
// (hi and lo terms) live in registers, or with kQSmem in shared memory, written
// once for all warps by stage_q ([k-step][lane] 16-byte entries: one
// conflict-free 16-byte load per lane and k-step), which frees HD/2 registers.
template <int HD, typename KVT, bool kQSmem = false>
struct GqaWarp {
    static constexpr int QD = HD / 4;   // dims of a lane in S (4 lanes per key row)
    static constexpr int VD = HD / 8;   // dims of a lane in O (8 lanes per V row)
    static constexpr int KSTEPS = HD / 8;
    static constexpr int MT = HD / 16;
    static constexpr int QREG = kQSmem ? 1 : QD;
    uint32_t qhi[QREG], qlo[QREG];
    const uint4* qs;
    float o[MT][4];
    float m[2], l[2];
    uint32_t g, c, lane_;

    // Shared-memory q fragments of heads 0 .. nh - 1 (q + head * HD), written by
    // threads tid of nthreads; 32 * KSTEPS entries.  The caller synchronises the
    // threads before the warps use them.
    __device__ static void stage_q(uint4* qs, const float* q, uint32_t nh, uint32_t tid, uint32_t nthreads) {
        for (uint32_t e = tid; e < 32u * KSTEPS; e += nthreads) {
            const uint32_t j = e >> 5, ln = e & 31, hg = ln >> 2, hc = ln & 3;
            float v0 = 0.0f, v1 = 0.0f;
            if (hg < nh) {
                const float* qp = q + (size_t)hg * HD + hc * QD + 2 * j;
                v0 = __ldcg(qp);
                v1 = __ldcg(qp + 1);
            }
            uint4 f;
            split_tf32(v0, f.x, f.z);
            split_tf32(v1, f.y, f.w);
            qs[e] = f;
        }
    }

    // q rows of heads 0 .. nh - 1 (heads >= nh are zero): q + head * HD (registers),
    // or the fragments stage_q wrote at qsm (kQSmem)
    __device__ __forceinline__ void init(const float* q, uint32_t nh, uint32_t lane, const uint4* qsm = nullptr) {
        g = lane >> 2;
        c = lane & 3;
        lane_ = lane;
        qs = qsm;
        if constexpr (!kQSmem) {
#pragma unroll
            for (int i = 0; i < QD; ++i) {
                const float v = g < nh ? __ldcg(q + (size_t)g * HD + c * QD + i) : 0.0f;
                split_tf32(v, qhi[i], qlo[i]);
            }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int k = 0; k < 4; ++k) o[t][k] = 0.0f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.0f;
    }

    // A tile's cache rows in registers: K rows g and g + 8, dims [c QD, c QD + QD)
    // (for S); V rows c, c + 4, 8 + c, 12 + c, dims [g VD, g VD + VD) (for O).
    struct Tile {
        RowTf32<KVT, QD> ka, kb;
        RowTf32<KVT, VD> v0, v1, v2, v3;
    };

    // Loads keys k0 .. k0 + 15 (rows >= t1 read as zero), rows at kc/vc + row(key).
    template <class RowOf>
    __device__ __forceinline__ void load(Tile& f, const KVT* kc, const KVT* vc, uint32_t k0, uint32_t t1,
                                         RowOf row) const {
        if (k0 + g < t1) f.ka.load(kc + row(k0 + g) + c * QD); else f.ka.zero();
        if (k0 + g + 8 < t1) f.kb.load(kc + row(k0 + g + 8) + c * QD); else f.kb.zero();
        if (k0 + c < t1) f.v0.load(vc + row(k0 + c) + g * VD); else f.v0.zero();
        if (k0 + c + 4 < t1) f.v1.load(vc + row(k0 + c + 4) + g * VD); else f.v1.zero();
        if (k0 + 8 + c < t1) f.v2.load(vc + row(k0 + 8 + c) + g * VD); else f.v2.zero();
        if (k0 + 12 + c < t1) f.v3.load(vc + row(k0 + 12 + c) + g * VD); else f.v3.zero();
    }

    // Keys k0 .. k0 + 15 (those >= t1 masked), rows at kc/vc + row(key).
    template <class RowOf>
    __device__ __forceinline__ void tile(const KVT* kc, const KVT* vc, uint32_t k0, uint32_t t1, float scale,
                                         RowOf row) {
        Tile f;
        load(f, kc, vc, k0, t1, row);
        compute(f, k0, t1, scale);
    }

    // The tile's scores, softmax update and P V (keys >= t1 masked).
    __device__ __forceinline__ void compute(const Tile& f, uint32_t k0, uint32_t t1, float scale) {
        const auto& ka = f.ka;
        const auto& kb = f.kb;
        const auto& v0 = f.v0;
        const auto& v1 = f.v1;
        const auto& v2 = f.v2;
        const auto& v3 = f.v3;
        const bool va = k0 + g < t1, vb = k0 + g + 8 < t1;
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < KSTEPS; ++j) {
            uint32_t h0, h1, l0, l1;
            if constexpr (kQSmem) {
                const uint4 f = qs[j * 32 + lane_];
                h0 = f.x; h1 = f.y; l0 = f.z; l1 = f.w;
            } else {
                h0 = qhi[2 * j]; h1 = qhi[2 * j + 1]; l0 = qlo[2 * j]; l1 = qlo[2 * j + 1];
            }
            const uint32_t a0 = ka.hi(2 * j), a1 = kb.hi(2 * j), a2 = ka.hi(2 * j + 1), a3 = kb.hi(2 * j + 1);
            mma_tf32(s, a0, a1, a2, a3, h0, h1);
            mma_tf32(s, a0, a1, a2, a3, l0, l1);
            if constexpr (RowTf32<KVT, QD>::kTwo)
                mma_tf32(s, ka.lo(2 * j), kb.lo(2 * j), ka.lo(2 * j + 1), kb.lo(2 * j + 1), h0, h1);
        }
        // ---- scores, masked; online softmax of heads 2c, 2c + 1 over the tile
        s[0] = va ? __fmul_rn(s[0], scale) : -INFINITY;
        s[1] = va ? __fmul_rn(s[1], scale) : -INFINITY;
        s[2] = vb ? __fmul_rn(s[2], scale) : -INFINITY;
        s[3] = vb ? __fmul_rn(s[3], scale) : -INFINITY;
        float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
        }
        const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
        // nothing seen yet (mn = -inf): scale 1, weights 0
        const float al0 = mn0 == -INFINITY ? 1.0f : expf(m[0] - mn0);
        const float al1 = mn1 == -INFINITY ? 1.0f : expf(m[1] - mn1);
        float p[4];
        p[0] = mn0 == -INFINITY ? 0.0f : expf(s[0] - mn0);
        p[1] = mn1 == -INFINITY ? 0.0f : expf(s[1] - mn1);
        p[2] = mn0 == -INFINITY ? 0.0f : expf(s[2] - mn0);
        p[3] = mn1 == -INFINITY ? 0.0f : expf(s[3] - mn1);
        l[0] = fmaf(l[0], al0, p[0] + p[2]);
        l[1] = fmaf(l[1], al1, p[1] + p[3]);
        m[0] = mn0;
        m[1] = mn1;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            o[t][0] *= al0;
            o[t][1] *= al1;
            o[t][2] *= al0;
            o[t][3] *= al1;
        }
        // ---- P^T fragments: b0 = P[head g][key 8 ks + c], b1 = P[head g][key 8 ks + c + 4], held by
        // lanes (g' = key mod 8, c' = g / 2) in p[ks * 2 + (g & 1)]
        const uint32_t srcA = (c << 2) | (g >> 1), srcB = ((c + 4) << 2) | (g >> 1);
        uint32_t bh[2][2], bl[2][2];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            const float xa0 = __shfl_sync(0xffffffffu, p[2 * ks], srcA);
            const float xa1 = __shfl_sync(0xffffffffu, p[2 * ks + 1], srcA);
            const float xb0 = __shfl_sync(0xffffffffu, p[2 * ks], srcB);
            const float xb1 = __shfl_sync(0xffffffffu, p[2 * ks + 1], srcB);
            split_tf32((g & 1) ? xa1 : xa0, bh[ks][0], bl[ks][0]);
            split_tf32((g & 1) ? xb1 : xb0, bh[ks][1], bl[ks][1]);
        }
        // ---- O^T += V^T P^T: tile mt rows g (dim g VD + 2 mt) and g + 8 (dim + 1)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const uint32_t x0 = v0.hi(2 * t), x1 = v0.hi(2 * t + 1), x2 = v1.hi(2 * t), x3 = v1.hi(2 * t + 1);
            const uint32_t y0 = v2.hi(2 * t), y1 = v2.hi(2 * t + 1), y2 = v3.hi(2 * t), y3 = v3.hi(2 * t + 1);
            mma_tf32(o[t], x0, x1, x2, x3, bh[0][0], bh[0][1]);
            mma_tf32(o[t], x0, x1, x2, x3, bl[0][0], bl[0][1]);
            mma_tf32(o[t], y0, y1, y2, y3, bh[1][0], bh[1][1]);
            mma_tf32(o[t], y0, y1, y2, y3, bl[1][0], bl[1][1]);
            if constexpr (RowTf32<KVT, VD>::kTwo) {
                mma_tf32(o[t], v0.lo(2 * t), v0.lo(2 * t + 1), v1.lo(2 * t), v1.lo(2 * t + 1), bh[0][0], bh[0][1]);
                mma_tf32(o[t], v2.lo(2 * t), v2.lo(2 * t + 1), v3.lo(2 * t), v3.lo(2 * t + 1), bh[1][0], bh[1][1]);
            }
        }
    }

    // The warp's (m, l, o) of heads < nh into out[head][HD + 2] = (m, l, o[0..HD)).
    __device__ __forceinline__ void store(float* out, uint32_t nh) {
        float lt0 = l[0], lt1 = l[1];
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
            lt0 += __shfl_xor_sync(0xffffffffu, lt0, sh);
            lt1 += __shfl_xor_sync(0xffffffffu, lt1, sh);
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const uint32_t h = 2 * c + hh;
            if (h >= nh) continue;
            float* p = out + (size_t)h * (HD + 2);
            if (g == 0) {
                p[0] = m[hh];
                p[1] = hh ? lt1 : lt0;
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                p[2 + g * VD + 2 * t] = o[t][hh];
                p[2 + g * VD + 2 * t + 1] = o[t][2 + hh];
            }
        }
    }
};

// ---------------------------------------------------------------- fp16 variant
// For fp16 caches the same products run as mma.sync m16n8k16 (f16 in, fp32
// accumulate): half the MMAs of the tf32 form, and the cache elements go to the
// tensor cores as loaded (no conversion).  q and p enter as two fp16 terms each,
// x = hi + lo (22 significant bits), scaled by a power of two first so neither
// term leaves fp16's normal range: q of head h by 2^e_h with max |q_h| 2^e_h in
// [2^13, 2^14) (per head, undone on the scores), p in [0, 1] by 2^14 (undone on
// o).  Fragments (m16n8k16 f16): A a0 (g, 2c..2c+1), a1 (g + 8, 2c..), a2 (g,
// 2c+8..2c+9), a3 (g + 8, 2c+8..); B b0 (k 2c..2c+1, n g), b1 (k 2c+8..2c+9,
// n g); C as above.  In S, k-step j of lane c covers dims c hd/4 + 4j .. + 3
// (the row's halves as loaded); in O the K index is the key (lane c holds keys
// 2c, 2c + 1, 2c + 8, 2c + 9 of the tile, pairs of halves of two V rows packed
// with one byte permute) and the M index as above.

__device__ __forceinline__ float attn_pow2(int k) { return __int_as_float((127 + k) << 23); }
// v 2^e for e in [-149, 149], in two exact steps
__device__ __forceinline__ float attn_scale2(float v, int e) {
    return __fmul_rn(__fmul_rn(v, attn_pow2(e / 2)), attn_pow2(e - e / 2));
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// x (already scaled) as fp16 hi and lo terms
__device__ __forceinline__ void split_f16(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

template <int HD>
struct GqaWarp16 {
    static constexpr int QD = HD / 4;  // dims of a lane in S
    static constexpr int VD = HD / 8;  // dims of a lane in O
    static constexpr int KSTEPS = HD / 16;
    static constexpr int MT = HD / 16;
    static constexpr float kPScale = 16384.0f;  // 2^14
    const uint4* qs;
    float o[MT][4];
    float m[2], l[2];
    int e0, e1;  // q exponents of heads 2c, 2c + 1
    uint32_t g, c, lane_;

    // Exponent of head w (warp w < nh, all lanes): max |q_w| 2^e in [2^13, 2^14); 0 for a zero or
    // non-finite head (inf / NaN then reach the scores as in fp32).
    __device__ static void head_exponent(int* qe, const float* q, uint32_t nh, uint32_t w, uint32_t lane) {
        if (w >= nh) return;
        float am = 0.0f;
        for (uint32_t d = lane; d < (uint32_t)HD; d += 32) am = fmaxf(am, fabsf(__ldcg(q + (size_t)w * HD + d)));
        am = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am)));
        int e = 0;
        if (am > 0.0f && isfinite(am)) {
            int ex;  // am = fr 2^ex, fr in [0.5, 1)
            if (am >= 1.17549435e-38f)
                ex = ((__float_as_int(am) >> 23) & 255) - 126;
            else
                frexpf(am, &ex);
            e = 14 - ex;
            if (e > 149) e = 149;
        }
        if (lane == 0) qe[w] = e;
    }

    // B fragments of q ([k-step][lane] 16-byte entries: hi of dims 4j..4j+3 of the lane's
    // share, then lo), heads >= nh zero; qe from head_exponent (visible to the threads).
    __device__ static void stage_q(uint4* qs, const float* q, const int* qe, uint32_t nh, uint32_t tid,
                                   uint32_t nthreads) {
        for (uint32_t e = tid; e < 32u * KSTEPS; e += nthreads) {
            const uint32_t j = e >> 5, ln = e & 31, hg = ln >> 2, hc = ln & 3;
            __half hi[4], lo[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float v = hg < nh ? attn_scale2(__ldcg(q + (size_t)hg * HD + hc * QD + 4 * j + i), qe[hg]) : 0.0f;
                split_f16(v, hi[i], lo[i]);
            }
            qs[e] = make_uint4(pack_h2(hi[0], hi[1]), pack_h2(hi[2], hi[3]), pack_h2(lo[0], lo[1]), pack_h2(lo[2], lo[3]));
        }
    }

    __device__ __forceinline__ void init(uint32_t nh, uint32_t lane, const uint4* qsm, const int* qe) {
        g = lane >> 2;
        c = lane & 3;
        lane_ = lane;
        qs = qsm;
        e0 = 2 * c < nh ? qe[2 * c] : 0;
        e1 = 2 * c + 1 < nh ? qe[2 * c + 1] : 0;
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int k = 0; k < 4; ++k) o[t][k] = 0.0f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.0f;
    }

    // K rows g and g + 8, dims [c QD, c QD + QD); V rows 2c, 2c + 1, 2c + 8, 2c + 9, dims
    // [g VD, g VD + VD)
    struct Tile {
        RowTf32<__half, QD> ka, kb;
        RowTf32<__half, VD> v0, v1, v2, v3;
    };

    template <class RowOf>
    __device__ __forceinline__ void load(Tile& f, const __half* kc, const __half* vc, uint32_t k0, uint32_t t1,
                                         RowOf row) const {
        if (k0 + g < t1) f.ka.load(kc + row(k0 + g) + c * QD); else f.ka.zero();
        if (k0 + g + 8 < t1) f.kb.load(kc + row(k0 + g + 8) + c * QD); else f.kb.zero();
        if (k0 + 2 * c < t1) f.v0.load(vc + row(k0 + 2 * c) + g * VD); else f.v0.zero();
        if (k0 + 2 * c + 1 < t1) f.v1.load(vc + row(k0 + 2 * c + 1) + g * VD); else f.v1.zero();
        if (k0 + 2 * c + 8 < t1) f.v2.load(vc + row(k0 + 2 * c + 8) + g * VD); else f.v2.zero();
        if (k0 + 2 * c + 9 < t1) f.v3.load(vc + row(k0 + 2 * c + 9) + g * VD); else f.v3.zero();
    }

    // Keys k0 .. k0 + 15 (those >= t1 masked), rows at kc/vc + row(key), loaded and computed.
    template <class RowOf>
    __device__ __forceinline__ void tile(const __half* kc, const __half* vc, uint32_t k0, uint32_t t1, float scale,
                                         RowOf row) {
        Tile f;
        load(f, kc, vc, k0, t1, row);
        compute(f, k0, t1, scale);
    }

    // The same from shared memory: key t's K (V) row at ks (vs) + (t - kb) HD.
    __device__ __forceinline__ void load_s(Tile& f, const __half* ks, const __half* vs, uint32_t kb, uint32_t k0,
                                           uint32_t t1) const {
        auto r = [&](uint32_t t) { return (size_t)(t - kb) * HD; };
        if (k0 + g < t1) f.ka.load_s(ks + r(k0 + g) + c * QD); else f.ka.zero();
        if (k0 + g + 8 < t1) f.kb.load_s(ks + r(k0 + g + 8) + c * QD); else f.kb.zero();
        if (k0 + 2 * c < t1) f.v0.load_s(vs + r(k0 + 2 * c) + g * VD); else f.v0.zero();
        if (k0 + 2 * c + 1 < t1) f.v1.load_s(vs + r(k0 + 2 * c + 1) + g * VD); else f.v1.zero();
        if (k0 + 2 * c + 8 < t1) f.v2.load_s(vs + r(k0 + 2 * c + 8) + g * VD); else f.v2.zero();
        if (k0 + 2 * c + 9 < t1) f.v3.load_s(vs + r(k0 + 2 * c + 9) + g * VD); else f.v3.zero();
    }

    __device__ __forceinline__ void compute(const Tile& f, uint32_t k0, uint32_t t1, float scale) {
        const bool va = k0 + g < t1, vb = k0 + g + 8 < t1;
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < KSTEPS; ++j) {
            const uint4 q = qs[j * 32 + lane_];
            const uint32_t a0 = f.ka.w[2 * j], a1 = f.kb.w[2 * j], a2 = f.ka.w[2 * j + 1], a3 = f.kb.w[2 * j + 1];
            mma_f16(s, a0, a1, a2, a3, q.x, q.y);
            mma_f16(s, a0, a1, a2, a3, q.z, q.w);
        }
        // ---- scores (q's scale undone exactly, then 1/sqrt(hd)), masked; online softmax
        s[0] = va ? __fmul_rn(attn_scale2(s[0], -e0), scale) : -INFINITY;
        s[1] = va ? __fmul_rn(attn_scale2(s[1], -e1), scale) : -INFINITY;
        s[2] = vb ? __fmul_rn(attn_scale2(s[2], -e0), scale) : -INFINITY;
        s[3] = vb ? __fmul_rn(attn_scale2(s[3], -e1), scale) : -INFINITY;
        float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
        }
        const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
        const float al0 = mn0 == -INFINITY ? 1.0f : expf(m[0] - mn0);
        const float al1 = mn1 == -INFINITY ? 1.0f : expf(m[1] - mn1);
        float p[4];
        p[0] = mn0 == -INFINITY ? 0.0f : expf(s[0] - mn0);
        p[1] = mn1 == -INFINITY ? 0.0f : expf(s[1] - mn1);
        p[2] = mn0 == -INFINITY ? 0.0f : expf(s[2] - mn0);
        p[3] = mn1 == -INFINITY ? 0.0f : expf(s[3] - mn1);
        l[0] = fmaf(l[0], al0, p[0] + p[2]);
        l[1] = fmaf(l[1], al1, p[1] + p[3]);
        m[0] = mn0;
        m[1] = mn1;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            o[t][0] *= al0;
            o[t][1] *= al1;
            o[t][2] *= al0;
            o[t][3] *= al1;
        }
        // ---- P^T fragments: P[head g][key k] for keys 2c, 2c + 1 (b0) and 2c + 8, 2c + 9 (b1);
        // key k < 8 (k + 8) of head g is p[g & 1] (p[2 + (g & 1)]) of lane 4 k + g / 2
        const uint32_t srcA = ((2 * c) << 2) | (g >> 1), srcB = ((2 * c + 1) << 2) | (g >> 1);
        float pa[4], pb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            pa[i] = __shfl_sync(0xffffffffu, p[i], srcA);
            pb[i] = __shfl_sync(0xffffffffu, p[i], srcB);
        }
        const uint32_t hs = g & 1;
        __half h00, l00, h01, l01, h10, l10, h11, l11;
        split_f16(__fmul_rn(hs ? pa[1] : pa[0], kPScale), h00, l00);  // key 2c
        split_f16(__fmul_rn(hs ? pb[1] : pb[0], kPScale), h01, l01);  // key 2c + 1
        split_f16(__fmul_rn(hs ? pa[3] : pa[2], kPScale), h10, l10);  // key 2c + 8
        split_f16(__fmul_rn(hs ? pb[3] : pb[2], kPScale), h11, l11);  // key 2c + 9
        const uint32_t bh0 = pack_h2(h00, h01), bh1 = pack_h2(h10, h11);
        const uint32_t bl0 = pack_h2(l00, l01), bl1 = pack_h2(l10, l11);
        // ---- O^T += V^T P^T: tile t rows g (dim g VD + 2t) and g + 8 (dim g VD + 2t + 1)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const uint32_t x0 = __byte_perm(f.v0.w[t], f.v1.w[t], 0x5410);  // dim 2t of keys 2c, 2c + 1
            const uint32_t x1 = __byte_perm(f.v0.w[t], f.v1.w[t], 0x7632);  // dim 2t + 1
            const uint32_t x2 = __byte_perm(f.v2.w[t], f.v3.w[t], 0x5410);
            const uint32_t x3 = __byte_perm(f.v2.w[t], f.v3.w[t], 0x7632);
            mma_f16(o[t], x0, x1, x2, x3, bh0, bh1);
            mma_f16(o[t], x0, x1, x2, x3, bl0, bl1);
        }
    }

    // The warp's (m, l, o) of heads < nh into out[head][HD + 2] (o with p's 2^14 undone).
    __device__ __forceinline__ void store(float* out, uint32_t nh) {
        float lt0 = l[0], lt1 = l[1];
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
            lt0 += __shfl_xor_sync(0xffffffffu, lt0, sh);
            lt1 += __shfl_xor_sync(0xffffffffu, lt1, sh);
        }
        constexpr float kInv = 1.0f / kPScale;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const uint32_t h = 2 * c + hh;
            if (h >= nh) continue;
            float* p = out + (size_t)h * (HD + 2);
            if (g == 0) {
                p[0] = m[hh];
                p[1] = hh ? lt1 : lt0;
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                p[2 + g * VD + 2 * t] = o[t][hh] * kInv;
                p[2 + g * VD + 2 * t + 1] = o[t][2 + hh] * kInv;
            }
        }
    }
};

}  // namespace bt
