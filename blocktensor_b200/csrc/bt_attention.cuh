// bt_attention.cuh -- split-K decode attention over the device KV cache.
//
// The reference computes attention on the host for every token
// (runtime/src/transformer_engine.cpp:148-184): per query head h,
// s_t = (q_h . k_t) / sqrt(hd), p = softmax(s) (kernels/cpu_ref.hpp:55-72),
// o_h = sum_t p_t v_t, with the GQA map kv_h = h / (H / KVH) (:161).
//
// Here: grid (KVH, S).  CTA (kvh, s) owns keys [s*L, min(c, (s+1)*L)),
// L = ceil(c/S), c = pos + 1, for the G = H/KVH query heads of kv head kvh.
// The cache layout [kv_head][max_seq][hd] makes the CTA's K rows and V rows two
// contiguous ranges, which arrive by two cp.async.bulk copies.  Rows before
// `pos` were written by earlier steps, so those copies are issued before
// griddepcontrol.wait and overlap the previous kernel; the row at `pos` (this
// step's K/V append) is loaded after it.  Each CTA writes an unnormalised
// partial (max m, sum l, o = sum e^(s-m) v); the last CTA of a KV head (atomic
// ticket) merges the S partials.
#pragma once

#include "bt_common.cuh"
#include "bt_gemv.cuh"
#include "bt_ptx.cuh"

namespace bt {

struct AttnArgs {
    const float* q;       // [H][hd] (after RoPE)
    const void* k;        // layer base [KVH][max_seq][hd]
    const void* v;
    float* out;           // [H][hd]
    float* part;          // [H][S][hd + 2]: m, l, o[hd]
    uint32_t* ticket;     // [KVH], zero between launches
    const DevState* st;   // position source; when null, `ctx` is the context length
    uint32_t* err;        // bounded-wait error flag (may be null)
    uint32_t hd, G, max_seq, lmax, ctx;
    float scale;          // 1/sqrt(hd) (transformer_engine.cpp:158)
    int bulk;             // rows are 16-byte multiples: stage K/V with bulk copies
};

template <int NV, int GT, typename KVT>
__global__ void __launch_bounds__(128) attn_decode_kernel(AttnArgs a) {
    extern __shared__ __align__(128) uint8_t sm_raw[];
    __shared__ float s_m[16], s_l[16];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t s_last;
    pdl_trigger();
    const uint32_t kvh = blockIdx.x, sidx = blockIdx.y, S = gridDim.y;
    const uint32_t HD = a.hd, G = a.G;
    // position of this step: written by the previous step (or the host) before this graph ran
    const uint32_t pos = a.st ? a.st->pos : a.ctx - 1;
    const uint32_t c = min(pos + 1, a.max_seq);
    const uint32_t L = (c + S - 1) / S;
    const uint32_t t0 = sidx * L;
    const uint32_t t1 = min(c, t0 + L);
    const uint32_t nk = t1 > t0 ? t1 - t0 : 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;

    const size_t row_bytes = (size_t)HD * sizeof(KVT);
    KVT* ks = reinterpret_cast<KVT*>(sm_raw);                      // [lmax][HD]
    KVT* vs = ks + (size_t)a.lmax * HD;                            // [lmax][HD]
    float* qs = reinterpret_cast<float*>(vs + (size_t)a.lmax * HD);  // [G][HD]
    float* sc = qs + G * HD;                                       // [G][lmax]
    const KVT* kb = reinterpret_cast<const KVT*>(a.k) + (size_t)kvh * a.max_seq * HD;
    const KVT* vb = reinterpret_cast<const KVT*>(a.v) + (size_t)kvh * a.max_seq * HD;

    // rows that no kernel of this step writes: in the engine every row before
    // `pos` (the row at `pos` is this step's append); standalone, all rows
    const uint32_t n_old = !a.bulk ? 0 : (a.st ? (pos > t0 ? min(nk, pos - t0) : 0) : nk);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && n_old > 0) {
        const uint32_t bytes = (uint32_t)(n_old * row_bytes);
        mbar_expect_tx(&bar, 2 * bytes);
        bulk_g2s(ks, kb + (size_t)t0 * HD, bytes, &bar);
        bulk_g2s(vs, vb + (size_t)t0 * HD, bytes, &bar);
    }
    pdl_wait();
    // remaining rows (this step's append, or all rows without bulk staging) and q
    for (uint32_t i = threadIdx.x; i < (nk - n_old) * HD; i += blockDim.x) {
        const uint32_t t = n_old + i / HD, d = i % HD;
        ks[(size_t)t * HD + d] = kb[(size_t)(t0 + t) * HD + d];
        vs[(size_t)t * HD + d] = vb[(size_t)(t0 + t) * HD + d];
    }
    for (uint32_t i = threadIdx.x; i < G * HD; i += blockDim.x) qs[i] = a.q[(size_t)kvh * G * HD + i];
    if (n_old > 0) mbar_wait(&bar, 0, a.err);
    __syncthreads();

    // scores: one warp per key, lanes over head dims (conflict-free rows in shared memory)
    for (uint32_t t = warp; t < nk; t += nw) {
        const KVT* kr = ks + (size_t)t * HD;
        float kv[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const uint32_t d = lane + 32 * i;
            kv[i] = d < HD ? KVConv<KVT>::to_f(kr[d]) : 0.0f;
        }
#pragma unroll
        for (int g = 0; g < GT; ++g) {
            if ((uint32_t)g >= G) break;
            float p = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const uint32_t d = lane + 32 * i;
                if (d < HD) p = fmaf(qs[g * HD + d], kv[i], p);
            }
            p = warp_sum(p);
            if (lane == 0) sc[g * a.lmax + t] = __fmul_rn(p, a.scale);
        }
    }
    __syncthreads();
    // per query head: max and sum of exponentials (cpu_ref.hpp:55-72)
    for (uint32_t g = warp; g < G; g += nw) {
        float m = -INFINITY;
        for (uint32_t t = lane; t < nk; t += 32) m = fmaxf(m, sc[g * a.lmax + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (uint32_t t = lane; t < nk; t += 32) {
            const float e = expf(sc[g * a.lmax + t] - m);
            sc[g * a.lmax + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { s_m[g] = m; s_l[g] = l; }
    }
    __syncthreads();
    // o = sum_t p_t v_t, threads over head dims
    const size_t pstride = HD + 2;
    for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x) {
        float acc[GT];
#pragma unroll
        for (int g = 0; g < GT; ++g) acc[g] = 0.0f;
        for (uint32_t t = 0; t < nk; ++t) {
            const float vv = KVConv<KVT>::to_f(vs[(size_t)t * HD + d]);
#pragma unroll
            for (int g = 0; g < GT; ++g)
                if ((uint32_t)g < G) acc[g] = fmaf(sc[g * a.lmax + t], vv, acc[g]);
        }
#pragma unroll
        for (int g = 0; g < GT; ++g)
            if ((uint32_t)g < G) a.part[((size_t)(kvh * G + g) * S + sidx) * pstride + 2 + d] = acc[g];
    }
    if (threadIdx.x < G) {
        float* p = a.part + ((size_t)(kvh * G + threadIdx.x) * S + sidx) * pstride;
        p[0] = s_m[threadIdx.x];
        p[1] = s_l[threadIdx.x];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(a.ticket + kvh, 1u) == S - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // merge: per-head maxima and weights of the S splits in shared memory, then o
    float* wts = sc;  // reuse: [G][S] weights e^(m_s - M) (0 for empty splits)
    for (uint32_t g = warp; g < G; g += nw) {
        const float* pb = a.part + (size_t)(kvh * G + g) * S * pstride;
        float M = -INFINITY;
        for (uint32_t s = lane; s < S; s += 32)
            if (__ldcg(pb + s * pstride + 1) > 0.0f) M = fmaxf(M, __ldcg(pb + s * pstride));
        M = warp_max(M);
        float l = 0.0f;
        for (uint32_t s = lane; s < S; s += 32) {
            const float ls = __ldcg(pb + s * pstride + 1);
            const float f = ls > 0.0f ? expf(__ldcg(pb + s * pstride) - M) : 0.0f;
            wts[g * S + s] = f;
            l = fmaf(ls, f, l);
        }
        l = warp_sum(l);
        if (lane == 0) s_l[g] = l;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const uint32_t g = i / HD, d = i % HD;
        const float* pb = a.part + (size_t)(kvh * G + g) * S * pstride + 2 + d;
        float o = 0.0f;
        uint32_t s = 0;
        for (; s + 8 <= S; s += 8) {  // 8 partials in flight
            float ov[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) ov[u] = __ldcg(pb + (s + u) * pstride);
#pragma unroll
            for (int u = 0; u < 8; ++u) o = fmaf(ov[u], wts[g * S + s + u], o);
        }
        for (; s < S; ++s) o = fmaf(__ldcg(pb + s * pstride), wts[g * S + s], o);
        a.out[(size_t)(kvh * G + g) * HD + d] = __fdiv_rn(o, s_l[g]);
    }
    if (threadIdx.x == 0) a.ticket[kvh] = 0;
}

// Split count and rows per split for a cache of max_seq rows.
inline void attn_plan(uint32_t kv_heads, uint32_t head_dim, uint32_t G, uint32_t max_seq, size_t esz, uint32_t nsm,
                      uint32_t& splits, uint32_t& lmax) {
    // >= 2 CTAs per SM over all KV heads, and K+V tiles of at most 32 KB per CTA
    uint32_t S = (2 * nsm + kv_heads - 1) / kv_heads;
    const uint64_t per_row = 2ull * head_dim * esz;
    const uint32_t s_mem = (uint32_t)((max_seq * per_row + 32767) / 32768);
    if (s_mem > S) S = s_mem;
    if (S > max_seq) S = max_seq;
    if (S < 1) S = 1;
    splits = S;
    lmax = (max_seq + S - 1) / S;
    (void)G;
}

inline size_t attn_smem(const AttnArgs& a, size_t esz, uint32_t S) {
    const size_t tiles = 2 * (size_t)a.lmax * a.hd * esz;
    const size_t sc = (size_t)a.G * (a.lmax > S ? a.lmax : S) * 4;
    return (tiles + 15) / 16 * 16 + (size_t)a.G * a.hd * 4 + sc;
}

template <int NV, int GT, typename KVT>
cudaError_t launch_attn_g(const AttnArgs& a, uint32_t KVH, uint32_t S, cudaStream_t s, bool pdl) {
    auto kern = attn_decode_kernel<NV, GT, KVT>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    return launch_pdl(kern, dim3(KVH, S), dim3(128), attn_smem(a, sizeof(KVT), S), s, pdl, a);
}

template <int NV, typename KVT>
cudaError_t launch_attn_t(const AttnArgs& a, uint32_t KVH, uint32_t S, cudaStream_t s, bool pdl) {
    if (a.G <= 1) return launch_attn_g<NV, 1, KVT>(a, KVH, S, s, pdl);
    if (a.G <= 2) return launch_attn_g<NV, 2, KVT>(a, KVH, S, s, pdl);
    if (a.G <= 4) return launch_attn_g<NV, 4, KVT>(a, KVH, S, s, pdl);
    if (a.G <= 8) return launch_attn_g<NV, 8, KVT>(a, KVH, S, s, pdl);
    return launch_attn_g<NV, 16, KVT>(a, KVH, S, s, pdl);
}

template <typename KVT>
cudaError_t launch_attn(const AttnArgs& a, uint32_t KVH, uint32_t S, cudaStream_t s, bool pdl) {
    const uint32_t nv = (a.hd + 31) / 32;
    if (nv <= 1) return launch_attn_t<1, KVT>(a, KVH, S, s, pdl);
    if (nv <= 2) return launch_attn_t<2, KVT>(a, KVH, S, s, pdl);
    if (nv <= 4) return launch_attn_t<4, KVT>(a, KVH, S, s, pdl);
    return launch_attn_t<8, KVT>(a, KVH, S, s, pdl);
}

}  // namespace bt
