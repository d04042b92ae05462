// bt_batch.cu -- batched decode: many independent sequences stepped together.
//
// The reference's KV cache holds one sequence (runtime/src/kv_cache.cpp:6-15)
// and forward_single_token processes one token (transformer_engine.cpp:228-251);
// a batch of n sequences is, by definition, n independent runs of that loop.
// Here one step processes the current token of every sequence of the batch at
// once: the projections as many-token tensor-core GEMMs (bt_gemm.cuh, one token
// row per sequence: the weights stream once for the whole batch), attention
// per sequence over its own cache, then the head GEMM with a greedy argmax per
// sequence.  Sequences may be at different positions (ragged contexts).
//
//   layer input  : token image of x * attn_norm (embedding rows for layer 0)
//   qkv GEMM     : RoPE at each sequence's position, K/V append into its cache (:117-146)
//   attention    : per (sequence, KV head, split of keys), then the splits merged (:148-184)
//   o GEMM       : x += o                                               (:186-195)
//   gate/up GEMM : silu(gate) * up                                      (:197-215)
//   down GEMM    : x += down                                            (:217-225)
//   head GEMM    : logits and a per-32-row argmax, reduced per sequence  (:244-250, sampler.hpp:11-13)
#include "bt_attn_mma.cuh"
#include "bt_common.cuh"
#include "bt_gemm.cuh"
#include "bt_step.cuh"
#include "bt_engine_impl.h"
#include "bt_internal.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

using namespace bt;

struct bt_batch {
    bt_engine* e = nullptr;
    uint32_t n_seq = 0, max_seq = 0;
    int dtype = BT_KV_FP32;
    std::vector<void*> allocs;
    void* k = nullptr;           // contiguous: [n_seq][L][KVH][max_seq][hd]; paged: [n_pages][L][KVH][P][hd]
    void* v = nullptr;
    size_t seq_stride = 0;       // contiguous: elements between two sequences' caches
    size_t layer_stride = 0;     // elements between two layers' bases (per sequence, or inside a page)
    KVMap map;                   // row addresses (the table pointer set when paged)
    // paged KV: a pool of n_pages pages of 2^page_shift positions shared by the sequences;
    // table[s][j] = the page holding positions j P .. j P + P - 1 of sequence s
    bool paged = false;
    uint32_t page_shift = 0, n_pages = 0, max_pages = 0;
    uint32_t* table = nullptr;              // device [n_seq][max_pages]
    std::vector<uint32_t> host_table;       // its host copy (kNoPage: none)
    std::vector<uint32_t> free_pages;       // pages no sequence holds (taken from the back)
    std::vector<uint32_t> seq_pages;        // pages held per sequence
    float2* rope = nullptr;      // [max_seq][hd/2]
    uint32_t* pos = nullptr;     // [n_seq] position of the token the next step processes
    uint32_t* cur = nullptr;     // [n_seq] the token it consumes
    uint32_t* n_fixed = nullptr; // [n_seq] tok_hist entries below this are given (the prompt)
    uint32_t* last_am = nullptr; // [n_seq] greedy token of the last step
    uint32_t* tok_hist = nullptr;// [n_seq][max_seq + 1]
    uint32_t* seq_idx = nullptr; // [n_seq] 0 .. n_seq - 1: the GEMM token -> sequence map
    uint32_t* err = nullptr;
    float* x = nullptr;          // [n_seq][D]
    float* q = nullptr;          // [n_seq][DQ]
    float* attn = nullptr;       // [n_seq][DQ]
    float* act = nullptr;        // [n_seq][F]
    float* logits = nullptr;     // [n_seq][V]
    float* ss = nullptr;         // [n_seq][D / 32]
    uint8_t* img[2] = {nullptr, nullptr};
    float* att_part = nullptr;   // [n_seq][KVH][S][GQ][hd + 2]
    uint32_t S = 1, kps = 1;     // attention splits, keys per split
    float* gpart = nullptr;      // split-K partial sums of the GEMMs with fewer units than SMs
    size_t gpart_floats = 0;
    float* am_val = nullptr;     // [n_seq][Mp(V) / 32]
    uint32_t* am_idx = nullptr;
    std::vector<uint32_t> host_pos;
    cudaGraphExec_t graph = nullptr;
    bool warmed = false;
    uint64_t launches_per_step = 0;  // kernels of one step (counted on the eager first step)
};

namespace bt {

// Greedy-argmax partials of the head GEMM: per token and 32-row block of the vocab,
// the best (value, row), first maximum winning (sampler.hpp:11-13).
struct GEpiLogits {
    float* logits;        // [T][V]
    float* pv;            // [T][nob]
    uint32_t* pi;
    uint32_t V, nob;
    template <class Bar>
    __device__ void rows(uint32_t r, uint32_t ob, uint32_t tok0, uint32_t nvalid, const float (&v)[16],
                         uint32_t lane, uint32_t, float*, Bar) const {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            if ((uint32_t)i >= nvalid) break;
            const uint32_t t = tok0 + i;
            float bv = -INFINITY;
            uint32_t bi = 0xFFFFFFFFu;
            if (r < V) {
                logits[(size_t)t * V + r] = v[i];
                bv = v[i];
                bi = r;
            }
            // NaN never wins (better()), as in std::max_element with operator<
            if (!(bv == bv)) { bv = -INFINITY; bi = 0xFFFFFFFFu; }
            warp_argmax(bv, bi);
            if (lane == 0 && ob < nob) {
                pv[(size_t)t * nob + ob] = bv;
                pi[(size_t)t * nob + ob] = bi;
            }
        }
    }
};

// Per sequence: the argmax over its partials in vocab order, then the next token
// (the prompt's while positions are given, else the argmax) and the position.
__global__ void batch_finish_kernel(const float* __restrict__ pv, const uint32_t* __restrict__ pi, uint32_t nob,
                                    uint32_t n_seq, uint32_t max_seq, uint32_t* pos, uint32_t* cur,
                                    const uint32_t* n_fixed, uint32_t* last_am, uint32_t* tok_hist) {
    const uint32_t s = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (s >= n_seq) return;
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t o = lane; o < nob; o += 32) {
        const float v = pv[(size_t)s * nob + o];
        const uint32_t i = pi[(size_t)s * nob + o];
        if (i != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || better(v, i, bv, bi))) { bv = v; bi = i; }
    }
    warp_argmax(bv, bi);
    if (lane == 0) {
        const uint32_t am = bi == 0xFFFFFFFFu ? 0 : bi;
        const uint32_t p = pos[s];
        if (p >= max_seq) return;  // the sequence is full: no further steps
        uint32_t* th = tok_hist + (size_t)s * (max_seq + 1);
        const uint32_t next = (p + 1 < n_fixed[s]) ? th[p + 1] : am;
        th[p + 1] = next;
        last_am[s] = am;
        cur[s] = next;
        pos[s] = p + 1;
    }
}

// Attention of a batch of decode tokens: block (split sp, KV head kvh, sequence s)
// takes keys [sp * kps, min(c_s, (sp + 1) * kps)) of sequence s's cache (c_s = its
// position + 1) for the query heads of kvh; warps take the keys round robin in
// batches of 8 (all loads in flight), online softmax per query head, lane i
// holding head dims NV i .. NV i + NV - 1; the warps' (m, l, o) are merged in
// shared memory and the split's written to part (l = 0: no keys).
// The CTA's partial of a split: its 8 warps' (m, l, o) [8][GQ][HD + 2] in shared
// memory merged (empty warps, l = 0, skipped) into out[GQ][HD + 2].
__device__ __forceinline__ void cta_merge_partials(const float* wm, float* out, uint32_t GQ, uint32_t HD,
                                                   uint32_t tid = threadIdx.x, uint32_t nthreads = blockDim.x) {
    const uint32_t pstride = HD + 2;
    for (uint32_t e = tid; e < GQ * HD; e += nthreads) {
        const uint32_t g = e / HD, d = e % HD;
        float M = -INFINITY;
        for (uint32_t ww = 0; ww < 8; ++ww) {
            const float* p = wm + ((size_t)ww * GQ + g) * pstride;
            if (p[1] > 0.0f) M = fmaxf(M, p[0]);
        }
        float lsum = 0.0f, acc = 0.0f;
        for (uint32_t ww = 0; ww < 8; ++ww) {
            const float* p = wm + ((size_t)ww * GQ + g) * pstride;
            if (p[1] > 0.0f) {
                const float f = expf(p[0] - M);
                lsum = fmaf(p[1], f, lsum);
                acc = fmaf(p[2 + d], f, acc);
            }
        }
        float* po = out + (size_t)g * pstride;
        po[2 + d] = acc;
        if (d == 0) { po[0] = M; po[1] = lsum; }
    }
}

struct BatchAttnArgs {
    const float* q;          // [B][DQ]
    const void* kc;          // this layer's K base (row addresses from map)
    const void* vc;
    KVMap map;
    const uint32_t* pos;     // [B]
    float* part;             // [B][KVH][S][GQ][hd + 2]
    uint32_t S, kps, KVH, GQ, hd, max_seq;
    float scale;
    uint32_t* err;           // set when a bounded wait gives up
};

template <int NV, int GQM, typename KVT>
__global__ void __launch_bounds__(256) batch_attn_kernel(BatchAttnArgs a) {
    extern __shared__ float wm[];  // [8 warps][GQ][hd + 2]
    constexpr int BW = 16 / RowWords<NV, KVT>::W / (GQM > 1 ? 2 : 1);
    constexpr int B = BW > 8 ? 8 : (BW < 2 ? 2 : BW);
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t sp = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
    const uint32_t HD = a.hd, GQ = a.GQ, pstride = HD + 2;
    const uint32_t c = min(a.pos[s] + 1, a.max_seq);
    const uint32_t t0 = sp * a.kps, t1 = min(c, t0 + a.kps);
    float* out = a.part + ((((size_t)s * a.KVH + kvh) * a.S + sp) * GQ) * pstride;
    if (t0 >= t1) {
        for (uint32_t g = threadIdx.x; g < GQ; g += blockDim.x) {
            out[(size_t)g * pstride] = -INFINITY;
            out[(size_t)g * pstride + 1] = 0.0f;
        }
        return;
    }
    const KVT* kc = static_cast<const KVT*>(a.kc);
    const KVT* vc = static_cast<const KVT*>(a.vc);
    const uint32_t d0 = lane * NV;
    const bool active = d0 < HD;
    const size_t DQ = (size_t)a.KVH * GQ * HD;
    for (uint32_t g0 = 0; g0 < GQ; g0 += GQM) {
        float qv[GQM][NV], o[GQM][NV], m[GQM], ls[GQM];
#pragma unroll
        for (int g = 0; g < GQM; ++g) {
            m[g] = -INFINITY;
            ls[g] = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                o[g][i] = 0.0f;
                qv[g][i] = (g0 + g < GQ && active) ? a.q[(size_t)s * DQ + (size_t)(kvh * GQ + g0 + g) * HD + d0 + i] : 0.0f;
            }
        }
        for (uint32_t base = t0 + w; base < t1; base += B * 8) {
            RowWords<NV, KVT> kr[B], vr[B];
#pragma unroll
            for (int j = 0; j < B; ++j) {
                const uint32_t t = base + j * 8;
                if (t < t1 && active) {
                    const size_t ro = a.map.row(s, kvh, t) + d0;
                    kr[j].load(kc + ro);
                    vr[j].load(vc + ro);
                } else {
                    kr[j].zero();
                    vr[j].zero();
                }
            }
#pragma unroll
            for (int g = 0; g < GQM; ++g) {
                if (g0 + g >= GQ) break;
                float sc[B];
                float mb = -INFINITY;
#pragma unroll
                for (int j = 0; j < B; ++j) {
                    float p = 0.0f;
#pragma unroll
                    for (int i = 0; i < NV; ++i) p = fmaf(qv[g][i], kr[j].at(i), p);
                    p = warp_sum(p);
                    sc[j] = base + j * 8 < t1 ? __fmul_rn(p, a.scale) : -INFINITY;
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
                    const float ev = expf(sc[j] - mn);  // 0 for keys past t1
                    lsum += ev;
#pragma unroll
                    for (int i = 0; i < NV; ++i) acc[i] = fmaf(ev, vr[j].at(i), acc[i]);
                }
                ls[g] = lsum;
                m[g] = mn;
#pragma unroll
                for (int i = 0; i < NV; ++i) o[g][i] = acc[i];
            }
        }
        for (uint32_t g = 0; g0 + g < GQ && g < (uint32_t)GQM; ++g) {
            float* p = wm + ((size_t)w * GQ + g0 + g) * pstride;
            if (lane == 0) { p[0] = m[g]; p[1] = ls[g]; }
#pragma unroll
            for (int i = 0; i < NV; ++i)
                if (active) p[2 + d0 + i] = o[g][i];
        }
    }
    __syncthreads();
    cta_merge_partials(wm, out, GQ, HD);
}

// Tensor-core variant (bt_attn_mma.cuh) for up to 8 query heads per KV head:
// warps take 16-key tiles of the split round robin.
template <int HD, typename KVT>
__global__ void __launch_bounds__(256, (HD == 64 && sizeof(KVT) == 2) ? 2 : 1) batch_attn_mma_kernel(BatchAttnArgs a) {
    extern __shared__ float wm[];  // [8 warps][GQ][HD + 2]
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t sp = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
    const uint32_t GQ = a.GQ, pstride = HD + 2;
    const uint32_t c = min(a.pos[s] + 1, a.max_seq);
    const uint32_t t0 = sp * a.kps, t1 = min(c, t0 + a.kps);
    float* out = a.part + ((((size_t)s * a.KVH + kvh) * a.S + sp) * GQ) * pstride;
    if (t0 >= t1) {
        for (uint32_t g = threadIdx.x; g < GQ; g += blockDim.x) {
            out[(size_t)g * pstride] = -INFINITY;
            out[(size_t)g * pstride + 1] = 0.0f;
        }
        return;
    }
    const KVT* kc = static_cast<const KVT*>(a.kc);
    const KVT* vc = static_cast<const KVT*>(a.vc);
    const size_t DQ = (size_t)a.KVH * GQ * HD;
    // q's fragments once for the 8 warps, after their partials
    using GW = GqaWarp<HD, KVT, true>;
    uint4* qs = reinterpret_cast<uint4*>(wm + ((size_t)8 * GQ * pstride + 3) / 4 * 4);
    GW::stage_q(qs, a.q + (size_t)s * DQ + (size_t)kvh * GQ * HD, GQ, threadIdx.x, blockDim.x);
    __syncthreads();
    GW st;
    st.init(nullptr, GQ, lane, qs);
    const KVMap map = a.map;
    auto row = [&](uint32_t t) { return map.row(s, kvh, t); };
    // the warp's tiles k0, k0 + 128, ...: the next tile's rows load while this one computes
    uint32_t k0 = t0 + 16 * w;
    typename GW::Tile cur, nxt;
    if (k0 < t1) st.load(cur, kc, vc, k0, t1, row);
    for (; k0 < t1; k0 += 16 * 8) {
        if (k0 + 16 * 8 < t1) st.load(nxt, kc, vc, k0 + 16 * 8, t1, row);
        st.compute(cur, k0, t1, a.scale);
        cur = nxt;
    }
    st.store(wm + (size_t)w * GQ * pstride, GQ);
    __syncthreads();
    cta_merge_partials(wm, out, GQ, HD);
}

// fp16 caches: a producer warp (warp 8) streams the split's K and V rows into a
// ring of shared-memory stages of 64 keys with bulk copies (one per contiguous
// run of rows: the whole stage, or a page's piece of it), and the 8 consumer
// warps take the 16-key tiles round robin (tile i: warp i mod 8; stage j's
// four tiles go to four warps, which release it), the products on f16 MMAs
// (GqaWarp16).  Copies run NS stages ahead of the slowest consumer, so the
// split's rows stream at the copy engine's pace instead of one 4 KB tile per
// warp and round trip.
constexpr uint32_t kAttnStageKeys = 64;
template <int HD>
constexpr uint32_t attn_bulk_stages() { return HD == 64 ? 4 : 5; }
template <int HD>
constexpr size_t attn_bulk_smem(uint32_t GQ) {
    // ring [NS][K | V][64 keys][HD] halves, the warps' partials [8][GQ][HD + 2], q's fragments, q's exponents
    return (size_t)attn_bulk_stages<HD>() * 2 * kAttnStageKeys * HD * 2 + (size_t)8 * GQ * (HD + 2) * 4 +
           (size_t)32 * (HD / 16) * 16 + 8 * 4;
}

template <int HD>
__global__ void __launch_bounds__(288, HD == 64 ? 2 : 1) batch_attn_bulk_kernel(BatchAttnArgs a) {
    constexpr uint32_t NS = attn_bulk_stages<HD>();
    constexpr uint32_t RB = HD * 2;                    // bytes per cache row
    constexpr uint32_t SB = kAttnStageKeys * RB;       // K (or V) bytes of a stage
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ __align__(8) uint64_t full[NS], empty[NS];
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t sp = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
    const uint32_t GQ = a.GQ, pstride = HD + 2;
    const uint32_t c = min(a.pos[s] + 1, a.max_seq);
    const uint32_t t0 = sp * a.kps, t1 = min(c, t0 + a.kps);
    float* out = a.part + ((((size_t)s * a.KVH + kvh) * a.S + sp) * GQ) * pstride;
    if (t0 >= t1) {
        for (uint32_t g = threadIdx.x; g < GQ; g += blockDim.x) {
            out[(size_t)g * pstride] = -INFINITY;
            out[(size_t)g * pstride + 1] = 0.0f;
        }
        return;
    }
    uint8_t* ring = sm;
    float* wm = reinterpret_cast<float*>(sm + (size_t)NS * 2 * SB);
    using GW = GqaWarp16<HD>;
    uint4* qs = reinterpret_cast<uint4*>(wm + (size_t)8 * GQ * pstride);
    int* qe = reinterpret_cast<int*>(qs + 32 * GW::KSTEPS);
    const uint32_t nst = (t1 - t0 + kAttnStageKeys - 1) / kAttnStageKeys;
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 4);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const KVMap map = a.map;
    if (w == 8) {
        // ---------------- producer
        if (lane == 0) {
            const uint8_t* kc = static_cast<const uint8_t*>(a.kc);
            const uint8_t* vc = static_cast<const uint8_t*>(a.vc);
            const uint32_t run_max = map.paged() ? (1u << map.page_shift) : 0xFFFFFFFFu;
            bool ok = true;
            for (uint32_t j = 0; j < nst && ok; ++j) {
                const uint32_t slot = j % NS;
                if (j >= NS) ok = mbar_wait(&empty[slot], ((j / NS) - 1) & 1, a.err);
                if (!ok) break;
                const uint32_t k0 = t0 + j * kAttnStageKeys, k1 = min(t1, k0 + kAttnStageKeys);
                mbar_expect_tx(&full[slot], 2 * (k1 - k0) * RB);
                uint8_t* dk = ring + (size_t)slot * 2 * SB;
                for (uint32_t t = k0; t < k1;) {
                    // rows t .. t + n - 1 are contiguous (one sequence's head, or one page's piece)
                    const uint32_t n = min(k1 - t, run_max - (t & (run_max - 1u)));
                    const size_t off = map.row(s, kvh, t) * 2;
                    bulk_g2s(dk + (size_t)(t - k0) * RB, kc + off, n * RB, &full[slot]);
                    bulk_g2s(dk + SB + (size_t)(t - k0) * RB, vc + off, n * RB, &full[slot]);
                    t += n;
                }
            }
            // the ring's copies still in flight land before the CTA may end
            const uint32_t first = nst > NS ? nst - NS : 0;
            for (uint32_t j = first; j < nst && ok; ++j) ok = mbar_wait(&full[j % NS], (j / NS) & 1, a.err);
        }
        return;
    }
    // ---------------- consumers (warps 0-7)
    auto csync = []() { asm volatile("bar.sync 1, 256;" ::: "memory"); };
    const float* qh = a.q + (size_t)s * ((size_t)a.KVH * GQ * HD) + (size_t)kvh * GQ * HD;
    GW::head_exponent(qe, qh, GQ, w, lane);
    csync();
    GW::stage_q(qs, qh, qe, GQ, threadIdx.x, 256);
    csync();
    GW st;
    st.init(GQ, lane, qs, qe);
    bool ok = true;
    for (uint32_t i = w; i < 4 * nst; i += 8) {
        const uint32_t j = i >> 2, slot = j % NS;
        if (ok) ok = mbar_wait(&full[slot], (j / NS) & 1, a.err);
        const uint32_t kb = t0 + j * kAttnStageKeys, k0 = t0 + 16 * i;
        const __half* ks = reinterpret_cast<const __half*>(ring + (size_t)slot * 2 * SB);
        typename GW::Tile f;
        st.load_s(f, ks, ks + SB / 2, kb, k0, ok ? t1 : 0);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // the tile is in registers
        st.compute(f, k0, ok ? t1 : 0, a.scale);
    }
    st.store(wm + (size_t)w * GQ * pstride, GQ);
    csync();
    cta_merge_partials(wm, out, GQ, HD, threadIdx.x, 256);
}

// attn[s][h hd + d] from the splits of (s, kv head, query head): the splits'
// maxima and sums first (lane i holds split i, i + 32, ...), then o as the
// weighted sum over the splits in split order.  One warp per (sequence, query
// head).  With img (head_dim a multiple of 32: a warp's 32 values are one
// block of the o-proj input) it also writes the o-proj GEMM's token image.
__global__ void batch_attn_merge_kernel(const float* __restrict__ part, float* __restrict__ attn, uint32_t B,
                                        uint32_t KVH, uint32_t GQ, uint32_t S, uint32_t hd, uint8_t* img) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t item = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const uint32_t H = KVH * GQ;
    if (item >= B * H) return;
    const uint32_t s = item / H, h = item % H, kvh = h / GQ, g = h % GQ;
    const uint32_t pstride = hd + 2;
    const float* base = part + (((size_t)s * KVH + kvh) * S * GQ + g) * pstride;  // split sp at + sp GQ pstride
    const size_t sstride = (size_t)GQ * pstride;
    float M = -INFINITY;
    for (uint32_t sp = lane; sp < S; sp += 32) {
        const float* p = base + sp * sstride;
        if (__ldg(p + 1) > 0.0f) M = fmaxf(M, __ldg(p));
    }
    M = warp_max(M);
    float L = 0.0f;
    for (uint32_t sp = lane; sp < S; sp += 32) {
        const float* p = base + sp * sstride;
        const float ls = __ldg(p + 1);
        if (ls > 0.0f) L = fmaf(ls, expf(__ldg(p) - M), L);
    }
    L = warp_sum(L);
    for (uint32_t d = lane; d < hd; d += 32) {
        float acc = 0.0f;
        for (uint32_t sp0 = 0; sp0 < S; sp0 += 8) {
            float ov[8], wv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t sp = sp0 + k;
                ov[k] = 0.0f;
                wv[k] = 0.0f;
                if (sp < S) {
                    const float* p = base + sp * sstride;
                    const float ls = __ldg(p + 1);
                    if (ls > 0.0f) {
                        wv[k] = expf(__ldg(p) - M);
                        ov[k] = __ldg(p + 2 + d);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) acc = fmaf(ov[k], wv[k], acc);
        }
        const float o = __fdiv_rn(acc, L);
        attn[(size_t)s * H * hd + (size_t)h * hd + d] = o;
        if (img) token_terms(img, H * hd / 32, s, (h * hd + d - lane) / 32, o, lane);  // warp-uniform
    }
}

namespace {

template <int NV, int GQM, typename KVT>
cudaError_t launch_batch_attn_t(const BatchAttnArgs& a, uint32_t B, cudaStream_t st) {
    const size_t smem = (size_t)8 * a.GQ * (a.hd + 2) * sizeof(float);
    auto kern = batch_attn_kernel<NV, GQM, KVT>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(kern, dim3(a.S, a.KVH, B), dim3(256), smem, st, false, a);
}

template <int HD, typename KVT>
cudaError_t launch_batch_attn_mma(const BatchAttnArgs& a, uint32_t B, cudaStream_t st) {
    // the warps' partials, then q's fragments (16 bytes per lane and k-step)
    const size_t smem = ((size_t)8 * a.GQ * (HD + 2) + 3) / 4 * 4 * sizeof(float) + (size_t)32 * (HD / 8) * 16;
    auto kern = batch_attn_mma_kernel<HD, KVT>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(kern, dim3(a.S, a.KVH, B), dim3(256), smem, st, false, a);
}

template <int HD>
cudaError_t launch_batch_attn_bulk(const BatchAttnArgs& a, uint32_t B, cudaStream_t st) {
    const size_t smem = attn_bulk_smem<HD>(a.GQ);
    auto kern = batch_attn_bulk_kernel<HD>;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(a.S, a.KVH, B), dim3(288), smem, st, false, a);
}

template <typename KVT>
cudaError_t launch_batch_attn(const BatchAttnArgs& a, uint32_t B, cudaStream_t st) {
    // the tensor-core kernels for head_dim 64 / 128 and up to 8 query heads per KV head
    if constexpr (sizeof(KVT) == 2) {
        if (a.GQ <= 8 && a.hd == 64) return launch_batch_attn_bulk<64>(a, B, st);
        if (a.GQ <= 8 && a.hd == 128) return launch_batch_attn_bulk<128>(a, B, st);
    } else {
        if (a.GQ <= 8 && a.hd == 64) return launch_batch_attn_mma<64, KVT>(a, B, st);
        if (a.GQ <= 8 && a.hd == 128) return launch_batch_attn_mma<128, KVT>(a, B, st);
    }
    const bool mha = a.GQ == 1;
#define BT_BATCH_ATTN(NV_)                                                                               \
    return mha ? launch_batch_attn_t<NV_, 1, KVT>(a, B, st) : launch_batch_attn_t<NV_, 16 / NV_, KVT>(a, B, st)
    if (a.hd <= 64) { BT_BATCH_ATTN(2); }
    if (a.hd <= 128) { BT_BATCH_ATTN(4); }
    BT_BATCH_ATTN(8);
#undef BT_BATCH_ATTN
}

template <typename KVT>
int enqueue_batch_step(bt_batch* b, cudaStream_t s) {
    bt_engine* e = b->e;
    const auto& c = e->lc;
    const uint32_t D = c.dim, F = c.hidden_dim, Q = qd(c), KV = kvd(c), hd = c.head_dim, V = c.vocab_size;
    const uint32_t QKV = Q + 2 * KV, L = c.num_layers, nsm = e->num_sms, B = b->n_seq;
    const uint32_t GQ = c.num_heads / c.num_kv_heads;
    uint32_t* err = b->err;
    // GEMM inputs with the split-K workspace (used when a GEMM has fewer units than SMs)
    auto gin = [&](const uint8_t* img, const float* ss, float eps) {
        GemmIn g{img, ss, eps, B};
        g.part = b->gpart;
        g.part_floats = b->gpart_floats;
        return g;
    };
    BT_CUDA_CHECK(launch_token_image(e->embed, b->cur, e->layers[0].attn_norm, B, D, b->img[0], b->ss, b->x, s));
    for (uint32_t l = 0; l < L; ++l) {
        const LayerDev& Ld = e->layers[l];
        KVT* kl = static_cast<KVT*>(b->k) + l * b->layer_stride;
        KVT* vl = static_cast<KVT*>(b->v) + l * b->layer_stride;
        {
            GEpiQKV<KVT> epi{b->q, kl, vl, b->map, b->rope, GemmTok{B, b->pos, b->seq_idx}, Q, KV, hd};
            BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.qkv, QKV, unit_rows(QKV), D}, gin(b->img[0], b->ss, c.rms_norm_eps),
                                             epi, err, nsm, s));
        }
        BatchAttnArgs aa{b->q, kl, vl, b->map, b->pos, b->att_part, b->S, b->kps, c.num_kv_heads, GQ, hd,
                         b->max_seq, 1.0f / std::sqrt((float)hd), err};
        BT_CUDA_CHECK(launch_batch_attn<KVT>(aa, B, s));
        {
            const uint32_t items = B * c.num_heads;
            // the merge writes the o-proj input's token image too when a head is whole 32-blocks
            uint8_t* oimg = hd % 32 == 0 ? b->img[1] : nullptr;
            BT_CUDA_CHECK(launch_pdl(batch_attn_merge_kernel, dim3((items + 7) / 8), dim3(256), 0, s, false,
                                     (const float*)b->att_part, b->attn, B, c.num_kv_heads, GQ, b->S, hd, oimg));
            if (!oimg) BT_CUDA_CHECK(launch_token_image(b->attn, nullptr, nullptr, B, Q, b->img[1], nullptr, nullptr, s));
        }
        BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.o, D, unit_rows(D), Q}, gin(b->img[1], nullptr, 0.0f),
                                         GEpiResidual{b->x, Ld.ffn_norm, b->img[0], b->ss, nullptr, D}, err, nsm, s));
        BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.gu, 2 * F, unit_rows(2 * F), D}, gin(b->img[0], b->ss, c.rms_norm_eps),
                                         GEpiSwiGLU{b->act, b->img[1], F}, err, nsm, s));
        const float* wn = l + 1 < L ? e->layers[l + 1].attn_norm : e->out_norm;
        BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.d, D, unit_rows(D), F}, gin(b->img[1], nullptr, 0.0f),
                                         GEpiResidual{b->x, wn, b->img[0], b->ss, nullptr, D}, err, nsm, s));
    }
    const uint32_t nob = unit_rows(V) / 32;
    BT_CUDA_CHECK(launch_gemm_tokens(UnitW{e->head, V, unit_rows(V), D}, gin(b->img[0], b->ss, c.rms_norm_eps),
                                     GEpiLogits{b->logits, b->am_val, b->am_idx, V, nob}, err, nsm, s));
    BT_CUDA_CHECK(launch_pdl(batch_finish_kernel, dim3((B + 7) / 8), dim3(256), 0, s, false, (const float*)b->am_val,
                             (const uint32_t*)b->am_idx, nob, B, b->max_seq, b->pos, b->cur,
                             (const uint32_t*)b->n_fixed, b->last_am, b->tok_hist));
    return BT_OK;
}

int enqueue_batch(bt_batch* b, cudaStream_t s) {
    return b->dtype == BT_KV_FP16 ? enqueue_batch_step<__half>(b, s) : enqueue_batch_step<float>(b, s);
}

int check_batch(bt_batch* b) {
    if (!b) return fail(BT_ERR_INVALID_ARGUMENT, "null batch");
    if (!b->e) return fail(BT_ERR_INVALID_ARGUMENT, "batch outlived its engine");
    return BT_OK;
}

}  // namespace
}  // namespace bt

extern "C" {

}  // extern "C"

namespace {

constexpr uint32_t kNoPage = 0xFFFFFFFFu;

// Paged KV: gives sequence s pages for its positions [0, n), taking pages from
// the pool for the page-sized runs it does not hold yet and uploading those
// table entries on stream st (ordered before the kernels that use them).
// BT_ERR_OUT_OF_MEMORY, with nothing taken, when the pool has too few pages.
int ensure_pages(bt_batch* b, uint32_t s, uint32_t n, cudaStream_t st) {
    if (!b->paged || n == 0) return BT_OK;
    const uint32_t need = (n + (1u << b->page_shift) - 1u) >> b->page_shift;
    if (need > b->max_pages) return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    const uint32_t have = b->seq_pages[s];
    if (need <= have) return BT_OK;
    if (need - have > b->free_pages.size())
        return fail(BT_ERR_OUT_OF_MEMORY, "paged KV: the page pool has too few free pages");
    uint32_t* row = b->host_table.data() + (size_t)s * b->max_pages;
    for (uint32_t j = have; j < need; ++j) {
        row[j] = b->free_pages.back();
        b->free_pages.pop_back();
    }
    b->seq_pages[s] = need;
    // from pageable memory: staged before the call returns, so the host table may change afterwards
    BT_CUDA_CHECK(cudaMemcpyAsync(b->table + (size_t)s * b->max_pages + have, row + have,
                                  sizeof(uint32_t) * (need - have), cudaMemcpyHostToDevice, st));
    return BT_OK;
}

// Paged KV: returns sequence s's pages to the pool and marks it idle (no work in
// later steps).  The caller has synchronised the streams that used the pages.
int drop_pages(bt_batch* b, uint32_t s, cudaStream_t st) {
    uint32_t* row = b->host_table.data() + (size_t)s * b->max_pages;
    for (uint32_t j = 0; j < b->seq_pages[s]; ++j) {
        b->free_pages.push_back(row[j]);
        row[j] = kNoPage;
    }
    b->seq_pages[s] = 0;
    const uint32_t idle = 0xFFFFFFFFu;  // position "not started": the kernels skip the sequence
    BT_CUDA_CHECK(cudaMemcpyAsync(b->table + (size_t)s * b->max_pages, row, sizeof(uint32_t) * b->max_pages,
                                  cudaMemcpyHostToDevice, st));
    BT_CUDA_CHECK(cudaMemcpyAsync(b->pos + s, &idle, sizeof(idle), cudaMemcpyHostToDevice, st));
    BT_CUDA_CHECK(cudaStreamSynchronize(st));
    b->host_pos[s] = b->max_seq;
    return BT_OK;
}

// A batch with contiguous per-sequence caches (page_tokens 0) or with its KV in a
// pool of n_pages pages of page_tokens positions.
int batch_create(bt_engine* e, uint32_t n_seq, uint32_t max_seq, int kv_dtype, uint32_t page_tokens,
                 uint32_t n_pages, bt_batch** out) {
    if (!e || !out) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: null argument");
    *out = nullptr;
    if (n_seq == 0 || max_seq == 0) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: n_seq and max_seq must be > 0");
    if (kv_dtype != BT_KV_FP32 && kv_dtype != BT_KV_FP16) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: bad kv dtype");
    if (e->tp_world > 1) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: not available under tensor parallelism");
    if (page_tokens) {
        if (page_tokens < 16 || page_tokens > 4096 || (page_tokens & (page_tokens - 1)))
            return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create_paged: page_tokens must be a power of two in [16, 4096]");
        if (n_pages == 0) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create_paged: n_pages must be > 0");
    }
    DeviceGuard guard(e->device);
    const auto& c = e->lc;
    auto b = new bt_batch();
    b->e = e;
    b->n_seq = n_seq;
    b->max_seq = max_seq;
    b->dtype = kv_dtype;
    auto cleanup = [&](int rc) {
        std::string msg = bt_cuda_last_error();
        bt_batch_destroy(b);
        set_error(msg);
        return rc;
    };
    const size_t esz = kv_dtype == BT_KV_FP16 ? 2 : 4;
    const uint32_t D = c.dim, F = c.hidden_dim, Q = qd(c), V = c.vocab_size, hd = c.head_dim;
    const uint32_t GQ = c.num_heads / c.num_kv_heads;
    size_t n = 0;  // cache elements (K, and again V)
    b->map.hd = hd;
    b->map.max_seq = max_seq;
    if (page_tokens) {
        b->paged = true;
        while ((1u << b->page_shift) < page_tokens) ++b->page_shift;
        b->n_pages = n_pages;
        b->max_pages = (max_seq + page_tokens - 1) / page_tokens;
        b->layer_stride = (size_t)c.num_kv_heads * page_tokens * hd;
        b->map.page_stride = b->layer_stride * c.num_layers;
        b->map.page_shift = b->page_shift;
        b->map.max_pages = b->max_pages;
        n = b->map.page_stride * n_pages;
    } else {
        b->seq_stride = (size_t)c.num_layers * c.num_kv_heads * max_seq * hd;
        b->layer_stride = (size_t)c.num_kv_heads * max_seq * hd;
        b->map.seq_stride = b->seq_stride;
        n = b->seq_stride * n_seq;
    }
    uint8_t *kb = nullptr, *vb = nullptr;
    int rc;
    if ((rc = dev_alloc(b->allocs, &kb, n * esz, "batch K cache"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &vb, n * esz, "batch V cache"))) return cleanup(rc);
    b->k = kb;
    b->v = vb;
    if (b->paged) {
        if ((rc = dev_alloc(b->allocs, &b->table, (size_t)n_seq * b->max_pages, "page table"))) return cleanup(rc);
        b->map.table = b->table;
        b->host_table.assign((size_t)n_seq * b->max_pages, kNoPage);
        b->seq_pages.assign(n_seq, 0);
        b->free_pages.resize(n_pages);
        for (uint32_t i = 0; i < n_pages; ++i) b->free_pages[i] = n_pages - 1 - i;  // page 0 is taken first
    }
    if ((rc = dev_alloc(b->allocs, &b->rope, (size_t)max_seq * (hd / 2), "rope table"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->pos, n_seq, "positions"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->cur, n_seq, "current tokens"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->n_fixed, n_seq, "prompt lengths"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->last_am, n_seq, "argmax"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->tok_hist, (size_t)n_seq * (max_seq + 1), "token history"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->seq_idx, n_seq, "sequence index"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->err, 4, "error flag"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->x, (size_t)n_seq * D, "x"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->q, (size_t)n_seq * Q, "q"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->attn, (size_t)n_seq * Q, "attention"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->act, (size_t)n_seq * F, "act"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->logits, (size_t)n_seq * V, "logits"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->ss, (size_t)n_seq * (D / 32), "norm sums"))) return cleanup(rc);
    const uint32_t k0 = std::max(D, Q), k1 = std::max(F, Q);
    if ((rc = dev_alloc(b->allocs, &b->img[0], token_image_bytes(n_seq, k0), "token image"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->img[1], token_image_bytes(n_seq, k1), "token image"))) return cleanup(rc);
    // attention splits (per sequence and KV head) of kps keys, a multiple of 128 (the 8 warps'
    // 16-key tiles): about 6 splits per SM over the batch's (sequence, KV head) pairs at
    // max_seq (64 TinyLlama-shaped sequences of up to 4k keys: 1152; measured 256, 512, 1024,
    // 1408, 2048: 14.2k, 15.0k, 15.1k, 14.6k, 14.6k tokens/s); BT_BATCH_KPS (a multiple of 16)
    // overrides
    {
        const uint32_t pairs = n_seq * c.num_kv_heads, tiles = (max_seq + 127) / 128;
        uint32_t S = (6 * e->num_sms + pairs - 1) / pairs;
        S = std::max(1u, std::min(S, tiles));
        b->kps = (max_seq + S - 1) / S;
        b->kps = (b->kps + 127) / 128 * 128;
        if (const char* v = std::getenv("BT_BATCH_KPS")) {
            const long k = std::atol(v);
            if (k >= 16 && k <= 65536 && k % 16 == 0) b->kps = (uint32_t)k;
        }
        b->S = (max_seq + b->kps - 1) / b->kps;
    }
    if ((rc = dev_alloc(b->allocs, &b->att_part, (size_t)n_seq * c.num_kv_heads * b->S * GQ * (hd + 2), "splits")))
        return cleanup(rc);
    // split-K partials: a GEMM with fewer units than SMs is cut into up to about two units per SM
    b->gpart_floats = gemm_split_floats(e->num_sms);
    if ((rc = dev_alloc(b->allocs, &b->gpart, b->gpart_floats, "GEMM split partials"))) return cleanup(rc);
    const size_t nob = unit_rows(V) / 32;
    if ((rc = dev_alloc(b->allocs, &b->am_val, (size_t)n_seq * nob, "argmax partials"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &b->am_idx, (size_t)n_seq * nob, "argmax partials"))) return cleanup(rc);
    cudaStream_t s = e->stream;
    std::vector<uint32_t> idx(n_seq);
    for (uint32_t i = 0; i < n_seq; ++i) idx[i] = i;
    cudaError_t ce = cudaMemcpyAsync(b->seq_idx, idx.data(), sizeof(uint32_t) * n_seq, cudaMemcpyHostToDevice, s);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b->pos, 0xFF, sizeof(uint32_t) * n_seq, s);  // not started: "full"
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b->err, 0, 4, s);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b->cur, 0, sizeof(uint32_t) * n_seq, s);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b->n_fixed, 0, sizeof(uint32_t) * n_seq, s);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b->tok_hist, 0, sizeof(uint32_t) * n_seq * (max_seq + 1), s);
    if (ce == cudaSuccess && b->paged)
        ce = cudaMemcpyAsync(b->table, b->host_table.data(), sizeof(uint32_t) * b->host_table.size(),
                             cudaMemcpyHostToDevice, s);
    std::vector<float2> tab((size_t)max_seq * (hd / 2));
    for (uint32_t i = 0; i < hd / 2; ++i) {
        const float freq = 1.0f / std::pow(e->theta, (float)(2 * i) / (float)hd);  // kernels/cpu_ref.hpp:40-43
        for (uint32_t p = 0; p < max_seq; ++p) {
            const float val = (float)p * freq;
            tab[(size_t)p * (hd / 2) + i] = make_float2(std::cos(val), std::sin(val));
        }
    }
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(b->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) return cleanup(fail(BT_ERR_CUDA, cudaGetErrorString(ce)));
    b->host_pos.assign(n_seq, max_seq);
    *out = b;
    return BT_OK;
}

}  // namespace

extern "C" {

int bt_batch_create(bt_engine* e, uint32_t n_seq, uint32_t max_seq, int kv_dtype, bt_batch** out) {
    return batch_create(e, n_seq, max_seq, kv_dtype, 0, 0, out);
}

int bt_batch_create_paged(bt_engine* e, uint32_t n_seq, uint32_t max_seq, uint32_t page_tokens, uint32_t n_pages,
                          int kv_dtype, bt_batch** out) {
    return batch_create(e, n_seq, max_seq, kv_dtype, page_tokens, n_pages, out);
}

int bt_batch_release(bt_batch* b, uint32_t s) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    if (s >= b->n_seq) return fail(BT_ERR_OUT_OF_RANGE, "bt_batch_release: sequence index out of range");
    if (!b->paged) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_release: the batch has no page pool");
    DeviceGuard guard(b->e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(b->e->stream));
    return drop_pages(b, s, b->e->stream);
}

int bt_batch_pages(bt_batch* b, uint32_t* free_pages, uint32_t* total_pages) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    if (free_pages) *free_pages = b->paged ? (uint32_t)b->free_pages.size() : 0u;
    if (total_pages) *total_pages = b->paged ? b->n_pages : 0u;
    return BT_OK;
}

int bt_batch_destroy(bt_batch* b) {
    if (!b) return BT_OK;
    if (b->e) {
        DeviceGuard guard(b->e->device);
        cudaStreamSynchronize(b->e->stream);
        if (b->graph) cudaGraphExecDestroy(b->graph);
        for (void* p : b->allocs) cudaFree(p);
    }
    delete b;
    return BT_OK;
}

int bt_batch_prefill(bt_batch* b, uint32_t s, const uint32_t* prompt, uint32_t n_prompt) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    bt_engine* e = b->e;
    if (s >= b->n_seq) return fail(BT_ERR_OUT_OF_RANGE, "bt_batch_prefill: sequence index out of range");
    if (!prompt || n_prompt == 0) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_prefill: empty prompt");
    if (n_prompt > b->max_seq) return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] >= e->cfg.vocab_size) return fail(BT_ERR_OUT_OF_RANGE, "Token ID out of vocab bounds");
    if (!e->loaded) return fail(BT_ERR_RUNTIME, "engine has no weights (call bt_engine_load or bt_engine_generate)");
    DeviceGuard guard(e->device);
    rc = ensure_prefill_buffers(e);
    if (rc != BT_OK) return rc;
    cudaStream_t st = e->stream;
    const size_t esz = b->dtype == BT_KV_FP16 ? 2 : 4;
    CacheRef cr{static_cast<uint8_t*>(b->k), static_cast<uint8_t*>(b->v), b->rope, b->max_seq, b->err,
                kv_map_flat(b->max_seq, e->lc.head_dim), b->layer_stride};
    if (b->paged) {
        // a new sequence in this slot: the previous one's pages go back to the pool first
        BT_CUDA_CHECK(cudaStreamSynchronize(st));
        if (b->seq_pages[s] && (rc = drop_pages(b, s, st)) != BT_OK) return rc;
        if ((rc = ensure_pages(b, s, n_prompt, st)) != BT_OK) return rc;
        cr.map = b->map;
        cr.map.table = b->table + (size_t)s * b->max_pages;  // the sequence's row: index 0 in the map
    } else {
        cr.k = static_cast<uint8_t*>(b->k) + (size_t)s * b->seq_stride * esz;
        cr.v = static_cast<uint8_t*>(b->v) + (size_t)s * b->seq_stride * esz;
    }
    const uint32_t n_fill = n_prompt - 1;
    for (uint32_t done = 0; done < n_fill;) {
        const uint32_t T = std::min(n_fill - done, e->pf_cap);
        BT_CUDA_CHECK(cudaMemcpyAsync(e->pf_tok, prompt + done, sizeof(uint32_t) * T, cudaMemcpyHostToDevice, st));
        rc = b->dtype == BT_KV_FP16 ? prefill_chunk_t<__half>(e, cr, T, done, st) : prefill_chunk_t<float>(e, cr, T, done, st);
        if (rc != BT_OK) return rc;
        BT_CUDA_CHECK(cudaStreamSynchronize(st));
        done += T;
    }
    // sequence s: position n_prompt - 1 consuming the last prompt token next
    const uint32_t hs[3] = {n_fill, prompt[n_fill], n_prompt};
    BT_CUDA_CHECK(cudaMemcpyAsync(b->tok_hist + (size_t)s * (b->max_seq + 1), prompt, sizeof(uint32_t) * n_prompt,
                                  cudaMemcpyHostToDevice, st));
    BT_CUDA_CHECK(cudaMemcpyAsync(b->pos + s, &hs[0], sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    BT_CUDA_CHECK(cudaMemcpyAsync(b->cur + s, &hs[1], sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    BT_CUDA_CHECK(cudaMemcpyAsync(b->n_fixed + s, &hs[2], sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    BT_CUDA_CHECK(cudaStreamSynchronize(st));
    uint32_t flag = 0;
    BT_CUDA_CHECK(cudaMemcpy(&flag, b->err, sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag) return fail(BT_ERR_DEVICE_TIMEOUT, "batch prefill: a device wait timed out");
    b->host_pos[s] = n_fill;
    return BT_OK;
}

int bt_batch_steps(bt_batch* b, uint32_t n, void* stream) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    bt_engine* e = b->e;
    for (uint32_t s = 0; s < b->n_seq; ++s) {
        if (b->paged && b->seq_pages[s] == 0) continue;  // an idle slot of the page pool: no work
        if ((uint64_t)b->host_pos[s] + n > b->max_seq)
            return fail(BT_ERR_OUT_OF_RANGE, "bt_batch_steps: a sequence would pass max_seq (or was not prefilled)");
    }
    DeviceGuard guard(e->device);
    cudaStream_t s = stream ? as_stream(stream) : e->stream;
    if (b->paged) {
        // pages for every position the n steps write (all or nothing: count them first)
        size_t need = 0;
        for (uint32_t q = 0; q < b->n_seq; ++q) {
            if (b->seq_pages[q] == 0) continue;
            const uint32_t want = (b->host_pos[q] + n + (1u << b->page_shift) - 1u) >> b->page_shift;
            if (want > b->seq_pages[q]) need += want - b->seq_pages[q];
        }
        if (need > b->free_pages.size())
            return fail(BT_ERR_OUT_OF_MEMORY, "paged KV: the page pool has too few free pages for these steps");
        for (uint32_t q = 0; q < b->n_seq; ++q)
            if (b->seq_pages[q] && (rc = ensure_pages(b, q, b->host_pos[q] + n, s)) != BT_OK) return rc;
    }
    for (uint32_t i = 0; i < n; ++i) {
        if (!b->warmed) {
            // the first step runs eagerly: it sets every kernel's attributes outside capture
            const uint64_t l0 = g_launches.load();
            rc = enqueue_batch(b, s);
            if (rc != BT_OK) return rc;
            b->launches_per_step = g_launches.load() - l0;
            b->warmed = true;
        } else {
            if (!b->graph) {
                cudaStream_t cs = e->stream;
                BT_CUDA_CHECK(cudaStreamSynchronize(s));
                cudaGraph_t g = nullptr;
                BT_CUDA_CHECK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
                const uint64_t l0 = g_launches.load();
                rc = enqueue_batch(b, cs);
                g_launches.store(l0);  // captured, not launched
                const cudaError_t ce = cudaStreamEndCapture(cs, &g);
                if (rc != BT_OK) {
                    if (g) cudaGraphDestroy(g);
                    return rc;
                }
                if (ce != cudaSuccess) return fail(BT_ERR_CUDA, std::string("batch graph capture: ") + cudaGetErrorString(ce));
                const cudaError_t ie = cudaGraphInstantiate(&b->graph, g, 0);
                cudaGraphDestroy(g);
                if (ie != cudaSuccess) {
                    b->graph = nullptr;
                    return fail(BT_ERR_CUDA, std::string("batch graph instantiate: ") + cudaGetErrorString(ie));
                }
            }
            g_launches.fetch_add(b->launches_per_step, std::memory_order_relaxed);
            BT_CUDA_CHECK(cudaGraphLaunch(b->graph, s));
        }
    }
    for (uint32_t q = 0; q < b->n_seq; ++q)
        if (!(b->paged && b->seq_pages[q] == 0)) b->host_pos[q] += n;
    return BT_OK;
}

int bt_batch_read_tokens(bt_batch* b, uint32_t s, uint32_t pos0, uint32_t n, uint32_t* out) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    if (s >= b->n_seq) return fail(BT_ERR_OUT_OF_RANGE, "bt_batch_read_tokens: sequence index out of range");
    if (!out && n) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_read_tokens: null output");
    if ((uint64_t)pos0 + n > (uint64_t)b->max_seq + 1) return fail(BT_ERR_OUT_OF_RANGE, "bt_batch_read_tokens: past max_seq");
    DeviceGuard guard(b->e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(b->e->stream));
    if (n)
        BT_CUDA_CHECK(cudaMemcpy(out, b->tok_hist + (size_t)s * (b->max_seq + 1) + pos0, sizeof(uint32_t) * n,
                                 cudaMemcpyDeviceToHost));
    uint32_t flag = 0;
    BT_CUDA_CHECK(cudaMemcpy(&flag, b->err, sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag) return fail(BT_ERR_DEVICE_TIMEOUT, "batch decode: a device wait timed out");
    return BT_OK;
}

int bt_batch_read_current(bt_batch* b, uint32_t* out) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    if (!out) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_read_current: null output");
    DeviceGuard guard(b->e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(b->e->stream));
    BT_CUDA_CHECK(cudaMemcpy(out, b->cur, sizeof(uint32_t) * b->n_seq, cudaMemcpyDeviceToHost));
    uint32_t flag = 0;
    BT_CUDA_CHECK(cudaMemcpy(&flag, b->err, sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag) return fail(BT_ERR_DEVICE_TIMEOUT, "batch decode: a device wait timed out");
    return BT_OK;
}

int bt_batch_read_logits(bt_batch* b, float* out) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    if (!out) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_read_logits: null output");
    DeviceGuard guard(b->e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(b->e->stream));
    BT_CUDA_CHECK(cudaMemcpy(out, b->logits, sizeof(float) * b->n_seq * b->e->lc.vocab_size, cudaMemcpyDeviceToHost));
    return BT_OK;
}

int bt_batch_step_info(bt_batch* b, uint64_t* bytes) {
    int rc = check_batch(b);
    if (rc != BT_OK) return rc;
    if (!bytes) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_step_info: null output");
    const auto& c = b->e->lc;
    const uint64_t D = c.dim, F = c.hidden_dim, KV = kvd(c), V = c.vocab_size, L = c.num_layers, Q = qd(c);
    const uint64_t params = L * (Q * D * 2 + KV * D * 2 + F * D * 3) + V * D;
    const uint64_t esz = b->dtype == BT_KV_FP16 ? 2 : 4;
    uint64_t kvb = 0;
    for (uint32_t s = 0; s < b->n_seq; ++s)
        kvb += 2 * L * KV * esz * ((uint64_t)std::min(b->host_pos[s], b->max_seq - 1) + 2);  // read c keys, write 1
    *bytes = params + params / 32 * 4 + 4 * D * (2 * L + 1) + 4 * D * b->n_seq + kvb;
    return BT_OK;
}

}  // extern "C"
