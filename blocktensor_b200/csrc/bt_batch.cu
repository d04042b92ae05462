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
#include "bt_common.cuh"
#include "bt_gemm.cuh"
#include "bt_step.cuh"
#include "bt_engine_impl.h"
#include "bt_internal.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

using namespace bt;

struct bt_batch {
    bt_engine* e = nullptr;
    uint32_t n_seq = 0, max_seq = 0;
    int dtype = BT_KV_FP32;
    std::vector<void*> allocs;
    void* k = nullptr;           // [n_seq][L][KVH][max_seq][hd]
    void* v = nullptr;
    size_t seq_stride = 0;       // elements between two sequences' caches
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
struct BatchAttnArgs {
    const float* q;          // [B][DQ]
    const void* kc;          // this layer's cache of sequence 0
    const void* vc;
    size_t seq_stride;       // elements between sequences
    const uint32_t* pos;     // [B]
    float* part;             // [B][KVH][S][GQ][hd + 2]
    uint32_t S, kps, KVH, GQ, hd, max_seq;
    float scale;
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
    const KVT* kb = static_cast<const KVT*>(a.kc) + (size_t)s * a.seq_stride + (size_t)kvh * a.max_seq * HD;
    const KVT* vb = static_cast<const KVT*>(a.vc) + (size_t)s * a.seq_stride + (size_t)kvh * a.max_seq * HD;
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
                    kr[j].load(kb + (size_t)t * HD + d0);
                    vr[j].load(vb + (size_t)t * HD + d0);
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
    // the CTA's partial of this split: the 8 warps' (m, l, o) merged
    for (uint32_t e = threadIdx.x; e < GQ * HD; e += blockDim.x) {
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

// attn[s][h hd + d] from the splits of (s, kv head, query head), in split order with
// online rescaling.  One warp per (sequence, query head).
__global__ void batch_attn_merge_kernel(const float* __restrict__ part, float* __restrict__ attn, uint32_t B,
                                        uint32_t KVH, uint32_t GQ, uint32_t S, uint32_t hd) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t item = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const uint32_t H = KVH * GQ;
    if (item >= B * H) return;
    const uint32_t s = item / H, h = item % H, kvh = h / GQ, g = h % GQ;
    const uint32_t pstride = hd + 2;
    for (uint32_t d = lane; d < hd; d += 32) {
        float Mr = -INFINITY, lr = 0.0f, ar = 0.0f;
        for (uint32_t sp = 0; sp < S; ++sp) {
            const float* p = part + ((((size_t)s * KVH + kvh) * S + sp) * GQ + g) * pstride;
            const float ms = p[0], ls = p[1], os = p[2 + d];
            if (!(ls > 0.0f)) continue;
            if (ms > Mr) {
                const float r = expf(Mr - ms);
                lr = fmaf(lr, r, ls);
                ar = fmaf(ar, r, os);
                Mr = ms;
            } else {
                const float f = expf(ms - Mr);
                lr = fmaf(ls, f, lr);
                ar = fmaf(os, f, ar);
            }
        }
        attn[(size_t)s * H * hd + (size_t)h * hd + d] = __fdiv_rn(ar, lr);
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
    g_launches.fetch_add(1, std::memory_order_relaxed);
    kern<<<dim3(a.S, a.KVH, B), 256, smem, st>>>(a);
    return cudaGetLastError();
}

template <typename KVT>
cudaError_t launch_batch_attn(const BatchAttnArgs& a, uint32_t B, cudaStream_t st) {
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
    BT_CUDA_CHECK(launch_token_image(e->embed, b->cur, e->layers[0].attn_norm, B, D, b->img[0], b->ss, b->x, s));
    const size_t kv_layer = (size_t)c.num_kv_heads * b->max_seq * hd;
    for (uint32_t l = 0; l < L; ++l) {
        const LayerDev& Ld = e->layers[l];
        KVT* kl = static_cast<KVT*>(b->k) + l * kv_layer;
        KVT* vl = static_cast<KVT*>(b->v) + l * kv_layer;
        {
            GEpiQKV<KVT> epi{b->q, kl, vl, b->seq_stride, b->rope, GemmTok{B, b->pos, b->seq_idx}, Q, KV, hd, b->max_seq};
            BT_CUDA_CHECK(launch_gemm_digits(UnitW{Ld.qkv, QKV, unit_rows(QKV), D},
                                             GemmIn{b->img[0], b->ss, c.rms_norm_eps, B}, epi, err, nsm, s));
        }
        BatchAttnArgs aa{b->q, kl, vl, b->seq_stride, b->pos, b->att_part, b->S, b->kps, c.num_kv_heads, GQ, hd,
                         b->max_seq, 1.0f / std::sqrt((float)hd)};
        BT_CUDA_CHECK(launch_batch_attn<KVT>(aa, B, s));
        {
            const uint32_t items = B * c.num_heads;
            g_launches.fetch_add(1, std::memory_order_relaxed);
            batch_attn_merge_kernel<<<(items + 7) / 8, 256, 0, s>>>(b->att_part, b->attn, B, c.num_kv_heads, GQ, b->S,
                                                                   hd);
            BT_CUDA_CHECK(cudaGetLastError());
        }
        BT_CUDA_CHECK(launch_token_image(b->attn, nullptr, nullptr, B, Q, b->img[1], nullptr, nullptr, s));
        BT_CUDA_CHECK(launch_gemm_digits(UnitW{Ld.o, D, unit_rows(D), Q}, GemmIn{b->img[1], nullptr, 0.0f, B},
                                         GEpiResidual{b->x, Ld.ffn_norm, b->img[0], b->ss, nullptr, D}, err, nsm, s));
        BT_CUDA_CHECK(launch_gemm_digits(UnitW{Ld.gu, 2 * F, unit_rows(2 * F), D},
                                         GemmIn{b->img[0], b->ss, c.rms_norm_eps, B},
                                         GEpiSwiGLU{b->act, b->img[1], F}, err, nsm, s));
        const float* wn = l + 1 < L ? e->layers[l + 1].attn_norm : e->out_norm;
        BT_CUDA_CHECK(launch_gemm_digits(UnitW{Ld.d, D, unit_rows(D), F}, GemmIn{b->img[1], nullptr, 0.0f, B},
                                         GEpiResidual{b->x, wn, b->img[0], b->ss, nullptr, D}, err, nsm, s));
    }
    const uint32_t nob = unit_rows(V) / 32;
    BT_CUDA_CHECK(launch_gemm_digits(UnitW{e->head, V, unit_rows(V), D}, GemmIn{b->img[0], b->ss, c.rms_norm_eps, B},
                                     GEpiLogits{b->logits, b->am_val, b->am_idx, V, nob}, err, nsm, s));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    batch_finish_kernel<<<(B + 7) / 8, 256, 0, s>>>(b->am_val, b->am_idx, nob, B, b->max_seq, b->pos, b->cur,
                                                    b->n_fixed, b->last_am, b->tok_hist);
    BT_CUDA_CHECK(cudaGetLastError());
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

int bt_batch_create(bt_engine* e, uint32_t n_seq, uint32_t max_seq, int kv_dtype, bt_batch** out) {
    if (!e || !out) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: null argument");
    *out = nullptr;
    if (n_seq == 0 || max_seq == 0) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: n_seq and max_seq must be > 0");
    if (kv_dtype != BT_KV_FP32 && kv_dtype != BT_KV_FP16) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: bad kv dtype");
    if (e->tp_world > 1) return fail(BT_ERR_INVALID_ARGUMENT, "bt_batch_create: not available under tensor parallelism");
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
    b->seq_stride = (size_t)c.num_layers * c.num_kv_heads * max_seq * hd;
    const size_t n = b->seq_stride * n_seq;
    uint8_t *kb = nullptr, *vb = nullptr;
    int rc;
    if ((rc = dev_alloc(b->allocs, &kb, n * esz, "batch K cache"))) return cleanup(rc);
    if ((rc = dev_alloc(b->allocs, &vb, n * esz, "batch V cache"))) return cleanup(rc);
    b->k = kb;
    b->v = vb;
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
    // attention splits of at most 256 keys (per sequence, KV head)
    b->kps = 256;
    b->S = (max_seq + b->kps - 1) / b->kps;
    if ((rc = dev_alloc(b->allocs, &b->att_part, (size_t)n_seq * c.num_kv_heads * b->S * GQ * (hd + 2), "splits")))
        return cleanup(rc);
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
    const CacheRef cr{static_cast<uint8_t*>(b->k) + (size_t)s * b->seq_stride * esz,
                      static_cast<uint8_t*>(b->v) + (size_t)s * b->seq_stride * esz, b->rope, b->max_seq, b->err};
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
    for (uint32_t s = 0; s < b->n_seq; ++s)
        if ((uint64_t)b->host_pos[s] + n > b->max_seq)
            return fail(BT_ERR_OUT_OF_RANGE, "bt_batch_steps: a sequence would pass max_seq (or was not prefilled)");
    DeviceGuard guard(e->device);
    cudaStream_t s = stream ? as_stream(stream) : e->stream;
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
    for (uint32_t q = 0; q < b->n_seq; ++q) b->host_pos[q] += n;
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
