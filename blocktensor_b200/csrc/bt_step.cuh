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

#include "bt_attn_mma.cuh"
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
    uint64_t* split_part;     // [G][2][128] tagged partial sums: (tag << 32) | float bits
    float* am_val;            // [G]
    uint32_t* am_idx;
    uint32_t* am_ticket;
    uint64_t* att_part;       // [KVH][GQ][S][hd + 2] tagged (m, l, o) of the splits (S <= kAttnMaxSplits)
    uint32_t* cnt;            // [5 L + 1] phase counters
    uint8_t* dimg[2];         // digit images of GEMV inputs, by phase parity (layout of the shared digit area)
    float* ssp[2];            // per-128-row-tile sums of x^2 of the next RMSNorm input, by phase parity
    uint32_t L, D, KVD, F, hd, KVH, GQ, max_seq, S_att;
    uint32_t DQ;              // query rows (heads of this rank x hd; D without tensor parallelism)
    uint32_t v0;              // first vocab row of this rank's head matrix
    // tensor parallelism over tp_world GPUs (1: none): every rank's exchange buffer, mapped here;
    // [0] o-proj and [1] down partials, [tp_world][D] tagged words each, then the argmax slots
    uint64_t* const* tp_xch;
    uint32_t tp_rank, tp_world;
    float eps, scale;
    uint32_t NS, xstride, tmem_cols, scratch_off;
    // L2 prefetch of upcoming weight stages while the consumers are held up (0: off), and
    // kStepFlag* options
    uint32_t pf_stages, flags;
    // fewest weight tiles a CTA takes in a GEMV phase (0: no floor): a small matrix then runs
    // on U / min_tiles CTAs, its row tiles cut into fewer pieces
    uint32_t min_tiles;
    // per-phase device timestamps (null: off): [P][G][kTraceSlots] of %globaltimer
    uint64_t* trace;
};

constexpr uint32_t kStepFlagEvictFirst = 1;  // ring copies mark their L2 lines evict-first

// Timestamps of the trace (per phase and CTA), in %globaltimer nanoseconds.
enum : uint32_t {
    kTrStart = 0,     // consumers pass the phase's counter wait
    kTrDigits = 1,    // the input's digits are in shared memory
    kTrFirstAcc = 2,  // the finisher receives its first row tile's sums
    kTrEnd = 3,       // the CTA's writes of the phase are done (its counter release)
    kTrCopy0 = 4,     // the producer issues the phase's first ring copy
    kTrCopy1 = 5,     // ... and its last
    kTraceSlots = 8
};

// Stage timeline (a build with BT_STAGE_TRACE defined, for latency analysis):
// after the phase part of the trace, per CTA and ring stage (the first
// kStageTraceMax of the step), kStageSlots timestamps: [0] the producer issues
// the stage's copy, [1] issuer 1 sees it landed, [2] accumulator warp 5 sees
// its MMAs complete, [3] that warp has read the results and releases the slot,
// [4] issuer 1 has issued and committed its MMAs of the stage, [5] accumulator
// warp 5 starts waiting for the stage's MMAs, [6] it has added the stage's sums,
// [7] it has formed the stage's digit sums (before adding them).
constexpr uint32_t kStageTraceMax = 2048;
constexpr uint32_t kStageSlots = 8;

__device__ __forceinline__ void stage_trace_at(const StepArgs& a, uint32_t P, uint32_t stage, uint32_t slot,
                                               float dep = 0.0f) {
#ifdef BT_STAGE_TRACE
    if (a.trace && stage < kStageTraceMax)
        a.trace[(size_t)P * gridDim.x * kTraceSlots + ((size_t)blockIdx.x * kStageTraceMax + stage) * kStageSlots +
                slot] = global_ns_after(dep);
#endif
}

constexpr uint32_t kTpMaxWorld = 8;  // GPUs of one tensor parallel group

enum : uint32_t { kPhQKV = 0, kPhAttn = 1, kPhO = 2, kPhGU = 3, kPhDown = 4, kPhHead = 5 };

__device__ __forceinline__ uint32_t phase_kind(uint32_t p, uint32_t L) { return p == 5 * L ? kPhHead : p % 5; }

__device__ __forceinline__ StepMat phase_mat(const StepArgs& a, uint32_t p) {
    const uint32_t k = phase_kind(p, a.L);
    if (k == kPhHead) return a.head;
    const StepLayer& l = a.layers[p / 5];
    return k == kPhQKV ? l.qkv : k == kPhO ? l.o : k == kPhGU ? l.gu : l.d;
}

// Tile range of CTA c in the stream-K split of matrix m over Gm = min(G, U,
// U / min_tiles) CTAs (every CTA of the split owns at least one tile; CTAs
// c >= Gm own none).
struct Geo {
    uint32_t NB, U, Gm, u0, u1, g_first, g_last, nstages;
};

__device__ __forceinline__ Geo phase_geo(const StepMat& m, uint32_t c, uint32_t G, uint32_t min_tiles) {
    Geo r;
    r.NB = m.K / kTileK;
    r.U = (m.Mp / kTileRows) * r.NB;
    const uint32_t gmax = min_tiles ? max(1u, r.U / min_tiles) : r.U;
    r.Gm = gmax < G ? gmax : G;
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

// Position of a CTA in the stream of its weight stages over the GEMV phases of
// the step (the producer copies them in this order, and prefetches ahead of
// the copies in the same order).
struct StageCursor {
    uint32_t p, j, nst, u0, u1;
    const uint8_t* units;
};

// Moves k to stage 0 of the first phase >= k.p that has stages for CTA c (k.p = P: the end).
__device__ __forceinline__ void cursor_settle(StageCursor& k, const StepArgs& a, uint32_t P, uint32_t c, uint32_t G) {
    for (; k.p < P; ++k.p) {
        if (phase_kind(k.p, a.L) == kPhAttn) continue;
        const StepMat mt = phase_mat(a, k.p);
        const Geo gm = phase_geo(mt, c, G, a.min_tiles);
        if (gm.nstages) {
            k.j = 0;
            k.nst = gm.nstages;
            k.u0 = gm.u0;
            k.u1 = gm.u1;
            k.units = mt.units;
            return;
        }
    }
}

__device__ __forceinline__ void cursor_next(StageCursor& k, const StepArgs& a, uint32_t P, uint32_t c, uint32_t G) {
    if (++k.j < k.nst) return;
    ++k.p;
    cursor_settle(k, a, P, c, G);
}

// Source and size of the stage at k.
__device__ __forceinline__ const uint8_t* cursor_src(const StageCursor& k, uint32_t& bytes) {
    const uint32_t ub = k.u0 + k.j * kStageTiles;
    bytes = min(kStageTiles, k.u1 - ub) * kTileBytes;
    return k.units + (size_t)ub * kTileBytes;
}

__device__ __forceinline__ void trace_at(const StepArgs& a, uint32_t p, uint32_t slot) {
    if (a.trace) a.trace[((size_t)p * gridDim.x + blockIdx.x) * kTraceSlots + slot] = global_ns();
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
// or, when w is null, a plain copy.  With `embed` the source is the embedding
// row of the current token and CTA 0 also writes it to x_out.  Activations are
// read through L2.
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
    // x (embedding row, or activations through L2), p = x * w (or p = x), and the sums the norm needs
    __device__ float4 load(const float* s, uint32_t k, float& ss, float& mx) const {
        const float4 v = embed ? *reinterpret_cast<const float4*>(s + k) : ldcg4(s + k);
        if (!w) {
            amax4(mx, v);
            return v;
        }
        const float4 g = *reinterpret_cast<const float4*>(w + k);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
        if (embed && blockIdx.x == 0) *reinterpret_cast<float4*>(x_out + k) = v;
        const float4 p = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
        amax4(mx, p);
        return p;
    }
};

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

// ---------------------------------------------------------------- digit images
// The B operand of a GEMV phase, block by block: for block b (32 elements) of
// the input, the signed base-256 digits (hi, mid, lo) of v = round(p * 2^e_b),
// p the block's values (times the next RMSNorm weight) and e_b the block's own
// exponent (max |p| * 2^e_b in [2^20, 2^21)), laid out as the shared digit
// area: half c (elements 16c .. 16c+15) of digit row d at c * xstride + 48 b
// + 16 d, then the block scales 2^-e_b (NaN for a block holding an inf or NaN)
// as floats at 2 * xstride.  The RMSNorm factor is a per-vector scalar and is
// applied to the GEMV results.  The warps that finalize a phase's values write
// the next phase's image to global memory; the next phase fetches it with
// bulk copies.

// Digits of block b of the shared-area layout (see warp_digits).
__device__ __forceinline__ void warp_block_digits(uint8_t* img, uint32_t xstride, uint32_t b, float p, uint32_t lane) {
    warp_digits(img + b * 48, xstride, reinterpret_cast<float*>(img + blk_off(xstride)) + b, p, lane);
}

// RMSNorm factor of a phase fed by a digit image: 1/sqrt(sum of the row-tile
// sums of x^2 / K + eps), summed in a fixed order (one warp).
__device__ __forceinline__ float image_inv(const float* ssp, uint32_t K, float eps, uint32_t lane) {
    const uint32_t tiles = (K + kTileRows - 1) / kTileRows;
    float ss = 0.0f;
    for (uint32_t t = lane; t < tiles; t += 32) ss += __ldcg(ssp + t);
    ss = warp_sum(ss);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
}

// ---------------------------------------------------------------- attention phase
// Items (kv head, split) are dealt to the CTAs round robin; the 9 consumer
// warps of a CTA take the item's keys round robin in batches (2 to 8 keys,
// up to 64 bytes of K and V per lane, all loads of a batch in flight at once), with an online softmax per query head (lane i
// holds head dims NV*i .. NV*i+NV-1), merge in shared memory, write the CTA's
// partial (max m, sum l, o = sum e^(s-m) v), and the last CTA of a KV head
// (ticket) merges the splits into attn (:148-184) and, with img (head_dim a
// multiple of 32, so that blocks of 32 never straddle heads), writes the
// o-proj input's digit image.

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

// Splits of a KV head's keys: about one attention item per SM, so models with
// few KV heads (8 for the 70B shape) split each head's long cache many ways.
constexpr uint32_t kAttnMaxSplits = 32;

// Splits this step uses at context c: S_att (about one item per SM), but no
// more than one per 64 keys, so that short caches are not cut into slivers
// whose merge costs more than their keys.  Every CTA computes the same value;
// the split partials of the step are laid out by it (tags tell steps apart).
__device__ __forceinline__ uint32_t attn_splits(const StepArgs& a, uint32_t c) {
    return max(1u, min(a.S_att, (c + 63) / 64));
}

template <int NV, int GQM, typename KVT>
__device__ void attn_phase(const StepArgs& a, uint32_t l, uint8_t* scratch, uint32_t tid, uint8_t* img, uint32_t tag,
                           bool& ok) {
    // grouped-query variants with head_dim 64 or 128 run the key loop on the tensor cores (bt_attn_mma.cuh)
    constexpr bool kAttnMma = GQM > 1 && (NV == 2 || NV == 4);
    // GQM: query heads per KV head held in registers; B: keys per batch and warp
    // (half the batch when several query heads share the keys: their registers)
    constexpr int BW = 16 / RowWords<NV, KVT>::W / (GQM > 1 ? 2 : 1);
    constexpr int B = BW > 8 ? 8 : (BW < 2 ? 2 : BW);
    const uint32_t lane = tid & 31, w = tid >> 5, G = gridDim.x;
    const uint32_t HD = a.hd, GQ = a.GQ;
    const uint32_t pos = a.st->pos;
    const uint32_t c = min(pos + 1, a.max_seq);
    const uint32_t S = attn_splits(a, c);
    const size_t layer_off = (size_t)l * a.KVH * a.max_seq * HD;
    const KVT* kl = reinterpret_cast<const KVT*>(a.kc) + layer_off;
    const KVT* vl = reinterpret_cast<const KVT*>(a.vc) + layer_off;
    float* wm = reinterpret_cast<float*>(scratch);  // [9][GQ][HD + 2]
    const uint32_t pstride = HD + 2;
    const uint64_t tagw = (uint64_t)tag << 32;
    const uint32_t d0 = lane * NV;
    const bool active = d0 < HD;
    for (uint32_t it = blockIdx.x; it < a.KVH * S; it += G) {
        const uint32_t kvh = it / S, sidx = it % S;
        const uint32_t Lk = (c + S - 1) / S;
        const uint32_t t0 = sidx * Lk, t1 = min(c, t0 + Lk);
        const KVT* kb = kl + (size_t)kvh * a.max_seq * HD + d0;
        const KVT* vb = vl + (size_t)kvh * a.max_seq * HD + d0;
        bool on_tensor_cores = false;
        if constexpr (kAttnMma) {
            if (GQ <= 8 && HD == 32 * NV) {  // NV = 2 also serves head_dim < 64: those stay on the CUDA cores
                // grouped heads on the tensor cores: the warps take 16-key tiles round robin; q's
                // fragments in shared memory after the warps' partials
                uint4* qs = reinterpret_cast<uint4*>(scratch + ((size_t)kDigitWarps * GQ * pstride * 4 + 15) / 16 * 16);
                const float* qh = a.q + (size_t)kvh * GQ * HD;
                const size_t head_row0 = (size_t)kvh * a.max_seq;
                auto row = [&](uint32_t t) { return (head_row0 + t) * (32 * NV); };
                if constexpr (sizeof(KVT) == 2) {
                    // fp16 cache: f16 MMAs, q in two fp16 terms scaled per head (exponents after the fragments)
                    using GW = GqaWarp16<32 * NV>;
                    int* qe = reinterpret_cast<int*>(qs + 32 * GW::KSTEPS);
                    GW::head_exponent(qe, qh, GQ, w, lane);
                    digit_sync();
                    GW::stage_q(qs, qh, qe, GQ, tid, kDigitThreads);
                    digit_sync();
                    GW st;
                    st.init(GQ, lane, qs, qe);
                    for (uint32_t k0 = t0 + 16 * w; k0 < t1; k0 += 16 * kDigitWarps) st.tile(kl, vl, k0, t1, a.scale, row);
                    st.store(wm + (size_t)w * GQ * pstride, GQ);
                } else {
                    using GW = GqaWarp<32 * NV, KVT, true>;
                    GW::stage_q(qs, qh, GQ, tid, kDigitThreads);
                    digit_sync();
                    GW st;
                    st.init(nullptr, GQ, lane, qs);
                    for (uint32_t k0 = t0 + 16 * w; k0 < t1; k0 += 16 * kDigitWarps) st.tile(kl, vl, k0, t1, a.scale, row);
                    st.store(wm + (size_t)w * GQ * pstride, GQ);
                }
                on_tensor_cores = true;
            }
        }
        // query heads g0 .. g0 + GQM - 1 of this KV head per pass (K/V re-read from L2 by later passes)
        for (uint32_t g0 = 0; g0 < GQ && !on_tensor_cores; g0 += GQM) {
        float qv[GQM][NV], o[GQM][NV], m[GQM], ls[GQM];
#pragma unroll
        for (int g = 0; g < GQM; ++g) {
            m[g] = -INFINITY;
            ls[g] = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                o[g][i] = 0.0f;
                qv[g][i] = (g0 + g < GQ && active) ? __ldcg(a.q + (size_t)(kvh * GQ + g0 + g) * HD + d0 + i) : 0.0f;
            }
        }
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
                if (g0 + g >= GQ) break;
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
        for (uint32_t g = 0; g0 + g < GQ && g < (uint32_t)GQM; ++g) {
            float* p = wm + ((size_t)w * GQ + g0 + g) * pstride;
            if (lane == 0) { p[0] = m[g]; p[1] = ls[g]; }
#pragma unroll
            for (int i = 0; i < NV; ++i)
                if (active) p[2 + d0 + i] = o[g][i];
        }
        }
        digit_sync();
        // CTA partial of this split (the warps' (m, l, o) merged).  When every CTA holds at most one
        // item (KVH S <= G), all splits publish theirs as (tag, value) words and then all of them
        // merge: split s's CTA takes the 32-element blocks s, s + S, ... of the KV head's query
        // outputs, so no single CTA merges every split.  Otherwise the splits other than 0 publish
        // and move on, and split 0's CTA keeps its own (o in warp 0's row of wm, which only this
        // element's thread reads; m and l in mls) and merges the others.
        const bool spread = a.KVH * S <= G;
        uint64_t* pg = a.att_part + (size_t)kvh * GQ * S * pstride;
        // [GQ][S][3] (m, l, weight) of the splits, then [GQ] totals, after the warps' partials
        float* mls = reinterpret_cast<float*>(scratch + ((size_t)kDigitWarps * GQ * pstride * 4 + 15) / 16 * 16);
        float* ltot = mls + (size_t)GQ * S * 3;
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
            if (sidx != 0 || spread) {
                uint64_t* dst = pg + ((size_t)g * S + sidx) * pstride;
                st_relaxed_u64(dst + 2 + d, tagw | __float_as_uint(acc));
                if (d == 0) {
                    st_relaxed_u64(dst, tagw | __float_as_uint(M));
                    st_relaxed_u64(dst + 1, tagw | __float_as_uint(lsum));
                }
                continue;
            }
            wm[(size_t)g * pstride + 2 + d] = acc;  // warp 0's row: read by this thread only
            if (d == 0) {
                mls[(size_t)g * S * 3] = M;
                mls[(size_t)g * S * 3 + 1] = lsum;
            }
        }
        if (spread) {
            // this split's blocks of the KV head's GQ HD outputs, one warp per block, lane = element;
            // (m, l, o) of every split added in split order with online rescaling (:148-184)
            const uint32_t nblk = (GQ * HD + 31) / 32;
            const uint64_t tw = global_ns();
            for (uint32_t bk = sidx + S * w; bk < nblk; bk += S * kDigitWarps) {
                const uint32_t e = bk * 32 + lane;
                const bool valid = e < GQ * HD;
                const uint32_t g = valid ? e / HD : 0, d = valid ? e % HD : 0;
                const uint64_t* src = pg + (size_t)g * S * pstride;
                float Mr = -INFINITY, lr = 0.0f, ar = 0.0f;
                for (uint32_t s0 = 0; s0 < S; s0 += 4) {
                    uint64_t wmv[4], wl[4], wo[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        wmv[k] = wl[k] = wo[k] = (uint64_t)tag << 32;  // splits past S: l = 0, skipped
                        if (valid && s0 + k < S) {
                            const uint64_t* q = src + (size_t)(s0 + k) * pstride;
                            wmv[k] = ld_relaxed_u64(q);
                            wl[k] = ld_relaxed_u64(q + 1);
                            wo[k] = ld_relaxed_u64(q + 2 + d);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (!(valid && s0 + k < S)) continue;
                        const uint64_t* q = src + (size_t)(s0 + k) * pstride;
                        while (ok && ((uint32_t)(wmv[k] >> 32) != tag || (uint32_t)(wl[k] >> 32) != tag ||
                                      (uint32_t)(wo[k] >> 32) != tag)) {
                            if (global_ns() - tw > kWaitNs) {
                                atomicExch(&a.st->error, 1u);
                                ok = false;
                                break;
                            }
                            wmv[k] = ld_relaxed_u64(q);
                            wl[k] = ld_relaxed_u64(q + 1);
                            wo[k] = ld_relaxed_u64(q + 2 + d);
                        }
                        const float ms = __uint_as_float((uint32_t)wmv[k]), ls_ = __uint_as_float((uint32_t)wl[k]);
                        const float os = __uint_as_float((uint32_t)wo[k]);
                        if (!(ls_ > 0.0f)) continue;
                        if (ms > Mr) {
                            const float r = expf(Mr - ms);  // 0 while nothing is accumulated (Mr = -inf)
                            lr = fmaf(lr, r, ls_);
                            ar = fmaf(ar, r, os);
                            Mr = ms;
                        } else {
                            const float f = expf(ms - Mr);
                            lr = fmaf(ls_, f, lr);
                            ar = fmaf(os, f, ar);
                        }
                    }
                }
                const float o = __fdiv_rn(ar, lr);
                if (valid) a.attn[(size_t)(kvh * GQ) * HD + e] = o;
                // digits of the o-proj input: the warp's 32 elements are one block when HD % 32 == 0
                if (img) warp_block_digits(img, a.xstride, (kvh * GQ * HD) / 32 + bk, o, lane);
            }
        } else if (sidx == 0) {
            digit_sync();
            // every other split's (m, l) of every head, polled in parallel (bounded)
            const uint64_t tw = global_ns();
            for (uint32_t i = tid; i < GQ * (S - 1); i += kDigitThreads) {
                const uint32_t g = i / (S - 1), sp = 1 + i % (S - 1);
                const uint64_t* src = pg + ((size_t)g * S + sp) * pstride;
                uint64_t wmv = ld_relaxed_u64(src), wl = ld_relaxed_u64(src + 1);
                while (ok && ((uint32_t)(wmv >> 32) != tag || (uint32_t)(wl >> 32) != tag)) {
                    if (global_ns() - tw > kWaitNs) {
                        atomicExch(&a.st->error, 1u);
                        ok = false;
                        break;
                    }
                    wmv = ld_relaxed_u64(src);
                    wl = ld_relaxed_u64(src + 1);
                }
                mls[((size_t)g * S + sp) * 3] = __uint_as_float((uint32_t)wmv);
                mls[((size_t)g * S + sp) * 3 + 1] = __uint_as_float((uint32_t)wl);
            }
            digit_sync();
            // per head: the maximum over the splits that saw keys, each split's weight, the total
            for (uint32_t g = tid; g < GQ; g += kDigitThreads) {
                float* mg = mls + (size_t)g * S * 3;
                float Mx = -INFINITY;
                for (uint32_t sp = 0; sp < S; ++sp)
                    if (mg[3 * sp + 1] > 0.0f) Mx = fmaxf(Mx, mg[3 * sp]);
                float L = 0.0f;
                for (uint32_t sp = 0; sp < S; ++sp) {
                    const float w = mg[3 * sp + 1] > 0.0f ? expf(mg[3 * sp] - Mx) : 0.0f;
                    mg[3 * sp + 2] = w;
                    L = fmaf(mg[3 * sp + 1], w, L);
                }
                ltot[g] = L;
            }
            digit_sync();
            // elements: o = (sum over the splits, in split order, of weight * o_split) / total
            for (uint32_t e = tid; e < GQ * HD; e += kDigitThreads) {
                const uint32_t g = e / HD, d = e % HD;
                const float* mg = mls + (size_t)g * S * 3;
                float acc = mg[2] * wm[(size_t)g * pstride + 2 + d];
                for (uint32_t s0 = 1; s0 < S; s0 += 8) {
                    float ov[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint32_t sp = s0 + k;
                        ov[k] = 0.0f;
                        if (sp < S) {
                            const uint64_t* src = pg + ((size_t)g * S + sp) * pstride + 2 + d;
                            uint64_t w = ld_relaxed_u64(src);
                            while (ok && (uint32_t)(w >> 32) != tag) {
                                if (global_ns() - tw > kWaitNs) {
                                    atomicExch(&a.st->error, 1u);
                                    ok = false;
                                    break;
                                }
                                w = ld_relaxed_u64(src);
                            }
                            ov[k] = __uint_as_float((uint32_t)w);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (s0 + k < S) acc = fmaf(mg[3 * (s0 + k) + 2], ov[k], acc);
                }
                const float o = __fdiv_rn(acc, ltot[g]);
                a.attn[(size_t)(kvh * GQ + g) * HD + d] = o;
                // digits of the o-proj input: this warp holds the 32 elements of one block
                if (img) warp_block_digits(img, a.xstride, (kvh * GQ * HD + e) >> 5, o, lane);
            }
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
    const uint32_t c = min(a.st->pos + 1, a.max_seq), S = attn_splits(a, c);
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
    __shared__ __align__(8) uint64_t dbar;  // digit image copies
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
            mbar_init(&mma_done[s], kIssuers);
        }
        for (int r = 0; r < kRedSlots; ++r) {
            mbar_init(&red_full[r], kAccWarps);
            mbar_init(&red_free[r], 1);
        }
        mbar_init(&dbar, 1);
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
            uint32_t s_last = 0, ph_last = 0;  // ring slot and barrier parity of the latest copy
            bool ok = true;
            StageCursor cp{0, 0, 0, 0, 0, nullptr};
            cursor_settle(cp, a, P, c, G);
            // L2 prefetch: pf runs pf_ahead stages in front of the copies (pf == cp when 0)
            StageCursor pf = cp;
            uint32_t pf_ahead = 0;
            const uint64_t pol = policy_evict_first();
            const bool hint = (a.flags & kStepFlagEvictFirst) != 0;
            uint32_t p_traced = 0xFFFFFFFFu;
            while (cp.p < P && ok) {
                if (issued >= NS) {
                    // slot s is free once the accumulators release it.  While it is not, and every
                    // copy issued so far has landed, the consumers are held up (a phase boundary,
                    // attention) and this CTA's HBM stream is idle: bring upcoming stages into L2.
                    const uint64_t t0 = global_ns();
                    while (!mbar_try_wait(&empty[s], ph ^ 1)) {
                        if (pf_ahead < a.pf_stages && pf.p < P && mbar_try_wait(&full[s_last], ph_last)) {
                            while (pf_ahead < a.pf_stages && pf.p < P) {
                                uint32_t nb;
                                const uint8_t* src = cursor_src(pf, nb);
                                bulk_prefetch_l2(src, nb);
                                ++pf_ahead;
                                cursor_next(pf, a, P, c, G);
                            }
                        }
                        if (mbar_try_wait_sleep(&empty[s], ph ^ 1, pf_ahead < a.pf_stages ? 1000u : 100000u)) break;
                        if (global_ns() - t0 > kWaitNs) {
                            atomicExch(err, 1u);
                            ok = false;
                            break;
                        }
                    }
                    if (!ok) break;
                }
                if (a.trace && cp.p != p_traced) {
                    if (p_traced != 0xFFFFFFFFu) trace_at(a, p_traced, kTrCopy1);
                    trace_at(a, cp.p, kTrCopy0);
                    p_traced = cp.p;
                }
                uint32_t nb;
                const uint8_t* src = cursor_src(cp, nb);
                stage_trace_at(a, P, issued, 0);
                mbar_expect_tx(&full[s], nb);
                if (hint)
                    bulk_g2s_hint(ring + (size_t)s * kStageBytes, src, nb, &full[s], pol);
                else
                    bulk_g2s(ring + (size_t)s * kStageBytes, src, nb, &full[s]);
                s_last = s;
                ph_last = ph;
                ++issued;
                cursor_next(cp, a, P, c, G);
                if (pf_ahead > 0) --pf_ahead;
                else pf = cp;
                if (++s == NS) { s = 0; ph ^= 1; }
            }
            if (a.trace && p_traced != 0xFFFFFFFFu) trace_at(a, p_traced, kTrCopy1);
            const uint32_t first = issued > NS ? issued - NS : 0;
            for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, nullptr);
        }
        return;
    }

    // ---------------- consumers (warps 1-9)
    const uint32_t tid = threadIdx.x - 32;
    const uint32_t epoch = a.st->pad[0];
    const uint32_t target = G * (epoch + 1);
    const uint32_t pos = a.st->pos;  // changed only by the head phase's last CTA, at the very end
    const uint32_t launch = a.am_ticket[1];  // step launches of the engine so far (bumped at the very end)
    // Tag of this launch's phase-p partials: ((launch mod (2^22 - 1)) + 1) << 10 | p.  Its launch
    // bits are never 0 (zeroed buffers never match) and consecutive launches never share a tag,
    // also across the wrap of the 32-bit launch count, so a slot still holding the previous
    // launch's words is never taken for this launch's.
    const uint32_t tag_base = ((launch % 0x3FFFFFu) + 1u) << 10;
    bool ok = true;
    // per-role pipeline state, carried across phases
    uint32_t rs = 0, rph = 0;              // ring slot (issuers, accumulators)
    uint32_t rcount = 0;                   // stages passed through the ring so far
    uint32_t qs = 0, qph = 0, qn = 0;      // reduction slot (accumulators, finisher) and slots used
    uint32_t dph = 0;                      // digit-image barrier phase
    StreamState est{-INFINITY, 0xFFFFFFFFu};
    for (uint32_t p = 0; p < P; ++p) {
        const uint32_t kind = phase_kind(p, a.L);
        const uint32_t l = p / 5;
        const StepMat mt = phase_mat(a, p);
        if (p > 0) {
            if (tid == 0) wait_count(a.cnt + (p - 1), target, err);  // acquire
            digit_sync();
        }
        if (tid == 0) trace_at(a, p, kTrStart);
        if (kind == kPhQKV && tid == 32 * 8) prefetch_attn_rows<KVT>(a, l);  // the finisher warp, before its first group
        uint8_t* img_next = a.dimg[(p + 1) & 1];
        float* ssp_next = a.ssp[(p + 1) & 1];
        if (kind == kPhAttn) {
            attn_phase<NV, GQM, KVT>(a, l, xb, tid, a.hd % 32 == 0 ? img_next : nullptr, tag_base | p, ok);
            // the CTA's writes are ordered before the release by the barrier that ends the item
            if (tid == 0) {
                trace_at(a, p, kTrEnd);
                red_add_release_gpu(a.cnt + p, 1u);
            }
            continue;
        }
        const Geo gm = phase_geo(mt, c, G, a.min_tiles);
        const uint32_t NB = mt.K / kTileK;
        const bool norm = kind == kPhQKV || kind == kPhGU || kind == kPhHead;
        // the input's digits: a bulk copy of the image the previous phase wrote, or built here
        const bool from_img = (kind == kPhQKV && l > 0) || kind == kPhGU || kind == kPhDown || kind == kPhHead ||
                              (kind == kPhO && a.hd % 32 == 0);
        float inv = 1.0f;
        if (from_img) {
            if (tid == 0) {
                const uint8_t* src = a.dimg[p & 1];
                const uint32_t hb = NB * 48 + 128, bb = (NB * 4 + 15) & ~15u;
                fence_proxy_async_global();  // the image was written by generic stores of other SMs
                mbar_expect_tx(&dbar, 2 * hb + bb);
                bulk_g2s(xb, src, hb, &dbar);
                bulk_g2s(xb + a.xstride, src + a.xstride, hb, &dbar);
                bulk_g2s(xb + blk_off(a.xstride), src + blk_off(a.xstride), bb, &dbar);
            }
            if (ok) ok = mbar_wait(&dbar, dph, err);
            dph ^= 1;
        } else {
            MProStep pro{kind == kPhO ? a.attn : a.x, nullptr, a.eps, nullptr, a.st, a.x};
            if (kind == kPhQKV) {
                pro.w = a.layers[l].attn_norm;
                pro.embed = a.embed;  // layer 0
            }
            inv = block_digits(pro, mt.K, xb, a.xstride, redd, tid);  // the image an input no finisher writes
        }
        if (tid == 0) trace_at(a, p, kTrDigits);
        const float* blk = reinterpret_cast<const float*>(xb + blk_off(a.xstride));

        if (warp < kAccWarp0) {
            // ---------------- MMA issue
            const uint32_t t = warp - kMmaWarp0;
            if (lane == 0) {
                uint32_t b = (gm.u0 + t) % NB;
                const uint64_t a0 = umma_desc(smem_u32(ring + t * kTileBytes), 128, 256);
                const uint64_t b0 = umma_desc(smem_u32(xb), a.xstride, 128);
                const uint32_t d0 = tmem + t * kTileCols;
                uint32_t s = rs, ph = rph;
                for (uint32_t j = 0; j < gm.nstages; ++j) {
                    if (ok) ok = mbar_wait(&full[s], ph, err);
                    if (t == 0) stage_trace_at(a, P, rcount + j, 1);
                    tcgen05_fence_after();
                    if (ok) issue_stage(t, min(kStageTiles, gm.u1 - (gm.u0 + j * kStageTiles)), s, b, NB, a0, b0, d0);
                    umma_commit(&mma_done[s]);
                    if (t == 0) stage_trace_at(a, P, rcount + j, 4);
                    if (++s == NS) { s = 0; ph ^= 1; }
                    b += kStageTiles;
                    while (b >= NB) b -= NB;
                }
            }
            // every issuer lane tracks the ring position
            for (uint32_t j = 0; j < gm.nstages; ++j)
                if (++rs == NS) { rs = 0; rph ^= 1; }
            rcount += gm.nstages;
            __syncwarp();
            continue;
        }

        if (warp == kFinWarp) {
            // ---------------- finisher
            if (norm && from_img) inv = image_inv(a.ssp[p & 1], mt.K, a.eps, lane);
            const bool resid = kind == kPhO || kind == kPhDown;
            // the next RMSNorm's weight, for the digits of the next phase's input (residual phases)
            const float* wnext = kind == kPhO ? a.layers[l].ffn_norm
                                 : kind == kPhDown ? (l + 1 < a.L ? a.layers[l + 1].attn_norm : a.out_norm)
                                                   : nullptr;
            const uint32_t NBn = kind == kPhGU ? a.F / kTileK : a.D / kTileK;  // blocks of the next input
            const uint32_t tag = tag_base | p;
            const uint32_t half = a.hd >> 1;
            KVT* kl = reinterpret_cast<KVT*>(a.kc) + (size_t)l * a.KVH * a.max_seq * a.hd;
            KVT* vl = reinterpret_cast<KVT*>(a.vc) + (size_t)l * a.KVH * a.max_seq * a.hd;
            for (uint32_t g = gm.g_first; g <= gm.g_last; ++g) {
                const uint32_t row0 = g * kTileRows;
                // epilogue inputs that do not depend on this phase, loaded before the merge wait
                float xv[4], wv[4];
                float2 cs[2];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t r = row0 + lane + 32 * i;
                    xv[i] = (resid && r < mt.M) ? __ldcg(a.x + r) : 0.0f;
                    wv[i] = (resid && r < mt.M) ? wnext[r] : 0.0f;
                }
                if (kind == kPhQKV) {
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const uint32_t r = row0 + 2 * (lane + 32 * i);
                        const uint32_t local = r < a.DQ ? r : r - a.DQ;
                        cs[i] = (r < a.DQ + a.KVD && pos < a.max_seq) ? a.rope[(size_t)pos * half + ((local % a.hd) >> 1)]
                                                                     : make_float2(1.0f, 0.0f);
                    }
                }
                if (ok) ok = mbar_wait(&red_full[qs], qph, err);
                if (g == gm.g_first && lane == 0) trace_at(a, p, kTrFirstAcc);
                float v[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = red[qs][lane + 32 * i] * inv;
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_free[qs]);
                if (++qs == kRedSlots) { qs = 0; qph ^= 1; }
                const uint32_t c_lo = split_cta((uint64_t)g * gm.NB, gm.U, gm.Gm);
                const uint32_t c_hi = split_cta((uint64_t)(g + 1) * gm.NB - 1, gm.U, gm.Gm);
                if (c_lo != c_hi) {
                    if (c != c_lo) {
                        // publish this piece for CTA c_lo (value and tag in one 64-bit word) and move on
                        uint64_t* part = a.split_part + ((size_t)c * 2 + (g == gm.g_first ? 0 : 1)) * kTileRows;
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            st_relaxed_u64(part + lane + 32 * i, ((uint64_t)tag << 32) | __float_as_uint(v[i]));
                        continue;
                    }
                    // CTA c_lo finishes the row tile (its own piece is its range's last): add the other
                    // pieces in CTA order once their tags say they are this phase's
                    for (uint32_t cb = c_lo + 1; cb <= c_hi && ok; cb += 4) {
                        uint64_t pv[4][4];
                        const uint64_t t0 = global_ns();
                        while (true) {
                            bool have = true;
#pragma unroll
                            for (uint32_t u = 0; u < 4; ++u) {
                                const uint32_t cc = cb + u;
                                if (cc > c_hi) break;
                                const uint32_t first_cc = (uint32_t)(((uint64_t)gm.U * cc) / gm.Gm) / gm.NB;
                                const uint64_t* pc = a.split_part + ((size_t)cc * 2 + (g == first_cc ? 0 : 1)) * kTileRows;
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    pv[u][i] = ld_relaxed_u64(pc + lane + 32 * i);
                                    have = have && (uint32_t)(pv[u][i] >> 32) == tag;
                                }
                            }
                            if (__all_sync(0xffffffffu, have)) break;
                            if (global_ns() - t0 > kWaitNs) {
                                if (lane == 0) atomicExch(err, 1u);
                                ok = false;
                                break;
                            }
                        }
#pragma unroll
                        for (uint32_t u = 0; u < 4; ++u) {
                            if (cb + u > c_hi) break;
#pragma unroll
                            for (int i = 0; i < 4; ++i) v[i] += __uint_as_float((uint32_t)pv[u][i]);
                        }
                    }
                }
                if (resid && a.tp_world > 1 && ok) {
                    // tensor parallelism: y is this rank's partial over its input columns.  Send it to
                    // every rank, then add all ranks' partials in rank order (the same sum on every rank,
                    // so the replicated x stays identical)
                    const uint32_t W = a.tp_world, region = kind == kPhO ? 0 : 1;
                    const uint64_t tagw = (uint64_t)tag << 32;
                    for (uint32_t q = 0; q < W; ++q) {
                        uint64_t* dst = a.tp_xch[q] + ((size_t)region * W + a.tp_rank) * a.D + row0;
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            if (row0 + lane + 32 * i < mt.M) st_relaxed_sys_u64(dst + lane + 32 * i, tagw | __float_as_uint(v[i]));
                    }
                    const uint64_t* own = a.tp_xch[a.tp_rank] + (size_t)region * W * a.D + row0;
                    float y[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    const uint64_t t0 = global_ns();
                    for (uint32_t qb = 0; qb < W && ok;) {
                        // 4 ranks' words in flight; a poll that finds one missing reads the group again
                        float ys[4] = {y[0], y[1], y[2], y[3]};
                        bool have = true;
#pragma unroll
                        for (uint32_t u = 0; u < 4; ++u) {
                            const uint32_t q = qb + u;
                            if (q >= W) break;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t r = row0 + lane + 32 * i;
                                if (r >= mt.M) continue;
                                const uint64_t w = ld_relaxed_sys_u64(own + (size_t)q * a.D + lane + 32 * i);
                                have = have && (uint32_t)(w >> 32) == tag;
                                ys[i] += __uint_as_float((uint32_t)w);
                            }
                        }
                        if (__all_sync(0xffffffffu, have)) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) y[i] = ys[i];
                            qb += 4;
                        } else if (global_ns() - t0 > kWaitNs) {
                            if (lane == 0) atomicExch(err, 1u);
                            ok = false;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) v[i] = y[i];
                }
                if (resid) {
                    // x += y (transformer_engine.cpp:191-195, 222-225), optional per-layer tap, then the
                    // next phase's digits of x * w_next and this tile's sum of x^2
                    float* tap = (kind == kPhDown && a.taps) ? a.taps + (size_t)l * a.D : nullptr;
                    float ss = 0.0f;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t r = row0 + lane + 32 * i;
                        float xn = 0.0f;
                        if (r < mt.M) {
                            xn = __fadd_rn(xv[i], v[i]);
                            a.x[r] = xn;
                            if (tap) tap[r] = xn;
                            ss = fmaf(xn, xn, ss);
                        }
                        if (4 * g + i < NBn) warp_block_digits(img_next, a.xstride, 4 * g + i, xn * wv[i], lane);
                    }
                    ss = warp_sum(ss);
                    if (lane == 0) ssp_next[g] = ss;
                } else if (kind == kPhGU) {
                    // act = silu(gate) * up (cpu_ref.hpp:74-79, transformer_engine.cpp:212-215): rows (2j, 2j+1)
#pragma unroll
                    for (int i = 0; i < 4; ++i) fin[lane + 32 * i] = v[i];
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const uint32_t pp = lane + 32 * i;
                        const float gt = fin[2 * pp], up = fin[2 * pp + 1];
                        float act = 0.0f;
                        if (row0 + 2 * pp + 1 < mt.M) {
                            act = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
                            a.act[(row0 >> 1) + pp] = act;
                        }
                        if (2 * g + i < NBn) warp_block_digits(img_next, a.xstride, 2 * g + i, act, lane);
                    }
                } else if (kind == kPhQKV) {
                    // RoPE on (i, i + hd/2) pairs, q and the K/V append at pos (:117-146)
#pragma unroll
                    for (int i = 0; i < 4; ++i) fin[lane + 32 * i] = v[i];
                    __syncwarp();
                    if (pos < a.max_seq) {
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            const uint32_t pp = lane + 32 * i;
                            const uint32_t r = row0 + 2 * pp;
                            if (r >= mt.M) continue;
                            const float x0 = fin[2 * pp], x1 = fin[2 * pp + 1];
                            if (r < a.DQ + a.KVD) {
                                const bool isq = r < a.DQ;
                                const uint32_t local = isq ? r : r - a.DQ;
                                const uint32_t h = local / a.hd, j = (local % a.hd) >> 1;
                                const float o1 = __fsub_rn(__fmul_rn(x0, cs[i].x), __fmul_rn(x1, cs[i].y));
                                const float o2 = __fadd_rn(__fmul_rn(x0, cs[i].y), __fmul_rn(x1, cs[i].x));
                                if (isq) {
                                    a.q[h * a.hd + j] = o1;
                                    a.q[h * a.hd + j + half] = o2;
                                } else {
                                    KVT* dst = kl + ((size_t)h * a.max_seq + pos) * a.hd;
                                    dst[j] = KVConv<KVT>::from_f(o1);
                                    dst[j + half] = KVConv<KVT>::from_f(o2);
                                }
                            } else {
                                const uint32_t local = r - a.DQ - a.KVD;
                                const uint32_t h = local / a.hd, d = local % a.hd;
                                KVT* dst = vl + ((size_t)h * a.max_seq + pos) * a.hd;
                                dst[d] = KVConv<KVT>::from_f(x0);
                                dst[d + 1] = KVConv<KVT>::from_f(x1);
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) fin[lane + 32 * i] = v[i];
                    __syncwarp();
                    EpiLogits lg{a.logits, a.am_val, a.am_idx, a.am_ticket, a.st, a.tok_hist, a.max_seq};
                    SEpiLogits{lg}.tile(est, row0, kTileRows, mt.M, lane, [&](uint32_t t) { return fin[t]; });
                }
                __syncwarp();
            }
            if (lane == 0) trace_at(a, p, kTrEnd);
            if (kind == kPhHead) {
                EpiLogits lg{a.logits, a.am_val, a.am_idx, a.am_ticket, a.st, a.tok_hist, a.max_seq, true};
                lg.v0 = a.v0;
                lg.tp_rank = a.tp_rank;
                lg.tp_world = a.tp_world;
                lg.tag = tag;
                lg.xch = a.tp_xch;
                lg.xch_off = 2 * (size_t)a.tp_world * a.D;
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
#ifdef BT_STAGE_TRACE
            auto st_hook = [&](uint32_t j, uint32_t slot, float dep = 0.0f) {
                if (warp == kAccWarp0 && lane == 0) stage_trace_at(a, P, rcount + j, slot, dep);
            };
#else
            auto st_hook = [](uint32_t, uint32_t, float = 0.0f) {};
#endif
            acc_stages(gm.u0, gm.u1, NB, gm.nstages, ring, NS, taddr, row, blk, mma_done, empty, rs, rph, ok, err, acc,
                       cur_g, flush, st_hook);
            rcount += gm.nstages;
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
