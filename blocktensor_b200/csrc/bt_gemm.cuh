// bt_gemm.cuh -- int8-weight GEMM over many tokens on the 5th-generation
// tensor cores: prompt prefill and batched decode.
//
// Y[t][m] = sum_b scale[m][b] * sum_{i<32} q[m][32b+i] * x[t][32b+i] for T
// token rows x[t], the reference's per-row arithmetic
// (quantization/quant_types.cpp:101-121): the block dot product of the exact
// int8 weights with x, times the block's scale, summed over the blocks.
//
// Formulation.  Every 32-element block of every token is scaled by its own
// power of two (max |x| 2^e in [2^14, 2^15)) and written as two fp16 terms,
// x 2^e = hi + lo (hi the nearest fp16, lo the next 11 bits), so the pair
// carries 22 significant bits of each element.  The int8 weights are exact in
// fp16.  One block of a weight row tile is then two K-steps of
// tcgen05.mma kind::f16 (M = 128 rows, N = 64 tokens, K = 16) for each term,
// four MMAs accumulating in fp32 in one tensor-memory slot: the slot holds
// sum_i q_i x_i 2^e for every (row, token) -- exact products, fp32 sums -- and
// the reader warps add scale[m][b] * 2^-e[t][b] * slot into their
// accumulators (two operations per row, token and block).  The weight scale
// varies per (row, block), so the blocks are read out one by one.
//
// Layouts.  Weights: the 4608-byte tiles of bt_gemv_mma.cuh (128 rows x one
// 32-column block of int8 in the K-major no-swizzle canonical layout, then 128
// fp32 scales); two converter warps rewrite each tile as fp16 in shared memory
// (8 KB: K-step k's 128 x 16 halves in the same canonical layout at k * 4096).
// Token terms ("token image"): per group of 64 tokens and block b an
// 8448-byte tile: term (hi, lo) at term * 4096, K-step k at + k * 2048, each
// K-step the 64 tokens' 16 halves in the canonical layout (8-token core
// matrices of 16 bytes per token, the two 8-element K halves 128 bytes apart,
// token groups 256 bytes apart), then the 64 block factors 2^-e (NaN for a
// block holding an inf or NaN); tiles ordered [group][b].
//
// Work: a unit is (row tile g, token group tg, K-split ks); CTAs take units
// round robin, consecutive units sharing a row tile.  Warp 0 streams the
// unit's weight tiles and token tiles in stages of 4 blocks (one mbarrier
// ring); warps 1-4 convert the weight tiles to fp16 (a ring of 6 converted
// tiles; converting a 4 KB tile takes one warp ~0.5 us); warps 5-7 issue the
// four MMAs of a block (issuer i takes blocks i, i + 3, ...; one thread spends
// ~0.3 us on a block's four MMAs and two commits) into one of 8
// tensor-memory slots of 64 columns; 8 reader warps 8-15 (4 lane quarters x 2
// token halves of 32) read the slot, accumulate 32 tokens x their 32 rows in
// registers and, after the unit's last block, run the epilogue on them, 16
// tokens at a time (a warp's 32 rows are one 32-element block of the output,
// so the epilogue can write the next GEMM's token image directly).  All waits
// are bounded (2 s).
#pragma once

#include <cuda_fp16.h>

#include "bt_common.cuh"
#include "bt_gemv_mma.cuh"
#include "bt_ptx.cuh"

namespace bt {

constexpr uint32_t kGTok = 64;                            // tokens per group (MMA N)
constexpr uint32_t kGKStep = kGTok * 32;                  // bytes of one K-step of one term (64 tokens x 16 halves)
constexpr uint32_t kGTerm = 2 * kGKStep;                  // bytes of one term (two K-steps)
constexpr uint32_t kGDTile = 2 * kGTerm + kGTok * 4;      // token tile: 8448 bytes
constexpr uint32_t kGA16 = 2 * kTileQBytes;               // a weight tile in fp16: 8192 bytes
constexpr uint32_t kGStageBlocks = 4;
constexpr uint32_t kGStageW = kGStageBlocks * kTileBytes;  // weight part of a stage
constexpr uint32_t kGStageBytes = kGStageW + kGStageBlocks * kGDTile;  // 52224
constexpr uint32_t kGSlots = 8;                           // tensor-memory slots of kGTok columns (all 512)
constexpr uint32_t kGA16Slots = 6;                        // converted weight tiles in flight
constexpr int kGConv0 = 1, kGConvs = 4;                   // converter warps 1-4
constexpr int kGIssuer0 = 5, kGIssuers = 3;               // issuer warps 5-7
constexpr int kGReader0 = 8, kGReaders = 8;               // reader warps 8-15
constexpr int kGThreads = 32 * (kGReader0 + kGReaders);   // 512
constexpr uint32_t kGMaxStages = 3;
constexpr uint32_t kGSmem = kGMaxStages * kGStageBytes + kGA16Slots * kGA16 + 2 * 16 * 64 * 4;  // + SwiGLU exchange

// Instruction descriptor: D f32, A and B f16, both K-major, N = 64, M = 128.
constexpr uint32_t kIdescG = (1u << 4) | (0u << 7) | (0u << 10) | ((kGTok >> 3) << 17) | ((128u >> 4) << 24);

inline __host__ __device__ uint32_t token_groups(uint32_t T) { return (T + kGTok - 1) / kGTok; }
inline __host__ __device__ size_t token_image_bytes(uint32_t T, uint32_t K) {
    return (size_t)token_groups(T) * (K / 32) * kGDTile;
}

// v * 2^e for e in [-149, 149]: two exact power-of-two factors (each within the
// normal range), so the product is exact unless it underflows.
__device__ __forceinline__ float scale_pow2(float v, int e) { return __fmul_rn(__fmul_rn(v, pow2i(e / 2)), pow2i(e - e / 2)); }

// The fp16 terms of block b of token t in a token image of NB blocks per token:
// warp-uniform call, lane i holding element 32 b + i.  The block's max |p| is
// one redux.sync on the bit patterns; an inf or NaN anywhere makes the block
// factor NaN, so it propagates to every output as in fp32 arithmetic.
__device__ __forceinline__ void token_terms(uint8_t* img, uint32_t NB, uint32_t t, uint32_t b, float p, uint32_t lane) {
    uint8_t* tile = img + ((size_t)(t / kGTok) * NB + b) * kGDTile;
    const uint32_t ti = t % kGTok;
    const float am = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(p))));
    const bool finite = isfinite(am);
    int e = 0;
    if (am > 0.0f && finite) {
        int ex;  // am = fr * 2^ex, fr in [0.5, 1)
        if (am >= 1.17549435e-38f)
            ex = ((__float_as_int(am) >> 23) & 255) - 126;
        else
            frexpf(am, &ex);
        e = 15 - ex;  // am * 2^e in [2^14, 2^15)
        if (e > 149) e = 149;
    }
    const float v = finite ? scale_pow2(p, e) : 0.0f;
    const __half h = __float2half_rn(v);
    const __half l = __float2half_rn(__fsub_rn(v, __half2float(h)));
    const uint32_t hb = __half_as_ushort(h), lb = __half_as_ushort(l);
    const uint32_t hn = __shfl_down_sync(0xffffffffu, hb, 1), ln = __shfl_down_sync(0xffffffffu, lb, 1);
    if ((lane & 1) == 0) {
        // element lane of the block: K-step lane / 16, K half (lane % 16) / 8, half lane % 8
        const uint32_t off = (lane >> 4) * kGKStep + ((lane >> 3) & 1) * 128 + (ti >> 3) * 256 + (ti & 7) * 16 +
                             (lane & 7) * 2;
        *reinterpret_cast<uint32_t*>(tile + off) = hb | (hn << 16);
        *reinterpret_cast<uint32_t*>(tile + kGTerm + off) = lb | (ln << 16);
    }
    if (lane == 0)
        reinterpret_cast<float*>(tile + 2 * kGTerm)[ti] = finite ? scale_pow2(1.0f, -e) : __int_as_float(0x7fc00000);
}

// Per-token inputs of the epilogues.
struct GemmTok {
    uint32_t T;              // tokens
    const uint32_t* pos;     // position of token t (RoPE, KV slot)
    const uint32_t* seq;     // sequence (KV cache) of token t; null: all tokens in cache 0
};

// RMSNorm factors of tokens tok0 .. tok0 + nvalid - 1, multiplied into v[i]:
// token_inv for 16 tokens with every token's loads in flight together (the same
// sums in the same order).
__device__ __forceinline__ void scale_by_token_inv(float (&v)[16], const float* ss, uint32_t NB, uint32_t K, float eps,
                                                   uint32_t tok0, uint32_t nvalid, uint32_t lane) {
    float s[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) s[i] = 0.0f;
    for (uint32_t b = lane; b < NB; b += 32) {
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) t[i] = (uint32_t)i < nvalid ? __ldcg(ss + (size_t)(tok0 + i) * NB + b) : 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) s[i] += t[i];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float tot = warp_sum(s[i]);
        if ((uint32_t)i < nvalid) v[i] *= __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
    }
}

// ---------------------------------------------------------------- epilogues
// rows(): called by each reader warp after a unit, lane = row r = row0 + lane
// of its 32-row output block ob (= r / 32), v[i] the final value of token
// tok0 + i (i < 16; tokens >= T are skipped by the caller's `valid` mask).
// ex: 4 KB of shared memory of the warp's token half; bar(): named barrier of
// the 4 warps of that half.

// Y[t][m] (the standalone GEMM).
struct GEpiStore {
    float* y;
    uint32_t M;
    template <class Bar>
    __device__ void rows(uint32_t r, uint32_t, uint32_t tok0, uint32_t nvalid, const float (&v)[16], uint32_t,
                         uint32_t, float*, Bar) const {
        if (r >= M) return;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if ((uint32_t)i < nvalid) y[(size_t)(tok0 + i) * M + r] = v[i];
    }
};

// x[t] += y (transformer_engine.cpp:191-195, 222-225); then the next GEMM's token
// image of x * w_next and the per-block sums of x^2 for its RMSNorm.
struct GEpiResidual {
    float* x;              // [T][D]
    const float* w_next;   // next RMSNorm weight
    uint8_t* img_next;     // token image of the next GEMM (NB = D / 32)
    float* ss_next;        // [T][D / 32]
    float* tap;            // [T][D] copy of x (null: none)
    uint32_t D;
    template <class Bar>
    __device__ void rows(uint32_t r, uint32_t ob, uint32_t tok0, uint32_t nvalid, const float (&v)[16],
                         uint32_t lane, uint32_t, float*, Bar) const {
        const uint32_t NB = D / 32;
        if (ob >= NB) return;  // padding rows of the last row tile (warp-uniform: D is a multiple of 32)
        const float w = w_next[r];
        // the 16 tokens' x first, all loads in flight (the stores below would order them otherwise)
        float xo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) xo[i] = (uint32_t)i < nvalid ? __ldcg(x + (size_t)(tok0 + i) * D + r) : 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            if ((uint32_t)i >= nvalid) break;
            const uint32_t t = tok0 + i;
            float* xp = x + (size_t)t * D + r;
            const float xn = __fadd_rn(xo[i], v[i]);
            *xp = xn;
            if (tap) tap[(size_t)t * D + r] = xn;
            token_terms(img_next, NB, t, ob, xn * w, lane);
            const float ss = warp_sum(xn * xn);
            if (lane == 0) ss_next[(size_t)t * NB + ob] = ss;
        }
    }
};

// (gate, up) row pairs (2j, 2j+1): act[t][j] = silu(gate) * up (cpu_ref.hpp:74-79,
// transformer_engine.cpp:212-215), then the down GEMM's token image of act.  A
// warp holds 16 act values of a token, half a 32-block: the four warps of a
// token half exchange them through shared memory and the warps of quarters 0
// and 2 write the token terms of the row tile's two act blocks.
struct GEpiSwiGLU {
    float* act;            // [T][F]
    uint8_t* img_next;     // token image of the down GEMM (NB = F / 32)
    uint32_t F;
    template <class Bar>
    __device__ void rows(uint32_t r, uint32_t, uint32_t tok0, uint32_t nvalid, const float (&v)[16], uint32_t lane,
                         uint32_t q, float* ex, Bar bar) const {
        // ex: [16 tokens][64 act values of the row tile]
        bar();  // the previous unit's readers of ex are done
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float up = __shfl_down_sync(0xffffffffu, v[i], 1);
            if ((lane & 1) == 0 && (uint32_t)i < nvalid) {
                const float g = v[i];
                const float a = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up);
                const uint32_t j = r >> 1;
                if (j < F) act[(size_t)(tok0 + i) * F + j] = a;
                ex[i * 64 + 16 * q + (lane >> 1)] = a;
            }
        }
        bar();
        if (q == 0 || q == 2) {
            const uint32_t NB = F / 32;
            const uint32_t ob = (r - lane) >> 6;  // act block of this warp pair: 2 g + q / 2
            if (ob < NB) {
#pragma unroll 1
                for (uint32_t i = 0; i < nvalid; ++i)
                    token_terms(img_next, NB, tok0 + i, ob, ex[i * 64 + 32 * (q >> 1) + lane], lane);
            }
        }
    }
};

// q/k/v rows (RoPE pairs (i, i + hd/2) of each head adjacent, as the decode
// layout), RoPE at each token's position and the K/V append (:117-146).
template <typename KVT>
struct GEpiQKV {
    float* q;              // [T][DQ]
    KVT* kc;               // this layer's K cache base (row addresses from map)
    KVT* vc;
    KVMap map;             // contiguous or paged rows; map.max_seq bounds the positions
    const float2* rope;    // [max_seq][hd/2]
    GemmTok tk;
    uint32_t DQ, KVD, hd;
    template <class Bar>
    __device__ void rows(uint32_t r, uint32_t, uint32_t tok0, uint32_t nvalid, const float (&v)[16], uint32_t lane,
                         uint32_t, float*, Bar) const {
        const uint32_t half = hd >> 1;
        const bool isq = r < DQ, isk = !isq && r < DQ + KVD, isv = r >= DQ + KVD && r < DQ + 2 * KVD;
        const uint32_t local = isq ? r : isk ? r - DQ : r - DQ - KVD;
        const uint32_t h = local / hd, j = (local % hd) >> 1;
        // every token's position, RoPE factors and cache row first, all loads in flight (the
        // stores below would order them otherwise)
        uint32_t pos[16];
        float2 cs[16];
        size_t ro[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            pos[i] = (uint32_t)i < nvalid ? tk.pos[tok0 + i] : 0xFFFFFFFFu;
            const bool live = pos[i] < map.max_seq;
            cs[i] = (live && (isq || isk)) ? rope[(size_t)pos[i] * half + j] : make_float2(1.0f, 0.0f);
            const uint32_t seq = (live && tk.seq) ? tk.seq[tok0 + i] : 0u;
            ro[i] = (live && (isk || isv)) ? map.row(seq, h, pos[i]) : 0;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float partner = __shfl_xor_sync(0xffffffffu, v[i], 1);
            if (pos[i] >= map.max_seq) continue;  // also tokens >= nvalid
            const uint32_t t = tok0 + i;
            if (isq || isk) {
                float o;
                uint32_t d;
                if ((lane & 1) == 0) {  // first of the pair: a cos - b sin
                    o = __fsub_rn(__fmul_rn(v[i], cs[i].x), __fmul_rn(partner, cs[i].y));
                    d = j;
                } else {                // second: a sin + b cos
                    o = __fadd_rn(__fmul_rn(partner, cs[i].y), __fmul_rn(v[i], cs[i].x));
                    d = j + half;
                }
                if (isq) q[(size_t)t * DQ + h * hd + d] = o;
                else kc[ro[i] + d] = KVConv<KVT>::from_f(o);
            } else if (isv) {
                vc[ro[i] + local % hd] = KVConv<KVT>::from_f(v[i]);
            }
        }
    }
};

// ---------------------------------------------------------------- kernel

struct GemmIn {
    const uint8_t* img;    // token image of the input, [NTG][NB][kGDTile]
    const float* ss;       // per-block sums of squares [T][NB] of the RMSNorm input (null: no norm)
    float eps;
    uint32_t T;
    // split-K workspace: with more splits than one the units write their partial sums
    // [KS][T][Mp] here and gemm_reduce_kernel sums them and runs the epilogue
    float* part = nullptr;
    size_t part_floats = 0;
    uint32_t KS = 1;       // set by launch_gemm_tokens
};

// Sum of the KS splits' partials of rows r, tokens tok0 .. tok0 + nvalid - 1, in
// split order: F splits at a time, the 16 tokens' loads of all F in flight together.
template <int F = 4>
__device__ __forceinline__ void sum_splits(float (&v)[16], const GemmIn& in, uint32_t Mp, uint32_t r, uint32_t tok0,
                                           uint32_t nvalid) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.0f;
    for (uint32_t ks0 = 0; ks0 < in.KS; ks0 += F) {
        float t[F][16];
#pragma unroll
        for (int k = 0; k < F; ++k) {
            const float* pk = in.part + ((size_t)(ks0 + k) * in.T + tok0) * Mp + r;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                t[k][i] = (ks0 + k < in.KS && (uint32_t)i < nvalid) ? __ldcg(pk + (size_t)i * Mp) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < F; ++k)
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] += t[k][i];
    }
}

// Blocks [b0, b1) of K-split ks of KS.
__device__ __forceinline__ void split_blocks(uint32_t NB, uint32_t ks, uint32_t KS, uint32_t& b0, uint32_t& b1) {
    b0 = (uint32_t)(((uint64_t)NB * ks) / KS);
    b1 = (uint32_t)(((uint64_t)NB * (ks + 1)) / KS);
}

template <class Epi>
__global__ void __launch_bounds__(kGThreads, 1) gemm_tokens_kernel(UnitW W, GemmIn in, Epi epi, uint32_t NS,
                                                                   uint32_t* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kGMaxStages], empty[kGMaxStages];
    __shared__ __align__(8) uint64_t afull[kGA16Slots], afree[kGA16Slots];
    __shared__ __align__(8) uint64_t tfull[kGSlots], tfree[kGSlots];
    __shared__ uint32_t s_tmem;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t NB = W.K / kTileK, NTG = token_groups(in.T), KS = in.KS;
    // a unit: (row tile g, token group tg, K-split ks), consecutive units sharing a row tile
    const uint32_t units = (W.Mp / kTileRows) * NTG * KS;
    uint8_t* ring = smem;
    uint8_t* a16 = smem + (size_t)kGMaxStages * kGStageBytes;
    float* exch = reinterpret_cast<float*>(a16 + (size_t)kGA16Slots * kGA16);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGReaders);
        }
        for (uint32_t s = 0; s < kGA16Slots; ++s) {
            mbar_init(&afull[s], 1);
            mbar_init(&afree[s], 1);
        }
        for (uint32_t s = 0; s < kGSlots; ++s) {
            mbar_init(&tfull[s], 1);
            mbar_init(&tfree[s], kGReaders);
        }
        fence_mbar_init();
    }
    if (warp == kGIssuer0) {
        tmem_alloc(&s_tmem, 512);
        tmem_relinquish();
    }
    tcgen05_fence_before();
    __syncthreads();
    tcgen05_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0) {
        // ---------------- producer
        if (lane == 0) {
            uint32_t s = 0, ph = 0, issued = 0;
            bool ok = true;
            for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const uint32_t ks = u % KS, g = (u / KS) / NTG, tg = (u / KS) % NTG;
                uint32_t bs, be;
                split_blocks(NB, ks, KS, bs, be);
                for (uint32_t b0 = bs; b0 < be; b0 += kGStageBlocks) {
                    if (issued >= NS && !(ok = mbar_wait(&empty[s], ph ^ 1, err))) break;
                    const uint32_t n = min(kGStageBlocks, be - b0);
                    mbar_expect_tx(&full[s], n * (kTileBytes + kGDTile));
                    uint8_t* dst = ring + (size_t)s * kGStageBytes;
                    bulk_g2s(dst, W.units + ((size_t)g * NB + b0) * kTileBytes, n * kTileBytes, &full[s]);
                    bulk_g2s(dst + kGStageW, in.img + ((size_t)tg * NB + b0) * kGDTile, n * kGDTile, &full[s]);
                    ++issued;
                    if (++s == NS) { s = 0; ph ^= 1; }
                }
            }
            const uint32_t first = issued > NS ? issued - NS : 0;
            for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, nullptr);
        }
        return;
    }

    if (warp < kGIssuer0) {
        // ---------------- converters: converter c takes the blocks j with j % 4 == c; each lane
        // turns 8 of the tile's 256 16-byte int8 chunks into fp16 (int8 + 128 as the low byte of
        // 0x6400 = 1024, minus 1152: exact)
        const uint32_t cv = warp - kGConv0;
        bool ok = true;
        uint32_t s = 0, ph = 0, j = 0;
        for (uint32_t u = blockIdx.x; u < units; u += gridDim.x) {
            uint32_t bs, be;
            split_blocks(NB, u % KS, KS, bs, be);
            for (uint32_t b0 = bs; b0 < be; b0 += kGStageBlocks) {
                const uint32_t n = min(kGStageBlocks, be - b0);
                bool waited = false;
                for (uint32_t k = 0; k < n; ++k, ++j) {
                    if ((j % kGConvs) != cv) continue;
                    if (!waited) {
                        if (ok) ok = mbar_wait(&full[s], ph, err);
                        waited = true;
                    }
                    const uint32_t as = j % kGA16Slots, use = j / kGA16Slots;
                    if (use > 0 && ok) ok = mbar_wait(&afree[as], (use - 1) & 1, err);
                    const uint8_t* src = ring + (size_t)s * kGStageBytes + k * kTileBytes;
                    uint8_t* dst = a16 + (size_t)as * kGA16;
                    const __half2 off = __floats2half2_rn(1152.0f, 1152.0f);
#pragma unroll 2
                    for (uint32_t c = lane; c < kTileQBytes / 16; c += 32) {
                        // chunk c: row 8 (c / 16) + c % 8, K half (c / 8) % 2 = the fp16 K-step
                        const uint4 w = *reinterpret_cast<const uint4*>(src + 16 * c);
                        const uint32_t ws[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u,
                                                w.w ^ 0x80808080u};
                        uint32_t hv[8];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t p0 = __byte_perm(ws[i], 0x64646464u, 0x5140);
                            const uint32_t p1 = __byte_perm(ws[i], 0x64646464u, 0x5342);
                            const __half2 h0 = __hsub2(*reinterpret_cast<const __half2*>(&p0), off);
                            const __half2 h1 = __hsub2(*reinterpret_cast<const __half2*>(&p1), off);
                            hv[2 * i] = *reinterpret_cast<const uint32_t*>(&h0);
                            hv[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&h1);
                        }
                        const uint32_t base = ((c >> 3) & 1) * kTileQBytes + (c >> 4) * 256 + (c & 7) * 16;
                        *reinterpret_cast<uint4*>(dst + base) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                        *reinterpret_cast<uint4*>(dst + base + 128) = make_uint4(hv[4], hv[5], hv[6], hv[7]);
                    }
                    fence_proxy_async();  // the generic writes, then the tensor cores' reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&afull[as]);
                }
                if (++s == NS) { s = 0; ph ^= 1; }
            }
        }
        return;
    }

    if (warp < kGReader0) {
        // ---------------- issuers: issuer i takes the blocks j with j % 3 == i
        const uint32_t i = warp - kGIssuer0;
        if (lane == 0) {
            bool ok = true;
            uint32_t s = 0, ph = 0, j = 0;
            for (uint32_t u = blockIdx.x; u < units; u += gridDim.x) {
                uint32_t bs, be;
                split_blocks(NB, u % KS, KS, bs, be);
                for (uint32_t b0 = bs; b0 < be; b0 += kGStageBlocks) {
                    const uint32_t n = min(kGStageBlocks, be - b0);
                    bool waited = false;
                    const uint8_t* stage = ring + (size_t)s * kGStageBytes;
                    for (uint32_t k = 0; k < n; ++k, ++j) {
                        if ((j % kGIssuers) != i) continue;
                        if (!waited) {
                            if (ok) ok = mbar_wait(&full[s], ph, err);  // the token tiles
                            waited = true;
                        }
                        const uint32_t as = j % kGA16Slots, slot = j % kGSlots, tuse = j / kGSlots;
                        if (ok) ok = mbar_wait(&afull[as], (j / kGA16Slots) & 1, err);
                        if (tuse > 0 && ok) ok = mbar_wait(&tfree[slot], (tuse - 1) & 1, err);
                        tcgen05_fence_after();
                        const uint32_t abase = smem_u32(a16 + (size_t)as * kGA16);
                        const uint32_t bbase = smem_u32(stage + kGStageW + k * kGDTile);
#pragma unroll
                        for (uint32_t kk = 0; kk < 2; ++kk)
#pragma unroll
                            for (uint32_t term = 0; term < 2; ++term) {
                                const uint64_t a = umma_desc(abase + kk * kTileQBytes, 128, 256);
                                const uint64_t b = umma_desc(bbase + term * kGTerm + kk * kGKStep, 128, 256);
                                if (ok) umma_f16(tmem + slot * kGTok, a, b, kIdescG, (kk | term) ? 1u : 0u);
                            }
                        umma_commit(&tfull[slot]);  // arrives once the block's MMAs are complete
                        umma_commit(&afree[as]);    // and the converted tile is free again
                    }
                    if (++s == NS) { s = 0; ph ^= 1; }
                }
            }
        }
        __syncwarp();
        // tensor memory is freed after every reader is done with it
        asm volatile("bar.sync 3, %0;" ::"n"(32 * (kGIssuers + kGReaders)) : "memory");
        if (warp == kGIssuer0) {
            tcgen05_fence_after();
            tmem_dealloc(tmem, 512);
        }
        return;
    }

    // ---------------- readers: lane quarter q (TMEM lanes 32 q ..), token half h (tokens 32 h .. 32 h + 31)
    const uint32_t q = warp & 3, h = (warp - kGReader0) >> 2;
    const uint32_t row = 32 * q + lane;
    const uint32_t taddr = tmem + ((32 * q) << 16) + 32 * h;
    float* ex = exch + h * (16 * 64);
    auto bar = [h]() { asm volatile("bar.sync %0, 128;" ::"r"(4 + h) : "memory"); };
    bool ok = true;
    uint32_t s = 0, ph = 0, j = 0;
    for (uint32_t u = blockIdx.x; u < units; u += gridDim.x) {
        const uint32_t ks = u % KS, g = (u / KS) / NTG, tg = (u / KS) % NTG;
        uint32_t bs, be;
        split_blocks(NB, ks, KS, bs, be);
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
        for (uint32_t b0 = bs; b0 < be; b0 += kGStageBlocks) {
            const uint32_t n = min(kGStageBlocks, be - b0);
            const uint8_t* stage = ring + (size_t)s * kGStageBytes;
            // the scales and block factors this warp reads were written by the stage's bulk copies
            if (ok) ok = mbar_wait(&full[s], ph, err);
            for (uint32_t k = 0; k < n; ++k, ++j) {
                const uint32_t slot = j % kGSlots, use = j / kGSlots;
                if (ok) ok = mbar_wait(&tfull[slot], use & 1, err);
                tcgen05_fence_after();
                uint32_t d[32];
                tmem_ld32(taddr + slot * kGTok, d);
                const float sc = *reinterpret_cast<const float*>(stage + k * kTileBytes + kTileQBytes + row * 4);
                const float4* bfp = reinterpret_cast<const float4*>(stage + kGStageW + k * kGDTile + 2 * kGTerm) + 8 * h;
                float f[32];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 v = bfp[i];
                    f[4 * i] = sc * v.x; f[4 * i + 1] = sc * v.y; f[4 * i + 2] = sc * v.z; f[4 * i + 3] = sc * v.w;
                }
                tmem_wait_ld();
                tcgen05_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tfree[slot]);
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[i] = fmaf(f[i], __uint_as_float(d[i]), acc[i]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage's shared memory
            if (++s == NS) { s = 0; ph ^= 1; }
        }
        // ---------------- epilogue of the unit, 16 tokens at a time
        const uint32_t r = g * kTileRows + row;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const uint32_t tok0 = tg * kGTok + 32 * h + 16 * hh;
            const uint32_t nvalid = tok0 < in.T ? min(16u, in.T - tok0) : 0u;
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = acc[16 * hh + i];
            if (KS > 1) {
                // one K-split's partial sums; gemm_reduce_kernel adds the splits and runs the epilogue
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if ((uint32_t)i < nvalid) in.part[((size_t)ks * in.T + tok0 + i) * W.Mp + r] = v[i];
                continue;
            }
            if (in.ss) scale_by_token_inv(v, in.ss, NB, W.K, in.eps, tok0, nvalid, lane);
            epi.rows(r, r >> 5, tok0, nvalid, v, lane, q, ex, bar);
        }
    }
    tcgen05_fence_before();
    asm volatile("bar.sync 3, %0;" ::"n"(32 * (kGIssuers + kGReaders)) : "memory");
}

// The token image of an input that no GEMM epilogue writes: src rows (or the
// embedding rows of `tokens`) times the RMSNorm weight w (null: none), plus the
// per-block sums of squares of the unweighted rows; x_out (non-null) receives
// the rows themselves (the residual stream of layer 0).  One warp per (token, block).
static __global__ void __launch_bounds__(256) token_image_kernel(const float* __restrict__ src,
                                                          const uint32_t* __restrict__ tokens,
                                                          const float* __restrict__ w, uint32_t T, uint32_t K,
                                                          uint8_t* img, float* ss, float* x_out) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t NB = K / 32;
    const uint64_t item = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= (uint64_t)T * NB) return;
    const uint32_t t = (uint32_t)(item / NB), b = (uint32_t)(item % NB);
    const float* row = tokens ? src + (size_t)tokens[t] * K : src + (size_t)t * K;
    const uint32_t k = 32 * b + lane;
    const float x = __ldcg(row + k);
    if (x_out) x_out[(size_t)t * K + k] = x;
    token_terms(img, NB, t, b, w ? x * w[k] : x, lane);
    if (ss) {
        const float s = warp_sum(x * x);
        if (lane == 0) ss[(size_t)t * NB + b] = s;
    }
}

// The K-splits of a GEMM added in split order, the RMSNorm factor applied, and
// the epilogue run as the GEMM's readers run it: one CTA of 4 warps per (row
// tile, token group, 16 tokens), warp q holding rows 32 q .. 32 q + 31.
template <class Epi>
__global__ void __launch_bounds__(128) gemm_reduce_kernel(UnitW W, GemmIn in, Epi epi) {
    __shared__ float ex[16 * 64];
    const uint32_t q = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t NTG = token_groups(in.T), NB = W.K / kTileK;
    constexpr uint32_t kSix = kGTok / 16;  // 16-token pieces of a group
    const uint32_t h = blockIdx.x % kSix, tg = (blockIdx.x / kSix) % NTG, g = (blockIdx.x / kSix) / NTG;
    const uint32_t r = g * kTileRows + 32 * q + lane;
    const uint32_t tok0 = tg * kGTok + 16 * h;
    const uint32_t nvalid = tok0 < in.T ? min(16u, in.T - tok0) : 0u;
    float v[16];
    sum_splits<4>(v, in, W.Mp, r, tok0, nvalid);
    if (in.ss) scale_by_token_inv(v, in.ss, NB, W.K, in.eps, tok0, nvalid, lane);
    auto bar = []() { __syncthreads(); };
    epi.rows(r, r >> 5, tok0, nvalid, v, lane, q, ex, bar);
}

// ---------------------------------------------------------------- host side

inline uint32_t gemm_stages() { return (uint32_t)kGMaxStages; }

// K-splits of a GEMM: as many as keep every unit on an SM of its own (at least
// 8 blocks per split), within the workspace; 1 when there is no workspace.
inline uint32_t gemm_splits(uint32_t Mp, uint32_t K, uint32_t T, uint32_t nsm, size_t part_floats) {
    const uint32_t units = (Mp / kTileRows) * token_groups(T), NB = K / kTileK;
    if (units == 0 || units >= nsm || part_floats == 0) return 1;
    uint32_t ks = nsm / units;  // KS * units <= nsm: no CTA takes two units
    ks = ks < NB / 8 ? ks : NB / 8;
    while (ks > 1 && (size_t)ks * T * Mp > part_floats) --ks;
    return ks < 1 ? 1 : ks;
}

// Size of a split-K workspace that lets every GEMM reach about one unit per SM:
// KS splits of U < nsm units need KS * T * Mp floats with KS * U <= ~2 nsm, and a
// unit covers at most 128 rows x kGTok tokens.
inline size_t gemm_split_floats(uint32_t nsm) { return (size_t)2 * nsm * kTileRows * kGTok; }

template <class Epi>
cudaError_t launch_gemm_tokens(const UnitW& W, const GemmIn& in_, const Epi& epi, uint32_t* err, uint32_t nsm,
                               cudaStream_t s) {
    if (W.K % kTileK || W.Mp % kTileRows || W.K == 0 || W.Mp == 0) return cudaErrorInvalidValue;
    GemmIn in = in_;
    in.KS = gemm_splits(W.Mp, W.K, in.T, nsm, in.part ? in.part_floats : 0);
    const uint32_t units = (W.Mp / kTileRows) * token_groups(in.T) * in.KS;
    if (units == 0) return cudaSuccess;
    auto kern = gemm_tokens_kernel<Epi>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const uint32_t grid = units < nsm ? units : nsm;
    cudaError_t ce = launch_pdl(kern, dim3(grid), dim3(kGThreads), (size_t)kGSmem, s, false, W, in, epi,
                                gemm_stages(), err);
    if (ce != cudaSuccess || in.KS == 1) return ce;
    const uint32_t reduce_ctas = (W.Mp / kTileRows) * token_groups(in.T) * (kGTok / 16);
    return launch_pdl(gemm_reduce_kernel<Epi>, dim3(reduce_ctas), dim3(128), 0, s, false, W, in, epi);
}

}  // namespace bt
