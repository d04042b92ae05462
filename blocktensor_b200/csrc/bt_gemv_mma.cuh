// bt_gemv_mma.cuh -- batch-1 int8 GEMV on the 5th-generation tensor cores.
//
// Arithmetic.  The reference computes y[r] = sum_b scale[r][b] * sum_{i<32}
// q[r][32b+i] * x[32b+i] in fp32 (quantization/quant_types.cpp:101-121).  Here
// every 32-element block b of x is first written in 22-bit fixed point,
// v = round(x * 2^e_b) with the block's own power-of-two exponent e_b
// (max |x| of the block times 2^e_b in [2^20, 2^21)), and v as three signed
// base-256 digits hi/mid/lo.  One tcgen05.mma (kind::i8, M=128, N=8, K=32) per
// 128-row x 32-column tile gives, for every row, the three digit dot products
// sum_i q_i * digit_i exactly as int32 in tensor memory; they are combined in
// fp32 ((256*hi + mid)*256 + lo), multiplied by the weight's block scale and
// by 2^-e_b, and accumulated in fp32 across blocks.  The only rounding besides
// fp32 accumulation is x's quantisation step of 2^-21 relative to the max |x|
// of its own block, so a block of small values next to an outlier block keeps
// its full precision.
//
// Layout (written by the pack kernel): rows in tiles of 128; a matrix is the
// stream of its (row tile, 32-column block) tiles, row-tile-major.  A tile is
// 4608 bytes: the 128x32 int8 block in the UMMA K-major no-swizzle canonical
// layout (core matrix of 8 rows x 16 bytes = 128 contiguous bytes; core
// matrices of the two 16-byte K halves 128 bytes apart, 8-row groups 256
// bytes apart), then the 128 fp32 block scales in row order.
//
// Work split (stream-K).  CTA c of G owns tiles [U c/G, U (c+1)/G): every CTA
// moves the same number of bytes, whatever M.  A row tile cut between several
// CTAs is finished by the one that completes last, adding the CTAs' partial
// sums in CTA order, so results are deterministic.
//
// Warp roles (320 threads): warp 0 produces (cp.async.bulk of 8-tile, 36 KB
// stages into an mbarrier ring; weights never depend on the previous kernel,
// so under programmatic dependent launch the ring fills while the previous
// kernel drains); warps 1-4 issue the MMAs, warp 1+t for tiles t and t+4 of
// every stage (one thread issuing back-to-back tcgen05.mma spends ~230 cycles
// per MMA whatever N up to 64 and however often it commits; four issuers reach
// ~58 cycles per MMA together, eight ~39 -- measured with a probe kernel -- so
// a single issuer could not keep up with HBM); warps 5-8 read the
// digit sums from tensor memory (warp w reads TMEM lanes 32 (w%4) .. +31, all
// eight tiles of a stage with one load) and accumulate; warp 9 finishes each
// row tile (cross-CTA merge, epilogue).  Stages are 36 KB because every stage
// costs ~0.4 us of mbarrier hand-offs between the roles whatever its size.
// Warps 1-9 build the digits first.  Warp 1 owns the tensor memory.  No
// thread loads weights into registers: the tensor cores read them from the
// ring.  All waits are bounded (2 s); an expired wait sets *err and the CTA
// still finishes and frees its tensor memory.
#pragma once

#include "bt_common.cuh"
#include "bt_gemv.cuh"
#include "bt_ptx.cuh"

namespace bt {

constexpr uint32_t kTileRows = 128;
constexpr uint32_t kTileK = 32;
constexpr uint32_t kTileQBytes = 4096;   // 128 x 32 int8
constexpr uint32_t kTileBytes = 4608;    // + 128 fp32 scales
constexpr uint32_t kStageTiles = 8;      // 36 KB stages
constexpr uint32_t kStageBytes = kStageTiles * kTileBytes;
constexpr uint32_t kTileCols = 8;        // TMEM columns per tile (N = 8)
constexpr int kMmaThreads = 320;
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp0 = 1;             // MMA issuers 1..4 (warp 1 owns the tensor memory)
constexpr uint32_t kIssuers = 4;
constexpr int kAccWarp0 = 5;             // accumulator warps 5..8
constexpr int kAccWarps = 4;
constexpr int kFinWarp = 9;
constexpr int kDigitWarps = 9;           // warps 1..9
constexpr int kDigitThreads = 32 * kDigitWarps;
constexpr int kRedSlots = 4;
constexpr uint32_t kMmaMaxRing = 8;      // stages (8 x 64 TMEM columns = 512)

// Instruction descriptor: D s32, A and B s8, both K-major, N = 8, M = 128.
constexpr uint32_t kIdescS8 = (2u << 4) | (1u << 7) | (1u << 10) | ((8u >> 3) << 17) | ((128u >> 4) << 24);

inline __host__ __device__ uint32_t unit_rows(uint32_t M) { return (M + kTileRows - 1) / kTileRows * kTileRows; }

// A matrix in the tile layout.
struct UnitW {
    const uint8_t* units;  // [Mp/128][K/32][4608]
    uint32_t M;            // rows the epilogue writes
    uint32_t Mp;           // rows in the layout (multiple of 128)
    uint32_t K;            // multiple of 32
};

// Partial sums of row tiles cut between CTAs: part[cta][side][128] (side 0 =
// the CTA's first row tile, 1 = its last), ticket[row tile] counts the pieces.
struct SplitScratch {
    float* part;
    uint32_t* ticket;
};

struct MmaShape {
    uint32_t NS;           // ring stages
    uint32_t xstride;      // bytes between the two digit arrays (K halves)
    uint32_t tmem_cols;    // power of two >= 64 * NS (8 columns per tile)
};

// ---------------------------------------------------------------- prologues
// Digit threads build the input vector's digits.  load() reads four
// consecutive elements (16-byte aligned), accumulates what the prologue needs
// (sum of squares, max |p| as a bit pattern) and returns p, the value before
// the per-vector factor; factor() turns the sum of squares into that factor.

// Running max of |v| over the bit patterns: unlike fmaxf it keeps a NaN (whose
// pattern is above inf's), so a block holding a NaN or inf is seen as one.
__device__ __forceinline__ void amax4(float& mx, const float4& v) {
    uint32_t m = __float_as_uint(mx);
    m = max(m, __float_as_uint(fabsf(v.x)));
    m = max(m, __float_as_uint(fabsf(v.y)));
    m = max(m, __float_as_uint(fabsf(v.z)));
    m = max(m, __float_as_uint(fabsf(v.w)));
    mx = __uint_as_float(m);
}

struct MProCopy {
    const float* src;
    __device__ const float* base(uint32_t) const { return src; }
    __device__ float4 load(const float* s, uint32_t k, float&, float& mx) const {
        const float4 v = *reinterpret_cast<const float4*>(s + k);
        amax4(mx, v);
        return v;
    }
    __device__ float factor(float, uint32_t) const { return 1.0f; }
};

// RMSNorm (kernels/cpu_ref.hpp:11-28): value = x * w * inv.  With `embed`
// the source row is embed[st->cur_token] and CTA 0 also writes it to x_out.
struct MProNorm {
    const float* src;
    const float* w;
    float eps;
    const float* embed;
    const DevState* st;
    float* x_out;
    __device__ const float* base(uint32_t K) const { return embed ? embed + (size_t)st->cur_token * K : src; }
    __device__ float4 load(const float* s, uint32_t k, float& ss, float& mx) const {
        const float4 v = *reinterpret_cast<const float4*>(s + k);
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
    __device__ float factor(float ss, uint32_t K) const {
        return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
    }
};

// Signed base-256 digits of v, |v| <= 2^21: v = 65536*hi + 256*mid + lo.
__device__ __forceinline__ void digits3(int v, int& hi, int& mid, int& lo) {
    lo = ((v + 128) & 255) - 128;
    const int v1 = (v - lo) >> 8;
    mid = ((v1 + 128) & 255) - 128;
    hi = (v1 - mid) >> 8;
}

// Digit area of the B operand: for each K half c (0, 1), block b's three digit
// rows (hi, mid, lo; 16 bytes each = the 16 elements of that half) at xb + c *
// xstride + 48 b, then the block factors 2^-e_b as floats at 2 * xstride.  The
// B tile of block b (N = 8 rows of 16 bytes per K half) starts at its hi row:
// rows 3..7 are the next blocks' digits, which only reach D columns 3..7,
// never read.  128 bytes of padding end each digit array.

__device__ __forceinline__ uint32_t blk_off(uint32_t xstride) { return 2 * xstride; }

// Block exponent e with max |p| * 2^e in [2^20, 2^21), so that round(p * 2^e)
// fits 22 bits; finite = false for a block holding an inf or NaN.
__device__ __forceinline__ int block_exponent(float am, bool& finite) {
    finite = isfinite(am);
    int e = 0;
    if (am > 0.0f && finite) {
        int ex;  // am = fr * 2^ex, fr in [0.5, 1)
        if (am >= 1.17549435e-38f)
            ex = ((__float_as_int(am) >> 23) & 255) - 126;
        else
            frexpf(am, &ex);
        e = 21 - ex;
        if (e > 149) e = 149;  // 2^-e stays representable
    }
    return e;
}

// 2^k for |k| <= 126, exactly.
__device__ __forceinline__ float pow2i(int k) { return __int_as_float((127 + k) << 23); }

// 2^-e for the block exponents above (subnormal below 2^-126).
__device__ __forceinline__ float pow2neg(int e) { return e <= 126 ? pow2i(-e) : ldexpf(1.0f, -e); }

// Writes the digits of one item (8 elements: block idx/4, elements 4 (idx%4)
// + {0..3} of each K half), v = round(p * c1 * c2).
__device__ __forceinline__ void pack_item(uint8_t* xb, uint32_t xstride, uint32_t idx, const float4& a,
                                          const float4& b, float c1, float c2) {
    const float va[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t r[3][2] = {{0, 0}, {0, 0}, {0, 0}};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int v = __float2int_rn(__fmul_rn(__fmul_rn(va[j], c1), c2));
        int hi, mid, lo;
        digits3(v, hi, mid, lo);
        const int sh = 8 * (j & 3);
        r[0][j >> 2] |= (uint32_t)(hi & 255) << sh;
        r[1][j >> 2] |= (uint32_t)(mid & 255) << sh;
        r[2][j >> 2] |= (uint32_t)(lo & 255) << sh;
    }
    const uint32_t blk = idx >> 2, tig = idx & 3;
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int d = 0; d < 3; ++d)
            *reinterpret_cast<uint32_t*>(xb + c * xstride + blk * 48 + d * 16 + tig * 4) = r[d][c];
}

// round(p * 2^e) for |p * 2^e| <= 2^21 (round half to even, as cvt.rni).
__device__ __forceinline__ int scaled_round(float p, int e) {
    const float t = __fmul_rn(__fmul_rn(p, pow2i(e / 2)), pow2i(e - e / 2));
    return __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
}

// One warp writes the digits of one 32-element block, lane i holding element i
// (warp-uniform call).  The block's max |p| is one redux.sync on the bit
// patterns (monotonic for non-negative floats; an inf or NaN anywhere makes
// the block factor NaN, so it propagates to every output as in fp32
// arithmetic); each lane packs its three digit bytes into one word and three
// shuffles bring the next lanes' words for the 4-element digit words of lanes
// 0, 4, ... .  hi_row: the block's hi digit row of K half 0 (16 bytes; the mid
// and lo rows follow at +16 and +32, K half 1 at hi_row + half_stride);
// factor: where the block factor 2^-e goes.
__device__ __forceinline__ void warp_digits(uint8_t* hi_row, uint32_t half_stride, float* factor, float p,
                                            uint32_t lane) {
    const float am = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(p))));
    bool finite;
    const int e = block_exponent(am, finite);
    const int v = finite ? scaled_round(p, e) : 0;
    int hi, mid, lo;
    digits3(v, hi, mid, lo);
    const uint32_t w0 = ((uint32_t)hi & 255u) | (((uint32_t)mid & 255u) << 8) | (((uint32_t)lo & 255u) << 16);
    const uint32_t w1 = __shfl_down_sync(0xffffffffu, w0, 1);
    const uint32_t w2 = __shfl_down_sync(0xffffffffu, w0, 2);
    const uint32_t w3 = __shfl_down_sync(0xffffffffu, w0, 3);
    if ((lane & 3) == 0) {
        // digit d of elements lane .. lane+3: byte d of w0, w1, w2, w3
        const uint32_t a01 = __byte_perm(w0, w1, 0x5140), a23 = __byte_perm(w2, w3, 0x5140);  // hi, mid bytes
        const uint32_t b01 = __byte_perm(w0, w1, 0x0062), b23 = __byte_perm(w2, w3, 0x0062);  // lo bytes
        uint8_t* q = hi_row + (lane >> 4) * half_stride + (lane & 15);
        *reinterpret_cast<uint32_t*>(q) = __byte_perm(a01, a23, 0x5410);        // hi
        *reinterpret_cast<uint32_t*>(q + 16) = __byte_perm(a01, a23, 0x7632);   // mid
        *reinterpret_cast<uint32_t*>(q + 32) = __byte_perm(b01, b23, 0x5410);   // lo
    }
    if (lane == 0) *factor = finite ? pow2neg(e) : __int_as_float(0x7fc00000);
}

// Builds the digit area of a whole input vector with one exponent per 32-element
// block, and returns the per-vector factor (the RMSNorm factor; 1 without a
// norm).  Item idx (8 elements) goes to digit thread idx % 288; the four items
// of a block sit in four consecutive lanes, which share the block's max |p|
// by two shuffles.  A block holding an inf or NaN gets a NaN factor, so every
// output it reaches is NaN, as in fp32 arithmetic.  Called by the 288 threads
// of the digit warps (tid = 0..287); ends with the digits visible to the
// tensor cores.
template <class Pro>
__device__ float block_digits(const Pro& pro, uint32_t K, uint8_t* xb, uint32_t xstride, float* red, uint32_t tid) {
    const float* s = pro.base(K);
    const uint32_t items = K >> 3;
    float ss = 0.0f;
    for (uint32_t i0 = 0; i0 < items; i0 += kDigitThreads) {  // same trip count in every thread (shuffles below)
        const uint32_t idx = i0 + tid;
        const bool valid = idx < items;
        const uint32_t k = (idx >> 2) * 32 + (idx & 3) * 4;
        float4 pa = make_float4(0.f, 0.f, 0.f, 0.f), pb = pa;
        float mx = 0.0f;
        if (valid) {
            pa = pro.load(s, k, ss, mx);
            pb = pro.load(s, k + 16, ss, mx);
        }
        uint32_t mb = __float_as_uint(mx);
        mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
        mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
        bool finite;
        const int e = block_exponent(__uint_as_float(mb), finite);
        if (valid) {
            pack_item(xb, xstride, idx, pa, pb, pow2i(e / 2), pow2i(e - e / 2));
            if ((idx & 3) == 0)
                *reinterpret_cast<float*>(xb + blk_off(xstride) + 4 * (idx >> 2)) =
                    finite ? pow2neg(e) : __int_as_float(0x7fc00000);
        }
    }
    ss = warp_sum(ss);
    const uint32_t lane = tid & 31, w = tid >> 5;
    if (lane == 0) red[w] = ss;
    fence_proxy_async();  // generic-proxy writes -> visible to the tensor cores
    digit_sync();
    float tss = 0.0f;
#pragma unroll
    for (int i = 0; i < kDigitWarps; ++i) tss += red[i];
    return pro.factor(tss, K);
}

// ---------------------------------------------------------------- epilogues (epilogue warp)
// tile(): the 32 lanes of the finisher warp, once per finished row tile;
// rs(t) is the final value of row row0 + t.  end(): after the CTA's last tile.

struct StreamState {
    float bv;     // running argmax value of this lane (logits epilogue)
    uint32_t bi;  // running argmax index, 0xFFFFFFFF = none
};

struct SEpiStore {
    float* y;
    template <class F>
    __device__ void tile(StreamState&, uint32_t row0, uint32_t T, uint32_t M, int lane, F rs) const {
        for (uint32_t t = lane; t < T; t += 32)
            if (row0 + t < M) y[row0 + t] = rs(t);
    }
    __device__ void end(StreamState&, int) const {}
};

// x[m] += y[m] (transformer_engine.cpp:191-195, 222-225); optional per-layer tap.
struct SEpiResidual {
    float* x;
    float* tap;
    template <class F>
    __device__ void tile(StreamState&, uint32_t row0, uint32_t T, uint32_t M, int lane, F rs) const {
        for (uint32_t t = lane; t < T; t += 32) {
            const uint32_t r = row0 + t;
            if (r >= M) continue;
            const float v = __fadd_rn(__ldcg(x + r), rs(t));  // x may have been written by another SM
            x[r] = v;
            if (tap) tap[r] = v;
        }
    }
    __device__ void end(StreamState&, int) const {}
};

// (gate, up) row pairs: act[j] = silu(gate) * up (cpu_ref.hpp:74-79, transformer_engine.cpp:212-215).
struct SEpiSwiGLU {
    float* act;
    template <class F>
    __device__ void tile(StreamState&, uint32_t row0, uint32_t T, uint32_t M, int lane, F rs) const {
        for (uint32_t p = lane; p < T / 2; p += 32) {
            if (row0 + 2 * p + 1 >= M) continue;
            const float g = rs(2 * p), u = rs(2 * p + 1);
            const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            act[(row0 >> 1) + p] = __fmul_rn(s, u);
        }
    }
    __device__ void end(StreamState&, int) const {}
};

// q/k/v rows with RoPE pairs and the KV append (see EpiQKV in bt_gemv.cuh).
template <typename KVT>
struct SEpiQKV {
    EpiQKV<KVT> e;
    template <class F>
    __device__ void tile(StreamState&, uint32_t row0, uint32_t T, uint32_t M, int lane, F rs) const {
        const uint32_t pos = e.st->pos;
        if (pos >= e.max_seq) return;
        for (uint32_t p = lane; p < T / 2; p += 32) {
            const uint32_t r = row0 + 2 * p;
            if (r >= M) continue;
            const float a = rs(2 * p), b = rs(2 * p + 1);
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
    }
    __device__ void end(StreamState&, int) const {}
};

// Logits + greedy argmax: per-lane running best, per-CTA partial; the last CTA
// (atomic ticket) reduces the partials and advances the sequence state.
struct SEpiLogits {
    EpiLogits e;
    template <class F>
    __device__ void tile(StreamState& s, uint32_t row0, uint32_t T, uint32_t M, int lane, F rs) const {
        for (uint32_t t = lane; t < T; t += 32) {
            const uint32_t r = row0 + t;
            if (r >= M) continue;
            const float v = rs(t);
            e.logits[r] = v;
            if (s.bi == 0xFFFFFFFFu || better(v, r, s.bv, s.bi)) { s.bv = v; s.bi = r; }
        }
    }
    __device__ void end(StreamState& s, int lane) const {
        float bv = s.bv;
        uint32_t bi = s.bi;
        warp_argmax(bv, bi);
        uint32_t last = 0;
        if (lane == 0) {
            e.part_val[blockIdx.x] = bv;
            e.part_idx[blockIdx.x] = bi;
            __threadfence();
            last = atomicAdd(e.ticket, 1u) == gridDim.x - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence();
        bv = -INFINITY;
        bi = 0xFFFFFFFFu;
        for (uint32_t i = lane; i < gridDim.x; i += 32) {
            const float v = __ldcg(e.part_val + i);
            const uint32_t ix = __ldcg(e.part_idx + i);
            if (ix != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || better(v, ix, bv, bi))) { bv = v; bi = ix; }
        }
        warp_argmax(bv, bi);
        if (lane == 0) {
            if (bi != 0xFFFFFFFFu) bi += e.v0;  // vocab index
            if (e.tp_world > 1) {
                // every rank's best to every rank, then the best of all in rank (= vocab) order
                const uint64_t tagw = (uint64_t)e.tag << 32;
                for (uint32_t q = 0; q < e.tp_world; ++q) {
                    uint64_t* slot = e.xch[q] + e.xch_off + 2 * e.tp_rank;
                    st_relaxed_sys_u64(slot, tagw | __float_as_uint(bv));
                    st_relaxed_sys_u64(slot + 1, tagw | bi);
                }
                const uint64_t* own = e.xch[e.tp_rank] + e.xch_off;
                float gv = -INFINITY;
                uint32_t gi = 0xFFFFFFFFu;
                const uint64_t t0 = global_ns();
                for (uint32_t q = 0; q < e.tp_world; ++q) {
                    uint64_t wv = 0, wi = 0;
                    while (true) {
                        wv = ld_relaxed_sys_u64(own + 2 * q);
                        wi = ld_relaxed_sys_u64(own + 2 * q + 1);
                        if ((uint32_t)(wv >> 32) == e.tag && (uint32_t)(wi >> 32) == e.tag) break;
                        if (global_ns() - t0 > kWaitNs) {
                            atomicExch(&e.st->error, 1u);
                            break;
                        }
                    }
                    const float v = __uint_as_float((uint32_t)wv);
                    const uint32_t ix = (uint32_t)wi;
                    if (ix != 0xFFFFFFFFu && (gi == 0xFFFFFFFFu || better(v, ix, gv, gi))) { gv = v; gi = ix; }
                }
                bv = gv;
                bi = gi;
            }
            const uint32_t ix = bi == 0xFFFFFFFFu ? 0 : bi;
            DevState* st = e.st;
            const uint32_t pos = st->pos;
            const uint32_t next = (pos + 1 < st->n_fixed) ? e.tok_hist[pos + 1] : ix;
            if (pos < e.max_seq) e.tok_hist[pos + 1] = next;
            st->last_argmax = ix;
            st->cur_token = next;
            st->pos = pos + 1;
            if (e.bump_epoch) {
                st->pad[0] += 1;
                e.ticket[1] += 1;
            }
            *e.ticket = 0;
        }
    }
};

// ---------------------------------------------------------------- MMA issue
// Lane 0 of issuer warp t, one stage (n tiles, ring slot s): tiles t, t + 4,
// ... of the stage.  a0/d0: the descriptor of tile t of slot 0 and its TMEM
// columns; bt: the block index of tile t.  Descriptors advance by adding to
// the start-address field (shared addresses < 256 KB: no carry).
__device__ __forceinline__ void issue_stage(uint32_t t, uint32_t n, uint32_t s, uint32_t bt, uint32_t NB, uint64_t a0,
                                            uint64_t b0, uint32_t d0) {
#pragma unroll
    for (uint32_t k = 0; k < kStageTiles / kIssuers; ++k) {
        const uint32_t tt = t + k * kIssuers;
        if (tt < n)
            umma_s8(d0 + s * (kStageTiles * kTileCols) + k * kIssuers * kTileCols,
                    a0 + ((s * kStageBytes + k * kIssuers * kTileBytes) >> 4), b0 + bt * 3, kIdescS8, 0);
        bt += kIssuers;
        while (bt >= NB) bt -= NB;
    }
}

// ---------------------------------------------------------------- accumulator warp
// Stages of an accumulator warp's loop handled together (their waits, tensor
// memory loads and scale loads overlap).  Measured: 2 is slower than 1 (the
// release of a stage then waits for the next stage's MMAs).
constexpr uint32_t kAccBatch = 1;

// Accumulator warp over tiles [u0, u1) in nstages stages: lane's row `row` of
// every tile, y = (256 hi + mid) 256 + lo from the tile's three TMEM columns,
// acc += scale(row, tile) * blk[block] * y.  blk: per-block factors (null: 1).
// Before a tile of a new row tile, flush() hands acc on (and must zero it and
// advance cur_g).  s/ph: the ring position, carried by the caller.
struct NoStageHook {
    __device__ void operator()(uint32_t, uint32_t, float = 0.0f) const {}
};

template <class Flush, class Hook = NoStageHook>
__device__ __forceinline__ void acc_stages(uint32_t u0, uint32_t u1, uint32_t NB, uint32_t nstages, const uint8_t* ring,
                                           uint32_t NS, uint32_t taddr, uint32_t row, const float* blk,
                                           uint64_t* mma_done, uint64_t* empty, uint32_t& s, uint32_t& ph, bool& ok,
                                           uint32_t* err, float& acc, uint32_t& cur_g, Flush flush,
                                           Hook hook = Hook()) {
    const uint32_t lane = threadIdx.x & 31;
    uint32_t g = NB ? u0 / NB : 0, b = u0 - g * NB;  // row tile and block of the next tile
    for (uint32_t j = 0; j < nstages; j += kAccBatch) {
        const uint32_t m = min(kAccBatch, nstages - j);  // stages in this batch (warp-uniform)
        uint32_t d[kAccBatch][kStageTiles * kTileCols];
        float sc[kAccBatch][kStageTiles];
        uint32_t sl[kAccBatch], nt[kAccBatch];
#pragma unroll
        for (uint32_t k = 0; k < kAccBatch; ++k) {
            sl[k] = s;
            nt[k] = 0;
            if (k < m) {
                hook(j + k, 5);
                if (ok) ok = mbar_wait(&mma_done[s], ph, err);
                hook(j + k, 2);
                tcgen05_fence_after();
                tmem_ld64(taddr + s * (kStageTiles * kTileCols), d[k]);
                nt[k] = min(kStageTiles, u1 - (u0 + (j + k) * kStageTiles));
                const uint8_t* st = ring + (size_t)s * kStageBytes + kTileQBytes + row * 4;
#pragma unroll
                for (uint32_t t = 0; t < kStageTiles; ++t)
                    sc[k][t] = t < nt[k] ? *reinterpret_cast<const float*>(st + t * kTileBytes) : 0.0f;
                if (++s == NS) { s = 0; ph ^= 1; }
            }
        }
        tmem_wait_ld();
        tcgen05_fence_before();
        __syncwarp();
        if (lane == 0)
            for (uint32_t k = 0; k < m; ++k) mbar_arrive(&empty[sl[k]]);  // stages (smem and TMEM columns) free
        hook(j, 3);
#pragma unroll
        for (uint32_t k = 0; k < kAccBatch; ++k) {
            if (k >= m) break;
            // block factors (read after the release) and digit sums before the first possible flush
            float y[kStageTiles], bs[kStageTiles];
#pragma unroll
            for (uint32_t t = 0, bt = b; t < kStageTiles; ++t) {
                const uint32_t* dt = d[k] + kTileCols * t;  // columns hi, mid, lo of tile t
                y[t] = fmaf(fmaf(small_i2f((int)dt[0]), 256.0f, small_i2f((int)dt[1])), 256.0f, small_i2f((int)dt[2]));
                bs[t] = blk ? blk[bt] : 1.0f;
                if (++bt == NB) bt = 0;
            }
            hook(j + k, 7, [&] {
                float z = 0.0f;  // every digit sum and factor (the timestamp waits for them)
#pragma unroll
                for (uint32_t t = 0; t < kStageTiles; ++t) z += y[t] + bs[t];
                return z;
            }());
            if (cur_g == g && b + nt[k] <= NB) {
                // no row tile ends before the stage's last tile: one FMA chain, no flush
#pragma unroll
                for (uint32_t t = 0; t < kStageTiles; ++t)
                    if (t < nt[k]) acc = fmaf(sc[k][t] * bs[t], y[t], acc);  // weight scale x the block's factor
                b += kStageTiles;
                while (b >= NB) { b -= NB; ++g; }
            } else {
#pragma unroll
                for (uint32_t t = 0; t < kStageTiles; ++t) {
                    if (t < nt[k]) {
                        while (cur_g < g) flush();
                        acc = fmaf(sc[k][t] * bs[t], y[t], acc);
                    }
                    if (++b == NB) { b = 0; ++g; }
                }
            }
        }
        hook(j, 6, acc);
    }
}

// ---------------------------------------------------------------- kernel

// The next GEMV of the sequence: the producer prefetches into L2 the first
// bytes of the tile range that CTA blockIdx.x of that GEMV will stream, so its
// first stages hit in L2 while this kernel drains.
struct NextW {
    const uint8_t* units;  // null: nothing to prefetch
    uint32_t Mp, K, grid;
    uint32_t bytes;        // prefetch budget per CTA
};

// CTA of a G-way split of U tiles that owns tile u: the largest c with U c / G <= u.
__device__ __forceinline__ uint32_t split_cta(uint64_t u, uint64_t U, uint32_t G) {
    return (uint32_t)(((u + 1) * G + U - 1) / U) - 1;
}

template <class Pro, class Epi>
__global__ void __launch_bounds__(kMmaThreads, 2)
gemv_mma_kernel(UnitW W, MmaShape sh, Pro pro, Epi epi, SplitScratch sp, NextW nx, uint32_t* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMmaMaxRing], empty[kMmaMaxRing], mma_done[kMmaMaxRing];
    __shared__ __align__(8) uint64_t red_full[kRedSlots], red_free[kRedSlots];
    __shared__ float red[kRedSlots][kTileRows];
    __shared__ float fin[kTileRows];
    __shared__ float redd[2 * kDigitWarps];
    __shared__ uint32_t s_tmem;

    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t K = W.K, NB = K / kTileK, NS = sh.NS;
    const uint32_t U = (W.Mp / kTileRows) * NB;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const uint32_t u0 = (uint32_t)(((uint64_t)U * c) / G);
    const uint32_t u1 = (uint32_t)(((uint64_t)U * (c + 1)) / G);
    const uint32_t g_first = u0 / NB, g_last = (u1 - 1) / NB;
    const uint32_t ngroups = g_last - g_first + 1;
    const uint32_t nstages = (u1 - u0 + kStageTiles - 1) / kStageTiles;
    uint8_t* ring = smem;
    uint8_t* xb = smem + (size_t)NS * kStageBytes;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kAccWarps);
            mbar_init(&mma_done[s], kIssuers);  // one commit per issuer
        }
        for (int r = 0; r < kRedSlots; ++r) {
            mbar_init(&red_full[r], kAccWarps);
            mbar_init(&red_free[r], 1);
        }
        fence_mbar_init();
    }
    if (warp == kMmaWarp0) {
        tmem_alloc(&s_tmem, sh.tmem_cols);
        tmem_relinquish();
    }
    tcgen05_fence_before();
    __syncthreads();
    tcgen05_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == kProducerWarp) {
        // ---------------- producer
        if (lane == 0) {
            uint32_t issued = 0, s = 0, ph = 0;
            for (uint32_t j = 0; j < nstages; ++j) {
                if (j >= NS && !mbar_wait(&empty[s], ph ^ 1, err)) break;
                const uint32_t ub = u0 + j * kStageTiles;
                const uint32_t n = min(kStageTiles, u1 - ub);
                mbar_expect_tx(&full[s], n * kTileBytes);
                bulk_g2s(ring + (size_t)s * kStageBytes, W.units + (size_t)ub * kTileBytes, n * kTileBytes, &full[s]);
                issued = j + 1;
                if (++s == NS) { s = 0; ph ^= 1; }
            }
            // warm L2 with the start of this CTA's share of the next GEMV
            if (nx.units && c < nx.grid) {
                const uint64_t U2 = (uint64_t)(nx.Mp / kTileRows) * (nx.K / kTileK);
                const uint64_t v0 = U2 * c / nx.grid, v1 = U2 * (c + 1) / nx.grid;
                uint64_t bytes = (v1 - v0) * kTileBytes;
                if (bytes > nx.bytes) bytes = nx.bytes;
                const uint8_t* p = nx.units + v0 * kTileBytes;
                for (uint64_t o = 0; o < bytes; o += 32768) {
                    const uint32_t n = (uint32_t)((bytes - o) < 32768 ? (bytes - o) : 32768);
                    bulk_prefetch_l2(p + o, n & ~15u);
                }
            }
            // copies still in flight must land before the CTA may exit
            const uint32_t first = issued > NS ? issued - NS : 0;
            for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, nullptr);
        }
        return;
    }

    // ---------------- warps 1-9: the input vector's digits (every thread gets the per-vector factor)
    pdl_wait();
    const float f = block_digits(pro, K, xb, sh.xstride, redd, threadIdx.x - 32);
    const float* blk = reinterpret_cast<const float*>(xb + blk_off(sh.xstride));

    if (warp < kAccWarp0) {
        // ---------------- MMA issue: lane 0 of warp 1+t issues tiles t, t+4 of every stage
        const uint32_t t = warp - kMmaWarp0;
        if (lane == 0) {
            bool ok = true;
            uint32_t s = 0, ph = 0, b = (u0 + t) % NB;
            // descriptors advance by adding to the start-address field (addresses < 256 KB: no carry)
            const uint64_t a0 = umma_desc(smem_u32(ring + t * kTileBytes), 128, 256);
            const uint64_t b0 = umma_desc(smem_u32(xb), sh.xstride, 128);
            const uint32_t d0 = tmem + t * kTileCols;
            for (uint32_t j = 0; j < nstages; ++j) {
                if (ok) ok = mbar_wait(&full[s], ph, err);
                tcgen05_fence_after();
                if (ok) issue_stage(t, min(kStageTiles, u1 - (u0 + j * kStageTiles)), s, b, NB, a0, b0, d0);
                umma_commit(&mma_done[s]);  // arrives once this issuer's MMAs are complete
                if (++s == NS) { s = 0; ph ^= 1; }
                b += kStageTiles;
                while (b >= NB) b -= NB;
            }
        }
        __syncwarp();
        tmem_sync();  // every accumulator warp is done with tensor memory
        if (warp == kMmaWarp0) {
            tcgen05_fence_after();
            tmem_dealloc(tmem, sh.tmem_cols);
        }
        return;
    }

    if (warp == kFinWarp) {
        // ---------------- finisher: per-vector factor, cross-CTA merge, epilogue
        StreamState est{-INFINITY, 0xFFFFFFFFu};
        bool ok = true;
        uint32_t slot = 0, ph = 0;
        for (uint32_t gi = 0; gi < ngroups; ++gi) {
            if (ok) ok = mbar_wait(&red_full[slot], ph, err);
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[i] = red[slot][lane + 32 * i] * f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_free[slot]);
            if (++slot == kRedSlots) { slot = 0; ph ^= 1; }
            const uint32_t g = g_first + gi;
            const uint32_t c_lo = split_cta((uint64_t)g * NB, U, G);
            const uint32_t c_hi = split_cta((uint64_t)(g + 1) * NB - 1, U, G);
            if (c_lo != c_hi) {
                const uint32_t side = g == g_first ? 0 : 1;
                float* part = sp.part + ((size_t)c * 2 + side) * kTileRows;
#pragma unroll
                for (int i = 0; i < 4; ++i) part[lane + 32 * i] = v[i];
                __threadfence();
                __syncwarp();
                uint32_t last = 0;
                if (lane == 0) last = atomicAdd(sp.ticket + g, 1u) == c_hi - c_lo;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;  // a later CTA finishes this row tile
                __threadfence();
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = 0.0f;
                for (uint32_t cb = c_lo; cb <= c_hi; cb += 4) {  // 4 CTAs' partials in flight, summed in CTA order
                    float pv[4][4];
#pragma unroll
                    for (uint32_t u = 0; u < 4; ++u) {
                        const uint32_t cc = cb + u;
                        if (cc > c_hi) break;
                        const uint32_t first_cc = (uint32_t)(((uint64_t)U * cc) / G) / NB;
                        const float* pc = sp.part + ((size_t)cc * 2 + (g == first_cc ? 0 : 1)) * kTileRows;
#pragma unroll
                        for (int i = 0; i < 4; ++i) pv[u][i] = __ldcg(pc + lane + 32 * i);
                    }
#pragma unroll
                    for (uint32_t u = 0; u < 4; ++u) {
                        if (cb + u > c_hi) break;
#pragma unroll
                        for (int i = 0; i < 4; ++i) v[i] += pv[u][i];
                    }
                }
                if (lane == 0) sp.ticket[g] = 0;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) fin[lane + 32 * i] = v[i];
            __syncwarp();
            epi.tile(est, g * kTileRows, kTileRows, W.M, lane, [&](uint32_t t) { return fin[t]; });
            __syncwarp();
        }
        epi.end(est, lane);
        return;
    }

    // ---------------- accumulators: warp 5+i reads TMEM lane quarter (5+i)%4, all tiles of every stage
    const uint32_t q = warp & 3;
    const uint32_t row = 32 * q + lane;
    const uint32_t taddr = tmem + ((32 * q) << 16);
    float acc = 0.0f;
    bool ok = true;
    uint32_t cur_g = g_first, rslot = 0, rph = 0, gi = 0;
    auto flush = [&]() {
        if (gi >= kRedSlots && ok) ok = mbar_wait(&red_free[rslot], rph ^ 1, err);
        red[rslot][row] = acc;
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_full[rslot]);
        acc = 0.0f;
        ++gi;
        if (++rslot == kRedSlots) { rslot = 0; rph ^= 1; }
        ++cur_g;
    };
    uint32_t s = 0, ph = 0;
    acc_stages(u0, u1, NB, nstages, ring, NS, taddr, row, blk, mma_done, empty, s, ph, ok, err, acc, cur_g, flush);
    while (cur_g <= g_last) flush();
    tcgen05_fence_before();
    tmem_sync();
}

// ---------------------------------------------------------------- host side

inline uint32_t mma_xstride(uint32_t K) { return ((K / 32) * 48 + 128 + 15) & ~15u; }

// Shared digit area: two digit arrays, then the block factors.
inline uint32_t mma_digit_bytes(uint32_t K) { return 2 * mma_xstride(K) + (((K / 32) * 4 + 15) & ~15u); }

// Largest K whose digit area fits beside a two-stage ring (220 KB of dynamic shared memory).
constexpr uint32_t kGemvMaxK = 48384;

inline size_t mma_smem(const MmaShape& sh, uint32_t K) {
    // at least 80 KB, so that no more than two CTAs share an SM's tensor memory
    const size_t need = (size_t)sh.NS * kStageBytes + mma_digit_bytes(K);
    return need > 80 * 1024 ? need : 80 * 1024;
}

// Ring of about ring_bytes (2..8 stages); one CTA per SM (at most U).
inline bool mma_plan(uint32_t Mp, uint32_t K, uint32_t nsm, uint32_t ring_bytes, MmaShape& sh, uint32_t& grid) {
    if (K % kTileK || Mp % kTileRows || Mp == 0 || K == 0) return false;
    uint32_t ns = ring_bytes / kStageBytes;
    if (ns < 2) ns = 2;
    if (ns > kMmaMaxRing) ns = kMmaMaxRing;
    sh.NS = ns;
    sh.xstride = mma_xstride(K);
    uint32_t cols = 32;
    while (cols < ns * kStageTiles * kTileCols) cols <<= 1;
    sh.tmem_cols = cols;
    const uint64_t U = (uint64_t)(Mp / kTileRows) * (K / kTileK);
    grid = (uint32_t)(U < nsm ? U : nsm);
    return mma_smem(sh, K) <= 220 * 1024 && (cols <= 256 || mma_smem(sh, K) > 114 * 1024);
}

// Default ring: about 200 KB of shared memory per CTA (one CTA per SM).
// Measured on the 7B decode step, a deep ring beats two co-resident CTAs with
// half the ring each (the next GEMV then streams under programmatic dependent
// launch, but every GEMV has half the bytes in flight).
constexpr uint32_t kMmaCoResidentDyn = 200 * 1024;

inline uint32_t mma_ring_bytes(uint32_t K) {
    static int env_kb = -1;
    if (env_kb < 0) {
        const char* v = std::getenv("BT_GEMV_RING_KB");
        env_kb = v ? std::atoi(v) : 0;
    }
    if (env_kb >= 36 && env_kb <= 200) return (uint32_t)env_kb * 1024;
    const uint32_t digits = mma_digit_bytes(K), two = 2 * kStageBytes;
    return kMmaCoResidentDyn > digits + two ? kMmaCoResidentDyn - digits : two;
}

inline uint32_t mma_grid(uint32_t Mp, uint32_t K, uint32_t nsm) {
    const uint64_t U = (uint64_t)(Mp / kTileRows) * (K / kTileK);
    return (uint32_t)(U < nsm ? U : nsm);
}

// Row tiles of an Mp-row matrix: the split scratch needs one ticket per row tile.
inline uint32_t mma_row_tiles(uint32_t Mp) { return Mp / kTileRows; }

template <class Pro, class Epi>
cudaError_t launch_gemv_mma(const UnitW& W, const Pro& pro, const Epi& epi, SplitScratch sp, uint32_t* err,
                            uint32_t nsm, cudaStream_t s, bool pdl, NextW nx = NextW{nullptr, 0, 0, 0, 0},
                            uint32_t ring_bytes = 0) {
    MmaShape sh;
    uint32_t grid = 0;
    if (ring_bytes == 0) ring_bytes = mma_ring_bytes(W.K);
    if (!mma_plan(W.Mp, W.K, nsm, ring_bytes, sh, grid)) return cudaErrorInvalidValue;
    auto kern = gemv_mma_kernel<Pro, Epi>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    return launch_pdl(kern, dim3(grid), dim3(kMmaThreads), mma_smem(sh, W.K), s, pdl, W, sh, pro, epi, sp, nx, err);
}

}  // namespace bt
