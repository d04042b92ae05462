// bt_gemv_mma.cuh -- batch-1 int8 GEMV on the tensor cores, stream-K over HBM.
//
// Arithmetic.  The reference computes y[r] = sum_b scale[r][b] * sum_{i<32}
// q[r][32b+i] * x[32b+i] in fp32 (quantization/quant_types.cpp:101-121).  Here
// x is first written as a 22-bit fixed-point vector v = round(x * 2^e) with one
// power-of-two exponent e per vector (|v| < 2^22), and v as three signed
// base-256 digits hi/mid/lo (|hi| <= 64).  One mma.sync.m16n8k32 s8*s8->s32
// per (16 rows, 32 columns) gives, for every row, the three digit dot products
// sum_i q_i * digit_i exactly in integers; they are combined in fp32
// ((256*hi + mid)*256 + lo), scaled by the block scale and accumulated in fp32
// across blocks, and 2^-e is applied at the end.  The only rounding besides fp32
// accumulation is x's quantisation step of 2^-21 relative to max|x|.
//
// Layout (written by the repack kernel): rows in groups of 16, each group as
// K/32 units of 576 bytes: the 16x32 int8 block in mma fragment order (lane t's
// 16 bytes = its four A registers) followed by the 16 fp32 block scales in
// row order 0, 8, 1, 9, ..., 7, 15 (the two rows a lane pair finishes are
// adjacent).  A matrix is one contiguous stream of units, group-major.
//
// Work split (stream-K).  CTA c of G owns units [U c/G, U (c+1)/G): every CTA
// moves the same number of bytes, whatever M.  A 16-row group cut between two
// CTAs is finished by the one that completes second, adding the two partial
// sums in a fixed order (lower columns first), so results are deterministic.
//
// Warp roles (320 threads): warps 0-7 consume, warp 8 produces (cp.async.bulk
// of 32-unit stages into an mbarrier ring; it never waits for the previous
// kernel, so under programmatic dependent launch the ring fills while the
// previous kernel drains), warp 9 runs the epilogue of each finished group.
// All waits are bounded (2 s); an expired wait sets *err and the CTA still
// finishes (consumers stop waiting but keep arriving on every barrier).
#pragma once

#include "bt_common.cuh"
#include "bt_gemv.cuh"
#include "bt_ptx.cuh"

namespace bt {

constexpr uint32_t kUnitRows = 16;
constexpr uint32_t kUnitK = 32;
constexpr uint32_t kUnitQBytes = 512;   // 16 x 32 int8
constexpr uint32_t kUnitBytes = 576;    // + 16 fp32 scales
constexpr int kMmaConsumers = 8;
constexpr int kMmaProducerWarp = 8;
constexpr int kMmaEpilogueWarp = 9;
constexpr int kMmaThreads = 320;
constexpr int kMmaRedSlots = 8;
constexpr uint32_t kMmaMaxRing = 16;
constexpr uint32_t kMmaStageUnits = 32;  // 18 KB stages

// A matrix in the unit layout.
struct UnitW {
    const uint8_t* units;  // [Mp/16][K/32][576]
    uint32_t M;            // rows the epilogue writes
    uint32_t Mp;           // rows in the layout (multiple of 16)
    uint32_t K;            // multiple of 32
};

// Partial sums of 16-row groups cut between CTA c and c+1: part[c][side][16], ticket[c].
struct SplitScratch {
    float* part;
    uint32_t* ticket;
};

struct MmaShape {
    uint32_t NS;           // ring stages
    uint32_t stage_bytes;  // kMmaStageUnits * kUnitBytes
};

// ---------------------------------------------------------------- prologues
// Consumer threads build the digit fragments of the input vector.  load()
// reads four consecutive elements (16-byte aligned), accumulates what the
// prologue needs (sum of squares, max |p|) and returns p, the value before the
// per-vector factor; factor() turns the sum of squares into that factor.

struct MProCopy {
    const float* src;
    __device__ const float* base(uint32_t) const { return src; }
    __device__ float4 load(const float* s, uint32_t k, float&, float& mx) const {
        const float4 v = *reinterpret_cast<const float4*>(s + k);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
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
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(p.x), fabsf(p.y)), fmaxf(fabsf(p.z), fabsf(p.w))));
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

// Writes the mma B fragments of one item: 8 elements (block blk, lanes tig of
// each digit) as xf[blk][digit * 4 + tig].
__device__ __forceinline__ void pack_item(uint2* xf, uint32_t idx, const float4& a, const float4& b, float c1,
                                          float c2) {
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
    for (int p = 0; p < 3; ++p) xf[blk * 12 + p * 4 + tig] = make_uint2(r[p][0], r[p][1]);
}

// Builds xf[b][lane] (lane < 12: digit lane/4 of the 8 elements that mma B
// fragment lane holds) and returns the exponent e; *bad when the vector holds
// an inf or NaN (the outputs are then NaN).  One global round trip: item idx
// (block idx/4, lane tig = idx%4, elements 32 b + 4 tig + {0..3, 16..19}) is
// loaded once into registers by consumer thread idx % 256 (K <= 12288; larger
// vectors load their tail twice).  Consumer threads only.
template <class Pro>
__device__ int build_digits(const Pro& pro, uint32_t K, uint2* xf, float* red, bool& bad) {
    constexpr int R = 6;
    const float* s = pro.base(K);
    const uint32_t items = K >> 3;
    float ss = 0.0f, mx = 0.0f;
    float4 pa[R], pb[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const uint32_t idx = threadIdx.x + 256u * i;
        if (idx < items) {
            const uint32_t k = (idx >> 2) * 32 + (idx & 3) * 4;
            pa[i] = pro.load(s, k, ss, mx);
            pb[i] = pro.load(s, k + 16, ss, mx);
        }
    }
    for (uint32_t idx = threadIdx.x + 256u * R; idx < items; idx += 256) {
        const uint32_t k = (idx >> 2) * 32 + (idx & 3) * 4;
        pro.load(s, k, ss, mx);
        pro.load(s, k + 16, ss, mx);
    }
    // sum and max over the 256 consumers
    ss = warp_sum(ss);
    mx = warp_max(mx);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { red[warp] = ss; red[8 + warp] = mx; }
    consumer_sync();
    float tss = 0.0f, tmx = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) { tss += red[i]; tmx = fmaxf(tmx, red[8 + i]); }
    const float f = pro.factor(tss, K);
    const float m = tmx * f;
    // m * 2^e in [2^20, 2^21): values round to |v| <= 2^21 (slack for the rounding of m)
    int e = 0;
    bad = !isfinite(m);
    if (m > 0.0f && !bad) {
        int ex;
        frexpf(m, &ex);  // m = fr * 2^ex, fr in [0.5, 1)
        e = 21 - ex;
    }
    // v = p * f * 2^e as two products that cannot overflow
    const float c1 = ldexpf(1.0f, e / 2), c2 = ldexpf(f, e - e / 2);
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const uint32_t idx = threadIdx.x + 256u * i;
        if (idx < items) pack_item(xf, idx, pa[i], pb[i], c1, c2);
    }
    for (uint32_t idx = threadIdx.x + 256u * R; idx < items; idx += 256) {
        const uint32_t k = (idx >> 2) * 32 + (idx & 3) * 4;
        float d0 = 0.0f, d1 = 0.0f;
        const float4 a = pro.load(s, k, d0, d1), b = pro.load(s, k + 16, d0, d1);
        pack_item(xf, idx, a, b, c1, c2);
    }
    consumer_sync();
    return e;
}

// ---------------------------------------------------------------- epilogues (epilogue warp)
// tile(): the 32 lanes of the epilogue warp, once per finished 16-row group;
// rs(t) is the final value of row row0 + t.  end(): after the CTA's last group.

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
            const float v = __fadd_rn(x[r], rs(t));
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
            const uint32_t ix = bi == 0xFFFFFFFFu ? 0 : bi;
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

// The next GEMV of the sequence: this CTA prefetches into L2 the first bytes
// of the unit range that CTA blockIdx.x of that GEMV will stream, so its first
// stages hit in L2 while this kernel drains.
struct NextW {
    const uint8_t* units;  // null: nothing to prefetch
    uint32_t Mp, K, grid;
    uint32_t bytes;        // prefetch budget per CTA
};

template <class Pro, class Epi>
__global__ void __launch_bounds__(kMmaThreads, 2)
gemv_mma_kernel(UnitW W, MmaShape sh, Pro pro, Epi epi, SplitScratch sp, NextW nx, uint32_t* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMmaMaxRing], empty[kMmaMaxRing];
    __shared__ __align__(8) uint64_t red_full[kMmaRedSlots], red_free[kMmaRedSlots];
    __shared__ float red[kMmaRedSlots][kMmaConsumers][16];
    __shared__ float fin[16];
    __shared__ float red32[32];
    __shared__ int s_e;
    __shared__ bool s_bad;

    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t K = W.K, NB = K / kUnitK, NS = sh.NS;
    const uint32_t U = (W.Mp / kUnitRows) * NB;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const uint32_t u0 = (uint32_t)(((uint64_t)U * c) / G);
    const uint32_t u1 = (uint32_t)(((uint64_t)U * (c + 1)) / G);
    const uint32_t g_first = u0 / NB, g_last = (u1 - 1) / NB;
    const uint32_t ngroups = g_last - g_first + 1;
    const uint32_t nstages = (u1 - u0 + kMmaStageUnits - 1) / kMmaStageUnits;
    uint8_t* ring = smem;
    uint2* xf = reinterpret_cast<uint2*>(smem + (size_t)NS * sh.stage_bytes);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMmaConsumers);
        }
        for (int r = 0; r < kMmaRedSlots; ++r) {
            mbar_init(&red_full[r], kMmaConsumers);
            mbar_init(&red_free[r], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kMmaProducerWarp) {
        // ---------------- producer: weights never depend on the previous kernel
        if (lane == 0) {
            uint32_t issued = 0, s = 0, ph = 0;
            for (uint32_t j = 0; j < nstages; ++j) {
                if (j >= NS && !mbar_wait(&empty[s], ph ^ 1, err)) break;
                const uint32_t ub = u0 + j * kMmaStageUnits;
                const uint32_t n = min(kMmaStageUnits, u1 - ub);
                mbar_expect_tx(&full[s], n * kUnitBytes);
                bulk_g2s(ring + (size_t)s * sh.stage_bytes, W.units + (size_t)ub * kUnitBytes, n * kUnitBytes, &full[s]);
                issued = j + 1;
                if (++s == NS) { s = 0; ph ^= 1; }
            }
            // warm L2 with the start of this CTA's share of the next GEMV
            if (nx.units && c < nx.grid) {
                const uint32_t nb2 = nx.K / kUnitK;
                const uint64_t U2 = (uint64_t)(nx.Mp / kUnitRows) * nb2;
                const uint64_t v0 = U2 * c / nx.grid, v1 = U2 * (c + 1) / nx.grid;
                uint64_t bytes = (v1 - v0) * kUnitBytes;
                if (bytes > nx.bytes) bytes = nx.bytes;
                const uint8_t* p = nx.units + v0 * kUnitBytes;
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

    if (warp == kMmaEpilogueWarp) {
        // ---------------- epilogue: finished groups, cross-CTA merge of cut groups
        pdl_wait();
        StreamState est{-INFINITY, 0xFFFFFFFFu};
        bool ok = true;
        const bool hi_cut = (u0 % NB) != 0;   // g_first began in CTA c-1
        const bool lo_cut = (u1 % NB) != 0;   // g_last continues in CTA c+1
        uint32_t slot = 0, ph = 0;
        for (uint32_t gi = 0; gi < ngroups; ++gi) {
            if (ok) ok = mbar_wait(&red_full[slot], ph, err);
            float v = 0.0f;
            if (lane < 16) {
#pragma unroll
                for (int w = 0; w < kMmaConsumers; ++w) v += red[slot][w][lane];
                v = s_bad ? __int_as_float(0x7fc00000) : ldexpf(v, -s_e);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_free[slot]);
            if (++slot == kMmaRedSlots) { slot = 0; ph ^= 1; }
            const int side = (gi == 0 && hi_cut) ? 1 : ((gi == ngroups - 1 && lo_cut) ? 0 : -1);
            if (side >= 0) {
                const uint32_t bnd = side == 1 ? c - 1 : c;
                float* part = sp.part + (size_t)bnd * 32;
                if (lane < 16) part[side * 16 + lane] = v;
                __threadfence();
                __syncwarp();
                uint32_t second = 0;
                if (lane == 0) second = atomicAdd(sp.ticket + bnd, 1u);
                second = __shfl_sync(0xffffffffu, second, 0);
                if (!second) continue;  // the other CTA finishes this group
                __threadfence();
                if (lane < 16) v = __ldcg(part + lane) + __ldcg(part + 16 + lane);  // lower columns first
                if (lane == 0) sp.ticket[bnd] = 0;
            }
            if (lane < 16) fin[lane] = v;
            __syncwarp();
            epi.tile(est, (g_first + gi) * kUnitRows, kUnitRows, W.M, lane, [&](uint32_t t) { return fin[t]; });
            __syncwarp();
        }
        epi.end(est, lane);
        return;
    }

    // ---------------- consumers
    pdl_wait();
    bool bad = false;
    const int e = build_digits(pro, K, xf, red32, bad);
    if (threadIdx.x == 0) {
        s_e = e;
        s_bad = bad;
    }

    // C fragment: lane (grp, tig) holds rows grp and grp+8 at columns 2 tig, 2 tig+1,
    // i.e. tig 0 the hi and mid sums, tig 1 the lo sums (tig 2, 3: zero columns).
    // After one exchange, even lanes finish row grp and odd lanes row grp + 8.
    const int grp = lane >> 2, odd = lane & 1;
    const float mA = odd ? 1.0f : 256.0f;
    const uint32_t soff = kUnitQBytes + (uint32_t)(grp * 2 + odd) * 4;  // scales stored as (r, r+8) pairs
    float acc = 0.0f;
    bool ok = true;
    uint32_t cur_g = g_first, rslot = 0, rph = 0, gi = 0;
    auto flush = [&]() {
        if (gi >= kMmaRedSlots && ok) ok = mbar_wait(&red_free[rslot], rph ^ 1, err);
        if ((lane & 3) < 2) red[rslot][warp][grp + 8 * odd] = acc;
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_full[rslot]);
        acc = 0.0f;
        ++gi;
        if (++rslot == kMmaRedSlots) { rslot = 0; rph ^= 1; }
        ++cur_g;
    };

    // warp w takes the 4 consecutive units 4w..4w+3 of every stage
    constexpr int kPerWarp = kMmaStageUnits / kMmaConsumers;
    uint32_t g = (u0 + kPerWarp * warp) / NB;            // group and block of the warp's next unit
    uint32_t b = (u0 + kPerWarp * warp) - g * NB;
    uint32_t s = 0, ph = 0;
    for (uint32_t j = 0; j < nstages; ++j) {
        if (ok) ok = mbar_wait(&full[s], ph, err);
        const uint32_t n = min(kMmaStageUnits, u1 - (u0 + j * kMmaStageUnits));
        const uint8_t* wb = ring + (size_t)s * sh.stage_bytes + (size_t)(kPerWarp * warp) * kUnitBytes;
        float y[kPerWarp], sc[kPerWarp];
        uint32_t gq[kPerWarp];
#pragma unroll
        for (int q = 0; q < kPerWarp; ++q) {
            gq[q] = g;
            y[q] = sc[q] = 0.0f;
            if ((uint32_t)(kPerWarp * warp + q) < n) {
                const uint8_t* up = wb + q * kUnitBytes;
                const uint4 a = *reinterpret_cast<const uint4*>(up + lane * 16);
                const uint2 bx = lane < 12 ? xf[b * 12 + lane] : make_uint2(0u, 0u);
                int d0, d1, d2, d3;
                mma_s8_16832(a, bx, d0, d1, d2, d3);
                const float fa = fmaf(small_i2f(d0), mA, small_i2f(d1));  // even: 256 hi + mid, odd: lo
                const float fb = fmaf(small_i2f(d2), mA, small_i2f(d3));
                const float r = __shfl_xor_sync(0xffffffffu, odd ? fa : fb, 1);
                y[q] = fmaf(odd ? r : fa, 256.0f, odd ? fb : r);
                sc[q] = *reinterpret_cast<const float*>(up + soff);
            }
            if (++b == NB) { b = 0; ++g; }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // slot free for the producer
        if (++s == NS) { s = 0; ph ^= 1; }
#pragma unroll
        for (int q = 0; q < kPerWarp; ++q) {
            if ((uint32_t)(kPerWarp * warp + q) >= n) break;
            while (cur_g < gq[q]) flush();
            acc = fmaf(sc[q], y[q], acc);
        }
        b += kMmaStageUnits - kPerWarp;  // the other warps' units of the stage
        while (b >= NB) { b -= NB; ++g; }
    }
    while (cur_g <= g_last) flush();
}

// ---------------------------------------------------------------- host side

inline size_t mma_smem(const MmaShape& sh, uint32_t K) {
    return (size_t)sh.NS * sh.stage_bytes + (size_t)(K / kUnitK) * 12 * sizeof(uint2);
}

// Ring of about ring_bytes (2..16 stages); grid so that every CTA owns at least
// one group's worth of units (a group is then cut between at most two CTAs).
inline bool mma_plan(uint32_t Mp, uint32_t K, uint32_t nsm, uint32_t ring_bytes, MmaShape& sh, uint32_t& grid) {
    if (K % kUnitK || Mp % kUnitRows || Mp == 0) return false;
    sh.stage_bytes = kMmaStageUnits * kUnitBytes;
    uint32_t ns = ring_bytes / sh.stage_bytes;
    if (ns < 2) ns = 2;
    if (ns > kMmaMaxRing) ns = kMmaMaxRing;
    sh.NS = ns;
    const uint32_t groups = Mp / kUnitRows;
    grid = nsm < groups ? nsm : groups;
    return mma_smem(sh, K) <= 220 * 1024;
}

// Default ring: what leaves two CTAs per SM co-resident (228 KB of shared
// memory per SM, 1 KB reserved per CTA, ~4.7 KB static), so that under
// programmatic dependent launch the next GEMV's CTAs start streaming their
// weights while this one drains.
constexpr uint32_t kMmaCoResidentDyn = 108 * 1024;

inline uint32_t mma_ring_bytes(uint32_t K) {
    static int env_kb = -1;
    if (env_kb < 0) {
        const char* v = std::getenv("BT_GEMV_RING_KB");
        env_kb = v ? std::atoi(v) : 0;
    }
    if (env_kb >= 36 && env_kb <= 200) return (uint32_t)env_kb * 1024;
    const uint32_t digits = (K / kUnitK) * 96, two = 2 * kMmaStageUnits * kUnitBytes;
    return kMmaCoResidentDyn > digits + two ? kMmaCoResidentDyn - digits : two;
}

inline uint32_t mma_grid(uint32_t Mp, uint32_t nsm) {
    const uint32_t groups = Mp / kUnitRows;
    return nsm < groups ? nsm : groups;
}

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
