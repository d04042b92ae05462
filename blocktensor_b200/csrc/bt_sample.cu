// bt_sample.cu -- top-k / top-p sampling on the device.
//
// sampling::sample_top_p_top_k (runtime/include/blocktensor/sampler.hpp:15-85)
// on the host: temperature <= 0 is greedy; otherwise the logits are divided by
// the temperature, sorted in decreasing order, cut to top_k, turned into
// probabilities with exp(l - max) / sum, cut where the running sum first
// reaches top_p, renormalised, and the first token whose running sum reaches
// r is returned, r the first draw of std::uniform_real_distribution<float>(0, 1)
// from std::mt19937(seed).  Here one CTA of 1024 threads:
//   1. radix select (four 8-bit passes over order-preserving keys) finds the
//      k-th largest scaled logit; candidates are the larger ones and, among
//      those equal to it, the lowest ids (the reference's sort leaves the order
//      of equal logits unspecified);
//   2. a bitonic sort orders the k candidates (logit decreasing, id increasing);
//   3. every thread takes one exp; one thread then runs the reference's
//      sequential sums, cutoff and draw in the same order and precision.
// r is computed on the host with the same standard-library engine and
// distribution the reference uses, so only the device's expf (within 2 ulp of
// the host's) can move a draw that falls within rounding of a boundary.
#include "bt_common.cuh"
#include "bt_internal.h"

#include <random>

namespace bt {

constexpr uint32_t kSampleMaxK = 4096;

__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // larger float -> larger key
}

__global__ void __launch_bounds__(1024) sample_kernel(const float* __restrict__ logits, uint32_t V, float temp,
                                                      float top_p, uint32_t K, float r, uint32_t* out) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_need, s_ngt;
    __shared__ float cl[kSampleMaxK];     // candidate scaled logits (sorted), then probabilities
    __shared__ uint32_t cid[kSampleMaxK];
    __shared__ uint32_t scan[1024];
    const uint32_t tid = threadIdx.x, nt = blockDim.x;

    // ---- 1. the k-th largest key, 8 bits at a time from the top
    uint32_t prefix = 0, need = K;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
        for (uint32_t i = tid; i < 256; i += nt) hist[i] = 0;
        __syncthreads();
        for (uint32_t i = tid; i < V; i += nt) {
            const uint32_t k = order_key(__fdiv_rn(logits[i], temp));
            if ((k & hmask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t acc = 0, d = 255;
            for (;; --d) {  // from the largest digit down
                if (acc + hist[d] >= need || d == 0) break;
                acc += hist[d];
            }
            s_prefix = prefix | (d << shift);
            s_need = need - acc;
        }
        __syncthreads();
        prefix = s_prefix;
        need = s_need;
        __syncthreads();
    }
    const uint32_t T = prefix;  // the k-th largest key; `need` of the keys equal to T are taken
    // ---- collect: keys > T in any order, keys == T by increasing id
    if (tid == 0) s_ngt = 0;
    __syncthreads();
    const uint32_t chunk = (V + nt - 1) / nt, lo = tid * chunk, hi = min(V, lo + chunk);
    uint32_t my_eq = 0;
    for (uint32_t i = lo; i < hi; ++i) {
        const float l = __fdiv_rn(logits[i], temp);
        const uint32_t k = order_key(l);
        if (k > T) {
            const uint32_t slot = atomicAdd(&s_ngt, 1u);
            cl[slot] = l;
            cid[slot] = i;
        } else if (k == T) {
            ++my_eq;
        }
    }
    scan[tid] = my_eq;
    __syncthreads();
    for (uint32_t off = 1; off < nt; off <<= 1) {  // inclusive scan of the equal counts by thread (= id order)
        const uint32_t v = tid >= off ? scan[tid - off] : 0u;
        __syncthreads();
        scan[tid] += v;
        __syncthreads();
    }
    const uint32_t ngt = s_ngt;
    uint32_t rank = scan[tid] - my_eq;
    for (uint32_t i = lo; i < hi && rank < need; ++i) {
        const float l = __fdiv_rn(logits[i], temp);
        if (order_key(l) == T) {
            cl[ngt + rank] = l;
            cid[ngt + rank] = i;
            ++rank;
        }
    }
    __syncthreads();
    // ---- 2. bitonic sort of the K candidates: logit decreasing, id increasing
    uint32_t P = 1;
    while (P < K) P <<= 1;
    for (uint32_t i = K + tid; i < P; i += nt) {
        cl[i] = -INFINITY;
        cid[i] = 0xFFFFFFFFu;
    }
    __syncthreads();
    for (uint32_t size = 2; size <= P; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t t = tid; t < P / 2; t += nt) {
                const uint32_t a = 2 * t - (t & (stride - 1)), b = a + stride;
                const bool up = (a & size) == 0;  // this half sorts "first before second"
                const float la = cl[a], lb = cl[b];
                const uint32_t ia = cid[a], ib = cid[b];
                // a before b when (la > lb) or (la == lb and ia < ib)
                const bool a_first = (la > lb) || (la == lb && ia < ib);
                if (a_first != up) {
                    cl[a] = lb; cl[b] = la;
                    cid[a] = ib; cid[b] = ia;
                }
            }
            __syncthreads();
        }
    }
    // ---- 3. probabilities in the reference's order and precision
    const float max_l = cl[0];
    __syncthreads();
    for (uint32_t i = tid; i < K; i += nt) cl[i] = expf(__fsub_rn(cl[i], max_l));
    __syncthreads();
    if (tid == 0) {
        float sum_exp = 0.0f;
        for (uint32_t i = 0; i < K; ++i) sum_exp = __fadd_rn(sum_exp, cl[i]);
        float cum = 0.0f;
        uint32_t cutoff = K;
        for (uint32_t i = 0; i < K; ++i) {
            cl[i] = __fdiv_rn(cl[i], sum_exp);
            if (cutoff == K) {
                cum = __fadd_rn(cum, cl[i]);
                if (cum >= top_p) cutoff = i + 1;
            }
        }
        float p_sum = 0.0f;
        for (uint32_t i = 0; i < cutoff; ++i) p_sum = __fadd_rn(p_sum, cl[i]);
        float acc = 0.0f;
        uint32_t pick = cid[cutoff - 1];
        for (uint32_t i = 0; i < cutoff; ++i) {
            acc = __fadd_rn(acc, __fdiv_rn(cl[i], p_sum));
            if (r <= acc) {
                pick = cid[i];
                break;
            }
        }
        *out = pick;
    }
}

}  // namespace bt

using namespace bt;

extern "C" int bt_cuda_sample_top_p_top_k(const float* logits, uint32_t vocab, float temperature, float top_p,
                                          uint32_t top_k, uint64_t seed, uint32_t* out, void* stream) {
    BT_CHECK_ARG(logits && out, "sample_top_p_top_k: null buffer");
    BT_CHECK_ARG(vocab > 0, "sample_top_p_top_k: empty logits");
    if (temperature <= 0.0f) return bt_cuda_argmax(logits, vocab, out, stream);  // sampler.hpp:23-25
    const uint32_t K = (top_k > 0 && top_k < vocab) ? top_k : vocab;
    BT_CHECK_ARG(K <= kSampleMaxK, "sample_top_p_top_k: at most 4096 candidates (top_k in 1..4096, or vocab <= 4096)");
    // the reference's draw: std::mt19937(seed), std::uniform_real_distribution<float>(0, 1) (sampler.hpp:76-78)
    std::mt19937 gen(static_cast<unsigned int>(seed));
    std::uniform_real_distribution<float> dis(0.0f, 1.0f);
    const float r = dis(gen);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    sample_kernel<<<1, 1024, 0, as_stream(stream)>>>(logits, vocab, temperature, top_p, K, r, out);
    BT_CUDA_CHECK(cudaGetLastError());
    return BT_OK;
}
