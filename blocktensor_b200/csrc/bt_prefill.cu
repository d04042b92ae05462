// bt_prefill.cu -- prompt prefill: the positions of a prompt processed as
// many-token GEMMs on the tensor cores instead of one decode step each.
//
// The reference runs a prompt through TransformerEngine::forward_single_token
// one position at a time (benchmarks/bench_runner.cpp:107-109,
// tools/bt_infer.cpp:116-125) and keeps only the K/V rows and, for the last
// position, the logits.  Here the positions pos0 .. pos0 + n - 2 go through
// every layer together (execute_layer, runtime/src/transformer_engine.cpp:114-226,
// for each of them), in chunks of up to kPrefillChunk tokens:
//
//   layer input  : token image of x * attn_norm (embedding rows for layer 0)
//   qkv GEMM     : RoPE at each position, q rows and the K/V append   (:117-146)
//   attention    : causal, each query over the cache up to its own position (:148-184)
//   o GEMM       : x += o; token image of x * ffn_norm                 (:186-197)
//   gate/up GEMM : silu(gate) * up; token image of act                 (:197-215)
//   down GEMM    : x += down; token image of x * next attn_norm        (:217-225)
//
// The last prompt token is then processed by the decode step kernel, which
// produces its logits and greedy token exactly as a decode step does, and
// decoding continues from there.
#include "bt_common.cuh"
#include "bt_gemm.cuh"
#include "bt_engine_impl.h"
#include "bt_internal.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

using namespace bt;

namespace bt {

constexpr uint32_t kPrefillChunk = 512;  // tokens per chunk (buffers are sized for it)

// Causal attention of a prompt chunk: query token t (position pos0 + t) of
// head h attends to the cache's keys 0 .. pos0 + t (those of earlier chunks and
// the chunk's own, appended by the qkv GEMM).  One warp per (head, token);
// lane i holds head dims i, i + 32, ...; keys in batches of 8 with all loads in
// flight, online softmax in fp32 (mathematically the reference's softmax over
// the scores s = q.k / sqrt(hd)).
template <int NVM, typename KVT>
__global__ void __launch_bounds__(256) prefill_attn_kernel(const float* __restrict__ q, const KVT* __restrict__ kc,
                                                           const KVT* __restrict__ vc, float* __restrict__ out,
                                                           uint32_t T, uint32_t pos0, uint32_t H, uint32_t GQ,
                                                           uint32_t hd, KVMap map, float scale) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t t = blockIdx.y * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    const uint32_t h = blockIdx.x, kvh = h / GQ;
    const uint32_t P = pos0 + t;
    const size_t DQ = (size_t)H * hd;
    const float* qp = q + (size_t)t * DQ + (size_t)h * hd;
    float qv[NVM], o[NVM];
#pragma unroll
    for (int i = 0; i < NVM; ++i) {
        const uint32_t d = lane + 32 * i;
        qv[i] = d < hd ? qp[d] : 0.0f;
        o[i] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    constexpr int B = 8;
    for (uint32_t base = 0; base <= P; base += B) {
        float kr[B][NVM], vr[B][NVM];
#pragma unroll
        for (int j = 0; j < B; ++j) {
            const uint32_t key = base + j;
            const size_t ro = key <= P ? map.row(0, kvh, key) : 0;
#pragma unroll
            for (int i = 0; i < NVM; ++i) {
                const uint32_t d = lane + 32 * i;
                const bool ok = key <= P && d < hd;
                kr[j][i] = ok ? KVConv<KVT>::to_f(kc[ro + d]) : 0.0f;
                vr[j][i] = ok ? KVConv<KVT>::to_f(vc[ro + d]) : 0.0f;
            }
        }
        float sc[B];
        float mb = -INFINITY;
#pragma unroll
        for (int j = 0; j < B; ++j) {
            float p = 0.0f;
#pragma unroll
            for (int i = 0; i < NVM; ++i) p = fmaf(qv[i], kr[j][i], p);
            p = warp_sum(p);
            sc[j] = base + j <= P ? __fmul_rn(p, scale) : -INFINITY;
            mb = fmaxf(mb, sc[j]);
        }
        const float mn = fmaxf(m, mb);
        const float alpha = expf(m - mn);
        l *= alpha;
#pragma unroll
        for (int i = 0; i < NVM; ++i) o[i] *= alpha;
#pragma unroll
        for (int j = 0; j < B; ++j) {
            const float ev = expf(sc[j] - mn);
            l += ev;
#pragma unroll
            for (int i = 0; i < NVM; ++i) o[i] = fmaf(ev, vr[j][i], o[i]);
        }
        m = mn;
    }
    float* op = out + (size_t)t * DQ + (size_t)h * hd;
#pragma unroll
    for (int i = 0; i < NVM; ++i) {
        const uint32_t d = lane + 32 * i;
        if (d < hd) op[d] = __fdiv_rn(o[i], l);
    }
}

__global__ void positions_kernel(uint32_t* pos, uint32_t T, uint32_t pos0) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < T) pos[t] = pos0 + t;
}

template <typename KVT>
cudaError_t launch_prefill_attn(const float* q, const KVT* kc, const KVT* vc, float* out, uint32_t T, uint32_t pos0,
                                uint32_t H, uint32_t GQ, uint32_t hd, const KVMap& map, float scale, cudaStream_t s) {
    const dim3 grid(H, (T + 7) / 8);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    const uint32_t nv = (hd + 31) / 32;
    if (nv <= 1) prefill_attn_kernel<1, KVT><<<grid, 256, 0, s>>>(q, kc, vc, out, T, pos0, H, GQ, hd, map, scale);
    else if (nv == 2) prefill_attn_kernel<2, KVT><<<grid, 256, 0, s>>>(q, kc, vc, out, T, pos0, H, GQ, hd, map, scale);
    else if (nv <= 4) prefill_attn_kernel<4, KVT><<<grid, 256, 0, s>>>(q, kc, vc, out, T, pos0, H, GQ, hd, map, scale);
    else prefill_attn_kernel<8, KVT><<<grid, 256, 0, s>>>(q, kc, vc, out, T, pos0, H, GQ, hd, map, scale);
    return cudaGetLastError();
}

cudaError_t launch_token_image(const float* src, const uint32_t* tokens, const float* w, uint32_t T, uint32_t K,
                               uint8_t* img, float* ss, float* x_out, cudaStream_t s) {
    const uint64_t items = (uint64_t)T * (K / 32);
    if (items == 0) return cudaSuccess;
    return launch_pdl(token_image_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0, s, false, src, tokens, w, T,
                      K, img, ss, x_out);
}

int ensure_prefill_buffers(bt_engine* e) {
    if (e->pf_cap) return BT_OK;
    const auto& c = e->lc;
    const size_t cap = kPrefillChunk, D = c.dim, F = c.hidden_dim, Q = qd(c);
    auto& A = e->allocs;
    BT_TRY_ALLOC(A, &e->pf_x, cap * D, "prefill x");
    BT_TRY_ALLOC(A, &e->pf_q, cap * Q, "prefill q");
    BT_TRY_ALLOC(A, &e->pf_attn, cap * Q, "prefill attention");
    BT_TRY_ALLOC(A, &e->pf_act, cap * F, "prefill act");
    BT_TRY_ALLOC(A, &e->pf_ss, cap * (D / 32), "prefill norm sums");
    const uint32_t k0 = (uint32_t)std::max(D, Q), k1 = (uint32_t)std::max(F, Q);
    BT_TRY_ALLOC(A, &e->pf_img[0], token_image_bytes((uint32_t)cap, k0), "prefill token image");
    BT_TRY_ALLOC(A, &e->pf_img[1], token_image_bytes((uint32_t)cap, k1), "prefill token image");
    BT_TRY_ALLOC(A, &e->pf_tok, cap, "prefill tokens");
    BT_TRY_ALLOC(A, &e->pf_pos, cap, "prefill positions");
    e->pf_part_floats = gemm_split_floats(e->num_sms);
    BT_TRY_ALLOC(A, &e->pf_part, e->pf_part_floats, "prefill GEMM split partials");
    e->pf_cap = (uint32_t)cap;
    return BT_OK;
}

template <typename KVT>
int prefill_chunk_t(bt_engine* e, const CacheRef& kv, uint32_t T, uint32_t pos0, cudaStream_t s) {
    const auto& c = e->lc;
    const uint32_t D = c.dim, F = c.hidden_dim, Q = qd(c), KV = kvd(c), hd = c.head_dim;
    const uint32_t QKV = Q + 2 * KV, L = c.num_layers, nsm = e->num_sms;
    uint32_t* err = kv.err;
    const float scale = 1.0f / std::sqrt((float)hd);
    // GEMM inputs with the split-K workspace (used by short chunks: fewer units than SMs)
    auto gin = [&](const uint8_t* img, const float* ss, float eps) {
        GemmIn g{img, ss, eps, T};
        g.part = e->pf_part;
        g.part_floats = e->pf_part_floats;
        return g;
    };
    positions_kernel<<<(T + 255) / 256, 256, 0, s>>>(e->pf_pos, T, pos0);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    BT_CUDA_CHECK(cudaGetLastError());
    // layer 0 input: the embedding rows (also the residual stream) times attn_norm
    BT_CUDA_CHECK(launch_token_image(e->embed, e->pf_tok, e->layers[0].attn_norm, T, D, e->pf_img[0], e->pf_ss,
                                     e->pf_x, s));
    for (uint32_t l = 0; l < L; ++l) {
        const LayerDev& Ld = e->layers[l];
        KVT* kl = static_cast<KVT*>(kv.k) + l * kv.layer_stride;
        KVT* vl = static_cast<KVT*>(kv.v) + l * kv.layer_stride;
        // qkv + RoPE + K/V append
        {
            GEpiQKV<KVT> epi{e->pf_q, kl, vl, kv.map, kv.rope, GemmTok{T, e->pf_pos, nullptr}, Q, KV, hd};
            BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.qkv, QKV, unit_rows(QKV), D},
                                             gin(e->pf_img[0], e->pf_ss, c.rms_norm_eps), epi, err, nsm, s));
        }
        // causal attention over the cache, then the o-proj input's token image
        BT_CUDA_CHECK(launch_prefill_attn<KVT>(e->pf_q, kl, vl, e->pf_attn, T, pos0, c.num_heads,
                                               c.num_heads / c.num_kv_heads, hd, kv.map, scale, s));
        BT_CUDA_CHECK(launch_token_image(e->pf_attn, nullptr, nullptr, T, Q, e->pf_img[1], nullptr, nullptr, s));
        // o-proj + residual; token image of x * ffn_norm
        BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.o, D, unit_rows(D), Q}, gin(e->pf_img[1], nullptr, 0.0f),
                                         GEpiResidual{e->pf_x, Ld.ffn_norm, e->pf_img[0], e->pf_ss, nullptr, D}, err,
                                         nsm, s));
        // gate/up + SwiGLU; token image of act
        BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.gu, 2 * F, unit_rows(2 * F), D},
                                         gin(e->pf_img[0], e->pf_ss, c.rms_norm_eps),
                                         GEpiSwiGLU{e->pf_act, e->pf_img[1], F}, err, nsm, s));
        // down + residual; token image of x * the next layer's attn_norm (the last layer's output
        // is not used: the decode step processes the final prompt token)
        const float* wn = l + 1 < L ? e->layers[l + 1].attn_norm : e->out_norm;
        BT_CUDA_CHECK(launch_gemm_tokens(UnitW{Ld.d, D, unit_rows(D), F}, gin(e->pf_img[1], nullptr, 0.0f),
                                         GEpiResidual{e->pf_x, wn, e->pf_img[0], e->pf_ss, nullptr, D}, err, nsm,
                                         s));
    }
    return BT_OK;
}

template int prefill_chunk_t<float>(bt_engine*, const CacheRef&, uint32_t, uint32_t, cudaStream_t);
template int prefill_chunk_t<__half>(bt_engine*, const CacheRef&, uint32_t, uint32_t, cudaStream_t);

// Workspace of gemm_units_launch: the token image, then the split-K partials.
static size_t image_part_offset(uint32_t K, uint32_t T) { return (token_image_bytes(T, K) + 255) / 256 * 256; }

cudaError_t gemm_units_launch(const void* units, const float* X, float* Y, uint32_t M, uint32_t K, uint32_t T,
                              uint8_t* ws, uint32_t* err, uint32_t nsm, cudaStream_t s) {
    cudaError_t ce = launch_token_image(X, nullptr, nullptr, T, K, ws, nullptr, nullptr, s);
    if (ce != cudaSuccess) return ce;
    GemmIn in{ws, nullptr, 0.0f, T};
    in.part = reinterpret_cast<float*>(ws + image_part_offset(K, T));
    in.part_floats = gemm_split_floats(nsm);
    return launch_gemm_tokens(UnitW{static_cast<const uint8_t*>(units), M, unit_rows(M), K}, in, GEpiStore{Y, M}, err,
                              nsm, s);
}

size_t gemm_units_scratch(uint32_t K, uint32_t T, uint32_t nsm) {
    return image_part_offset(K, T) + gemm_split_floats(nsm) * sizeof(float);
}

}  // namespace bt

extern "C" {

int bt_engine_prefill(bt_engine* e, bt_kv* kv, const uint32_t* prompt, uint32_t n_prompt, uint32_t pos0) {
    if (!e || !kv) return fail(BT_ERR_INVALID_ARGUMENT, "prefill: null engine or KV cache");
    if (!e->loaded) return fail(BT_ERR_RUNTIME, "engine has no weights (call bt_engine_load or bt_engine_generate)");
    if (kv->e != e) return fail(BT_ERR_INVALID_ARGUMENT, "KV cache belongs to another engine");
    if (!prompt || n_prompt == 0) return fail(BT_ERR_INVALID_ARGUMENT, "prefill: empty prompt");
    if ((uint64_t)pos0 + n_prompt > kv->max_seq) return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] >= e->cfg.vocab_size) return fail(BT_ERR_OUT_OF_RANGE, "Token ID out of vocab bounds");
    if (e->tp_world > 1) return fail(BT_ERR_INVALID_ARGUMENT, "prefill: not available under tensor parallelism");
    if (!(e->use_step && e->step_ok))
        return fail(BT_ERR_INVALID_ARGUMENT, "prefill: the engine does not run the persistent step kernel");
    DeviceGuard guard(e->device);
    int rc = ensure_prefill_buffers(e);
    if (rc != BT_OK) return rc;
    cudaStream_t s = e->stream;
    // a fresh error flag for the chunks' bounded waits
    BT_CUDA_CHECK(cudaMemsetAsync(&kv->st->error, 0, sizeof(uint32_t), s));
    const uint32_t n_fill = n_prompt - 1;  // the last prompt token goes through the decode step
    for (uint32_t done = 0; done < n_fill;) {
        const uint32_t T = std::min(n_fill - done, e->pf_cap);
        BT_CUDA_CHECK(cudaMemcpyAsync(e->pf_tok, prompt + done, sizeof(uint32_t) * T, cudaMemcpyHostToDevice, s));
        const CacheRef cr{kv->k, kv->v, kv->rope, kv->max_seq, &kv->st->error,
                          kv_map_flat(kv->max_seq, e->lc.head_dim),
                          (size_t)e->lc.num_kv_heads * kv->max_seq * e->lc.head_dim};
        rc = kv->dtype == BT_KV_FP16 ? prefill_chunk_t<__half>(e, cr, T, pos0 + done, s)
                                     : prefill_chunk_t<float>(e, cr, T, pos0 + done, s);
        if (rc != BT_OK) return rc;
        BT_CUDA_CHECK(cudaStreamSynchronize(s));  // pf_tok is refilled from the host by the next chunk
        done += T;
    }
    uint32_t flag = 0;
    BT_CUDA_CHECK(cudaMemcpy(&flag, &kv->st->error, sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag) return fail(BT_ERR_DEVICE_TIMEOUT, "prefill: a device wait timed out");
    // the sequence state as after n_prompt - 1 decode steps of bt_engine_begin(prompt, pos0)
    BT_CUDA_CHECK(cudaMemcpyAsync(kv->tok_hist + pos0, prompt, sizeof(uint32_t) * n_prompt, cudaMemcpyHostToDevice, s));
    DevState* h = kv->h_st;
    std::memset(h, 0, sizeof(DevState));
    h->pos = pos0 + n_fill;
    h->cur_token = prompt[n_fill];
    h->n_fixed = pos0 + n_prompt;
    BT_CUDA_CHECK(cudaMemcpyAsync(kv->st, h, sizeof(DevState), cudaMemcpyHostToDevice, s));
    BT_CUDA_CHECK(cudaMemsetAsync(kv->step_cnt, 0, sizeof(uint32_t) * (5 * e->cfg.num_layers + 1), s));
    BT_CUDA_CHECK(cudaStreamSynchronize(s));
    kv->host_pos = pos0 + n_fill;
    return BT_OK;
}

int bt_kv_read_tokens(bt_kv* kv, uint32_t pos0, uint32_t n, uint32_t* out) {
    if (!kv || (!out && n)) return fail(BT_ERR_INVALID_ARGUMENT, "read_tokens: null argument");
    if (!kv->e) return fail(BT_ERR_INVALID_ARGUMENT, "KV cache outlived its engine");
    if ((uint64_t)pos0 + n > (uint64_t)kv->max_seq + 1) return fail(BT_ERR_OUT_OF_RANGE, "read_tokens: past max_seq");
    DeviceGuard guard(kv->e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(kv->e->stream));
    if (n) BT_CUDA_CHECK(cudaMemcpy(out, kv->tok_hist + pos0, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost));
    return BT_OK;
}

int bt_cuda_gemm_q8_units(const void* units, const float* X, float* Y, uint32_t M, uint32_t K, uint32_t T,
                          void* stream) {
    BT_CHECK_ARG(K % 32 == 0 && K > 0, "gemm_q8_units: K must be a positive multiple of 32");
    BT_CHECK_ARG(units && X && Y, "gemm_q8_units: null buffer");
    BT_CHECK_ARG(((uintptr_t)units & 15) == 0 && ((uintptr_t)X & 15) == 0,
                 "gemm_q8_units: units and X must be 16-byte aligned");
    if (M == 0 || T == 0) return BT_OK;
    cudaStream_t s = as_stream(stream);
    int dev = 0, nsm = 0;
    BT_CUDA_CHECK(cudaGetDevice(&dev));
    BT_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    // token image and split-K partials, then the error flag; stream-ordered
    const size_t img_bytes = gemm_units_scratch(K, T, (uint32_t)nsm);
    uint8_t* ws = nullptr;
    BT_CUDA_CHECK(cudaMallocAsync(reinterpret_cast<void**>(&ws), img_bytes + 256, s));
    uint32_t* err = reinterpret_cast<uint32_t*>(ws + img_bytes);
    cudaError_t ce = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
    if (ce == cudaSuccess) ce = gemm_units_launch(units, X, Y, M, K, T, ws, err, (uint32_t)nsm, s);
    uint32_t flag = 0;
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&flag, err, sizeof(flag), cudaMemcpyDeviceToHost, s);
    const cudaError_t ce2 = cudaFreeAsync(ws, s);
    if (ce == cudaSuccess) ce = ce2;
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) return fail(BT_ERR_CUDA, std::string("gemm_q8_units: ") + cudaGetErrorString(ce));
    if (flag) return fail(BT_ERR_DEVICE_TIMEOUT, "gemm_q8_units: a device wait timed out; the output is not valid");
    return BT_OK;
}

}  // extern "C"
