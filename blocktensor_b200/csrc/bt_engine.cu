// bt_engine.cu -- the device-resident single-token decode engine.
//
// Replaces TransformerEngine::forward_single_token
// (runtime/src/transformer_engine.cpp:228-251) for the CUDA backend.  One
// token is 5 launches per layer plus one for the head, captured once in a
// CUDA graph and replayed with the position and token in device memory:
//
//   qkv   : RMSNorm(x) -> [Wq;Wk;Wv] GEMV -> RoPE -> q, K/V cache append   (:117-146)
//   attn  : split-K flash-decode over the cache, last CTA per KV head combines (:148-184)
//   oproj : Wo GEMV -> x += o                                             (:186-195)
//   gateup: RMSNorm(x) -> [Wg;Wu] GEMV -> silu(g)*u                       (:197-215)
//   down  : Wd GEMV -> x += d                                             (:217-225)
//   head  : RMSNorm(x) -> Whead GEMV -> logits, greedy argmax, next token (:244-250)
//
// Layer 0's qkv reads the embedding row of the current token directly
// (:233-238) instead of copying the whole table to the host.
#include "bt_common.cuh"
#include "bt_gemv.cuh"
#include "bt_gemv_mma.cuh"
#include "bt_attention.cuh"
#include "bt_step.cuh"
#include "bt_internal.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

using namespace bt;

#include "bt_engine_impl.h"

namespace {

int validate_config(const bt_model_config& c) {
    if (c.vocab_size == 0 || c.dim == 0 || c.hidden_dim == 0 || c.num_layers == 0 || c.num_heads == 0 ||
        c.num_kv_heads == 0 || c.head_dim == 0)
        return fail(BT_ERR_INVALID_ARGUMENT, "model config: zero-sized dimension");
    if (c.dim % 32 || c.hidden_dim % 32)
        return fail(BT_ERR_INVALID_ARGUMENT, "model config: dim and hidden_dim must be multiples of 32 (Q8_0 blocks)");
    if (c.num_heads * c.head_dim != c.dim)
        return fail(BT_ERR_INVALID_ARGUMENT, "model config: num_heads * head_dim must equal dim");
    if (c.num_heads % c.num_kv_heads)
        return fail(BT_ERR_INVALID_ARGUMENT, "model config: num_heads must be a multiple of num_kv_heads");
    if (c.head_dim % 2 || c.head_dim > 256)
        return fail(BT_ERR_INVALID_ARGUMENT, "model config: head_dim must be even and <= 256");
    if (c.num_heads / c.num_kv_heads > 16)
        return fail(BT_ERR_INVALID_ARGUMENT, "model config: at most 16 query heads per KV head");
    if (c.dim > 48 * 1024 || c.hidden_dim > 48 * 1024)
        return fail(BT_ERR_INVALID_ARGUMENT, "model config: dim/hidden_dim above 49152 not supported");
    return BT_OK;
}

// Destination of each of the 9 per-layer tensors inside the fused device layout.
struct Slot {
    uint8_t* units;
    uint32_t rows, cols;  // of this rank's share
    RowMap map;
    uint32_t grow0;       // its first row in the model's tensor
    uint32_t gcols;       // columns of the model's tensor (its share: blocks cb0 .. cb0 + cols/32 - 1)
    uint32_t cb0;
};

// Tensor parallelism: q/k/v, gate and up split by output rows (whole heads,
// FFN rows), o and down by input columns (whole 32-blocks), so that o and
// down give partial sums of x that the ranks add.
Slot layer_slot(bt_engine* e, uint32_t l, int j) {
    const auto& c = e->lc;
    LayerDev& L = e->layers[l];
    const uint32_t D = c.dim, F = c.hidden_dim, KV = kvd(c), Q = qd(c), hd = c.head_dim, r = e->tp_rank;
    const uint32_t Fg = e->cfg.hidden_dim, Qg = qd(e->cfg);
    switch (j) {
        case 2: return {L.qkv, Q, D, RowMap{1, hd, 0, 0, 0}, r * Q, D, 0};
        case 3: return {L.qkv, KV, D, RowMap{1, hd, 0, 0, Q}, r * KV, D, 0};
        case 4: return {L.qkv, KV, D, RowMap{0, 0, 0, 0, Q + KV}, r * KV, D, 0};
        case 5: return {L.o, D, Q, RowMap{0, 0, 0, 0, 0}, 0, Qg, r * Q / 32};
        case 6: return {L.gu, F, D, RowMap{2, 0, 0, 0, 0}, r * F, D, 0};
        case 7: return {L.gu, F, D, RowMap{2, 0, 1, 0, 0}, r * F, D, 0};
        default: return {L.d, D, F, RowMap{0, 0, 0, 0, 0}, 0, Fg, r * F / 32};
    }
}

// Tile-layout matrix of M x K rows (padding rows zero).
int alloc_units(bt_engine* e, uint8_t** out, uint32_t M, uint32_t K, const char* what) {
    const uint64_t bytes = unit_bytes(M, K);
    int rc = dev_alloc(e->allocs, out, bytes, what);
    if (rc != BT_OK) return rc;
    BT_CUDA_CHECK(cudaMemsetAsync(*out, 0, bytes, e->stream));
    return BT_OK;
}

// Shape of the persistent step kernel: head dims per lane, ring depth, shared
// memory (ring + a scratch area for digits or attention partials).  Configs
// whose attention partials leave no room for a two-stage ring use the
// launch-per-kernel step.
int plan_step(bt_engine* e) {
    const auto& c = e->lc;
    const uint32_t hd = c.head_dim, GQ = c.num_heads / c.num_kv_heads;
    e->step_nv = hd <= 64 ? 2 : hd <= 128 ? 4 : 8;
    // phases 5 L + 1 < 1024: the phase index is the low 10 bits of the split partials' tags
    // (query heads per KV head beyond 16 / NV are taken in several passes over the keys)
    e->step_ok = hd % e->step_nv == 0 && 5 * c.num_layers + 1 < 1024;
    uint32_t kmax = c.dim > c.hidden_dim ? c.dim : c.hidden_dim;
    if (qd(c) > kmax) kmax = qd(c);
    const size_t img_bytes = mma_digit_bytes(kmax);  // digits + block factors
    size_t scratch = img_bytes;
    // attention: the warps' partials [9][GQ][hd + 2], then, 16-byte aligned, either q's
    // tensor-core fragments (grouped heads: 16 bytes per lane and k-step) or, after the key
    // loop, the split merge's (m, l, weight) of every head and split and the heads' totals
    const size_t frag = (size_t)32 * (hd / 8) * 16, merge = ((size_t)GQ * kAttnMaxSplits * 3 + GQ) * 4;
    const size_t attn = ((size_t)kDigitWarps * GQ * (hd + 2) * 4 + 15) / 16 * 16 + (frag > merge ? frag : merge);
    if (attn > scratch) scratch = attn;
    scratch = (scratch + 127) / 128 * 128;
    const size_t budget = 220 * 1024;
    if (scratch + 2 * kStageBytes > budget) e->step_ok = false;
    uint32_t ns = scratch < budget ? (uint32_t)((budget - scratch) / kStageBytes) : 0;
    if (ns > kMmaMaxRing) ns = kMmaMaxRing;
    e->step_ns = ns;
    e->step_xstride = mma_xstride(kmax);
    e->step_scratch_off = ns * kStageBytes;
    e->step_smem = (size_t)ns * kStageBytes + scratch;
    uint32_t cols = 32;
    while (cols < ns * kStageTiles * kTileCols) cols <<= 1;
    e->step_tmem = cols;
    if (const char* v = std::getenv("BT_STEP_KERNEL")) e->use_step = (v[0] != '0');
    if (const char* v = std::getenv("BT_STEP_PF")) {
        const long n = std::atol(v);
        if (n >= 0 && n <= 64) e->step_pf = (uint32_t)n;
    }
    if (const char* v = std::getenv("BT_STEP_MIN_TILES")) {
        const long n = std::atol(v);
        if (n >= 0 && n <= 4096) e->step_min_tiles = (uint32_t)n;
    }
    if (const char* v = std::getenv("BT_STEP_EVICT_FIRST")) {
        if (v[0] != '0') e->step_flags |= kStepFlagEvictFirst;
        else e->step_flags &= ~kStepFlagEvictFirst;
    }
    // the per-layer matrix table the kernel walks
    std::vector<StepLayer> tab(c.num_layers);
    const uint32_t D = c.dim, F = c.hidden_dim, Q = qd(c), QKV = Q + 2 * kvd(c);
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        const LayerDev& L = e->layers[l];
        tab[l].qkv = StepMat{L.qkv, QKV, unit_rows(QKV), D};
        tab[l].o = StepMat{L.o, D, unit_rows(D), Q};
        tab[l].gu = StepMat{L.gu, 2 * F, unit_rows(2 * F), D};
        tab[l].d = StepMat{L.d, D, unit_rows(D), F};
        tab[l].attn_norm = L.attn_norm;
        tab[l].ffn_norm = L.ffn_norm;
    }
    BT_TRY_ALLOC(e->allocs, &e->d_layers, c.num_layers, "step layer table");
    for (int i = 0; i < 2; ++i) {
        BT_TRY_ALLOC(e->allocs, &e->step_img[i], img_bytes, "step digit image");
        BT_TRY_ALLOC(e->allocs, &e->step_ssp[i], (c.dim + kTileRows - 1) / kTileRows, "step norm partials");
    }
    BT_CUDA_CHECK(cudaMemcpyAsync(e->d_layers, tab.data(), sizeof(StepLayer) * c.num_layers, cudaMemcpyHostToDevice,
                                  e->stream));
    BT_CUDA_CHECK(cudaStreamSynchronize(e->stream));
    return BT_OK;
}

template <int NV, int GQM, typename KVT>
cudaError_t launch_step_t(const StepArgs& a, uint32_t grid, size_t smem, cudaStream_t s) {
    auto kern = decode_step_kernel<NV, GQM, KVT>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_set[dev]) {
        cudaError_t ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (ce != cudaSuccess) return ce;
        int blocks = 0;
        ce = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, kMmaThreads, smem);
        if (ce != cudaSuccess) return ce;
        if (blocks < 1) return cudaErrorCooperativeLaunchTooLarge;
        attr_set[dev] = true;
    }
    if (g_dry_run) return cudaSuccess;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// One decode step as one cooperative launch of the persistent kernel.
int launch_step(bt_engine* e, bt_kv* kv, cudaStream_t s) {
    const auto& c = e->lc;
    if (e->tp_world > 1 && !e->tp_ready)
        return fail(BT_ERR_INVALID_ARGUMENT, "tensor parallel engine: bt_engine_tp_connect has not been called");
    StepArgs a{};
    a.layers = e->d_layers;
    a.head = StepMat{e->head, c.vocab_size, unit_rows(c.vocab_size), c.dim};
    a.embed = e->embed;
    a.out_norm = e->out_norm;
    a.x = e->x;
    a.q = e->q;
    a.attn = e->attn;
    a.act = e->act;
    a.logits = e->logits;
    a.taps = e->taps_on ? e->taps : nullptr;
    a.kc = kv->k;
    a.vc = kv->v;
    a.rope = kv->rope;
    a.st = kv->st;
    a.tok_hist = kv->tok_hist;
    a.split_part = reinterpret_cast<uint64_t*>(e->split_part);
    a.am_val = e->am_val;
    a.am_idx = e->am_idx;
    a.am_ticket = e->am_ticket;
    a.att_part = kv->step_att_part;
    a.cnt = kv->step_cnt;
    for (int i = 0; i < 2; ++i) {
        a.dimg[i] = e->step_img[i];
        a.ssp[i] = e->step_ssp[i];
    }
    a.L = c.num_layers;
    a.D = c.dim;
    a.DQ = qd(c);
    a.v0 = e->v0;
    a.tp_xch = e->tp_peers;
    a.tp_rank = e->tp_rank;
    a.tp_world = e->tp_world;
    a.F = c.hidden_dim;
    a.KVD = kvd(c);
    a.hd = c.head_dim;
    a.KVH = c.num_kv_heads;
    a.GQ = c.num_heads / c.num_kv_heads;
    a.max_seq = kv->max_seq;
    a.S_att = kv->step_S;
    a.eps = c.rms_norm_eps;
    a.scale = 1.0f / std::sqrt((float)c.head_dim);
    a.NS = e->step_ns;
    a.xstride = e->step_xstride;
    a.tmem_cols = e->step_tmem;
    a.scratch_off = e->step_scratch_off;
    a.pf_stages = e->step_pf;
    a.min_tiles = e->step_min_tiles;
    a.flags = e->step_flags;
    a.trace = e->trace;
    const uint32_t grid = e->num_sms;
    cudaError_t ce;
    const bool f16 = kv->dtype == BT_KV_FP16;
    // query heads per KV head: 1 (multi-head) or up to 16 / NV (grouped-query)
    const bool mha = a.GQ == 1;
#define BT_STEP_LAUNCH(NV_)                                                                                      \
    ce = mha ? (f16 ? launch_step_t<NV_, 1, __half>(a, grid, e->step_smem, s)                                   \
                    : launch_step_t<NV_, 1, float>(a, grid, e->step_smem, s))                                   \
             : (f16 ? launch_step_t<NV_, 16 / NV_, __half>(a, grid, e->step_smem, s)                            \
                    : launch_step_t<NV_, 16 / NV_, float>(a, grid, e->step_smem, s))
    switch (e->step_nv) {
        case 2: BT_STEP_LAUNCH(2); break;
        case 4: BT_STEP_LAUNCH(4); break;
        default: BT_STEP_LAUNCH(8); break;
    }
#undef BT_STEP_LAUNCH
    BT_CUDA_CHECK(ce);
    return BT_OK;
}

bool step_path(const bt_engine* e) { return e->use_step && e->step_ok; }

int alloc_weights(bt_engine* e) {
    const auto& c = e->lc;
    const size_t D = c.dim, F = c.hidden_dim, KV = kvd(c), V = c.vocab_size, Q = qd(c);
    auto& A = e->allocs;
    BT_TRY_ALLOC(A, &e->embed, (size_t)e->cfg.vocab_size * D, "embed");  // every token's row on every rank
    BT_TRY_ALLOC(A, &e->out_norm, D, "out_norm");
    int rc = alloc_units(e, &e->head, (uint32_t)V, (uint32_t)D, "head");
    if (rc != BT_OK) return rc;
    e->layers.resize(c.num_layers);
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        LayerDev& L = e->layers[l];
        if ((rc = alloc_units(e, &L.qkv, (uint32_t)(Q + 2 * KV), (uint32_t)D, "wqkv"))) return rc;
        if ((rc = alloc_units(e, &L.o, (uint32_t)D, (uint32_t)Q, "wo"))) return rc;
        if ((rc = alloc_units(e, &L.gu, (uint32_t)(2 * F), (uint32_t)D, "wgu"))) return rc;
        if ((rc = alloc_units(e, &L.d, (uint32_t)D, (uint32_t)F, "wd"))) return rc;
        BT_TRY_ALLOC(A, &L.attn_norm, D, "attn_norm");
        BT_TRY_ALLOC(A, &L.ffn_norm, D, "ffn_norm");
    }
    BT_TRY_ALLOC(A, &e->x, D, "x");
    BT_TRY_ALLOC(A, &e->q, Q, "q");
    BT_TRY_ALLOC(A, &e->attn, Q, "attn");
    BT_TRY_ALLOC(A, &e->act, F, "act");
    BT_TRY_ALLOC(A, &e->logits, V, "logits");
    BT_TRY_ALLOC(A, &e->taps, (size_t)c.num_layers * D, "taps");
    const size_t nblk = V + 1;  // one partial per CTA, at least one row per CTA
    BT_TRY_ALLOC(A, &e->am_val, nblk, "argmax val");
    BT_TRY_ALLOC(A, &e->am_idx, nblk, "argmax idx");
    BT_TRY_ALLOC(A, &e->am_ticket, 4, "argmax ticket");
    BT_CUDA_CHECK(cudaMemsetAsync(e->am_ticket, 0, 16, e->stream));
    // split scratch of the GEMVs: partials [SM][2][128], one ticket per row tile of the tallest matrix
    uint32_t rows = (uint32_t)V;
    if (2 * F > rows) rows = (uint32_t)(2 * F);
    if (Q + 2 * KV > rows) rows = (uint32_t)(Q + 2 * KV);
    if (D > rows) rows = (uint32_t)D;
    const size_t tickets = mma_row_tiles(unit_rows(rows));
    // floats for the standalone GEMVs; (tag, value) words for the step kernel, zeroed (tag 0 is never valid)
    BT_TRY_ALLOC(A, &e->split_part, (size_t)e->num_sms * 2 * kTileRows * 2, "split partials");
    BT_CUDA_CHECK(cudaMemsetAsync(e->split_part, 0, sizeof(float) * e->num_sms * 2 * kTileRows * 2, e->stream));
    BT_TRY_ALLOC(A, &e->split_ticket, tickets, "split tickets");
    BT_CUDA_CHECK(cudaMemsetAsync(e->split_ticket, 0, sizeof(uint32_t) * tickets, e->stream));
    return plan_step(e);
}

void drop_graphs_of(bt_kv* kv) {
    if (kv->graph) {
        cudaGraphExecDestroy(kv->graph);
        kv->graph = nullptr;
    }
}

// Frees the device side of a cache (graph, buffers, pinned staging); the handle stays.
void release_kv_device(bt_kv* kv) {
    drop_graphs_of(kv);
    for (void* p : kv->allocs) cudaFree(p);
    kv->allocs.clear();
    if (kv->h_st) cudaFreeHost(kv->h_st);
    kv->h_st = nullptr;
    kv->k = kv->v = nullptr;
}

// Events recorded after every launch of a step (per-kernel profiling; no PDL).
struct Marks {
    cudaEvent_t* ev;
    int n;
};

#define BT_MARK()                                                   \
    do {                                                            \
        if (marks) BT_CUDA_CHECK(cudaEventRecord(marks->ev[marks->n++], s)); \
    } while (0)

// Enqueue one decode step (all launches) on stream s.
int enqueue_step(bt_engine* e, bt_kv* kv, cudaStream_t s, Marks* marks = nullptr) {
    const auto& c = e->cfg;
    const uint32_t D = c.dim, F = c.hidden_dim, KV = kvd(c), hd = c.head_dim;
    const uint32_t G = c.num_heads / c.num_kv_heads;
    const bool pdl = e->pdl && !marks;
    const uint32_t nsm = e->num_sms;
    const SplitScratch sp{e->split_part, e->split_ticket};
    const uint32_t QKV = D + 2 * KV;
    // the GEMV that follows each one, for the producer's L2 prefetch
    auto next = [&](const uint8_t* u, uint32_t M, uint32_t K) {
        return e->prefetch_bytes ? NextW{u, unit_rows(M), K, mma_grid(unit_rows(M), K, nsm), e->prefetch_bytes}
                                 : NextW{nullptr, 0, 0, 0, 0};
    };
    uint32_t* errp = &kv->st->error;
    const size_t kv_layer = (size_t)c.num_kv_heads * kv->max_seq * hd;
    const size_t esz = kv->dtype == BT_KV_FP16 ? 2 : 4;
    const float scale = 1.0f / std::sqrt((float)hd);
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        const LayerDev& L = e->layers[l];
        char* kl = static_cast<char*>(kv->k) + l * kv_layer * esz;
        char* vl = static_cast<char*>(kv->v) + l * kv_layer * esz;
        // qkv
        {
            const UnitW w{L.qkv, QKV, unit_rows(QKV), D};
            const NextW nx = next(L.o, D, D);
            MProNorm pro{e->x, L.attn_norm, c.rms_norm_eps, l == 0 ? e->embed : nullptr, kv->st, e->x};
            cudaError_t err;
            if (kv->dtype == BT_KV_FP16) {
                EpiQKV<__half> epi{e->q, reinterpret_cast<__half*>(kl), reinterpret_cast<__half*>(vl), kv->rope, kv->st,
                                   D, KV, hd, kv->max_seq};
                err = launch_gemv_mma(w, pro, SEpiQKV<__half>{epi}, sp, errp, nsm, s, pdl, nx);
            } else {
                EpiQKV<float> epi{e->q, reinterpret_cast<float*>(kl), reinterpret_cast<float*>(vl), kv->rope, kv->st,
                                  D, KV, hd, kv->max_seq};
                err = launch_gemv_mma(w, pro, SEpiQKV<float>{epi}, sp, errp, nsm, s, pdl, nx);
            }
            BT_CUDA_CHECK(err);
            BT_MARK();
        }
        // attention
        {
            AttnArgs a{e->q, kl, vl, e->attn, kv->att_part, kv->att_ticket + l * c.num_kv_heads, kv->st, errp,
                       hd, G, kv->max_seq, kv->lmax, 0, scale, (hd * esz) % 16 == 0 ? 1 : 0};
            cudaError_t err = kv->dtype == BT_KV_FP16 ? launch_attn<__half>(a, c.num_kv_heads, kv->splits, s, pdl)
                                                       : launch_attn<float>(a, c.num_kv_heads, kv->splits, s, pdl);
            BT_CUDA_CHECK(err);
            BT_MARK();
        }
        // o-proj + residual
        BT_CUDA_CHECK(launch_gemv_mma(UnitW{L.o, D, unit_rows(D), D}, MProCopy{e->attn}, SEpiResidual{e->x, nullptr}, sp,
                                      errp, nsm, s, pdl, next(L.gu, 2 * F, D)));
        BT_MARK();
        // gate/up + SwiGLU
        BT_CUDA_CHECK(launch_gemv_mma(UnitW{L.gu, 2 * F, unit_rows(2 * F), D},
                                      MProNorm{e->x, L.ffn_norm, c.rms_norm_eps, nullptr, nullptr, nullptr},
                                      SEpiSwiGLU{e->act}, sp, errp, nsm, s, pdl, next(L.d, D, F)));
        BT_MARK();
        // down + residual (+ tap)
        {
            float* tap = e->taps_on ? e->taps + (size_t)l * D : nullptr;
            const NextW nx = l + 1 < c.num_layers ? next(e->layers[l + 1].qkv, QKV, D) : next(e->head, c.vocab_size, D);
            BT_CUDA_CHECK(launch_gemv_mma(UnitW{L.d, D, unit_rows(D), F}, MProCopy{e->act}, SEpiResidual{e->x, tap}, sp,
                                          errp, nsm, s, pdl, nx));
            BT_MARK();
        }
    }
    {
        EpiLogits epi{e->logits, e->am_val, e->am_idx, e->am_ticket, kv->st, kv->tok_hist, kv->max_seq};
        BT_CUDA_CHECK(launch_gemv_mma(UnitW{e->head, c.vocab_size, unit_rows(c.vocab_size), D},
                                      MProNorm{e->x, e->out_norm, c.rms_norm_eps, nullptr, nullptr, nullptr},
                                      SEpiLogits{epi}, sp, errp, nsm, s, pdl, next(e->layers[0].qkv, QKV, D)));
        BT_MARK();
    }
    return BT_OK;
}

int ensure_graph(bt_engine* e, bt_kv* kv) {
    if (!e->use_graph) return BT_OK;
    if (kv->graph && kv->graph_taps == e->taps_on) return BT_OK;
    drop_graphs_of(kv);
    // configure every kernel of the step (shared-memory attributes) outside capture
    g_dry_run = true;
    int drc = enqueue_step(e, kv, e->stream);
    g_dry_run = false;
    if (drc != BT_OK) return drc;
    cudaGraph_t g = nullptr;
    BT_CUDA_CHECK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(e, kv, e->stream);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (rc != BT_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (ce != cudaSuccess) return fail(BT_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
    ce = cudaGraphInstantiate(&kv->graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) {
        kv->graph = nullptr;
        return fail(BT_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
    }
    kv->graph_taps = e->taps_on;
    return BT_OK;
}

int run_steps(bt_engine* e, bt_kv* kv, uint32_t n, cudaStream_t s) {
    if (kv->host_pos + n > kv->max_seq) return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    if (step_path(e)) {
        for (uint32_t i = 0; i < n; ++i) {
            int rc = launch_step(e, kv, s);
            if (rc != BT_OK) return rc;
            kv->host_pos += 1;
        }
        return BT_OK;
    }
    int rc = ensure_graph(e, kv);
    if (rc != BT_OK) return rc;
    for (uint32_t i = 0; i < n; ++i) {
        if (e->use_graph) {
            g_launches.fetch_add(5ull * e->cfg.num_layers + 1, std::memory_order_relaxed);
            BT_CUDA_CHECK(cudaGraphLaunch(kv->graph, s));
        } else {
            rc = enqueue_step(e, kv, s);
            if (rc != BT_OK) return rc;
        }
        kv->host_pos += 1;
    }
    return BT_OK;
}

int check_engine(bt_engine* e) {
    if (!e) return fail(BT_ERR_INVALID_ARGUMENT, "null engine");
    if (!e->loaded) return fail(BT_ERR_RUNTIME, "engine has no weights (call bt_engine_load or bt_engine_generate)");
    return BT_OK;
}

int check_kv(bt_engine* e, bt_kv* kv) {
    if (!kv) return fail(BT_ERR_INVALID_ARGUMENT, "null KV cache");
    if (kv->e != e) return fail(BT_ERR_INVALID_ARGUMENT, "KV cache belongs to another engine");
    return BT_OK;
}

}  // namespace

extern "C" {

int bt_engine_create(int device, const bt_model_config* cfg, const bt_engine_options* opt, bt_engine** out) {
    if (!cfg || !out) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_create: null argument");
    *out = nullptr;
    int rc = validate_config(*cfg);
    if (rc != BT_OK) return rc;
    int ndev = 0;
    BT_CUDA_CHECK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_create: bad device index");
    DeviceGuard guard(device);
    auto e = std::make_unique<bt_engine>();
    e->device = device;
    e->cfg = *cfg;
    e->lc = *cfg;
    if (opt && opt->rope_theta > 0.0f) e->theta = opt->rope_theta;
    if (opt && opt->tp_world > 1) {
        // tensor parallelism: rank tp_rank of tp_world takes whole heads, KV heads and 32-blocks of FFN
        // rows (o and down are split by these as input columns), and a contiguous slice of the vocab
        const uint32_t W = opt->tp_world, r = opt->tp_rank;
        if (W > kTpMaxWorld || r >= W)
            return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_create: tp_rank must be < tp_world <= 8");
        if (cfg->num_kv_heads % W || cfg->num_heads % W || (cfg->num_heads / W * cfg->head_dim) % 32 ||
            cfg->hidden_dim % (32 * W))
            return fail(BT_ERR_INVALID_ARGUMENT,
                        "bt_engine_create: tp_world must divide the KV heads, and each rank's query rows and FFN rows "
                        "must be whole 32-blocks");
        e->tp_rank = r;
        e->tp_world = W;
        e->lc.num_heads = cfg->num_heads / W;
        e->lc.num_kv_heads = cfg->num_kv_heads / W;
        e->lc.hidden_dim = cfg->hidden_dim / W;
        const uint32_t vl = (cfg->vocab_size + W - 1) / W;
        e->v0 = r * vl;
        e->lc.vocab_size = e->v0 < cfg->vocab_size ? std::min(vl, cfg->vocab_size - e->v0) : 0;
        if (e->lc.vocab_size == 0) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_create: tp_world above the vocab");
    }
    if (const char* v = std::getenv("BT_NO_PDL")) e->pdl = (v[0] == '0');
    if (const char* v = std::getenv("BT_NO_GRAPH")) e->use_graph = (v[0] == '0');
    if (const char* v = std::getenv("BT_GEMV_PREFETCH_KB")) {
        const long kb = std::atol(v);
        if (kb >= 0 && kb <= 1024) e->prefetch_bytes = (uint32_t)kb * 1024;
    }
    int nsm = 0;
    BT_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device));
    e->num_sms = nsm > 0 ? (uint32_t)nsm : 148;
    BT_CUDA_CHECK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    rc = alloc_weights(e.get());
    if (rc == BT_OK && e->tp_world > 1) {
        if (!step_path(e.get()))
            rc = fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_create: tensor parallelism needs the persistent step kernel");
        // exchange buffer: o-proj and down partials [2][tp_world][dim], then [tp_world][2] argmax words
        e->tp_bytes = sizeof(uint64_t) * (2 * (size_t)e->tp_world * cfg->dim + 2 * e->tp_world);
        cudaError_t ce = cudaSuccess;
        if (rc == BT_OK) ce = cudaMalloc(&e->tp_xbuf, e->tp_bytes);
        if (rc == BT_OK && ce == cudaSuccess) ce = cudaMemset(e->tp_xbuf, 0, e->tp_bytes);  // tag 0: never valid
        if (rc == BT_OK && ce == cudaSuccess) ce = cudaMalloc(&e->tp_peers, sizeof(uint64_t*) * e->tp_world);
        if (rc == BT_OK && ce != cudaSuccess) rc = fail(BT_ERR_CUDA, cudaGetErrorString(ce));
    }
    if (rc != BT_OK) {
        std::string msg = bt_cuda_last_error();
        bt_engine_destroy(e.release());
        set_error(msg);
        return rc;
    }
    *out = e.release();
    return BT_OK;
}

int bt_engine_tp_handle(bt_engine* e, void* handle) {
    if (!e || !handle) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_tp_handle: null argument");
    if (e->tp_world < 2) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_tp_handle: not a tensor parallel engine");
    DeviceGuard guard(e->device);
    cudaIpcMemHandle_t h;
    BT_CUDA_CHECK(cudaIpcGetMemHandle(&h, e->tp_xbuf));
    static_assert(sizeof(h) == BT_TP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    return BT_OK;
}

int bt_engine_tp_connect(bt_engine* e, const void* handles) {
    if (!e || !handles) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_tp_connect: null argument");
    if (e->tp_world < 2) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_tp_connect: not a tensor parallel engine");
    if (e->tp_ready) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_tp_connect: already connected");
    DeviceGuard guard(e->device);
    std::vector<uint64_t*> ptrs(e->tp_world, nullptr);
    for (uint32_t q = 0; q < e->tp_world; ++q) {
        if (q == e->tp_rank) {
            ptrs[q] = e->tp_xbuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)q * BT_TP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        const cudaError_t ce = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (ce != cudaSuccess) {
            for (void* o : e->tp_opened) cudaIpcCloseMemHandle(o);
            e->tp_opened.clear();
            return fail(BT_ERR_CUDA, std::string("bt_engine_tp_connect: rank ") + std::to_string(q) + ": " +
                                         cudaGetErrorString(ce));
        }
        e->tp_opened.push_back(p);
        ptrs[q] = static_cast<uint64_t*>(p);
    }
    BT_CUDA_CHECK(cudaMemcpy(e->tp_peers, ptrs.data(), sizeof(uint64_t*) * e->tp_world, cudaMemcpyHostToDevice));
    e->tp_ready = true;
    return BT_OK;
}

int bt_engine_destroy(bt_engine* e) {
    if (!e) return BT_OK;
    DeviceGuard guard(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    // caches still alive are detached: their device memory goes with the engine,
    // and a later bt_kv_destroy only frees the handle
    for (bt_kv* kv : e->kvs) {
        release_kv_device(kv);
        kv->e = nullptr;
    }
    e->kvs.clear();
    for (void* p : e->tp_opened) cudaIpcCloseMemHandle(p);
    if (e->tp_peers) cudaFree(e->tp_peers);
    if (e->tp_xbuf) cudaFree(e->tp_xbuf);
    for (void* p : e->allocs) cudaFree(p);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return BT_OK;
}

int bt_engine_load(bt_engine* e, const bt_tensor_view* t, uint32_t n, int on_device) {
    if (!e || !t) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_load: null argument");
    const auto& c = e->cfg;
    if (n != 3 + 9 * c.num_layers)
        return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_load: expected 3 + 9*num_layers tensors");
    DeviceGuard guard(e->device);
    const size_t D = c.dim, F = c.hidden_dim, KV = kvd(c), V = c.vocab_size;
    // Q8_0 (36-byte blocks) or Q4_0 (20-byte blocks, quant_types.hpp:17-20) matrices, told apart
    // by the head matrix's size; every matrix of a model has the same type (one quant_type per
    // .btmodel, model_importer.cpp:55-57)
    const size_t blk_bytes = (n > 2 && t[2].bytes == V * D / 32 * 20) ? 20 : 36;
    auto qbytes = [blk_bytes](size_t r, size_t k) { return r * k / 32 * blk_bytes; };
    // size checks (the reference reads raw sizes; a mismatch is a corrupt model)
    auto expect = [&](uint32_t i, size_t bytes, const char* what) -> int {
        if (t[i].bytes != bytes || (!t[i].data && bytes))
            return fail(BT_ERR_RUNTIME, std::string("bt_engine_load: tensor ") + std::to_string(i) + " (" + what +
                                            ") has " + std::to_string(t[i].bytes) + " bytes, expected " +
                                            std::to_string(bytes));
        return BT_OK;
    };
    int rc;
    if ((rc = expect(0, V * D * 4, "embed"))) return rc;
    if ((rc = expect(1, D * 4, "out_norm"))) return rc;
    if ((rc = expect(2, qbytes(V, D), "head"))) return rc;
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        const size_t sizes[9] = {D * 4, D * 4, qbytes(D, D), qbytes(KV, D), qbytes(KV, D), qbytes(D, D),
                                 qbytes(F, D), qbytes(F, D), qbytes(D, F)};
        for (int j = 0; j < 9; ++j)
            if ((rc = expect(3 + 9 * l + j, sizes[j], "layer tensor"))) return rc;
    }
    const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaStream_t s = e->stream;
    BT_CUDA_CHECK(cudaMemcpyAsync(e->embed, t[0].data, t[0].bytes, kind, s));
    BT_CUDA_CHECK(cudaMemcpyAsync(e->out_norm, t[1].data, t[1].bytes, kind, s));
    // staging buffer for 36-byte blocks (device copy when the source is on the host)
    size_t max_q = qbytes(V, D);
    for (size_t b : {qbytes(F, D), qbytes(D, F)}) max_q = b > max_q ? b : max_q;
    void* stage = nullptr;
    if (!on_device) BT_CUDA_CHECK(cudaMalloc(&stage, max_q));
    // this rank's rows (and, for o and down, its columns) of a tensor
    auto load_q = [&](const bt_tensor_view& tv, const Slot& sl) -> int {
        const size_t row_bytes = (size_t)sl.gcols / 32 * blk_bytes;
        const void* src = static_cast<const uint8_t*>(tv.data) + (size_t)sl.grow0 * row_bytes;
        if (!on_device) {
            BT_CUDA_CHECK(cudaMemcpyAsync(stage, src, (size_t)sl.rows * row_bytes, cudaMemcpyHostToDevice, s));
            src = stage;
        }
        if (blk_bytes == 20)
            BT_CUDA_CHECK(launch_pack_units_q4(src, sl.units, sl.rows, sl.cols, sl.map, s, sl.gcols / 32, sl.cb0));
        else
            BT_CUDA_CHECK(launch_pack_units(src, sl.units, sl.rows, sl.cols, sl.map, s, sl.gcols / 32, sl.cb0));
        if (!on_device) BT_CUDA_CHECK(cudaStreamSynchronize(s));  // stage is reused
        return BT_OK;
    };
    rc = load_q(t[2], Slot{e->head, e->lc.vocab_size, c.dim, RowMap{0, 0, 0, 0, 0}, e->v0, c.dim, 0});
    for (uint32_t l = 0; rc == BT_OK && l < c.num_layers; ++l) {
        LayerDev& L = e->layers[l];
        const bt_tensor_view* tl = t + 3 + 9 * l;
        cudaError_t ce = cudaMemcpyAsync(L.attn_norm, tl[0].data, tl[0].bytes, kind, s);
        if (ce == cudaSuccess) ce = cudaMemcpyAsync(L.ffn_norm, tl[1].data, tl[1].bytes, kind, s);
        if (ce != cudaSuccess) { rc = fail(BT_ERR_CUDA, cudaGetErrorString(ce)); break; }
        for (int j = 2; j < 9 && rc == BT_OK; ++j) rc = load_q(tl[j], layer_slot(e, l, j));
    }
    cudaError_t ce = cudaStreamSynchronize(s);
    if (stage) cudaFree(stage);
    if (rc != BT_OK) return rc;
    if (ce != cudaSuccess) return fail(BT_ERR_CUDA, std::string("bt_engine_load: ") + cudaGetErrorString(ce));
    e->loaded = true;
    return BT_OK;
}

int bt_engine_generate(bt_engine* e, uint64_t seed, float sigma) {
    if (!e) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_generate: null engine");
    DeviceGuard guard(e->device);
    const auto& c = e->cfg;
    const size_t D = c.dim, F = c.hidden_dim, KV = kvd(c), V = c.vocab_size;
    const float k = normal_k(sigma);
    cudaStream_t s = e->stream;
    // slabs of at most 32M elements: fp32 values, then their 36-byte blocks
    const size_t slab = 32u << 20;
    float* tmp = nullptr;
    void* blk = nullptr;
    BT_CUDA_CHECK(cudaMalloc(&tmp, slab * sizeof(float)));
    cudaError_t ce = cudaMalloc(&blk, slab / 32 * 36);
    if (ce != cudaSuccess) {
        cudaFree(tmp);
        return fail(BT_ERR_OUT_OF_MEMORY, "bt_engine_generate: staging allocation failed");
    }
    int rc = BT_OK;
    // this rank's rows of the model's tensor (whole rows generated, its columns packed)
    auto gen_q = [&](uint32_t stream_id, const Slot& sl) -> int {
        const size_t gcols = sl.gcols, rows = sl.rows;
        const size_t rows_per = slab / gcols;
        for (size_t r0 = 0; r0 < rows; r0 += rows_per) {
            const size_t nr = (rows - r0) < rows_per ? (rows - r0) : rows_per;
            BT_CUDA_CHECK(launch_gen_normal(seed, stream_id, (sl.grow0 + r0) * gcols, nr * gcols, k, tmp, s));
            BT_CUDA_CHECK(launch_quantize_q8_0(tmp, blk, nr * gcols / 32, s));
            RowMap mm = sl.map;
            mm.src_off = (uint32_t)r0;
            BT_CUDA_CHECK(launch_pack_units(blk, sl.units, (uint32_t)nr, sl.cols, mm, s, (uint32_t)(gcols / 32), sl.cb0));
        }
        return BT_OK;
    };
    ce = launch_gen_normal(seed, 0, 0, V * D, k, e->embed, s);
    if (ce == cudaSuccess) ce = launch_fill(e->out_norm, D, 1.0f, s);
    if (ce != cudaSuccess) rc = fail(BT_ERR_CUDA, cudaGetErrorString(ce));
    if (rc == BT_OK) rc = gen_q(2, Slot{e->head, e->lc.vocab_size, (uint32_t)D, RowMap{0, 0, 0, 0, 0}, e->v0, (uint32_t)D, 0});
    for (uint32_t l = 0; rc == BT_OK && l < c.num_layers; ++l) {
        LayerDev& L = e->layers[l];
        ce = launch_fill(L.attn_norm, D, 1.0f, s);
        if (ce == cudaSuccess) ce = launch_fill(L.ffn_norm, D, 1.0f, s);
        if (ce != cudaSuccess) { rc = fail(BT_ERR_CUDA, cudaGetErrorString(ce)); break; }
        for (int j = 2; j < 9 && rc == BT_OK; ++j) rc = gen_q(16 + 16 * l + j, layer_slot(e, l, j));
    }
    (void)KV; (void)F;
    ce = cudaStreamSynchronize(s);
    cudaFree(tmp);
    cudaFree(blk);
    if (rc != BT_OK) return rc;
    if (ce != cudaSuccess) return fail(BT_ERR_CUDA, std::string("bt_engine_generate: ") + cudaGetErrorString(ce));
    e->loaded = true;
    return BT_OK;
}

int bt_kv_create(bt_engine* e, uint32_t max_seq, int dtype, bt_kv** out) {
    if (!e || !out) return fail(BT_ERR_INVALID_ARGUMENT, "bt_kv_create: null argument");
    if (max_seq == 0) return fail(BT_ERR_INVALID_ARGUMENT, "bt_kv_create: max_seq must be > 0");
    if (dtype != BT_KV_FP32 && dtype != BT_KV_FP16) return fail(BT_ERR_INVALID_ARGUMENT, "bt_kv_create: bad kv dtype");
    *out = nullptr;
    DeviceGuard guard(e->device);
    const auto& c = e->lc;
    auto kv = std::make_unique<bt_kv>();
    kv->e = e;
    kv->max_seq = max_seq;
    kv->dtype = dtype;
    const size_t esz = dtype == BT_KV_FP16 ? 2 : 4;
    const size_t n = (size_t)c.num_layers * c.num_kv_heads * max_seq * c.head_dim;
    auto cleanup = [&](int rc) {
        std::string msg = bt_cuda_last_error();
        bt_kv_destroy(kv.release());
        set_error(msg);
        return rc;
    };
    int rc;
    uint8_t* kb = nullptr;
    uint8_t* vb = nullptr;
    if ((rc = dev_alloc(kv->allocs, &kb, n * esz, "K cache"))) return cleanup(rc);
    if ((rc = dev_alloc(kv->allocs, &vb, n * esz, "V cache"))) return cleanup(rc);
    kv->k = kb;
    kv->v = vb;
    const uint32_t half = c.head_dim / 2;
    if ((rc = dev_alloc(kv->allocs, &kv->rope, (size_t)max_seq * half, "rope table"))) return cleanup(rc);
    if ((rc = dev_alloc(kv->allocs, &kv->st, 1, "state"))) return cleanup(rc);
    if ((rc = dev_alloc(kv->allocs, &kv->tok_hist, (size_t)max_seq + 1, "token history"))) return cleanup(rc);
    // attention splits: >= 2 CTAs per SM over the KV heads, K+V tiles <= 32 KB per CTA
    attn_plan(c.num_kv_heads, c.head_dim, c.num_heads / c.num_kv_heads, max_seq, esz, e->num_sms, kv->splits,
              kv->lmax);
    const uint32_t S = kv->splits;
    if ((rc = dev_alloc(kv->allocs, &kv->att_part, (size_t)c.num_heads * S * (c.head_dim + 2), "attention partials")))
        return cleanup(rc);
    if ((rc = dev_alloc(kv->allocs, &kv->att_ticket, (size_t)c.num_layers * c.num_kv_heads, "attention tickets")))
        return cleanup(rc);
    // persistent step kernel: one attention item per (KV head, split), about one per SM, at most
    // kAttnMaxSplits splits per head (split 0's CTA merges the others' partials in split order)
    kv->step_S = e->num_sms / c.num_kv_heads;
    if (kv->step_S < 1) kv->step_S = 1;
    if (kv->step_S > kAttnMaxSplits) kv->step_S = kAttnMaxSplits;
    const uint32_t GQ = c.num_heads / c.num_kv_heads;
    if ((rc = dev_alloc(kv->allocs, &kv->step_cnt, (size_t)5 * c.num_layers + 1, "phase counters")))
        return cleanup(rc);
    if ((rc = dev_alloc(kv->allocs, &kv->step_att_part,
                        (size_t)c.num_kv_heads * GQ * kv->step_S * (c.head_dim + 2), "step attention partials")))
        return cleanup(rc);
    cudaError_t ce = cudaMemsetAsync(kv->att_ticket, 0, sizeof(uint32_t) * c.num_layers * c.num_kv_heads, e->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(kv->step_cnt, 0, sizeof(uint32_t) * (5 * c.num_layers + 1), e->stream);
    // tag 0 is never a valid tag: zeroed partials are never taken for a split's
    if (ce == cudaSuccess)
        ce = cudaMemsetAsync(kv->step_att_part, 0,
                             sizeof(uint64_t) * c.num_kv_heads * GQ * kv->step_S * (c.head_dim + 2), e->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(kb, 0, n * esz, e->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(vb, 0, n * esz, e->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(kv->st, 0, sizeof(DevState), e->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(kv->tok_hist, 0, sizeof(uint32_t) * (max_seq + 1), e->stream);
    if (ce != cudaSuccess) return cleanup(fail(BT_ERR_CUDA, cudaGetErrorString(ce)));
    // RoPE table with the reference formula (kernels/cpu_ref.hpp:40-43), host libm
    std::vector<float2> tab((size_t)max_seq * half);
    for (uint32_t i = 0; i < half; ++i) {
        const float freq = 1.0f / std::pow(e->theta, (float)(2 * i) / (float)c.head_dim);
        for (uint32_t p = 0; p < max_seq; ++p) {
            const float val = (float)p * freq;
            tab[(size_t)p * half + i] = make_float2(std::cos(val), std::sin(val));
        }
    }
    ce = cudaMemcpyAsync(kv->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, e->stream);
    if (ce == cudaSuccess) ce = cudaMallocHost(&kv->h_st, sizeof(DevState));
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
    if (ce != cudaSuccess) return cleanup(fail(BT_ERR_CUDA, cudaGetErrorString(ce)));
    e->kvs.push_back(kv.get());
    *out = kv.release();
    return BT_OK;
}

int bt_kv_destroy(bt_kv* kv) {
    if (!kv) return BT_OK;
    if (kv->e) {  // still attached: free its device memory and unregister it
        bt_engine* e = kv->e;
        DeviceGuard guard(e->device);
        cudaStreamSynchronize(e->stream);
        release_kv_device(kv);
        for (size_t i = 0; i < e->kvs.size(); ++i)
            if (e->kvs[i] == kv) {
                e->kvs.erase(e->kvs.begin() + (long)i);
                break;
            }
    }
    delete kv;
    return BT_OK;
}

int bt_kv_read_layer(bt_kv* kv, uint32_t layer, float* k, float* v) {
    if (!kv || !k || !v) return fail(BT_ERR_INVALID_ARGUMENT, "bt_kv_read_layer: null argument");
    if (!kv->e) return fail(BT_ERR_INVALID_ARGUMENT, "KV cache outlived its engine");
    bt_engine* e = kv->e;
    const auto& c = e->lc;  // this rank's KV heads
    if (layer >= c.num_layers) return fail(BT_ERR_OUT_OF_RANGE, "KVCache layer out of bounds");
    DeviceGuard guard(e->device);
    const size_t per = (size_t)c.num_kv_heads * kv->max_seq * c.head_dim;
    const size_t esz = kv->dtype == BT_KV_FP16 ? 2 : 4;
    std::vector<uint8_t> hk(per * esz), hv(per * esz);
    BT_CUDA_CHECK(cudaStreamSynchronize(e->stream));
    BT_CUDA_CHECK(cudaMemcpy(hk.data(), static_cast<uint8_t*>(kv->k) + layer * per * esz, per * esz, cudaMemcpyDeviceToHost));
    BT_CUDA_CHECK(cudaMemcpy(hv.data(), static_cast<uint8_t*>(kv->v) + layer * per * esz, per * esz, cudaMemcpyDeviceToHost));
    const uint32_t H = c.num_kv_heads, hd = c.head_dim, S = kv->max_seq;
    for (uint32_t h = 0; h < H; ++h)
        for (uint32_t p = 0; p < S; ++p)
            for (uint32_t d = 0; d < hd; ++d) {
                const size_t src = ((size_t)h * S + p) * hd + d, dst = ((size_t)p * H + h) * hd + d;
                if (esz == 2) {
                    k[dst] = __half2float(reinterpret_cast<const __half*>(hk.data())[src]);
                    v[dst] = __half2float(reinterpret_cast<const __half*>(hv.data())[src]);
                } else {
                    k[dst] = reinterpret_cast<const float*>(hk.data())[src];
                    v[dst] = reinterpret_cast<const float*>(hv.data())[src];
                }
            }
    return BT_OK;
}

int bt_engine_forward_token(bt_engine* e, bt_kv* kv, uint32_t token, uint32_t pos, float* logits, uint32_t* argmax) {
    int rc = check_engine(e);
    if (rc == BT_OK) rc = check_kv(e, kv);
    if (rc != BT_OK) return rc;
    if (token >= e->cfg.vocab_size) return fail(BT_ERR_OUT_OF_RANGE, "Token ID out of vocab bounds");
    if (pos >= kv->max_seq) return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    DeviceGuard guard(e->device);
    cudaStream_t s = e->stream;
    DevState* h = kv->h_st;
    std::memset(h, 0, sizeof(DevState));
    h->pos = pos;
    h->cur_token = token;
    h->n_fixed = 0;
    BT_CUDA_CHECK(cudaMemcpyAsync(kv->st, h, sizeof(DevState), cudaMemcpyHostToDevice, s));
    // the state's step count restarts at 0, and so do the phase counters
    BT_CUDA_CHECK(cudaMemsetAsync(kv->step_cnt, 0, sizeof(uint32_t) * (5 * e->cfg.num_layers + 1), s));
    kv->host_pos = pos;
    rc = run_steps(e, kv, 1, s);
    if (rc != BT_OK) return rc;
    if (logits)
        BT_CUDA_CHECK(cudaMemcpyAsync(logits + e->v0, e->logits, sizeof(float) * e->lc.vocab_size,
                                      cudaMemcpyDeviceToHost, s));  // this rank's vocab rows
    BT_CUDA_CHECK(cudaMemcpyAsync(h, kv->st, sizeof(DevState), cudaMemcpyDeviceToHost, s));
    BT_CUDA_CHECK(cudaStreamSynchronize(s));
    if (h->error) return fail(BT_ERR_DEVICE_TIMEOUT, "device wait timed out during the decode step");
    if (argmax) *argmax = h->last_argmax;
    return BT_OK;
}

int bt_engine_begin(bt_engine* e, bt_kv* kv, const uint32_t* prompt, uint32_t n_prompt, uint32_t pos0) {
    int rc = check_engine(e);
    if (rc == BT_OK) rc = check_kv(e, kv);
    if (rc != BT_OK) return rc;
    if (!prompt || n_prompt == 0) return fail(BT_ERR_INVALID_ARGUMENT, "decode: empty prompt");
    if ((uint64_t)pos0 + n_prompt > kv->max_seq) return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] >= e->cfg.vocab_size) return fail(BT_ERR_OUT_OF_RANGE, "Token ID out of vocab bounds");
    DeviceGuard guard(e->device);
    cudaStream_t s = e->stream;
    BT_CUDA_CHECK(cudaMemcpyAsync(kv->tok_hist + pos0, prompt, sizeof(uint32_t) * n_prompt, cudaMemcpyHostToDevice, s));
    DevState* h = kv->h_st;
    std::memset(h, 0, sizeof(DevState));
    h->pos = pos0;
    h->cur_token = prompt[0];
    h->n_fixed = pos0 + n_prompt;
    BT_CUDA_CHECK(cudaMemcpyAsync(kv->st, h, sizeof(DevState), cudaMemcpyHostToDevice, s));
    BT_CUDA_CHECK(cudaMemsetAsync(kv->step_cnt, 0, sizeof(uint32_t) * (5 * e->cfg.num_layers + 1), s));
    BT_CUDA_CHECK(cudaStreamSynchronize(s));
    kv->host_pos = pos0;
    return step_path(e) ? BT_OK : ensure_graph(e, kv);
}

int bt_engine_steps(bt_engine* e, bt_kv* kv, uint32_t n, void* stream) {
    int rc = check_engine(e);
    if (rc == BT_OK) rc = check_kv(e, kv);
    if (rc != BT_OK) return rc;
    DeviceGuard guard(e->device);
    return run_steps(e, kv, n, stream ? as_stream(stream) : e->stream);
}

int bt_engine_decode(bt_engine* e, bt_kv* kv, const uint32_t* prompt, uint32_t n_prompt, uint32_t pos0,
                     uint32_t n_gen, uint32_t* tokens_out) {
    if (!tokens_out) return fail(BT_ERR_INVALID_ARGUMENT, "decode: null tokens_out");
    if (kv && (uint64_t)pos0 + n_prompt + n_gen > kv->max_seq)
        return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    int rc = bt_engine_begin(e, kv, prompt, n_prompt, pos0);
    if (rc != BT_OK) return rc;
    DeviceGuard guard(e->device);
    rc = run_steps(e, kv, n_prompt + n_gen, e->stream);
    if (rc != BT_OK) return rc;
    BT_CUDA_CHECK(cudaMemcpyAsync(tokens_out, kv->tok_hist + pos0, sizeof(uint32_t) * (n_prompt + n_gen + 1),
                                  cudaMemcpyDeviceToHost, e->stream));
    BT_CUDA_CHECK(cudaMemcpyAsync(kv->h_st, kv->st, sizeof(DevState), cudaMemcpyDeviceToHost, e->stream));
    BT_CUDA_CHECK(cudaStreamSynchronize(e->stream));
    if (kv->h_st->error) return fail(BT_ERR_DEVICE_TIMEOUT, "device wait timed out during decode");
    return BT_OK;
}

int bt_engine_set_taps(bt_engine* e, int enable) {
    if (!e) return fail(BT_ERR_INVALID_ARGUMENT, "null engine");
    e->taps_on = enable != 0;
    return BT_OK;
}

int bt_engine_set_trace(bt_engine* e, int enable) {
    if (!e) return fail(BT_ERR_INVALID_ARGUMENT, "null engine");
    if (enable && !step_path(e)) return fail(BT_ERR_INVALID_ARGUMENT, "trace: the engine does not run the step kernel");
    DeviceGuard guard(e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(e->stream));
    if (enable && !e->trace) {
        size_t n = (size_t)(5 * e->lc.num_layers + 1) * e->num_sms * kTraceSlots;
#ifdef BT_STAGE_TRACE
        n += (size_t)e->num_sms * kStageTraceMax * kStageSlots;
#endif
        BT_TRY_ALLOC(e->allocs, &e->trace, n, "step trace");
        BT_CUDA_CHECK(cudaMemset(e->trace, 0, n * sizeof(uint64_t)));
    }
    if (!enable && e->trace) {
        for (size_t i = 0; i < e->allocs.size(); ++i)
            if (e->allocs[i] == e->trace) {
                e->allocs.erase(e->allocs.begin() + (long)i);
                break;
            }
        cudaFree(e->trace);
        e->trace = nullptr;
    }
    return BT_OK;
}

int bt_engine_read_trace(bt_engine* e, uint64_t* out, uint64_t n_words) {
    if (!e || !out) return fail(BT_ERR_INVALID_ARGUMENT, "null argument");
    if (!e->trace) return fail(BT_ERR_INVALID_ARGUMENT, "trace is off (bt_engine_set_trace)");
    uint64_t n = (uint64_t)(5 * e->lc.num_layers + 1) * e->num_sms * kTraceSlots;
#ifdef BT_STAGE_TRACE
    n += (uint64_t)e->num_sms * kStageTraceMax * kStageSlots;  // a stage-trace build: the stage timeline follows
#endif
    if (n_words != n) return fail(BT_ERR_INVALID_ARGUMENT, "read_trace: n_words does not match the trace size");
    DeviceGuard guard(e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(e->stream));
    BT_CUDA_CHECK(cudaMemcpy(out, e->trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    return BT_OK;
}

int bt_engine_read_taps(bt_engine* e, float* taps) {
    if (!e || !taps) return fail(BT_ERR_INVALID_ARGUMENT, "null argument");
    DeviceGuard guard(e->device);
    BT_CUDA_CHECK(cudaStreamSynchronize(e->stream));
    BT_CUDA_CHECK(cudaMemcpy(taps, e->taps, sizeof(float) * e->cfg.num_layers * e->cfg.dim, cudaMemcpyDeviceToHost));
    return BT_OK;
}

int bt_kv_step_info(bt_kv* kv, uint32_t context, uint64_t* launches, uint64_t* bytes) {
    if (!kv) return fail(BT_ERR_INVALID_ARGUMENT, "null KV cache");
    if (!kv->e) return fail(BT_ERR_INVALID_ARGUMENT, "KV cache outlived its engine");
    const auto& c = kv->e->lc;  // this rank's share
    const uint64_t D = c.dim, F = c.hidden_dim, KV = kvd(c), V = c.vocab_size, L = c.num_layers, Q = qd(c);
    const uint64_t params = L * (Q * D * 2 + KV * D * 2 + F * D * 3) + V * D;
    const uint64_t weight_bytes = params + params / 32 * 4;
    const uint64_t norms = 4 * D * (2 * L + 1);
    const uint64_t emb = 4 * D;
    const uint64_t esz = kv->dtype == BT_KV_FP16 ? 2 : 4;
    const uint64_t kv_bytes = 2 * L * KV * esz * ((uint64_t)context + 1);  // read c positions, write 1
    if (launches) *launches = step_path(kv->e) ? 1 : 5 * L + 1;
    if (bytes) *bytes = weight_bytes + norms + emb + kv_bytes;
    return BT_OK;
}

int bt_kv_state(bt_kv* kv, uint32_t* pos, uint32_t* token, uint32_t* last_argmax) {
    if (!kv) return fail(BT_ERR_INVALID_ARGUMENT, "null KV cache");
    if (!kv->e) return fail(BT_ERR_INVALID_ARGUMENT, "KV cache outlived its engine");
    DeviceGuard guard(kv->e->device);
    DevState h{};
    BT_CUDA_CHECK(cudaStreamSynchronize(kv->e->stream));
    BT_CUDA_CHECK(cudaMemcpy(&h, kv->st, sizeof(DevState), cudaMemcpyDeviceToHost));
    if (pos) *pos = h.pos;
    if (token) *token = h.cur_token;
    if (last_argmax) *last_argmax = h.last_argmax;
    if (h.error) return fail(BT_ERR_DEVICE_TIMEOUT, "device wait timed out during an earlier step");
    return BT_OK;
}

int bt_kv_inject_stall(bt_kv* kv) {
    if (!kv) return fail(BT_ERR_INVALID_ARGUMENT, "null KV cache");
    bt_engine* e = kv->e;
    if (!e) return fail(BT_ERR_INVALID_ARGUMENT, "KV cache outlived its engine");
    if (!step_path(e)) return fail(BT_ERR_INVALID_ARGUMENT, "inject_stall: the engine does not run the step kernel");
    DeviceGuard guard(e->device);
    // the step count 2^20: a phase's CTAs wait for G (2^20 + 1) arrivals while only G can come
    // (the signed difference stays negative for any grid below 2048 CTAs)
    const uint32_t far = 1u << 20;
    BT_CUDA_CHECK(cudaStreamSynchronize(e->stream));
    BT_CUDA_CHECK(cudaMemcpy(&kv->st->pad[0], &far, sizeof(far), cudaMemcpyHostToDevice));
    return BT_OK;
}

void* bt_engine_stream(bt_engine* e) { return e ? (void*)e->stream : nullptr; }

int bt_engine_profile(bt_engine* e, bt_kv* kv, uint32_t n_steps, float* ms_by_kind) {
    int rc = check_engine(e);
    if (rc == BT_OK) rc = check_kv(e, kv);
    if (rc != BT_OK) return rc;
    if (!ms_by_kind || n_steps == 0) return fail(BT_ERR_INVALID_ARGUMENT, "bt_engine_profile: bad argument");
    if (kv->host_pos + n_steps > kv->max_seq) return fail(BT_ERR_OUT_OF_RANGE, "KVCache pos out of bounds");
    DeviceGuard guard(e->device);
    const int per_step = 5 * (int)e->cfg.num_layers + 1;
    std::vector<cudaEvent_t> ev((size_t)per_step + 1);
    for (auto& x : ev) BT_CUDA_CHECK(cudaEventCreate(&x));
    for (int k = 0; k < 6; ++k) ms_by_kind[k] = 0.0f;
    cudaStream_t s = e->stream;
    for (uint32_t it = 0; it < n_steps && rc == BT_OK; ++it) {
        Marks m{ev.data() + 1, 0};
        cudaError_t ce = cudaEventRecord(ev[0], s);
        if (ce != cudaSuccess) { rc = fail(BT_ERR_CUDA, cudaGetErrorString(ce)); break; }
        g_launches.fetch_add((uint64_t)per_step, std::memory_order_relaxed);
        rc = enqueue_step(e, kv, s, &m);
        if (rc != BT_OK) break;
        kv->host_pos += 1;
        ce = cudaEventSynchronize(ev[per_step]);
        if (ce != cudaSuccess) { rc = fail(BT_ERR_CUDA, cudaGetErrorString(ce)); break; }
        for (int i = 0; i < per_step; ++i) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            const int kind = (i == per_step - 1) ? 5 : (i % 5);
            ms_by_kind[kind] += ms;
        }
    }
    for (auto& x : ev) cudaEventDestroy(x);
    return rc;
}

}  // extern "C"
