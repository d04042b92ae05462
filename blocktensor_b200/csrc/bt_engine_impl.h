// bt_engine_impl.h -- the engine and KV-cache objects behind the C ABI
// (bt_engine, bt_kv), shared by the decode engine (bt_engine.cu) and the
// prompt prefill (bt_prefill.cu).
#pragma once

#include "bt_common.cuh"
#include "bt_gemv.cuh"
#include "bt_step.cuh"

#include <string>
#include <vector>


// Matrices in the 4608-byte tile layout of bt_gemv_mma.cuh (rows padded to 128).
struct LayerDev {
    uint8_t* qkv;   // [D + 2 KVD] x D, q and k rows as RoPE pairs (i, i + hd/2) of each head
    uint8_t* o;     // D x D
    uint8_t* gu;    // 2F x D, (gate, up) rows interleaved
    uint8_t* d;     // D x F
    float* attn_norm;
    float* ffn_norm;
};

struct bt_engine {
    int device = 0;
    bt_model_config cfg{};  // the model
    // this GPU's share of it (tensor parallelism over tp_world GPUs; the whole model when 1):
    // heads, KV heads, FFN rows and head-matrix (vocab) rows of rank tp_rank, dim unchanged
    bt_model_config lc{};
    uint32_t tp_rank = 0, tp_world = 1;
    uint32_t v0 = 0;  // first vocab row of this rank
    uint64_t* tp_xbuf = nullptr;     // exchange buffer of this rank (own allocation, shared by IPC)
    size_t tp_bytes = 0;
    uint64_t** tp_peers = nullptr;   // [tp_world] every rank's exchange buffer as mapped here (device array)
    std::vector<void*> tp_opened;    // peer buffers opened by IPC
    bool tp_ready = false;
    float theta = 10000.0f;
    cudaStream_t stream = nullptr;
    bool pdl = true;
    bool use_graph = true;
    uint32_t prefetch_bytes = 98304;  // L2 prefetch of the next GEMV's weights, per CTA
    // persistent step kernel (one launch per token); the launch-per-kernel step stays for profiling
    bool use_step = true;
    bool step_ok = false;
    uint32_t step_nv = 0, step_ns = 0, step_xstride = 0, step_tmem = 0, step_scratch_off = 0;
    size_t step_smem = 0;
    bt::StepLayer* d_layers = nullptr;  // device copy of the per-layer matrix table
    uint8_t* step_img[2] = {nullptr, nullptr};  // digit images of GEMV inputs, by phase parity
    float* step_ssp[2] = {nullptr, nullptr};    // row-tile sums of x^2, by phase parity
    uint32_t num_sms = 148;
    // stages of L2 prefetch ahead of the ring while the consumers are held up (BT_STEP_PF; off by
    // default: measured slower on the 7B step, the prefetched weights evict the K/V rows attention reads)
    uint32_t step_pf = 0;
    // StepArgs::min_tiles: 32 tiles (4 stages) per CTA at least; the 7B-shaped o-proj at 1 GPU
    // (4096 tiles) then runs on 128 CTAs, each row tile in 4 aligned pieces (481 -> 486 tokens/s),
    // and under tensor parallelism the small per-rank matrices are cut into fewer pieces (4 GPUs:
    // 510 -> 671 tokens/s); BT_STEP_MIN_TILES overrides (0: every SM)
    uint32_t step_min_tiles = 32;
    uint32_t step_flags = 0;   // kStepFlag* options of the step kernel
    uint64_t* trace = nullptr; // per-phase timestamps of the last step ([5 L + 1][num_sms][kTraceSlots])
    bool taps_on = false;
    std::vector<void*> allocs;
    std::vector<LayerDev> layers;
    float* embed = nullptr;
    float* out_norm = nullptr;
    uint8_t* head = nullptr;  // V x D units
    // partial sums of row tiles cut between CTAs of a GEMV ([num_sms][2][128] floats, or 64-bit tagged
    // words in the step kernel) + one ticket per row tile (standalone GEMVs)
    float* split_part = nullptr;
    uint32_t* split_ticket = nullptr;
    // activations
    float* x = nullptr;
    float* q = nullptr;
    float* attn = nullptr;
    float* act = nullptr;
    float* logits = nullptr;
    float* taps = nullptr;
    // argmax scratch
    float* am_val = nullptr;
    uint32_t* am_idx = nullptr;
    uint32_t* am_ticket = nullptr;
    bool loaded = false;
    std::vector<bt_kv*> kvs;  // caches created on this engine and not yet destroyed
    // prompt prefill (bt_prefill.cu): token-major buffers for chunks of up to pf_cap tokens,
    // allocated on the first prefill
    uint32_t pf_cap = 0;
    float* pf_x = nullptr;      // [cap][D] residual stream
    float* pf_q = nullptr;      // [cap][DQ]
    float* pf_attn = nullptr;   // [cap][DQ]
    float* pf_act = nullptr;    // [cap][F]
    float* pf_ss = nullptr;     // [cap][D / 32] sums of squares of the next RMSNorm input
    uint8_t* pf_img[2] = {nullptr, nullptr};  // token images (K = D or DQ; K = F or DQ)
    uint32_t* pf_tok = nullptr; // [cap] token ids
    uint32_t* pf_pos = nullptr; // [cap] positions
    float* pf_part = nullptr;   // split-K partial sums of chunk GEMMs with fewer units than SMs
    size_t pf_part_floats = 0;
};

struct bt_kv {
    bt_engine* e = nullptr;
    uint32_t max_seq = 0;
    int dtype = BT_KV_FP32;
    std::vector<void*> allocs;
    void* k = nullptr;          // [L][KVH][max_seq][hd]
    void* v = nullptr;
    float2* rope = nullptr;     // [max_seq][hd/2]
    bt::DevState* st = nullptr;
    uint32_t* tok_hist = nullptr;  // [max_seq + 1]
    float* att_part = nullptr;
    uint32_t* att_ticket = nullptr;
    uint32_t splits = 1, lmax = 1;
    bt::DevState* h_st = nullptr;   // pinned staging
    uint64_t host_pos = 0;      // position of the next step, mirrored on the host for bounds checks
    cudaGraphExec_t graph = nullptr;
    bool graph_taps = false;
    // persistent step kernel: phase counters [5 L + 1], attention split partials and tickets
    uint32_t* step_cnt = nullptr;
    uint64_t* step_att_part = nullptr;  // tagged attention split partials of the step kernel
    uint32_t step_S = 1;
};

namespace bt {

// One sequence's KV cache as prefill sees it: K and V [L][KVH][max_seq][hd] (fp32 or
// fp16 by the engine call), the RoPE table, and the flag bounded waits set.
struct CacheRef {
    void* k;              // layer 0's K base (row addresses from map)
    void* v;
    const float2* rope;
    uint32_t max_seq;     // positions the sequence may hold
    uint32_t* err;
    KVMap map;            // rows of the sequence (index 0 of the map)
    size_t layer_stride;  // elements between two layers' bases
};

// Prompt prefill building blocks (bt_prefill.cu).
int ensure_prefill_buffers(bt_engine* e);
template <typename KVT>
int prefill_chunk_t(bt_engine* e, const CacheRef& kv, uint32_t T, uint32_t pos0, cudaStream_t s);
cudaError_t launch_token_image(const float* src, const uint32_t* tokens, const float* w, uint32_t T, uint32_t K,
                               uint8_t* img, float* ss, float* x_out, cudaStream_t s);

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

template <typename T>
int dev_alloc(std::vector<void*>& list, T** out, size_t count, const char* what) {
    void* p = nullptr;
    const size_t bytes = count * sizeof(T);
    cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(e == cudaErrorMemoryAllocation ? BT_ERR_OUT_OF_MEMORY : BT_ERR_CUDA,
                    std::string("cudaMalloc(") + what + ", " + std::to_string(bytes) + " B): " + cudaGetErrorString(e));
    }
    list.push_back(p);
    *out = static_cast<T*>(p);
    return BT_OK;
}

#define BT_TRY_ALLOC(list, ptr, count, what)                         \
    do {                                                             \
        int _rc = dev_alloc(list, ptr, count, what);                 \
        if (_rc != BT_OK) return _rc;                                \
    } while (0)

inline uint32_t kvd(const bt_model_config& c) { return c.num_kv_heads * c.head_dim; }
inline uint32_t qd(const bt_model_config& c) { return c.num_heads * c.head_dim; }  // query rows (dim without TP)


}  // namespace bt
