// cuda_engine.hpp -- blocktensor::CudaTransformerEngine: the device-resident
// replacement of TransformerEngine (runtime/include/blocktensor/transformer_engine.hpp:12-56)
// with the same constructor and forward_single_token signature.
//
// The reference engine runs device work only for backend_name() ==
// "Vulkan_Compute" (runtime/src/transformer_engine.cpp:55,75,102,123,201) and
// keeps attention, KV append, residual and SwiGLU on the host; this class runs
// the whole token on the GPU through bt_engine_forward_token.  Weights come
// from the TransformerWeights buffers: CudaBuffers are loaded device-to-device,
// any other buffers are read to the host first.  Each KVCache object seen is
// paired with a device cache of the same max_seq_len (fp32 by default, as
// runtime/src/kv_cache.cpp:9).  The pairing is by the identity of the
// KVCache's buffers (it holds them; they die with it), so a new KVCache that
// happens to reuse a destroyed one's address gets a fresh device cache.  The
// device cache is the one the kernels read and write; sync_to_reference copies
// it into the KVCache's own buffers for callers that read K/V through the
// reference object (k_cache / v_cache).
#pragma once

#include <cstdint>
#include <memory>
#include <unordered_map>
#include <vector>

#include "blocktensor/kv_cache.hpp"
#include "blocktensor/transformer_weights.hpp"
#include "bt_cuda.h"
#include "cuda_backend.hpp"

namespace blocktensor {

class CudaTransformerEngine {
public:
    CudaTransformerEngine(std::shared_ptr<IComputeBackend> backend, const TransformerWeights& weights,
                          float rope_theta = 10000.0f, int kv_dtype = BT_KV_FP32);
    ~CudaTransformerEngine();
    CudaTransformerEngine(const CudaTransformerEngine&) = delete;
    CudaTransformerEngine& operator=(const CudaTransformerEngine&) = delete;

    std::vector<float> forward_single_token(uint32_t token_id, uint32_t pos, KVCache& kv_cache);

    // Copies the device K/V of kv_cache's sequence into its reference buffers, layout
    // [max_seq][kv_heads][head_dim] fp32 per layer (runtime/src/kv_cache.cpp:21-23).
    void sync_to_reference(KVCache& kv_cache);

    // Greedy token of the last forward_single_token (sampling::sample_greedy of its logits).
    uint32_t last_argmax() const { return last_argmax_; }
    bt_engine* handle() const { return eng_; }

private:
    bt_kv* kv_for(const KVCache& kv);

    std::shared_ptr<IComputeBackend> backend_;
    ModelConfig cfg_;
    int device_ = 0;
    int kv_dtype_;
    bt_engine* eng_ = nullptr;
    struct KvBinding {
        std::weak_ptr<IComputeBuffer> k0;  // the KVCache's layer-0 K buffer: expires with the KVCache
        bt_kv* h = nullptr;
    };
    std::unordered_map<const KVCache*, KvBinding> kvs_;
    uint32_t last_argmax_ = 0;
};

}  // namespace blocktensor
