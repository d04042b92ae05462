// cuda_engine.cpp -- see cuda_engine.hpp.
#include "cuda_engine.hpp"

#include <cstring>
#include <stdexcept>

namespace blocktensor {

static_assert(sizeof(ModelConfig) == sizeof(bt_model_config), "ModelConfig layout");

CudaTransformerEngine::CudaTransformerEngine(std::shared_ptr<IComputeBackend> backend,
                                             const TransformerWeights& weights, float rope_theta, int kv_dtype)
    : backend_(std::move(backend)), cfg_(weights.config), kv_dtype_(kv_dtype) {
    if (!backend_) throw std::invalid_argument("CudaTransformerEngine: null backend");
    if (weights.quant_type != DataType::INT8 && weights.quant_type != DataType::INT4)
        throw std::invalid_argument("CudaTransformerEngine: weights must be INT8 (Q8_0) or INT4 (Q4_0)");
    if (auto cb = std::dynamic_pointer_cast<CudaBackend>(backend_)) device_ = cb->device();
    bt_model_config c;
    static_assert(sizeof(c) == sizeof(cfg_), "config size");
    std::memcpy(&c, &cfg_, sizeof(c));
    bt_engine_options opt{};
    opt.rope_theta = rope_theta;
    bt_throw_if_error(bt_engine_create(device_, &c, &opt, &eng_), "bt_engine_create");

    // tensors in .btmodel order (models/model_importer.cpp:69-85)
    std::vector<std::shared_ptr<IComputeBuffer>> bufs = {weights.embed_tokens_w, weights.output_norm_w,
                                                         weights.output_head_w};
    for (const auto& L : weights.layers) {
        bufs.insert(bufs.end(), {L.attn_norm_w, L.ffn_norm_w, L.q_proj_w, L.k_proj_w, L.v_proj_w, L.o_proj_w,
                                 L.gate_proj_w, L.up_proj_w, L.down_proj_w});
    }
    bool all_device = true;
    for (const auto& b : bufs) {
        if (!b) throw std::invalid_argument("CudaTransformerEngine: null weight buffer");
        auto cb = std::dynamic_pointer_cast<CudaBuffer>(b);
        all_device = all_device && cb && cb->device() == device_;
    }
    std::vector<bt_tensor_view> views(bufs.size());
    std::vector<std::vector<uint8_t>> host;
    if (all_device) {
        for (size_t i = 0; i < bufs.size(); ++i)
            views[i] = {std::dynamic_pointer_cast<CudaBuffer>(bufs[i])->device_ptr(), bufs[i]->size()};
    } else {
        host.resize(bufs.size());
        for (size_t i = 0; i < bufs.size(); ++i) {
            host[i].resize(bufs[i]->size());
            bufs[i]->read(host[i].data(), host[i].size(), 0);
            views[i] = {host[i].data(), host[i].size()};
        }
    }
    int rc = bt_engine_load(eng_, views.data(), (uint32_t)views.size(), all_device ? 1 : 0);
    if (rc != BT_OK) {
        bt_engine_destroy(eng_);
        eng_ = nullptr;
        bt_throw_if_error(rc, "bt_engine_load");
    }
}

CudaTransformerEngine::~CudaTransformerEngine() {
    for (auto& kv : kvs_) bt_kv_destroy(kv.second.h);
    bt_engine_destroy(eng_);
}

bt_kv* CudaTransformerEngine::kv_for(const KVCache& kv) {
    if (cfg_.num_layers == 0) throw std::invalid_argument("CudaTransformerEngine: model without layers");
    const std::shared_ptr<IComputeBuffer> k0 = kv.k_cache(0);
    auto it = kvs_.find(&kv);
    if (it != kvs_.end()) {
        if (it->second.k0.lock() == k0) return it->second.h;
        bt_kv_destroy(it->second.h);  // a destroyed KVCache's address, reused by a new one
        kvs_.erase(it);
    }
    // device caches of KVCaches that no longer exist
    for (auto i = kvs_.begin(); i != kvs_.end();) {
        if (i->second.k0.expired()) {
            bt_kv_destroy(i->second.h);
            i = kvs_.erase(i);
        } else {
            ++i;
        }
    }
    bt_kv* h = nullptr;
    bt_throw_if_error(bt_kv_create(eng_, kv.max_seq_len(), kv_dtype_, &h), "bt_kv_create");
    kvs_[&kv] = KvBinding{k0, h};
    return h;
}

void CudaTransformerEngine::sync_to_reference(KVCache& kv_cache) {
    bt_kv* h = kv_for(kv_cache);
    const size_t n = (size_t)kv_cache.max_seq_len() * cfg_.num_kv_heads * cfg_.head_dim;
    std::vector<float> k(n), v(n);
    for (uint32_t l = 0; l < cfg_.num_layers; ++l) {
        bt_throw_if_error(bt_kv_read_layer(h, l, k.data(), v.data()), "bt_kv_read_layer");
        kv_cache.k_cache(l)->write(k.data(), n * sizeof(float), 0);
        kv_cache.v_cache(l)->write(v.data(), n * sizeof(float), 0);
    }
}

std::vector<float> CudaTransformerEngine::forward_single_token(uint32_t token_id, uint32_t pos, KVCache& kv_cache) {
    if (token_id >= cfg_.vocab_size) throw std::out_of_range("Token ID out of vocab bounds");
    std::vector<float> logits(cfg_.vocab_size);
    bt_throw_if_error(bt_engine_forward_token(eng_, kv_for(kv_cache), token_id, pos, logits.data(), &last_argmax_),
                      "forward_single_token");
    return logits;
}

}  // namespace blocktensor
