// ref_shim.cpp -- C entry points over the UNMODIFIED reference CPU path.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's own sources (quantization/quant_types.cpp,
// backends/cpu/cpu_backend.cpp, memory/memory_manager.cpp,
// runtime/src/{kv_cache,transformer_engine}.cpp, models/model_importer.cpp)
// into oracle/_ref/libbtref.so.  It is used to pin the C restatement in
// oracle/bt_oracle.c and as the timed CPU baseline ("kind": "reference").
//
// Exceptions of the reference are mapped to return codes:
//   0 ok, -2 std::out_of_range, -3 std::runtime_error, -4 std::invalid_argument, -1 other.

#include "backends/cpu/cpu_backend.hpp"
#include "blocktensor/kv_cache.hpp"
#include "blocktensor/sampler.hpp"
#include "blocktensor/transformer_engine.hpp"
#include "kernels/cpu_ref.hpp"
#include "memory/memory_manager.hpp"
#include "models/model_importer.hpp"
#include "quantization/quant_types.hpp"

#include <cstring>
#include <memory>
#include <stdexcept>
#include <vector>

using namespace blocktensor;

#define BTR_TRY try {
#define BTR_CATCH                                           \
    }                                                       \
    catch (const std::out_of_range&) { return -2; }        \
    catch (const std::invalid_argument&) { return -4; }    \
    catch (const std::runtime_error&) { return -3; }       \
    catch (...) { return -1; }                              \
    return 0;

extern "C" {

int btr_quantize_q8_0(const float* src, void* dst, size_t n) {
    BTR_TRY quantization::quantize_q8_0(src, static_cast<quantization::BlockQ8_0*>(dst), n); BTR_CATCH
}
int btr_dequantize_q8_0(const void* src, float* dst, size_t n) {
    BTR_TRY quantization::dequantize_q8_0(static_cast<const quantization::BlockQ8_0*>(src), dst, n); BTR_CATCH
}
int btr_matvec_q8_0(const void* W, const float* X, float* Y, uint32_t M, uint32_t N) {
    BTR_TRY quantization::matvec_q8_0(static_cast<const quantization::BlockQ8_0*>(W), X, Y, M, N); BTR_CATCH
}
int btr_quantize_q4_0(const float* src, void* dst, size_t n) {
    BTR_TRY quantization::quantize_q4_0(src, static_cast<quantization::BlockQ4_0*>(dst), n); BTR_CATCH
}
void btr_rmsnorm(const float* in, const float* w, float* out, uint32_t rows, uint32_t dim, float eps) {
    cpu_ref::rmsnorm(in, w, out, rows, dim, eps);
}
void btr_rope(const float* in, float* out, uint32_t seq, uint32_t heads, uint32_t hd, uint32_t pos) {
    cpu_ref::rope(in, out, seq, heads, hd, pos);
}
void btr_softmax(const float* in, float* out, uint32_t rows, uint32_t dim) { cpu_ref::softmax(in, out, rows, dim); }
void btr_silu(const float* in, float* out, uint32_t n) { cpu_ref::silu(in, out, n); }
uint32_t btr_sample_greedy(const float* logits, uint32_t n) { return sampling::sample_greedy(logits, n); }
uint32_t btr_sample_top_p_top_k(const float* logits, uint32_t n, float temp, float top_p, uint32_t top_k, uint64_t seed) {
    return sampling::sample_top_p_top_k(logits, n, temp, top_p, top_k, seed);
}
size_t btr_sizeof_config() { return sizeof(ModelConfig); }
size_t btr_sizeof_block_q8_0() { return sizeof(quantization::BlockQ8_0); }

// ---------------------------------------------------------------------------
// Engine: the reference TransformerEngine over the reference CPUBackend.
// ---------------------------------------------------------------------------
struct btr_engine {
    std::shared_ptr<CPUBackend> backend;
    std::unique_ptr<MemoryManager> mem;
    TransformerWeights weights;
    std::unique_ptr<TransformerEngine> engine;
    std::unique_ptr<KVCache> kv;
};

struct btr_tensor { const void* data; uint64_t bytes; };

static std::shared_ptr<IComputeBuffer> upload(MemoryManager& mem, const btr_tensor& t, DataType dt) {
    auto b = mem.allocate(t.bytes, dt, BufferUsage::STORAGE, MemoryLocation::HOST_VISIBLE);
    mem.copy_host_to_device(t.data, b, t.bytes);
    return b;
}

static void finish(btr_engine* e, uint32_t kv_max_seq) {
    e->engine = std::make_unique<TransformerEngine>(e->backend, e->weights);
    const ModelConfig& c = e->weights.config;
    e->kv = std::make_unique<KVCache>(*e->mem, c.num_layers, kv_max_seq, c.num_kv_heads, c.head_dim);
}

// tensors: .btmodel order (model_importer.cpp:69-85): embed, out_norm, head, then per layer
// attn_norm, ffn_norm, q, k, v, o, gate, up, down.  cfg points at a 36-byte ModelConfig.
int btr_engine_create(const void* cfg, const btr_tensor* tensors, uint32_t n_tensors,
                      uint32_t kv_max_seq, btr_engine** out) {
    BTR_TRY
        auto e = std::make_unique<btr_engine>();
        e->backend = std::make_shared<CPUBackend>();
        e->mem = std::make_unique<MemoryManager>(e->backend);
        std::memcpy(&e->weights.config, cfg, sizeof(ModelConfig));
        e->weights.quant_type = DataType::INT8;
        const ModelConfig& c = e->weights.config;
        if (n_tensors != 3 + 9 * c.num_layers) throw std::invalid_argument("tensor count");
        e->weights.embed_tokens_w = upload(*e->mem, tensors[0], DataType::FLOAT32);
        e->weights.output_norm_w = upload(*e->mem, tensors[1], DataType::FLOAT32);
        e->weights.output_head_w = upload(*e->mem, tensors[2], DataType::INT8);
        for (uint32_t l = 0; l < c.num_layers; ++l) {
            const btr_tensor* t = tensors + 3 + 9 * l;
            LayerWeights L;
            L.attn_norm_w = upload(*e->mem, t[0], DataType::FLOAT32);
            L.ffn_norm_w = upload(*e->mem, t[1], DataType::FLOAT32);
            L.q_proj_w = upload(*e->mem, t[2], DataType::INT8);
            L.k_proj_w = upload(*e->mem, t[3], DataType::INT8);
            L.v_proj_w = upload(*e->mem, t[4], DataType::INT8);
            L.o_proj_w = upload(*e->mem, t[5], DataType::INT8);
            L.gate_proj_w = upload(*e->mem, t[6], DataType::INT8);
            L.up_proj_w = upload(*e->mem, t[7], DataType::INT8);
            L.down_proj_w = upload(*e->mem, t[8], DataType::INT8);
            e->weights.layers.push_back(L);
        }
        finish(e.get(), kv_max_seq ? kv_max_seq : c.max_seq_len);
        *out = e.release();
    BTR_CATCH
}

// The reference .btmodel loader (models/model_importer.cpp:44-88).
int btr_engine_import(const char* path, uint32_t kv_max_seq, btr_engine** out) {
    BTR_TRY
        auto e = std::make_unique<btr_engine>();
        e->backend = std::make_shared<CPUBackend>();
        e->mem = std::make_unique<MemoryManager>(e->backend);
        e->weights = importer::import_btmodel(path, e->backend, *e->mem);
        finish(e.get(), kv_max_seq ? kv_max_seq : e->weights.config.max_seq_len);
        *out = e.release();
    BTR_CATCH
}

// The reference .btmodel writer (models/model_importer.cpp:10-42).
int btr_engine_export(btr_engine* e, const char* path) {
    BTR_TRY importer::export_btmodel(path, e->weights, *e->mem); BTR_CATCH
}

int btr_engine_config(btr_engine* e, void* cfg_out) {
    std::memcpy(cfg_out, &e->weights.config, sizeof(ModelConfig));
    return 0;
}

uint64_t btr_engine_allocated_bytes(btr_engine* e) { return e->mem->total_allocated_bytes(); }

int btr_engine_forward(btr_engine* e, uint32_t token, uint32_t pos, float* logits) {
    BTR_TRY
        std::vector<float> out = e->engine->forward_single_token(token, pos, *e->kv);
        if (logits) std::memcpy(logits, out.data(), out.size() * sizeof(float));
    BTR_CATCH
}

// Reads the reference KV cache of one layer ([max_seq][kv_heads][head_dim] fp32).
int btr_engine_read_kv(btr_engine* e, uint32_t layer, float* k, float* v, uint64_t bytes) {
    BTR_TRY
        e->mem->copy_device_to_host(e->kv->k_cache(layer), k, bytes);
        e->mem->copy_device_to_host(e->kv->v_cache(layer), v, bytes);
    BTR_CATCH
}

void btr_engine_destroy(btr_engine* e) { delete e; }

// KVCache::update on a standalone cache (runtime/src/kv_cache.cpp:17-27).
int btr_kv_update_probe(uint32_t layers, uint32_t max_seq, uint32_t kvh, uint32_t hd,
                        uint32_t layer, uint32_t pos) {
    BTR_TRY
        auto be = std::make_shared<CPUBackend>();
        MemoryManager mem(be);
        KVCache kv(mem, layers, max_seq, kvh, hd);
        std::vector<float> d((size_t)kvh * hd, 1.0f);
        kv.update(layer, pos, d.data(), d.data());
    BTR_CATCH
}

}  // extern "C"
