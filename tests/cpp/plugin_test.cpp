// plugin_test.cpp -- the CUDA backend driven through the reference's own C++
// interfaces, checked against the reference CPU path.
//
// Built by `make -C oracle plugin` against the reference sources (it links the
// reference importer, MemoryManager, KVCache, CPUBackend and TransformerEngine
// as the checker) into oracle/_ref/bt_plugin_test; run by tests/test_gpu_plugin.py.
//
//  1. writes a seeded model with the reference exporter (models/model_importer.cpp:10-42)
//  2. imports it twice with the reference importer: onto CPUBackend and onto
//     CudaBackend (the buffers become device memory through MemoryManager)
//  3. runs TransformerEngine (CPU) and CudaTransformerEngine (GPU) token by
//     token and compares logits (|a-b| <= 1e-2 (1+|a|)) and greedy tokens
//  4. dispatches the pipelines by name on the ramps of
//     tests/test_stage3_kernels.cpp and test_stage4_quant.cpp and compares with
//     cpu_ref / matvec_q8_0 at those tests' tolerances
//  5. checks the exception contract (out_of_range, runtime_error)
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "backends/cpu/cpu_backend.hpp"
#include "blocktensor/kv_cache.hpp"
#include "blocktensor/sampler.hpp"
#include "blocktensor/transformer_engine.hpp"
#include "cuda_backend.hpp"
#include "cuda_engine.hpp"
#include "kernels/cpu_ref.hpp"
#include "memory/memory_manager.hpp"
#include "models/model_importer.hpp"
#include "quantization/quant_types.hpp"

using namespace blocktensor;

static int g_fail = 0;
#define CHECK(cond, ...)                                 \
    do {                                                 \
        if (!(cond)) {                                   \
            std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
            std::fprintf(stderr, __VA_ARGS__);           \
            std::fprintf(stderr, "\n");                  \
            ++g_fail;                                    \
        }                                                \
    } while (0)

static bool approx(float a, float b, float tol) { return std::fabs(a - b) <= tol * (1.0f + std::fabs(a)); }

// deterministic values in [-1, 1)
static float lcg(uint64_t& s) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return (float)((s >> 40) & 0xFFFFFF) / 8388608.0f - 1.0f;
}

static std::shared_ptr<IComputeBuffer> upload(MemoryManager& mem, const void* p, size_t bytes, DataType dt) {
    auto b = mem.allocate(bytes, dt, BufferUsage::STORAGE, MemoryLocation::HOST_VISIBLE);
    mem.copy_host_to_device(p, b, bytes);
    return b;
}

static TransformerWeights make_weights(const ModelConfig& cfg, MemoryManager& mem, uint64_t seed) {
    TransformerWeights w;
    w.config = cfg;
    w.quant_type = DataType::INT8;
    auto vec = [&](size_t n, float scale, float bias) {
        std::vector<float> v(n);
        for (auto& x : v) x = bias + scale * lcg(seed);
        return v;
    };
    auto mat = [&](uint32_t rows, uint32_t cols) {
        auto raw = vec((size_t)rows * cols, 0.04f, 0.0f);
        std::vector<quantization::BlockQ8_0> q(raw.size() / 32);
        quantization::quantize_q8_0(raw.data(), q.data(), raw.size());
        return upload(mem, q.data(), q.size() * sizeof(q[0]), DataType::INT8);
    };
    auto e = vec((size_t)cfg.vocab_size * cfg.dim, 0.05f, 0.0f);
    w.embed_tokens_w = upload(mem, e.data(), e.size() * 4, DataType::FLOAT32);
    auto n = vec(cfg.dim, 0.1f, 1.0f);
    w.output_norm_w = upload(mem, n.data(), n.size() * 4, DataType::FLOAT32);
    w.output_head_w = mat(cfg.vocab_size, cfg.dim);
    const uint32_t kv = cfg.num_kv_heads * cfg.head_dim;
    for (uint32_t l = 0; l < cfg.num_layers; ++l) {
        LayerWeights L;
        auto a = vec(cfg.dim, 0.1f, 1.0f);
        auto f = vec(cfg.dim, 0.1f, 1.0f);
        L.attn_norm_w = upload(mem, a.data(), a.size() * 4, DataType::FLOAT32);
        L.ffn_norm_w = upload(mem, f.data(), f.size() * 4, DataType::FLOAT32);
        L.q_proj_w = mat(cfg.dim, cfg.dim);
        L.k_proj_w = mat(kv, cfg.dim);
        L.v_proj_w = mat(kv, cfg.dim);
        L.o_proj_w = mat(cfg.dim, cfg.dim);
        L.gate_proj_w = mat(cfg.hidden_dim, cfg.dim);
        L.up_proj_w = mat(cfg.hidden_dim, cfg.dim);
        L.down_proj_w = mat(cfg.dim, cfg.hidden_dim);
        w.layers.push_back(L);
    }
    return w;
}

static void engine_parity(const std::string& path, const ModelConfig& cfg) {
    auto cpu = std::make_shared<CPUBackend>();
    MemoryManager cmem(cpu);
    auto cw = importer::import_btmodel(path, cpu, cmem);
    TransformerEngine ref(cpu, cw);
    KVCache ckv(cmem, cfg.num_layers, cfg.max_seq_len, cfg.num_kv_heads, cfg.head_dim);

    auto gpu = std::make_shared<CudaBackend>(0);
    MemoryManager gmem(gpu);
    auto gw = importer::import_btmodel(path, gpu, gmem);  // reference loader, device buffers
    CHECK(std::dynamic_pointer_cast<CudaBuffer>(gw.output_head_w) != nullptr, "importer did not allocate CudaBuffers");
    CudaTransformerEngine eng(gpu, gw);
    KVCache gkv(gmem, cfg.num_layers, cfg.max_seq_len, cfg.num_kv_heads, cfg.head_dim);

    uint32_t tok = 5;
    int steps = 24, bad = 0, tok_diff = 0;
    for (int p = 0; p < steps; ++p) {
        auto a = ref.forward_single_token(tok, p, ckv);
        auto b = eng.forward_single_token(tok, p, gkv);
        for (size_t i = 0; i < a.size(); ++i) bad += !approx(a[i], b[i], 1e-2f);
        uint32_t ta = sampling::sample_greedy(a.data(), cfg.vocab_size);
        uint32_t tb = sampling::sample_greedy(b.data(), cfg.vocab_size);
        tok_diff += ta != tb;
        CHECK(tb == eng.last_argmax(), "device argmax %u != host greedy %u", eng.last_argmax(), tb);
        tok = ta;
    }
    CHECK(bad == 0, "%d logits outside 1e-2", bad);
    CHECK(tok_diff == 0, "%d greedy tokens differ", tok_diff);
    std::printf("engine parity (%d steps through import_btmodel + CudaBackend): %s\n", steps,
                (bad == 0 && tok_diff == 0) ? "PASSED" : "FAILED");

    // the device K/V written back into the reference KVCache equals the CPU engine's cache
    eng.sync_to_reference(gkv);
    const size_t n = (size_t)cfg.max_seq_len * cfg.num_kv_heads * cfg.head_dim;
    std::vector<float> a(n), b(n);
    int kv_bad = 0;
    for (uint32_t l = 0; l < cfg.num_layers; ++l) {
        for (int kv = 0; kv < 2; ++kv) {
            (kv ? ckv.v_cache(l) : ckv.k_cache(l))->read(a.data(), n * sizeof(float), 0);
            (kv ? gkv.v_cache(l) : gkv.k_cache(l))->read(b.data(), n * sizeof(float), 0);
            const size_t used = (size_t)steps * cfg.num_kv_heads * cfg.head_dim;  // positions 0 .. steps - 1
            for (size_t i = 0; i < used; ++i) kv_bad += !approx(a[i], b[i], 1e-2f);
        }
    }
    CHECK(kv_bad == 0, "%d K/V elements outside 1e-2 after sync_to_reference", kv_bad);
    std::printf("KV write-back into the reference KVCache: %s\n", kv_bad == 0 ? "PASSED" : "FAILED");

    // a new KVCache (possibly at the destroyed one's address) starts from an empty device cache
    {
        auto fresh = std::make_unique<KVCache>(gmem, cfg.num_layers, cfg.max_seq_len, cfg.num_kv_heads, cfg.head_dim);
        auto c0 = eng.forward_single_token(5, 0, *fresh);
        KVCache ckv2(cmem, cfg.num_layers, cfg.max_seq_len, cfg.num_kv_heads, cfg.head_dim);
        auto r0 = ref.forward_single_token(5, 0, ckv2);
        int fb = 0;
        for (size_t i = 0; i < r0.size(); ++i) fb += !approx(r0[i], c0[i], 1e-2f);
        CHECK(fb == 0, "fresh KVCache: %d logits outside 1e-2", fb);
    }

    bool caught = false;
    try { eng.forward_single_token(cfg.vocab_size, 0, gkv); } catch (const std::out_of_range&) { caught = true; }
    CHECK(caught, "token >= vocab did not throw out_of_range");
    caught = false;
    try { eng.forward_single_token(1, cfg.max_seq_len, gkv); } catch (const std::out_of_range&) { caught = true; }
    CHECK(caught, "pos >= max_seq did not throw out_of_range");
}

static void pipelines() {
    auto gpu = std::make_shared<CudaBackend>(0);
    MemoryManager mem(gpu);
    auto buf = [&](size_t n) {
        return mem.allocate(n * 4, DataType::FLOAT32, BufferUsage::STORAGE, MemoryLocation::HOST_VISIBLE);
    };
    auto ramp = [](size_t n, int mod, float a, float b) {
        std::vector<float> v(n);
        for (size_t i = 0; i < n; ++i) v[i] = static_cast<float>(i % mod) * a - b;
        return v;
    };
    int bad = 0;
    {   // rmsnorm 4x512 (test_stage3_kernels.cpp:49-89)
        auto x = ramp(4 * 512, 100, 0.1f, 5.0f);
        std::vector<float> w(512), ref(x.size()), out(x.size());
        for (size_t i = 0; i < w.size(); ++i) w[i] = 1.0f + static_cast<float>(i % 10) * 0.05f;
        cpu_ref::rmsnorm(x.data(), w.data(), ref.data(), 4, 512, 1e-5f);
        auto bx = buf(x.size()), bw = buf(w.size()), bo = buf(x.size());
        mem.copy_host_to_device(x.data(), bx, x.size() * 4);
        mem.copy_host_to_device(w.data(), bw, w.size() * 4);
        struct { uint32_t dim; float eps; } pc{512, 1e-5f};
        gpu->dispatch(gpu->create_pipeline_from_spirv("rmsnorm", {}, 3, 8), {bx, bw, bo}, {4, 1, 1}, &pc, sizeof(pc));
        mem.copy_device_to_host(bo, out.data(), out.size() * 4);
        for (size_t i = 0; i < out.size(); ++i) bad += !approx(out[i], ref[i], 1e-4f);
    }
    {   // rope in place, seq 2 x 4 heads x hd 64 (test_stage3_kernels.cpp:91-130, engine binds in==out)
        auto x = ramp(2 * 4 * 64, 30, 0.2f, 3.0f);
        std::vector<float> ref(x.size()), out(x.size());
        cpu_ref::rope(x.data(), ref.data(), 2, 4, 64, 9);
        auto bx = buf(x.size());
        mem.copy_host_to_device(x.data(), bx, x.size() * 4);
        struct { uint32_t s, h, d, p; } pc{2, 4, 64, 9};
        gpu->dispatch(gpu->create_pipeline_from_spirv("rope", {}, 2, 16), {bx, bx}, {2, 1, 1}, &pc, sizeof(pc));
        mem.copy_device_to_host(bx, out.data(), out.size() * 4);
        for (size_t i = 0; i < out.size(); ++i) bad += !approx(out[i], ref[i], 1e-4f);
    }
    {   // softmax 4x256 and silu 1024
        auto x = ramp(4 * 256, 50, 0.1f, 2.5f);
        std::vector<float> ref(x.size()), out(x.size());
        cpu_ref::softmax(x.data(), ref.data(), 4, 256);
        auto bx = buf(x.size()), bo = buf(x.size());
        mem.copy_host_to_device(x.data(), bx, x.size() * 4);
        struct { uint32_t r, d; } pc{4, 256};
        gpu->dispatch(gpu->create_pipeline_from_spirv("softmax", {}, 2, 8), {bx, bo}, {4, 1, 1}, &pc, sizeof(pc));
        mem.copy_device_to_host(bo, out.data(), out.size() * 4);
        for (size_t i = 0; i < out.size(); ++i) bad += !approx(out[i], ref[i], 1e-4f);
        auto s = ramp(1024, 100, 0.1f, 5.0f);
        std::vector<float> sref(s.size()), sout(s.size());
        cpu_ref::silu(s.data(), sref.data(), 1024);
        auto bs = buf(s.size()), bso = buf(s.size());
        mem.copy_host_to_device(s.data(), bs, s.size() * 4);
        uint32_t n = 1024;
        gpu->dispatch(gpu->create_pipeline_from_spirv("silu", {}, 2, 4), {bs, bso}, {4, 1, 1}, &n, 4);
        mem.copy_device_to_host(bso, sout.data(), sout.size() * 4);
        for (size_t i = 0; i < sout.size(); ++i) bad += !approx(sout[i], sref[i], 1e-4f);
    }
    {   // Q8_0 matvec 16x256 (test_stage4_quant.cpp:47-94)
        auto raw = ramp(16 * 256, 50, 0.1f, 2.5f);
        auto x = ramp(256, 20, 0.15f, 1.5f);
        std::vector<quantization::BlockQ8_0> q(16 * 8);
        quantization::quantize_q8_0(raw.data(), q.data(), raw.size());
        std::vector<float> ref(16), out(16);
        quantization::matvec_q8_0(q.data(), x.data(), ref.data(), 16, 256);
        auto bw = mem.allocate(q.size() * sizeof(q[0]), DataType::INT8, BufferUsage::STORAGE, MemoryLocation::HOST_VISIBLE);
        auto bx = buf(256), by = buf(16);
        mem.copy_host_to_device(q.data(), bw, q.size() * sizeof(q[0]));
        mem.copy_host_to_device(x.data(), bx, 256 * 4);
        struct { uint32_t M, N; } pc{16, 256};
        gpu->dispatch(gpu->create_pipeline_from_spirv("matvec_q8_0", {}, 3, 8), {bw, bx, by}, {16, 1, 1}, &pc, sizeof(pc));
        gpu->synchronize();
        mem.copy_device_to_host(by, out.data(), 16 * 4);
        for (int i = 0; i < 16; ++i) bad += !approx(out[i], ref[i], 1e-2f);
    }
    CHECK(bad == 0, "%d pipeline outputs outside tolerance", bad);
    std::printf("pipelines by name (rmsnorm, rope, softmax, silu, matvec_q8_0): %s\n", bad == 0 ? "PASSED" : "FAILED");

    auto b = buf(4);
    bool caught = false;
    float tmp[8] = {0};
    try { b->write(tmp, 32, 0); } catch (const std::runtime_error&) { caught = true; }
    CHECK(caught, "CudaBuffer::write out of bounds did not throw");
}

int main(int argc, char** argv) {
    std::string path = argc > 1 ? argv[1] : "/tmp/bt_plugin_test.btmodel";
    ModelConfig cfg;
    cfg.vocab_size = 1000;
    cfg.dim = 256;
    cfg.hidden_dim = 512;
    cfg.num_layers = 4;
    cfg.num_heads = 4;
    cfg.num_kv_heads = 4;
    cfg.head_dim = 64;
    cfg.max_seq_len = 64;
    {
        auto cpu = std::make_shared<CPUBackend>();
        MemoryManager mem(cpu);
        auto w = make_weights(cfg, mem, 42);
        importer::export_btmodel(path, w, mem);
    }
    try {
        engine_parity(path, cfg);
        pipelines();
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FAIL: exception %s\n", e.what());
        return 2;
    }
    std::printf("%s\n", g_fail ? "PLUGIN TEST FAILED" : "PLUGIN TEST PASSED");
    return g_fail ? 1 : 0;
}
