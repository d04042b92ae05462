/*
 * bt_oracle.h -- CPU oracle for the BlockTensor int8 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * CPU path (ulusluyz/BlockTensor) that the CUDA backend is checked against.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it, and only as the checker.  The product path never calls it.
 *
 * Every function cites the reference file:line whose arithmetic it restates.
 * Parity is pinned: tests/test_oracle_pins.py checks this restatement
 * bit-for-bit against the reference's own sources compiled into
 * oracle/_ref/libbtref.so (recipe: oracle/Makefile), and against the
 * known-answer values of the reference's tests (tests/golden/).
 *
 * Build flags matter for bit-exactness: -O2 -ffp-contract=off, no -ffast-math,
 * no -march (the reference is compiled with g++ -O2 -std=c++20 for baseline
 * x86-64, which has no FMA contraction).
 */
#ifndef BT_ORACLE_H
#define BT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BTO_Q8_BLOCK 32

/* Byte-identical to blocktensor::quantization::BlockQ8_0
 * (quantization/quant_types.hpp:12-15): 4-byte scale then 32 int8. */
typedef struct bto_block_q8_0 {
    float scale;
    int8_t qs[BTO_Q8_BLOCK];
} bto_block_q8_0;

/* Field order and size (36 bytes) of blocktensor::ModelConfig
 * (runtime/include/blocktensor/model_config.hpp:9-19). */
typedef struct bto_config {
    uint32_t vocab_size;
    uint32_t dim;
    uint32_t hidden_dim;
    uint32_t num_layers;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t max_seq_len;
    float rms_norm_eps;
} bto_config;

/* ---- quantization (quantization/quant_types.cpp) ---- */
int  bto_quantize_q8_0(const float* src, bto_block_q8_0* dst, size_t n);       /* :8-34, returns -1 if n%32 */
void bto_dequantize_q8_0(const bto_block_q8_0* src, float* dst, size_t n);     /* :36-48 */
void bto_matvec_q8_0(const bto_block_q8_0* W, const float* X, float* Y,
                     uint32_t M, uint32_t N);                                   /* :101-121 */
/* Same arithmetic per row, rows split over nthreads (bit-identical to 1 thread). */
void bto_matvec_q8_0_mt(const bto_block_q8_0* W, const float* X, float* Y,
                        uint32_t M, uint32_t N, int nthreads);

/* ---- math kernels (kernels/cpu_ref.hpp) ---- */
void bto_rmsnorm(const float* in, const float* w, float* out, uint32_t rows, uint32_t dim, float eps); /* :11-28 */
void bto_rope(const float* in, float* out, uint32_t seq, uint32_t heads, uint32_t head_dim,
              uint32_t pos_offset, float theta);                                 /* :30-53, theta=10000 there */
void bto_softmax(const float* in, float* out, uint32_t rows, uint32_t dim);     /* :55-72 */
void bto_silu(const float* in, float* out, uint32_t n);                          /* :74-79 */
uint32_t bto_sample_greedy(const float* logits, uint32_t n);                     /* sampler.hpp:11-13 */

/* ---- seeded synthetic inputs (shared spec with the CUDA generator) ---- */
uint64_t bto_splitmix64(uint64_t z);
uint64_t bto_stream_base(uint64_t seed, uint64_t stream);
/* value i = (float)(sum of four 16-bit uniforms - 131070) * k, k = sigma/37837.2271 */
void bto_gen_normal(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, float k, float* out);
float bto_normal_k(float sigma);
/* uniform int8 in [-127,127] */
void bto_gen_int8(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, int8_t* out);
/* uniform float lo + u24 * ((hi-lo)/2^24) */
void bto_gen_uniform(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, float lo, float hi, float* out);
/* uniform token ids in [0, vocab) */
void bto_gen_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab, uint32_t* out);

/* Stream ids of the synthetic model (tensor order of models/model_importer.cpp:69-85). */
#define BTO_STREAM_EMBED    0u
#define BTO_STREAM_OUT_NORM 1u
#define BTO_STREAM_HEAD     2u
#define BTO_STREAM_LAYER(l, j) (16u + 16u * (uint32_t)(l) + (uint32_t)(j))
enum { BTO_T_ATTN_NORM = 0, BTO_T_FFN_NORM, BTO_T_Q, BTO_T_K, BTO_T_V, BTO_T_O,
       BTO_T_GATE, BTO_T_UP, BTO_T_DOWN, BTO_T_COUNT };
#define BTO_STREAM_PROMPT 0xF000u

/* ---- model + engine restatement (runtime/src/transformer_engine.cpp) ---- */
typedef struct bto_layer {
    float* attn_norm;                 /* [dim] */
    float* ffn_norm;                  /* [dim] */
    bto_block_q8_0 *q, *k, *v, *o;    /* [rows*cols/32] */
    bto_block_q8_0 *gate, *up, *down;
} bto_layer;

typedef struct bto_model {
    bto_config cfg;
    float* embed;                     /* [vocab][dim] fp32 */
    float* out_norm;                  /* [dim] */
    bto_block_q8_0* head;             /* [vocab*dim/32] */
    bto_layer* layers;
    int owns;                         /* 1 if arrays were malloc'ed by the oracle */
} bto_model;

/* Matrices N(0,sigma) -> Q8_0 via bto_quantize_q8_0, embeddings N(0,sigma), norms 1.0. */
bto_model* bto_model_generate(const bto_config* cfg, uint64_t seed, float sigma, int nthreads);
/* Wrap caller-owned arrays (no copy). layers[] must hold cfg.num_layers entries. */
bto_model* bto_model_wrap(const bto_config* cfg, float* embed, float* out_norm,
                          bto_block_q8_0* head, const bto_layer* layers);
void bto_model_free(bto_model* m);

/* KV cache: per layer [max_seq][kv_heads][head_dim] as in runtime/src/kv_cache.cpp:9,21-23.
 * kv_fp16 != 0 rounds every appended K/V value to IEEE binary16 (round-to-nearest-even),
 * which is the restatement used for the fp16-KV configurations (the reference is fp32 only). */
typedef struct bto_kv {
    uint32_t num_layers, max_seq, kv_heads, head_dim;
    int kv_fp16;
    float* k;                         /* [layers][max_seq][kv_heads][head_dim] */
    float* v;
} bto_kv;

bto_kv* bto_kv_create(uint32_t num_layers, uint32_t max_seq, uint32_t kv_heads, uint32_t head_dim, int kv_fp16);
void bto_kv_free(bto_kv* kv);

/* One token (transformer_engine.cpp:228-251).  logits: [vocab] or NULL.
 * taps: NULL or [num_layers][dim] residual stream after each layer.
 * Returns 0, or -2 for token >= vocab / pos >= max_seq (the reference throws out_of_range). */
int bto_forward_token(const bto_model* m, bto_kv* kv, uint32_t token, uint32_t pos,
                      float rope_theta, float* logits, float* taps, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
