/*
 * bt_oracle.c -- CPU oracle (test infrastructure only; see bt_oracle.h).
 *
 * A plain-C restatement of the reference CPU path.  Each function names the
 * reference lines it follows; the float operations are written in the same
 * order so that, compiled with -O2 -ffp-contract=off, results are
 * bit-identical to the reference's g++ -O2 build.
 */
#define _GNU_SOURCE
#include "bt_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* quantization/quant_types.cpp                                         */
/* ------------------------------------------------------------------ */

/* x86-64 cvttss2si semantics of static_cast<int>(float): NaN and values
 * outside int range give INT32_MIN. */
static int to_int_trunc(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int)v;
}

/* quant_types.cpp:8-34 */
int bto_quantize_q8_0(const float* src, bto_block_q8_0* dst, size_t n) {
    if (n % BTO_Q8_BLOCK != 0) return -1;            /* :9-11 invalid_argument */
    size_t nb = n / BTO_Q8_BLOCK;
    for (size_t b = 0; b < nb; ++b) {
        const float* s = src + b * BTO_Q8_BLOCK;
        float amax = 0.0f;
        for (int i = 0; i < BTO_Q8_BLOCK; ++i) {     /* :19-22 std::max(amax, std::abs(x)) */
            float a = fabsf(s[i]);
            amax = (amax < a) ? a : amax;
        }
        float scale = amax / 127.0f;                 /* :24 */
        dst[b].scale = scale;
        float inv = (scale != 0.0f) ? (1.0f / scale) : 0.0f;   /* :27 */
        for (int i = 0; i < BTO_Q8_BLOCK; ++i) {     /* :28-32 */
            int q = to_int_trunc(roundf(s[i] * inv));
            q = q < -128 ? -128 : (q > 127 ? 127 : q);
            dst[b].qs[i] = (int8_t)q;
        }
    }
    return 0;
}

/* quant_types.cpp:36-48 */
void bto_dequantize_q8_0(const bto_block_q8_0* src, float* dst, size_t n) {
    size_t nb = n / BTO_Q8_BLOCK;
    for (size_t b = 0; b < nb; ++b) {
        float scale = src[b].scale;
        for (int i = 0; i < BTO_Q8_BLOCK; ++i) dst[b * BTO_Q8_BLOCK + i] = (float)src[b].qs[i] * scale;
    }
}

/* quant_types.cpp:101-121 for rows [r0, r1) */
static void matvec_rows(const bto_block_q8_0* W, const float* X, float* Y,
                        uint32_t r0, uint32_t r1, uint32_t N) {
    uint32_t bpr = N / BTO_Q8_BLOCK;
    for (uint32_t row = r0; row < r1; ++row) {
        float sum = 0.0f;
        const bto_block_q8_0* rw = W + (size_t)row * bpr;
        for (uint32_t b = 0; b < bpr; ++b) {
            const float* xb = X + (size_t)b * BTO_Q8_BLOCK;
            float bs = 0.0f;
            for (int i = 0; i < BTO_Q8_BLOCK; ++i) bs += (float)rw[b].qs[i] * xb[i];
            sum += bs * rw[b].scale;
        }
        Y[row] = sum;
    }
}

void bto_matvec_q8_0(const bto_block_q8_0* W, const float* X, float* Y, uint32_t M, uint32_t N) {
    matvec_rows(W, X, Y, 0, M, N);
}

typedef struct mv_job {
    const bto_block_q8_0* W; const float* X; float* Y;
    uint32_t r0, r1, N;
} mv_job;

static void* mv_worker(void* p) {
    mv_job* j = (mv_job*)p;
    matvec_rows(j->W, j->X, j->Y, j->r0, j->r1, j->N);
    return NULL;
}

void bto_matvec_q8_0_mt(const bto_block_q8_0* W, const float* X, float* Y,
                        uint32_t M, uint32_t N, int nthreads) {
    if (nthreads <= 1 || M < 64) { matvec_rows(W, X, Y, 0, M, N); return; }
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    mv_job jobs[256];
    uint32_t per = (M + (uint32_t)nthreads - 1) / (uint32_t)nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; ++t) {
        uint32_t r0 = (uint32_t)t * per, r1 = r0 + per;
        if (r0 >= M) break;
        if (r1 > M) r1 = M;
        jobs[t] = (mv_job){W, X, Y, r0, r1, N};
        if (pthread_create(&th[t], NULL, mv_worker, &jobs[t]) != 0) { mv_worker(&jobs[t]); th[t] = 0; }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t) if (th[t]) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------ */
/* kernels/cpu_ref.hpp                                                  */
/* ------------------------------------------------------------------ */

/* cpu_ref.hpp:11-28 */
void bto_rmsnorm(const float* in, const float* w, float* out, uint32_t rows, uint32_t dim, float eps) {
    for (uint32_t r = 0; r < rows; ++r) {
        const float* x = in + (size_t)r * dim;
        float* o = out + (size_t)r * dim;
        float ss = 0.0f;
        for (uint32_t d = 0; d < dim; ++d) ss += x[d] * x[d];
        float mean = ss / (float)dim;
        float inv = 1.0f / sqrtf(mean + eps);
        for (uint32_t d = 0; d < dim; ++d) o[d] = x[d] * inv * w[d];
    }
}

/* cpu_ref.hpp:30-53, with the hard-coded 10000.0f base (:40) as a parameter */
void bto_rope(const float* in, float* out, uint32_t seq, uint32_t heads, uint32_t hd,
              uint32_t pos_offset, float theta) {
    uint32_t half = hd / 2;
    for (uint32_t s = 0; s < seq; ++s) {
        uint32_t pos = s + pos_offset;
        for (uint32_t h = 0; h < heads; ++h) {
            const float* ih = in + ((size_t)s * heads + h) * hd;
            float* oh = out + ((size_t)s * heads + h) * hd;
            for (uint32_t i = 0; i < half; ++i) {
                float freq = 1.0f / powf(theta, (float)(2 * i) / (float)hd);
                float val = (float)pos * freq;
                float c = cosf(val), sn = sinf(val);
                float x1 = ih[i], x2 = ih[i + half];
                oh[i] = x1 * c - x2 * sn;
                oh[i + half] = x1 * sn + x2 * c;
            }
        }
    }
}

/* cpu_ref.hpp:55-72 */
void bto_softmax(const float* in, float* out, uint32_t rows, uint32_t dim) {
    for (uint32_t r = 0; r < rows; ++r) {
        const float* x = in + (size_t)r * dim;
        float* o = out + (size_t)r * dim;
        float mx = x[0];                                  /* std::max_element: first largest */
        for (uint32_t d = 1; d < dim; ++d) if (mx < x[d]) mx = x[d];
        float sum = 0.0f;
        for (uint32_t d = 0; d < dim; ++d) { o[d] = expf(x[d] - mx); sum += o[d]; }
        for (uint32_t d = 0; d < dim; ++d) o[d] /= sum;
    }
}

/* cpu_ref.hpp:74-79 */
void bto_silu(const float* in, float* out, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) { float x = in[i]; out[i] = x / (1.0f + expf(-x)); }
}

/* runtime/include/blocktensor/sampler.hpp:11-13: std::max_element, first max wins */
uint32_t bto_sample_greedy(const float* logits, uint32_t n) {
    uint32_t best = 0;
    for (uint32_t i = 1; i < n; ++i) if (logits[best] < logits[i]) best = i;
    return best;
}

/* ------------------------------------------------------------------ */
/* Seeded synthetic inputs.  Integer hashing plus one correctly rounded */
/* float multiply, so CPU and GPU generators agree bit for bit.         */
/* ------------------------------------------------------------------ */

uint64_t bto_splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t bto_stream_base(uint64_t seed, uint64_t stream) {
    return bto_splitmix64(bto_splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}

float bto_normal_k(float sigma) {
    /* std of the sum of four uniforms on {0..65535}: sqrt(4*(65536^2-1)/12) */
    return (float)((double)sigma / 37837.22712838299);
}

void bto_gen_normal(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, float k, float* out) {
    uint64_t base = bto_stream_base(seed, stream);
    for (size_t i = 0; i < n; ++i) {
        uint64_t h = bto_splitmix64(base + offset + i);
        int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF)
                  + (int32_t)((h >> 32) & 0xFFFF) + (int32_t)(h >> 48);
        out[i] = (float)(s - 131070) * k;
    }
}

void bto_gen_int8(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, int8_t* out) {
    uint64_t base = bto_stream_base(seed, stream);
    for (size_t i = 0; i < n; ++i) {
        uint64_t h = bto_splitmix64(base + offset + i);
        out[i] = (int8_t)((int32_t)((h >> 32) % 255u) - 127);
    }
}

void bto_gen_uniform(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, float lo, float hi, float* out) {
    uint64_t base = bto_stream_base(seed, stream);
    float step = (hi - lo) / 16777216.0f;
    for (size_t i = 0; i < n; ++i) {
        uint64_t h = bto_splitmix64(base + offset + i);
        out[i] = lo + (float)(uint32_t)(h >> 40) * step;
    }
}

void bto_gen_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab, uint32_t* out) {
    uint64_t base = bto_stream_base(seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)((bto_splitmix64(base + i) >> 32) % vocab);
}

/* ------------------------------------------------------------------ */
/* Model                                                                */
/* ------------------------------------------------------------------ */

static bto_block_q8_0* gen_matrix(uint64_t seed, uint32_t stream, size_t rows, size_t cols, float k) {
    size_t n = rows * cols;
    bto_block_q8_0* q = (bto_block_q8_0*)malloc(sizeof(bto_block_q8_0) * (n / BTO_Q8_BLOCK));
    /* generate and quantize a row slab at a time to bound memory */
    size_t slab_rows = rows < 256 ? rows : 256;
    float* tmp = (float*)malloc(sizeof(float) * slab_rows * cols);
    for (size_t r = 0; r < rows; r += slab_rows) {
        size_t nr = (rows - r) < slab_rows ? (rows - r) : slab_rows;
        bto_gen_normal(seed, stream, r * cols, nr * cols, k, tmp);
        bto_quantize_q8_0(tmp, q + r * cols / BTO_Q8_BLOCK, nr * cols);
    }
    free(tmp);
    return q;
}

static float* gen_ones(size_t n) {
    float* p = (float*)malloc(sizeof(float) * n);
    for (size_t i = 0; i < n; ++i) p[i] = 1.0f;
    return p;
}

typedef struct gen_job { const bto_config* c; uint64_t seed; float k; bto_model* m; uint32_t l; } gen_job;

static void gen_layer(const bto_config* c, uint64_t seed, float k, bto_layer* L, uint32_t l) {
    size_t D = c->dim, F = c->hidden_dim, KV = (size_t)c->num_kv_heads * c->head_dim;
    L->attn_norm = gen_ones(D);
    L->ffn_norm = gen_ones(D);
    L->q = gen_matrix(seed, BTO_STREAM_LAYER(l, BTO_T_Q), D, D, k);
    L->k = gen_matrix(seed, BTO_STREAM_LAYER(l, BTO_T_K), KV, D, k);
    L->v = gen_matrix(seed, BTO_STREAM_LAYER(l, BTO_T_V), KV, D, k);
    L->o = gen_matrix(seed, BTO_STREAM_LAYER(l, BTO_T_O), D, D, k);
    L->gate = gen_matrix(seed, BTO_STREAM_LAYER(l, BTO_T_GATE), F, D, k);
    L->up = gen_matrix(seed, BTO_STREAM_LAYER(l, BTO_T_UP), F, D, k);
    L->down = gen_matrix(seed, BTO_STREAM_LAYER(l, BTO_T_DOWN), D, F, k);
}

typedef struct layer_range { const bto_config* c; uint64_t seed; float k; bto_model* m; uint32_t l0, l1, step; } layer_range;
static void* gen_worker(void* p) {
    layer_range* r = (layer_range*)p;
    for (uint32_t l = r->l0; l < r->l1; l += r->step) gen_layer(r->c, r->seed, r->k, &r->m->layers[l], l);
    return NULL;
}

bto_model* bto_model_generate(const bto_config* c, uint64_t seed, float sigma, int nthreads) {
    bto_model* m = (bto_model*)calloc(1, sizeof(bto_model));
    m->cfg = *c;
    m->owns = 1;
    float k = bto_normal_k(sigma);
    size_t V = c->vocab_size, D = c->dim;
    m->embed = (float*)malloc(sizeof(float) * V * D);
    bto_gen_normal(seed, BTO_STREAM_EMBED, 0, V * D, k, m->embed);
    m->out_norm = gen_ones(D);
    m->head = gen_matrix(seed, BTO_STREAM_HEAD, V, D, k);
    m->layers = (bto_layer*)calloc(c->num_layers, sizeof(bto_layer));
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 64) nthreads = 64;
    pthread_t th[64];
    layer_range jobs[64];
    int started = 0;
    for (int t = 0; t < nthreads && (uint32_t)t < c->num_layers; ++t) {
        jobs[t] = (layer_range){c, seed, k, m, (uint32_t)t, c->num_layers, (uint32_t)nthreads};
        if (pthread_create(&th[t], NULL, gen_worker, &jobs[t]) != 0) { gen_worker(&jobs[t]); th[t] = 0; }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t) if (th[t]) pthread_join(th[t], NULL);
    return m;
}

bto_model* bto_model_wrap(const bto_config* c, float* embed, float* out_norm,
                          bto_block_q8_0* head, const bto_layer* layers) {
    bto_model* m = (bto_model*)calloc(1, sizeof(bto_model));
    m->cfg = *c;
    m->embed = embed; m->out_norm = out_norm; m->head = head;
    m->layers = (bto_layer*)calloc(c->num_layers, sizeof(bto_layer));
    memcpy(m->layers, layers, sizeof(bto_layer) * c->num_layers);
    m->owns = 0;
    return m;
}

void bto_model_free(bto_model* m) {
    if (!m) return;
    if (m->owns) {
        free(m->embed); free(m->out_norm); free(m->head);
        for (uint32_t l = 0; l < m->cfg.num_layers; ++l) {
            bto_layer* L = &m->layers[l];
            free(L->attn_norm); free(L->ffn_norm); free(L->q); free(L->k); free(L->v);
            free(L->o); free(L->gate); free(L->up); free(L->down);
        }
    }
    free(m->layers);
    free(m);
}

/* ------------------------------------------------------------------ */
/* KV cache (runtime/src/kv_cache.cpp)                                  */
/* ------------------------------------------------------------------ */

bto_kv* bto_kv_create(uint32_t L, uint32_t max_seq, uint32_t kvh, uint32_t hd, int kv_fp16) {
    bto_kv* kv = (bto_kv*)calloc(1, sizeof(bto_kv));
    kv->num_layers = L; kv->max_seq = max_seq; kv->kv_heads = kvh; kv->head_dim = hd;
    kv->kv_fp16 = kv_fp16;
    size_t n = (size_t)L * max_seq * kvh * hd;
    kv->k = (float*)calloc(n, sizeof(float));
    kv->v = (float*)calloc(n, sizeof(float));
    return kv;
}

void bto_kv_free(bto_kv* kv) {
    if (!kv) return;
    free(kv->k); free(kv->v); free(kv);
}

static float round_fp16(float x) { return (float)(_Float16)x; }

/* ------------------------------------------------------------------ */
/* Engine: transformer_engine.cpp:114-251                               */
/* ------------------------------------------------------------------ */

static void mv(const bto_block_q8_0* W, const float* X, float* Y, uint32_t M, uint32_t N, int nt) {
    bto_matvec_q8_0_mt(W, X, Y, M, N, nt);
}

int bto_forward_token(const bto_model* m, bto_kv* kv, uint32_t token, uint32_t pos,
                      float theta, float* logits, float* taps, int nt) {
    const bto_config* c = &m->cfg;
    if (token >= c->vocab_size) return -2;            /* :229-231 */
    if (pos >= kv->max_seq) return -2;                /* kv_cache.cpp:18-19 */
    uint32_t D = c->dim, F = c->hidden_dim, H = c->num_heads, KVH = c->num_kv_heads, hd = c->head_dim;
    uint32_t KVD = KVH * hd;
    float* x = (float*)malloc(sizeof(float) * D);
    float* xn = (float*)malloc(sizeof(float) * D);
    float* q = (float*)malloc(sizeof(float) * D);
    float* k = (float*)malloc(sizeof(float) * KVD);
    float* v = (float*)malloc(sizeof(float) * KVD);
    float* att = (float*)malloc(sizeof(float) * D);
    float* o = (float*)malloc(sizeof(float) * D);
    float* g = (float*)malloc(sizeof(float) * F);
    float* u = (float*)malloc(sizeof(float) * F);
    float* a = (float*)malloc(sizeof(float) * F);
    float* scores = (float*)malloc(sizeof(float) * (pos + 1));

    memcpy(x, m->embed + (size_t)token * D, sizeof(float) * D);   /* :233-238 */

    for (uint32_t l = 0; l < c->num_layers; ++l) {              /* execute_layer :114-226 */
        const bto_layer* Lw = &m->layers[l];
        bto_rmsnorm(x, Lw->attn_norm, xn, 1, D, c->rms_norm_eps);  /* :117 */
        mv(Lw->q, xn, q, D, D, nt);                               /* :119-121 */
        mv(Lw->k, xn, k, KVD, D, nt);
        mv(Lw->v, xn, v, KVD, D, nt);
        bto_rope(q, q, 1, H, hd, pos, theta);                     /* :136-137 */
        bto_rope(k, k, 1, KVH, hd, pos, theta);
        size_t lo = (size_t)l * kv->max_seq * KVD;                /* kv_cache.cpp:21-26 */
        float* kc = kv->k + lo;
        float* vc = kv->v + lo;
        for (uint32_t i = 0; i < KVD; ++i) {
            kc[(size_t)pos * KVD + i] = kv->kv_fp16 ? round_fp16(k[i]) : k[i];
            vc[(size_t)pos * KVD + i] = kv->kv_fp16 ? round_fp16(v[i]) : v[i];
        }
        uint32_t ctx = pos + 1;                                   /* :148 */
        for (uint32_t i = 0; i < D; ++i) att[i] = 0.0f;
        float scale = 1.0f / sqrtf((float)hd);                    /* :158 */
        for (uint32_t h = 0; h < H; ++h) {                        /* :160-184 */
            uint32_t kvh = h / (H / KVH);
            const float* qh = q + (size_t)h * hd;
            for (uint32_t t = 0; t < ctx; ++t) {
                const float* kt = kc + ((size_t)t * KVH + kvh) * hd;
                float s = 0.0f;
                for (uint32_t d = 0; d < hd; ++d) s += qh[d] * kt[d];
                scores[t] = s * scale;
            }
            bto_softmax(scores, scores, 1, ctx);
            float* oh = att + (size_t)h * hd;
            for (uint32_t t = 0; t < ctx; ++t) {
                const float* vt = vc + ((size_t)t * KVH + kvh) * hd;
                float p = scores[t];
                for (uint32_t d = 0; d < hd; ++d) oh[d] += p * vt[d];
            }
        }
        mv(Lw->o, att, o, D, D, nt);                              /* :188-195 */
        for (uint32_t d = 0; d < D; ++d) x[d] += o[d];
        bto_rmsnorm(x, Lw->ffn_norm, xn, 1, D, c->rms_norm_eps);  /* :197-199 */
        mv(Lw->gate, xn, g, F, D, nt);
        mv(Lw->up, xn, u, F, D, nt);
        bto_silu(g, g, F);                                        /* :201-210 */
        for (uint32_t i = 0; i < F; ++i) a[i] = g[i] * u[i];      /* :212-215 */
        mv(Lw->down, a, o, D, F, nt);                             /* :220-225 */
        for (uint32_t d = 0; d < D; ++d) x[d] += o[d];
        if (taps) memcpy(taps + (size_t)l * D, x, sizeof(float) * D);
    }
    if (logits) {                                                 /* :244-250 */
        bto_rmsnorm(x, m->out_norm, xn, 1, D, c->rms_norm_eps);
        mv(m->head, xn, logits, c->vocab_size, D, nt);
    }
    free(x); free(xn); free(q); free(k); free(v); free(att); free(o);
    free(g); free(u); free(a); free(scores);
    return 0;
}
