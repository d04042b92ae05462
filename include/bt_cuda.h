/*
 * bt_cuda.h -- C ABI of the B200 (sm_100a) backend for BlockTensor's int8
 * single-token decode path.
 *
 * Plain C: pointers, sizes and status codes only.  Device pointers are CUDA
 * global-memory addresses on the current device; `stream` is a cudaStream_t
 * passed as void* (NULL = legacy default stream).  Every entry point returns a
 * status code (0 = success); bt_cuda_last_error() gives the message of the
 * last failure on the calling thread.
 *
 * Status codes mirror the exceptions of the reference so that a C++ wrapper
 * can rethrow the same types:
 *   BT_ERR_OUT_OF_RANGE      std::out_of_range     (token >= vocab,
 *                            runtime/src/transformer_engine.cpp:229-231;
 *                            pos >= max_seq, runtime/src/kv_cache.cpp:18-19)
 *   BT_ERR_RUNTIME           std::runtime_error    (I/O, bad magic,
 *                            models/model_importer.cpp:12,46,50)
 *   BT_ERR_INVALID_ARGUMENT  std::invalid_argument (n % 32 != 0,
 *                            quantization/quant_types.cpp:9-11; null buffers,
 *                            memory/memory_manager.cpp:10,29,52)
 */
#ifndef BT_CUDA_H
#define BT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BT_API __attribute__((visibility("default")))
#else
#define BT_API
#endif

#define BT_OK                    0
#define BT_ERR_UNKNOWN          -1
#define BT_ERR_OUT_OF_RANGE     -2
#define BT_ERR_RUNTIME          -3
#define BT_ERR_INVALID_ARGUMENT -4
#define BT_ERR_CUDA             -5
#define BT_ERR_OUT_OF_MEMORY    -6
#define BT_ERR_DEVICE_TIMEOUT   -7

#define BT_ABI_VERSION 1

/* KV-cache element types. */
#define BT_KV_FP32 0
#define BT_KV_FP16 1

/* Layout and field order of blocktensor::ModelConfig
 * (runtime/include/blocktensor/model_config.hpp:9-19); 36 bytes, so a
 * .btmodel header (models/model_importer.cpp:15,53) can be passed as-is. */
typedef struct bt_model_config {
    uint32_t vocab_size;
    uint32_t dim;
    uint32_t hidden_dim;
    uint32_t num_layers;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t max_seq_len;
    float    rms_norm_eps;
} bt_model_config;

/* Engine options that the reference hard-codes. */
typedef struct bt_engine_options {
    float    rope_theta;   /* 10000.0f in kernels/cpu_ref.hpp:40; 500000 for Llama-3 shapes */
    /* Tensor parallelism (no counterpart in the reference): this engine is rank
     * tp_rank of tp_world <= 8 GPUs, one process per GPU.  0 or 1: the whole
     * model on one GPU.  Rank r holds heads and KV heads [r H/W, (r+1) H/W),
     * the same FFN share of gate/up rows and of down's input columns, o-proj's
     * input columns of its heads, and vocab rows [r ceil(V/W), ...) of the
     * head matrix; embeddings and norms are whole on every rank. */
    uint32_t tp_rank;
    uint32_t tp_world;
    uint32_t reserved[5];
} bt_engine_options;

/* Bytes of a tensor-parallel exchange handle (a CUDA IPC memory handle). */
#define BT_TP_HANDLE_BYTES 64

/* One tensor of a model, as the .btmodel file stores it
 * (models/model_importer.cpp:27-41): fp32 for embeddings and norms, an array
 * of 36-byte BlockQ8_0 {float scale; int8 qs[32]} (quantization/quant_types.hpp:12-15)
 * for every projection matrix. */
typedef struct bt_tensor_view {
    const void* data;
    uint64_t    bytes;
} bt_tensor_view;

typedef struct bt_engine bt_engine;
typedef struct bt_kv bt_kv;
typedef struct bt_batch bt_batch;

/* ------------------------------------------------------------------ */
/* Library                                                              */
/* ------------------------------------------------------------------ */
BT_API int         bt_cuda_abi_version(void);
BT_API const char* bt_cuda_last_error(void);
/* Number of kernel launches this library has issued on the calling process. */
BT_API uint64_t    bt_cuda_launch_count(void);

/* ------------------------------------------------------------------ */
/* Device memory for IComputeBuffer implementations                     */
/* (runtime/include/blocktensor/backend.hpp:32-43, memory/memory_manager.cpp) */
/* ------------------------------------------------------------------ */
/* Device name, total memory and the limits that DeviceInfo
 * (backend.hpp:56-66) reports. name: at least 256 bytes. */
BT_API int bt_cuda_device_info(int device, char* name, uint64_t* total_bytes, uint32_t* max_threads_per_block,
                               uint32_t* max_shared_bytes);
/* Allocates `bytes` (zero-filled) on `device`. */
BT_API int bt_cuda_alloc(int device, uint64_t bytes, void** ptr);
BT_API int bt_cuda_free(int device, void* ptr);
/* Synchronous copies (IComputeBuffer::write / read). */
BT_API int bt_cuda_copy_h2d(int device, void* dst, const void* src, uint64_t bytes);
BT_API int bt_cuda_copy_d2h(int device, void* dst, const void* src, uint64_t bytes);
/* IComputeBackend::synchronize (backend.hpp:91). */
BT_API int bt_cuda_synchronize(int device);

/* ------------------------------------------------------------------ */
/* Quantization on device (quantization/quant_types.cpp)               */
/* ------------------------------------------------------------------ */

/* Replaces quantization::quantize_q8_0 (quant_types.cpp:8-34, decl.
 * quant_types.hpp:22).  src: n fp32; dst: n/32 BlockQ8_0 (36 B each).
 * Bit-exact with the reference for finite inputs.  n % 32 != 0 ->
 * BT_ERR_INVALID_ARGUMENT. */
BT_API int bt_cuda_quantize_q8_0(const float* src, void* dst_blocks, uint64_t n, void* stream);

/* Replaces quantization::dequantize_q8_0 (quant_types.cpp:36-48, decl. quant_types.hpp:23). */
BT_API int bt_cuda_dequantize_q8_0(const void* src_blocks, float* dst, uint64_t n, void* stream);

/* Replaces quantization::quantize_q4_0 (quant_types.cpp:50-79, decl.
 * quant_types.hpp:25): dst gets n/32 BlockQ4_0 of 20 bytes (fp32 scale, then
 * 16 bytes of 4-bit codes, element 2i in the low nibble of byte i).  Bit-exact
 * with the reference for finite inputs; n % 32 != 0 -> BT_ERR_INVALID_ARGUMENT. */
BT_API int bt_cuda_quantize_q4_0(const float* src, void* dst_blocks, uint64_t n, void* stream);
/* Replaces quantization::dequantize_q4_0 (quant_types.cpp:81-99, decl. quant_types.hpp:26). */
BT_API int bt_cuda_dequantize_q4_0(const void* src_blocks, float* dst, uint64_t n, void* stream);
/* Replaces quantization::matvec_q4_0 (quant_types.cpp:123-147, decl.
 * quant_types.hpp:29) and the "matvec_q4_0" pipeline (transformer_engine.cpp:63-65,
 * 87-91): Y[M] = W[M x N] X[N], W in the reference's 20-byte block layout. */
BT_API int bt_cuda_matvec_q4_0(const void* W_blocks, const float* X, float* Y, uint32_t M, uint32_t N, void* stream);

/* Replaces quantization::matvec_q8_0 (quant_types.cpp:101-121, decl.
 * quant_types.hpp:28) and the "matvec_q8_0" pipeline of the Vulkan backend
 * (kernels/glsl/matvec_q8_0.comp, bound at transformer_engine.cpp:76-77):
 * Y[M] = W[M x N] X[N] with W in the reference's 36-byte block layout. */
BT_API int bt_cuda_matvec_q8_0(const void* W_blocks, const float* X, float* Y,
                        uint32_t M, uint32_t N, void* stream);

/* Split reference blocks into the device layout: qs[M][K] int8 (rows 16-byte
 * aligned) and scales[M][K/32] fp32.  No reference counterpart (the reference
 * keeps the 36-byte blocks); this is the upload repack of
 * MemoryManager::copy_host_to_device (memory/memory_manager.cpp:22-42). */
BT_API int bt_cuda_repack_q8_0(const void* W_blocks, int8_t* qs, float* scales,
                        uint32_t M, uint32_t K, void* stream);

/* Repack reference blocks into the tensor-core tile layout used by the decode
 * engine: rows in tiles of 128, each row tile as K/32 tiles of 4608 bytes (the
 * 128x32 int8 block in the UMMA K-major no-swizzle canonical layout, then its
 * 128 fp32 scales in row order).  `units` must be 16-byte aligned and hold
 * ceil(M/128) * (K/32) * 4608 bytes; padding rows are zeroed.  Upload
 * repack of MemoryManager::copy_host_to_device (memory/memory_manager.cpp:22-42). */
BT_API int bt_cuda_pack_q8_units(const void* W_blocks, void* units, uint32_t M, uint32_t K, void* stream);

/* y[m] = sum_k W[m][k] x[k] on the tile layout: quantization::matvec_q8_0
 * (quant_types.cpp:101-121) on the tensor cores (tcgen05 int8 MMA: exact block
 * dot products, every 32-element block of x in 22-bit fixed point with its own
 * exponent, fp32 block accumulation), split evenly over all SMs.  units and x
 * must be 16-byte aligned; M <= 1048576, K <= 48384.  Scratch for row tiles
 * split between CTAs comes from a per-device workspace the library allocates
 * on the first call.  Returns once the GEMV has finished on `stream` (like the
 * reference's synchronous matvec): BT_ERR_DEVICE_TIMEOUT when a wait inside
 * the kernel gave up after its 2 s limit (y is then not valid). */
BT_API int bt_cuda_gemv_q8_units(const void* units, const float* x, float* y, uint32_t M, uint32_t K,
                                 void* stream);

/* bt_cuda_gemv_q8_units for callers that cannot allocate device memory (no
 * counterpart in the reference).  An engine that reserves all device memory up
 * front in its own pool, a runtime whose allocator must account for every
 * byte, or a decode loop that must never hit cudaMalloc's implicit device
 * synchronisation cannot let the library cudaMalloc a workspace on first use.
 * This variant calls no cudaMalloc, cudaFree or allocating library routine: its
 * scratch (partial sums of row groups split between CTAs, arrival tickets, a
 * timeout flag) is a fixed 288 KB device array inside the library, held by
 * every GPU that loads the library until the process exits.  Limits: M <=
 * 1048576 rows, K <= 48384, at most 256 SMs; larger sizes return
 * BT_ERR_INVALID_ARGUMENT.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make that
 * first call before any stream capture.  Every call on a device shares the one
 * array and each call clears its tickets first, so calls that overlap on the
 * GPU (concurrent streams) race and must be serialised by the caller.  Same
 * inputs, outputs, alignment, arithmetic and completion (returns once the GEMV
 * has finished; BT_ERR_DEVICE_TIMEOUT when a device wait gave up) as
 * bt_cuda_gemv_q8_units. */
BT_API int bt_cuda_gemv_q8_units_noalloc(const void* units, const float* x, float* y, uint32_t M, uint32_t K,
                                         void* stream);

/* Microbenchmark of the standalone int8 GEMV/GEMM kernels (no counterpart in
 * the reference; the dequant-GEMV benchmark): `iters` launches of kernel
 * `kind` back to back on `stream` after 3 warm-up launches, cycling through
 * n_copies weight copies copy_stride bytes apart (together larger than L2,
 * every launch streams its weights from HBM), reporting the mean device time
 * per launch from CUDA events.  kind 0: tensor-core GEMV on the tile layout
 * (B = 1); kind 1: tensor-core GEMM on the tile layout for B token rows (its
 * token image included); kind 2: CUDA-core GEMV on the split layout, qs
 * [M][K] followed by the scales [M][K/32] (B <= 16).  X [B][K], Y [B][M]. */
BT_API int bt_cuda_gemv_bench(int kind, const void* w, const float* X, float* Y, uint32_t M, uint32_t K, uint32_t B,
                              uint32_t n_copies, uint64_t copy_stride, uint32_t iters, void* stream,
                              float* us_per_call);

/* Fault injection on the host, for tests of the standalone GEMVs' timeout
 * reporting (no counterpart in the reference): sets the bounded-wait flag of
 * bt_cuda_gemv_q8_units (noalloc = 0) or of bt_cuda_gemv_q8_units_noalloc
 * (noalloc = 1) on `device`, as an expired device wait would, so that the next
 * call of that entry point returns BT_ERR_DEVICE_TIMEOUT and clears it.  No
 * GPU fault, no hang. */
BT_API int bt_cuda_gemv_inject_timeout(int device, int noalloc);

/* Y[t][m] = sum_k W[m][k] X[t][k] for T token rows on the tile layout: the
 * reference's matvec_q8_0 (quant_types.cpp:101-121) for every row of X, as one
 * tensor-core GEMM (tcgen05 int8 MMA over 32-token groups: exact block dot
 * products of every token's 22-bit per-block fixed point digits, fp32 block
 * accumulation in the reference's block order).  This is the contraction of
 * prompt prefill and batched decode, exposed for its parity tests.  X [T][K]
 * and Y [T][M] are fp32 row-major; units and X 16-byte aligned.  Returns once
 * finished on `stream`; scratch (the digit image of X) is allocated
 * stream-ordered per call.  BT_ERR_DEVICE_TIMEOUT when a device wait gave up. */
BT_API int bt_cuda_gemm_q8_units(const void* units, const float* X, float* Y, uint32_t M, uint32_t K, uint32_t T,
                                 void* stream);

/* Batched int8 GEMV on the device layout: Y[b][m] = sum_k W[m][k] X[b][k],
 * b < B, for the dequant-GEMV microbenchmark.  B = 1 is the
 * reference's matvec_q8_0 (quant_types.cpp:101-121) on repacked weights. */
BT_API int bt_cuda_gemv_q8(const int8_t* qs, const float* scales, const float* X, float* Y,
                    uint32_t M, uint32_t K, uint32_t B, void* stream);

/* ------------------------------------------------------------------ */
/* Math primitives (kernels/cpu_ref.hpp, sampler.hpp) on device         */
/* ------------------------------------------------------------------ */
/* cpu_ref::rmsnorm (cpu_ref.hpp:11-28); pipeline "rmsnorm", push {dim, eps}. */
BT_API int bt_cuda_rmsnorm(const float* in, const float* w, float* out, uint32_t rows, uint32_t dim,
                    float eps, void* stream);
/* cpu_ref::rope (cpu_ref.hpp:30-53) with the base as a parameter; pipeline "rope". */
BT_API int bt_cuda_rope(const float* in, float* out, uint32_t seq, uint32_t heads, uint32_t head_dim,
                 uint32_t pos, float theta, void* stream);
/* cpu_ref::softmax (cpu_ref.hpp:55-72); pipeline "softmax". */
BT_API int bt_cuda_softmax(const float* in, float* out, uint32_t rows, uint32_t dim, void* stream);
/* cpu_ref::silu (cpu_ref.hpp:74-79); pipeline "silu". */
BT_API int bt_cuda_silu(const float* in, float* out, uint32_t n, void* stream);
/* sampling::sample_greedy (sampler.hpp:11-13): first maximum wins. out: device uint32. */
BT_API int bt_cuda_argmax(const float* logits, uint32_t n, uint32_t* out, void* stream);
/* sampling::sample_top_p_top_k (sampler.hpp:15-85) on the device: logits
 * [vocab] divided by the temperature, the top_k largest kept in decreasing
 * order, probabilities exp(l - max) / sum, cut where the running sum reaches
 * top_p, renormalised, and the token where the running sum first reaches r, r
 * the first std::uniform_real_distribution<float>(0, 1) draw of
 * std::mt19937(seed) (computed on the host as the reference does).
 * temperature <= 0: greedy.  Candidates: top_k in 1..4096 (or all of a vocab
 * of at most 4096); equal logits are ordered by id.  out: device uint32. */
BT_API int bt_cuda_sample_top_p_top_k(const float* logits, uint32_t vocab, float temperature, float top_p,
                                      uint32_t top_k, uint64_t seed, uint32_t* out, void* stream);

/* ------------------------------------------------------------------ */
/* Engine (runtime/include/blocktensor/transformer_engine.hpp:12-56)    */
/* ------------------------------------------------------------------ */

/* Replaces TransformerEngine::TransformerEngine(backend, weights)
 * (transformer_engine.hpp:14): creates the device context and allocates
 * device-resident weights for `cfg` on CUDA device `device`.  opt may be NULL
 * (rope_theta 10000).  Weights are loaded next by bt_engine_load or
 * bt_engine_generate. */
BT_API int bt_engine_create(int device, const bt_model_config* cfg, const bt_engine_options* opt,
                     bt_engine** out);
BT_API int bt_engine_destroy(bt_engine* e);

/* Loads the 3 + 9*num_layers tensors of a model in .btmodel order
 * (models/model_importer.cpp:69-85: embed, out_norm, head, then per layer
 * attn_norm, ffn_norm, q, k, v, o, gate, up, down).  on_device = 0: host
 * pointers (importer output, IComputeBuffer::map of HOST_VISIBLE buffers);
 * on_device = 1: device pointers.  Matrices are Q8_0 (36-byte blocks) or, for
 * an INT4 model, Q4_0 (20-byte blocks; told apart by the head's size), and are
 * repacked on the device into int8 tiles (Q4_0 codes as code - 8 with the
 * block scale, the values matvec_q4_0 multiplies). */
BT_API int bt_engine_load(bt_engine* e, const bt_tensor_view* tensors, uint32_t n_tensors, int on_device);

/* Seeded synthetic weights generated on the device: matrices
 * approximately N(0, sigma) (sum of four 16-bit uniforms), quantized with the
 * device quantizer; embeddings N(0, sigma) fp32; norms 1.0.  Bit-identical to
 * the CPU oracle's generator for the same seed. */
BT_API int bt_engine_generate(bt_engine* e, uint64_t seed, float sigma);

/* Replaces KVCache(MemoryManager&, num_layers, max_seq_len, kv_heads, head_dim)
 * (runtime/include/blocktensor/kv_cache.hpp:12): device-resident cache of
 * max_seq positions in fp32 (BT_KV_FP32) or fp16 (BT_KV_FP16). */
BT_API int bt_kv_create(bt_engine* e, uint32_t max_seq, int kv_dtype, bt_kv** out);
BT_API int bt_kv_destroy(bt_kv* kv);
/* Reads one layer in the reference layout [max_seq][kv_heads][head_dim] as fp32
 * (runtime/src/kv_cache.cpp:21-23).  k, v: host, max_seq*kv_heads*head_dim floats. */
BT_API int bt_kv_read_layer(bt_kv* kv, uint32_t layer, float* k, float* v);

/* Replaces TransformerEngine::forward_single_token(token, pos, KVCache&)
 * (transformer_engine.hpp:17, transformer_engine.cpp:228-251): one decode
 * step.  logits: host [vocab] or NULL; argmax: host or NULL (greedy token,
 * sampler.hpp:11-13).  token >= vocab or pos >= max_seq -> BT_ERR_OUT_OF_RANGE. */
BT_API int bt_engine_forward_token(bt_engine* e, bt_kv* kv, uint32_t token, uint32_t pos,
                            float* logits, uint32_t* argmax);

/* The prompt-then-greedy loop of bt_infer/bench_runner
 * (tools/bt_infer.cpp:116-136, benchmarks/bench_runner.cpp:105-119) on the
 * device: positions pos0 .. pos0+n_prompt+n_gen-1, the step at position p
 * consuming prompt[p-pos0] while p-pos0 < n_prompt and the previous step's
 * argmax afterwards.  tokens_out (host, n_prompt + n_gen + 1 entries) gets the
 * token consumed at each position plus the final argmax.  No host round trip
 * between steps. */
BT_API int bt_engine_decode(bt_engine* e, bt_kv* kv, const uint32_t* prompt, uint32_t n_prompt,
                     uint32_t pos0, uint32_t n_gen, uint32_t* tokens_out);

/* Prompt prefill: the batched form of the reference's prompt loop
 * (benchmarks/bench_runner.cpp:107-109, tools/bt_infer.cpp:116-125).  The
 * positions pos0 .. pos0 + n_prompt - 2 run through every layer together as
 * tensor-core GEMMs (chunks of up to 512 tokens) with causal attention over the
 * cache, filling their K/V rows; the sequence is then left as
 * bt_engine_begin(prompt, n_prompt, pos0) leaves it after n_prompt - 1 steps:
 * the next bt_engine_steps step processes prompt[n_prompt - 1] at position
 * pos0 + n_prompt - 1 (its logits and greedy token come from the decode step)
 * and decoding continues greedily.  Needs the persistent step kernel and no
 * tensor parallelism.  Errors as bt_engine_begin; BT_ERR_DEVICE_TIMEOUT when a
 * device wait gave up. */
BT_API int bt_engine_prefill(bt_engine* e, bt_kv* kv, const uint32_t* prompt, uint32_t n_prompt, uint32_t pos0);
/* Token consumed at positions pos0 .. pos0 + n - 1 (the prompt, then the
 * greedy tokens; entry max_seq is the argmax after the last position). */
BT_API int bt_kv_read_tokens(bt_kv* kv, uint32_t pos0, uint32_t n, uint32_t* out);

/* Per-layer residual-stream taps: when enabled, every subsequent step records
 * x after each layer; bt_engine_read_taps copies [num_layers][dim] fp32 of the
 * last step to host. */
BT_API int bt_engine_set_taps(bt_engine* e, int enable);
BT_API int bt_engine_read_taps(bt_engine* e, float* taps);

/* Per-phase device timestamps of the persistent step kernel, for latency
 * analysis (no counterpart in the reference).  When enabled, every subsequent
 * step records, for every phase p (5 per layer, then the head) and CTA c, the
 * %globaltimer nanoseconds of: [0] the consumers passing the phase's counter
 * wait, [1] the input digits ready in shared memory, [2] the first row tile's
 * sums reaching the finisher, [3] the CTA's last write of the phase, [4] and
 * [5] the producer issuing the phase's first and last weight copy; slots 6-7
 * are unused.  bt_engine_read_trace copies the last step's
 * [5 L + 1][SMs][8] words (n_words must equal that count).  The recording
 * costs a few stores per phase; off by default. */
BT_API int bt_engine_set_trace(bt_engine* e, int enable);
BT_API int bt_engine_read_trace(bt_engine* e, uint64_t* out, uint64_t n_words);

/* Device-side timing hooks for benchmarks: run n decode steps on `stream`
 * with no host synchronisation; the device state (position, current token)
 * continues from the last call. */
BT_API int bt_engine_begin(bt_engine* e, bt_kv* kv, const uint32_t* prompt, uint32_t n_prompt, uint32_t pos0);
BT_API int bt_engine_steps(bt_engine* e, bt_kv* kv, uint32_t n, void* stream);
/* The engine's own stream (cudaStream_t), on which every call above runs. */
BT_API void* bt_engine_stream(bt_engine* e);
/* Per-kernel timing: runs n_steps decode steps eagerly (no graph, no
 * overlap between kernels) with a CUDA event after every launch and adds the
 * device time of each kernel kind into ms_by_kind[6] = {qkv, attention,
 * o-proj, gate/up, down, head}.  Advances the sequence like bt_engine_steps. */
BT_API int bt_engine_profile(bt_engine* e, bt_kv* kv, uint32_t n_steps, float* ms_by_kind);
/* Position, current token and last argmax of the sequence (host copy).
 * Returns BT_ERR_DEVICE_TIMEOUT (outputs still filled) when a device wait of
 * an earlier step expired. */
BT_API int bt_kv_state(bt_kv* kv, uint32_t* pos, uint32_t* token, uint32_t* last_argmax);
/* Tensor parallelism, after bt_engine_create with tp_world > 1 and before the
 * first decode step: every rank writes its exchange handle
 * (BT_TP_HANDLE_BYTES bytes) with bt_engine_tp_handle, the ranks gather the
 * handles in rank order (torch.distributed, MPI, a file, ...), and every rank
 * passes all tp_world handles to bt_engine_tp_connect, which maps the other
 * ranks' buffers (CUDA IPC over NVLink).  The decode step then adds o-proj's
 * and down's partial sums across the ranks inside the persistent kernel
 * (every rank stores its row tiles into every rank's buffer and adds all ranks'
 * in rank order) and agrees on the greedy token the same way; all ranks must
 * run the same calls in the same order.  Logits of bt_engine_forward_token
 * are this rank's vocab rows only (written at their offset). */
BT_API int bt_engine_tp_handle(bt_engine* e, void* handle);
BT_API int bt_engine_tp_connect(bt_engine* e, const void* handles);
/* Fault injection on the host, for tests of the device timeouts (no
 * counterpart in the reference): sets the sequence's device step count so
 * that the phase barriers of its next persistent-kernel step can never be
 * reached.  That step's waits then expire after their 2 s limit, the kernel
 * finishes (every later wait of the step returns at once), and the error flag
 * is set for bt_kv_state / bt_engine_decode to report.  No GPU fault and no
 * hang: the context stays usable, and bt_engine_begin or
 * bt_engine_forward_token resets the state.  BT_ERR_INVALID_ARGUMENT when the
 * engine runs the launch-per-operation step. */
BT_API int bt_kv_inject_stall(bt_kv* kv);
/* Kernel launches of one decode step and the algorithmic HBM bytes it moves
 * when the step processes position context-1: weights (int8 + fp32 scales),
 * norms, one embedding row, KV read of `context` positions and the KV write. */
BT_API int bt_kv_step_info(bt_kv* kv, uint32_t context, uint64_t* launches, uint64_t* bytes);

/* ------------------------------------------------------------------ */
/* Batched decode (no reference counterpart: the reference KVCache holds one */
/* sequence, runtime/src/kv_cache.cpp:6-15; a batch of n sequences is n     */
/* independent forward_single_token loops, decoded here in one pass)        */
/* ------------------------------------------------------------------ */

/* n_seq sequences of up to max_seq positions each (KV caches fp32 or fp16) on
 * the engine's device.  Each step processes every sequence's current token at
 * its own position: the projections as tensor-core GEMMs over the batch (the
 * weights stream once per step), attention per sequence over its own cache,
 * the head with a greedy argmax per sequence.  No tensor parallelism; shard
 * sequences over GPUs by giving each GPU its own engine and batch. */
BT_API int bt_batch_create(bt_engine* e, uint32_t n_seq, uint32_t max_seq, int kv_dtype, bt_batch** out);
BT_API int bt_batch_destroy(bt_batch* b);
/* Sequence s starts with `prompt`: positions 0 .. n_prompt - 2 are prefilled
 * (as bt_engine_prefill), and its next step processes prompt[n_prompt - 1] at
 * position n_prompt - 1.  Every sequence of a contiguous batch must be started
 * before steps run; in a paged batch a slot's previous sequence is released
 * first. */
BT_API int bt_batch_prefill(bt_batch* b, uint32_t s, const uint32_t* prompt, uint32_t n_prompt);
/* n decode steps of every sequence (greedy), on `stream` (NULL: the engine's);
 * BT_ERR_OUT_OF_RANGE when a sequence would pass max_seq. */
BT_API int bt_batch_steps(bt_batch* b, uint32_t n, void* stream);
/* Token consumed by sequence s at positions pos0 .. pos0 + n - 1 (prompt, then
 * greedy tokens); BT_ERR_DEVICE_TIMEOUT when a device wait gave up. */
BT_API int bt_batch_read_tokens(bt_batch* b, uint32_t s, uint32_t pos0, uint32_t n, uint32_t* out);
/* Each sequence's newest token (the greedy token of its last step; for a
 * sequence that has not stepped, its last prompt token), [n_seq] in one copy:
 * the per-step read-back of a serving loop.  BT_ERR_DEVICE_TIMEOUT as above. */
BT_API int bt_batch_read_current(bt_batch* b, uint32_t* out);
/* Logits of every sequence's last step, [n_seq][vocab] fp32 (host). */
BT_API int bt_batch_read_logits(bt_batch* b, float* out);
/* Algorithmic HBM bytes of the next step: weights once, norms, one embedding
 * row per sequence, every sequence's K/V read and written. */
BT_API int bt_batch_step_info(bt_batch* b, uint64_t* bytes);

/* Paged KV for serving (replaces the reference's one contiguous single-
 * sequence buffer per layer, runtime/src/kv_cache.cpp:6-15): a batch of n_seq
 * sequence slots whose K/V live in one pool of n_pages pages of page_tokens
 * positions (a power of two in [16, 4096]); a page holds every layer's
 * [kv_heads][page_tokens][head_dim] rows, K and V in two pools.  A slot takes
 * pages as its sequence grows (bt_batch_prefill, bt_batch_steps) and gives
 * them back with bt_batch_release; max_seq bounds one sequence.  Slots that
 * hold no sequence are skipped by the steps.  Results are those of
 * bt_batch_create's contiguous caches.  A prefill or steps call that needs
 * more pages than are free returns BT_ERR_OUT_OF_MEMORY and takes none.
 * Calls on one batch are made from one host thread; prefill and release
 * synchronise the engine's stream. */
BT_API int bt_batch_create_paged(bt_engine* e, uint32_t n_seq, uint32_t max_seq, uint32_t page_tokens,
                                 uint32_t n_pages, int kv_dtype, bt_batch** out);
/* Ends the sequence of slot s: its pages return to the pool, the slot idles
 * until the next bt_batch_prefill of s.  BT_ERR_INVALID_ARGUMENT on a batch
 * without a page pool. */
BT_API int bt_batch_release(bt_batch* b, uint32_t s);
/* Free and total pages of the pool (0 and 0 for a contiguous batch). */
BT_API int bt_batch_pages(bt_batch* b, uint32_t* free_pages, uint32_t* total_pages);

#ifdef __cplusplus
}
#endif
#endif /* BT_CUDA_H */
