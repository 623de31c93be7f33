/*
 * b200_infer.h -- C ABI of the B200-native (sm_100a) kernels and runtime for the
 * Infer-LLM F32 Qwen3 inference path.
 *
 * The reference's kernel seam is
 *     namespace CUDA_F32 { cudaError_t compute_<op>(Tensor* dst, cudaStream_t); }
 * (include/kernels/cuda/kernel_f32.hpp:8-28), which hands the whole C++ Tensor
 * struct across the call. This header replaces it with plain pointers, int64
 * sizes and explicit strides, so any host language can bind it (ctypes, cgo,
 * JNI). Conventions shared by every entry point:
 *
 *   - Layouts follow the reference's ggml convention (dims[0] fastest): a
 *     weight "[K, N]" is N rows of K contiguous floats; activations "[K, M]"
 *     are M rows (tokens) of K floats.
 *   - All tensor pointers are device pointers on the current CUDA device unless
 *     the name says host_. `stream` is a cudaStream_t (NULL = legacy stream).
 *   - Entry points validate sizes on the host, enqueue work and return; they
 *     never allocate, never synchronize and never trap. Scratch memory comes
 *     from a caller-provided workspace whose size a *_workspace_bytes() query
 *     returns.
 *   - Device-side checks (token ids, positions) never fault: an offending row
 *     is skipped and the first error is recorded in an optional device status
 *     word (int32, 0 = ok) that the caller reads after the step.
 *   - Return value: B200_OK or a B200_ERR_* code. The reference maps CUDA
 *     failures to std::errc::io_error (include/cuda_util.hpp:7-16) and an
 *     unknown op to std::errc::not_supported (src/backends/cuda_backend.cpp:237).
 */
#ifndef B200_INFER_H
#define B200_INFER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_OK 0
#define B200_ERR_INVALID_ARGUMENT 1 /* std::errc::invalid_argument */
#define B200_ERR_NOT_SUPPORTED 2    /* std::errc::not_supported */
#define B200_ERR_OUT_OF_RANGE 3     /* bad token id / position / KV capacity */
#define B200_ERR_CUDA 4             /* std::errc::io_error in the reference */
#define B200_ERR_NO_MEMORY 5        /* std::errc::not_enough_memory */
#define B200_ERR_DEVICE_CHECK 6     /* a device-side check set the status word */
#define B200_ERR_TIMEOUT 7          /* a bounded device wait gave up */
#define B200_ERR_NUMERIC 8          /* NaN / +inf logits (sampler.cpp:53) */

/* Device status word codes (written by kernels, read by the host). */
#define B200_DEV_BAD_TOKEN 1
#define B200_DEV_BAD_POSITION 2
#define B200_DEV_BAD_LOGITS 3
#define B200_DEV_TIMEOUT 4

/* Precision of a matrix product. */
#define B200_PREC_FFMA 0 /* exact F32 FFMA (reference tolerance 1e-5) */
#define B200_PREC_TF32 1 /* tcgen05 tensor cores, TF32 inputs, F32 accumulate */

const char *b200_status_string(int status);
/* 1 if the library was built for and runs on an sm_100 device, else 0. */
int b200_device_supported(int device);

/* ------------------------------------------------------------------------
 * Single ops: one entry point per reference CUDA_F32::compute_* function.
 * ------------------------------------------------------------------------ */

/* out[t*N + n] = sum_k x[t*K + k] * w[n*K + k]   (y = x . W^T)
 * Replaces CUDA_F32::compute_mul_mat (kernel_f32.hpp:18, kernel_f32.cu:180-205).
 * M <= 4 uses the HBM-streaming GEMV (TMA bulk-staged weight tiles); larger M
 * uses the tiled GEMM selected by `precision`. */
int b200_mul_mat(const float *w, const float *x, float *out, int64_t K, int64_t N, int64_t M,
                 int precision, void *stream);
/* b200_mul_mat with a split-K workspace: where the M x N tiles leave SMs idle
 * (prompts up to a few hundred tokens on the layer shapes) K is split across CTAs,
 * each split's partial sums go to the workspace and are added in split order
 * (deterministic), so every SM takes part. `workspace` (16-byte aligned, contents
 * ignored) of b200_mul_mat_workspace_bytes(K, N, M, precision) bytes enables every
 * split; a smaller one fewer, NULL none. */
int b200_mul_mat_ws(const float *w, const float *x, float *out, int64_t K, int64_t N, int64_t M,
                    int precision, void *workspace, size_t workspace_bytes, void *stream);
size_t b200_mul_mat_workspace_bytes(int64_t K, int64_t N, int64_t M, int precision);

/* Row-wise RMSNorm over D contiguous floats: y = x * rsqrt(mean(x^2) + eps) * gamma.
 * Replaces CUDA_F32::compute_rms_norm (kernel_f32.hpp:14, kernel_f32.cu:60-90). */
int b200_rms_norm(const float *x, const float *gamma, float *out, int64_t D, int64_t rows,
                  float eps, void *stream);

/* NeoX half-split RoPE of x [D, H, T] (x may equal out). Angles come from the
 * reference's table layout [n_ctx][D/2] (theta_table, device memory), row pos[t].
 * A position outside [0, n_ctx) leaves its rows untouched and records
 * B200_DEV_BAD_POSITION (the reference kernel traps instead, kernel_f32.cu:250-253).
 * Replaces CUDA_F32::compute_rope (kernel_f32.hpp:22, kernel_f32.cu:273-301). */
int b200_rope(const float *x, const int32_t *pos, const float *theta_table, int64_t n_ctx,
              float *out, int64_t D, int64_t H, int64_t T, int32_t *dev_status, void *stream);

/* Fused per-head RMSNorm + RoPE (+ optional KV-cache write) for Q and K of one step.
 * q_in [Dq*Hq] and k_in [D*Hkv] per token (row strides q_ld / k_ld floats), gammas
 * [D]. Angles are float(double(pos) * freq[j]) with freq[j] = 1.0f/powf(theta, 2j/D),
 * which reproduces the reference table (graph.cpp:119-131) bit for bit. q_out gets
 * [D, Hq, T]; k_out (may be a KV-cache slot) gets [D, Hkv, T] with token stride
 * k_out_ld floats. v_in/v_out optionally copy V into its cache slot in the same pass.
 * Chains reference nodes rms_norm(q), rms_norm(k), rope(q), rope(k), cpy(k), cpy(v)
 * (Qwen3.cpp:66-84). */
int b200_qk_norm_rope(const float *q_in, int64_t q_ld, const float *k_in, int64_t k_ld,
                      const float *v_in, int64_t v_ld, const float *q_gamma,
                      const float *k_gamma, const float *freq, const int32_t *pos,
                      float *q_out, float *k_out, int64_t k_out_ld, float *v_out,
                      int64_t v_out_ld, int64_t D, int64_t Hq, int64_t Hkv, int64_t T,
                      int64_t n_ctx, float eps, int32_t *dev_status, void *stream);

/* Host helper: freq[j] = 1.0f / powf(theta, 2.0f*j/D), j < D/2 (host memory). */
void b200_rope_freqs(float theta, int64_t D, float *host_freq);

/* Causal GQA attention over a KV cache.
 * q [D, Hq, Tq] contiguous; K/V element (token t, kv head h, dim d) at
 * k[t*k_tok_stride + h*k_head_stride + d] (the reference cache is token-major:
 * k_tok_stride = Hkv*D, k_head_stride = D); out [D, Hq, Tq].
 * Key j is visible to query i iff j <= n_past + i; Tkv = n_past + Tq.
 * scale <= 0 selects 1/sqrt(D). Decode (Tq == 1) uses split-KV flash-decoding over
 * about 128 keys per CTA: with a workspace of b200_flash_attn_workspace_bytes(...)
 * bytes the K/V rows are staged by bulk copies (TMA engine) into a shared-memory
 * ring and the splits' partials are merged through the workspace by the last CTA
 * of each KV head. The workspace must be zero-filled before its first use and may
 * be reused by later calls (every completed call leaves it ready); after a call that
 * reported a device error, zero it again. With `workspace` NULL (or smaller), at
 * most 16 splits per KV head form a thread-block cluster and merge through
 * distributed shared memory instead. Tq > 1 uses a tiled online-softmax kernel and
 * needs no workspace.
 * Replaces CUDA_F32::compute_flash_attn (kernel_f32.hpp:24, kernel_f32.cu:452-511),
 * which mallocs an Hq*Tq*Tkv score matrix and synchronizes on every call. */
int b200_flash_attn(const float *q, const float *k, const float *v, float *out, int64_t D,
                    int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tkv, int64_t n_past,
                    float scale, int64_t k_tok_stride, int64_t k_head_stride,
                    int64_t v_tok_stride, int64_t v_head_stride, void *workspace,
                    size_t workspace_bytes, void *stream);
size_t b200_flash_attn_workspace_bytes(int64_t D, int64_t Hq, int64_t Hkv, int64_t Tq,
                                       int64_t Tkv);
/* b200_flash_attn with a precision for Tq > 1: B200_PREC_FFMA (exact F32, as
 * b200_flash_attn) or B200_PREC_TF32 (head_dim 128: S = Q K^T and O = P V on the
 * tcgen05 tensor cores with TF32 inputs and F32 accumulation, scores and O in tensor
 * memory; other head sizes fall back to the exact kernel). Decode is unaffected. */
int b200_flash_attn_ex(const float *q, const float *k, const float *v, float *out, int64_t D,
                       int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tkv, int64_t n_past,
                       float scale, int64_t k_tok_stride, int64_t k_head_stride,
                       int64_t v_tok_stride, int64_t v_head_stride, void *workspace,
                       size_t workspace_bytes, void *stream, int32_t precision);

/* Paged KV cache (the kernel side of a paged KVStrategy: KVCacheConfig::block_tokens
 * > 0, include/kvcache/kvutil.hpp:43-44, which the reference declares but does not
 * implement). K and V live in blocks of block_tokens tokens; k_blocks / v_blocks are
 * device arrays of n_blocks device pointers, entry i the block of positions
 * [i * block_tokens, (i + 1) * block_tokens) of the sequence, in the NaiveKVStorage
 * layout with capacity block_tokens: element (token t of the block, KV head h, dim d)
 * at block[(t * Hkv + h) * D + d]. The blocks may be anywhere (the reference's own
 * storage objects, or slices of one pool).
 *
 * b200_paged_kv_write: the K / V rows of T new tokens (k_src, v_src: [T][Hkv][D] with
 * token stride src_tok_stride floats, 16-byte aligned) into their blocks at positions
 * pos0 .. pos0 + T - 1 (B200_ERR_OUT_OF_RANGE past n_blocks * block_tokens). */
int b200_paged_kv_write(const float *k_src, const float *v_src, int64_t src_tok_stride,
                        float *const *k_blocks, float *const *v_blocks, int64_t n_blocks,
                        int64_t block_tokens, int64_t pos0, int64_t T, int64_t Hkv, int64_t D,
                        int32_t *dev_status, void *stream);
/* Causal GQA attention of q [Tq][Hq][D] against the paged cache's positions
 * [0, Tkv) (Tkv = n_past + Tq, already written), out [Tq][Hq][D]; the same numerics
 * contract as b200_flash_attn. Decode (Tq == 1) reads K / V through the block tables
 * (split-KV, splits merged through the workspace; its counters must be zero before
 * the first use, as for b200_flash_attn); Tq > 1 gathers [0, Tkv) into the workspace
 * and runs the tiled prefill kernel. A null block pointer met on the way records
 * B200_DEV_BAD_POSITION in dev_status and reads as zeros. head_dim 64 or 128. */
int b200_flash_attn_paged(const float *q, const float *const *k_blocks, const float *const *v_blocks,
                          int64_t n_blocks, int64_t block_tokens, float *out, int64_t D, int64_t Hq,
                          int64_t Hkv, int64_t Tq, int64_t Tkv, int64_t n_past, float scale,
                          void *workspace, size_t workspace_bytes, int32_t *dev_status, void *stream);
size_t b200_flash_attn_paged_workspace_bytes(int64_t D, int64_t Hq, int64_t Hkv, int64_t Tq,
                                             int64_t Tkv);

/* Elementwise ops of the reference graph (n elements).
 * CUDA_F32::compute_silu / compute_mul / compute_add (kernel_f32.cu:529-630). */
int b200_silu(const float *x, float *out, int64_t n, void *stream);
int b200_mul(const float *a, const float *b, float *out, int64_t n, void *stream);
int b200_add(const float *a, const float *b, float *out, int64_t n, void *stream);
/* out = up * silu(gate): silu + mul of Qwen3.cpp:109-112 in one pass. */
int b200_swiglu(const float *gate, const float *up, float *out, int64_t n, void *stream);

/* Embedding gather out[t] = table[ids[t]] (rows of D floats, n_rows rows).
 * An id outside [0, n_rows) leaves its row untouched and records B200_DEV_BAD_TOKEN.
 * Replaces CUDA_F32::compute_get_rows (kernel_f32.hpp:16, kernel_f32.cu:107-138). */
int b200_get_rows(const float *table, const int32_t *ids, float *out, int64_t D, int64_t n,
                  int64_t n_rows, int32_t *dev_status, void *stream);

/* Device-to-device copy of `bytes` (the reference's CPY / RESHAPE nodes,
 * kernel_f32.cu:210-240, 305-319). */
int b200_copy(void *dst, const void *src, size_t bytes, void *stream);

/* Greedy sampler on the device: out_id = first index of the maximum of logits[n];
 * NaN or +inf -> out_id = -1 and B200_DEV_BAD_LOGITS (sampler.cpp:42-65).
 * workspace: b200_argmax_workspace_bytes(n). */
int b200_argmax(const float *logits, int64_t n, int32_t *out_id, void *workspace,
                size_t workspace_bytes, int32_t *dev_status, void *stream);
size_t b200_argmax_workspace_bytes(int64_t n);

/* Allocation-free b200_argmax. This entry point has no counterpart in the
 * reference: it serves callers that cannot allocate a device workspace, such as a
 * kernel seam that receives only tensors and a stream (the reference's
 * CUDA_F32::compute_* has no workspace argument) or a host that must not call
 * cudaMalloc between steps (an allocation synchronises the device). Its scratch
 * is a fixed library-owned device array of B200_ARGMAX_NOALLOC_SCRATCH bytes,
 * held by every GPU that loads the library until the process exits; the call
 * itself allocates nothing. Limits: n <= B200_ARGMAX_NOALLOC_MAX_N (larger n is
 * rejected with B200_ERR_INVALID_ARGUMENT). Every call looks up the array's device
 * address (cudaGetSymbolAddress); the first call on a device also loads the
 * library's device code there, so make it before any stream capture on that
 * device. All calls share the one array (the counter in it
 * is cleared at the start of every call): calls that overlap on the GPU, on any
 * streams of the same device, race and must be serialised by the caller.
 * Results equal b200_argmax's. */
#define B200_ARGMAX_NOALLOC_SCRATCH 8192
#define B200_ARGMAX_NOALLOC_MAX_N 2147483647LL
int b200_argmax_noalloc(const float *logits, int64_t n, int32_t *out_id, int32_t *dev_status,
                        void *stream);

/* ------------------------------------------------------------------------
 * Qwen3 engine: device-resident weights, KV cache and activation arenas, the
 * fused per-layer kernel sequence, CUDA-graph decode. It is the runtime behind
 * the reference's Backend::compute for a Qwen3 graph (Qwen3.cpp:4-136,
 * scheduler.cpp:4-28) without per-step graph building or allocation.
 * ------------------------------------------------------------------------ */
typedef struct b200_qwen3_config {
    int32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, head_dim, n_ff;
    int32_t n_ctx_train;
    float rope_theta, rms_eps;
    int32_t tied;          /* LM head = token_embd (model.cpp:203-206) */
    int32_t kv_capacity;   /* max tokens per sequence (KVCacheConfig) */
    int32_t max_batch;     /* max tokens per eval call (prefill chunk) */
    int32_t precision;     /* B200_PREC_* for prefill matrix products */
    /* tensor parallelism (1 = single GPU); rank/world index this process */
    int32_t tp_rank, tp_world;
    /* decode step: B200_DECODE_AUTO or B200_DECODE_SINGLE (the persistent
     * single-launch kernel where the shape allows it on one GPU, else the
     * multi-kernel chain) or B200_DECODE_MULTI (always the multi-kernel chain) */
    int32_t decode_mode;
    /* 1: the engine allocates no KV cache; the caller binds each layer's KV object
     * (b200_engine_bind_kv) before finalize, e.g. the reference's KV storage
     * objects. 0: the engine owns a KV arena of kv_capacity tokens. */
    int32_t external_kv;
} b200_qwen3_config;

#define B200_DECODE_AUTO 0
#define B200_DECODE_MULTI 1
#define B200_DECODE_SINGLE 2

typedef struct b200_engine b200_engine;

/* Creates an engine on `device` and allocates its arenas once (weights, KV,
 * activations, workspaces). Returns B200_ERR_NO_MEMORY if they do not fit. */
int b200_engine_create(const b200_qwen3_config *cfg, int device, b200_engine **out);
void b200_engine_destroy(b200_engine *e);
/* Bytes the engine allocated, by arena (weights, kv, activations). */
int b200_engine_memory(const b200_engine *e, size_t *weights, size_t *kv, size_t *act);

/* Uploads one GGUF tensor (F32, numpy-style row-major (N, K); host memory or device
 * memory, told apart by unified addressing) by its GGUF name, e.g.
 * "blk.3.attn_q.weight". Under tensor parallelism the engine keeps only its rank's
 * shard of the full tensor passed here. Synchronous: the source may be released on
 * return. */
int b200_engine_set_weight(b200_engine *e, const char *name, const float *host_data,
                           int64_t n_elements);
/* Loads every tensor of a GGUF v3 file (F32 tensors named as above) into the
 * weight arena: the file is memory-mapped and streamed through a pinned staging
 * ring of `staging_bytes` (<= 0: 256 MiB) with asynchronous copies, and the call
 * synchronizes once at the end. Every tensor is validated (name, size, type,
 * bounds in the file) before the first copy. Replaces the reference's
 * per-tensor synchronous upload (ModelBase::alloc_weight, model.cpp:562-572, and
 * CUDABackend::copy_tensor_set, cuda_backend.cpp:106-112). */
int b200_engine_load_gguf(b200_engine *e, const char *path, int64_t staging_bytes);
/* Copies one weight tensor back to host memory in its GGUF shape (the inverse of
 * b200_engine_set_weight; like CUDABackend::copy_tensor_get, cuda_backend.cpp).
 * Single-GPU engines only (B200_ERR_NOT_SUPPORTED under tensor parallelism). */
int b200_engine_get_weight(b200_engine *e, const char *name, float *host_out, int64_t n_elements);
/* Fills every weight from the seeded generator of the given seed directly on the
 * device: matrices N(0, std), norm weights 1.0 (used when no GGUF is at hand). */
int b200_engine_init_random(b200_engine *e, uint64_t seed, float std);
/* Checks that every weight is set and prepares the decode CUDA graph. */
int b200_engine_finalize(b200_engine *e);

/* Drops the sequence (n_past = 0). */
int b200_engine_reset(b200_engine *e);
/* Precision of the prefill matrix products from the next step on (B200_PREC_FFMA:
 * exact F32; B200_PREC_TF32: tcgen05 tensor cores). Decode is unaffected (its
 * matrix-vector products are F32 FFMA either way). */
int b200_engine_set_precision(b200_engine *e, int32_t precision);
int64_t b200_engine_n_past(const b200_engine *e);

/* Kernel launches of this library per decode step after finalize: 1 when the
 * single-launch decode kernel runs the step, else the multi-kernel count
 * (5 per layer + LM head, + 2 token-selection kernels under tensor parallelism;
 * NCCL's own kernels not counted). < 0 on error. */
int b200_engine_decode_launches(const b200_engine *e);

/* Evaluates n tokens (prefill if n > 1, decode if n == 1) at positions
 * n_past..n_past+n-1, appends their K/V and samples greedily from the last row.
 * host_ids: host memory; host_last_logits (nullable): receives the last row [V];
 * host_token receives the greedy token. Synchronous (like read_logits +
 * Sampler::sample, sampler.cpp:5-65). On error nothing is committed. */
int b200_engine_eval(b200_engine *e, const int32_t *host_ids, int64_t n,
                     float *host_last_logits, int32_t *host_token);

/* As b200_engine_eval, but the last row's logits (nullable) go to device memory of
 * the engine's device (the logits tensor of a reference graph, for example). */
int b200_engine_eval_device(b200_engine *e, const int32_t *host_ids, int64_t n,
                            float *dev_last_logits, int32_t *host_token);

/* Sets the sequence position (tokens already in the KV cache; <= kv_capacity), for
 * a caller that keeps its own KV bookkeeping (the reference's KVCacheManager). */
int b200_engine_set_n_past(b200_engine *e, int64_t n_past);

/* Rotation frequencies freq[j], j < head_dim / 2 (host memory), replacing those the
 * engine derived from rope_theta; the angle of position p stays
 * float(double(p) * freq[j]). Row 1 of the reference's angle table
 * (GraphContext::get_rope_theta_table, graph.cpp:92-135) is exactly freq. */
int b200_engine_set_rope_freqs(b200_engine *e, const float *host_freq);

/* external_kv engines: layer `layer` reads and appends K/V in the KV object at
 * k_base / v_base (device memory of the engine's device, 16-byte aligned; token-major
 * [kv_capacity][n_head_kv][head_dim] floats each, the NaiveKVStorage layout,
 * naiveKVStorage.cpp:28-40). May be called again after finalize to move to another
 * sequence's objects (the decode graph is captured again at the next step). */
int b200_engine_bind_kv(b200_engine *e, int32_t layer, float *k_base, float *v_base);

/* Greedy decode of n_steps tokens entirely on the device: each step feeds the
 * previous step's token back (CUDA-graph replay, no host round trip); the first
 * input is the token sampled by the last eval. host_tokens (nullable) receives
 * the n_steps generated tokens after the final synchronization. */
int b200_engine_generate(b200_engine *e, int64_t n_steps, int32_t *host_tokens);

/* Per-op timing of one decode step (CUDA events around each launch, no graph):
 * writes up to max_ops (name, microseconds) pairs; returns the count or <0. */
int b200_engine_profile_step(b200_engine *e, char *names, int name_len, float *us,
                             int max_ops);

/* Device-side timeline of one graph-replayed decode step: for each launch, in
 * order (per layer: QKV GEMV, attention, o_proj, gate/up, down; then LM head),
 * 8 global-timer words in ns: [CTA 0 start, CTA 0 after its dependency wait,
 * last CTA end, first CTA start of any CTA, CTA 0 after its prologue, CTA 0
 * after its main loop, 0, 0]. With the single-launch decode kernel the entries
 * are its phases in the same order, stamped by CTA 0: [0, 0, after the grid
 * barrier that ends the phase, phase start, after the input load, after the
 * main loop, 0, 0]. Returns the number of entries written (<= max_kernels) or
 * < 0. The step leaves n_past and the token unchanged. */
int b200_engine_trace_step(b200_engine *e, unsigned long long *host_trace, int max_kernels);

/* Failure injection for tests of the single-launch decode step (no counterpart in
 * the reference): after `after_steps` more decode steps, CTA `cta` of every step
 * does not publish its layer-0 QKV outputs, as if it had stopped; the CTAs waiting
 * for them give up after their bounded wait (2 s), the call returns
 * B200_ERR_TIMEOUT and commits nothing (eval and generate leave n_past and the
 * next input token as before the call), and the engine stays usable without a
 * reset. cta < 0 ends the injection. B200_ERR_NOT_SUPPORTED when the multi-kernel
 * decode path is in use. */
int b200_engine_inject_withhold(b200_engine *e, int32_t cta, int32_t after_steps);

/* Test hook of the single-launch decode step (no counterpart in the reference):
 * sets its launch counter as if `launches` steps had run, so a test can take the
 * step's exchange tags across their wrap-around (every 2^24 - 1 launches) without
 * running millions of steps. Results must not change. B200_ERR_NOT_SUPPORTED when
 * the multi-kernel decode path is in use. */
int b200_engine_set_decode_launch_counter(b200_engine *e, uint64_t launches);

/* Raw handles for in-process callers (bench / tests): the engine's stream and
 * device status word. */
void *b200_engine_stream(b200_engine *e);
int b200_engine_read_status(b200_engine *e, int32_t *status);

/* Tensor parallelism over NCCL: every rank calls with the same 128-byte
 * ncclUniqueId (created by rank 0 with b200_tp_unique_id) before finalize. */
int b200_tp_unique_id(unsigned char out_id[128]);
int b200_engine_tp_init(b200_engine *e, const unsigned char id[128]);
/* 1 if the engine's decode step exchanges its all-reduces and token selection over
 * NVLink peer memory (its own kernels: CUDA IPC buffers, tagged words, bounded
 * waits), 0 if over NCCL (a peer not reachable by peer access, or B200_TP_NCCL=1
 * at tp_init). Prefill all-reduces always use NCCL. */
int b200_engine_tp_peer_exchange(const b200_engine *e);

#ifdef __cplusplus
}
#endif
#endif /* B200_INFER_H */
