/*
 * oracle/cpu_ops.h -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A CPU restatement of the Infer-LLM reference CPU backend
 * (src/backends/cpu_backend.cpp) for the F32 Qwen3 inference path. It is the
 * checker the B200 kernels are compared against. Only tests/, the smoke check
 * in __graft_entry__.py and the cpu_baseline / reference legs of bench.py load
 * it; the product library never links or calls it.
 *
 * Every function reproduces the reference arithmetic: the same accumulation
 * type, the same summation order and the same libm calls, so its outputs are
 * bit-identical to the reference CPU backend when both are compiled without
 * FMA contraction (checked by tests/test_oracle_vs_reference.py against the
 * reference built from source, and by committed golden fixtures).
 *
 * Layout convention (ggml style, dims[0] fastest):
 *   matrix "[K, N]" = N rows of K contiguous floats.
 */
#ifndef B200_ORACLE_CPU_OPS_H
#define B200_ORACLE_CPU_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[t*N + n] = sum_k x[t*K + k] * w[n*K + k], float accumulation in k order.
 * cpu_backend.cpp:386-424 (CPUBackend::compute_mul_mat). */
void orc_mul_mat(const float *w, const float *x, float *out,
                 int64_t K, int64_t N, int64_t M, int nthreads);

/* Row-wise RMSNorm over D contiguous floats, sum of squares in double.
 * cpu_backend.cpp:335-382 (CPUBackend::compute_rms_norm). */
void orc_rms_norm(const float *x, const float *gamma, float *out,
                  int64_t D, int64_t rows, float eps, int nthreads);

/* RoPE angle table [n_ctx][head_dim/2]: row[pos][i] = float(double(pos) * freq_i),
 * freq_i = 1.0f / powf(theta, 2.0f*i/head_dim).
 * graph.cpp:92-135 (GraphContext::get_rope_theta_table). */
void orc_rope_theta_table(float theta_base, uint32_t head_dim, uint32_t n_ctx, float *out);

/* NeoX half-split rotation of x [D, H, T] by the table rows at pos[t].
 * cpu_backend.cpp:443-523 (CPUBackend::compute_rope). table_row = D/2 floats. */
void orc_rope(const float *x, const int32_t *pos, const float *table, float *out,
              int64_t D, int64_t H, int64_t T, int nthreads);

/* Causal GQA attention. q [D, Hq, Tq]; k, v [D, Hkv, Tkv] token-major
 * (token stride Hkv*D); out [D, Hq, Tq]. Key j is masked for query t when
 * j > n_past + t. Scale is always 1/sqrt(D).
 * cpu_backend.cpp:525-634 (CPUBackend::compute_flash_attn). */
void orc_flash_attn(const float *q, const float *k, const float *v, float *out,
                    int64_t D, int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tkv,
                    int64_t n_past, int nthreads);

/* cpu_backend.cpp:662-677 */
void orc_silu(const float *x, float *out, int64_t n);
/* cpu_backend.cpp:681-703 (dst = a * b) */
void orc_mul(const float *a, const float *b, float *out, int64_t n);
/* cpu_backend.cpp:638-659 (dst = a + b) */
void orc_add(const float *a, const float *b, float *out, int64_t n);
/* Row gather: out[t] = table[ids[t]], rows of D floats. cpu_backend.cpp:259-332.
 * Returns -1 (and writes nothing for that row) for an id outside [0, n_rows). */
int orc_get_rows(const float *table, const int32_t *ids, float *out,
                 int64_t D, int64_t n, int64_t n_rows);

/* Greedy sampler: first index of the maximum; NaN or +inf anywhere -> -1;
 * all -inf -> -1. sampler.cpp:42-65 (sample_greedy). */
int32_t orc_argmax(const float *logits, int64_t n);

/* ------------------------------------------------------------------------
 * Whole-model restatement of Qwen3Model::build_graph (src/models/Qwen3.cpp:4-136)
 * executed in graph order, with the contiguous per-layer KV object of
 * NaiveKVStorage (K block [cap][Hkv][Dk] then V block [cap][Hkv][Dv],
 * src/kvcache/KVStorages/naiveKVStorage.cpp:28-40).
 * ------------------------------------------------------------------------ */
typedef struct orc_qwen3_config {
    int32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, head_dim, n_ff;
    int32_t n_ctx_train;   /* rows of the RoPE angle table */
    float rope_theta, rms_eps;
    int32_t kv_capacity;   /* max tokens per sequence */
} orc_qwen3_config;

/* Per-layer weight pointers, host memory, row-major as stored in GGUF. */
typedef struct orc_qwen3_layer {
    const float *attn_norm, *wq, *wk, *wv, *wo, *q_norm, *k_norm;
    const float *ffn_norm, *ffn_gate, *ffn_up, *ffn_down;
} orc_qwen3_layer;

typedef struct orc_qwen3 orc_qwen3;

orc_qwen3 *orc_qwen3_create(const orc_qwen3_config *cfg, const float *token_embd,
                            const float *output_norm, const float *output,
                            const orc_qwen3_layer *layers);
void orc_qwen3_destroy(orc_qwen3 *m);
/* Reset the sequence (n_past = 0). */
void orc_qwen3_reset(orc_qwen3 *m);
int64_t orc_qwen3_n_past(const orc_qwen3 *m);
/* Evaluate n tokens at positions n_past..n_past+n-1, append their K/V and
 * write logits. all_rows != 0 writes [n][V] (what the reference graph
 * computes); otherwise only the last row [V]. Returns 0, or -1 on a bad id or
 * KV overflow (nothing is committed then). */
int orc_qwen3_eval(orc_qwen3 *m, const int32_t *ids, int64_t n, float *logits,
                   int all_rows, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
