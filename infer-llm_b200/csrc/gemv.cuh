// Decode GEMV (M <= 4 tokens): y[m][n] = sum_k W[n][k] * x[m][k] with fused
// prologues (embedding gather, RMSNorm) and epilogues (residual add, SwiGLU, greedy
// argmax). Replaces the reference's one-CTA-per-output mul_mat (kernel_f32.cu:142-205).
#pragma once

#include "common.cuh"

namespace b200 {

enum GemvEpi : int {
    GEMV_STORE = 0,     // out = W.x
    GEMV_RESIDUAL = 1,  // out = W.x + residual        (o_proj / ffn_down + add)
    GEMV_SWIGLU = 2,    // rows interleaved (gate_i, up_i): out_i = up_i * silu(gate_i)
    GEMV_ARGMAX = 3,    // LM head: optional logits store + first-max token id (M == 1)
};

struct GemvArgs {
    const float *w = nullptr;      // [N][K] row-major, 16-byte aligned, K % 4 == 0
    const float *x = nullptr;      // [M][K] activations (unused when embed_table is set)
    int64_t x_ld = 0;              // row stride of x in floats (0 = K)
    const float *gamma = nullptr;  // RMSNorm prologue weight [K] (nullptr: no norm)
    float eps = 0.f;
    const float *embed_table = nullptr;  // gather prologue: x[m] = table[ids[m]]
    const int32_t *embed_ids = nullptr;
    int64_t embed_rows = 0;
    float *x_store = nullptr;      // with embed: CTA 0 stores the gathered rows here [M][K]
    float *out = nullptr;          // [M][N] ([M][N/2] for SWIGLU); ARGMAX: logits or nullptr
    int64_t out_ld = 0;            // row stride of out in floats (0 = natural)
    const float *residual = nullptr;  // RESIDUAL: [M][out_ld] (may alias out)
    int64_t K = 0, N = 0;
    int M = 1;
    int epi = GEMV_STORE;
    // ARGMAX
    float *part_val = nullptr;     // [gridDim.x]
    int32_t *part_idx = nullptr;   // [gridDim.x]
    unsigned *counter = nullptr;   // zero before the first launch; the last CTA re-zeroes it
    int32_t *argmax_out = nullptr; // token id (-1 on NaN / +inf logits)
    int32_t *token_log = nullptr;  // optional: token also appended to token_log[*log_pos]
    int32_t *log_pos = nullptr;
    int32_t log_cap = 0;
    int32_t *n_past = nullptr;     // optional: advanced by n_past_add by the last CTA
    int32_t n_past_add = 1;
    int64_t idx_offset = 0;        // added to the winning row (vocab shard offset)
    float *best_val_out = nullptr; // optional: winning logit (tensor-parallel selection)
    int32_t *status = nullptr;
    unsigned long long *trace = nullptr;  // optional step trace slot (common.cuh)
    // Signal dependents only after this kernel's own dependency wait, so the next
    // kernel may read, before its wait, anything produced two or more launches back.
    bool late_launch = false;
    // Weights of the next kernel in the step, prefetched into L2 by this kernel's
    // CTAs before their dependency wait (keeps HBM busy across kernel boundaries).
    const void *next_w = nullptr;
    size_t next_w_bytes = 0;
};

// Launches the GEMV on `stream` (with programmatic dependent launch if pdl): the
// direct-streaming kernel (gemv_direct.cu) for even N, else the bulk-copy ring.
cudaError_t gemv_launch(const GemvArgs &a, cudaStream_t stream, bool pdl);
cudaError_t gemv_direct_launch(const GemvArgs &a, cudaStream_t stream, bool pdl);
cudaError_t gemv_ring_launch(const GemvArgs &a, cudaStream_t stream, bool pdl);
int gemv_grid_size(int64_t N, int epi);      // CTAs of the ring kernel
int gemv_direct_ks(int64_t N, int64_t K);    // K-slices per row of the direct kernel
int gemv_direct_grid(int64_t N, int64_t K, int M = 1, bool norm = true);  // its CTAs
// Size of part_val / part_idx an ARGMAX launch over N rows of length K needs.
int gemv_argmax_slots(int64_t N, int64_t K);
int device_sm_count();

}  // namespace b200
