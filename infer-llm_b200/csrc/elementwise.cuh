// Normalisation, RoPE, gather, activation and sampling kernels.
#pragma once

#include "common.cuh"

namespace b200 {

// round_tf32: outputs rounded to the nearest TF32 value (they feed a TF32 product)
cudaError_t rms_norm_launch(const float *x, const float *gamma, float *out, int64_t D, int64_t rows,
                            float eps, cudaStream_t stream, bool pdl, bool round_tf32 = false);

cudaError_t rope_table_launch(const float *x, const int32_t *pos, const float *table, int64_t n_ctx,
                              float *out, int64_t D, int64_t H, int64_t T, int32_t *status,
                              cudaStream_t stream, bool pdl);

struct QkNormRopeArgs {
    const float *q_in = nullptr;   // token t, head h at q_in[t*q_ld + h*D]
    int64_t q_ld = 0;
    const float *k_in = nullptr;
    int64_t k_ld = 0;
    const float *v_in = nullptr;   // optional V copy into its cache slot
    int64_t v_ld = 0;
    const float *q_gamma = nullptr, *k_gamma = nullptr;  // [D]
    const float *freq = nullptr;   // [D/2]
    const int32_t *pos = nullptr;  // [T] positions, or nullptr to use pos_base
    const int32_t *pos_base = nullptr;  // device scalar: position of token 0 (pos = base + t)
    float *q_out = nullptr;        // [T][Hq][D]
    float *k_out = nullptr;        // token t at k_out[(koff + t) * k_out_ld + h*D]
    int64_t k_out_ld = 0;
    float *v_out = nullptr;
    int64_t v_out_ld = 0;
    const int32_t *out_offset = nullptr;  // device scalar added to the K/V row index (n_past)
    int64_t D = 0, Hq = 0, Hkv = 0, T = 0, n_ctx = 0;
    float eps = 0.f;
    int32_t *status = nullptr;
};
cudaError_t qk_norm_rope_launch(const QkNormRopeArgs &a, cudaStream_t stream, bool pdl);

// op: 0 silu(a), 1 a*b, 2 a+b, 3 b*silu(a) (swiglu: a = gate, b = up)
cudaError_t eltwise_launch(int op, const float *a, const float *b, float *out, int64_t n,
                           cudaStream_t stream, bool pdl);

cudaError_t get_rows_launch(const float *table, const int32_t *ids, float *out, int64_t D, int64_t n,
                            int64_t n_rows, int32_t *status, cudaStream_t stream, bool pdl);

size_t argmax_workspace(int64_t n);
cudaError_t argmax_launch(const float *logits, int64_t n, int32_t *out_id, void *ws, int32_t *status,
                          cudaStream_t stream, bool pdl);

}  // namespace b200
