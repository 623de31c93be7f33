// Prefill matrix products C[M][N] = X[M][K] . W[N][K]^T with fused epilogues.
#pragma once

#include "common.cuh"

namespace b200 {

enum GemmEpi : int {
    GEMM_STORE = 0,
    GEMM_RESIDUAL = 1,  // C = X.W^T + R (R may alias C)
    GEMM_SWIGLU = 2,    // W rows interleaved (gate_i, up_i): C[:, i] = up * silu(gate)
};

struct GemmArgs {
    const float *x = nullptr;  // [M][ldx]
    int64_t ldx = 0;
    const float *w = nullptr;  // [N][K]
    float *c = nullptr;        // [M][ldc]
    int64_t ldc = 0;
    const float *r = nullptr;  // residual [M][ldc]
    int64_t M = 0, N = 0, K = 0;
    int epi = GEMM_STORE;
    // Optional split-K workspace (floats). When the M x N tile grid is too small to
    // fill the GPU, the FFMA GEMM splits K, writes per-split partials here and
    // reduces them in split order (deterministic) with the epilogue.
    float *ws = nullptr;
    int64_t ws_floats = 0;
    int64_t k_split = 0;  // set by the launcher: K per split (0 = no split)
    int32_t *status = nullptr;  // device status word for bounded-wait timeouts (tcgen05 GEMM)
    // Outputs rounded to the nearest TF32 value (they only feed a later TF32 product;
    // honoured by the tcgen05 GEMM and the split-K reduction).
    bool round_out = false;
};

// Exact F32 FFMA tiled GEMM (any M; K % 4 == 0).
cudaError_t gemm_ffma_launch(const GemmArgs &a, cudaStream_t stream, bool pdl);
// tcgen05 TF32 tensor-core GEMM (TMA-staged 128-byte-swizzled operands, TMEM
// accumulators). Returns cudaErrorNotSupported for operands TMA cannot describe
// (unaligned bases or strides).
cudaError_t gemm_tf32_launch(const GemmArgs &a, cudaStream_t stream, bool pdl);
// Sums a.ws[0..splits) (split-K partials, [M][N] each) in split order and applies
// a.epi into a.c.
cudaError_t gemm_splitk_reduce_launch(const GemmArgs &a, int splits, cudaStream_t stream, bool pdl);
// Split-K workspace (floats) that lets each GEMM use all its splits at M x N x K
// (0: no split at this shape).
int64_t gemm_ffma_ws_floats(int64_t M, int64_t N, int64_t K);
int64_t gemm_tf32_ws_floats(int64_t M, int64_t N, int64_t K);
int device_sm_count();

}  // namespace b200
