// extern "C" single-op entry points declared in include/b200_infer.h. Each one
// validates sizes and alignment on the host, then enqueues the sm_100a kernel on
// the caller's stream. No allocation, no synchronization.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "attention.cuh"
#include "elementwise.cuh"
#include "gemm.cuh"
#include "gemv.cuh"

using namespace b200;

namespace {

inline cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline int from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return B200_OK;
    if (e == cudaErrorInvalidValue) return B200_ERR_INVALID_ARGUMENT;
    if (e == cudaErrorNotSupported) return B200_ERR_NOT_SUPPORTED;
    return B200_ERR_CUDA;
}

}  // namespace

extern "C" {

const char *b200_status_string(int s) {
    switch (s) {
        case B200_OK: return "ok";
        case B200_ERR_INVALID_ARGUMENT: return "invalid argument";
        case B200_ERR_NOT_SUPPORTED: return "not supported";
        case B200_ERR_OUT_OF_RANGE: return "out of range";
        case B200_ERR_CUDA: return "CUDA error";
        case B200_ERR_NO_MEMORY: return "out of memory";
        case B200_ERR_DEVICE_CHECK: return "device-side check failed";
        case B200_ERR_TIMEOUT: return "device wait timed out";
        case B200_ERR_NUMERIC: return "NaN or +inf logits";
    }
    return "unknown status";
}

int b200_device_supported(int device) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return 0;
    return p.major == 10 && p.minor == 0 ? 1 : 0;
}

size_t b200_mul_mat_workspace_bytes(int64_t K, int64_t N, int64_t M, int precision) {
    if (K <= 0 || N <= 0 || M <= 4) return 0;
    int64_t f = gemm_ffma_ws_floats(M, N, K);
    if (precision == B200_PREC_TF32) f = std::max(f, gemm_tf32_ws_floats(M, N, K));
    return static_cast<size_t>(f) * 4;
}

int b200_mul_mat(const float *w, const float *x, float *out, int64_t K, int64_t N, int64_t M,
                 int precision, void *stream) {
    return b200_mul_mat_ws(w, x, out, K, N, M, precision, nullptr, 0, stream);
}

int b200_mul_mat_ws(const float *w, const float *x, float *out, int64_t K, int64_t N, int64_t M,
                    int precision, void *workspace, size_t workspace_bytes, void *stream) {
    if (K <= 0 || N <= 0 || M < 0) return B200_ERR_INVALID_ARGUMENT;
    if (M == 0) return B200_OK;
    if (!w || !x || !out) return B200_ERR_INVALID_ARGUMENT;
    if (precision != B200_PREC_FFMA && precision != B200_PREC_TF32) return B200_ERR_INVALID_ARGUMENT;
    if ((K & 3) || !aligned16(w) || !aligned16(x)) return B200_ERR_NOT_SUPPORTED;
    if (M <= 4) {
        GemvArgs a;
        a.w = w;
        a.x = x;
        a.out = out;
        a.K = K;
        a.N = N;
        a.M = static_cast<int>(M);
        a.epi = GEMV_STORE;
        return from_cuda(gemv_launch(a, as_stream(stream), false));
    }
    GemmArgs g;
    g.x = x;
    g.ldx = K;
    g.w = w;
    g.c = out;
    g.ldc = N;
    g.M = M;
    g.N = N;
    g.K = K;
    g.epi = GEMM_STORE;
    if (workspace && !(reinterpret_cast<uintptr_t>(workspace) & 15)) {
        g.ws = static_cast<float *>(workspace);
        g.ws_floats = static_cast<int64_t>(workspace_bytes / 4);
    }
    if (precision == B200_PREC_TF32) {
        const cudaError_t e = gemm_tf32_launch(g, as_stream(stream), false);
        if (e != cudaErrorNotSupported) return from_cuda(e);
    }
    return from_cuda(gemm_ffma_launch(g, as_stream(stream), false));
}

int b200_rms_norm(const float *x, const float *gamma, float *out, int64_t D, int64_t rows, float eps,
                  void *stream) {
    if (D <= 0 || rows < 0 || !x || !gamma || !out) return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(rms_norm_launch(x, gamma, out, D, rows, eps, as_stream(stream), false));
}

int b200_rope(const float *x, const int32_t *pos, const float *theta_table, int64_t n_ctx, float *out,
              int64_t D, int64_t H, int64_t T, int32_t *dev_status, void *stream) {
    if (D <= 0 || (D & 1) || H < 0 || T < 0 || n_ctx <= 0 || !x || !pos || !theta_table || !out)
        return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(rope_table_launch(x, pos, theta_table, n_ctx, out, D, H, T, dev_status,
                                       as_stream(stream), false));
}

void b200_rope_freqs(float theta, int64_t D, float *host_freq) {
    // graph.cpp:119-121: freq_i = 1.0f / pow(theta, 2.0f * i / head_dim), float arithmetic
    for (int64_t i = 0; i < D / 2; ++i) {
        const float expo = 2.0f * static_cast<float>(i) / static_cast<float>(D);
        host_freq[i] = 1.0f / powf(theta, expo);
    }
}

int b200_qk_norm_rope(const float *q_in, int64_t q_ld, const float *k_in, int64_t k_ld, const float *v_in,
                      int64_t v_ld, const float *q_gamma, const float *k_gamma, const float *freq,
                      const int32_t *pos, float *q_out, float *k_out, int64_t k_out_ld, float *v_out,
                      int64_t v_out_ld, int64_t D, int64_t Hq, int64_t Hkv, int64_t T, int64_t n_ctx,
                      float eps, int32_t *dev_status, void *stream) {
    if (!q_in || !k_in || !q_gamma || !k_gamma || !freq || !pos || !q_out || !k_out || T < 0 || Hq <= 0 ||
        Hkv <= 0 || n_ctx <= 0)
        return B200_ERR_INVALID_ARGUMENT;
    if (D != 32 && D != 64 && D != 128 && D != 256) return B200_ERR_NOT_SUPPORTED;
    if ((v_out != nullptr) != (v_in != nullptr)) return B200_ERR_INVALID_ARGUMENT;
    QkNormRopeArgs a;
    a.q_in = q_in;
    a.q_ld = q_ld;
    a.k_in = k_in;
    a.k_ld = k_ld;
    a.v_in = v_in;
    a.v_ld = v_ld;
    a.q_gamma = q_gamma;
    a.k_gamma = k_gamma;
    a.freq = freq;
    a.pos = pos;
    a.q_out = q_out;
    a.k_out = k_out;
    a.k_out_ld = k_out_ld;
    a.v_out = v_out;
    a.v_out_ld = v_out_ld;
    a.D = D;
    a.Hq = Hq;
    a.Hkv = Hkv;
    a.T = T;
    a.n_ctx = n_ctx;
    a.eps = eps;
    a.status = dev_status;
    return from_cuda(qk_norm_rope_launch(a, as_stream(stream), false));
}

size_t b200_flash_attn_workspace_bytes(int64_t D, int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tkv) {
    if (Tq != 1) return 256;
    return attn_decode_ws_bytes(D, Hq, Hkv, attn_decode_splits(Tkv, Hkv));
}

int b200_flash_attn_ex(const float *q, const float *k, const float *v, float *out, int64_t D, int64_t Hq,
                       int64_t Hkv, int64_t Tq, int64_t Tkv, int64_t n_past, float scale, int64_t k_tok_stride,
                       int64_t k_head_stride, int64_t v_tok_stride, int64_t v_head_stride, void *workspace,
                       size_t workspace_bytes, void *stream, int32_t precision) {
    if (precision != B200_PREC_FFMA && precision != B200_PREC_TF32) return B200_ERR_INVALID_ARGUMENT;
    if (!q || !k || !v || !out || D <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Tq < 0 || n_past < 0)
        return B200_ERR_INVALID_ARGUMENT;
    if (Tkv != n_past + Tq) return B200_ERR_INVALID_ARGUMENT;
    if (Tq == 0) return B200_OK;
    AttnArgs a;
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.k_tok = k_tok_stride;
    a.k_head = k_head_stride;
    a.v_tok = v_tok_stride;
    a.v_head = v_head_stride;
    a.D = D;
    a.Hq = Hq;
    a.Hkv = Hkv;
    a.Tq = Tq;
    a.n_past = n_past;
    a.scale = scale;
    a.precision = precision;
    a.ws = workspace;
    a.ws_bytes = workspace_bytes;
    cudaStream_t st = as_stream(stream);
    if (Tq == 1) {
        // split-KV decode: with the workspace of b200_flash_attn_workspace_bytes the
        // K/V tiles are bulk-copied and the splits merged through it; without one the
        // splits of a KV head merge in distributed shared memory (one cluster)
        const int S = attn_decode_splits(Tkv, Hkv);
        return from_cuda(attn_decode_launch(a, S, st, false));
    }
    return from_cuda(attn_prefill_launch(a, st, false));
}

int b200_flash_attn(const float *q, const float *k, const float *v, float *out, int64_t D, int64_t Hq,
                    int64_t Hkv, int64_t Tq, int64_t Tkv, int64_t n_past, float scale, int64_t k_tok_stride,
                    int64_t k_head_stride, int64_t v_tok_stride, int64_t v_head_stride, void *workspace,
                    size_t workspace_bytes, void *stream) {
    return b200_flash_attn_ex(q, k, v, out, D, Hq, Hkv, Tq, Tkv, n_past, scale, k_tok_stride, k_head_stride,
                              v_tok_stride, v_head_stride, workspace, workspace_bytes, stream, B200_PREC_FFMA);
}

int b200_silu(const float *x, float *out, int64_t n, void *stream) {
    if (n < 0 || (n && (!x || !out))) return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(eltwise_launch(0, x, nullptr, out, n, as_stream(stream), false));
}
int b200_mul(const float *a, const float *b, float *out, int64_t n, void *stream) {
    if (n < 0 || (n && (!a || !b || !out))) return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(eltwise_launch(1, a, b, out, n, as_stream(stream), false));
}
int b200_add(const float *a, const float *b, float *out, int64_t n, void *stream) {
    if (n < 0 || (n && (!a || !b || !out))) return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(eltwise_launch(2, a, b, out, n, as_stream(stream), false));
}
int b200_swiglu(const float *gate, const float *up, float *out, int64_t n, void *stream) {
    if (n < 0 || (n && (!gate || !up || !out))) return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(eltwise_launch(3, gate, up, out, n, as_stream(stream), false));
}

int b200_get_rows(const float *table, const int32_t *ids, float *out, int64_t D, int64_t n, int64_t n_rows,
                  int32_t *dev_status, void *stream) {
    if (D <= 0 || n < 0 || n_rows <= 0 || (n && (!table || !ids || !out))) return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(get_rows_launch(table, ids, out, D, n, n_rows, dev_status, as_stream(stream), false));
}

int b200_copy(void *dst, const void *src, size_t bytes, void *stream) {
    if (bytes == 0 || dst == src) return B200_OK;
    if (!dst || !src) return B200_ERR_INVALID_ARGUMENT;
    return from_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
}

size_t b200_argmax_workspace_bytes(int64_t n) { return argmax_workspace(n); }

int b200_argmax(const float *logits, int64_t n, int32_t *out_id, void *workspace, size_t workspace_bytes,
                int32_t *dev_status, void *stream) {
    if (n <= 0 || !logits || !out_id || !workspace) return B200_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < argmax_workspace(n)) return B200_ERR_INVALID_ARGUMENT;
    cudaStream_t st = as_stream(stream);
    cudaError_t e = cudaMemsetAsync(workspace, 0, 4, st);
    if (e != cudaSuccess) return from_cuda(e);
    return from_cuda(argmax_launch(logits, n, out_id, workspace, dev_status, st, false));
}

}  // extern "C"
