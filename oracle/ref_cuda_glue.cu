// TEST-ONLY checker: the reference's own CUDA kernels behind a flat C interface.
//
// The reference's CUDA path is CUDA_F32::compute_<op>(Tensor *dst, cudaStream_t)
// (include/kernels/cuda/kernel_f32.hpp:8-28, src/kernels/cuda/kernel_f32.cu). The
// `ref-cuda` target of oracle/Makefile compiles that .cu unmodified for sm_100a and
// links it with this file into oracle/_ref/libref_cuda_ops.so, so the GPU tests can
// run the reference's kernels and the B200 kernels on the same device buffers and
// compare them (the reference's second implementation of every op, next to its CPU
// backend). Each refc_* function builds the Tensor graph node the reference's
// Qwen3 graph builds for that op (src/models/Qwen3.cpp, src/op_factory.cpp) around
// caller-owned device pointers, calls compute_<op> and synchronizes the stream.
// Never part of the product: nothing under infer-llm_b200/ links it.
//
// Positions passed to refc_rope must lie in [0, n_ctx): the reference kernel
// traps on any other (kernel_f32.cu:250-253), so callers keep them in range.
#include <cstring>
#include <initializer_list>

#include "kernels/cuda/kernel_f32.hpp"
#include "op_params.hpp"
#include "tensor.hpp"

namespace {

Tensor make(const char *name, DataType type, std::initializer_list<int64_t> shape, const void *data) {
    Tensor t(name, type, shape);
    t.data = const_cast<void *>(data);
    t.device = DeviceType::CUDA;
    return t;
}

int finish(cudaError_t launched, void *stream) {
    if (launched != cudaSuccess) return static_cast<int>(launched);
    return static_cast<int>(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
}

}  // namespace

extern "C" {

// out [N, M] = W [K, N]^T x [K, M]   (Qwen3.cpp mul_mat nodes, op_factory.cpp:98-107)
int refc_mul_mat(const float *w, const float *x, float *out, int64_t K, int64_t N, int64_t M, void *stream) {
    Tensor tw = make("w", GGML_TYPE_F32, {K, N}, w), tx = make("x", GGML_TYPE_F32, {K, M}, x);
    Tensor d = make("out", GGML_TYPE_F32, {N, M}, out);
    d.src[0] = &tw;
    d.src[1] = &tx;
    return finish(CUDA_F32::compute_mul_mat(&d, static_cast<cudaStream_t>(stream)), stream);
}

// RMSNorm over D of `rows` rows; eps in op_params[0] (op_factory.cpp:110-121)
int refc_rms_norm(const float *x, const float *gamma, float *out, int64_t D, int64_t rows, float eps, void *stream) {
    Tensor tx = make("x", GGML_TYPE_F32, {D, rows}, x), tg = make("g", GGML_TYPE_F32, {D}, gamma);
    Tensor d = make("out", GGML_TYPE_F32, {D, rows}, out);
    d.src[0] = &tx;
    d.src[1] = &tg;
    std::memcpy(&d.op_params[0], &eps, sizeof eps);
    return finish(CUDA_F32::compute_rms_norm(&d, static_cast<cudaStream_t>(stream)), stream);
}

// NeoX RoPE of x [D, H, T] with the angle table [D/2, n_ctx] (op_factory.cpp:138-147)
int refc_rope(const float *x, const int32_t *pos, const float *table, int64_t n_ctx, float *out, int64_t D,
              int64_t H, int64_t T, void *stream) {
    Tensor tx = make("x", GGML_TYPE_F32, {D, H, T}, x), tp = make("pos", GGML_TYPE_I32, {T}, pos);
    Tensor tt = make("theta", GGML_TYPE_F32, {D / 2, n_ctx}, table);
    Tensor d = make("out", GGML_TYPE_F32, {D, H, T}, out);
    d.src[0] = &tx;
    d.src[1] = &tp;
    d.src[2] = &tt;
    return finish(CUDA_F32::compute_rope(&d, static_cast<cudaStream_t>(stream)), stream);
}

// Causal GQA attention: q [D, Hq, Tq], contiguous k / v [D, Hkv, Tkv], AttnParams
// with n_ctx = n_past (Qwen3.cpp:38-44,80; op_factory.cpp:151-163)
int refc_flash_attn(const float *q, const float *k, const float *v, float *out, int64_t D, int64_t Hq, int64_t Hkv,
                    int64_t Tq, int64_t Tkv, int64_t n_past, float scale, void *stream) {
    Tensor tq = make("q", GGML_TYPE_F32, {D, Hq, Tq}, q), tk = make("k", GGML_TYPE_F32, {D, Hkv, Tkv}, k);
    Tensor tv = make("v", GGML_TYPE_F32, {D, Hkv, Tkv}, v);
    Tensor d = make("out", GGML_TYPE_F32, {D, Hq, Tq}, out);
    d.src[0] = &tq;
    d.src[1] = &tk;
    d.src[2] = &tv;
    AttnParams p{};
    p.n_head = static_cast<uint32_t>(Hq);
    p.n_head_kv = static_cast<uint32_t>(Hkv);
    p.head_dim = static_cast<uint32_t>(D);
    p.scale = scale;
    p.causal = true;
    p.n_ctx = static_cast<uint32_t>(n_past);
    static_assert(sizeof(AttnParams) <= sizeof(d.op_params), "AttnParams fits op_params");
    std::memcpy(d.op_params, &p, sizeof p);
    return finish(CUDA_F32::compute_flash_attn(&d, static_cast<cudaStream_t>(stream)), stream);
}

// Embedding gather: table [H, V], ids [n] -> out [H, n] (op_factory.cpp:78-94)
int refc_get_rows(const float *table, const int32_t *ids, float *out, int64_t H, int64_t V, int64_t n, void *stream) {
    Tensor tt = make("table", GGML_TYPE_F32, {H, V}, table), ti = make("ids", GGML_TYPE_I32, {n}, ids);
    Tensor d = make("out", GGML_TYPE_F32, {H, n}, out);
    d.src[0] = &tt;
    d.src[1] = &ti;
    return finish(CUDA_F32::compute_get_rows(&d, static_cast<cudaStream_t>(stream)), stream);
}

// Elementwise ops over n floats (op_factory.cpp:46-60,126-134)
int refc_silu(const float *x, float *out, int64_t n, void *stream) {
    Tensor tx = make("x", GGML_TYPE_F32, {n}, x), d = make("out", GGML_TYPE_F32, {n}, out);
    d.src[0] = &tx;
    return finish(CUDA_F32::compute_silu(&d, static_cast<cudaStream_t>(stream)), stream);
}

int refc_add(const float *a, const float *b, float *out, int64_t n, void *stream) {
    Tensor ta = make("a", GGML_TYPE_F32, {n}, a), tb = make("b", GGML_TYPE_F32, {n}, b);
    Tensor d = make("out", GGML_TYPE_F32, {n}, out);
    d.src[0] = &ta;
    d.src[1] = &tb;
    return finish(CUDA_F32::compute_add(&d, static_cast<cudaStream_t>(stream)), stream);
}

int refc_mul(const float *a, const float *b, float *out, int64_t n, void *stream) {
    Tensor ta = make("a", GGML_TYPE_F32, {n}, a), tb = make("b", GGML_TYPE_F32, {n}, b);
    Tensor d = make("out", GGML_TYPE_F32, {n}, out);
    d.src[0] = &ta;
    d.src[1] = &tb;
    return finish(CUDA_F32::compute_mul(&d, static_cast<cudaStream_t>(stream)), stream);
}

}  // extern "C"
