// Drop-in replacement for the reference's src/kernels/cuda/kernel_f32.cu.
//
// A maintainer of the reference keeps its CUDA backend (src/backends/cuda_backend.cpp,
// which dispatches every graph node to CUDA_F32::compute_<op>, cuda_backend.cpp:211-238)
// and swaps kernel_f32.cu for this file: each compute_<op>(Tensor *dst, cudaStream_t)
// of include/kernels/cuda/kernel_f32.hpp:8-28 becomes one call into the B200 C ABI
// (include/b200_infer.h) with the tensor's raw pointers, sizes and strides. Built
// against the reference headers with INFERLLM_WITH_CUDA defined and linked with
// libb200infer.so (oracle/Makefile target `ref-b200` does exactly that for the
// end-to-end drop-in test).
//
// Semantics follow the reference kernels: mul_mat out[N, M] = W[K, N]^T x[K, M]
// (kernel_f32.cu:180-205); RMSNorm over dims[0] with eps in op_params[0] (60-90);
// RoPE with the GraphContext angle table as src[2] (273-301); attention with
// AttnParams in op_params, scale defaulting to 1/sqrt(head_dim) (452-511); CPY /
// RESHAPE are device copies, VIEW is a no-op (210-240, 305-326).
#include <cmath>
#include <cstring>
#include <mutex>

#include "b200_infer.h"
#include "kernels/cuda/kernel_f32.hpp"
#include "op_params.hpp"
#include "tensor.hpp"

namespace {

cudaError_t as_cuda(int rc) {
    switch (rc) {
        case B200_OK: return cudaSuccess;
        case B200_ERR_INVALID_ARGUMENT:
        case B200_ERR_OUT_OF_RANGE: return cudaErrorInvalidValue;
        case B200_ERR_NOT_SUPPORTED: return cudaErrorNotSupported;
        case B200_ERR_NO_MEMORY: return cudaErrorMemoryAllocation;
        default: return cudaErrorUnknown;
    }
}

const float *cf(const Tensor *t) { return static_cast<const float *>(t->data); }
float *mf(Tensor *t) { return static_cast<float *>(t->data); }

// The decode attention's split workspace, one per device: the reference places
// layers on several CUDA devices (src/model.cpp:400-437), and a kernel may only be
// given memory of the device it runs on. Zero-filled when allocated, grown with the
// context, and zeroed again after a call that failed (an aborted call can leave
// split-merge counters behind; every completed call leaves them at zero).
struct AttnWorkspace {
    void *ptr = nullptr;
    size_t bytes = 0;
    bool dirty = false;
};
constexpr int kMaxDevices = 64;
AttnWorkspace g_attn_ws[kMaxDevices];
std::mutex g_attn_ws_mu;

// The prefill GEMM's split-K partials, one grow-only buffer per device (contents
// need no initialisation: every split writes its whole partial tile).
struct GemmWorkspace {
    void *ptr = nullptr;
    size_t bytes = 0;
};
GemmWorkspace g_gemm_ws[kMaxDevices];
std::mutex g_gemm_ws_mu;

// Device that holds `p` (device memory only), or -1.
int device_of(const void *p) {
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, p) != cudaSuccess || pa.type != cudaMemoryTypeDevice || pa.device < 0 ||
        pa.device >= kMaxDevices) {
        cudaGetLastError();
        return -1;
    }
    return pa.device;
}

// Restores the current device on scope exit.
struct CurrentDevice {
    int prev = -1;
    explicit CurrentDevice(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~CurrentDevice() {
        int now = -1;
        if (prev >= 0 && cudaGetDevice(&now) == cudaSuccess && now != prev) cudaSetDevice(prev);
    }
};

}  // namespace

namespace CUDA_F32 {

cudaError_t compute_mul_mat(Tensor *dst, cudaStream_t s) {
    const Tensor *w = dst->src[0], *x = dst->src[1];
    if (w->dims[0] != x->dims[0] || w->dims[1] != dst->dims[0] || x->dims[1] != dst->dims[1])
        return cudaErrorInvalidValue;
    const int64_t K = w->dims[0], N = w->dims[1], M = x->dims[1];
    const size_t need = b200_mul_mat_workspace_bytes(K, N, M, B200_PREC_FFMA);
    if (need == 0) return as_cuda(b200_mul_mat(cf(w), cf(x), mf(dst), K, N, M, B200_PREC_FFMA, s));
    // prompts of a few hundred tokens: split K across the SMs through the workspace
    // of the device that holds x
    const int dev = device_of(x->data);
    if (dev < 0) return cudaErrorInvalidValue;
    CurrentDevice on(dev);
    std::lock_guard<std::mutex> lock(g_gemm_ws_mu);
    GemmWorkspace &ws = g_gemm_ws[dev];
    if (need > ws.bytes) {
        if (ws.ptr && cudaFree(ws.ptr) != cudaSuccess) return cudaErrorUnknown;
        ws.ptr = nullptr;
        ws.bytes = 0;
        if (cudaMalloc(&ws.ptr, need) != cudaSuccess) return cudaErrorMemoryAllocation;
        ws.bytes = need;
    }
    return as_cuda(b200_mul_mat_ws(cf(w), cf(x), mf(dst), K, N, M, B200_PREC_FFMA, ws.ptr, ws.bytes, s));
}

cudaError_t compute_rms_norm(Tensor *dst, cudaStream_t s) {
    const Tensor *x = dst->src[0], *gamma = dst->src[1];
    float eps = 0.f;
    std::memcpy(&eps, &dst->op_params[0], sizeof eps);
    return as_cuda(b200_rms_norm(cf(x), cf(gamma), mf(dst), x->dims[0], x->dims[1] * x->dims[2] * x->dims[3], eps, s));
}

cudaError_t compute_rope(Tensor *dst, cudaStream_t s) {
    const Tensor *x = dst->src[0], *pos = dst->src[1], *tab = dst->src[2];
    return as_cuda(b200_rope(cf(x), static_cast<const int32_t *>(pos->data), cf(tab), tab->dims[1], mf(dst),
                             x->dims[0], x->dims[1], x->dims[2], nullptr, s));
}

cudaError_t compute_flash_attn(Tensor *dst, cudaStream_t s) {
    const Tensor *q = dst->src[0], *k = dst->src[1], *v = dst->src[2];
    AttnParams p{};
    std::memcpy(&p, dst->op_params, sizeof p);
    const int64_t D = q->dims[0];
    const float scale = p.scale > 0.0f ? p.scale : 1.0f / std::sqrt(static_cast<float>(D));
    // Decode splits merge through a zero-filled workspace that later calls reuse; it
    // grows with the context (the reference kernel mallocs a score matrix per call,
    // kernel_f32.cu:484-510). The workspace is the one of the device that holds q.
    const int dev = device_of(q->data);
    if (dev < 0) return cudaErrorInvalidValue;
    CurrentDevice on(dev);
    std::lock_guard<std::mutex> lock(g_attn_ws_mu);
    AttnWorkspace &ws = g_attn_ws[dev];
    const size_t need = b200_flash_attn_workspace_bytes(D, q->dims[1], k->dims[1], q->dims[2], k->dims[2]);
    if (need > ws.bytes) {
        if (ws.ptr && cudaFree(ws.ptr) != cudaSuccess) return cudaErrorUnknown;
        ws.ptr = nullptr;
        ws.bytes = 0;
        if (cudaMalloc(&ws.ptr, need) != cudaSuccess) return cudaErrorMemoryAllocation;
        ws.bytes = need;
        ws.dirty = true;
    }
    if (ws.dirty) {
        if (cudaMemsetAsync(ws.ptr, 0, ws.bytes, s) != cudaSuccess) return cudaErrorUnknown;
        ws.dirty = false;
    }
    // K / V are views of the cache: token stride strides[2], head stride strides[1] (bytes)
    const cudaError_t rc =
        as_cuda(b200_flash_attn(cf(q), cf(k), cf(v), mf(dst), D, q->dims[1], k->dims[1], q->dims[2], k->dims[2],
                                static_cast<int64_t>(p.n_ctx), scale, k->strides[2] / 4, k->strides[1] / 4,
                                v->strides[2] / 4, v->strides[1] / 4, ws.ptr, ws.bytes, s));
    if (rc != cudaSuccess) ws.dirty = true;
    return rc;
}

cudaError_t compute_get_rows(Tensor *dst, cudaStream_t s) {
    const Tensor *table = dst->src[0], *ids = dst->src[1];
    return as_cuda(b200_get_rows(cf(table), static_cast<const int32_t *>(ids->data), mf(dst), table->dims[0],
                                 ids->dims[0], table->dims[1], nullptr, s));
}

cudaError_t compute_silu(Tensor *dst, cudaStream_t s) {
    return as_cuda(b200_silu(cf(dst->src[0]), mf(dst), static_cast<int64_t>(dst->element_count()), s));
}

cudaError_t compute_mul(Tensor *dst, cudaStream_t s) {
    return as_cuda(b200_mul(cf(dst->src[0]), cf(dst->src[1]), mf(dst), static_cast<int64_t>(dst->element_count()), s));
}

cudaError_t compute_add(Tensor *dst, cudaStream_t s) {
    return as_cuda(b200_add(cf(dst->src[0]), cf(dst->src[1]), mf(dst), static_cast<int64_t>(dst->element_count()), s));
}

cudaError_t compute_cpy(Tensor *dst, cudaStream_t s) {
    const Tensor *src = dst->src[0];
    if (src->dataType != dst->dataType || src->dims != dst->dims) return cudaErrorInvalidValue;
    return as_cuda(b200_copy(dst->data, src->data, src->byte_size(), s));
}

cudaError_t compute_reshape(Tensor *dst, cudaStream_t s) {
    const Tensor *src = dst->src[0];
    if (src->dataType != dst->dataType || src->element_count() != dst->element_count()) return cudaErrorInvalidValue;
    return as_cuda(b200_copy(dst->data, src->data, src->byte_size(), s));
}

cudaError_t compute_view(Tensor *, cudaStream_t) { return cudaSuccess; }

}  // namespace CUDA_F32
