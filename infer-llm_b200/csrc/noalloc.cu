// Allocation-free greedy argmax: b200_argmax with its scratch in a fixed,
// library-owned device array instead of a caller-provided workspace.
//
// Some callers cannot allocate device memory for a workspace: a kernel seam that
// receives only tensors and a stream (like the reference's
// CUDA_F32::compute_*(Tensor*, cudaStream_t), which has no workspace argument
// and no allocator), or a host that must not call cudaMalloc between steps,
// where an allocation would synchronise the device and stall the pipeline.
// This entry point serves them. Its scratch is a file-scope __device__ array of
// B200_ARGMAX_NOALLOC_SCRATCH bytes that every GPU loading the library holds
// until exit; every call shares it.
#include "elementwise.cuh"

namespace {

constexpr size_t kScratchBytes = B200_ARGMAX_NOALLOC_SCRATCH;
__device__ __align__(256) unsigned char g_argmax_scratch[kScratchBytes];

// The device address of g_argmax_scratch on the current device. In host code the
// array's name is only a host-side stand-in, never a device address. It is looked
// up on every call (a cheap query once the module is loaded), so it stays right
// after a device reset reloads the module at another address. The first call on a
// device loads the module there; make it before any stream capture.
int scratch_for_current_device(void **out) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return B200_ERR_CUDA;
    }
    *out = p;
    return B200_OK;
}

}  // namespace

extern "C" int b200_argmax_noalloc(const float *logits, int64_t n, int32_t *out_id, int32_t *dev_status,
                                   void *stream) {
    if (!logits || !out_id || n <= 0) return B200_ERR_INVALID_ARGUMENT;
    if (n > B200_ARGMAX_NOALLOC_MAX_N) return B200_ERR_INVALID_ARGUMENT;  // ids are int32
    if (b200::argmax_workspace(n) > kScratchBytes) return B200_ERR_INVALID_ARGUMENT;
    void *ws = nullptr;
    const int rc = scratch_for_current_device(&ws);
    if (rc != B200_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The finishing CTA counter must start at zero: a call that was interrupted
    // could have left it set, so it is cleared on every call.
    if (cudaMemsetAsync(ws, 0, 4, st) != cudaSuccess) return B200_ERR_CUDA;
    const cudaError_t e = b200::argmax_launch(logits, n, out_id, ws, dev_status, st, false);
    return e == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}
