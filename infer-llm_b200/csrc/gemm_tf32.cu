// Placeholder until the tcgen05 TF32 GEMM lands: the engine and b200_mul_mat
// treat cudaErrorNotSupported as "use the FFMA GEMM".
#include "gemm.cuh"

namespace b200 {
cudaError_t gemm_tf32_launch(const GemmArgs &, cudaStream_t, bool) { return cudaErrorNotSupported; }
}  // namespace b200
