// Per-head RMSNorm + NeoX RoPE for one warp (shared by the fused QK-norm kernel
// and the fused decode-attention prologue).
#pragma once

#include "common.cuh"

namespace b200 {

// One warp normalises one head of D = 32*E floats and rotates it by position
// `pos`. Lane l holds elements [l*E, l*E+E), so the rotation partner j + D/2 of
// element j sits in lane l^16. Rounding follows the reference: squares are float
// products summed in double (cpu_backend.cpp:369-376), y = (x * scale) * gamma,
// angle = float(double(pos) * freq_j) (graph.cpp:119-131), separately rounded
// products in the rotation (cpu_backend.cpp:514-519).
// L2_ONLY: read `src` with ld.global.cg (for data other SMs rewrote since this SM
// last read the same address, e.g. inside a persistent kernel).
template <int E, bool L2_ONLY = false>
B200_DEVICE void warp_norm_rope_head(const float *__restrict__ src, const float *__restrict__ gamma,
                                     const float *__restrict__ freq, int64_t pos, float eps,
                                     float *__restrict__ dst) {
    constexpr int D = 32 * E;
    const int lane = threadIdx.x & 31;
    float v[E];
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        v[e] = L2_ONLY ? __ldcg(src + lane * E + e) : src[lane * E + e];
        const float sq = v[e] * v[e];
        ss += static_cast<double>(sq);
    }
    ss = warp_sum(ss);
    const float sc = rms_scale_from_sumsq(ss, D, eps);
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], sc), gamma[lane * E + e]);
    const bool lo = lane < 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const float other = __shfl_xor_sync(0xffffffffu, v[e], 16);
        const int j = (lo ? lane : lane - 16) * E + e;
        const float ang = static_cast<float>(static_cast<double>(pos) * static_cast<double>(freq[j]));
        float s, c;
        sincosf(ang, &s, &c);
        dst[lane * E + e] = lo ? __fsub_rn(__fmul_rn(v[e], c), __fmul_rn(other, s))
                               : __fadd_rn(__fmul_rn(other, s), __fmul_rn(v[e], c));
    }
}

}  // namespace b200
