// Normalisation, RoPE, gather, activation and sampling kernels (sm_100a).
//
// Rounding follows the reference CPU backend where it is cheap to do so:
// RMSNorm squares are float products accumulated in double with
// scale = float(1/sqrt(mean + eps)) (cpu_backend.cpp:369-376); RoPE angles are
// float(double(pos) * freq_j) exactly as the reference's host table
// (graph.cpp:119-131); products that the reference rounds separately are kept
// unfused (__fmul_rn) so only sin/cos differ (CUDA sincosf vs glibc, <= 1-2 ulp).
#include "elementwise.cuh"
#include "rope.cuh"

namespace b200 {
namespace {

// ---------------------------------------------------------------------------
// RMSNorm: one warp per row.
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *__restrict__ x,
                                                       const float *__restrict__ gamma,
                                                       float *__restrict__ out, int64_t D,
                                                       int64_t rows, float eps, bool round_tf32) {
    grid_launch_dependents();
    grid_wait();
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *xr = x + row * D;
    float *yr = out + row * D;
    double ss = 0.0;
    for (int64_t k = lane; k < D; k += 32) {
        const float v = xr[k];
        const float sq = v * v;
        ss += static_cast<double>(sq);
    }
    ss = warp_sum(ss);
    const float sc = rms_scale_from_sumsq(ss, D, eps);
    for (int64_t k = lane; k < D; k += 32) {
        const float y = __fmul_rn(__fmul_rn(xr[k], sc), gamma[k]);
        yr[k] = round_tf32 ? tf32_rn(y) : y;
    }
}

// ---------------------------------------------------------------------------
// RoPE from the reference's angle table [n_ctx][D/2]: one warp per (token, head).
__global__ void __launch_bounds__(256) rope_table_kernel(const float *__restrict__ x,
                                                         const int32_t *__restrict__ pos,
                                                         const float *__restrict__ table,
                                                         int64_t n_ctx, float *out, int64_t D,
                                                         int64_t H, int64_t T, int32_t *status) {
    grid_launch_dependents();
    grid_wait();
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= H * T) return;
    const int64_t t = row / H;
    const int64_t p = pos[t];
    if (p < 0 || p >= n_ctx) {
        if (lane == 0) set_status(status, B200_DEV_BAD_POSITION);
        return;
    }
    const int64_t half = D / 2;
    const float *src = x + row * D;
    float *dst = out + row * D;
    const float *ang = table + p * half;
    for (int64_t j = lane; j < half; j += 32) {
        float s, c;
        sincosf(ang[j], &s, &c);
        const float x0 = src[j], x1 = src[j + half];
        dst[j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        dst[j + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

// ---------------------------------------------------------------------------
// Fused QK RMSNorm + RoPE + KV-cache write: one warp per (token, head); lane l
// holds elements [l*E, l*E+E) so the rotation partner (j + D/2) is lane l^16.
template <int E>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const QkNormRopeArgs a) {
    grid_launch_dependents();
    grid_wait();
    const int64_t D = a.D;
    const int64_t heads = a.Hq + 2 * a.Hkv;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gw >= heads * a.T) return;
    const int64_t t = gw / heads, h = gw % heads;
    const int64_t p = a.pos ? static_cast<int64_t>(a.pos[t]) : static_cast<int64_t>(*a.pos_base) + t;
    const int64_t row = (a.out_offset ? static_cast<int64_t>(*a.out_offset) : 0) + t;
    if (p < 0 || p >= a.n_ctx) {
        if (lane == 0) set_status(a.status, B200_DEV_BAD_POSITION);
        return;
    }
    if (h >= a.Hq + a.Hkv) {  // V: plain copy into the cache slot
        if (!a.v_out) return;
        const int64_t hv = h - a.Hq - a.Hkv;
        const float *src = a.v_in + t * a.v_ld + hv * D;
        float *dst = a.v_out + row * a.v_out_ld + hv * D;
#pragma unroll
        for (int e = 0; e < E; ++e) dst[lane * E + e] = src[lane * E + e];
        return;
    }
    const bool is_q = h < a.Hq;
    const int64_t hh = is_q ? h : h - a.Hq;
    const float *src = is_q ? a.q_in + t * a.q_ld + hh * D : a.k_in + t * a.k_ld + hh * D;
    float *dst = is_q ? a.q_out + (t * a.Hq + hh) * D : a.k_out + row * a.k_out_ld + hh * D;
    warp_norm_rope_head<E>(src, is_q ? a.q_gamma : a.k_gamma, a.freq, p, a.eps, dst);
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

__global__ void __launch_bounds__(256) eltwise_kernel(int op, const float *__restrict__ a,
                                                      const float *__restrict__ b,
                                                      float *__restrict__ out, int64_t n) {
    grid_launch_dependents();
    grid_wait();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        float r;
        switch (op) {
            case 0: r = silu_f(a[i]); break;
            case 1: r = __fmul_rn(a[i], b[i]); break;
            case 2: r = __fadd_rn(a[i], b[i]); break;
            default: r = __fmul_rn(b[i], silu_f(a[i])); break;
        }
        out[i] = r;
    }
}

__global__ void __launch_bounds__(256) get_rows_kernel(const float *__restrict__ table,
                                                       const int32_t *__restrict__ ids,
                                                       float *__restrict__ out, int64_t D,
                                                       int64_t n_rows, int32_t *status) {
    grid_launch_dependents();
    grid_wait();
    const int64_t t = blockIdx.x;
    const int32_t id = ids[t];
    if (id < 0 || id >= n_rows) {
        if (threadIdx.x == 0) set_status(status, B200_DEV_BAD_TOKEN);
        return;
    }
    const float *src = table + static_cast<int64_t>(id) * D;
    float *dst = out + t * D;
    if ((D & 3) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int64_t k = threadIdx.x; k < D / 4; k += blockDim.x) d4[k] = s4[k];
    } else {
        for (int64_t k = threadIdx.x; k < D; k += blockDim.x) dst[k] = src[k];
    }
}

// ---------------------------------------------------------------------------
// Two-level greedy argmax: per-CTA first maximum, then the last CTA to finish
// reduces the CTA results in CTA order (lowest index wins ties, like
// sampler.cpp:51-59). NaN or +inf anywhere -> -1 and B200_DEV_BAD_LOGITS.
constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxMaxBlocks = 592;

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float *__restrict__ logits,
                                                                int64_t n, int32_t *out_id,
                                                                unsigned *counter, float *pv,
                                                                int32_t *pi, int32_t *status) {
    grid_launch_dependents();
    grid_wait();
    const int G = gridDim.x;
    const int64_t beg = n * blockIdx.x / G, end = n * (blockIdx.x + 1) / G;
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    bool bad = false;
    for (int64_t i = beg + threadIdx.x; i < end; i += kArgmaxThreads) {
        const float v = logits[i];
        if (isnan(v) || v == INFINITY) bad = true;
        if (v > bv) {  // per-thread indices increase: strict '>' keeps the first
            bv = v;
            bi = i;
        }
    }
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int64_t si[kArgmaxThreads / 32];
    __shared__ int sbad;
    if (threadIdx.x == 0) sbad = 0;
    __syncthreads();
    if (bad) sbad = 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[w] = bv;
        si[w] = bi;
    }
    __syncthreads();
    __shared__ unsigned ticket;
    if (threadIdx.x == 0) {
        float v = sv[0];
        int64_t i = si[0];
        for (int k = 1; k < kArgmaxThreads / 32; ++k)
            if (sv[k] > v || (sv[k] == v && si[k] < i)) {
                v = sv[k];
                i = si[k];
            }
        pv[blockIdx.x] = sbad ? NAN : v;
        pi[blockIdx.x] = sbad ? -2 : (i == INT64_MAX ? -1 : static_cast<int32_t>(i));
        __threadfence();
        ticket = atomicAdd(counter, 1u);
    }
    __syncthreads();
    if (ticket == static_cast<unsigned>(G - 1) && threadIdx.x == 0) {
        __threadfence();
        float v = -INFINITY;
        int32_t id = -1;
        bool any_bad = false;
        for (int b = 0; b < G; ++b) {
            const float bvv = __ldcg(pv + b);
            const int32_t bii = __ldcg(pi + b);
            if (bii == -2) any_bad = true;
            if (bvv > v) {
                v = bvv;
                id = bii;
            }
        }
        if (any_bad || id < 0) {
            id = -1;
            set_status(status, B200_DEV_BAD_LOGITS);
        }
        *out_id = id;
        *counter = 0u;
    }
}

int argmax_blocks(int64_t n) {
    int64_t b = (n + 4095) / 4096;
    if (b < 1) b = 1;
    if (b > kArgmaxMaxBlocks) b = kArgmaxMaxBlocks;
    return static_cast<int>(b);
}

unsigned grid_for(int64_t items, int per_block) {
    int64_t g = (items + per_block - 1) / per_block;
    if (g < 1) g = 1;
    return static_cast<unsigned>(g);
}

}  // namespace

cudaError_t rms_norm_launch(const float *x, const float *gamma, float *out, int64_t D, int64_t rows,
                            float eps, cudaStream_t stream, bool pdl, bool round_tf32) {
    if (rows == 0) return cudaSuccess;
    return b200_launch(rms_norm_kernel, dim3(grid_for(rows, 8)), dim3(256), 0, stream, pdl, x, gamma,
                       out, D, rows, eps, round_tf32);
}

cudaError_t rope_table_launch(const float *x, const int32_t *pos, const float *table, int64_t n_ctx,
                              float *out, int64_t D, int64_t H, int64_t T, int32_t *status,
                              cudaStream_t stream, bool pdl) {
    if (H * T == 0) return cudaSuccess;
    return b200_launch(rope_table_kernel, dim3(grid_for(H * T, 8)), dim3(256), 0, stream, pdl, x, pos,
                       table, n_ctx, out, D, H, T, status);
}

cudaError_t qk_norm_rope_launch(const QkNormRopeArgs &a, cudaStream_t stream, bool pdl) {
    if (a.T == 0) return cudaSuccess;
    const int64_t warps = a.T * (a.Hq + 2 * a.Hkv);
    const dim3 grid(grid_for(warps, 8)), block(256);
    switch (a.D) {
        case 32: return b200_launch(qk_norm_rope_kernel<1>, grid, block, 0, stream, pdl, a);
        case 64: return b200_launch(qk_norm_rope_kernel<2>, grid, block, 0, stream, pdl, a);
        case 128: return b200_launch(qk_norm_rope_kernel<4>, grid, block, 0, stream, pdl, a);
        case 256: return b200_launch(qk_norm_rope_kernel<8>, grid, block, 0, stream, pdl, a);
    }
    return cudaErrorInvalidValue;
}

cudaError_t eltwise_launch(int op, const float *a, const float *b, float *out, int64_t n,
                           cudaStream_t stream, bool pdl) {
    if (n == 0) return cudaSuccess;
    int64_t g = (n + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    return b200_launch(eltwise_kernel, dim3(static_cast<unsigned>(g)), dim3(256), 0, stream, pdl, op, a,
                       b, out, n);
}

cudaError_t get_rows_launch(const float *table, const int32_t *ids, float *out, int64_t D, int64_t n,
                            int64_t n_rows, int32_t *status, cudaStream_t stream, bool pdl) {
    if (n == 0) return cudaSuccess;
    return b200_launch(get_rows_kernel, dim3(static_cast<unsigned>(n)), dim3(256), 0, stream, pdl,
                       table, ids, out, D, n_rows, status);
}

size_t argmax_workspace(int64_t n) {
    return 256 + static_cast<size_t>(argmax_blocks(n)) * 8;
}

cudaError_t argmax_launch(const float *logits, int64_t n, int32_t *out_id, void *ws, int32_t *status,
                          cudaStream_t stream, bool pdl) {
    const int G = argmax_blocks(n);
    unsigned char *base = static_cast<unsigned char *>(ws);
    unsigned *counter = reinterpret_cast<unsigned *>(base);
    float *pv = reinterpret_cast<float *>(base + 256);
    int32_t *pi = reinterpret_cast<int32_t *>(base + 256 + static_cast<size_t>(G) * 4);
    return b200_launch(argmax_kernel, dim3(G), dim3(kArgmaxThreads), 0, stream, pdl, logits, n, out_id,
                       counter, pv, pi, status);
}

}  // namespace b200
