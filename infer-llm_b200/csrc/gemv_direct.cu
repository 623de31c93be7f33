// Decode GEMV, direct-streaming form (the default for even N).
//
// Critical-path design for batch-1 decode, where a step is ~140 short dependent
// kernels chained with programmatic dependent launch (PDL):
//   * Weights never depend on the previous kernel. Each warp therefore loads its
//     whole weight slice (2 rows x one K-slice, up to 8 x 16 B per lane per row)
//     into registers BEFORE griddepcontrol.wait, and asks the TMA engine to
//     prefetch any remainder into L2 (cp.async.bulk.prefetch.L2). The RMSNorm
//     gamma is staged in shared memory before the wait as well.
//   * After the wait only the activation vector is read: 128-bit loads, all
//     issued at once (one L2 round trip), the RMSNorm reduction, then FMAs from
//     registers.
// A CTA is 8 warps = (8/KS) row pairs x KS K-slices; KS is chosen per shape so
// the 8 MB projections still spread over >= 2 CTAs per SM. K-slices and warps
// are combined in a fixed order (deterministic results).
#include <algorithm>

#include "gemv.cuh"

namespace b200 {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxVpl = 8;  // float4 per lane per row held in registers

B200_DEVICE void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <int M, int EPI, int KS, int VPL>
__global__ void __launch_bounds__(kThreads) gemv_direct_kernel(const GemvArgs a, const int late_launch) {
    extern __shared__ __align__(16) float smem[];  // xs [M][K] | gamma [K]
    __shared__ float part[kWarps][2][M];
    __shared__ double s_red[kWarps][M];
    __shared__ float s_scale[M];

    constexpr int PAIRS = kWarps / KS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t K = a.K, K4 = K >> 2;
    const int pair = warp % PAIRS, sl = warp / PAIRS;
    const int64_t L4 = K4 / KS;  // host guarantees K4 % KS == 0
    const int64_t k4_beg = sl * L4;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * PAIRS + pair) * 2;
    const bool active = row < a.N;  // N is even
    float *xs = smem;
    float *gam = smem + static_cast<int64_t>(M) * K;

    const TraceMark tm(a.trace);
    if (!late_launch) grid_launch_dependents();

    // ---- before the dependency wait: weights -> registers, gamma -> smem
    const float4 *w0 = reinterpret_cast<const float4 *>(a.w + row * K) + k4_beg;
    const float4 *w1 = reinterpret_cast<const float4 *>(a.w + (row + 1) * K) + k4_beg;
    float4 r0[VPL], r1[VPL];
    if (active) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int64_t i = lane + 32 * j;
            if (i < L4) {
                r0[j] = ld_stream4(w0 + i);
                r1[j] = ld_stream4(w1 + i);
            }
        }
        const int64_t rest = L4 - 32 * VPL;  // float4s streamed after the wait
        if (rest > 0 && lane < 2)
            prefetch_l2((lane ? w1 : w0) + 32 * VPL, static_cast<uint32_t>(rest * 16));
    }
    if (a.gamma) {
        const float4 *g4 = reinterpret_cast<const float4 *>(a.gamma);
        for (int64_t i = tid; i < K4; i += kThreads) reinterpret_cast<float4 *>(gam)[i] = g4[i];
    }

    grid_wait();
    tm.waited();
    if (late_launch) grid_launch_dependents();

    // ---- activations: one 128-bit load per (thread, float4), all in flight together
    const int64_t x_ld = a.x_ld ? a.x_ld : K;
    double ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        ss[m] = 0.0;
        const float *src = a.x + m * x_ld;
        bool zero = false;
        if (a.embed_table) {
            const int32_t id = a.embed_ids[m];
            zero = id < 0 || id >= a.embed_rows;
            if (zero && tid == 0) set_status(a.status, B200_DEV_BAD_TOKEN);
            src = a.embed_table + (zero ? 0 : static_cast<int64_t>(id) * K);
        }
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *x4s = reinterpret_cast<float4 *>(xs + m * K);
        float4 *st4 = (a.x_store && blockIdx.x == 0) ? reinterpret_cast<float4 *>(a.x_store + m * K) : nullptr;
        for (int64_t i = tid; i < K4; i += kThreads) {
            float4 v = zero ? make_float4(0.f, 0.f, 0.f, 0.f) : s4[i];
            x4s[i] = v;
            if (st4) st4[i] = v;
            const float q0 = v.x * v.x, q1 = v.y * v.y, q2 = v.z * v.z, q3 = v.w * v.w;
            ss[m] += static_cast<double>(q0);
            ss[m] += static_cast<double>(q1);
            ss[m] += static_cast<double>(q2);
            ss[m] += static_cast<double>(q3);
        }
    }
    if (a.gamma) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const double w = warp_sum(ss[m]);
            if (lane == 0) s_red[warp][m] = w;
        }
    }
    __syncthreads();
    if (a.gamma && tid < M) {
        double t = 0.0;
        for (int w = 0; w < kWarps; ++w) t += s_red[w][tid];
        s_scale[tid] = rms_scale_from_sumsq(t, K, a.eps);
    }
    if (a.gamma) __syncthreads();
    tm.at(4);

    // ---- dot products: registers (and the streamed remainder) against x
    float acc0[M], acc1[M], sc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        acc0[m] = acc1[m] = 0.f;
        sc[m] = a.gamma ? s_scale[m] : 1.f;
    }
    const float4 *x4 = reinterpret_cast<const float4 *>(xs) + k4_beg;
    const float4 *gm4 = reinterpret_cast<const float4 *>(gam) + k4_beg;
    auto fma_step = [&](const float4 &u, const float4 &v, int64_t i) {
        float4 g = make_float4(1.f, 1.f, 1.f, 1.f);
        if (a.gamma) g = gm4[i];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float4 xv = x4[m * K4 + i];
            if (a.gamma) {  // reference order: (x * scale) * gamma, each rounded
                xv.x = __fmul_rn(__fmul_rn(xv.x, sc[m]), g.x);
                xv.y = __fmul_rn(__fmul_rn(xv.y, sc[m]), g.y);
                xv.z = __fmul_rn(__fmul_rn(xv.z, sc[m]), g.z);
                xv.w = __fmul_rn(__fmul_rn(xv.w, sc[m]), g.w);
            }
            acc0[m] = fmaf(u.x, xv.x, acc0[m]);
            acc0[m] = fmaf(u.y, xv.y, acc0[m]);
            acc0[m] = fmaf(u.z, xv.z, acc0[m]);
            acc0[m] = fmaf(u.w, xv.w, acc0[m]);
            acc1[m] = fmaf(v.x, xv.x, acc1[m]);
            acc1[m] = fmaf(v.y, xv.y, acc1[m]);
            acc1[m] = fmaf(v.z, xv.z, acc1[m]);
            acc1[m] = fmaf(v.w, xv.w, acc1[m]);
        }
    };
    if (active) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int64_t i = lane + 32 * j;
            if (i < L4) fma_step(r0[j], r1[j], i);
        }
#pragma unroll 4
        for (int64_t i = lane + 32 * VPL; i < L4; i += 32) fma_step(ld_stream4(w0 + i), ld_stream4(w1 + i), i);
    }
    tm.at(5);
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float s0 = warp_sum(acc0[m]), s1 = warp_sum(acc1[m]);
        if (lane == 0) {
            part[warp][0][m] = s0;
            part[warp][1][m] = s1;
        }
    }
    __syncthreads();
    tm.done();

    // combine K-slices (slice order) + epilogue
    if (EPI == GEMV_ARGMAX) {
        // M == 1; rows of this CTA in increasing order -> first maximum
        __shared__ unsigned s_ticket;
        if (tid == 0) {
            float bv = -INFINITY;
            int64_t bi = -1;
            bool bad = false;
            for (int p = 0; p < PAIRS; ++p)
                for (int h = 0; h < 2; ++h) {
                    const int64_t r = (static_cast<int64_t>(blockIdx.x) * PAIRS + p) * 2 + h;
                    if (r >= a.N) continue;
                    float v = 0.f;
                    for (int s = 0; s < KS; ++s) v += part[s * PAIRS + p][h][0];
                    if (a.out) a.out[r] = v;
                    if (isnan(v) || v == INFINITY) bad = true;
                    if (v > bv) {
                        bv = v;
                        bi = r;
                    }
                }
            a.part_val[blockIdx.x] = bad ? NAN : bv;
            a.part_idx[blockIdx.x] = bad ? -2 : static_cast<int32_t>(bi);
            __threadfence();
            s_ticket = atomicAdd(a.counter, 1u);
        }
        __syncthreads();
        const unsigned G = gridDim.x;
        if (s_ticket != G - 1) return;
        __threadfence();
        // last CTA: reduce the per-CTA results (CTAs own increasing row ranges)
        float bv = -INFINITY;
        int64_t bi = INT64_MAX;
        bool bad = false;
        for (unsigned b = tid; b < G; b += kThreads) {  // per thread: increasing b
            const float v = __ldcg(a.part_val + b);
            const int32_t i = __ldcg(a.part_idx + b);
            if (i == -2) bad = true;
            if (v > bv) {
                bv = v;
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        bad = __any_sync(0xffffffffu, bad);
        __shared__ float fv[kWarps];
        __shared__ int64_t fi[kWarps];
        __shared__ int fb[kWarps];
        if (lane == 0) {
            fv[warp] = bv;
            fi[warp] = bi;
            fb[warp] = bad;
        }
        __syncthreads();
        if (tid == 0) {
            float v = fv[0];
            int64_t i = fi[0];
            bool anyb = fb[0];
            for (int w = 1; w < kWarps; ++w) {
                anyb |= fb[w] != 0;
                if (fv[w] > v || (fv[w] == v && fi[w] < i)) {
                    v = fv[w];
                    i = fi[w];
                }
            }
            int32_t gi;
            if (anyb || i < 0 || i == INT64_MAX) {
                gi = -1;
                set_status(a.status, B200_DEV_BAD_LOGITS);
            } else {
                gi = static_cast<int32_t>(i + a.idx_offset);
            }
            *a.argmax_out = gi;
            if (a.best_val_out) *a.best_val_out = anyb ? NAN : v;
            if (a.token_log) {
                const int32_t p = *a.log_pos;
                a.token_log[p % a.log_cap] = gi;
                *a.log_pos = p + 1;
            }
            if (a.n_past) *a.n_past += a.n_past_add;
            *a.counter = 0u;
        }
        return;
    }
    if (tid < PAIRS * 2 * M) {
        const int p = tid / (2 * M), h = (tid / M) % 2, m = tid % M;
        const int64_t r = (static_cast<int64_t>(blockIdx.x) * PAIRS + p) * 2 + h;
        if (r < a.N) {
            float v = 0.f;
            for (int s = 0; s < KS; ++s) v += part[s * PAIRS + p][h][m];
            if (EPI == GEMV_SWIGLU) {
                // rows (2i, 2i+1) = (gate_i, up_i): the h == 0 thread owns the pair
                float u = 0.f;
                for (int s = 0; s < KS; ++s) u += part[s * PAIRS + p][1][m];
                if (h == 0) {
                    const int64_t o_ld = a.out_ld ? a.out_ld : a.N / 2;
                    const float sg = v / (1.0f + expf(-v));
                    a.out[m * o_ld + r / 2] = u * sg;
                }
            } else {
                const int64_t o_ld = a.out_ld ? a.out_ld : a.N;
                const int64_t idx = m * o_ld + r;
                if (EPI == GEMV_RESIDUAL) v = v + a.residual[idx];
                a.out[idx] = v;
            }
        }
    }
}

int vpl_for(int64_t L4) {
    const int64_t v = (L4 + 31) / 32;
    if (v <= 1) return 1;
    if (v <= 2) return 2;
    if (v <= 3) return 3;
    if (v <= 4) return 4;
    if (v <= 6) return 6;
    return kMaxVpl;
}

template <int M, int EPI, int KS, int VPL>
cudaError_t launch4(const GemvArgs &a, cudaStream_t st, bool pdl) {
    constexpr int rows_cta = 2 * kWarps / KS;
    const unsigned grid = static_cast<unsigned>((a.N + rows_cta - 1) / rows_cta);
    const size_t smem = (static_cast<size_t>(M) + (a.gamma ? 1 : 0)) * a.K * 4;
    auto kern = gemv_direct_kernel<M, EPI, KS, VPL>;
    if (smem > 40 * 1024) {  // dynamic + static shared memory above the 48 KB default
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return b200_launch(kern, dim3(grid), dim3(kThreads), smem, st, pdl, a, a.late_launch ? 1 : 0);
}

template <int M, int EPI, int KS>
cudaError_t launch3(const GemvArgs &a, cudaStream_t st, bool pdl) {
    switch (vpl_for(a.K / 4 / KS)) {
        case 1: return launch4<M, EPI, KS, 1>(a, st, pdl);
        case 2: return launch4<M, EPI, KS, 2>(a, st, pdl);
        case 3: return launch4<M, EPI, KS, 3>(a, st, pdl);
        case 4: return launch4<M, EPI, KS, 4>(a, st, pdl);
        case 6: return launch4<M, EPI, KS, 6>(a, st, pdl);
        default: return launch4<M, EPI, KS, kMaxVpl>(a, st, pdl);
    }
}

template <int M, int EPI>
cudaError_t launch2(const GemvArgs &a, int ks, cudaStream_t st, bool pdl) {
    switch (ks) {
        case 1: return launch3<M, EPI, 1>(a, st, pdl);
        case 2: return launch3<M, EPI, 2>(a, st, pdl);
        case 4: return launch3<M, EPI, 4>(a, st, pdl);
        case 8: return launch3<M, EPI, 8>(a, st, pdl);
    }
    return cudaErrorInvalidValue;
}

template <int M>
cudaError_t launch1(const GemvArgs &a, int ks, cudaStream_t st, bool pdl) {
    switch (a.epi) {
        case GEMV_STORE: return launch2<M, GEMV_STORE>(a, ks, st, pdl);
        case GEMV_RESIDUAL: return launch2<M, GEMV_RESIDUAL>(a, ks, st, pdl);
        case GEMV_SWIGLU: return launch2<M, GEMV_SWIGLU>(a, ks, st, pdl);
        case GEMV_ARGMAX: return launch2<1, GEMV_ARGMAX>(a, ks, st, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

int gemv_direct_ks(int64_t N, int64_t K) {
    // fewest K-slices that still give >= 2 CTAs per SM (K4 must split evenly)
    const int64_t want = 2 * static_cast<int64_t>(device_sm_count());
    int ks = 1;
    while (ks < 8 && (N + 2 * kWarps / ks - 1) / (2 * kWarps / ks) < want && (K / 4) % (ks * 2) == 0) ks *= 2;
    return ks;
}

int gemv_direct_grid(int64_t N, int64_t K) {
    const int ks = gemv_direct_ks(N, K);
    const int rows_cta = 2 * kWarps / ks;
    return static_cast<int>((N + rows_cta - 1) / rows_cta);
}

cudaError_t gemv_direct_launch(const GemvArgs &a, cudaStream_t st, bool pdl) {
    if (a.M < 1 || a.M > 4 || (a.K & 3) || a.K <= 0 || a.N <= 0 || (a.N & 1)) return cudaErrorInvalidValue;
    if (a.epi == GEMV_ARGMAX && a.M != 1) return cudaErrorInvalidValue;
    if ((static_cast<size_t>(a.M) + 1) * a.K * 4 > 200 * 1024) return cudaErrorInvalidValue;
    const int ks = gemv_direct_ks(a.N, a.K);
    switch (a.M) {
        case 1: return launch1<1>(a, ks, st, pdl);
        case 2: return launch1<2>(a, ks, st, pdl);
        case 3: return launch1<3>(a, ks, st, pdl);
        case 4: return launch1<4>(a, ks, st, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace b200
