// Decode GEMV, direct-streaming form (the default for even N).
//
// Critical-path design for batch-1 decode, where a step is ~140 short dependent
// kernels chained with programmatic dependent launch (PDL):
//   * A persistent grid (<= 2 CTAs per SM) whose warps loop over row pairs; a
//     CTA is 8 warps = (8/KS) row pairs x KS K-slices, KS chosen so a warp holds
//     at most 4 x 16 B per lane per row.
//   * Weights never depend on the previous kernel: before griddepcontrol.wait
//     each warp loads its first row pair into registers and asks the TMA engine
//     to prefetch its next two row pairs into L2 (cp.async.bulk.prefetch.L2);
//     every CTA also prefetches its share of the NEXT kernel's weights into L2.
//     Inside the loop the next pair is loaded while the current one is used and
//     the prefetch runs two pairs ahead.
//   * After the wait only the activation vector is read (128-bit loads, one L2
//     round trip), RMS-normalised in shared memory if requested.
// K-slices, warps and CTAs are combined in a fixed order (deterministic).
#include <algorithm>

#include "gemv.cuh"

namespace b200 {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxVpl = 4;  // float4 per lane per row held in registers

// ONESHOT: the grid covers every row pair once and is small enough to be resident
// in full (so all weights are in registers before the wait); otherwise the grid is
// persistent and warps loop with a one-pair register double buffer.
template <int M, int EPI, int KS, int VPL, bool ONESHOT>
__global__ void __launch_bounds__(kThreads, ONESHOT ? 4 : 2) gemv_direct_kernel(const GemvArgs a, const int late_launch) {
    extern __shared__ __align__(16) float smem[];  // xs [M][K] | gamma [K]
    __shared__ float part[kWarps][2][M];
    __shared__ double s_red[kWarps][M];
    __shared__ float s_scale[M];
    __shared__ float s_bv[kWarps];
    __shared__ int64_t s_bi[kWarps];
    __shared__ int s_bad[kWarps];
    __shared__ unsigned s_ticket;

    constexpr int PAIRS = kWarps / KS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t K = a.K, K4 = K >> 2;
    const int pair = warp % PAIRS, sl = warp / PAIRS;
    const int64_t L4 = K4 / KS;  // host guarantees K4 % KS == 0 and L4 <= 32 * VPL
    const int64_t k4_beg = sl * L4;
    const int64_t n_pairs = a.N / 2;  // N is even
    const int64_t pstride = static_cast<int64_t>(gridDim.x) * PAIRS;
    const int64_t p0 = static_cast<int64_t>(blockIdx.x) * PAIRS + pair;
    const int iters =
        ONESHOT ? 1 : static_cast<int>((n_pairs - static_cast<int64_t>(blockIdx.x) * PAIRS + pstride - 1) / pstride);
    float *xs = smem;
    float *gam = smem + static_cast<int64_t>(M) * K;

    const TraceMark tm(a.trace);
    if (!late_launch) grid_launch_dependents();
    prefetch_share_l2(a.next_w, a.next_w_bytes);

    auto wrow = [&](int64_t p, int h) {
        return reinterpret_cast<const float4 *>(a.w + (2 * p + h) * K) + k4_beg;
    };
    auto load_pair = [&](int64_t p, float4 (&u)[VPL], float4 (&v)[VPL]) {
        if (p >= n_pairs) return;
        const float4 *w0 = wrow(p, 0), *w1 = wrow(p, 1);
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int64_t i = lane + 32 * j;
            if (i < L4) {
                u[j] = ld_stream4(w0 + i);
                v[j] = ld_stream4(w1 + i);
            }
        }
    };
    auto prefetch_pair = [&](int64_t p) {  // lanes 0, 1: the pair's two row slices
        if (p < n_pairs && lane < 2) prefetch_l2_bulk(wrow(p, lane), static_cast<uint32_t>(L4 * 16));
    };

    // ---- before the dependency wait: weights -> registers / L2, gamma -> smem
    float4 cu[VPL], cv[VPL], nu[VPL], nv[VPL];
    prefetch_pair(p0 + pstride);
    prefetch_pair(p0 + 2 * pstride);
    load_pair(p0, cu, cv);
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

    float sc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) sc[m] = a.gamma ? s_scale[m] : 1.f;
    const float4 *x4 = reinterpret_cast<const float4 *>(xs) + k4_beg;
    const float4 *gm4 = reinterpret_cast<const float4 *>(gam) + k4_beg;
    float best_v = -INFINITY;  // ARGMAX: the combining thread's running first maximum
    int64_t best_i = INT64_MAX;
    bool bad = false;

    for (int it = 0; it < iters; ++it) {
        const int64_t p = p0 + it * pstride;
        if (!ONESHOT && it + 1 < iters) load_pair(p + pstride, nu, nv);
        prefetch_pair(p + 3 * pstride);
        float acc0[M], acc1[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc0[m] = acc1[m] = 0.f;
        if (p < n_pairs) {
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const int64_t i = lane + 32 * j;
                if (i >= L4) continue;
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
                    acc0[m] = fmaf(cu[j].x, xv.x, acc0[m]);
                    acc0[m] = fmaf(cu[j].y, xv.y, acc0[m]);
                    acc0[m] = fmaf(cu[j].z, xv.z, acc0[m]);
                    acc0[m] = fmaf(cu[j].w, xv.w, acc0[m]);
                    acc1[m] = fmaf(cv[j].x, xv.x, acc1[m]);
                    acc1[m] = fmaf(cv[j].y, xv.y, acc1[m]);
                    acc1[m] = fmaf(cv[j].z, xv.z, acc1[m]);
                    acc1[m] = fmaf(cv[j].w, xv.w, acc1[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float s0 = warp_sum(acc0[m]), s1 = warp_sum(acc1[m]);
            if (lane == 0) {
                part[warp][0][m] = s0;
                part[warp][1][m] = s1;
            }
        }
        __syncthreads();
        // combine K-slices (slice order) + epilogue: thread t -> (pair, half, m)
        if (tid < PAIRS * 2 * M) {
            const int pp = tid / (2 * M), h = (tid / M) % 2, m = tid % M;
            const int64_t prow = static_cast<int64_t>(blockIdx.x) * PAIRS + pp + it * pstride;
            const int64_t r = 2 * prow + h;
            if (prow < n_pairs) {
                float v = 0.f;
                for (int s = 0; s < KS; ++s) v += part[s * PAIRS + pp][h][m];
                if (EPI == GEMV_ARGMAX) {
                    if (a.out) a.out[r] = v;
                    if (isnan(v) || v == INFINITY) bad = true;
                    if (v > best_v || (v == best_v && r < best_i)) {
                        best_v = v;
                        best_i = r;
                    }
                } else if (EPI == GEMV_SWIGLU) {
                    // rows (2i, 2i+1) = (gate_i, up_i): the h == 0 thread owns the pair
                    if (h == 0) {
                        float u = 0.f;
                        for (int s = 0; s < KS; ++s) u += part[s * PAIRS + pp][1][m];
                        const int64_t o_ld = a.out_ld ? a.out_ld : a.N / 2;
                        const float sg = v / (1.0f + expf(-v));
                        a.out[m * o_ld + prow] = u * sg;
                    }
                } else {
                    const int64_t o_ld = a.out_ld ? a.out_ld : a.N;
                    const int64_t idx = m * o_ld + r;
                    if (EPI == GEMV_RESIDUAL) v = v + a.residual[idx];
                    a.out[idx] = v;
                }
            }
        }
        __syncthreads();
        if (it + 1 < iters) {
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                cu[j] = nu[j];
                cv[j] = nv[j];
            }
        }
    }
    tm.at(5);
    tm.done();
    if constexpr (EPI == GEMV_ARGMAX) {

    // ---- ARGMAX (M == 1): CTA first maximum -> per-CTA slot -> last CTA reduces.
    // Ties go to the lower row everywhere (sampler.cpp:51-59).
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ov > best_v || (ov == best_v && oi < best_i)) {
            best_v = ov;
            best_i = oi;
        }
    }
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        s_bv[warp] = best_v;
        s_bi[warp] = best_i;
        s_bad[warp] = bad;
    }
    __syncthreads();
    if (tid == 0) {
        float v = s_bv[0];
        int64_t i = s_bi[0];
        bool anyb = s_bad[0];
        for (int w = 1; w < kWarps; ++w) {
            anyb |= s_bad[w] != 0;
            if (s_bv[w] > v || (s_bv[w] == v && s_bi[w] < i)) {
                v = s_bv[w];
                i = s_bi[w];
            }
        }
        a.part_val[blockIdx.x] = anyb ? NAN : v;
        a.part_idx[blockIdx.x] = anyb ? -2 : (i == INT64_MAX ? -1 : static_cast<int32_t>(i));
        __threadfence();
        s_ticket = atomicAdd(a.counter, 1u);
    }
    __syncthreads();
    const unsigned G = gridDim.x;
    if (s_ticket != G - 1) return;
    __threadfence();
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    bool gbad = false;
    for (unsigned b = tid; b < G; b += kThreads) {
        const float v = __ldcg(a.part_val + b);
        const int32_t i = __ldcg(a.part_idx + b);
        if (i == -2) gbad = true;
        if (i >= 0 && (v > bv || (v == bv && i < bi))) {
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
    gbad = __any_sync(0xffffffffu, gbad);
    __syncthreads();  // s_bv / s_bi reused
    if (lane == 0) {
        s_bv[warp] = bv;
        s_bi[warp] = bi;
        s_bad[warp] = gbad;
    }
    __syncthreads();
    if (tid == 0) {
        float v = s_bv[0];
        int64_t i = s_bi[0];
        bool anyb = s_bad[0];
        for (int w = 1; w < kWarps; ++w) {
            anyb |= s_bad[w] != 0;
            if (s_bv[w] > v || (s_bv[w] == v && s_bi[w] < i)) {
                v = s_bv[w];
                i = s_bi[w];
            }
        }
        int32_t gi;
        if (anyb || i == INT64_MAX) {
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
    }  // ARGMAX
}

int vpl_for(int64_t L4) {
    const int64_t v = (L4 + 31) / 32;
    return static_cast<int>(v < 1 ? 1 : v);
}

// One-shot when the covering grid fits 4 CTAs per SM (launch bound 4 caps the
// kernel at 64 registers per thread) and its shared memory allows 4 per SM.
bool use_oneshot(int64_t N, int64_t K, int M, bool norm) {
    const int ks = gemv_direct_ks(N, K);
    const int64_t pairs_cta = kWarps / ks;
    const int64_t need = (N / 2 + pairs_cta - 1) / pairs_cta;
    const size_t smem = (static_cast<size_t>(M) + (norm ? 1 : 0)) * K * 4;
    const int64_t vpl = (K / 4 / ks + 31) / 32;
    return need <= 4 * static_cast<int64_t>(device_sm_count()) && smem <= 56 * 1024 && M == 1 && vpl <= 3;
}

template <int M, int EPI, int KS, int VPL>
cudaError_t launch4(const GemvArgs &a, cudaStream_t st, bool pdl) {
    const int grid = gemv_direct_grid(a.N, a.K, a.M, a.gamma != nullptr);
    const size_t smem = (static_cast<size_t>(M) + (a.gamma ? 1 : 0)) * a.K * 4;
    auto kern = gemv_direct_kernel<M, EPI, KS, VPL, false>;
    if constexpr (M == 1 && VPL <= 3) {  // one-shot fits the 64-register bound without spills
        if (use_oneshot(a.N, a.K, a.M, a.gamma != nullptr)) kern = gemv_direct_kernel<M, EPI, KS, VPL, true>;
    }
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
    }
    return cudaErrorInvalidValue;
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

// K-slices per row: enough that a lane holds <= 4 float4 per row, then enough that
// the one-shot grid would give >= 2 CTAs per SM; 0 if K cannot be split that way.
int gemv_direct_ks(int64_t N, int64_t K) {
    const int64_t K4 = K / 4;
    const int64_t want = 2 * static_cast<int64_t>(device_sm_count());
    int ks = 1;
    while (ks <= 8 && (K4 % ks != 0 || K4 / ks > 32 * kMaxVpl)) ks *= 2;
    if (ks > 8) return 0;
    while (ks < 8 && K4 % (ks * 2) == 0 && (N / 2 + kWarps / ks - 1) / (kWarps / ks) < want) ks *= 2;
    return ks;
}

int gemv_direct_grid(int64_t N, int64_t K, int M, bool norm) {
    const int ks = gemv_direct_ks(N, K);
    if (ks == 0) return 1;
    const int64_t pairs_cta = kWarps / ks;
    const int64_t need = (N / 2 + pairs_cta - 1) / pairs_cta;
    if (use_oneshot(N, K, M, norm)) return static_cast<int>(need);
    return static_cast<int>(std::min<int64_t>(need, 2 * static_cast<int64_t>(device_sm_count())));
}

cudaError_t gemv_direct_launch(const GemvArgs &a, cudaStream_t st, bool pdl) {
    if (a.M < 1 || a.M > 4 || (a.K & 3) || a.K <= 0 || a.N <= 0 || (a.N & 1)) return cudaErrorInvalidValue;
    if (a.epi == GEMV_ARGMAX && a.M != 1) return cudaErrorInvalidValue;
    if ((static_cast<size_t>(a.M) + 1) * a.K * 4 > 200 * 1024) return cudaErrorInvalidValue;
    const int ks = gemv_direct_ks(a.N, a.K);
    if (ks == 0) return cudaErrorNotSupported;
    switch (a.M) {
        case 1: return launch1<1>(a, ks, st, pdl);
        case 2: return launch1<2>(a, ks, st, pdl);
        case 3: return launch1<3>(a, ks, st, pdl);
        case 4: return launch1<4>(a, ks, st, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace b200
