// HBM-streaming decode GEMV for sm_100a.
//
// Work split: CTA b owns a contiguous block of weight rows (a contiguous byte
// range of W) and streams it through a ring of shared-memory stages with
// cp.async.bulk (the bulk-copy form of the TMA engine) issued by one producer
// warp. The producer starts before griddepcontrol.wait, so under programmatic
// dependent launch the next kernel's weight traffic overlaps the previous
// kernel's tail; only the activations wait for the previous kernel. Eight
// consumer warps split each stage's rows x K-slices, reduce with warp shuffles
// and combine the K-slices in a fixed order (deterministic results).
#include "gemv.cuh"

#include <algorithm>
#include <cstdlib>

namespace b200 {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + producer warp
constexpr int kMaxRpc = 8;
constexpr uint32_t kStageTarget = 16384;   // bytes per stage (rows are kept whole)
constexpr uint32_t kStageBudget = 98304;   // ring size target

struct Layout {
    int rpc;          // weight rows per stage
    int stages;
    uint32_t stage_floats;
    size_t smem;      // dynamic shared memory bytes
    size_t off_x, off_stage, off_part, off_best;
};

Layout make_layout(int64_t K, int M, int epi, int64_t rows_cta) {
    Layout L;
    const uint32_t row_bytes = static_cast<uint32_t>(K * 4);
    int rpc = static_cast<int>(std::max<uint32_t>(1u, kStageTarget / row_bytes));
    int p = 1;
    while (p * 2 <= rpc && p * 2 <= kMaxRpc) p *= 2;
    rpc = p;
    if (epi == GEMV_SWIGLU && rpc < 2) rpc = 2;  // a (gate, up) pair never straddles stages
    L.rpc = rpc;
    const uint32_t stage_bytes = row_bytes * rpc;
    L.stages = static_cast<int>(std::min<uint32_t>(8u, std::max<uint32_t>(2u, kStageBudget / stage_bytes)));
    L.stage_floats = stage_bytes / 4;
    size_t off = 2 * 8 * 8;  // full[8] + empty[8] mbarriers
    L.off_x = off;
    off += static_cast<size_t>(M) * K * 4;
    off = (off + 127) & ~size_t(127);
    L.off_stage = off;
    off += static_cast<size_t>(L.stages) * stage_bytes;
    L.off_part = off;
    off += static_cast<size_t>(rows_cta) * (kConsumerWarps / rpc) * M * sizeof(float);  // [row][slice][m]
    off = (off + 15) & ~size_t(15);
    L.off_best = off;
    off += 64;
    L.smem = off;
    return L;
}

template <int M, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemv_kernel(const GemvArgs a, const int rpc, const int stages, const uint32_t stage_floats,
            const uint32_t off_x, const uint32_t off_stage, const uint32_t off_part,
            const uint32_t off_best) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + 8;
    float *xs = reinterpret_cast<float *>(smem + off_x);
    float *stage = reinterpret_cast<float *>(smem + off_stage);
    float *part = reinterpret_cast<float *>(smem + off_part);
    __shared__ int s_abort;
    __shared__ double s_red[kConsumerWarps][4];
    __shared__ float s_scale[4];

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t K = a.K;
    const int unit = (EPI == GEMV_SWIGLU) ? 2 : 1;
    const int64_t units = a.N / unit;
    const int G = gridDim.x;
    const int64_t u0 = units * blockIdx.x / G, u1 = units * (blockIdx.x + 1) / G;
    const int64_t r0 = u0 * unit, r1 = u1 * unit;
    const int n_chunks = static_cast<int>((r1 - r0 + rpc - 1) / rpc);

    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    grid_launch_dependents();

    if (warp == kConsumerWarps) {
        // ---------------- producer: stream this CTA's rows ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (int c = 0; c < n_chunks; ++c) {
                const int s = c % stages;
                if (c >= stages) {
                    if (!mbar_wait(&empty[s], ((c / stages) - 1) & 1)) {
                        set_status(a.status, B200_DEV_TIMEOUT);
                        s_abort = 1;
                        break;
                    }
                }
                if (*(volatile int *)&s_abort) break;
                const int64_t row = r0 + static_cast<int64_t>(c) * rpc;
                const int rows = static_cast<int>(min64(rpc, r1 - row));
                const uint32_t bytes = static_cast<uint32_t>(rows * K * 4);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(stage + static_cast<size_t>(s) * stage_floats, a.w + row * K, bytes,
                         &full[s], pol);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    grid_wait();  // activations (x / residual / ids) come from the previous kernel
    const int64_t x_ld = a.x_ld ? a.x_ld : K;
    {
        // Gather / load x into shared memory, optionally RMS-normalised.
        double ss[M];
#pragma unroll
        for (int m = 0; m < M; ++m) ss[m] = 0.0;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float *src = a.x + m * x_ld;
            bool zero = false;
            if (a.embed_table) {
                const int32_t id = a.embed_ids[m];
                if (id < 0 || id >= a.embed_rows) {
                    if (tid == 0) set_status(a.status, B200_DEV_BAD_TOKEN);
                    zero = true;
                    src = a.embed_table;
                } else {
                    src = a.embed_table + static_cast<int64_t>(id) * K;
                }
            }
            for (int64_t k = tid; k < K; k += kConsumers) {
                const float v = zero ? 0.f : src[k];
                xs[m * K + k] = v;
                if (a.x_store && blockIdx.x == 0) a.x_store[m * K + k] = v;
                const float sq = v * v;
                ss[m] += static_cast<double>(sq);
            }
        }
        if (a.gamma) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const double w = warp_sum(ss[m]);
                if (lane == 0) s_red[warp][m] = w;
            }
            named_sync(1, kConsumers);
            if (tid < M) {
                double t = 0.0;
                for (int w = 0; w < kConsumerWarps; ++w) t += s_red[w][tid];
                s_scale[tid] = rms_scale_from_sumsq(t, K, a.eps);
            }
            named_sync(1, kConsumers);
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float sc = s_scale[m];
                for (int64_t k = tid; k < K; k += kConsumers) xs[m * K + k] = xs[m * K + k] * sc * a.gamma[k];
            }
        }
        named_sync(1, kConsumers);
    }

    const int ks = kConsumerWarps / rpc;  // K-slices per row
    const int64_t K4 = K >> 2;
    const int64_t L4 = (K4 + ks - 1) / ks;
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
    const int item_r = warp % rpc, item_sl = warp / rpc;  // this warp's (row, K-slice) in every stage

    // Main loop: warps are coupled only through the stage mbarriers. Each warp
    // reduces its (row, K-slice) dot product with shuffles and parks it in
    // part[local_row][slice][m]; the slices are combined once, after the loop.
    for (int c = 0; c < n_chunks; ++c) {
        const int s = c % stages;
        if (!mbar_wait(&full[s], (c / stages) & 1)) {  // bounded: never a hang
            set_status(a.status, B200_DEV_TIMEOUT);
            s_abort = 1;
            break;
        }
        const int64_t row0 = r0 + static_cast<int64_t>(c) * rpc;
        const int rows = static_cast<int>(min64(rpc, r1 - row0));
        const float4 *st4 = reinterpret_cast<const float4 *>(stage + static_cast<size_t>(s) * stage_floats);
        if (item_r < rows) {
            float acc[M];
#pragma unroll
            for (int m = 0; m < M; ++m) acc[m] = 0.f;
            const int64_t beg = item_sl * L4, end = min64(K4, beg + L4);
            const float4 *wr = st4 + item_r * K4;
#pragma unroll 4
            for (int64_t i = beg + lane; i < end; i += 32) {
                const float4 wv = wr[i];
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const float4 xv = xs4[m * K4 + i];
                    acc[m] = fmaf(wv.x, xv.x, acc[m]);
                    acc[m] = fmaf(wv.y, xv.y, acc[m]);
                    acc[m] = fmaf(wv.z, xv.z, acc[m]);
                    acc[m] = fmaf(wv.w, xv.w, acc[m]);
                }
            }
            const int64_t lr = row0 - r0 + item_r;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float v = warp_sum(acc[m]);
                if (lane == 0) part[(lr * ks + item_sl) * M + m] = v;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    named_sync(1, kConsumers);  // every partial is in shared memory
    const bool aborted = *(volatile int *)&s_abort != 0;
    const int rows_cta = static_cast<int>(r1 - r0);

    // Combine the K-slices of every (row, token) in slice order, then the epilogue.
    if (EPI == GEMV_SWIGLU) {
        const int64_t o_ld = a.out_ld ? a.out_ld : a.N / 2;
        for (int t = tid; t < (rows_cta / 2) * M && !aborted; t += kConsumers) {
            const int p = t / M, m = t % M;
            float g = 0.f, u = 0.f;
            for (int sl = 0; sl < ks; ++sl) {
                g += part[((2 * p) * ks + sl) * M + m];
                u += part[((2 * p + 1) * ks + sl) * M + m];
            }
            const float sg = g / (1.0f + expf(-g));
            a.out[m * o_ld + (r0 / 2 + p)] = u * sg;
        }
    } else if (EPI == GEMV_ARGMAX) {
        // M == 1. Per thread: rows tid, tid+256, ... (increasing), strict '>' keeps
        // the first maximum; then a block reduction that prefers the lower row on ties.
        float bv = -INFINITY;
        int64_t bi = INT64_MAX;
        bool bad = aborted;
        for (int r = tid; r < rows_cta && !aborted; r += kConsumers) {
            float v = 0.f;
            for (int sl = 0; sl < ks; ++sl) v += part[r * ks + sl];
            if (a.out) a.out[r0 + r] = v;
            if (isnan(v) || v == INFINITY) bad = true;
            if (v > bv) {
                bv = v;
                bi = r0 + r;
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
        __shared__ float s_bv[kConsumerWarps];
        __shared__ int64_t s_bi[kConsumerWarps];
        __shared__ int s_bad[kConsumerWarps];
        __shared__ unsigned s_ticket;
        if (lane == 0) {
            s_bv[warp] = bv;
            s_bi[warp] = bi;
            s_bad[warp] = bad;
        }
        named_sync(1, kConsumers);
        if (tid == 0) {
            float v = s_bv[0];
            int64_t i = s_bi[0];
            bool anyb = s_bad[0];
            for (int w = 1; w < kConsumerWarps; ++w) {
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
        named_sync(1, kConsumers);
        if (s_ticket == static_cast<unsigned>(G - 1) && tid == 0) {
            __threadfence();
            float gv = -INFINITY;
            int32_t gi = -1;
            bool any_bad = false;
            for (int b = 0; b < G; ++b) {  // CTAs own increasing row ranges
                const float v = __ldcg(a.part_val + b);
                const int32_t i = __ldcg(a.part_idx + b);
                if (i == -2) any_bad = true;
                if (v > gv) {
                    gv = v;
                    gi = i;
                }
            }
            if (any_bad || gi < 0) {
                gi = -1;
                set_status(a.status, B200_DEV_BAD_LOGITS);
            } else {
                gi = static_cast<int32_t>(gi + a.idx_offset);
            }
            *a.argmax_out = gi;
            if (a.best_val_out) *a.best_val_out = any_bad ? NAN : gv;
            if (a.token_log) {
                const int32_t p = *a.log_pos;
                a.token_log[p % a.log_cap] = gi;
                *a.log_pos = p + 1;
            }
            if (a.n_past) *a.n_past += a.n_past_add;
            *a.counter = 0u;
        }
    } else {
        const int64_t o_ld = a.out_ld ? a.out_ld : a.N;
        for (int t = tid; t < rows_cta * M && !aborted; t += kConsumers) {
            const int r = t / M, m = t % M;
            float v = 0.f;
            for (int sl = 0; sl < ks; ++sl) v += part[(r * ks + sl) * M + m];
            const int64_t idx = m * o_ld + r0 + r;
            if (EPI == GEMV_RESIDUAL) v = v + a.residual[idx];
            a.out[idx] = v;
        }
    }
}

template <int M, int EPI>
cudaError_t launch_typed(const GemvArgs &a, const Layout &L, int grid, cudaStream_t stream, bool pdl) {
    auto kern = gemv_kernel<M, EPI>;
    {
        const cudaError_t e = once_per_device(reinterpret_cast<const void *>(kern), ATTR_SMEM, [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        });
        if (e != cudaSuccess) return e;
    }
    return b200_launch(kern, dim3(grid), dim3(kThreads), L.smem, stream, pdl, a, L.rpc, L.stages,
                       L.stage_floats, static_cast<uint32_t>(L.off_x),
                       static_cast<uint32_t>(L.off_stage), static_cast<uint32_t>(L.off_part),
                       static_cast<uint32_t>(L.off_best));
}

template <int M>
cudaError_t launch_m(const GemvArgs &a, const Layout &L, int grid, cudaStream_t stream, bool pdl) {
    switch (a.epi) {
        case GEMV_STORE: return launch_typed<M, GEMV_STORE>(a, L, grid, stream, pdl);
        case GEMV_RESIDUAL: return launch_typed<M, GEMV_RESIDUAL>(a, L, grid, stream, pdl);
        case GEMV_SWIGLU: return launch_typed<M, GEMV_SWIGLU>(a, L, grid, stream, pdl);
        case GEMV_ARGMAX: return launch_typed<1, GEMV_ARGMAX>(a, L, grid, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

int device_sm_count() {
    // per device (grids are sized from the SM count of the device they run on)
    constexpr int kMaxDev = 64;
    static int sms[kMaxDev] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
        cudaGetLastError();
        return 148;
    }
    if (!sms[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
        sms[dev] = n;
    }
    return sms[dev];
}

int gemv_grid_size(int64_t N, int epi) {
    const int64_t units = (epi == GEMV_SWIGLU) ? N / 2 : N;
    return static_cast<int>(b200::min64(units, device_sm_count()));
}

int gemv_use_ring() {
    static int v = -1;
    if (v < 0) {
        const char *e = std::getenv("B200_GEMV_IMPL");
        v = (e && e[0] == 'r') ? 1 : 0;
    }
    return v;
}

int gemv_argmax_slots(int64_t N, int64_t K) {
    return std::max(gemv_grid_size(N, GEMV_ARGMAX), gemv_direct_grid(N, K));
}

cudaError_t gemv_launch(const GemvArgs &a, cudaStream_t stream, bool pdl) {
    if (!gemv_use_ring() && (a.N & 1) == 0) {
        const cudaError_t e = gemv_direct_launch(a, stream, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    return gemv_ring_launch(a, stream, pdl);
}

cudaError_t gemv_ring_launch(const GemvArgs &a, cudaStream_t stream, bool pdl) {
    if (a.M < 1 || a.M > 4 || (a.K & 3) || a.K <= 0 || a.N <= 0) return cudaErrorInvalidValue;
    if (a.epi == GEMV_ARGMAX && a.M != 1) return cudaErrorInvalidValue;
    if (a.epi == GEMV_SWIGLU && (a.N & 1)) return cudaErrorInvalidValue;
    const int grid = gemv_grid_size(a.N, a.epi);
    const int unit = (a.epi == GEMV_SWIGLU) ? 2 : 1;
    const int64_t rows_cta = ((a.N / unit + grid - 1) / grid) * unit;
    const Layout L = make_layout(a.K, a.M, a.epi, rows_cta);
    if (L.smem > 200 * 1024) return cudaErrorInvalidValue;
    switch (a.M) {
        case 1: return launch_m<1>(a, L, grid, stream, pdl);
        case 2: return launch_m<2>(a, L, grid, stream, pdl);
        case 3: return launch_m<3>(a, L, grid, stream, pdl);
        case 4: return launch_m<4>(a, L, grid, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace b200
