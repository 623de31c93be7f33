// Exact F32 (FFMA) tiled GEMM for prefill: C[M][N] = X[M][K] . W[N][K]^T.
//
// 256 threads, tile BM x 128 x 16, each thread owns a (BM/16) x 8 block of C
// split into two column quads 64 apart so shared-memory reads are conflict free.
// Global tiles are read with 128-bit loads into registers one K-step ahead and
// stored transposed into a double-buffered shared tile. Epilogues fuse the
// residual add and SwiGLU of the reference graph (Qwen3.cpp:97,109-118).
#include <algorithm>

#include "gemm.cuh"
#include "gemv.cuh"

namespace b200 {
namespace {

constexpr int BN = 128, BK = 16, PAD = 4, NT = 256;

// Two CTAs per SM (at most 128 registers a thread): 16 warps to hide the shared-memory
// and FFMA latencies, and the split-K grid below is sized for two CTAs per SM.
template <int BM, int EPI>
__global__ void __launch_bounds__(NT, 2) sgemm_kernel(const GemmArgs a) {
    constexpr int TM = BM / 16;              // rows per thread
    constexpr int A_LD = (BM * BK / 4) / NT; // float4 loads of X per thread (BM=32 -> 0.5)
    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];

    grid_launch_dependents();
    grid_wait();

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    const int64_t K = a.K;  // row stride of W and X's K extent
    // split-K: this CTA's K range [kbeg, kend)
    const int64_t kbeg = a.k_split ? static_cast<int64_t>(blockIdx.z) * a.k_split : 0;
    const int64_t kend = a.k_split ? min64(K, kbeg + a.k_split) : K;

    // X tile: BM rows x 4 float4; W tile: 128 rows x 4 float4 (2 per thread)
    float4 ra[A_LD > 0 ? A_LD : 1], rb[2];
    auto load_tiles = [&](int64_t k0) {
        if (A_LD > 0) {
#pragma unroll
            for (int i = 0; i < A_LD; ++i) {
                const int f = tid + i * NT;
                const int row = f >> 2, k4 = f & 3;
                const int64_t gm = m0 + row, gk = k0 + k4 * 4;
                ra[i] = (gm < a.M && gk < kend) ? *reinterpret_cast<const float4 *>(a.x + gm * a.ldx + gk)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        } else if (tid < BM * 4) {
            const int row = tid >> 2, k4 = tid & 3;
            const int64_t gm = m0 + row, gk = k0 + k4 * 4;
            ra[0] = (gm < a.M && gk < kend) ? *reinterpret_cast<const float4 *>(a.x + gm * a.ldx + gk)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int f = tid + i * NT;
            const int row = f >> 2, k4 = f & 3;
            const int64_t gn = n0 + row, gk = k0 + k4 * 4;
            rb[i] = (gn < a.N && gk < kend) ? ld_stream4(reinterpret_cast<const float4 *>(a.w + gn * K + gk))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_tiles = [&](int buf) {
        if (A_LD > 0) {
#pragma unroll
            for (int i = 0; i < A_LD; ++i) {
                const int f = tid + i * NT;
                const int row = f >> 2, k4 = f & 3;
                As[buf][k4 * 4 + 0][row] = ra[i].x;
                As[buf][k4 * 4 + 1][row] = ra[i].y;
                As[buf][k4 * 4 + 2][row] = ra[i].z;
                As[buf][k4 * 4 + 3][row] = ra[i].w;
            }
        } else if (tid < BM * 4) {
            const int row = tid >> 2, k4 = tid & 3;
            As[buf][k4 * 4 + 0][row] = ra[0].x;
            As[buf][k4 * 4 + 1][row] = ra[0].y;
            As[buf][k4 * 4 + 2][row] = ra[0].z;
            As[buf][k4 * 4 + 3][row] = ra[0].w;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int f = tid + i * NT;
            const int row = f >> 2, k4 = f & 3;
            Bs[buf][k4 * 4 + 0][row] = rb[i].x;
            Bs[buf][k4 * 4 + 1][row] = rb[i].y;
            Bs[buf][k4 * 4 + 2][row] = rb[i].z;
            Bs[buf][k4 * 4 + 3][row] = rb[i].w;
        }
    };

    float acc[TM][8];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    // rows owned: TM=8 -> {ty*4..+3} U {BM/2 + ty*4..+3}; TM=4 -> ty*4..+3; TM=2 -> ty*2..+1
    auto row_of = [&](int i) -> int {
        if (TM == 8) return (i < 4) ? ty * 4 + i : BM / 2 + ty * 4 + (i - 4);
        return ty * TM + i;
    };

    const int64_t nk = (kend - kbeg + BK - 1) / BK;
    load_tiles(kbeg);
    store_tiles(0);
    __syncthreads();
    for (int64_t kt = 0; kt < nk; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load_tiles(kbeg + (kt + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float av[TM], bv[8];
            if (TM == 8) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 4]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][k][BM / 2 + ty * 4]);
                av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
                av[4 % TM] = a1.x; av[5 % TM] = a1.y; av[6 % TM] = a1.z; av[7 % TM] = a1.w;
            } else if (TM == 4) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 4]);
                av[0] = a0.x; av[1 % TM] = a0.y; av[2 % TM] = a0.z; av[3 % TM] = a0.w;
            } else {
                const float2 a0 = *reinterpret_cast<const float2 *>(&As[buf][k][ty * 2]);
                av[0] = a0.x; av[1 % TM] = a0.y;
            }
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][k][64 + tx * 4]);
            bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
            bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (kt + 1 < nk) {
            store_tiles(buf ^ 1);
        }
        __syncthreads();
    }

    // epilogue
    if (a.k_split) {  // raw partial sums of this split: ws[z][M][N]
        float *ws = a.ws + static_cast<int64_t>(blockIdx.z) * a.M * a.N;
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int64_t gm = m0 + row_of(i);
            if (gm >= a.M) continue;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t col = n0 + h * 64 + tx * 4 + j;
                    if (col < a.N) ws[gm * a.N + col] = acc[i][h * 4 + j];
                }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int64_t gm = m0 + row_of(i);
        if (gm >= a.M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t gn = n0 + h * 64 + tx * 4;
            if (EPI == GEMM_SWIGLU) {
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    const int64_t col = gn + 2 * p;
                    if (col + 1 < a.N) {
                        const float g = acc[i][h * 4 + 2 * p], u = acc[i][h * 4 + 2 * p + 1];
                        const float sg = g / (1.0f + expf(-g));
                        a.c[gm * a.ldc + col / 2] = u * sg;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t col = gn + j;
                    if (col < a.N) {
                        float v = acc[i][h * 4 + j];
                        if (EPI == GEMM_RESIDUAL) v = v + a.r[gm * a.ldc + col];
                        a.c[gm * a.ldc + col] = v;
                    }
                }
            }
        }
    }
}

// Sums the split partials in split order and applies the epilogue (same
// arithmetic as sgemm_kernel's): one thread per output (per gate/up pair for SwiGLU).
template <int EPI>
__global__ void splitk_reduce_kernel(const GemmArgs a, int splits) {
    grid_launch_dependents();
    grid_wait();
    const int64_t per_row = EPI == GEMM_SWIGLU ? a.N / 2 : a.N;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= a.M * per_row) return;
    const int64_t m = i / per_row, n = i % per_row;
    const int64_t plane = a.M * a.N;
    if (EPI == GEMM_SWIGLU) {
        float g = 0.f, u = 0.f;
        for (int z = 0; z < splits; ++z) {
            g += a.ws[z * plane + m * a.N + 2 * n];
            u += a.ws[z * plane + m * a.N + 2 * n + 1];
        }
        const float sg = g / (1.0f + expf(-g));
        a.c[m * a.ldc + n] = a.round_out ? tf32_rn(u * sg) : u * sg;
    } else {
        float v = 0.f;
        for (int z = 0; z < splits; ++z) v += a.ws[z * plane + m * a.N + n];
        if (EPI == GEMM_RESIDUAL) v = v + a.r[m * a.ldc + n];
        a.c[m * a.ldc + n] = a.round_out ? tf32_rn(v) : v;
    }
}

// K splits for an M x N x K product with BM-row tiles: when the tile grid leaves
// SMs idle (prompts up to a few hundred tokens on the layer shapes), as many splits
// as fit in one wave of two CTAs per SM (a partial second wave would double the
// time), at least 128 of K (8 k-steps) per split.
template <int BM>
int64_t ffma_splits(int64_t M, int64_t N, int64_t K) {
    const int64_t tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM), target = 2 * device_sm_count();
    if (tiles >= target || K < 256) return 1;
    return std::max<int64_t>(1, std::min<int64_t>(target / tiles, K / 128));
}

template <int BM>
cudaError_t launch_bm(const GemmArgs &a_in, cudaStream_t stream, bool pdl) {
    GemmArgs a = a_in;
    dim3 grid(static_cast<unsigned>((a.N + BN - 1) / BN), static_cast<unsigned>((a.M + BM - 1) / BM));
    // split K (partials in a.ws, reduced in split order) when the tiles leave SMs idle
    a.k_split = 0;
    if (a.ws) {
        int64_t splits = ffma_splits<BM>(a.M, a.N, a.K);
        while (splits > 1 && splits * a.M * a.N > a.ws_floats) --splits;
        if (splits > 1) {
            a.k_split = ((a.K + splits - 1) / splits + BK - 1) / BK * BK;
            grid.z = static_cast<unsigned>((a.K + a.k_split - 1) / a.k_split);
        }
    }
    if (a.k_split) {
        cudaError_t e = b200_launch(sgemm_kernel<BM, GEMM_STORE>, grid, dim3(NT), 0, stream, pdl, a);
        if (e != cudaSuccess) return e;
        return gemm_splitk_reduce_launch(a, static_cast<int>(grid.z), stream, pdl);
    }
    switch (a.epi) {
        case GEMM_STORE: return b200_launch(sgemm_kernel<BM, GEMM_STORE>, grid, dim3(NT), 0, stream, pdl, a);
        case GEMM_RESIDUAL: return b200_launch(sgemm_kernel<BM, GEMM_RESIDUAL>, grid, dim3(NT), 0, stream, pdl, a);
        case GEMM_SWIGLU: return b200_launch(sgemm_kernel<BM, GEMM_SWIGLU>, grid, dim3(NT), 0, stream, pdl, a);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t gemm_splitk_reduce_launch(const GemmArgs &a, int splits, cudaStream_t stream, bool pdl) {
    const int64_t outs = a.M * (a.epi == GEMM_SWIGLU ? a.N / 2 : a.N);
    const dim3 rg(static_cast<unsigned>((outs + 255) / 256));
    switch (a.epi) {
        case GEMM_STORE: return b200_launch(splitk_reduce_kernel<GEMM_STORE>, rg, dim3(256), 0, stream, pdl, a, splits);
        case GEMM_RESIDUAL:
            return b200_launch(splitk_reduce_kernel<GEMM_RESIDUAL>, rg, dim3(256), 0, stream, pdl, a, splits);
        case GEMM_SWIGLU: return b200_launch(splitk_reduce_kernel<GEMM_SWIGLU>, rg, dim3(256), 0, stream, pdl, a, splits);
    }
    return cudaErrorInvalidValue;
}

int64_t gemm_ffma_ws_floats(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const int64_t s = M <= 32 ? ffma_splits<32>(M, N, K) : M <= 64 ? ffma_splits<64>(M, N, K) : ffma_splits<128>(M, N, K);
    return s > 1 ? s * M * N : 0;
}

cudaError_t gemm_ffma_launch(const GemmArgs &a, cudaStream_t stream, bool pdl) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0 || (a.K & 3) || (a.ldx & 3)) return cudaErrorInvalidValue;
    if (a.epi == GEMM_SWIGLU && (a.N & 1)) return cudaErrorInvalidValue;
    if (a.M <= 32) return launch_bm<32>(a, stream, pdl);
    if (a.M <= 64) return launch_bm<64>(a, stream, pdl);
    return launch_bm<128>(a, stream, pdl);
}

}  // namespace b200
