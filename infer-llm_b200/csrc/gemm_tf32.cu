// Prefill matrix products on the 5th-generation tensor cores (tcgen05, kind::tf32):
// C[M][N] = X[M][K] . W[N][K]^T with the STORE / RESIDUAL / SWIGLU epilogues of the
// FFMA GEMM (gemm_ffma.cu), for B200_PREC_TF32.
//
// A persistent grid (one CTA per SM) walks the 128 x 256 tiles of C (and the K
// splits, when the tile grid alone leaves SMs idle). Both operands are K-major in
// HBM (X rows are tokens, W rows are output features), the layout tcgen05 reads
// directly:
//   * warp 0, one lane: TMA engine. 2-D tiled copies (cuTensorMapEncodeTiled,
//     128-byte swizzle) of a [128 x 32 floats] box of X and a [256 x 32 floats] box
//     of W per stage into a kTStages-deep shared-memory ring, completing on the
//     stage's mbarrier;
//   * warp 1, one lane: tensor cores. Per stage four tcgen05.mma (M 128, N 256,
//     K 8 each) from shared-memory descriptors into one of two 256-column F32
//     accumulators in tensor memory (the whole 512 columns of the SM);
//     tcgen05.commit hands the stage back to the copy engine once the MMAs that
//     read it are done, and signals the epilogue when a tile is complete;
//   * warps 2..5: epilogue. Warp w reads TMEM lanes 32(w % 4)..+31 (= tile rows)
//     with tcgen05.ld, 16 columns at a time, writes C (or split-K partials) and
//     frees the accumulator, while the tensor cores already fill the other one.
// TF32 multiplies use the top 19 bits of each F32 operand and accumulate in F32,
// so results differ from the exact F32 reference by ~1e-3 relative (the
// B200_PREC_TF32 tolerance); B200_PREC_FFMA is the exact path.
//
// Every mbarrier wait is bounded: a wait that runs out records B200_DEV_TIMEOUT in
// the status word, skips the remaining work, waits (bounded) for this CTA's copies
// in flight and frees its tensor memory before returning.
#include <algorithm>

#include "gemm.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace b200 {
namespace {

constexpr int kTBM = 128, kTBK = 32;  // kTBK floats = one 128-byte swizzle row
constexpr int kEpiWarps = 4;           // warps 2..5: TMEM lane quarters (warp % 4) 2, 3, 0, 1
constexpr int kTThreads = 32 * (2 + kEpiWarps);

// Tile width BN (output features per tile): 256 when the tiles fill the SMs, else 128.
// MB: 128-row halves per tile. MB = 1: 128 x BN tiles, two accumulators so a tile's
// epilogue overlaps the next tile's MMAs. MB = 2 (BN 256): 256 x 256 tiles, the two
// accumulators hold the two row halves of one tile and share every W stage, so each
// MMA needs 1.5x fewer operand bytes from L2 (32 KB per 128 x 256 x 32 product
// instead of 48 KB); chosen where it also leaves fewer rounds of tiles.
template <int BN, int MB = 1>
struct TCfg {
    static_assert(BN == 128 || BN == 256, "cta_group::1 MMA with M 128 takes N % 16 == 0, N <= 256");
    static_assert(MB == 1 || (MB == 2 && BN == 256), "two row halves use the 512 tensor-memory columns");
    static constexpr uint32_t kTileA = MB * kTBM * kTBK * 4;  // X rows per stage (16 KB per half)
    static constexpr uint32_t kTileB = BN * kTBK * 4;         // W rows per stage
    static constexpr uint32_t kStageBytes = kTileA + kTileB;
    static constexpr int kStages = MB == 2 ? 3 : BN == 256 ? 4 : 6;  // 192 KB of ring: one CTA per SM
    static constexpr uint32_t kAccCols = BN;            // one F32 accumulator: 128 lanes x BN columns
    static constexpr uint32_t kTmemCols = 2 * BN;       // two accumulators
    static constexpr size_t kSmem = 1024 /* alignment slack */ + static_cast<size_t>(kStages) * kStageBytes + 256;
    // kind::tf32, both operands K-major
    static constexpr uint32_t kIdesc = idesc_tf32(kTBM, BN, false, false);
};

B200_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x, int32_t y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ int32_t g_tf32_status;  // status word when the caller passes none

// Tile t of the persistent schedule: split z, then row block, then column block
// (consecutive CTAs share a column block of W while X stays in L2).
struct TileIx {
    int64_t m0, n0, kbeg, kend;
};
template <int BN, int MB>
B200_DEVICE TileIx tile_of(const GemmArgs &a, int64_t t, int64_t mt, int64_t nt) {
    const int64_t z = t / (mt * nt), r = t % (mt * nt);
    TileIx ix;
    ix.m0 = (r % mt) * kTBM * MB;
    ix.n0 = (r / mt) * BN;
    ix.kbeg = a.k_split ? z * a.k_split : 0;
    ix.kend = a.k_split ? min64(a.K, ix.kbeg + a.k_split) : a.K;
    return ix;
}

template <int EPI, int BN, int MB>
__global__ void __launch_bounds__(kTThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, const GemmArgs a,
                     int64_t n_tiles) {
    using C = TCfg<BN, MB>;
    constexpr uint32_t kTileA = C::kTileA;
    constexpr int kTStages = C::kStages;
    constexpr uint32_t kStageBytes = C::kStageBytes, kAccCols = C::kAccCols, kTmemCols = C::kTmemCols;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;  // swizzled tiles want 1024-byte alignment
    unsigned char *gbase = smem_raw + (sbase - raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(gbase + kTStages * kStageBytes);
    uint64_t *empty = full + kTStages;
    uint64_t *acc_full = empty + kTStages;  // [2] accumulator b complete (tcgen05.commit)
    uint64_t *acc_free = acc_full + 2;      // [2] accumulator b read out by the epilogue warps
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_free + 2);
    int32_t *status = a.status ? a.status : &g_tf32_status;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t mt = (a.M + kTBM * MB - 1) / (kTBM * MB), nt = (a.N + BN - 1) / BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_free[b], kEpiWarps);
        }
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmx)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmw)) : "memory");
    }
    if (warp == 2) {  // one warp owns the tensor-memory allocation
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    grid_launch_dependents();
    grid_wait();  // X (and the residual) come from the previous kernel

    if (warp == 0) {
        if (lane == 0) {
            // ---- copy engine: ring stage it % kTStages over all k-steps of all tiles
            int it = 0;
            bool ok = true;
#pragma unroll 1
            for (int64_t t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                const TileIx ix = tile_of<BN, MB>(a, t, mt, nt);
#pragma unroll 1
                for (int64_t k = ix.kbeg; k < ix.kend; k += kTBK, ++it) {
                    const int s = it % kTStages;
                    if (it >= kTStages && !wait_bounded(&empty[s], ((it / kTStages) - 1) & 1, status)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = sbase + s * kStageBytes;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tma_load_2d(dst, &tmx, static_cast<int32_t>(k), static_cast<int32_t>(ix.m0), smem_addr(&full[s]));
                    tma_load_2d(dst + kTileA, &tmw, static_cast<int32_t>(k), static_cast<int32_t>(ix.n0),
                                smem_addr(&full[s]));
                }
            }
            // copies still landing in this CTA's shared memory: the last kTStages issued
#pragma unroll 1
            for (int j = it > kTStages ? it - kTStages : 0; j < it; ++j)
                wait_bounded(&full[j % kTStages], (j / kTStages) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- tensor cores: tile j of this CTA accumulates into TMEM columns (j % 2) * kAccCols
            int it = 0, j = 0;
            bool ok = true;
#pragma unroll 1
            for (int64_t t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++j) {
                const TileIx ix = tile_of<BN, MB>(a, t, mt, nt);
                // MB = 1: accumulator b = j % 2, free again once tile j - 2 is read out;
                // MB = 2: both accumulators for tile j, free once tile j - 1 is read out
                const int b = MB == 2 ? 0 : (j & 1);
                if (MB == 1 && j >= 2 && !wait_bounded(&acc_free[b], ((j >> 1) - 1) & 1, status)) break;
                if (MB == 2 && j >= 1 && !wait_bounded(&acc_free[0], (j - 1) & 1, status)) break;
                tc_fence_after();
                const uint32_t acc = tmem + b * kAccCols;
                bool first = true;
#pragma unroll 1
                for (int64_t k = ix.kbeg; k < ix.kend; k += kTBK, ++it) {
                    const int s = it % kTStages;
                    if (!wait_bounded(&full[s], (it / kTStages) & 1, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = desc_k_sw128(sbase + s * kStageBytes);
                    const uint64_t db = desc_k_sw128(sbase + s * kStageBytes + kTileA);
#pragma unroll
                    for (int kk = 0; kk < kTBK / 8; ++kk) {  // K 8 per MMA: +32 bytes = +2 in the address field
#pragma unroll
                        for (int half = 0; half < MB; ++half)  // X rows 128 half.. (16 KB further), accumulator half
                            tc_mma_tf32(acc + half * kAccCols, da + half * (16384 >> 4) + 2 * kk, db + 2 * kk,
                                        C::kIdesc, first ? 0u : 1u);
                        first = false;
                    }
                    tc_commit(smem_addr(&empty[s]));
                }
                tc_commit(smem_addr(&acc_full[b]));  // this tile's accumulator is complete
            }
            // no MMA may still write tensor memory when it is freed (matters only if
            // the epilogue gave up early)
            if (j > 0) {
                if (MB == 2)
                    wait_bounded(&acc_full[0], (j - 1) & 1, nullptr);
                else
                    wait_bounded(&acc_full[(j - 1) & 1], ((j - 1) >> 1) & 1, nullptr);
            }
        }
    } else {
        // ---- epilogue warps: thread (warp w, lane t) owns tile row 32 * (w % 4) + t
        const int q = warp & 3;
        // 16-byte stores where C (and the split-K workspace) rows allow them
        const bool vec_c = !(a.ldc & 3) && !(reinterpret_cast<uintptr_t>(a.c) & 15);
        const bool vec_ws = !(a.N & 3) && !(reinterpret_cast<uintptr_t>(a.ws) & 15);
        int j = 0;
#pragma unroll 1
        for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x, ++j) {
            const TileIx ix = tile_of<BN, MB>(a, t, mt, nt);
            const int b = MB == 2 ? 0 : (j & 1);
            // warp-uniform: tcgen05.ld is a warp-collective (.sync.aligned) instruction
            if (!__all_sync(0xffffffffu, wait_bounded(&acc_full[b], MB == 2 ? (j & 1) : ((j >> 1) & 1), status))) break;
            tc_fence_after();
            const int64_t z = t / (mt * nt);
#pragma unroll 1
            for (int half = 0; half < MB; ++half) {  // row half of the tile: accumulator b + half
            const int64_t gm = ix.m0 + kTBM * half + 32 * q + lane;
            const uint32_t trow = tmem + (b + half) * kAccCols + (static_cast<uint32_t>(32 * q) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float v[16];
                __syncwarp();
                tc_ld16(trow + c0, v);  // every lane takes part
                const int64_t gn = ix.n0 + c0;
                if (gm >= a.M || gn >= a.N) continue;
                const bool whole = gn + 16 <= a.N;
                if (a.k_split) {  // raw partial sums of this split: ws[z][M][N]
                    float *ws = a.ws + z * a.M * a.N + gm * a.N + gn;
                    if (whole && vec_ws) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4 *>(ws + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (gn + i < a.N) ws[i] = v[i];
                    }
                } else if (EPI == GEMM_SWIGLU) {  // (gate, up) column pairs -> one output
                    float h[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float g = v[2 * i], u = v[2 * i + 1];
                        const float sg = g / (1.0f + expf(-g));
                        h[i] = a.round_out ? tf32_rn(u * sg) : u * sg;
                    }
                    float *dst = a.c + gm * a.ldc + gn / 2;
                    if (whole && vec_c) {
                        *reinterpret_cast<float4 *>(dst) = make_float4(h[0], h[1], h[2], h[3]);
                        *reinterpret_cast<float4 *>(dst + 4) = make_float4(h[4], h[5], h[6], h[7]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            if (gn + 2 * i + 1 < a.N) dst[i] = h[i];
                    }
                } else {
                    float *dst = a.c + gm * a.ldc + gn;
                    if (EPI == GEMM_RESIDUAL) {
                        const float *res = a.r + gm * a.ldc + gn;
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (gn + i < a.N) v[i] = v[i] + res[i];
                    }
                    if (a.round_out) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[i] = tf32_rn(v[i]);
                    }
                    if (whole && vec_c) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4 *>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (gn + i < a.N) dst[i] = v[i];
                    }
                }
            }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_free[b]);  // the MMA warp may reuse accumulator b (MB = 2: both)
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// [rows][cols] F32 matrix with row stride `ld` floats, boxes of [box_rows x 32 floats].
bool encode(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld, uint32_t box_rows) {
    const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 4};
    const uint32_t box[2] = {static_cast<uint32_t>(kTBK), box_rows};
    return tma_encode_f32(map, base, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int EPI, int BN, int MB = 1>
cudaError_t launch_epi(const CUtensorMap &mx, const CUtensorMap &mw, const GemmArgs &a, int64_t n_tiles,
                       cudaStream_t st, bool pdl) {
    auto kern = gemm_tf32_kernel<EPI, BN, MB>;
    {
        const cudaError_t e = once_per_device(reinterpret_cast<const void *>(kern), ATTR_SMEM, [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(TCfg<BN, MB>::kSmem));
        });
        if (e != cudaSuccess) return e;
    }
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>(n_tiles, device_sm_count())));
    return b200_launch(kern, grid, dim3(kTThreads), TCfg<BN, MB>::kSmem, st, pdl, mx, mw, a, n_tiles);
}

// 256 x 256 tiles, no K split.
cudaError_t launch_m2(const GemmArgs &a_in, cudaStream_t stream, bool pdl) {
    GemmArgs a = a_in;
    a.k_split = 0;
    CUtensorMap mx, mw;
    if (!encode(&mx, a.x, a.M, a.K, a.ldx, 2 * kTBM) || !encode(&mw, a.w, a.N, a.K, a.K, 256)) return cudaErrorNotSupported;
    const int64_t n_tiles = ((a.N + 255) / 256) * ((a.M + 2 * kTBM - 1) / (2 * kTBM));
    switch (a.epi) {
        case GEMM_STORE: return launch_epi<GEMM_STORE, 256, 2>(mx, mw, a, n_tiles, stream, pdl);
        case GEMM_RESIDUAL: return launch_epi<GEMM_RESIDUAL, 256, 2>(mx, mw, a, n_tiles, stream, pdl);
        case GEMM_SWIGLU: return launch_epi<GEMM_SWIGLU, 256, 2>(mx, mw, a, n_tiles, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

// K splits of the tcgen05 GEMM with BN-wide tiles, when the tile grid alone leaves
// SMs idle: as many as fit in one round of the persistent grid (one tile per SM; a
// partial second round would double the time), at least 256 of K per split.
template <int BN>
int64_t tf32_splits(int64_t M, int64_t N, int64_t K) {
    const int64_t tiles = ((N + BN - 1) / BN) * ((M + kTBM - 1) / kTBM), target = device_sm_count();
    if (tiles >= target || K < 512) return 1;
    return std::max<int64_t>(1, std::min<int64_t>(target / tiles, K / 256));
}

template <int BN>
cudaError_t launch_bn(const GemmArgs &a_in, cudaStream_t stream, bool pdl) {
    GemmArgs a = a_in;
    CUtensorMap mx, mw;
    if (!encode(&mx, a.x, a.M, a.K, a.ldx, kTBM) || !encode(&mw, a.w, a.N, a.K, a.K, BN)) return cudaErrorNotSupported;
    const int64_t tiles = ((a.N + BN - 1) / BN) * ((a.M + kTBM - 1) / kTBM);
    // Split K when the tile grid leaves SMs idle (short prompts): about one tile per
    // SM, at least 256 of K per split, partials reduced in split order.
    a.k_split = 0;
    int64_t splits = 1;
    if (a.ws) {
        splits = tf32_splits<BN>(a.M, a.N, a.K);
        while (splits > 1 && splits * a.M * a.N > a.ws_floats) --splits;
        if (splits > 1) {
            a.k_split = ((a.K + splits - 1) / splits + kTBK - 1) / kTBK * kTBK;
            splits = (a.K + a.k_split - 1) / a.k_split;
        } else {
            splits = 1;
        }
    }
    const int64_t n_tiles = tiles * splits;
    if (a.k_split) {
        const cudaError_t e = launch_epi<GEMM_STORE, BN>(mx, mw, a, n_tiles, stream, pdl);
        if (e != cudaSuccess) return e;
        return gemm_splitk_reduce_launch(a, static_cast<int>(splits), stream, pdl);
    }
    switch (a.epi) {
        case GEMM_STORE: return launch_epi<GEMM_STORE, BN>(mx, mw, a, n_tiles, stream, pdl);
        case GEMM_RESIDUAL: return launch_epi<GEMM_RESIDUAL, BN>(mx, mw, a, n_tiles, stream, pdl);
        case GEMM_SWIGLU: return launch_epi<GEMM_SWIGLU, BN>(mx, mw, a, n_tiles, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

int64_t gemm_tf32_ws_floats(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const int64_t tiles256 = ((N + 255) / 256) * ((M + kTBM - 1) / kTBM);
    const int64_t s = tiles256 >= device_sm_count() ? tf32_splits<256>(M, N, K) : tf32_splits<128>(M, N, K);
    return s > 1 ? s * M * N : 0;
}

cudaError_t gemm_tf32_launch(const GemmArgs &a, cudaStream_t stream, bool pdl) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return cudaErrorInvalidValue;
    if (a.epi == GEMM_SWIGLU && (a.N & 1)) return cudaErrorInvalidValue;
    // TMA: 16-byte aligned bases and row strides; the tile rows must fit 32-bit coordinates
    if ((a.K & 3) || (a.ldx & 3) || (reinterpret_cast<uintptr_t>(a.x) & 15) || (reinterpret_cast<uintptr_t>(a.w) & 15) ||
        a.M >= (int64_t(1) << 31) || a.N >= (int64_t(1) << 31) || a.K >= (int64_t(1) << 31))
        return cudaErrorNotSupported;
    // 256-wide tiles (half the X traffic per flop) once they alone fill the SMs; 256 x 256
    // tiles where they need at most half the rounds of 128 x 256 ones (measured: a
    // 256 x 256 tile takes ~1.9x a 128 x 256 one, so they win only on equal work per
    // SM, by their lower operand traffic: 4096^3 605 -> 699 TFLOP/s, 2048 x 4096 x 1024
    // 399 -> 420; with more rounds, e.g. 2048 x 6144 x 1024, they lose)
    const int64_t sms = device_sm_count();
    const int64_t tiles256 = ((a.N + 255) / 256) * ((a.M + kTBM - 1) / kTBM);
    const int64_t tiles2 = ((a.N + 255) / 256) * ((a.M + 2 * kTBM - 1) / (2 * kTBM));
    if (a.M > kTBM && 2 * tiles2 >= sms && 2 * ((tiles2 + sms - 1) / sms) <= (tiles256 + sms - 1) / sms) {
        const cudaError_t e = launch_m2(a, stream, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    return tiles256 >= sms ? launch_bn<256>(a, stream, pdl) : launch_bn<128>(a, stream, pdl);
}

}  // namespace b200
