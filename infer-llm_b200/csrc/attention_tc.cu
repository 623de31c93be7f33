// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05,
// kind::tf32) for B200_PREC_TF32, head_dim 128: the flash-attention schedule with
// the score tile S and the output O accumulated in tensor memory.
//
// A CTA owns 128 query rows (M of both products): the 128 / G tokens q0.. of one
// KV head times its G query heads, row r = token (r / G), head (r % G), so the G
// heads that share K / V also share every tile. Per 64-key tile t:
//   S  = Q . K_t^T         (M 128, N 64, K 128; A = Q and B = K_t K-major in
//                           shared memory, D = one of two 64-column S buffers)
//   P  = exp2(S * scale * log2 e - m), written over S in tensor memory
//   O += P . V_t           (M 128, N 128, K 64; A = P from tensor memory, B = V_t
//                           MN-major in shared memory, D = 128 O columns)
// Warp roles:
//   * warp 0, one lane: TMA engine. Q once (four 3-D boxes {32 dims, G heads,
//     128/G tokens}, 128-byte swizzle), then K_t and V_t (four boxes {32 dims, 1
//     head, 64 keys} each; K with the 128-byte swizzle, V with 32-byte chunks
//     swizzled in its 128-byte rows, the MN-major TF32 layout) into two-stage rings
//     with their own full / empty barriers;
//   * warp 1, one lane: tensor cores. S_{t+1} is issued before P_t V_t, so the
//     scores of the next tile are computed while the softmax warps work on this one;
//   * warps 2..5: softmax. Thread = one row (tensor-memory lane); row max in log2
//     units; O (and the row sum) is rescaled only when the row max grows by more than
//     2^8 (the running max otherwise stays, which leaves the result unchanged and
//     bounds every p by 2^8), so the correction pass over the O columns is rare.
//     P is rounded to the nearest TF32 value and the row sum is taken over the
//     rounded P, so the weights of the V rows sum to one without truncation bias.
//     The same warps read O at the end, divide by the row sum and store the rows.
//   * warps 6..7: converters. Q, then each K and V stage as it lands, rounded to the
//     nearest TF32 value in shared memory (the tensor cores would truncate, a bias
//     that compounds over the layers), released to the tensor cores by their own
//     ready barriers.
// Keys past the sequence in the last tile: their scores are masked and their V rows
// zeroed in shared memory (the cache may hold anything there; 0 x NaN is NaN).
// Numerics: TF32 products of operands rounded to nearest (P as well, by the softmax
// warps), F32 accumulation; on N(0, 1) inputs the output moves from exact attention
// by ~1e-3 of V's RMS, without the truncation bias.
//
// Every mbarrier wait is bounded (tcgen05.cuh): a wait that runs out records
// B200_DEV_TIMEOUT in the status word; the CTA then waits (bounded) for its copies
// and tensor-core work in flight and frees its tensor memory before returning.
#include "attention.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace b200 {
namespace {

constexpr int kTcRows = 128;  // query rows per CTA: M of both products
constexpr int kTcKeys = 64;   // keys per tile
constexpr int kTcD = 128;
constexpr uint32_t kQBox = kTcRows * 32 * 4;   // 16 KB: 128 rows x 32 dims
constexpr uint32_t kQBytes = 4 * kQBox;        // 64 KB
constexpr uint32_t kKvBox = kTcKeys * 32 * 4;  // 8 KB: 64 keys x 32 dims
constexpr uint32_t kKvTile = 4 * kKvBox;       // 32 KB
constexpr uint32_t kOffK = kQBytes;                 // K ring: 2 stages
constexpr uint32_t kOffV = kOffK + 2 * kKvTile;     // V ring: 2 stages
constexpr uint32_t kOffBar = kOffV + 2 * kKvTile;   // 192 KB
constexpr size_t kTcSmem = 1024 /* alignment slack */ + kOffBar + 256;
constexpr int kSoftWarps = 4;                       // warps 2..5: TMEM lane quarters 2, 3, 0, 1
constexpr int kCvtWarps = 2;                        // warps 6..7: round Q / K / V to TF32 in place
constexpr int kCvtThreads = 32 * kCvtWarps;
constexpr int kTcThreads = 32 * (2 + kSoftWarps + kCvtWarps);
constexpr uint32_t kTmemCols = 256;  // S / P buffers at columns 0 and 64, O at 128
constexpr uint32_t kColO = 128;
constexpr uint32_t kIdescS = idesc_tf32(kTcRows, kTcKeys, false, false);
constexpr uint32_t kIdescO = idesc_tf32(kTcRows, kTcD, false, true);
constexpr float kRescaleLog2 = 8.0f;

__device__ int32_t g_attn_tc_status;  // status word when the caller passes none

// Nearest TF32 value of an F32 bit pattern (ties away from zero): the tensor cores
// would otherwise truncate, which biases every product toward zero.
B200_DEVICE uint32_t tf32_round(uint32_t u) { return (u + 0x1000u) & 0xFFFFE000u; }

// Rounds n16 16-byte groups at p to TF32 (thread i of `threads` takes every
// threads-th group); groups >= zero_from are cleared instead.
B200_DEVICE void round_tf32_smem(unsigned char *p, int n16, int zero_from, int i, int threads) {
    uint4 *q = reinterpret_cast<uint4 *>(p);
#pragma unroll 4
    for (int j = i; j < n16; j += threads) {
        uint4 v = q[j];
        if (j >= zero_from) {
            v = make_uint4(0u, 0u, 0u, 0u);
        } else {
            v.x = tf32_round(v.x);
            v.y = tf32_round(v.y);
            v.z = tf32_round(v.z);
            v.w = tf32_round(v.w);
        }
        q[j] = v;
    }
}

template <int G>
__global__ void __launch_bounds__(kTcThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv, const AttnArgs a) {
    constexpr int BQ = kTcRows / G;
    extern __shared__ unsigned char tc_raw[];
    const uint32_t raw = smem_addr(tc_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;  // swizzled boxes want 1024-byte alignment
    unsigned char *base = tc_raw + (sbase - raw);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + kOffBar);
    uint64_t *q_full = bars;        // Q landed
    uint64_t *k_full = bars + 1;    // [2] K stage landed
    uint64_t *k_empty = bars + 3;   // [2] K stage read by its S product
    uint64_t *v_full = bars + 5;    // [2]
    uint64_t *v_empty = bars + 7;   // [2]
    uint64_t *s_full = bars + 9;    // [2] S buffer complete (and every earlier product)
    uint64_t *p_full = bars + 11;   // [2] P written over S (and O rescaled), 128 arrivals
    uint64_t *o_done = bars + 13;   // one phase per tile: P_t V_t complete
    uint64_t *o_final = bars + 14;  // the last P V complete
    uint64_t *mma_idle = bars + 15; // no tensor-core work in flight (exit)
    uint64_t *q_ready = bars + 16;  // Q rounded to TF32 (converter warps)
    uint64_t *k_ready = bars + 17;  // [2] K stage rounded
    uint64_t *v_ready = bars + 19;  // [2] V stage rounded (rows past the sequence cleared)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 21);
    int32_t *status = a.status ? a.status : &g_attn_tc_status;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t qb = gridDim.x - 1 - blockIdx.x;  // heaviest blocks first
    const int64_t kvh = blockIdx.y;
    const int64_t q0 = qb * BQ;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 32 * kSoftWarps);
        }
        mbar_init(o_done, 1);
        mbar_init(o_final, 1);
        mbar_init(mma_idle, 1);
        mbar_init(q_ready, kCvtThreads);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_ready[s], kCvtThreads);
            mbar_init(&v_ready[s], kCvtThreads);
        }
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tq)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
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
    grid_wait();  // q, the cache rows and n_past come from earlier kernels
    const int64_t n_past = a.n_past_dev ? static_cast<int64_t>(*a.n_past_dev) : a.n_past;
    const int64_t Tkv = n_past + a.Tq;
    const int64_t kv_end = min64(Tkv, n_past + min64(q0 + BQ, a.Tq));
    const int ntiles = static_cast<int>((kv_end + kTcKeys - 1) / kTcKeys);

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA engine
            const uint64_t pol = policy_evict_last();  // K / V tiles are re-read by the other query blocks
            mbar_arrive_expect_tx(q_full, kQBytes);
#pragma unroll
            for (int b = 0; b < 4; ++b)
                tma_load_3d(sbase + b * kQBox, &tq, 32 * b, static_cast<int32_t>(kvh * G), static_cast<int32_t>(q0),
                            smem_addr(q_full), pol);
            int nk = 0, nv = 0;
#pragma unroll 1
            for (int t = 0; t < ntiles; ++t) {
                const int st = t & 1;
                const int32_t z = t * kTcKeys, y = static_cast<int32_t>(kvh);
                if (t >= 2 && !wait_bounded(&k_empty[st], ((t >> 1) - 1) & 1, status)) break;
                mbar_arrive_expect_tx(&k_full[st], kKvTile);
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    tma_load_3d(sbase + kOffK + st * kKvTile + b * kKvBox, &tk, 32 * b, y, z, smem_addr(&k_full[st]),
                                pol);
                nk = t + 1;
                if (t >= 2 && !wait_bounded(&v_empty[st], ((t >> 1) - 1) & 1, status)) break;
                mbar_arrive_expect_tx(&v_full[st], kKvTile);
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    tma_load_3d(sbase + kOffV + st * kKvTile + b * kKvBox, &tv, 32 * b, y, z, smem_addr(&v_full[st]),
                                pol);
                nv = t + 1;
            }
            // copies still landing in this CTA's shared memory (bounded; no-ops when
            // every tile was consumed)
            wait_bounded(q_full, 0, nullptr);
#pragma unroll 1
            for (int t = nk > 2 ? nk - 2 : 0; t < nk; ++t) wait_bounded(&k_full[t & 1], (t >> 1) & 1, nullptr);
#pragma unroll 1
            for (int t = nv > 2 ? nv - 2 : 0; t < nv; ++t) wait_bounded(&v_full[t & 1], (t >> 1) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- tensor cores
            auto issue_s = [&](int t) {  // S_t = Q . K_t^T into buffer t % 2
                const int st = t & 1;
                if (!wait_bounded(&k_ready[st], (t >> 1) & 1, status)) return false;
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(st * kTcKeys);
#pragma unroll
                for (int kk = 0; kk < kTcD / 8; ++kk) {  // K 8 per MMA: +32 bytes inside a 128-byte row
                    const uint64_t da = desc_k_sw128(sbase + (kk >> 2) * kQBox) + 2 * (kk & 3);
                    const uint64_t db = desc_k_sw128(sbase + kOffK + st * kKvTile + (kk >> 2) * kKvBox) + 2 * (kk & 3);
                    tc_mma_tf32(d, da, db, kIdescS, kk > 0 ? 1u : 0u);
                }
                tc_commit(smem_addr(&s_full[st]));
                tc_commit(smem_addr(&k_empty[st]));
                return true;
            };
            bool ok = wait_bounded(q_ready, 0, status) && ntiles > 0 && issue_s(0);
#pragma unroll 1
            for (int t = 0; t < ntiles && ok; ++t) {
                const int st = t & 1;
                if (t + 1 < ntiles && !issue_s(t + 1)) break;
                if (!wait_bounded(&p_full[st], (t >> 1) & 1, status) ||
                    !wait_bounded(&v_ready[st], (t >> 1) & 1, status))
                    break;
                tc_fence_after();
                const uint32_t pa = tmem + static_cast<uint32_t>(st * kTcKeys);
#pragma unroll
                for (int kk = 0; kk < kTcKeys / 8; ++kk) {  // K 8 keys per MMA: one 1024-byte atom of V
                    const uint64_t db = desc_mn_sw128_b32(sbase + kOffV + st * kKvTile + kk * 1024, kKvBox);
                    tc_mma_tf32_ts(tmem + kColO, pa + 8 * kk, db, kIdescO, (t > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(smem_addr(&v_empty[st]));
                tc_commit(smem_addr(o_done));
                if (t + 1 == ntiles) tc_commit(smem_addr(o_final));
            }
            // no product may still use tensor memory or the rings when the CTA exits
            tc_commit(smem_addr(mma_idle));
            wait_bounded(mma_idle, 0, nullptr);
        }
    } else if (warp >= 2 + kSoftWarps) {
        // ---- converters: Q once, then every K / V stage as it lands, rounded to TF32
        // in place; V rows past the sequence (last tile) cleared: the cache may hold
        // anything there, and a zero P does not cancel a NaN
        const int ci = threadIdx.x - 32 * (2 + kSoftWarps);
        bool ok = __all_sync(0xffffffffu, wait_bounded(q_full, 0, status));
        if (ok) {
            round_tf32_smem(base, kQBytes / 16, kQBytes / 16, ci, kCvtThreads);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
            mbar_arrive(q_ready);
        }
#pragma unroll 1
        for (int t = 0; t < ntiles && ok; ++t) {
            const int st = t & 1;
            const int64_t k0 = static_cast<int64_t>(t) * kTcKeys;
            if (!__all_sync(0xffffffffu, wait_bounded(&k_full[st], (t >> 1) & 1, status))) break;
            round_tf32_smem(base + kOffK + st * kKvTile, kKvTile / 16, kKvTile / 16, ci, kCvtThreads);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&k_ready[st]);
            if (!__all_sync(0xffffffffu, wait_bounded(&v_full[st], (t >> 1) & 1, status))) break;
            const int nk = static_cast<int>(min64(kTcKeys, Tkv - k0));  // valid rows of this tile
#pragma unroll 1
            for (int b = 0; b < 4; ++b)  // per 32-dim box: rows of 128 bytes = 8 groups
                round_tf32_smem(base + kOffV + st * kKvTile + b * kKvBox, kKvBox / 16, nk * 8, ci, kCvtThreads);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&v_ready[st]);
        }
    } else {
        // ---- softmax: thread (warp w, lane l) owns row 32 (w % 4) + l = TMEM lane
        const int r = 32 * (warp & 3) + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        const int64_t tok = q0 + r / G;
        const int64_t qpos = n_past + tok;
        const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf(static_cast<float>(kTcD));
        const float sl2 = scale * 1.4426950408889634f;  // log2(e)
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
#pragma unroll 1
        for (int t = 0; t < ntiles; ++t) {
            const int st = t & 1;
            if (!__all_sync(0xffffffffu, wait_bounded(&s_full[st], (t >> 1) & 1, status))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t s0[32], s1[32];
            tc_ld32_nowait(trow + st * kTcKeys, s0);
            tc_ld32_nowait(trow + st * kTcKeys + 32, s1);
            tc_wait_ld();
            tc_reg_fence(s0);
            tc_reg_fence(s1);
            const int64_t k0 = static_cast<int64_t>(t) * kTcKeys;
            const bool all_vis = k0 + kTcKeys - 1 <= qpos && k0 + kTcKeys <= Tkv;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const bool v0 = all_vis || (k0 + c <= qpos && k0 + c < Tkv);
                const bool v1 = all_vis || (k0 + 32 + c <= qpos && k0 + 32 + c < Tkv);
                const float x0 = v0 ? __uint_as_float(s0[c]) * sl2 : -INFINITY;
                const float x1 = v1 ? __uint_as_float(s1[c]) * sl2 : -INFINITY;
                s0[c] = __float_as_uint(x0);
                s1[c] = __float_as_uint(x1);
                mx = fmaxf(mx, fmaxf(x0, x1));
            }
            float alpha = 1.f;
            bool rescale = false;
            if (t == 0) {
                m_run = mx;  // key 0 is visible to every row: finite
            } else if (mx > m_run + kRescaleLog2) {
                alpha = exp2f(m_run - mx);
                m_run = mx;
                rescale = true;
            }
            // P rounded to the nearest TF32 value here (the tensor cores would truncate
            // it), and the row sum taken over the same rounded values: the weights of
            // the V rows then sum to one exactly, with no downward bias
            float rs = 0.f;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const uint32_t p0 = (__float_as_uint(exp2f(__uint_as_float(s0[c]) - m_run)) + 0x1000u) & 0xFFFFE000u;
                const uint32_t p1 = (__float_as_uint(exp2f(__uint_as_float(s1[c]) - m_run)) + 0x1000u) & 0xFFFFE000u;
                rs += __uint_as_float(p0) + __uint_as_float(p1);
                s0[c] = p0;
                s1[c] = p1;
            }
            l_run = l_run * alpha + rs;
            if (__any_sync(0xffffffffu, rescale)) {
                // O holds tiles < t once P_{t-1} V_{t-1} is done (the products before
                // it completed ahead of s_full[t]); P_t V_t waits for this thread's P.
                if (!__all_sync(0xffffffffu, wait_bounded(o_done, (t - 1) & 1, status))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int cb = 0; cb < kTcD / 32; ++cb) {
                    uint32_t o[32];
                    tc_ld32_nowait(trow + kColO + 32 * cb, o);
                    tc_wait_ld();
                    tc_reg_fence(o);
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    tc_st32(trow + kColO + 32 * cb, o);
                }
            }
            tc_st32(trow + st * kTcKeys, s0);
            tc_st32(trow + st * kTcKeys + 32, s1);
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[st]);
        }
        if (ok && __all_sync(0xffffffffu, wait_bounded(o_final, 0, status))) {
            tc_fence_after();
            const float inv = 1.0f / l_run;
            float *dst = a.out + (tok * a.Hq + kvh * G + (r % G)) * kTcD;
#pragma unroll 1
            for (int cb = 0; cb < kTcD / 32; ++cb) {
                uint32_t o[32];
                tc_ld32_nowait(trow + kColO + 32 * cb, o);
                tc_wait_ld();
                tc_reg_fence(o);
                if (tok < a.Tq) {
#pragma unroll
                    for (int c = 0; c < 32; c += 4)
                        *reinterpret_cast<float4 *>(dst + 32 * cb + c) =
                            make_float4(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv,
                                        __uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// q [Tq][Hq][128] as a 3-D tensor {128, Hq, Tq}, boxes {32 dims, G heads, 128/G tokens}
bool q_map(CUtensorMap *m, const float *q, int64_t Hq, int64_t Tq, int G) {
    const uint64_t dims[3] = {static_cast<uint64_t>(kTcD), static_cast<uint64_t>(Hq), static_cast<uint64_t>(Tq)};
    const uint64_t strides[2] = {static_cast<uint64_t>(kTcD) * 4, static_cast<uint64_t>(Hq) * kTcD * 4};
    const uint32_t box[3] = {32, static_cast<uint32_t>(G), static_cast<uint32_t>(kTcRows / G)};
    return tma_encode_f32(m, q, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// K or V as {128, Hkv, rows} with boxes {32 dims, 1 head, 64 positions}: K with the
// 128-byte swizzle (K-major B operand of S), V with 32-byte chunks swizzled in the
// 128-byte rows (the MN-major B operand layout of O += P V)
bool kv_map(CUtensorMap *m, const float *base, int64_t Hkv, int64_t rows, int64_t head, int64_t tok,
            CUtensorMapSwizzle swizzle) {
    const uint64_t dims[3] = {static_cast<uint64_t>(kTcD), static_cast<uint64_t>(Hkv), static_cast<uint64_t>(rows)};
    const uint64_t strides[2] = {static_cast<uint64_t>(head) * 4, static_cast<uint64_t>(tok) * 4};
    const uint32_t box[3] = {32, 1, static_cast<uint32_t>(kTcKeys)};
    return tma_encode_f32(m, base, 3, dims, strides, box, swizzle);
}

template <int G>
cudaError_t tc_launch(const AttnArgs &a, cudaStream_t stream, bool pdl) {
    auto kern = attn_prefill_tc_kernel<G>;
    {
        const cudaError_t e = once_per_device(reinterpret_cast<const void *>(kern), ATTR_SMEM, [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTcSmem));
        });
        if (e != cudaSuccess) return e;
    }
    // positions the K / V maps cover: the sequence (host n_past), else the cache's capacity
    const int64_t rows = a.n_past_dev ? a.kv_rows : a.n_past + a.Tq;
    if (rows <= 0 || rows >= (int64_t(1) << 31) || a.Tq >= (int64_t(1) << 31)) return cudaErrorNotSupported;
    CUtensorMap mq, mk, mv;
    if (!q_map(&mq, a.q, a.Hq, a.Tq, G) ||
        !kv_map(&mk, a.k, a.Hkv, rows, a.k_head, a.k_tok, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !kv_map(&mv, a.v, a.Hkv, rows, a.v_head, a.v_tok, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
        return cudaErrorNotSupported;
    constexpr int BQ = kTcRows / G;
    const dim3 grid(static_cast<unsigned>((a.Tq + BQ - 1) / BQ), static_cast<unsigned>(a.Hkv));
    return b200_launch(kern, grid, dim3(kTcThreads), kTcSmem, stream, pdl, mq, mk, mv, a);
}

}  // namespace

cudaError_t attn_prefill_tc_launch(const AttnArgs &a, cudaStream_t stream, bool pdl) {
    if (a.D != kTcD || a.Hkv <= 0 || a.Hq % a.Hkv || a.Tq < 1) return cudaErrorNotSupported;
    // out rows are written as 16-byte vectors
    if (reinterpret_cast<uintptr_t>(a.out) & 15) return cudaErrorNotSupported;
    switch (a.Hq / a.Hkv) {
        case 1: return tc_launch<1>(a, stream, pdl);
        case 2: return tc_launch<2>(a, stream, pdl);
        case 4: return tc_launch<4>(a, stream, pdl);
        case 8: return tc_launch<8>(a, stream, pdl);
    }
    return cudaErrorNotSupported;
}

}  // namespace b200
