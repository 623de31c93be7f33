// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05,
// kind::tf32) for B200_PREC_TF32, head_dim 128: the flash-attention schedule with
// the score tile S and the output O accumulated in tensor memory.
//
// A CTA owns 128 query rows (M of both products): the 128 / G tokens q0.. of one
// KV head times its G query heads, row r = token (r / G), head (r % G), so the G
// heads that share K / V also share every tile. Per 64-key tile t:
//   S  = Q . K_t^T         (M 128, N 64, K 128; A = Q from tensor memory, B = K_t
//                           K-major in shared memory, D = one of two S buffers)
//   P  = exp2(S * scale * log2 e - m), written over S in tensor memory
//   O += P . V_t           (M 128, N 128, K 64; A = P from tensor memory, B = V_t
//                           MN-major in shared memory, D = 128 O columns)
// Tensor memory (512 columns): S / P buffers at 0 and 64, O at 128, Q at 256.
// Warp roles:
//   * warp 0 and warp 14, one lane each: TMA engine for K and for V. K_t and V_t
//     (four boxes {32 dims, 1 head, 64 keys} each; K with the 128-byte swizzle, V
//     with 32-byte chunks swizzled in its 128-byte rows, the MN-major TF32 layout)
//     go into three-stage rings with their own full / empty barriers, so neither
//     ring waits for the other;
//   * warp 1, one lane: tensor cores. S_{t+1} is issued before P_t V_t, so the
//     scores of the next tile are computed while the softmax warps work on this one;
//   * warps 2..9: softmax. Each row (tensor-memory lane) is owned by two threads,
//     one per half of the columns: warp w takes lane quarter w % 4 and column half
//     (w - 2) / 4. First each thread loads its half of its Q row, rounds it to TF32
//     and stores it into tensor memory. Then per tile: half-row max, exchanged with
//     the partner thread through shared memory (a 64-thread named barrier per
//     pair), row max in log2 units; O (and the row sum) is rescaled only when the
//     row max grows by more than 2^8 (the running max otherwise stays, which leaves
//     the result unchanged and bounds every p by 2^8), so the correction pass over
//     the O columns is rare. P is rounded to the nearest TF32 value and the row sum
//     (kept per half, combined at the end) is taken over the rounded P, so the
//     weights of the V rows sum to one without truncation bias. The same warps read
//     O at the end, divide by the row sum and store the rows;
//   * warps 10..13: converters. Each K and V stage, as it lands, rounded to the nearest
//     TF32 value in shared memory (the tensor cores would truncate, a bias that
//     compounds over the layers), released to the tensor cores by ready barriers.
// Keys past the sequence in the last tile: their scores are masked and their V rows
// zeroed in shared memory (the cache may hold anything there; 0 x NaN is NaN).
// Numerics: TF32 products of operands rounded to nearest, F32 accumulation; on
// N(0, 1) inputs the output moves from exact attention by ~1e-3 of V's RMS, without
// the truncation bias. The output is written rounded to the nearest TF32 value: in
// the B200_PREC_TF32 layer it feeds the o_proj product only.
//
// Every mbarrier wait is bounded (wait_poll, tcgen05.cuh): a wait that runs out records
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
constexpr int kStages = 3;                     // K and V ring depth
constexpr uint32_t kKvBox = kTcKeys * 32 * 4;  // 8 KB: 64 keys x 32 dims
constexpr uint32_t kKvTile = 4 * kKvBox;       // 32 KB
constexpr uint32_t kOffK = 0;                           // K ring
constexpr uint32_t kOffV = kOffK + kStages * kKvTile;   // V ring
// softmax pair exchange: [3][2][128] floats (tile max by tile parity, then the row
// sums in slot 2) and [2][2][128] ok flags
constexpr uint32_t kOffXch = kOffV + kStages * kKvTile;  // 192 KB
constexpr uint32_t kOffXok = kOffXch + 3 * 2 * kTcRows * 4;
constexpr uint32_t kOffBar = kOffXok + 2 * 2 * kTcRows * 4;
constexpr size_t kTcSmem = 1024 /* alignment slack */ + kOffBar + 256;
constexpr int kSoftWarps = 8;                       // warps 2..9: TMEM lane quarter w % 4, column half (w - 2) / 4
constexpr int kCvtWarps = 4;                        // warps 10..13: round K / V to TF32 in place
constexpr int kCvtThreads = 32 * kCvtWarps;
constexpr int kVWarp = 2 + kSoftWarps + kCvtWarps;  // warp 14: TMA engine for V
constexpr int kTcThreads = 32 * (kVWarp + 1);
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 128, kColQ = 256;
constexpr uint32_t kIdescS = idesc_tf32(kTcRows, kTcKeys, false, false);
constexpr uint32_t kIdescO = idesc_tf32(kTcRows, kTcD, false, true);
constexpr float kRescaleLog2 = 8.0f;

__device__ int32_t g_attn_tc_status;  // status word when the caller passes none

// Nearest TF32 value of an F32 bit pattern (ties away from zero): the tensor cores
// would otherwise truncate, which biases every product toward zero.
B200_DEVICE uint32_t tf32_round(uint32_t u) { return (u + 0x1000u) & 0xFFFFE000u; }

// 2^x (ex2.approx.ftz: relative error ~2^-22, far below the TF32 rounding of P)
B200_DEVICE float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Rounds the N16 16-byte groups of a K / V tile at p (8 KB boxes of 64 rows of 128
// bytes) to TF32; thread i of kCvtThreads takes groups i, i + kCvtThreads, ... (eight
// loads in flight); the groups of rows >= valid_rows are cleared instead (a whole
// tile passes valid_rows = 64).
template <int N16>
B200_DEVICE void round_tf32_smem(unsigned char *p, int valid_rows, int i) {
    static_assert(N16 % (8 * kCvtThreads) == 0, "whole rounds of eight groups per thread");
    uint4 *q = reinterpret_cast<uint4 *>(p);
#pragma unroll 1
    for (int j0 = i; j0 < N16; j0 += 8 * kCvtThreads) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = q[j0 + u * kCvtThreads];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + u * kCvtThreads;
            q[j] = ((j & 511) >> 3) >= valid_rows
                       ? make_uint4(0u, 0u, 0u, 0u)
                       : make_uint4(tf32_round(v[u].x), tf32_round(v[u].y), tf32_round(v[u].z), tf32_round(v[u].w));
        }
    }
}

template <int G>
__global__ void __launch_bounds__(kTcThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                           const AttnArgs a) {
    constexpr int BQ = kTcRows / G;
    extern __shared__ unsigned char tc_raw[];
    const uint32_t raw = smem_addr(tc_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;  // swizzled boxes want 1024-byte alignment
    unsigned char *base = tc_raw + (sbase - raw);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + kOffBar);
    uint64_t *k_full = bars;        // [3] K stage landed
    uint64_t *k_empty = bars + 3;   // [3] K stage read by its S product
    uint64_t *k_ready = bars + 6;   // [3] K stage rounded
    uint64_t *v_full = bars + 9;    // [3]
    uint64_t *v_empty = bars + 12;  // [3]
    uint64_t *v_ready = bars + 15;  // [3] V stage rounded (rows past the sequence cleared)
    uint64_t *s_full = bars + 18;   // [2] S buffer complete (and every earlier product)
    uint64_t *p_full = bars + 20;   // [2] P written over S (and O rescaled), one arrival per softmax thread
    uint64_t *q_ready = bars + 22;  // Q in tensor memory, one arrival per softmax thread
    uint64_t *o_done = bars + 23;   // one phase per tile: P_t V_t complete
    uint64_t *o_final = bars + 24;  // the last P V complete
    uint64_t *mma_idle = bars + 25; // no tensor-core work in flight (exit)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 26);
    int32_t *status = a.status ? a.status : &g_attn_tc_status;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // one CTA per (query block, KV head), the heaviest query blocks (most keys under
    // the causal mask) of every head first: the first wave takes the longest CTAs
    const int64_t nqb = gridDim.x / a.Hkv;
    const int64_t qb = nqb - 1 - blockIdx.x / a.Hkv;
    const int64_t kvh = blockIdx.x % a.Hkv;
    const int64_t q0 = qb * BQ;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&k_ready[s], kCvtThreads);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
            mbar_init(&v_ready[s], kCvtThreads);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 32 * kSoftWarps);
        }
        mbar_init(q_ready, 32 * kSoftWarps);
        mbar_init(o_done, 1);
        mbar_init(o_final, 1);
        mbar_init(mma_idle, 1);
        fence_barrier_init();
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

    if (warp == 0 || warp == kVWarp) {
        if (lane == 0) {
            // ---- TMA engine: K (warp 0) or V (warp kVWarp), stage t % 3
            const bool is_k = warp == 0;
            const CUtensorMap *map = is_k ? &tk : &tv;
            uint64_t *full = is_k ? k_full : v_full, *empty = is_k ? k_empty : v_empty;
            const uint32_t ring = sbase + (is_k ? kOffK : kOffV);
            const uint64_t pol = policy_evict_last();  // K / V tiles are re-read by the other query blocks
            int issued = 0;
#pragma unroll 1
            for (int t = 0; t < ntiles; ++t) {
                const int st = t % kStages;
                if (t >= kStages && !wait_poll(&empty[st], ((t / kStages) - 1) & 1, status)) break;
                mbar_arrive_expect_tx(&full[st], kKvTile);
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    tma_load_3d(ring + st * kKvTile + b * kKvBox, map, 32 * b, static_cast<int32_t>(kvh),
                                t * kTcKeys, smem_addr(&full[st]), pol);
                issued = t + 1;
            }
            // copies still landing in this CTA's shared memory (bounded; no-ops when
            // every tile was consumed)
#pragma unroll 1
            for (int t = issued > kStages ? issued - kStages : 0; t < issued; ++t)
                wait_poll(&full[t % kStages], (t / kStages) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- tensor cores
            auto issue_s = [&](int t) {  // S_t = Q . K_t^T into buffer t % 2
                const int ks = t % kStages;
                if (!wait_poll(&k_ready[ks], (t / kStages) & 1, status)) return false;
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>((t & 1) * kTcKeys);
#pragma unroll
                for (int kk = 0; kk < kTcD / 8; ++kk) {  // K 8 per MMA: +32 bytes inside a 128-byte row of K
                    const uint64_t db = desc_k_sw128(sbase + kOffK + ks * kKvTile + (kk >> 2) * kKvBox) + 2 * (kk & 3);
                    tc_mma_tf32_ts(d, tmem + kColQ + 8 * kk, db, kIdescS, kk > 0 ? 1u : 0u);
                }
                tc_commit(smem_addr(&s_full[t & 1]));
                tc_commit(smem_addr(&k_empty[ks]));
                return true;
            };
            bool ok = wait_poll(q_ready, 0, status) && ntiles > 0;
            if (ok) {
                tc_fence_after();
                ok = issue_s(0);
            }
#pragma unroll 1
            for (int t = 0; t < ntiles && ok; ++t) {
                const int sb = t & 1, vs = t % kStages;
                if (t + 1 < ntiles && !issue_s(t + 1)) break;
                if (!wait_poll(&p_full[sb], (t >> 1) & 1, status) ||
                    !wait_poll(&v_ready[vs], (t / kStages) & 1, status))
                    break;
                tc_fence_after();
                const uint32_t pa = tmem + static_cast<uint32_t>(sb * kTcKeys);
#pragma unroll
                for (int kk = 0; kk < kTcKeys / 8; ++kk) {  // K 8 keys per MMA: +1024 bytes of V
                    const uint64_t db = desc_mn_sw128_b32(sbase + kOffV + vs * kKvTile + kk * 1024, kKvBox);
                    tc_mma_tf32_ts(tmem + kColO, pa + 8 * kk, db, kIdescO, (t > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(smem_addr(&v_empty[vs]));
                tc_commit(smem_addr(o_done));
                if (t + 1 == ntiles) tc_commit(smem_addr(o_final));
            }
            // no product may still use tensor memory or the rings when the CTA exits
            tc_commit(smem_addr(mma_idle));
            wait_poll(mma_idle, 0, nullptr);
        }
    } else if (warp >= 2 + kSoftWarps) {
        // ---- converters: every K / V stage as it lands, rounded to TF32 in place; V
        // rows past the sequence (last tile) cleared: the cache may hold anything
        // there, and a zero P does not cancel a NaN
        const int ci = threadIdx.x - 32 * (2 + kSoftWarps);
#pragma unroll 1
        for (int t = 0; t < ntiles; ++t) {
            const int st = t % kStages;
            const uint32_t par = (t / kStages) & 1;
            const int64_t k0 = static_cast<int64_t>(t) * kTcKeys;
            if (!__all_sync(0xffffffffu, wait_poll(&k_full[st], par, status))) break;
            round_tf32_smem<kKvTile / 16>(base + kOffK + st * kKvTile, kTcKeys, ci);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
            mbar_arrive(&k_ready[st]);
            if (!__all_sync(0xffffffffu, wait_poll(&v_full[st], par, status))) break;
            const int nk = static_cast<int>(min64(kTcKeys, Tkv - k0));  // valid rows of this tile
            round_tf32_smem<kKvTile / 16>(base + kOffV + st * kKvTile, nk, ci);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&v_ready[st]);
        }
    } else {
        // ---- softmax: thread (warp w, lane l) owns row 32 (w % 4) + l = TMEM lane,
        // columns [32 h, 32 h + 32) of each S tile and [64 h, 64 h + 64) of Q and O,
        // h = (w - 2) / 4; its partner (warp w +- 4, same lane) owns the other half
        const int h = (warp - 2) >> 2, qq = warp & 3;
        const int r = 32 * qq + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * qq) << 16);
        float *xch = reinterpret_cast<float *>(base + kOffXch);   // [tile parity | 2: sums][half][row]
        int32_t *xok = reinterpret_cast<int32_t *>(base + kOffXok);
        auto pair_sync = [&] { asm volatile("bar.sync %0, 64;" ::"r"(1 + qq) : "memory"); };
        const int64_t tok = q0 + r / G;
        const int64_t qpos = n_past + tok;
        const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf(static_cast<float>(kTcD));
        const float sl2 = scale * 1.4426950408889634f;  // log2(e)
        {
            // this half of the row of Q, rounded to TF32, into tensor memory (rows past Tq: zero)
            const float4 *qrow =
                reinterpret_cast<const float4 *>(a.q + (tok * a.Hq + kvh * G + (r % G)) * kTcD + 64 * h);
#pragma unroll 1
            for (int cb = 0; cb < 2; ++cb) {
                uint32_t qv[32];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float4 v = tok < a.Tq ? qrow[8 * cb + c] : make_float4(0.f, 0.f, 0.f, 0.f);
                    qv[4 * c] = tf32_round(__float_as_uint(v.x));
                    qv[4 * c + 1] = tf32_round(__float_as_uint(v.y));
                    qv[4 * c + 2] = tf32_round(__float_as_uint(v.z));
                    qv[4 * c + 3] = tf32_round(__float_as_uint(v.w));
                }
                tc_st32(trow + kColQ + 64 * h + 32 * cb, qv);
            }
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(q_ready);
        }
        // A failed wait is carried to the next exchange, where both threads of the
        // pair see it and leave the tile loop together: every pair barrier is then
        // reached by both warps the same number of times.
        float m_run = -INFINITY, l_run = 0.f;  // l_run: this half's share of the row sum
        bool bad = false;
#pragma unroll 1
        for (int t = 0; t < ntiles; ++t) {
            const int sb = t & 1;
            const bool okw = !bad && __all_sync(0xffffffffu, wait_poll(&s_full[sb], (t >> 1) & 1, status));
            uint32_t sv[32];
            const int64_t k0 = static_cast<int64_t>(t) * kTcKeys + 32 * h;
            // keys k0 + c with c < nvis are visible to this row (causal and in the sequence)
            const int nvis = okw ? static_cast<int>(max64(0, min64(32, min64(qpos + 1, Tkv) - k0))) : 0;
            if (okw) {
                tc_fence_after();
                tc_ld32_nowait(trow + sb * kTcKeys + 32 * h, sv);
                tc_wait_ld();
                tc_reg_fence(sv);
            }
            // half-row max of the raw scores (the scale is positive: it is applied
            // after), masked keys set to -inf only in tiles that have some
            float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (nvis == 32) {
#pragma unroll
                for (int c = 0; c < 32; ++c) mxp[c & 3] = fmaxf(mxp[c & 3], __uint_as_float(sv[c]));
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float x = c < nvis ? __uint_as_float(sv[c]) : -INFINITY;
                    sv[c] = __float_as_uint(x);
                    mxp[c & 3] = fmaxf(mxp[c & 3], x);
                }
            }
            float mx = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3]));
            // row max = max of both halves (double-buffered by tile parity: the
            // partner may still read the previous tile's value)
            xch[(sb * 2 + h) * kTcRows + r] = mx;
            xok[(sb * 2 + h) * kTcRows + r] = okw ? 1 : 0;
            pair_sync();
            if (!okw || !xok[(sb * 2 + (h ^ 1)) * kTcRows + r]) {
                bad = true;
                break;
            }
            mx = fmaxf(mx, xch[(sb * 2 + (h ^ 1)) * kTcRows + r]) * sl2;  // log2 units
            float alpha = 1.f;
            bool rescale = false;
            if (t == 0) {
                m_run = mx;  // key 0 is visible to every row: finite
            } else if (mx > m_run + kRescaleLog2) {
                alpha = fast_exp2(m_run - mx);
                m_run = mx;
                rescale = true;
            }
            // P rounded to the nearest TF32 value here (the tensor cores would truncate
            // it), and the row sum taken over the same rounded values: the weights of
            // the V rows then sum to one exactly, with no downward bias
            float rsp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const uint32_t pv = tf32_round(__float_as_uint(fast_exp2(fmaf(__uint_as_float(sv[c]), sl2, -m_run))));
                rsp[c & 3] += __uint_as_float(pv);
                sv[c] = pv;
            }
            l_run = l_run * alpha + ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3]));
            if (__any_sync(0xffffffffu, rescale)) {
                // O holds tiles < t once P_{t-1} V_{t-1} is done (the products before
                // it completed ahead of s_full[t]); P_t V_t waits for this thread's P.
                if (!__all_sync(0xffffffffu, wait_poll(o_done, (t - 1) & 1, status))) bad = true;
                tc_fence_after();
#pragma unroll 1
                for (int cb = 0; cb < 2 && !bad; ++cb) {
                    uint32_t o[32];
                    tc_ld32_nowait(trow + kColO + 64 * h + 32 * cb, o);
                    tc_wait_ld();
                    tc_reg_fence(o);
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    tc_st32(trow + kColO + 64 * h + 32 * cb, o);
                }
            }
            tc_st32(trow + sb * kTcKeys + 32 * h, sv);
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[sb]);
        }
        // both halves take part in the final exchange, after a failure as well
        const bool ok = !bad && __all_sync(0xffffffffu, wait_poll(o_final, 0, status));
        xch[(2 * 2 + h) * kTcRows + r] = l_run;
        pair_sync();
        const float l_row = l_run + xch[(2 * 2 + (h ^ 1)) * kTcRows + r];
        if (ok) {
            tc_fence_after();
            const float inv = 1.0f / l_row;
            float *dst = a.out + (tok * a.Hq + kvh * G + (r % G)) * kTcD + 64 * h;
#pragma unroll 1
            for (int cb = 0; cb < 2; ++cb) {
                uint32_t o[32];
                tc_ld32_nowait(trow + kColO + 64 * h + 32 * cb, o);
                tc_wait_ld();
                tc_reg_fence(o);
                if (tok < a.Tq) {
#pragma unroll
                    for (int c = 0; c < 32; c += 4)
                        *reinterpret_cast<float4 *>(dst + 32 * cb + c) =
                            make_float4(tf32_rn(__uint_as_float(o[c]) * inv), tf32_rn(__uint_as_float(o[c + 1]) * inv),
                                        tf32_rn(__uint_as_float(o[c + 2]) * inv), tf32_rn(__uint_as_float(o[c + 3]) * inv));
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
    CUtensorMap mk, mv;
    if (!kv_map(&mk, a.k, a.Hkv, rows, a.k_head, a.k_tok, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !kv_map(&mv, a.v, a.Hkv, rows, a.v_head, a.v_tok, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
        return cudaErrorNotSupported;
    constexpr int BQ = kTcRows / G;
    const dim3 grid(static_cast<unsigned>(((a.Tq + BQ - 1) / BQ) * a.Hkv));
    return b200_launch(kern, grid, dim3(kTcThreads), kTcSmem, stream, pdl, mk, mv, a);
}

}  // namespace

cudaError_t attn_prefill_tc_launch(const AttnArgs &a, cudaStream_t stream, bool pdl) {
    if (a.D != kTcD || a.Hkv <= 0 || a.Hq % a.Hkv || a.Tq < 1) return cudaErrorNotSupported;
    // q rows are read and out rows written as 16-byte vectors
    if ((reinterpret_cast<uintptr_t>(a.out) & 15) || (reinterpret_cast<uintptr_t>(a.q) & 15)) return cudaErrorNotSupported;
    switch (a.Hq / a.Hkv) {
        case 1: return tc_launch<1>(a, stream, pdl);
        case 2: return tc_launch<2>(a, stream, pdl);
        case 4: return tc_launch<4>(a, stream, pdl);
        case 8: return tc_launch<8>(a, stream, pdl);
    }
    return cudaErrorNotSupported;
}

}  // namespace b200
