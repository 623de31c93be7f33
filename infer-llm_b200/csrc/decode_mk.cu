// Persistent decode megakernel: one cooperative launch runs a whole decode step
// (28 layers x [QKV, attention, o_proj, gate/up, down] + LM head + greedy argmax)
// with one CTA per SM: 8 consumer warps and a producer warpgroup.
//
// Weight streaming is decoupled from the activation dependency chain. The step's
// static weight schedule (this CTA's row slice of every projection, layer after
// layer, then the LM head) is cut into ring chunks of whole rows; a producer
// thread streams them through a 16-slot shared-memory ring with cp.async.bulk
// (TMA engine, mbarrier completion) and keeps L2 bulk prefetches further ahead,
// so HBM keeps streaming while the consumers wait on activations. Chunk c is
// read by consumer warp c % 8 from slot c % 16.
//
// There are no grid barriers. Every activation a CTA hands to others (q/k/v rows,
// attention split partials, residual rows, SwiGLU rows) is written as a tagged
// 64-bit word (phase tag | float); the next phase's readers poll exactly the
// words they need until the tag of that phase shows, which costs one store and
// one load round trip instead of a release, a counter update and a poll.
//
// Numerics match the multi-kernel path up to summation order: RMSNorm in double
// with the reference's rounding, row sums and split partials combined in a fixed
// order, so the step is deterministic.
#include <algorithm>
#include <cstdlib>

#include "decode_mk.cuh"
#include "gemv.cuh"

namespace b200 {
namespace {

constexpr int kCW = 8;               // consumer warps
constexpr int kCT = kCW * 32;        // consumer threads
// + one producer warpgroup (warp kCW streams weights, the other three exit).
// Launched at 168 registers a thread (3 warps per SM sub-partition); the producer
// warpgroup drops to kProdRegs and the consumers grow to kConsRegs:
// 4*32*kProdRegs + 8*32*kConsRegs == 12*32*168.
constexpr int kThreads = kCT + 128;
constexpr int kProdRegs = 72;
constexpr int kConsRegs = 216;
static_assert(4 * kProdRegs + 8 * kConsRegs == 12 * 168, "register split must equal the launch total");
constexpr int kStageFloats = 3072;   // 12 KB per ring stage (whole rows)
constexpr int kStages = 16;
// A ring slot is always read by the same warp (chunk c -> warp c % kCW, slot
// c % kStages), so a warp waits on a slot's full barrier only after it consumed
// the slot's previous chunk itself: the barrier is never two phases behind.
static_assert(kStages % kCW == 0, "ring slots must map to a fixed consumer warp");
constexpr int kMaxRpc = 8;           // rows per ring chunk at most
constexpr int kMaxK = 3072;          // largest projection input (= one ring stage)
constexpr int kMaxLayers = 40;
constexpr int kPartFloats = 2048;    // per-CTA row sums of one phase
constexpr int kResFloats = 64;       // this CTA's rows of the residual stream
constexpr int kMaxSplits = 18;
constexpr int kDefaultInflight = 8;  // measured: 8 copies (96 KB) per SM keep HBM busy; 3 starve the LM head
constexpr int kDefaultSplitKeys = 32;  // keys per attention split
constexpr int kMaxGq = 4;            // query heads per KV head (attention registers)
enum { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_PER_LAYER = 5 };

struct PhaseW {
    const float *w;
    int64_t N, K;
    int unit;  // 2: rows come in (gate, up) pairs
};

// The layer table, copied to shared memory at kernel start: the ring cursors cross
// phases constantly and every phase starts from a layer pointer, so none of them
// may wait on a global load to find its matrix or norm weights.
__shared__ MkLayer s_layers[kMaxLayers];
// cos / sin of this step's rotation angles (the position is the same in every
// layer): s_rope[j] = cos, s_rope[kMaxHalfD + j] = sin of float(double(pos) * freq_j).
constexpr int kMaxHalfD = 64;
__shared__ float s_rope[2 * kMaxHalfD];

B200_DEVICE PhaseW phase_w(const MkParams &p, int l, int ph) {
    if (l == p.n_layer) return {p.lm_head, p.V, p.H, 1};
    switch (ph) {
        case PH_QKV: return {s_layers[l].wqkv, static_cast<int64_t>(p.Hq + 2 * p.Hkv) * p.D, p.H, 1};
        case PH_O: return {s_layers[l].wo, p.H, static_cast<int64_t>(p.Hq) * p.D, 1};
        case PH_GU: return {s_layers[l].wgu, 2 * static_cast<int64_t>(p.F), p.H, 2};
        case PH_DOWN: return {s_layers[l].wdown, p.H, p.F, 1};
    }
    return {nullptr, 0, 0, 1};
}

// Rows per ring chunk: as many whole rows as one stage holds, at most kMaxRpc.
B200_HOST_DEVICE int rpc_for(int64_t K, int /*unit*/) {
    const int64_t r = kStageFloats / K;
    return static_cast<int>(r < kMaxRpc ? r : kMaxRpc);
}

// This CTA's row range of an N-row matrix, in whole units (32-bit arithmetic:
// units * G stays below 2^31 for every supported shape).
B200_DEVICE void rows_of(int64_t N, int unit, int b, int G, int64_t &r0, int64_t &r1) {
    const unsigned units = static_cast<unsigned>(N / unit);
    r0 = static_cast<int64_t>(units * static_cast<unsigned>(b) / static_cast<unsigned>(G)) * unit;
    r1 = static_cast<int64_t>(units * static_cast<unsigned>(b + 1) / static_cast<unsigned>(G)) * unit;
}

// This CTA's geometry of one projection kind: its rows [r0, r1), rows per ring
// chunk, chunks. The same in every layer, so it is computed once per launch (the
// integer divisions behind it cost hundreds of cycles on the critical path when
// redone at every phase). Index: PH_QKV, PH_O, PH_GU, PH_DOWN; kGeoLm = LM head.
struct Geo {
    int r0, r1, rpc, nch;
};
constexpr int kGeoLm = PH_ATTN;  // the attention slot holds the LM head (attention streams no weights)
__shared__ Geo s_geo[PH_PER_LAYER];
B200_DEVICE int geo_index(const MkParams &p, int l, int ph) { return l == p.n_layer ? kGeoLm : ph; }

// Walks this CTA's weight schedule chunk by chunk, in consumption order: per layer
// the QKV, o_proj, gate/up and down row slices (attention streams no weights), then
// the LM head. A chunk is rpc whole rows (at most one ring stage). Advancing by n
// chunks costs O(1) per phase crossed.
struct Cursor {
    int l = 0, ph = 0, k = 0, nch = 0, rpc = 1;
    int64_t r0 = 0, r1 = 0;  // this CTA's rows of the phase; the cursor is at chunk k of nch
    PhaseW pw{};

    B200_DEVICE void load_phase(const MkParams &p, int, int) {
        pw = phase_w(p, l, ph);
        const Geo &g = s_geo[geo_index(p, l, ph)];
        r0 = g.r0;
        r1 = g.r1;
        rpc = g.rpc;
        nch = g.nch;
    }
    // Positions the cursor at chunk n of the schedule; false if there is none.
    B200_DEVICE bool start(const MkParams &p, int b, int G, int n) {
        l = 0;
        ph = 0;
        k = 0;
        load_phase(p, b, G);
        return advance(p, b, G, n);
    }
    // Moves n chunks on; false once past the LM head.
    B200_DEVICE bool advance(const MkParams &p, int b, int G, int n) {
        k += n;
#pragma unroll 1
        while (k >= nch) {
            if (l == p.n_layer) return false;
            k -= nch;
            ph += (ph + 1 == PH_ATTN) ? 2 : 1;
            if (ph >= PH_PER_LAYER) {
                ++l;
                ph = 0;
            }
            load_phase(p, b, G);
        }
        return true;
    }
    B200_DEVICE uint32_t bytes() const {
        return static_cast<uint32_t>(min64(rpc, r1 - r0 - static_cast<int64_t>(k) * rpc) * pw.K * 4);
    }
    B200_DEVICE const float *src() const { return pw.w + (r0 + static_cast<int64_t>(k) * rpc) * pw.K; }
};

// L2-resident data on the critical path. The weight stream is read with an
// evict_first policy; the KV cache, the norm weights and the RoPE table are read
// and written with evict_last so that they stay in L2 from step to step instead of
// queueing behind the stream in HBM.
B200_DEVICE float4 ld_keep4(const float *p, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.cg.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}
B200_DEVICE float2 ld_keep2(const float *p, uint64_t pol) {
    float2 v;
    asm volatile("ld.global.cg.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;" : "=f"(v.x), "=f"(v.y) : "l"(p), "l"(pol));
    return v;
}
B200_DEVICE void prefetch_l2_keep(const float *p) {
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}
B200_DEVICE float ld_keep_f(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
B200_DEVICE void st_keep(float *p, float v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v), "l"(pol) : "memory");
}
// E consecutive floats (E = 2 or 4, 8- or 16-byte aligned) with the keep policy.
template <int E>
B200_DEVICE void ld_keep_vec(const float *src, float (&v)[E], uint64_t pol) {
    if constexpr (E == 4) {
        const float4 t = ld_keep4(src, pol);
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
    } else {
        static_assert(E == 2, "head_dim 64 or 128");
        const float2 t = ld_keep2(src, pol);
        v[0] = t.x, v[1] = t.y;
    }
}

B200_DEVICE int status_set(const int32_t *s) { return *reinterpret_cast<const volatile int32_t *>(s); }

constexpr uint64_t kWaitNs = 2000000000ull;  // every wait gives up after 2 s

// Bounded wait on an mbarrier phase: abandoned as soon as any CTA has reported an
// error (its peers may have stopped), and after kWaitNs (sets the timeout status).
// status == nullptr: wait for this CTA's own copies in flight, ignoring errors.
// The waiting thread sleeps in hardware between polls (woken when the phase
// completes), so it does not steal issue slots from the warps beside it.
B200_DEVICE bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int32_t *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
#pragma unroll 1
    for (uint32_t i = 0; i < B200_SPIN_LIMIT; ++i) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if ((i & 7) == 7) {
            if (status && status_set(status)) return false;
            if (global_ns() - t0 > kWaitNs) break;
        }
    }
    if (status) set_status(status, B200_DEV_TIMEOUT);
    return false;
}

// ---------------------------------------------------------------------------
// Tagged activation words. Every value one CTA hands to others is stored as one
// 64-bit word (tag << 32 | float bits) with a single relaxed gpu-scope store, so
// a reader that sees the tag it expects also sees the value of that phase: no
// fence, no flag, no grid barrier. Tags are (launch mod kMkTagPeriod + 1) *
// kTagStride + phase index (the launch counter advances on every launch, aborted
// ones included, and the host clears it with the words before a period can pass),
// so nothing left over from an earlier step ever matches.
// A buffer is rewritten only two phases after it was read, and every phase needs
// the previous phase's outputs of all CTAs, so no writer can overtake a reader.
constexpr uint32_t kTagStride = 256;  // > 5 * kMaxLayers + 1 phase indices
static_assert((kMkTagPeriod + 1) * kTagStride <= (1ull << 32), "tags fit 32 bits");
using u64 = unsigned long long;

B200_DEVICE uint32_t tag_hi(u64 w) { return static_cast<uint32_t>(w >> 32); }
B200_DEVICE float tag_val(u64 w) { return __uint_as_float(static_cast<uint32_t>(w)); }
B200_DEVICE void st_tagged(u64 *p, float v, uint32_t tag) {
    const u64 w = (static_cast<u64>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
B200_DEVICE u64 ld_tagged1(const u64 *p) {
    u64 a;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
    return a;
}
B200_DEVICE void ld_tagged2(const u64 *p, u64 &a, u64 &b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Polls word pairs until both carry `tag`: `pending` is a bit mask over the
// caller's pairs, `reload(j)` re-reads pair j. Gives up (status set) after
// kWaitNs or as soon as another CTA reported an error.
template <int N, class Check, class Reload>
B200_DEVICE bool poll_pairs(unsigned pending, const int32_t *status_p, int32_t *status, Check ok, Reload reload) {
    uint64_t t0 = 0;
#pragma unroll 1
    for (uint32_t it = 0; it < B200_SPIN_LIMIT; ++it) {
        unsigned still = 0;
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (((pending >> j) & 1u) && !ok(j)) still |= 1u << j;
        if (!still) return true;
        if ((it & 15) == 15) {
            if (status_set(status_p)) return false;
            const uint64_t t = global_ns();
            if (!t0) t0 = t;
            else if (t - t0 > kWaitNs) {
                set_status(status, B200_DEV_TIMEOUT);
                return false;
            }
        }
        // polls back to back: each retry already waits one L2 round trip
#pragma unroll
        for (int j = 0; j < N; ++j)
            if ((still >> j) & 1u) reload(j);
        pending = still;
    }
    set_status(status, B200_DEV_TIMEOUT);
    return false;
}

// Named barrier over `threads` threads that also ORs `pred` over them: every
// participant gets the same answer, so a decision taken on it is uniform over the
// CTA (a flag in shared memory set by some threads and cleared by one would need
// a barrier between the clear and the sets).
B200_DEVICE bool named_sync_or(int id, int threads, bool pred) {
    int r;
    asm volatile(
        "{\n .reg .pred p, q;\n"
        " setp.ne.s32 p, %1, 0;\n"
        " bar.red.or.pred q, %2, %3, p;\n"
        " selp.s32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(pred ? 1 : 0), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

// Device trace (CTA 0, thread 0): phase idx, slot k <- global time.
B200_DEVICE void stamp(const MkParams &p, int idx, int k) {
    if (p.trace && threadIdx.x == 0 && blockIdx.x == 0) p.trace[idx * 8 + k] = global_ns();
}

struct Smem {
    uint64_t *full, *empty;  // [kStages] copy-complete / slot-read barriers
    float *ring;   // [kStages][kStageFloats]
    float *xs;     // [kMaxK] phase input activation
    float *part;   // [kPartFloats]
    float *qs;     // [Gq][D] rotated queries of the KV group (attention)
    float *res;    // [kResFloats] this CTA's residual rows (o_proj / down row range)
};

// D: head_dim; GQ: query heads per KV head (compile time: the attention's per-head
// loops and warp shuffles then have no head conditions, so they pipeline).
template <int D, int GQ>
struct Mk {
    static constexpr int E = D / 32;  // head elements per lane
    const MkParams &p;
    const Smem &sm;
    const int tid, warp, lane, b, G;
    const uint32_t tag0;                        // this launch's tag base
    const uint64_t keep = policy_evict_last();  // KV cache, norm weights, RoPE table

    B200_DEVICE uint32_t tag(int layer, int ph) const { return tag0 + static_cast<uint32_t>(layer * PH_PER_LAYER + ph); }

    // ---- phase input from tagged words: xs = src (optionally RMS-normalised with
    // gamma), in rounds of kP word pairs per thread (all loads of a round in
    // flight together, only stale pairs re-read); gamma is applied from shared
    // memory once the sum of squares is known.
    B200_DEVICE bool load_act(const u64 *src, int64_t K, const float *gamma, uint32_t want) {
        // word pairs per thread per round: the largest input (kMaxK floats) is
        // requested in one round, so a phase waits one L2 round trip, not K / 512
        constexpr int kP = kMaxK / 2 / kCT;
        __shared__ double s_red[kCW];
        const int64_t K2 = K >> 1;
        constexpr int kG = 2;  // gamma pairs per thread loaded with the words (K <= 2 kG kCT)
        float2 gv[kG];
#pragma unroll
        for (int j = 0; j < kG; ++j)
            if (gamma && tid + j * kCT < K2) gv[j] = ld_keep2(gamma + 2 * (tid + j * kCT), keep);
        double ss = 0.0;
        bool ok = true;
#pragma unroll 1
        for (int64_t base = 0; base < K2 && ok; base += kP * kCT) {
            u64 a[kP], c[kP];
            unsigned pending = 0;
#pragma unroll
            for (int j = 0; j < kP; ++j) {
                const int64_t i = base + tid + j * kCT;
                if (i < K2) {
                    ld_tagged2(src + 2 * i, a[j], c[j]);
                    pending |= 1u << j;
                }
            }
            ok = poll_pairs<kP>(
                pending, p.status, p.status, [&](int j) { return tag_hi(a[j]) == want && tag_hi(c[j]) == want; },
                [&](int j) { ld_tagged2(src + 2 * (base + tid + j * kCT), a[j], c[j]); });
#pragma unroll
            for (int j = 0; j < kP; ++j) {
                if ((pending >> j) & 1u) {
                    const float x0 = tag_val(a[j]), x1 = tag_val(c[j]);
                    const float q0 = x0 * x0, q1 = x1 * x1;
                    ss += static_cast<double>(q0);
                    ss += static_cast<double>(q1);
                    reinterpret_cast<float2 *>(sm.xs)[base + tid + j * kCT] = make_float2(x0, x1);
                }
            }
        }
        if (gamma) {
            ss = warp_sum(ss);
            if (lane == 0) s_red[warp] = ss;
            named_sync(1, kCT);
            double t = 0.0;  // every thread sums the warp totals in the same order
#pragma unroll
            for (int w = 0; w < kCW; ++w) t += s_red[w];
            const float sc = rms_scale_from_sumsq(t, K, p.eps);
            auto apply = [&](int64_t i, float2 g) {  // only pairs this thread wrote
                float2 y = reinterpret_cast<float2 *>(sm.xs)[i];
                y.x = __fmul_rn(__fmul_rn(y.x, sc), g.x);
                y.y = __fmul_rn(__fmul_rn(y.y, sc), g.y);
                reinterpret_cast<float2 *>(sm.xs)[i] = y;
            };
#pragma unroll
            for (int j = 0; j < kG; ++j)
                if (tid + j * kCT < K2) apply(tid + j * kCT, gv[j]);
#pragma unroll 1
            for (int64_t i = tid + kG * kCT; i < K2; i += kCT) apply(i, ld_keep2(gamma + 2 * i, keep));
        }
        return !named_sync_or(1, kCT, !ok);  // uniform over the CTA
    }

    // ---- the same from plain floats (the token's embedding row).
    B200_DEVICE void load_act_plain(const float *src, int64_t K, const float *gamma) {
        constexpr int kV = kMaxK / 4 / kCT;
        __shared__ double s_red[kCW];
        const int64_t K4 = K >> 2;
        float4 v[kV], g[kV];
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int64_t i = tid + j * kCT;
            if (i < K4) {
                v[j] = __ldg(reinterpret_cast<const float4 *>(src) + i);
                g[j] = ld_keep4(gamma + 4 * i, keep);
            }
        }
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            if (tid + j * kCT < K4) {
                const float q0 = v[j].x * v[j].x, q1 = v[j].y * v[j].y, q2 = v[j].z * v[j].z, q3 = v[j].w * v[j].w;
                ss += static_cast<double>(q0);
                ss += static_cast<double>(q1);
                ss += static_cast<double>(q2);
                ss += static_cast<double>(q3);
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        named_sync(1, kCT);
        double t = 0.0;
#pragma unroll
        for (int w = 0; w < kCW; ++w) t += s_red[w];
        const float sc = rms_scale_from_sumsq(t, K, p.eps);
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int64_t i = tid + j * kCT;
            if (i < K4) {
                float4 y = v[j];
                y.x = __fmul_rn(__fmul_rn(y.x, sc), g[j].x);
                y.y = __fmul_rn(__fmul_rn(y.y, sc), g[j].y);
                y.z = __fmul_rn(__fmul_rn(y.z, sc), g[j].z);
                y.w = __fmul_rn(__fmul_rn(y.w, sc), g[j].w);
                reinterpret_cast<float4 *>(sm.xs)[i] = y;
            }
        }
        named_sync(1, kCT);
    }

    // ---- R rows of one ring chunk against x (both in shared memory): each lane
    // takes float4 columns lane, lane + 32, ...; U columns per row are loaded
    // together (U * (R + 1) shared loads in flight) and accumulated per component
    // so no FMA waits on the previous one; then reduces the R row sums across the
    // warp (fixed order) into dst[0..R).
    template <int R>
    B200_DEVICE void chunk_rows(uint32_t w_sa, uint32_t x_sa, int K4, float *dst) {
        constexpr int U = R == 1 ? 8 : (R <= 3 ? 4 : 2);
        float4 a[R];
#pragma unroll
        for (int r = 0; r < R; ++r) a[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        auto fma_block = [&](const float4 (&xv)[U], const float4 (&wv)[R][U]) {
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    a[r].x = fmaf(wv[r][u].x, xv[u].x, a[r].x);
                    a[r].y = fmaf(wv[r][u].y, xv[u].y, a[r].y);
                    a[r].z = fmaf(wv[r][u].z, xv[u].z, a[r].z);
                    a[r].w = fmaf(wv[r][u].w, xv[u].w, a[r].w);
                }
        };
        // whole blocks of 32 U columns: the loads carry no bounds conditions, so
        // they issue back to back in one basic block (every projection of the
        // supported shapes is whole blocks); a ragged tail block after them
        const int full = K4 / (32 * U) * (32 * U);
        int i0 = lane;
#pragma unroll 1
        for (; i0 < full; i0 += 32 * U) {
            float4 xv[U], wv[R][U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                xv[u] = lds4(x_sa + 16u * (i0 + 32 * u));
#pragma unroll
                for (int r = 0; r < R; ++r) wv[r][u] = lds4(w_sa + 16u * (r * K4 + i0 + 32 * u));
            }
            fma_block(xv, wv);
        }
        if (i0 < K4) {
            float4 xv[U], wv[R][U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + 32 * u;
                xv[u] = i < K4 ? lds4(x_sa + 16u * i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int r = 0; r < R; ++r)
                    wv[r][u] = i < K4 ? lds4(w_sa + 16u * (r * K4 + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            fma_block(xv, wv);
        }
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = (a[r].x + a[r].y) + (a[r].z + a[r].w);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) dst[r] = acc[r];
        }
    }

    // ---- consume this CTA's ring chunks of one projection: chunk k of the phase
    // (schedule chunk cc + k) belongs to warp (cc + k) % kCW, which computes its
    // rpc whole rows (x from shared memory, one lane-strided pass, one warp
    // reduction per row) while the other warps work on the next chunks, and
    // releases the slot to the producer. Row sums -> sm.part. With `out` set, the
    // warp also publishes its rows at once (residual added from sm.res when
    // `residual`): a phase's last row goes out as soon as it is computed, not after
    // the CTA's barrier. Returns false on a failed wait (uniform over the CTA).
    B200_DEVICE bool consume(const PhaseW &pw, const Geo &gm, int &cc, int trace_idx, u64 *out, uint32_t tag,
                             bool residual) {
        const bool tr = p.trace && b == 0;  // CTA 0 records its slowest warp's chunk waits
        __shared__ unsigned long long s_wait, s_loop;
        if (tr && tid == 0) s_wait = s_loop = 0;
        uint64_t t_wait = 0;
        const long long tl0 = tr ? clock64() : 0;
        const int rpc = gm.rpc, nch = gm.nch, r0 = gm.r0, r1 = gm.r1;
        const int K4 = static_cast<int>(pw.K >> 2);
        const uint32_t x_sa = smem_addr(sm.xs);
        bool failed = false;
        if (tr) named_sync(1, kCT);  // s_wait / s_loop are cleared before any warp records
#pragma unroll 1
        for (int k = ((warp - cc) % kCW + kCW) % kCW; k < nch; k += kCW) {
            const int c = cc + k;
            const int s = c % kStages;
            const long long tw0 = tr ? clock64() : 0;
            if (!mbar_wait_bounded(&sm.full[s], (c / kStages) & 1, p.status)) {
                failed = true;
                break;
            }
            if (tr) t_wait += clock64() - tw0;
            const int row = r0 + k * rpc;
            const int rows = min(rpc, r1 - row);
            const uint32_t w_sa = smem_addr(sm.ring) + 4u * kStageFloats * s;
            float *dst = sm.part + (row - r0);
#pragma unroll 1
            for (int r = 0; r < rows; r += 3) {  // sub-chunks of at most 3 rows
                const int n = min(3, rows - r);
                const uint32_t wr_sa = w_sa + 16u * r * K4;
                if (n == 3)
                    chunk_rows<3>(wr_sa, x_sa, K4, dst + r);
                else if (n == 2)
                    chunk_rows<2>(wr_sa, x_sa, K4, dst + r);
                else
                    chunk_rows<1>(wr_sa, x_sa, K4, dst + r);
            }
            __syncwarp();  // the stage is read (and lane 0's row sums are in sm.part)
            if (lane == 0) mbar_arrive(&sm.empty[s]);
            if (out && lane < rows) {
                float v = dst[lane];
                if (residual) {  // this CTA's own residual rows, kept in shared memory
                    v += sm.res[row - r0 + lane];
                    sm.res[row - r0 + lane] = v;
                }
                st_tagged(out + row + lane, v, tag);
            }
        }
        cc += nch;
        if (tr && lane == 0) {
            atomicMax(&s_wait, static_cast<unsigned long long>(t_wait));
            atomicMax(&s_loop, static_cast<unsigned long long>(clock64() - tl0));
        }
        failed = named_sync_or(1, kCT, failed);
        if (tr && tid == 0) {
            p.trace[trace_idx * 8 + 1] = s_loop;        // slowest warp's ring loop, SM cycles
            p.trace[trace_idx * 8 + 6] = s_wait;        // slowest warp's total chunk wait, SM cycles
            p.trace[trace_idx * 8 + 7] = global_ns();   // all chunks consumed
        }
        return !failed;
    }

    B200_DEVICE float row_sum(int64_t lr) const { return sm.part[lr]; }

    // Attention splits per KV head for L keys: about p.split_keys keys per split, at most
    // kMaxSplits and at most G / Hkv (one CTA per (KV head, split)).
    B200_DEVICE int attn_splits(int64_t L) const {
        const int S = static_cast<int>((L + p.split_keys - 1) / p.split_keys);
        return max(1, min(S, min(kMaxSplits, G / p.Hkv)));
    }

    // One lane's E consecutive tagged words of a head (E even), waiting for `want`.
    B200_DEVICE bool read_head_lane(const u64 *src, uint32_t want, float (&v)[E]) {
        constexpr int NP = E / 2;
        u64 a[NP], c[NP];
#pragma unroll
        for (int j = 0; j < NP; ++j) ld_tagged2(src + lane * E + 2 * j, a[j], c[j]);
        const bool ok = poll_pairs<NP>(
            (1u << NP) - 1, p.status, p.status, [&](int j) { return tag_hi(a[j]) == want && tag_hi(c[j]) == want; },
            [&](int j) { ld_tagged2(src + lane * E + 2 * j, a[j], c[j]); });
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            v[2 * j] = tag_val(a[j]);
            v[2 * j + 1] = tag_val(c[j]);
        }
        return ok;
    }

    // One warp: RMSNorm + NeoX RoPE of one head of D = 32 E floats (reference
    // rounding: float squares summed in double, y = (x * scale) * gamma, angle =
    // float(double(pos) * freq_j), separately rounded rotation products). The head
    // comes from tagged words; gamma and the frequency table are loaded with it.
    B200_DEVICE bool norm_rope_head(const u64 *src, uint32_t want, const float *gamma, float *dst) {
        const bool lo = lane < 16;
        float v[E], gm[E];
        ld_keep_vec(gamma + lane * E, gm, keep);
        const bool ok = read_head_lane(src, want, v);
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const float sq = v[e] * v[e];
            ss += static_cast<double>(sq);
        }
        ss = warp_sum(ss);
        const float sc = rms_scale_from_sumsq(ss, D, p.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], sc), gm[e]);
        float other[E];
#pragma unroll
        for (int e = 0; e < E; ++e) other[e] = __shfl_xor_sync(0xffffffffu, v[e], 16);
        const int j0 = (lo ? lane : lane - 16) * E;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const float c = s_rope[j0 + e], s = s_rope[kMaxHalfD + j0 + e];
            dst[lane * E + e] = lo ? __fsub_rn(__fmul_rn(v[e], c), __fmul_rn(other[e], s))
                                   : __fadd_rn(__fmul_rn(other[e], s), __fmul_rn(v[e], c));
        }
        return __all_sync(0xffffffffu, ok);
    }

    // The step's rotation table (every layer rotates at the same position n_past):
    // the reference's table entry float(double(pos) * freq_j), then its sine and
    // cosine, once per launch instead of once per head and layer.
    B200_DEVICE void rope_table(int64_t pos) {
        // one copy of the accurate sincosf (its large-argument path is big)
#pragma unroll 1
        for (int j = tid; j < D / 2; j += kCT) {
            const float ang = static_cast<float>(static_cast<double>(pos) * static_cast<double>(ld_keep_f(p.freq + j)));
            float sn, cs;
            sincosf(ang, &sn, &cs);
            s_rope[j] = cs;
            s_rope[kMaxHalfD + j] = sn;
        }
    }

    // ---- attention for one (KV head g, split s): the split's keys are cut into
    // kCW sub-ranges, one per warp, and every warp scores its keys against all Gq
    // query heads of the group (each cached K/V row is read once per CTA). Warps
    // 0..Gq-1 normalise + rotate the queries, warp Gq the new token's key and warp
    // Gq+1 copies its value (last split only; both are appended to the cache for
    // later steps and used from shared memory here). The first batch of cached
    // K/V rows is in flight while that happens. Online softmax in batches of kTB
    // keys; the kCW sub-range partials are merged in order and the split partial
    // (o, max, sum) per query head goes out as tagged words.
    B200_DEVICE bool attention(int layer, int64_t n_past) {
        constexpr int kTB = 4;
        const MkLayer &Lw = s_layers[layer];
        const uint32_t want = tag(layer, PH_QKV), mine = tag(layer, PH_ATTN);
        constexpr int Gq = GQ;
        const int64_t L = n_past + 1;
        const int S = attn_splits(L);
        if (b >= p.Hkv * S) return true;
        __shared__ int s_bad;
        if (tid == 0) s_bad = 0;
        named_sync(1, kCT);  // shared scratch is free: the QKV epilogue has read sm.part
        const int g = b / S, s = b % S;
        const int64_t j0 = L * s / S, j1 = L * (s + 1) / S;
        const bool last = (s == S - 1);
        const int64_t tok = static_cast<int64_t>(p.Hkv) * D;  // cache token stride
        const int64_t t0 = j0 + (j1 - j0) * warp / kCW, t1 = j0 + (j1 - j0) * (warp + 1) / kCW;
        const float *kb = Lw.kc + g * D + lane * E, *vb = Lw.vc + g * D + lane * E;
        float *kn = sm.part + kPartFloats - 2 * D, *vn = kn + D;  // the new token's k, v
        float *wpart = sm.xs;  // [kCW][Gq][D + 2] sub-range partials (xs and part are contiguous)
        float kv[kTB][E], vv[kTB][E];
        auto load_batch = [&](int64_t t, int n) {
#pragma unroll
            for (int j = 0; j < kTB; ++j) {
                if (j < n && t + j != n_past) {
                    ld_keep_vec(kb + (t + j) * tok, kv[j], keep);
                    ld_keep_vec(vb + (t + j) * tok, vv[j], keep);
                } else {
#pragma unroll
                    for (int e = 0; e < E; ++e) kv[j][e] = vv[j][e] = 0.f;
                }
            }
        };
        load_batch(t0, static_cast<int>(min64(kTB, t1 - t0)));
        {
            // the next kPreB batches' cached rows towards L2 meanwhile (the first
            // batch is in flight to registers): E lines of 128 B per row
            constexpr int kPreB = 3;
            const int64_t nk = min64(kPreB * kTB, max64(0, t1 - t0 - kTB));
            const float *kr = Lw.kc + g * D, *vr = Lw.vc + g * D;
#pragma unroll 1
            for (int64_t x = lane; x < nk * 2 * E; x += 32) {
                const int64_t key = t0 + kTB + x / (2 * E);
                const int line = static_cast<int>(x % E);
                prefetch_l2_keep(((x / E) & 1 ? vr : kr) + key * tok + line * 32);
            }
        }
        bool ok = true;
        const bool isq = warp < Gq, isk = last && warp == Gq;
        if (isq || isk) {  // one call site for the norm + RoPE code
            ok = norm_rope_head(p.tqkv + (isq ? g * Gq + warp : p.Hq + g) * D, want, isq ? Lw.q_norm : Lw.k_norm,
                                isq ? sm.qs + warp * D : kn);
            if (isk) {
                __syncwarp();
                float *dst = Lw.kc + n_past * tok + g * D;
#pragma unroll 1
                for (int d = lane; d < D; d += 32) st_keep(dst + d, kn[d], keep);
            }
        }
        if (last && warp == Gq + 1) {  // new token v as is
            float v[E];
            ok = __all_sync(0xffffffffu, read_head_lane(p.tqkv + (p.Hq + p.Hkv + g) * D, want, v));
            float *vdst = Lw.vc + n_past * tok + g * D;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                vn[lane * E + e] = v[e];
                st_keep(vdst + lane * E + e, v[e], keep);
            }
        }
        if (!ok && lane == 0) s_bad = 1;
        named_sync(1, kCT);
        if (s_bad) return false;
        const int tq = layer * PH_PER_LAYER + PH_ATTN;
        stamp(p, tq, 4);  // q / k / v in, normalised and rotated
        float q[Gq][E], m[Gq], l[Gq], o[Gq][E];
#pragma unroll
        for (int hh = 0; hh < Gq; ++hh) {
            m[hh] = -INFINITY;
            l[hh] = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                q[hh][e] = sm.qs[hh * D + lane * E + e];
                o[hh][e] = 0.f;
            }
        }
        const float scale = 1.0f / sqrtf(static_cast<float>(D));
#pragma unroll 1
        for (int64_t t = t0; t < t1; t += kTB) {
            const int n = static_cast<int>(min64(kTB, t1 - t));
            if (t != t0) load_batch(t, n);
            if (n_past >= t && n_past < t + n) {  // patch in the new token
                const int j = static_cast<int>(n_past - t);
#pragma unroll
                for (int jj = 0; jj < kTB; ++jj)
                    if (jj == j) {
#pragma unroll
                        for (int e = 0; e < E; ++e) {
                            kv[jj][e] = kn[lane * E + e];
                            vv[jj][e] = vn[lane * E + e];
                        }
                    }
            }
            float sc[kTB][Gq];
#pragma unroll
            for (int j = 0; j < kTB; ++j)
#pragma unroll
                for (int hh = 0; hh < Gq; ++hh) {
                    float d = 0.f;
#pragma unroll
                    for (int e = 0; e < E; ++e) d = fmaf(q[hh][e], kv[j][e], d);
                    sc[j][hh] = d;
                }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int j = 0; j < kTB; ++j)
#pragma unroll
                    for (int hh = 0; hh < Gq; ++hh)
                        sc[j][hh] += __shfl_xor_sync(0xffffffffu, sc[j][hh], off);
#pragma unroll
            for (int hh = 0; hh < Gq; ++hh) {
                float bm = m[hh];
#pragma unroll
                for (int j = 0; j < kTB; ++j) {
                    sc[j][hh] = j < n ? sc[j][hh] * scale : -INFINITY;
                    bm = fmaxf(bm, sc[j][hh]);
                }
                const float corr = (m[hh] == -INFINITY) ? 0.f : expf(m[hh] - bm);
                l[hh] *= corr;
#pragma unroll
                for (int e = 0; e < E; ++e) o[hh][e] *= corr;
#pragma unroll
                for (int j = 0; j < kTB; ++j) {  // keys past n: score -inf, weight 0, v 0
                    const float pr = expf(sc[j][hh] - bm);
                    l[hh] += pr;
#pragma unroll
                    for (int e = 0; e < E; ++e) o[hh][e] = fmaf(pr, vv[j][e], o[hh][e]);
                }
                m[hh] = bm;
            }
        }
#pragma unroll
        for (int hh = 0; hh < Gq; ++hh) {
            float *wp = wpart + (warp * Gq + hh) * (D + 2);
#pragma unroll
            for (int e = 0; e < E; ++e) wp[lane * E + e] = o[hh][e];
            if (lane == 0) {
                wp[D] = m[hh];
                wp[D + 1] = l[hh];
            }
        }
        named_sync(1, kCT);
        // merge the kCW sub-ranges of each head in order -> the split's partial
        // (or, with one split, the group's output: os / lsum is what the split
        // merge below yields for S == 1, exp(0) and fmaf(1, x, 0) being exact)
#pragma unroll 1
        for (int i = tid; i < Gq * D; i += kCT) {
            const int hh = i / D, d = i % D;
            float M = -INFINITY;
#pragma unroll 1
            for (int u = 0; u < kCW; ++u) M = fmaxf(M, wpart[(u * Gq + hh) * (D + 2) + D]);
            float lsum = 0.f, os = 0.f;
#pragma unroll 1
            for (int u = 0; u < kCW; ++u) {
                const float *w = wpart + (u * Gq + hh) * (D + 2);
                if (w[D] == -INFINITY) continue;
                const float f = expf(w[D] - M);
                lsum = fmaf(f, w[D + 1], lsum);
                os = fmaf(f, w[d], os);
            }
            if (S == 1) {
                st_tagged(p.tao + static_cast<int64_t>(g * Gq) * D + i, os / lsum, mine);
                continue;
            }
            const int64_t sh = static_cast<int64_t>(s) * p.Hq + g * Gq + hh;
            st_tagged(p.tpo + sh * D + d, os, mine);
            if (d == 0) {
                st_tagged(p.tpml + sh * 2, M, mine);
                st_tagged(p.tpml + sh * 2 + 1, lsum, mine);
            }
        }
        named_sync(1, kCT);  // sm.xs (the sub-range partials) is read before it is reused
        stamp(p, tq, 7);  // split partial stored
        return S == 1 || merge_group(layer, g, s, S);
    }

    // ---- split merge inside the attention CTAs: CTA (g, s) merges its slice
    // [n s / S, n (s + 1) / S) of the n = Gq D outputs of KV group g from the S
    // split partials (one round of word loads: every split's value of the slice
    // and every split's (max, sum) of the group's heads), in split order, and
    // writes the merged outputs as tagged words. The o_proj phase then reads the
    // Hq D outputs in one round instead of S partials in several.
    B200_DEVICE bool merge_group(int layer, int g, int s, int S) {
        constexpr int kW = 3;  // slice words per thread: S * ns <= n + S <= kW * kCT
        const uint32_t want = tag(layer, PH_ATTN);
        constexpr int Gq = GQ;
        const int n = Gq * D;
        const int e0 = n * s / S, e1 = n * (s + 1) / S, ns = e1 - e0;
        float *vals = sm.xs;            // [S][ns]
        float *ml = sm.xs + kMaxK / 2;  // [S][Gq][2]
        auto word = [&](int j) -> const u64 * {  // slice word j = (split, element)
            const int sp = j / ns, i = j % ns;
            return p.tpo + (static_cast<int64_t>(sp) * p.Hq + g * Gq) * D + e0 + i;
        };
        u64 w[kW], ma = 0, mb = 0;
        unsigned pending = 0;
#pragma unroll
        for (int k = 0; k < kW; ++k) {
            const int j = tid + k * kCT;
            if (j < S * ns) {
                w[k] = ld_tagged1(word(j));
                pending |= 1u << k;
            }
        }
        const bool has_ml = tid < S * Gq;  // (split, head) = (tid / Gq, tid % Gq)
        auto ml_src = [&]() { return p.tpml + (static_cast<int64_t>(tid / Gq) * p.Hq + g * Gq + tid % Gq) * 2; };
        if (has_ml) {
            ld_tagged2(ml_src(), ma, mb);
            pending |= 1u << kW;
        }
        const bool ok = poll_pairs<kW + 1>(
            pending, p.status, p.status,
            [&](int k) { return k < kW ? tag_hi(w[k]) == want : (tag_hi(ma) == want && tag_hi(mb) == want); },
            [&](int k) {
                if (k < kW)
                    w[k] = ld_tagged1(word(tid + k * kCT));
                else
                    ld_tagged2(ml_src(), ma, mb);
            });
#pragma unroll
        for (int k = 0; k < kW; ++k)
            if ((pending >> k) & 1u) vals[tid + k * kCT] = tag_val(w[k]);
        if (has_ml) {
            ml[2 * tid] = tag_val(ma);
            ml[2 * tid + 1] = tag_val(mb);
        }
        if (named_sync_or(1, kCT, !ok)) return false;
        const uint32_t mine = tag(layer, PH_ATTN);
#pragma unroll 1
        for (int i = tid; i < ns; i += kCT) {
            const int hh = (e0 + i) / D;
            float M = -INFINITY;
#pragma unroll 1
            for (int sp = 0; sp < S; ++sp) M = fmaxf(M, ml[2 * (sp * Gq + hh)]);
            float lsum = 0.f, acc = 0.f;
#pragma unroll 1
            for (int sp = 0; sp < S; ++sp) {
                const float ms = ml[2 * (sp * Gq + hh)];
                const float f = (ms == -INFINITY) ? 0.f : expf(ms - M);
                if (ms != -INFINITY) lsum = fmaf(f, ml[2 * (sp * Gq + hh) + 1], lsum);
                acc = fmaf(f, vals[sp * ns + i], acc);
            }
            st_tagged(p.tao + static_cast<int64_t>(g * Gq) * D + e0 + i, acc / lsum, mine);
        }
        named_sync(1, kCT);  // sm.xs is read before the o_proj input overwrites it
        return true;
    }

};


template <int D, int GQ>
B200_DEVICE void run_step(Mk<D, GQ> &mk, const MkParams &p);

// The producer thread: streams the step's weight schedule through the ring (slot
// c % kStages for chunk c, refilled as soon as its consumer warp releases it). It
// never waits on activations, so HBM keeps streaming while the consumers wait for
// other CTAs' outputs; 16 slots of 12 KB per SM keep enough bytes in flight.
// Every wait is bounded and abandoned on error.
B200_DEVICE void produce(const MkParams &p, const Smem &sm, int b, int G) {
    const uint64_t pol = policy_evict_first();
    Cursor cp;
    bool live = cp.start(p, b, G, 0);
    int cc = 0, landed = 0;  // chunks issued / chunks known to have landed
#pragma unroll 1
    while (live) {
        // At most max_inflight copies outstanding: enough bytes in flight for this
        // SM's share of HBM bandwidth, and no deeper queue in front of the
        // consumers' own latency-critical loads (activations, KV rows).
#pragma unroll 1
        while (cc - landed >= p.max_inflight) {
            if (!mbar_wait_bounded(&sm.full[landed % kStages], (landed / kStages) & 1, p.status)) {
                live = false;
                break;
            }
            ++landed;
        }
        if (!live) break;
        const int s = cc % kStages;
        // (a consumer that stopped leaves its slot unreleased: the wait sees the
        // status word then; no per-chunk global load on the issue path)
        if (cc >= kStages && !mbar_wait_bounded(&sm.empty[s], ((cc / kStages) - 1) & 1, p.status)) break;
        const uint32_t bytes = cp.bytes();
        mbar_arrive_expect_tx(&sm.full[s], bytes);
        bulk_g2s(sm.ring + static_cast<size_t>(s) * kStageFloats, cp.src(), bytes, &sm.full[s], pol);
        ++cc;
        live = cp.advance(p, b, G, 1);
    }
    // Before leaving, wait (bounded) for the copies still in flight into this
    // CTA's shared memory: the last min(cc, kStages) issued chunks.
#pragma unroll 1
    for (int c = max(0, cc - kStages); c < cc; ++c) mbar_wait_bounded(&sm.full[c % kStages], (c / kStages) & 1, nullptr);
}

template <int D, int GQ>
__global__ void __launch_bounds__(kThreads, 1) decode_mk_kernel(const MkParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ uint32_t s_tag0;
    Smem sm;
    sm.full = reinterpret_cast<uint64_t *>(smem_raw);
    sm.empty = sm.full + kStages;
    sm.ring = reinterpret_cast<float *>(smem_raw + 256);
    sm.xs = sm.ring + kStages * kStageFloats;
    sm.part = sm.xs + kMaxK;
    sm.qs = sm.part + kPartFloats;
    sm.res = sm.qs + kMaxGq * D;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x, G = gridDim.x;
    if (tid < PH_PER_LAYER) {  // this CTA's geometry of the four projections and the LM head
        const PhaseW pw = phase_w(p, tid == kGeoLm ? p.n_layer : 0, tid);
        int64_t r0 = 0, r1 = 0;
        rows_of(pw.N, pw.unit, b, G, r0, r1);
        const int rpc = rpc_for(pw.K, pw.unit);
        s_geo[tid] = Geo{static_cast<int>(r0), static_cast<int>(r1), rpc, static_cast<int>((r1 - r0 + rpc - 1) / rpc)};
    }
    if (tid == 0) {
        // every CTA of every launch takes one ticket: launch = ticket / G
        const unsigned long long ticket = atomicAdd(p.launches, 1ull);
        const unsigned long long launch = ticket / static_cast<unsigned long long>(G);
        s_tag0 = static_cast<uint32_t>(launch % kMkTagPeriod + 1ull) * kTagStride;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);  // the one warp that reads the slot's chunk
        }
        fence_barrier_init();
    }
    {
        constexpr int kWords = sizeof(MkLayer) / 8;
        static_assert(sizeof(MkLayer) % 8 == 0, "layer table copied in 8-byte words");
        const unsigned long long *src = reinterpret_cast<const unsigned long long *>(p.layers);
        unsigned long long *dst = reinterpret_cast<unsigned long long *>(s_layers);
#pragma unroll 1
        for (int i = tid; i < p.n_layer * kWords; i += kThreads) dst[i] = src[i];
    }
    __syncthreads();

    if (warp >= kCW) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProdRegs));
        if (warp == kCW && lane == 0) produce(p, sm, b, G);
        return;
    }
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsRegs));
    Mk<D, GQ> mk{p, sm, tid, warp, lane, b, G, s_tag0};
    run_step<D, GQ>(mk, p);
}

template <int D, int GQ>
B200_DEVICE void run_step(Mk<D, GQ> &mk, const MkParams &p) {
    const int tid = mk.tid, warp = mk.warp, lane = mk.lane, b = mk.b, G = mk.G;
    int cc = 0;
    const int64_t n_past = *p.n_past;
    const int32_t token = *p.token;
    // test hook, normally -1: CTA withhold[0] - 1 withholds its layer-0 QKV outputs
    // once withhold[1] more launches have passed (that CTA counts them down)
    __shared__ int s_withheld;
    if (tid == 0) {
        int w = -1;
        if (p.withhold && p.withhold[0] - 1 == b) {
            const int skip = p.withhold[1];
            if (skip > 0)
                p.withhold[1] = skip - 1;
            else
                w = b;
        }
        s_withheld = w;
    }
    bool ok = true;
    if (n_past < 0 || n_past >= p.n_ctx) {
        if (tid == 0) set_status(p.status, B200_DEV_BAD_POSITION);
        ok = false;
    }
    if (token < 0 || token >= p.V) {  // V == vocabulary on one GPU
        if (tid == 0) set_status(p.status, B200_DEV_BAD_TOKEN);
        ok = false;
    }
    const float *emb = p.tok_embd + static_cast<int64_t>(ok ? token : 0) * p.H;
    int64_t r0 = 0, r1 = 0;
    {
        // The o_proj and down phases own the same H rows per CTA: their residual
        // stays in shared memory from phase to phase (layer 0: the embedding).
        rows_of(p.H, 1, b, G, r0, r1);
#pragma unroll 1
        for (int64_t r = r0 + tid; r < r1; r += kCT) mk.sm.res[r - r0] = __ldg(emb + r);
    }
    mk.rope_table(ok ? n_past : 0);
    named_sync(1, kCT);
    const int withheld = s_withheld;
    // One pass over the step's phases (per layer QKV, attention, o_proj, gate/up,
    // down; then the LM head), each helper called from exactly one place so that
    // the kernel's code stays small enough for the instruction cache.
    const int n_ph = p.n_layer * PH_PER_LAYER + 1;
    for (int q = 0; q < n_ph && ok; ++q) {
        const int l = q / PH_PER_LAYER, ph = q % PH_PER_LAYER;
        stamp(p, q, 3);
        if (ph == PH_ATTN) {
            ok = mk.attention(l, n_past);
            stamp(p, q, 5);
            stamp(p, q, 2);
            continue;
        }
        const PhaseW pw = phase_w(p, l, ph);
        const Geo &gm = s_geo[geo_index(p, l, ph)];
        r0 = gm.r0;
        r1 = gm.r1;
        // phase input
        if (ph == PH_O) {
            ok = mk.load_act(p.tao, static_cast<int64_t>(p.Hq) * p.D, nullptr, mk.tag(l, PH_ATTN));
        } else if (q == 0) {
            mk.load_act_plain(emb, p.H, s_layers[0].attn_norm);
        } else {
            const bool lm = l == p.n_layer;
            const u64 *src = ph == PH_DOWN ? p.th : p.tx;
            const int64_t K = ph == PH_DOWN ? p.F : p.H;
            const float *gamma = lm ? p.out_norm
                                    : ph == PH_QKV ? s_layers[l].attn_norm : ph == PH_GU ? s_layers[l].ffn_norm : nullptr;
            const uint32_t want = lm || ph == PH_QKV ? mk.tag(l - 1, PH_DOWN) : mk.tag(l, ph == PH_GU ? PH_O : PH_GU);
            ok = mk.load_act(src, K, gamma, want);
        }
        if (!ok) break;
        stamp(p, q, 4);
        const bool lm_phase = l == p.n_layer;
        const uint32_t mine = lm_phase ? 0u : mk.tag(l, ph);
        // QKV / o_proj / down rows are published by the warp that computed them; the
        // gate / up pairs of a SwiGLU row may sit in two chunks: after the barrier
        u64 *early = (lm_phase || ph == PH_GU || (ph == PH_QKV && l == 0 && b == withheld)) ? nullptr
                     : ph == PH_QKV                                                       ? p.tqkv
                                                                                          : p.tx;
        ok = mk.consume(pw, gm, cc, q, early, mine, ph != PH_QKV);
        if (lm_phase) break;  // LM head: the argmax below
        if (ph == PH_GU) {
#pragma unroll 1
            for (int64_t pr = r0 / 2 + tid; pr < r1 / 2; pr += kCT) {
                const float gt = mk.row_sum(2 * pr - r0), up = mk.row_sum(2 * pr + 1 - r0);
                const float sg = gt / (1.0f + expf(-gt));
                st_tagged(p.th + pr, up * sg, mine);
            }
        }
        stamp(p, q, 5);
        stamp(p, q, 2);
    }
    // uniform: threads that read the status word at different times must not
    // split between returning and the argmax's barriers below
    if (named_sync_or(1, kCT, !ok || status_set(p.status) != 0)) return;
    const int lm = p.n_layer * PH_PER_LAYER;

    // ---- LM head greedy argmax over the row sums (first maximum; NaN / +inf -> -1)
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    bool bad = false;
#pragma unroll 1
    for (int64_t r = r0 + tid; r < r1; r += kCT) {  // per thread: increasing rows
        const float v = mk.row_sum(r - r0);
        if (p.logits) p.logits[r] = v;
        if (isnan(v) || v == INFINITY) bad = true;
        if (v > bv) {
            bv = v;
            bi = r;
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
    __shared__ float s_bv[kCW];
    __shared__ int64_t s_bi[kCW];
    __shared__ int s_bad[kCW];
    __shared__ unsigned s_ticket;
    if (lane == 0) {
        s_bv[warp] = bv;
        s_bi[warp] = bi;
        s_bad[warp] = bad;
    }
    named_sync(1, kCT);
    if (tid == 0) {
        float v = s_bv[0];
        int64_t i = s_bi[0];
        bool anyb = s_bad[0];
#pragma unroll 1
        for (int w = 1; w < kCW; ++w) {
            anyb |= s_bad[w] != 0;
            if (s_bv[w] > v || (s_bv[w] == v && s_bi[w] < i)) {
                v = s_bv[w];
                i = s_bi[w];
            }
        }
        p.am_val[b] = anyb ? NAN : v;
        p.am_idx[b] = anyb ? -2 : (i == INT64_MAX ? -1 : static_cast<int32_t>(i));
        __threadfence();
        s_ticket = atomicAdd(p.am_counter, 1u);
    }
    named_sync(1, kCT);
    stamp(p, lm, 5);
    if (s_ticket != static_cast<unsigned>(G - 1)) return;
    if (tid == 0) {
        __threadfence();
        float v = -INFINITY;
        int32_t id = -1;
        bool anyb = false;
#pragma unroll 1
        for (int c = 0; c < G; ++c) {  // CTAs own increasing row ranges
            const float cv = __ldcg(p.am_val + c);
            const int32_t ci = __ldcg(p.am_idx + c);
            if (ci == -2) anyb = true;
            if (cv > v) {
                v = cv;
                id = ci;
            }
        }
        if (anyb || id < 0) {
            id = -1;
            set_status(p.status, B200_DEV_BAD_LOGITS);
        }
        *p.token = id;
        if (p.token_log) {
            const int32_t q = *p.log_pos;
            p.token_log[q % p.log_cap] = id;
            *p.log_pos = q + 1;
        }
        *p.n_past = static_cast<int32_t>(n_past + 1);
        *p.am_counter = 0u;
        stamp(p, lm, 2);
    }
}

size_t smem_bytes(int D) {
    return 256 + static_cast<size_t>(kStages) * kStageFloats * 4 + static_cast<size_t>(kMaxK) * 4 +
           static_cast<size_t>(kPartFloats) * 4 + static_cast<size_t>(kMaxGq) * D * 4 +
           static_cast<size_t>(kResFloats) * 4;
}

}  // namespace

int mk_grid() { return device_sm_count(); }

// The instantiated (head_dim, query heads per KV head) pairs: the Qwen3 shapes
// (head_dim 128 with 1, 2 or 4 query heads per KV head) and head_dim 64 with 2.
static void *mk_kernel(int D, int gq) {
    if (D == 128 && gq == 1) return reinterpret_cast<void *>(decode_mk_kernel<128, 1>);
    if (D == 128 && gq == 2) return reinterpret_cast<void *>(decode_mk_kernel<128, 2>);
    if (D == 128 && gq == 4) return reinterpret_cast<void *>(decode_mk_kernel<128, 4>);
    if (D == 64 && gq == 2) return reinterpret_cast<void *>(decode_mk_kernel<64, 2>);
    return nullptr;
}

// Ring copies in flight per CTA (B200_MK_INFLIGHT overrides the default).
int mk_max_inflight() {
    static int v = -1;
    if (v < 0) {
        const char *e = std::getenv("B200_MK_INFLIGHT");
        const int x = (e && *e) ? std::atoi(e) : kDefaultInflight;
        v = std::min(std::max(x, 1), kStages);
    }
    return v;
}

// Keys per attention split (B200_MK_SPLIT_KEYS overrides the default).
int mk_split_keys() {
    static int v = -1;
    if (v < 0) {
        const char *e = std::getenv("B200_MK_SPLIT_KEYS");
        const int x = (e && *e) ? std::atoi(e) : kDefaultSplitKeys;
        v = std::min(std::max(x, 8), 1024);
    }
    return v;
}

int mk_max_splits() { return kMaxSplits; }
size_t mk_po_words(const MkParams &p) { return static_cast<size_t>(kMaxSplits) * p.Hq * p.D; }
size_t mk_pml_words(const MkParams &p) { return static_cast<size_t>(kMaxSplits) * p.Hq * 2; }

bool mk_supported(const MkParams &p) {
    if (p.D != 64 && p.D != 128) return false;
    if (p.n_layer < 1 || p.n_layer > kMaxLayers) return false;
    if (p.Hkv <= 0 || p.Hq % p.Hkv || !mk_kernel(p.D, p.Hq / p.Hkv)) return false;
    // attention scratch: kCW x Gq sub-range partials in xs + part below the new k/v
    if (kCW * (p.Hq / p.Hkv) * (p.D + 2) > kMaxK + kPartFloats - 2 * p.D) return false;
    const int G = mk_grid();
    if (p.Hkv > G) return false;
    if ((p.H + G - 1) / G > kResFloats) return false;  // residual rows per CTA
    // 32-bit row-range arithmetic (rows_of)
    const int64_t nmax = std::max<int64_t>({static_cast<int64_t>(p.V), 2 * static_cast<int64_t>(p.F),
                                            static_cast<int64_t>(p.Hq + 2 * p.Hkv) * p.D});
    if (nmax * (G + 1) >= (1LL << 32)) return false;
    // split merge in the attention CTAs (merge_group): one (split, head) pair and
    // kW = 3 slice words per thread; scratch in sm.xs
    const int Gq = p.Hq / p.Hkv;
    if (kMaxSplits * Gq > kCT || Gq * p.D + kMaxSplits > 3 * kCT || 2 * kMaxSplits * Gq > kMaxK / 2) return false;
    if (p.D / 2 > kMaxHalfD) return false;
    const int64_t Ks[] = {p.H, static_cast<int64_t>(p.Hq) * p.D, p.F};
    for (int64_t K : Ks)
        if (K > kMaxK || (K & 3) || K < 64) return false;
    // every projection: a chunk fits one ring stage, the per-CTA row sums fit sm.part
    const int64_t Ns[] = {static_cast<int64_t>(p.Hq + 2 * p.Hkv) * p.D, p.H, 2 * static_cast<int64_t>(p.F), p.H, p.V};
    const int64_t Kof[] = {p.H, static_cast<int64_t>(p.Hq) * p.D, p.H, p.F, p.H};
    const int units[] = {1, 1, 2, 1, 1};
    for (int i = 0; i < 5; ++i) {
        const int rpc = rpc_for(Kof[i], units[i]);
        if (rpc < 1 || rpc > kMaxRpc || static_cast<int64_t>(rpc) * Kof[i] > kStageFloats) return false;
        const int64_t rows = ((Ns[i] / units[i] + G - 1) / G) * units[i] + 1;
        if (rows > kPartFloats) return false;
    }
    return true;
}

cudaError_t mk_launch(const MkParams &p, cudaStream_t stream) {
    const size_t smem = smem_bytes(p.D);
    void *kern = p.Hkv > 0 ? mk_kernel(p.D, p.Hq / p.Hkv) : nullptr;
    if (!kern) return cudaErrorInvalidValue;
    // Per device and cheap: the launch is recorded once into the decode graph.
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    MkParams args = p;
    args.max_inflight = mk_max_inflight();
    args.split_keys = mk_split_keys();
    void *kargs[] = {&args};
    return cudaLaunchCooperativeKernel(kern, dim3(mk_grid()), dim3(kThreads), kargs, smem, stream);
}

}  // namespace b200
