// GQA causal attention for sm_100a over the reference's token-major KV cache
// (element (t, h, d) at base + t*tok_stride + h*head_stride + d; the reference's
// NaiveKVStorage object is K block then V block, naiveKVStorage.cpp:28-40).
//
// Semantics follow CPUBackend::compute_flash_attn (cpu_backend.cpp:555-632):
// key j is visible to query i iff j <= n_past + i, kv_head = q_head / (Hq/Hkv),
// softmax over the visible keys, out = sum p_j v_j. The softmax here is the
// online (flash) form: same math, different rounding order.
#include <algorithm>

#include "attention.cuh"
#include "gemv.cuh"
#include "tma.cuh"
#include "rope.cuh"

namespace b200 {
namespace {

constexpr int kDecThreads = 128;
constexpr int kDecTile = 32;

// Split-KV flash decoding for one query token. CTA (s, kvh) covers keys
// [L*s/S, L*(s+1)/S) of KV head kvh for its G query heads, in 32-key tiles
// (double-buffered cp.async), with an online softmax. The S CTAs of a KV head
// are one thread-block cluster; rank 0 merges the S partial (m, l, o) triples in
// split order through distributed shared memory.
//
// Fused prologue (a.qkv set): q/k come raw from the QKV projection; the CTA
// applies the per-head RMSNorm + RoPE to its q heads and the CTA holding
// position n_past also normalises/rotates k, appends k and v to the cache and
// patches that row into its shared-memory tile directly.
template <int D, int G>
__global__ void __launch_bounds__(2 * kDecThreads) attn_decode_kernel(const AttnArgs a, const int S) {
    // one warp per query head in the score step: 8 warps when G > 4
    constexpr int kDecThreads = G > 4 ? 2 * b200::kDecThreads : b200::kDecThreads;
    constexpr int LD = D + 4;
    constexpr int DPT = (D + kDecThreads - 1) / kDecThreads;  // dims per thread
    extern __shared__ __align__(16) float sm[];
    float *Ks = sm;                            // [2][32][LD]
    float *Vs = Ks + 2 * kDecTile * LD;        // [2][32][LD]
    float *qs = Vs + 2 * kDecTile * LD;        // [G][D]
    float *knew = qs + G * D;                  // [D] new token's k (normed, rotated)
    float *vnew = knew + D;                    // [D] new token's v
    float *P = vnew + D;                       // [G][32]
    float *alpha_s = P + G * kDecTile;         // [G], then pm [G], pl [G], po [G][D]

    const TraceMark tm(a.trace);
    grid_launch_dependents();
    prefetch_share_l2(a.next_w, a.next_w_bytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x;
    const int64_t kvh = blockIdx.y;
    const bool fused = a.qkv != nullptr;

    // n_past is final before this kernel starts when early_kv is set (see attention.cuh)
    if (!a.early_kv) grid_wait();
    const int64_t n_past = a.n_past_dev ? static_cast<int64_t>(*a.n_past_dev) : a.n_past;
    const int64_t L = n_past + 1;  // keys 0..n_past are visible to the single query
    const int64_t j0 = L * s / S, j1 = L * (s + 1) / S;
    const bool last = (s == S - 1);  // holds key n_past
    const int ntiles = static_cast<int>((j1 - j0 + kDecTile - 1) / kDecTile);
    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf(static_cast<float>(D));
    // In fused mode row n_past is produced by this kernel: it is zero-filled by the
    // tile load and patched from knew / vnew.
    const int64_t jload = fused ? min64(j1, n_past) : j1;

    const float *kb = a.k + kvh * a.k_head;
    const float *vb = a.v + kvh * a.v_head;
    auto load_tile = [&](int t, int buf) {
        const int64_t base = j0 + static_cast<int64_t>(t) * kDecTile;
        constexpr int C4 = D / 4;
        for (int i = tid; i < kDecTile * C4; i += kDecThreads) {
            const int r = i / C4, c = i % C4;
            const int64_t j = base + r;
            const bool ok = j < jload;
            const int64_t jj = ok ? j : 0;
            cp_async16_zfill(Ks + (buf * kDecTile + r) * LD + c * 4, kb + jj * a.k_tok + c * 4, ok);
            cp_async16_zfill(Vs + (buf * kDecTile + r) * LD + c * 4, vb + jj * a.v_tok + c * 4, ok);
        }
        cp_async_commit();
    };
    // cached keys stream in while the previous kernel finishes
    if (ntiles > 0) load_tile(0, 0);
    if (ntiles > 1) load_tile(1, 1);

    if (a.early_kv) grid_wait();
    tm.waited();
    if (fused) {
        if (n_past >= a.n_ctx) {
            if (tid == 0) set_status(a.status, B200_DEV_BAD_POSITION);
            cp_async_wait<0>();
            return;
        }
        const int jobs = G + (last ? 2 : 0);
        for (int h = warp; h < jobs; h += kDecThreads / 32) {
            if (h < G) {
                warp_norm_rope_head<D / 32>(a.qkv + (kvh * G + h) * D, a.q_gamma, a.freq, n_past, a.eps,
                                            qs + h * D);
            } else if (h == G) {
                warp_norm_rope_head<D / 32>(a.qkv + (a.Hq + kvh) * D, a.k_gamma, a.freq, n_past, a.eps, knew);
                __syncwarp();
                float *kdst = const_cast<float *>(a.k) + n_past * a.k_tok + kvh * a.k_head;
                for (int d = lane; d < D; d += 32) kdst[d] = knew[d];
            } else {
                const float *vsrc = a.qkv + (a.Hq + a.Hkv + kvh) * D;
                float *vdst = const_cast<float *>(a.v) + n_past * a.v_tok + kvh * a.v_head;
                for (int d = lane; d < D; d += 32) {
                    const float v = vsrc[d];
                    vnew[d] = v;
                    vdst[d] = v;
                }
            }
        }
    } else {
        for (int i = tid; i < G * D; i += kDecThreads) qs[i] = a.q[(kvh * G) * D + i];
    }
    __syncthreads();
    tm.at(4);

    float m_run = -INFINITY, l_run = 0.f;  // valid in warp g (< G), replicated over lanes
    float acc[G][DPT];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < DPT; ++e) acc[g][e] = 0.f;

    for (int t = 0; t < ntiles; ++t) {
        const int buf = t & 1;
        if (t + 1 < ntiles) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();
        const int64_t tbase = j0 + static_cast<int64_t>(t) * kDecTile;
        if (fused && last && n_past >= tbase && n_past < tbase + kDecTile) {
            const int r = static_cast<int>(n_past - tbase);
            for (int d = tid; d < D; d += kDecThreads) {
                Ks[(buf * kDecTile + r) * LD + d] = knew[d];
                Vs[(buf * kDecTile + r) * LD + d] = vnew[d];
            }
            __syncthreads();
        }
        if (warp < G) {
            const int64_t j = tbase + lane;
            const bool valid = j < j1;
            const float *kr = Ks + (buf * kDecTile + lane) * LD;
            const float *qr = qs + warp * D;
            float dot = 0.f;
#pragma unroll 8
            for (int k = 0; k < D; k += 4) {
                const float4 kv = *reinterpret_cast<const float4 *>(kr + k);
                const float4 qv = *reinterpret_cast<const float4 *>(qr + k);
                dot = fmaf(qv.x, kv.x, dot);
                dot = fmaf(qv.y, kv.y, dot);
                dot = fmaf(qv.z, kv.z, dot);
                dot = fmaf(qv.w, kv.w, dot);
            }
            const float sc = valid ? dot * scale : -INFINITY;
            const float m_new = fmaxf(m_run, warp_max(sc));
            const float p = valid ? expf(sc - m_new) : 0.f;
            const float al = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
            l_run = l_run * al + warp_sum(p);
            m_run = m_new;
            P[warp * kDecTile + lane] = p;
            if (lane == 0) alpha_s[warp] = al;
        }
        __syncthreads();
#pragma unroll
        for (int e = 0; e < DPT; ++e) {
            const int d = tid + e * kDecThreads;
            if (d < D) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float o = acc[g][e] * alpha_s[g];
                    const float *pg = P + g * kDecTile;
#pragma unroll 8
                    for (int c = 0; c < kDecTile; ++c) o = fmaf(pg[c], Vs[(buf * kDecTile + c) * LD + d], o);
                    acc[g][e] = o;
                }
            }
        }
        __syncthreads();
        if (t + 2 < ntiles) load_tile(t + 2, buf);
    }
    tm.at(5);

    // Partials stay in this CTA's shared memory; the S CTAs of a KV head form one
    // thread-block cluster and rank 0 merges them through distributed shared
    // memory, in split order, between two cluster barriers.
    float *pm = alpha_s + G;        // [G] running max
    float *pl = pm + G;             // [G] running sum
    float *po = pl + G;             // [G][D] unnormalised output
    if (warp < G && lane == 0) {
        pm[warp] = m_run;
        pl[warp] = l_run;
    }
#pragma unroll
    for (int e = 0; e < DPT; ++e) {
        const int d = tid + e * kDecThreads;
        if (d < D)
#pragma unroll
            for (int g = 0; g < G; ++g) po[g * D + d] = acc[g][e];
    }
    cluster_sync();
    if (s == 0) {
#pragma unroll
        for (int e = 0; e < DPT; ++e) {
            const int d = tid + e * kDecThreads;
            if (d >= D) continue;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float M = -INFINITY;
                for (int r = 0; r < S; ++r) M = fmaxf(M, ld_dsmem(dsmem_addr(pm + g, r)));
                float lsum = 0.f, o = 0.f;
                for (int r = 0; r < S; ++r) {
                    const float ms = ld_dsmem(dsmem_addr(pm + g, r));
                    if (ms == -INFINITY) continue;
                    const float f = expf(ms - M);
                    lsum = fmaf(f, ld_dsmem(dsmem_addr(pl + g, r)), lsum);
                    o = fmaf(f, ld_dsmem(dsmem_addr(po + g * D + d, r)), o);
                }
                a.out[(kvh * G + g) * D + d] = o / lsum;
            }
        }
    }
    cluster_sync();  // peers keep their shared memory until rank 0 has read it
    tm.done();
}

// ---------------------------------------------------------------------------
// Split-KV flash decoding with TMA-staged K/V tiles. CTA (s, kvh) covers keys
// [L*s/S, L*(s+1)/S) of KV head kvh for its G query heads:
//   * warp 8, one lane (loader): per 32-key tile two tiled TMA loads, K and V, each
//     a [32 positions][D] box of the cache viewed as a 3-D tensor {D, Hkv, positions}
//     (the head's rows are Hkv * D floats apart), into a kNS-stage ring, the stage's
//     mbarrier expecting both boxes; it runs kNS tiles ahead. (One bulk copy per
//     512-byte row instead costs ~2 us per tile in copy-engine operations.)
//   * warps 0..7: warp w owns keys 4w..4w+3 of every tile with its own online
//     softmax (lane l: dimensions [l*D/32, (l+1)*D/32) of q, K, V and the output;
//     scores reduced across the warp by xor shuffles), so no CTA barrier is taken
//     per tile; a stage goes back to the loader once all eight warps have read
//     their rows. The warps' (m, l, o) are merged in warp order at the end.
// The S partial (m, l, o) of every CTA go to the workspace; the CTA that finishes
// last for its KV head (wrap-around atomic counter, left at zero) merges them in
// split order, so the result does not depend on which CTA was last.
// Fused prologue (a.qkv set): as attn_decode_kernel.
constexpr int kD2Compute = 256;
constexpr int kD2Threads = kD2Compute + 32;
constexpr int kD2Tile = 32;
constexpr int kD2KeysPerSplit = 128;  // keys a split takes (four tiles)

template <int D>
struct D2Cfg {
    static constexpr int LD = D;                                     // dense rows, as the TMA box lands
    static constexpr int kNS = D <= 128 ? 4 : 2;                     // stages
    static constexpr int kStageFloats = 2 * kD2Tile * LD;            // K box then V box
};

B200_HOST_DEVICE int64_t d2_counter_words(int64_t Hkv) { return (Hkv + 15) / 16 * 16; }

template <int D, int G>
size_t d2_smem_bytes() {
    using C = D2Cfg<D>;
    return 128 + static_cast<size_t>(C::kNS) * C::kStageFloats * 4 + (G * D + 2 * D) * sizeof(float);
}

// Bounded mbarrier wait: false (status set) after ~2 s or once another CTA reported an error.
B200_DEVICE bool d2_wait(uint64_t *bar, uint32_t parity, int32_t *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
#pragma unroll 1
    for (uint32_t i = 0; i < B200_SPIN_LIMIT; ++i) {
        // plain try_wait polls: the thread resumes as soon as the phase completes
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255) {
            if (status && *reinterpret_cast<volatile int32_t *>(status)) return false;
            if (global_ns() - t0 > 2000000000ull) break;
        }
    }
    set_status(status, B200_DEV_TIMEOUT);
    return false;
}

template <int D, int G>
__global__ void __launch_bounds__(kD2Threads, 1)
    attn_decode_tma_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                           const AttnArgs a, const int S) {
    using C = D2Cfg<D>;
    constexpr int LD = C::LD, NS = C::kNS;
    static_assert(D % 32 == 0 && kD2Tile % (kD2Compute / 32) == 0, "thread mapping");
    static_assert(NS * C::kStageFloats >= (kD2Compute / 32) * G * (D + 2), "warp partials fit the ring");
    extern __shared__ __align__(128) unsigned char d2_raw[];
    uint64_t *full = reinterpret_cast<uint64_t *>(d2_raw), *empty = full + NS;
    float *ring = reinterpret_cast<float *>(d2_raw + 128);  // [NS][K rows | V rows][LD]
    float *qs = ring + NS * C::kStageFloats;                // [G][D]
    float *knew = qs + G * D, *vnew = knew + D;             // new token's k (normed, rotated), v
    __shared__ int s_last, s_fail;

    const TraceMark tm(a.trace);
    grid_launch_dependents();
    prefetch_share_l2(a.next_w, a.next_w_bytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x;
    const int64_t kvh = blockIdx.y;
    const bool fused = a.qkv != nullptr;
    int32_t *status = a.status;

    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kD2Compute / 32);
        }
        fence_barrier_init();
        s_fail = 0;
    }
    __syncthreads();

    // n_past is final before this kernel starts when early_kv is set (see attention.cuh)
    if (!a.early_kv) grid_wait();
    const int64_t n_past = a.n_past_dev ? static_cast<int64_t>(*a.n_past_dev) : a.n_past;
    const int64_t L = n_past + 1;
    // The grid has S splits for the longest context (the engine's graph is captured
    // once); this step uses about kD2KeysPerSplit keys per split. Splits past SE exit
    // at once, and with SE == 1 the one split writes the output itself (no workspace
    // round trip, no counter).
    const int SE = static_cast<int>(min64(S, max64(1, (L + kD2KeysPerSplit - 1) / kD2KeysPerSplit)));
    if (s >= SE) return;
    const int64_t j0 = L * s / SE, j1 = L * (s + 1) / SE;
    const bool last = (s == SE - 1);  // holds key n_past
    const int ntiles = static_cast<int>((j1 - j0 + kD2Tile - 1) / kD2Tile);
    // In fused mode row n_past is produced by this kernel: patched from knew / vnew.
    const int64_t jload = fused ? min64(j1, n_past) : j1;
    const bool bad_pos = fused && n_past >= a.n_ctx;

    if (warp == kD2Compute / 32) {
        // ---- loader: cached rows [j0, jload) never depend on the previous kernel
        // beyond n_past (early_kv), so they stream in before the dependency wait
        if (bad_pos || lane != 0) return;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
        const uint64_t pol = policy_evict_last();
        (void)jload;  // rows past jload in a box are loaded but never used (masked / patched)
#pragma unroll 1
        for (int t = 0; t < ntiles; ++t) {
            const int st = t % NS;
            if (t >= NS && !d2_wait(&empty[st], ((t / NS) - 1) & 1, status)) break;
            const int32_t base = static_cast<int32_t>(j0 + static_cast<int64_t>(t) * kD2Tile);
            const uint32_t kst = smem_addr(ring + st * C::kStageFloats);
            mbar_arrive_expect_tx(&full[st], 2u * kD2Tile * D * 4);
            tma_load_3d(kst, &tk, 0, static_cast<int32_t>(kvh), base, smem_addr(&full[st]), pol);
            tma_load_3d(kst + kD2Tile * LD * 4, &tv, 0, static_cast<int32_t>(kvh), base, smem_addr(&full[st]), pol);
        }
        return;
    }

    // ---- compute warps
    if (a.early_kv) grid_wait();
    tm.waited();
    if (bad_pos) {
        if (tid == 0) set_status(a.status, B200_DEV_BAD_POSITION);
        return;
    }
    if (fused) {
        const int jobs = G + (last ? 2 : 0);
        for (int h = warp; h < jobs; h += kD2Compute / 32) {
            if (h < G) {
                warp_norm_rope_head<D / 32>(a.qkv + (kvh * G + h) * D, a.q_gamma, a.freq, n_past, a.eps, qs + h * D);
            } else if (h == G) {
                warp_norm_rope_head<D / 32>(a.qkv + (a.Hq + kvh) * D, a.k_gamma, a.freq, n_past, a.eps, knew);
                __syncwarp();
                float *kdst = const_cast<float *>(a.k) + n_past * a.k_tok + kvh * a.k_head;
                for (int d = lane; d < D; d += 32) kdst[d] = knew[d];
            } else {
                const float *vsrc = a.qkv + (a.Hq + a.Hkv + kvh) * D;
                float *vdst = const_cast<float *>(a.v) + n_past * a.v_tok + kvh * a.v_head;
                for (int d = lane; d < D; d += 32) {
                    const float v = vsrc[d];
                    vnew[d] = v;
                    vdst[d] = v;
                }
            }
        }
    } else {
        for (int i = tid; i < G * D; i += kD2Compute) qs[i] = a.q[(kvh * G) * D + i];
    }
    named_sync(1, kD2Compute);
    tm.at(4);

    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf(static_cast<float>(D));
    // Warp w owns keys 4w .. 4w+3 of every tile with its own online softmax (no
    // CTA barrier per tile); lane l holds dimensions [E*l, E*l + E) of q and of
    // the output accumulators.
    constexpr int E = D / 32;
    constexpr int KW = kD2Tile / (kD2Compute / 32);  // keys per warp per tile
    float q[G][E], o[G][E], m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            q[g][e] = qs[g * D + E * lane + e];
            o[g][e] = 0.f;
        }
    }
    bool ok = true;

#pragma unroll 1
    for (int t = 0; t < ntiles; ++t) {
        const int st = t % NS;
        if (!d2_wait(&full[st], (t / NS) & 1, status)) {
            ok = false;
            break;
        }
        float *kst = ring + st * C::kStageFloats, *vst = kst + kD2Tile * LD;
        const int64_t base = j0 + static_cast<int64_t>(t) * kD2Tile;
        const int nrows = static_cast<int>(min64(kD2Tile, j1 - base));  // loaded + (last tile) row n_past
        const int prow = (fused && last && n_past >= base && n_past < base + kD2Tile) ? static_cast<int>(n_past - base) : -1;
        float sc[KW][G];
        float vv[KW][E];
#pragma unroll
        for (int u = 0; u < KW; ++u) {
            const int j = KW * warp + u;
            float kv[E];
            if (j == prow) {  // the new token: from shared memory, not the (stale) box row
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    kv[e] = knew[E * lane + e];
                    vv[u][e] = vnew[E * lane + e];
                }
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    kv[e] = kst[j * LD + E * lane + e];
                    vv[u][e] = vst[j * LD + E * lane + e];
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < E; ++e) d = fmaf(q[g][e], kv[e], d);
                sc[u][g] = d;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);  // the warp's rows are in registers
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < KW; ++u)
#pragma unroll
                for (int g = 0; g < G; ++g) sc[u][g] += __shfl_xor_sync(0xffffffffu, sc[u][g], off);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mn = m[g];
#pragma unroll
            for (int u = 0; u < KW; ++u) {
                sc[u][g] = (KW * warp + u < nrows) ? sc[u][g] * scale : -INFINITY;
                mn = fmaxf(mn, sc[u][g]);
            }
            if (mn == -INFINITY) continue;  // no visible key of this warp in the tile yet
            const float al = (m[g] == -INFINITY) ? 0.f : expf(m[g] - mn);
            l[g] *= al;
#pragma unroll
            for (int e = 0; e < E; ++e) o[g][e] *= al;
#pragma unroll
            for (int u = 0; u < KW; ++u) {
                if (KW * warp + u < nrows) {
                    const float pr = expf(sc[u][g] - mn);
                    l[g] += pr;
#pragma unroll
                    for (int e = 0; e < E; ++e) o[g][e] = fmaf(pr, vv[u][e], o[g][e]);
                }
            }
            m[g] = mn;
        }
    }
    tm.at(5);
    if (!__all_sync(0xffffffffu, ok)) {
        // copies the loader may still have in flight into this CTA's shared memory
        if (lane == 0)
            for (int t = 0; t < min(NS, ntiles); ++t) d2_wait(&full[t % NS], 0, nullptr);
    }
    // every compute thread reaches the barriers below (status decides afterwards)
    named_sync(1, kD2Compute);
    if (!ok) s_fail = 1;
    named_sync(1, kD2Compute);
    if (s_fail) return;

    // ---- the 8 warps' (m, l, o) -> this split's partial, warps merged in order
    float *wp = ring;  // the stages are free: every tile was consumed
    constexpr int WR = G * (D + 2);
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < E; ++e) wp[warp * WR + g * D + E * lane + e] = o[g][e];
        if (lane == 0) {
            wp[warp * WR + G * D + g] = m[g];
            wp[warp * WR + G * D + G + g] = l[g];
        }
    }
    named_sync(1, kD2Compute);
    if (SE == 1) {  // one split: the warps' merge is the output
        for (int i = tid; i < G * D; i += kD2Compute) {
            const int g = i / D;
            float M = -INFINITY;
            for (int w = 0; w < kD2Compute / 32; ++w) M = fmaxf(M, wp[w * WR + G * D + g]);
            float lsum = 0.f, os = 0.f;
            for (int w = 0; w < kD2Compute / 32; ++w) {
                const float mw = wp[w * WR + G * D + g];
                if (mw == -INFINITY) continue;
                const float f = expf(mw - M);
                lsum = fmaf(f, wp[w * WR + G * D + G + g], lsum);
                os = fmaf(f, wp[w * WR + i], os);
            }
            a.out[(kvh * G) * D + i] = os / lsum;
        }
        tm.done();
        return;
    }
    unsigned *cnt = static_cast<unsigned *>(a.ws);
    float *ws = static_cast<float *>(a.ws) + d2_counter_words(a.Hkv);
    const size_t rec = static_cast<size_t>(G) * (D + 2);  // per (kvh, split): o [G][D], m [G], l [G]
    float *mine = ws + (static_cast<size_t>(kvh) * S + s) * rec;
    for (int i = tid; i < G * D; i += kD2Compute) {
        const int g = i / D;
        float M = -INFINITY;
        for (int w = 0; w < kD2Compute / 32; ++w) M = fmaxf(M, wp[w * WR + G * D + g]);
        float lsum = 0.f, os = 0.f;
        for (int w = 0; w < kD2Compute / 32; ++w) {
            const float mw = wp[w * WR + G * D + g];
            if (mw == -INFINITY) continue;
            const float f = expf(mw - M);
            lsum = fmaf(f, wp[w * WR + G * D + G + g], lsum);
            os = fmaf(f, wp[w * WR + i], os);
        }
        mine[i] = os;
        if (i % D == 0) {
            mine[G * D + g] = M;
            mine[G * D + G + g] = lsum;
        }
    }
    __threadfence();
    named_sync(1, kD2Compute);
    if (tid == 0) s_last = atomicInc(cnt + kvh, static_cast<unsigned>(SE - 1)) == static_cast<unsigned>(SE - 1);
    named_sync(1, kD2Compute);
    if (s_last) {
        __threadfence();
        const float *all = ws + static_cast<size_t>(kvh) * S * rec;
        for (int i = tid; i < G * D; i += kD2Compute) {
            const int g = i / D;
            float M = -INFINITY;
            for (int r = 0; r < SE; ++r) M = fmaxf(M, __ldcg(all + r * rec + G * D + g));
            float lsum = 0.f, o = 0.f;
            for (int r = 0; r < SE; ++r) {
                const float ms = __ldcg(all + r * rec + G * D + g);
                if (ms == -INFINITY) continue;
                const float f = expf(ms - M);
                lsum = fmaf(f, __ldcg(all + r * rec + G * D + G + g), lsum);
                o = fmaf(f, __ldcg(all + r * rec + i), o);
            }
            a.out[(kvh * G) * D + i] = o / lsum;
        }
    }
    tm.done();
}

// ---------------------------------------------------------------------------
constexpr int kPreThreads = 256;
constexpr int kRows = 64;   // query rows (token, head) per CTA
constexpr int kKeys = 64;   // keys per tile

// Prefill / multi-token attention: a CTA owns 64 query rows (BQ = 64/G tokens x
// the G query heads of one KV head), streams 64-key K and V tiles (cp.async; V
// loads overlap QK^T, the next K tile overlaps PV) and keeps an online softmax
// per row. Tiles beyond the causal limit of the block are skipped; the heaviest
// blocks are scheduled first.
template <int D, int G>
__global__ void __launch_bounds__(kPreThreads, 1) attn_prefill_kernel(const AttnArgs a) {
    constexpr int LD = D + 4;
    constexpr int BQ = kRows / G;       // query tokens per CTA
    constexpr int DV = D / 16;          // output dims per thread (8 for D=128)
    constexpr int PLD = kKeys + 4;
    extern __shared__ __align__(16) float sm[];
    float *Qs = sm;                     // [64][LD]
    float *Ks = Qs + kRows * LD;        // [64][LD]
    float *Vs = Ks + kKeys * LD;        // [64][LD]
    float *Ps = Vs + kKeys * LD;        // [64][PLD]

    grid_launch_dependents();
    grid_wait();

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    // one CTA per (query block, KV head), the heaviest query blocks (most keys under
    // the causal mask) of every head first: the first wave takes the longest CTAs
    const int64_t nqb = gridDim.x / a.Hkv;
    const int64_t qb = nqb - 1 - blockIdx.x / a.Hkv;
    const int64_t kvh = blockIdx.x % a.Hkv;
    const int64_t q0 = qb * BQ;
    const int64_t n_past = a.n_past_dev ? static_cast<int64_t>(*a.n_past_dev) : a.n_past;
    const int64_t Tkv = n_past + a.Tq;
    const int64_t kv_end = min64(Tkv, n_past + min64(q0 + BQ, a.Tq));
    const int ntiles = static_cast<int>((kv_end + kKeys - 1) / kKeys);
    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf(static_cast<float>(D));
    constexpr int C4 = D / 4;

    // Q rows r = tl*G + g: token q0+tl, head kvh*G+g (the G heads are contiguous)
    for (int i = tid; i < kRows * C4; i += kPreThreads) {
        const int r = i / C4, c = i % C4;
        const int64_t tok = q0 + r / G;
        const bool ok = tok < a.Tq;
        const float *src = a.q + ((ok ? tok : 0) * a.Hq + kvh * G + (r % G)) * D + c * 4;
        cp_async16_zfill(Qs + r * LD + c * 4, src, ok);
    }
    const float *kb = a.k + kvh * a.k_head;
    const float *vb = a.v + kvh * a.v_head;
    auto load_kv = [&](float *dst, const float *base, int64_t tok_stride, int t) {
        for (int i = tid; i < kKeys * C4; i += kPreThreads) {
            const int r = i / C4, c = i % C4;
            const int64_t j = static_cast<int64_t>(t) * kKeys + r;
            const bool ok = j < kv_end;
            cp_async16_zfill(dst + r * LD + c * 4, base + (ok ? j : 0) * tok_stride + c * 4, ok);
        }
        cp_async_commit();
    };

    float m_run[4], l_run[4], o[4][DV];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m_run[i] = -INFINITY;
        l_run[i] = 0.f;
#pragma unroll
        for (int e = 0; e < DV; ++e) o[i][e] = 0.f;
    }
    int64_t qpos[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) qpos[i] = n_past + q0 + (ty + 16 * i) / G;

    if (ntiles > 0) load_kv(Ks, kb, a.k_tok, 0);  // commits Q + K0 together
    for (int t = 0; t < ntiles; ++t) {
        load_kv(Vs, vb, a.v_tok, t);
        cp_async_wait<1>();
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
        for (int k = 0; k < D; k += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4 *>(Qs + (ty + 16 * i) * LD + k);
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4 *>(Ks + (tx + 16 * j) * LD + k);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sc[i][j] = fmaf(qv[i].x, kv[j].x, sc[i][j]);
                    sc[i][j] = fmaf(qv[i].y, kv[j].y, sc[i][j]);
                    sc[i][j] = fmaf(qv[i].z, kv[j].z, sc[i][j]);
                    sc[i][j] = fmaf(qv[i].w, kv[j].w, sc[i][j]);
                }
        }
        float alpha[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t kpos = static_cast<int64_t>(t) * kKeys + tx + 16 * j;
                const bool vis = kpos <= qpos[i] && kpos < Tkv;
                sc[i][j] = vis ? sc[i][j] * scale : -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run[i], mx);
            float rs = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = (sc[i][j] == -INFINITY) ? 0.f : expf(sc[i][j] - m_new);
                sc[i][j] = p;
                rs += p;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            alpha[i] = (m_run[i] == -INFINITY) ? 0.f : expf(m_run[i] - m_new);
            l_run[i] = l_run[i] * alpha[i] + rs;
            m_run[i] = m_new;
#pragma unroll
            for (int j = 0; j < 4; ++j) Ps[(ty + 16 * i) * PLD + tx + 16 * j] = sc[i][j];
#pragma unroll
            for (int e = 0; e < DV; ++e) o[i][e] *= alpha[i];
        }
        __syncthreads();  // Ks free, Ps complete
        const bool more = t + 1 < ntiles;
        if (more) load_kv(Ks, kb, a.k_tok, t + 1);
        if (more) cp_async_wait<1>(); else cp_async_wait<0>();
        __syncthreads();  // Vs ready
#pragma unroll 4
        for (int c = 0; c < kKeys; ++c) {
            float4 v0 = *reinterpret_cast<const float4 *>(Vs + c * LD + tx * 4);
            float4 v1 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (DV == 8) v1 = *reinterpret_cast<const float4 *>(Vs + c * LD + 64 + tx * 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float p = Ps[(ty + 16 * i) * PLD + c];
                o[i][0] = fmaf(p, v0.x, o[i][0]);
                o[i][1] = fmaf(p, v0.y, o[i][1]);
                o[i][2] = fmaf(p, v0.z, o[i][2]);
                o[i][3] = fmaf(p, v0.w, o[i][3]);
                if (DV == 8) {
                    o[i][4 % DV] = fmaf(p, v1.x, o[i][4 % DV]);
                    o[i][5 % DV] = fmaf(p, v1.y, o[i][5 % DV]);
                    o[i][6 % DV] = fmaf(p, v1.z, o[i][6 % DV]);
                    o[i][7 % DV] = fmaf(p, v1.w, o[i][7 % DV]);
                }
            }
        }
        __syncthreads();  // Vs / Ps reused next tile
    }
    cp_async_wait<0>();

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = ty + 16 * i;
        const int64_t tok = q0 + r / G;
        if (tok >= a.Tq) continue;
        float *dst = a.out + (tok * a.Hq + kvh * G + (r % G)) * D;
        const float inv = 1.0f / l_run[i];
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[tx * 4 + e] = o[i][e] * inv;
        if (DV == 8)
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[64 + tx * 4 + e] = o[i][(4 + e) % DV] * inv;
    }
}

template <int D, int G>
cudaError_t dec_launch(const AttnArgs &a, int S, cudaStream_t stream, bool pdl) {
    const size_t smem =
        (4 * kDecTile * (D + 4) + G * D + 2 * D + G * kDecTile + G + 2 * G + G * D) * sizeof(float);
    auto kern = attn_decode_kernel<D, G>;
    {
        const cudaError_t e = once_per_device(reinterpret_cast<const void *>(kern), ATTR_SMEM, [&] {
            cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (r == cudaSuccess) r = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         cudaSharedmemCarveoutMaxShared);
            return r;
        });
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, static_cast<unsigned>(a.Hkv));
    cfg.blockDim = dim3(G > 4 ? 2 * kDecThreads : kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, a, S);
}

// The K (or V) cache as a 3-D tensor {D, Hkv, rows} (strides in floats: head, token),
// boxes of one head x 32 positions.
bool d2_map(CUtensorMap *m, const float *base, int64_t D, int64_t Hkv, int64_t rows, int64_t head, int64_t tok) {
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Hkv), static_cast<uint64_t>(rows)};
    const uint64_t strides[2] = {static_cast<uint64_t>(head) * 4, static_cast<uint64_t>(tok) * 4};
    const uint32_t box[3] = {static_cast<uint32_t>(D), 1, static_cast<uint32_t>(kD2Tile)};
    return tma_encode_f32(m, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int D, int G>
cudaError_t d2_launch(const AttnArgs &a, int S, cudaStream_t stream, bool pdl) {
    const size_t smem = d2_smem_bytes<D, G>();
    auto kern = attn_decode_tma_kernel<D, G>;
    {
        const cudaError_t e = once_per_device(reinterpret_cast<const void *>(kern), ATTR_SMEM, [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        });
        if (e != cudaSuccess) return e;
    }
    // positions the maps cover: the cache capacity (engine) or the keys of this call
    const int64_t rows = a.kv_rows > 0 ? a.kv_rows : a.n_past + 1;
    CUtensorMap tk, tv;
    if (!d2_map(&tk, a.k, D, a.Hkv, rows, a.k_head, a.k_tok) || !d2_map(&tv, a.v, D, a.Hkv, rows, a.v_head, a.v_tok))
        return cudaErrorNotSupported;
    return b200_launch(kern, dim3(S, static_cast<unsigned>(a.Hkv)), dim3(kD2Threads), smem, stream, pdl, tk, tv, a, S);
}

template <int D, int G>
cudaError_t pre_launch(const AttnArgs &a, cudaStream_t stream, bool pdl) {
    constexpr int BQ = kRows / G;
    const size_t smem = ((kRows + 2 * kKeys) * (D + 4) + kRows * (kKeys + 4)) * sizeof(float);
    auto kern = attn_prefill_kernel<D, G>;
    {
        const cudaError_t e = once_per_device(reinterpret_cast<const void *>(kern), ATTR_SMEM, [&] {
            return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        });
        if (e != cudaSuccess) return e;
    }
    const dim3 grid(static_cast<unsigned>(((a.Tq + BQ - 1) / BQ) * a.Hkv));
    return b200_launch(kern, grid, dim3(kPreThreads), smem, stream, pdl, a);
}

template <int D, int G>
cudaError_t dec_one(const AttnArgs &a, int S, bool tma, cudaStream_t st, bool pdl) {
    if constexpr (G * D <= 1024) {  // per-warp accumulators of G heads x D/32 dims fit the registers
        if (tma) return d2_launch<D, G>(a, S, st, pdl);
    }
    return dec_launch<D, G>(a, std::min(S, 16), st, pdl);
}

template <int D>
cudaError_t dec_by_g(const AttnArgs &a, int S, cudaStream_t st, bool pdl) {
    // the TMA-staged kernel needs the split workspace; without one, the cluster
    // kernel (at most 16 splits) merges through distributed shared memory
    const bool tma = a.ws && a.ws_bytes >= attn_decode_ws_bytes(D, a.Hq, a.Hkv, S);
    switch (a.Hq / a.Hkv) {
        case 1: return dec_one<D, 1>(a, S, tma, st, pdl);
        case 2: return dec_one<D, 2>(a, S, tma, st, pdl);
        case 4: return dec_one<D, 4>(a, S, tma, st, pdl);
        case 8: return dec_one<D, 8>(a, S, tma, st, pdl);
    }
    return cudaErrorInvalidValue;
}

template <int D>
cudaError_t pre_by_g(const AttnArgs &a, cudaStream_t st, bool pdl) {
    switch (a.Hq / a.Hkv) {
        case 1: return pre_launch<D, 1>(a, st, pdl);
        case 2: return pre_launch<D, 2>(a, st, pdl);
        case 4: return pre_launch<D, 4>(a, st, pdl);
        case 8: return pre_launch<D, 8>(a, st, pdl);
    }
    return cudaErrorInvalidValue;
}

bool strides_ok(const AttnArgs &a) {
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return a.Hkv > 0 && a.Hq % a.Hkv == 0 && (a.k_tok & 3) == 0 && (a.k_head & 3) == 0 &&
           (a.v_tok & 3) == 0 && (a.v_head & 3) == 0 && al(a.q ? a.q : a.qkv) && al(a.k) && al(a.v);
}

}  // namespace

int attn_decode_splits(int64_t max_len, int64_t Hkv) {
    // About kD2KeysPerSplit keys (four tiles) per split, at most one CTA per SM over all KV heads.
    int64_t s = (max_len + kD2KeysPerSplit - 1) / kD2KeysPerSplit;
    const int64_t cap = std::max<int64_t>(1, device_sm_count() / std::max<int64_t>(1, Hkv));
    s = std::min(s, cap);
    return static_cast<int>(std::max<int64_t>(1, s));
}

size_t attn_decode_ws_bytes(int64_t D, int64_t Hq, int64_t Hkv, int splits) {
    if (D <= 0 || Hkv <= 0 || Hq % Hkv || splits < 1) return 0;
    const size_t rec = static_cast<size_t>(Hq / Hkv) * (D + 2);
    return (static_cast<size_t>(d2_counter_words(Hkv)) + static_cast<size_t>(Hkv) * splits * rec) * 4;
}

cudaError_t attn_decode_launch(const AttnArgs &a, int splits, cudaStream_t stream, bool pdl) {
    if (!strides_ok(a) || a.Tq != 1 || splits < 1 || splits > 1024) return cudaErrorInvalidValue;
    switch (a.D) {
        case 64: return dec_by_g<64>(a, splits, stream, pdl);
        case 128: return dec_by_g<128>(a, splits, stream, pdl);
        case 256: return dec_by_g<256>(a, splits, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

cudaError_t attn_prefill_launch(const AttnArgs &a, cudaStream_t stream, bool pdl) {
    if (!strides_ok(a) || a.Tq < 1) return cudaErrorInvalidValue;
    if (a.precision == 1 && a.D == 128) {  // B200_PREC_TF32
        const cudaError_t e = attn_prefill_tc_launch(a, stream, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    switch (a.D) {
        case 64: return pre_by_g<64>(a, stream, pdl);
        case 128: return pre_by_g<128>(a, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace b200
