// GQA attention over a paged KV cache: K and V live in fixed-size blocks of
// `block_tokens` tokens, found through per-sequence tables of block pointers.
//
// This is the kernel side of a paged KV strategy (KVCacheConfig::block_tokens > 0,
// include/kvcache/kvutil.hpp:43-44, resolved by KVStrategy::lookup into one slice
// per block): a block is a KV storage object with the NaiveKVStorage layout
// (naiveKVStorage.cpp:28-40) and capacity block_tokens -- element (token t of the
// block, KV head h, dim d) at block[(t * Hkv + h) * D + d] -- so the reference's
// own block objects can be passed as they are, in any order and at any addresses.
//
//  * paged_kv_write_kernel: the K / V rows of T new tokens into their blocks.
//  * attn_decode_paged_kernel: one query token. CTA (split s, KV head h) takes keys
//    [L s / SE, L (s + 1) / SE) of the G query heads of h; each warp owns four keys
//    of every 32-key batch (lane l: dims [E l, E l + E)), with the next batch's K /
//    V rows loaded into registers while the current one is scored (online softmax
//    per warp and head); the warps merge in order; with one split the CTA writes the
//    output, otherwise the split partials merge through the workspace in the CTA
//    that finishes last for its KV head (split order: deterministic).
//  * Tq > 1 (prefill over a paged cache): the [0, Tkv) rows are gathered into the
//    workspace and the tiled prefill kernel runs on them.
#include "attention.cuh"
#include "gemv.cuh"

namespace b200 {
namespace {

constexpr int kPgThreads = 256;
constexpr int kPgWarps = kPgThreads / 32;
constexpr int kPgKeys = 4;                    // keys per warp per batch
constexpr int kPgBatch = kPgKeys * kPgWarps;  // 32 keys per CTA batch
constexpr int kPgKeysPerSplit = 128;
constexpr int kPgTab = 256;                   // block pointers a split stages in shared memory

struct PagedArgs {
    const float *q = nullptr;                  // [Hq][D] (one token)
    const float *const *kb = nullptr;          // [n_blocks] device pointers to K blocks
    const float *const *vb = nullptr;          // [n_blocks] V blocks
    int64_t n_blocks = 0, bt = 0;              // blocks, tokens per block
    float *out = nullptr;                      // [Hq][D]
    int64_t Hq = 0, Hkv = 0, L = 0;            // L = keys (n_past + 1)
    float scale = 0.f;
    void *ws = nullptr;                        // counters [round_up(Hkv, 64)] u32, then split records
    int32_t *status = nullptr;
};

B200_HOST_DEVICE size_t pg_counter_words(int64_t Hkv) { return static_cast<size_t>((Hkv + 63) / 64 * 64); }

int pg_splits(int64_t L, int64_t Hkv) {
    int64_t s = (L + kPgKeysPerSplit - 1) / kPgKeysPerSplit;
    s = min64(s, max64(1, device_sm_count() / max64(1, Hkv)));
    return static_cast<int>(max64(1, s));
}

template <int E>
B200_DEVICE void load_row(const float *p, float (&v)[E]) {
    if constexpr (E == 4) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
    } else {
        static_assert(E == 2, "head_dim 64 or 128");
        const float2 t = __ldg(reinterpret_cast<const float2 *>(p));
        v[0] = t.x, v[1] = t.y;
    }
}

template <int D, int G>
__global__ void __launch_bounds__(kPgThreads) attn_decode_paged_kernel(const PagedArgs a, const int S) {
    constexpr int E = D / 32;
    constexpr int WR = G * (D + 2);  // one warp's (o, m, l) record
    __shared__ float wp[kPgWarps * WR];
    __shared__ const float *s_kb[kPgTab];
    __shared__ const float *s_vb[kPgTab];
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x;
    const int64_t kvh = blockIdx.y;
    const int64_t L = a.L;
    const int SE = static_cast<int>(min64(S, max64(1, (L + kPgKeysPerSplit - 1) / kPgKeysPerSplit)));
    if (s >= SE) return;
    const int64_t j0 = L * s / SE, j1 = L * (s + 1) / SE;
    const int64_t tok = a.Hkv * D;  // token stride inside a block
    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf(static_cast<float>(D));

    float q[G][E], o[G][E], m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            q[g][e] = a.q[(kvh * G + g) * D + E * lane + e];
            o[g][e] = 0.f;
        }
    }
    bool bad = false;
    // The split's block pointers, staged in shared memory once (a row load then
    // needs no dependent global load of its block's address); a split spanning more
    // than kPgTab blocks reads the rest from the tables.
    const int64_t b0 = j0 / a.bt, nb = (j1 - 1) / a.bt - b0 + 1;
    for (int64_t i = tid; i < min64(nb, kPgTab); i += kPgThreads) {
        s_kb[i] = a.kb[b0 + i];
        s_vb[i] = a.vb[b0 + i];
    }
    __syncthreads();
    // K / V rows of this warp's keys of the batch at `base` (zeros past j1)
    auto load = [&](int64_t base, float (&kv)[kPgKeys][E], float (&vv)[kPgKeys][E]) {
#pragma unroll
        for (int u = 0; u < kPgKeys; ++u) {
            const int64_t j = base + kPgKeys * warp + u;
            const float *kp = nullptr, *vp = nullptr;
            if (j < j1) {
                const int64_t blk = j / a.bt, off = j - blk * a.bt;
                kp = blk - b0 < kPgTab ? s_kb[blk - b0] : a.kb[blk];
                vp = blk - b0 < kPgTab ? s_vb[blk - b0] : a.vb[blk];
                if (!kp || !vp) {
                    bad = true;
                    kp = vp = nullptr;
                } else {
                    kp += off * tok + kvh * D + E * lane;
                    vp += off * tok + kvh * D + E * lane;
                }
            }
            if (kp) {
                load_row<E>(kp, kv[u]);
                load_row<E>(vp, vv[u]);
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) kv[u][e] = vv[u][e] = 0.f;
            }
        }
    };
    float kc[kPgKeys][E], vc[kPgKeys][E], kn[kPgKeys][E], vn[kPgKeys][E];
    load(j0, kc, vc);
#pragma unroll 1
    for (int64_t base = j0; base < j1; base += kPgBatch) {
        if (base + kPgBatch < j1) load(base + kPgBatch, kn, vn);  // next batch in flight
        float sc[kPgKeys][G];
#pragma unroll
        for (int u = 0; u < kPgKeys; ++u)
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < E; ++e) d = fmaf(q[g][e], kc[u][e], d);
                sc[u][g] = d;
            }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < kPgKeys; ++u)
#pragma unroll
                for (int g = 0; g < G; ++g) sc[u][g] += __shfl_xor_sync(0xffffffffu, sc[u][g], off);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mn = m[g];
#pragma unroll
            for (int u = 0; u < kPgKeys; ++u) {
                sc[u][g] = (base + kPgKeys * warp + u < j1) ? sc[u][g] * scale : -INFINITY;
                mn = fmaxf(mn, sc[u][g]);
            }
            if (mn == -INFINITY) continue;  // no key of this warp in the batch
            const float al = (m[g] == -INFINITY) ? 0.f : expf(m[g] - mn);
            l[g] *= al;
#pragma unroll
            for (int e = 0; e < E; ++e) o[g][e] *= al;
#pragma unroll
            for (int u = 0; u < kPgKeys; ++u) {
                if (base + kPgKeys * warp + u < j1) {
                    const float pr = expf(sc[u][g] - mn);
                    l[g] += pr;
#pragma unroll
                    for (int e = 0; e < E; ++e) o[g][e] = fmaf(pr, vc[u][e], o[g][e]);
                }
            }
            m[g] = mn;
        }
#pragma unroll
        for (int u = 0; u < kPgKeys; ++u)
#pragma unroll
            for (int e = 0; e < E; ++e) {
                kc[u][e] = kn[u][e];
                vc[u][e] = vn[u][e];
            }
    }
    if (bad && lane == 0) set_status(a.status, B200_DEV_BAD_POSITION);
    // the warps' (m, l, o) -> this split's partial, warps merged in order
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < E; ++e) wp[warp * WR + g * D + E * lane + e] = o[g][e];
        if (lane == 0) {
            wp[warp * WR + G * D + g] = m[g];
            wp[warp * WR + G * D + G + g] = l[g];
        }
    }
    __syncthreads();
    const size_t rec = static_cast<size_t>(G) * (D + 2);  // per (kvh, split): o [G][D], m [G], l [G]
    float *ws = static_cast<float *>(a.ws) + pg_counter_words(a.Hkv);
    float *mine = ws + (static_cast<size_t>(kvh) * S + s) * rec;
    for (int i = tid; i < G * D; i += kPgThreads) {
        const int g = i / D;
        float M = -INFINITY;
        for (int w = 0; w < kPgWarps; ++w) M = fmaxf(M, wp[w * WR + G * D + g]);
        float lsum = 0.f, os = 0.f;
        for (int w = 0; w < kPgWarps; ++w) {
            const float mw = wp[w * WR + G * D + g];
            if (mw == -INFINITY) continue;
            const float f = expf(mw - M);
            lsum = fmaf(f, wp[w * WR + G * D + G + g], lsum);
            os = fmaf(f, wp[w * WR + i], os);
        }
        if (SE == 1) {
            a.out[(kvh * G) * D + i] = os / lsum;
            continue;
        }
        mine[i] = os;
        if (i % D == 0) {
            mine[G * D + g] = M;
            mine[G * D + G + g] = lsum;
        }
    }
    if (SE == 1) return;
    __threadfence();
    __syncthreads();
    unsigned *cnt = static_cast<unsigned *>(a.ws);
    if (tid == 0) s_last = atomicInc(cnt + kvh, static_cast<unsigned>(SE - 1)) == static_cast<unsigned>(SE - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float *all = ws + static_cast<size_t>(kvh) * S * rec;
    for (int i = tid; i < G * D; i += kPgThreads) {
        const int g = i / D;
        float M = -INFINITY;
        for (int r = 0; r < SE; ++r) M = fmaxf(M, __ldcg(all + r * rec + G * D + g));
        float lsum = 0.f, acc = 0.f;
        for (int r = 0; r < SE; ++r) {
            const float ms = __ldcg(all + r * rec + G * D + g);
            if (ms == -INFINITY) continue;
            const float f = expf(ms - M);
            lsum = fmaf(f, __ldcg(all + r * rec + G * D + G + g), lsum);
            acc = fmaf(f, __ldcg(all + r * rec + i), acc);
        }
        a.out[(kvh * G) * D + i] = acc / lsum;
    }
}

// Rows of T tokens ([T][Hkv][D] with token stride src_ld) into their blocks at
// positions pos0 .. pos0 + T - 1; a missing block records B200_DEV_BAD_POSITION.
__global__ void paged_kv_write_kernel(const float *k_src, const float *v_src, int64_t src_ld, float *const *kb,
                                      float *const *vb, int64_t bt, int64_t pos0, int64_t T, int64_t HD,
                                      int32_t *status) {
    const int64_t n4 = T * (HD / 4);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const int64_t t = i / (HD / 4), c = (i - t * (HD / 4)) * 4;
        const int64_t pos = pos0 + t, blk = pos / bt, off = pos - blk * bt;
        float *kd = kb[blk], *vd = vb[blk];
        if (!kd || !vd) {
            set_status(status, B200_DEV_BAD_POSITION);
            continue;
        }
        *reinterpret_cast<float4 *>(kd + off * HD + c) = *reinterpret_cast<const float4 *>(k_src + t * src_ld + c);
        *reinterpret_cast<float4 *>(vd + off * HD + c) = *reinterpret_cast<const float4 *>(v_src + t * src_ld + c);
    }
}

// Rows [0, Tkv) of the paged cache into contiguous [Tkv][Hkv][D] K and V.
__global__ void paged_gather_kernel(const float *const *kb, const float *const *vb, int64_t bt, int64_t Tkv,
                                    int64_t HD, float *k_out, float *v_out, int32_t *status) {
    const int64_t n4 = Tkv * (HD / 4);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const int64_t t = i / (HD / 4), c = (i - t * (HD / 4)) * 4;
        const int64_t blk = t / bt, off = t - blk * bt;
        const float *ks = kb[blk], *vs = vb[blk];
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
        if (ks && vs) {
            kv = __ldg(reinterpret_cast<const float4 *>(ks + off * HD + c));
            vv = __ldg(reinterpret_cast<const float4 *>(vs + off * HD + c));
        } else {
            set_status(status, B200_DEV_BAD_POSITION);
        }
        *reinterpret_cast<float4 *>(k_out + t * HD + c) = kv;
        *reinterpret_cast<float4 *>(v_out + t * HD + c) = vv;
    }
}

template <int D, int G>
cudaError_t paged_decode_launch(const PagedArgs &a, int S, cudaStream_t st) {
    return b200_launch(attn_decode_paged_kernel<D, G>, dim3(S, static_cast<unsigned>(a.Hkv)), dim3(kPgThreads), 0,
                       st, false, a, S);
}

template <int D>
cudaError_t paged_decode_by_g(const PagedArgs &a, int S, cudaStream_t st) {
    switch (a.Hq / a.Hkv) {
        case 1: return paged_decode_launch<D, 1>(a, S, st);
        case 2: return paged_decode_launch<D, 2>(a, S, st);
        case 4: return paged_decode_launch<D, 4>(a, S, st);
        case 8: return paged_decode_launch<D, 8>(a, S, st);
    }
    return cudaErrorNotSupported;
}

int grid_for(int64_t n4) { return static_cast<int>(min64(max64(1, (n4 + 255) / 256), 4 * device_sm_count())); }

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int b200_paged_kv_write(const float *k_src, const float *v_src, int64_t src_tok_stride, float *const *k_blocks,
                        float *const *v_blocks, int64_t n_blocks, int64_t block_tokens, int64_t pos0, int64_t T,
                        int64_t Hkv, int64_t D, int32_t *dev_status, void *stream) {
    if (T < 0 || pos0 < 0 || Hkv <= 0 || D <= 0 || block_tokens <= 0 || n_blocks <= 0) return B200_ERR_INVALID_ARGUMENT;
    if (T == 0) return B200_OK;
    if (!k_src || !v_src || !k_blocks || !v_blocks || ((Hkv * D) & 3) || (src_tok_stride & 3) ||
        src_tok_stride < Hkv * D)
        return B200_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(k_src) | reinterpret_cast<uintptr_t>(v_src)) & 15) return B200_ERR_INVALID_ARGUMENT;
    if (pos0 + T > n_blocks * block_tokens) return B200_ERR_OUT_OF_RANGE;
    const int64_t n4 = T * (Hkv * D / 4);
    paged_kv_write_kernel<<<grid_for(n4), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        k_src, v_src, src_tok_stride, k_blocks, v_blocks, block_tokens, pos0, T, Hkv * D, dev_status);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

size_t b200_flash_attn_paged_workspace_bytes(int64_t D, int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tkv) {
    if (D <= 0 || Hkv <= 0 || Hq % Hkv || Tq < 0 || Tkv < 0) return 0;
    if (Tq > 1) return align256(static_cast<size_t>(Tkv) * Hkv * D * 4) * 2;
    const int S = pg_splits(Tkv, Hkv);
    return (pg_counter_words(Hkv) + static_cast<size_t>(Hkv) * S * (Hq / Hkv) * (D + 2)) * 4;
}

int b200_flash_attn_paged(const float *q, const float *const *k_blocks, const float *const *v_blocks, int64_t n_blocks,
                          int64_t block_tokens, float *out, int64_t D, int64_t Hq, int64_t Hkv, int64_t Tq,
                          int64_t Tkv, int64_t n_past, float scale, void *workspace, size_t workspace_bytes,
                          int32_t *dev_status, void *stream) {
    if (!q || !k_blocks || !v_blocks || !out || D <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Tq < 0 || n_past < 0 ||
        block_tokens <= 0 || n_blocks <= 0)
        return B200_ERR_INVALID_ARGUMENT;
    if (Tkv != n_past + Tq) return B200_ERR_INVALID_ARGUMENT;
    if (Tq == 0) return B200_OK;
    if (D != 64 && D != 128) return B200_ERR_NOT_SUPPORTED;
    if (Tkv > n_blocks * block_tokens) return B200_ERR_OUT_OF_RANGE;
    if (!workspace || workspace_bytes < b200_flash_attn_paged_workspace_bytes(D, Hq, Hkv, Tq, Tkv))
        return B200_ERR_INVALID_ARGUMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (Tq == 1) {
        PagedArgs a;
        a.q = q;
        a.kb = k_blocks;
        a.vb = v_blocks;
        a.n_blocks = n_blocks;
        a.bt = block_tokens;
        a.out = out;
        a.Hq = Hq;
        a.Hkv = Hkv;
        a.L = Tkv;
        a.scale = scale;
        a.ws = workspace;
        a.status = dev_status;
        const int S = pg_splits(Tkv, Hkv);
        const cudaError_t e = D == 128 ? paged_decode_by_g<128>(a, S, st) : paged_decode_by_g<64>(a, S, st);
        return e == cudaSuccess ? B200_OK : (e == cudaErrorNotSupported ? B200_ERR_NOT_SUPPORTED : B200_ERR_CUDA);
    }
    // prefill over the paged cache: gather, then the tiled kernel
    float *kc = static_cast<float *>(workspace);
    float *vc = reinterpret_cast<float *>(static_cast<char *>(workspace) + align256(static_cast<size_t>(Tkv) * Hkv * D * 4));
    const int64_t n4 = Tkv * (Hkv * D / 4);
    paged_gather_kernel<<<grid_for(n4), 256, 0, st>>>(k_blocks, v_blocks, block_tokens, Tkv, Hkv * D, kc, vc, dev_status);
    if (cudaGetLastError() != cudaSuccess) return B200_ERR_CUDA;
    AttnArgs a;
    a.q = q;
    a.k = kc;
    a.v = vc;
    a.out = out;
    a.k_tok = Hkv * D;
    a.k_head = D;
    a.v_tok = Hkv * D;
    a.v_head = D;
    a.D = D;
    a.Hq = Hq;
    a.Hkv = Hkv;
    a.Tq = Tq;
    a.n_past = n_past;
    a.scale = scale;
    const cudaError_t e = attn_prefill_launch(a, st, false);
    return e == cudaSuccess ? B200_OK : (e == cudaErrorNotSupported ? B200_ERR_NOT_SUPPORTED : B200_ERR_CUDA);
}

}  // extern "C"
