// GQA causal attention over a token-major KV cache.
#pragma once

#include "common.cuh"

namespace b200 {

struct AttnArgs {
    const float *q = nullptr;   // [Tq][Hq][D]
    const float *k = nullptr;   // element (t, h, d) at k[t*k_tok + h*k_head + d]
    const float *v = nullptr;
    float *out = nullptr;       // [Tq][Hq][D]
    int64_t k_tok = 0, k_head = 0, v_tok = 0, v_head = 0;
    int64_t D = 0, Hq = 0, Hkv = 0, Tq = 0;
    int64_t n_past = 0;                  // host value, used when n_past_dev is null
    int64_t kv_rows = 0;                 // positions the K/V buffers hold (0: n_past + 1)
    const int32_t *n_past_dev = nullptr; // device scalar (graph-replayed decode)
    float scale = 0.f;
    int precision = 0;                   // B200_PREC_TF32: prefill on the tensor cores (head_dim 128)
    void *ws = nullptr;                  // decode split partials + counters
    size_t ws_bytes = 0;
    int32_t *status = nullptr;
    // Fused decode prologue (Tq == 1): when qkv is set, q/k/v of the new token are
    // read raw from the QKV projection [Hq*D | Hkv*D | Hkv*D]; every CTA applies the
    // per-head RMSNorm + RoPE to its q heads, and the CTA whose split holds position
    // n_past also normalises/rotates k and appends k and v to the cache (k, v must
    // then be writable cache pointers).
    const float *qkv = nullptr;
    const float *q_gamma = nullptr, *k_gamma = nullptr, *freq = nullptr;
    float eps = 0.f;
    int64_t n_ctx = 0;                   // positions >= n_ctx are rejected (status)
    unsigned long long *trace = nullptr;  // optional step trace slot (common.cuh)
    // The launch before this one signals its dependents only after its own wait
    // (GemvArgs::late_launch): n_past and the cached K/V rows [0, n_past) are then
    // complete when this kernel starts and are read before its dependency wait.
    bool early_kv = false;
    // Weights of the next kernel, prefetched into L2 by this kernel's CTAs.
    const void *next_w = nullptr;
    size_t next_w_bytes = 0;
};

// Decode (Tq == 1): fixed `splits` x Hkv CTAs, each a slice of [0, n_past+1),
// merged in-kernel by the last CTA of each KV head. With a workspace of at least
// attn_decode_ws_bytes(...) the K/V tiles are staged by bulk copies and the split
// partials merged through it; its counters (the last Hkv words) must be zero before
// the first launch and every completed launch leaves them zero. Without one, at
// most 16 splits form a thread-block cluster and merge in distributed shared memory.
int attn_decode_splits(int64_t max_len, int64_t Hkv);
size_t attn_decode_ws_bytes(int64_t D, int64_t Hq, int64_t Hkv, int splits);
cudaError_t attn_decode_launch(const AttnArgs &a, int splits, cudaStream_t stream, bool pdl);

// Prefill / multi-token (Tq >= 1): tiled online softmax, causal tile skipping;
// precision B200_PREC_TF32 with head_dim 128 runs attn_prefill_tc_launch.
cudaError_t attn_prefill_launch(const AttnArgs &a, cudaStream_t stream, bool pdl);
// Tensor-core (tcgen05 kind::tf32) prefill, head_dim 128, G = Hq / Hkv in {1, 2, 4, 8};
// cudaErrorNotSupported where its tensor maps cannot be built.
cudaError_t attn_prefill_tc_launch(const AttnArgs &a, cudaStream_t stream, bool pdl);

}  // namespace b200
