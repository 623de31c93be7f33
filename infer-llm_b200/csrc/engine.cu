// Qwen3 F32 inference engine for one B200 (or one tensor-parallel rank).
//
// It executes the per-step graph of Qwen3Model::build_graph (Qwen3.cpp:4-136)
// as a fixed sequence of fused sm_100a kernels over device-resident arenas that
// are sized once at creation (weights, KV cache, activations, workspaces), so no
// step allocates, copies the RoPE table or synchronizes mid-step:
//
//   decode (per layer): [RMSNorm+QKV GEMV] [QK-norm+RoPE+KV append]
//                       [split-KV attention + merge] [o_proj GEMV + residual]
//                       [RMSNorm+gate/up GEMV+SwiGLU] [down GEMV + residual]
//   then [final RMSNorm + LM head GEMV + greedy argmax (+ n_past advance)].
//   The first layer's QKV GEMV gathers the embedding row itself.
//
// The decode step reads the token and n_past from device memory and writes the
// next token back, so it is captured once as a CUDA graph and replayed with no
// host round trip (under tensor parallelism with the NCCL all-reduces and the
// token all-gather inside the graph). Prefill uses the tiled FFMA / tcgen05 GEMMs and the tiled
// attention kernel over all prompt rows and samples from the last row only.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "attention.cuh"
#include "decode_mk.cuh"
#include "elementwise.cuh"
#include "engine_tp.cuh"
#include "gemm.cuh"
#include "gemv.cuh"

using namespace b200;

namespace {

struct LayerW {
    float *attn_norm = nullptr, *wqkv = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    float *wo = nullptr, *ffn_norm = nullptr, *wgu = nullptr, *wdown = nullptr;
    float *kc = nullptr, *vc = nullptr;  // KV object: K block [cap][Hkv][D], V block
};

inline int from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return B200_OK;
    if (e == cudaErrorMemoryAllocation) return B200_ERR_NO_MEMORY;
    if (e == cudaErrorInvalidValue) return B200_ERR_INVALID_ARGUMENT;
    if (e == cudaErrorNotSupported) return B200_ERR_NOT_SUPPORTED;
    return B200_ERR_CUDA;
}

#define B200_TRY(expr)                               \
    do {                                             \
        const cudaError_t _e = (expr);               \
        if (_e != cudaSuccess) return from_cuda(_e); \
    } while (0)

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3",
// SC'11) keyed by the seed; counter = (element index, tensor id).
__device__ __forceinline__ uint4 philox(uint4 c, uint2 k) {
    constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
        const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += W0;
        k.y += W1;
    }
    return c;
}

// out[i] = std * N(0,1) via Box-Muller on two Philox words.
__global__ void fill_normal_kernel(float *out, int64_t n, uint64_t seed, uint32_t tensor_id, float std) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint4 r = philox(make_uint4(static_cast<uint32_t>(i), static_cast<uint32_t>(i >> 32), tensor_id, 0u),
                               make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32)));
        const float u1 = (static_cast<float>(r.x >> 8) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
        const float u2 = static_cast<float>(r.y >> 8) * (1.0f / 16777216.0f);
        out[i] = std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
}

__global__ void fill_value_kernel(float *out, int64_t n, float v) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = v;
}

}  // namespace

struct b200_engine {
    b200_qwen3_config c{};
    int device = 0;
    cudaStream_t stream = nullptr;
    int H = 0, D = 0, Hq = 0, Hkv = 0, F = 0, V = 0;   // per-rank sizes (Hq, Hkv, F, V sharded)
    int64_t vocab_off = 0;                              // first vocab row of this rank's LM head
    int qkv_rows = 0;
    // arenas
    unsigned char *w_arena = nullptr, *kv_arena = nullptr, *act_arena = nullptr;
    size_t w_bytes = 0, kv_bytes = 0, act_bytes = 0;
    std::vector<LayerW> L;
    float *tok_embd = nullptr, *out_norm = nullptr, *lm_head = nullptr, *freq = nullptr;
    // activations
    float *x = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr;
    float *logits = nullptr;
    int32_t *ids = nullptr, *token = nullptr, *n_past_dev = nullptr, *status = nullptr;
    int32_t *token_log = nullptr, *log_pos = nullptr;
    int32_t log_cap = 0;
    void *attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    int attn_splits = 1;
    float *am_val = nullptr;
    int32_t *am_idx = nullptr;
    unsigned *am_counter = nullptr;
    float *gemm_ws = nullptr;  // split-K partials of the prefill GEMMs
    int64_t gemm_ws_floats = 0;
    int am_slots = 0;  // per-CTA argmax partials of the LM head GEMV (+1 local winner slot)
    float *tp_pairs = nullptr;  // [world][2] (value, index) for the vocab-sharded argmax
    // state
    int64_t n_past = 0;
    std::vector<std::string> missing;
    bool finalized = false;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    bool graph_logits = false;
    b200_tp *tp = nullptr;
    int32_t *pinned_io = nullptr;  // pinned host buffer: [max_batch] step ids, then the sampled token
    int64_t io_tok = 0;            // index of the token slot in pinned_io (past the ids, 64-byte aligned)
    // device-side step trace (b200_engine_trace_step): 8 x u64 per launch
    unsigned long long *trace_buf = nullptr;
    int trace_cap = 0, trace_n = 0;
    bool trace_on = false;
    // per-op timing (b200_engine_profile_step): an event is recorded after each launch
    std::vector<cudaEvent_t> *prof_events = nullptr;
    std::vector<const char *> *prof_names = nullptr;
    // single-launch decode step (decode_mk.cu)
    bool use_mk = false;
    MkParams mk;
    MkLayer *mk_layers = nullptr;  // device table
    // the step's tagged exchange words (one contiguous range of the activation
    // arena), cleared with the launch counter before kMkClearEvery launches have run
    unsigned char *mk_words = nullptr;
    size_t mk_words_bytes = 0;
    long long mk_since_clear = 0;
};

namespace {

inline cudaError_t mark(b200_engine *e, const char *name, cudaError_t launched) {
    if (launched != cudaSuccess || !e->prof_events) return launched;
    cudaEvent_t ev;
    cudaError_t err = cudaEventCreate(&ev);
    if (err != cudaSuccess) return err;
    e->prof_events->push_back(ev);
    e->prof_names->push_back(name);
    return cudaEventRecord(ev, e->stream);
}

inline unsigned long long *next_trace(b200_engine *e) {
    if (!e->trace_on || e->trace_n >= e->trace_cap) return nullptr;
    return e->trace_buf + 8 * (e->trace_n++);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

bool parse_layer(const char *name, int *layer, const char **rest) {
    if (std::strncmp(name, "blk.", 4) != 0) return false;
    char *end = nullptr;
    const long v = std::strtol(name + 4, &end, 10);
    if (end == name + 4 || *end != '.') return false;
    *layer = static_cast<int>(v);
    *rest = end + 1;
    return true;
}

// One decode step (M tokens at most 4, all from device memory) on e->stream.
// `first_ids`: device ids for the embedding gather of layer 0.
int enqueue_small_step(b200_engine *e, const int32_t *first_ids, int M, bool want_logits, int n_past_add,
                       bool pdl) {
    cudaStream_t st = e->stream;
    const int H = e->H, D = e->D;
    // Weights streamed by decode launch idx (per layer: qkv, attention, o, gate/up,
    // down; then the LM head). Launch i prefetches launch i+2's weights into L2.
    auto wspan = [&](int idx) -> std::pair<const void *, size_t> {
        const int nl = e->c.n_layer;
        if (M != 1) return {nullptr, 0};
        if (idx >= 5 * nl) {  // an LM-head prefix (the rest streams in its own kernel)
            const size_t lm = static_cast<size_t>(e->V) * H * 4, part = size_t(48) << 20;
            const size_t off = (idx == 5 * nl) ? 0 : part;
            if (off >= lm) return {nullptr, 0};
            return {reinterpret_cast<const char *>(e->lm_head) + off, std::min(part, lm - off)};
        }
        const LayerW &lw = e->L[idx / 5];
        switch (idx % 5) {
            case 0: return {lw.wqkv, static_cast<size_t>(e->qkv_rows) * H * 4};
            case 2: return {lw.wo, static_cast<size_t>(H) * e->Hq * D * 4};
            case 3: return {lw.wgu, static_cast<size_t>(2) * e->F * H * 4};
            case 4: return {lw.wdown, static_cast<size_t>(H) * e->F * 4};
        }
        return {nullptr, 0};
    };
    for (int l = 0; l < e->c.n_layer; ++l) {
        const LayerW &w = e->L[l];
        GemvArgs g;
        g.w = w.wqkv;
        g.K = H;
        g.N = e->qkv_rows;
        g.M = M;
        g.gamma = w.attn_norm;
        g.eps = e->c.rms_eps;
        g.out = e->qkv;
        g.epi = GEMV_STORE;
        g.status = e->status;
        g.late_launch = (M == 1);  // lets the decode attention read n_past / cached K,V early
        if (l == 0) {
            g.embed_table = e->tok_embd;
            g.embed_ids = first_ids;
            g.embed_rows = e->c.n_vocab;
            g.x_store = e->x;
        } else {
            g.x = e->x;
        }
        g.trace = next_trace(e);
        std::tie(g.next_w, g.next_w_bytes) = wspan(5 * l + 2);
        B200_TRY(mark(e, "qkv_gemv", gemv_launch(g, st, pdl)));

        QkNormRopeArgs r;
        r.q_in = e->qkv;
        r.q_ld = e->qkv_rows;
        r.k_in = e->qkv + e->Hq * D;
        r.k_ld = e->qkv_rows;
        r.v_in = e->qkv + (e->Hq + e->Hkv) * D;
        r.v_ld = e->qkv_rows;
        r.q_gamma = w.q_norm;
        r.k_gamma = w.k_norm;
        r.freq = e->freq;
        r.pos_base = e->n_past_dev;
        r.out_offset = e->n_past_dev;
        r.q_out = e->q;
        r.k_out = w.kc;
        r.k_out_ld = static_cast<int64_t>(e->Hkv) * D;
        r.v_out = w.vc;
        r.v_out_ld = static_cast<int64_t>(e->Hkv) * D;
        r.D = D;
        r.Hq = e->Hq;
        r.Hkv = e->Hkv;
        r.T = M;
        r.n_ctx = e->c.kv_capacity;
        r.eps = e->c.rms_eps;
        r.status = e->status;
        // single-token decode: the attention kernel applies QK-norm + RoPE and appends K/V itself
        if (M > 1) B200_TRY(mark(e, "qk_norm_rope_kv", qk_norm_rope_launch(r, st, pdl)));

        AttnArgs a;
        a.q = e->q;
        a.k = w.kc;
        a.v = w.vc;
        a.out = e->attn;
        a.k_tok = static_cast<int64_t>(e->Hkv) * D;
        a.k_head = D;
        a.v_tok = static_cast<int64_t>(e->Hkv) * D;
        a.v_head = D;
        a.D = D;
        a.Hq = e->Hq;
        a.Hkv = e->Hkv;
        a.Tq = M;
        a.n_past_dev = e->n_past_dev;
        a.kv_rows = e->c.kv_capacity;
        a.ws = e->attn_ws;
        a.ws_bytes = e->attn_ws_bytes;
        a.status = e->status;
        a.qkv = e->qkv;
        a.q_gamma = w.q_norm;
        a.k_gamma = w.k_norm;
        a.freq = e->freq;
        a.eps = e->c.rms_eps;
        a.n_ctx = e->c.kv_capacity;
        if (M == 1) {
            a.trace = next_trace(e);
            std::tie(a.next_w, a.next_w_bytes) = wspan(5 * l + 3);
            a.early_kv = pdl;  // the QKV GEMV before it signals late (late_launch)
            B200_TRY(mark(e, "attn_decode", attn_decode_launch(a, e->attn_splits, st, pdl)));
        } else {
            a.precision = e->c.precision;
            B200_TRY(mark(e, "attn_prefill", attn_prefill_launch(a, st, pdl)));
        }

        GemvArgs o;
        o.w = w.wo;
        o.K = static_cast<int64_t>(e->Hq) * D;
        o.N = H;
        o.M = M;
        o.x = e->attn;
        o.out = e->x;
        o.residual = e->x;
        o.epi = (e->tp && e->c.tp_rank != 0) ? GEMV_STORE : GEMV_RESIDUAL;
        o.status = e->status;
        o.trace = next_trace(e);
        std::tie(o.next_w, o.next_w_bytes) = wspan(5 * l + 4);
        B200_TRY(mark(e, "o_proj_gemv", gemv_launch(o, st, pdl)));
        if (e->tp) B200_TRY(tp_allreduce(e->tp, e->x, static_cast<size_t>(M) * H, st, pdl, e->status));

        GemvArgs gu;
        gu.w = w.wgu;
        gu.K = H;
        gu.N = 2 * static_cast<int64_t>(e->F);
        gu.M = M;
        gu.x = e->x;
        gu.gamma = w.ffn_norm;
        gu.eps = e->c.rms_eps;
        gu.out = e->h;
        gu.epi = GEMV_SWIGLU;
        gu.status = e->status;
        gu.trace = next_trace(e);
        std::tie(gu.next_w, gu.next_w_bytes) = wspan(5 * l + 5);
        B200_TRY(mark(e, "gate_up_gemv", gemv_launch(gu, st, pdl)));

        GemvArgs dn;
        dn.w = w.wdown;
        dn.K = e->F;
        dn.N = H;
        dn.M = M;
        dn.x = e->h;
        dn.out = e->x;
        dn.residual = e->x;
        dn.epi = (e->tp && e->c.tp_rank != 0) ? GEMV_STORE : GEMV_RESIDUAL;
        dn.status = e->status;
        dn.trace = next_trace(e);
        std::tie(dn.next_w, dn.next_w_bytes) = wspan(5 * l + 6);
        B200_TRY(mark(e, "down_gemv", gemv_launch(dn, st, pdl)));
        if (e->tp) B200_TRY(tp_allreduce(e->tp, e->x, static_cast<size_t>(M) * H, st, pdl, e->status));
    }
    GemvArgs lm;
    lm.w = e->lm_head;
    lm.K = H;
    lm.N = e->V;
    lm.M = 1;
    lm.x = e->x + static_cast<int64_t>(M - 1) * H;
    lm.gamma = e->out_norm;
    lm.eps = e->c.rms_eps;
    lm.out = want_logits ? e->logits : nullptr;
    lm.epi = GEMV_ARGMAX;
    lm.part_val = e->am_val;
    lm.part_idx = e->am_idx;
    lm.counter = e->am_counter;
    lm.status = e->status;
    if (e->tp) {
        lm.argmax_out = e->am_idx + e->am_slots;     // local winner (scratch slot)
        lm.best_val_out = e->am_val + e->am_slots;
        lm.idx_offset = e->vocab_off;
        B200_TRY(gemv_launch(lm, st, pdl));
        B200_TRY(tp_select_token(e->tp, e->am_val + e->am_slots, e->am_idx + e->am_slots, e->tp_pairs, e->token, e->token_log,
                                 e->log_pos, e->log_cap, e->n_past_dev, n_past_add, st, pdl, e->status));
    } else {
        lm.argmax_out = e->token;
        lm.token_log = e->token_log;
        lm.log_pos = e->log_pos;
        lm.log_cap = e->log_cap;
        lm.n_past = e->n_past_dev;
        lm.n_past_add = n_past_add;
        lm.trace = next_trace(e);
        std::tie(lm.next_w, lm.next_w_bytes) = wspan(0);
        B200_TRY(mark(e, "lm_head_gemv", gemv_launch(lm, st, pdl)));
    }
    return B200_OK;
}

// Prefill of n > 4 tokens whose ids are already in e->ids.
int enqueue_prefill(b200_engine *e, int n, bool want_logits) {
    cudaStream_t st = e->stream;
    const int H = e->H, D = e->D;
    const bool pdl = true;
    B200_TRY(get_rows_launch(e->tok_embd, e->ids, e->x, H, n, e->c.n_vocab, e->status, st, pdl));
    for (int l = 0; l < e->c.n_layer; ++l) {
        const LayerW &w = e->L[l];
        // TF32: the normalised rows only feed TF32 products, written rounded to nearest
        const bool tf32 = e->c.precision == B200_PREC_TF32;
        B200_TRY(rms_norm_launch(e->x, w.attn_norm, e->xn, H, n, e->c.rms_eps, st, pdl, tf32));
        GemmArgs g;
        g.x = e->xn;
        g.ldx = H;
        g.w = w.wqkv;
        g.c = e->qkv;
        g.ldc = e->qkv_rows;
        g.M = n;
        g.N = e->qkv_rows;
        g.K = H;
        g.epi = GEMM_STORE;
        g.ws = e->gemm_ws;
        g.ws_floats = e->gemm_ws_floats;
        g.status = e->status;
        B200_TRY(e->c.precision == B200_PREC_TF32 ? gemm_tf32_launch(g, st, pdl) : gemm_ffma_launch(g, st, pdl));

        QkNormRopeArgs r;
        r.q_in = e->qkv;
        r.q_ld = e->qkv_rows;
        r.k_in = e->qkv + e->Hq * D;
        r.k_ld = e->qkv_rows;
        r.v_in = e->qkv + (e->Hq + e->Hkv) * D;
        r.v_ld = e->qkv_rows;
        r.q_gamma = w.q_norm;
        r.k_gamma = w.k_norm;
        r.freq = e->freq;
        r.pos_base = e->n_past_dev;
        r.out_offset = e->n_past_dev;
        r.q_out = e->q;
        r.k_out = w.kc;
        r.k_out_ld = static_cast<int64_t>(e->Hkv) * D;
        r.v_out = w.vc;
        r.v_out_ld = static_cast<int64_t>(e->Hkv) * D;
        r.D = D;
        r.Hq = e->Hq;
        r.Hkv = e->Hkv;
        r.T = n;
        r.n_ctx = e->c.kv_capacity;
        r.eps = e->c.rms_eps;
        r.status = e->status;
        B200_TRY(qk_norm_rope_launch(r, st, pdl));

        AttnArgs a;
        a.q = e->q;
        a.k = w.kc;
        a.v = w.vc;
        a.out = e->attn;
        a.k_tok = static_cast<int64_t>(e->Hkv) * D;
        a.k_head = D;
        a.v_tok = a.k_tok;
        a.v_head = D;
        a.D = D;
        a.Hq = e->Hq;
        a.Hkv = e->Hkv;
        a.Tq = n;
        a.n_past_dev = e->n_past_dev;
        a.kv_rows = e->c.kv_capacity;
        a.precision = e->c.precision;
        a.status = e->status;
        B200_TRY(attn_prefill_launch(a, st, pdl));

        GemmArgs o;
        o.x = e->attn;
        o.ldx = static_cast<int64_t>(e->Hq) * D;
        o.w = w.wo;
        o.c = e->x;
        o.ldc = H;
        o.r = e->x;
        o.M = n;
        o.N = H;
        o.K = static_cast<int64_t>(e->Hq) * D;
        o.epi = (e->tp && e->c.tp_rank != 0) ? GEMM_STORE : GEMM_RESIDUAL;
        o.ws = e->gemm_ws;
        o.ws_floats = e->gemm_ws_floats;
        o.status = e->status;
        B200_TRY(e->c.precision == B200_PREC_TF32 ? gemm_tf32_launch(o, st, pdl) : gemm_ffma_launch(o, st, pdl));
        if (e->tp) B200_TRY(tp_allreduce(e->tp, e->x, static_cast<size_t>(n) * H, st, false, e->status));

        B200_TRY(rms_norm_launch(e->x, w.ffn_norm, e->xn, H, n, e->c.rms_eps, st, pdl, tf32));
        GemmArgs gu;
        gu.x = e->xn;
        gu.ldx = H;
        gu.w = w.wgu;
        gu.c = e->h;
        gu.ldc = e->F;
        gu.M = n;
        gu.N = 2 * static_cast<int64_t>(e->F);
        gu.K = H;
        gu.epi = GEMM_SWIGLU;
        gu.round_out = tf32;  // h feeds the down product only
        gu.ws = e->gemm_ws;
        gu.ws_floats = e->gemm_ws_floats;
        gu.status = e->status;
        B200_TRY(e->c.precision == B200_PREC_TF32 ? gemm_tf32_launch(gu, st, pdl) : gemm_ffma_launch(gu, st, pdl));

        GemmArgs dn;
        dn.x = e->h;
        dn.ldx = e->F;
        dn.w = w.wdown;
        dn.c = e->x;
        dn.ldc = H;
        dn.r = e->x;
        dn.M = n;
        dn.N = H;
        dn.K = e->F;
        dn.epi = (e->tp && e->c.tp_rank != 0) ? GEMM_STORE : GEMM_RESIDUAL;
        dn.ws = e->gemm_ws;
        dn.ws_floats = e->gemm_ws_floats;
        dn.status = e->status;
        B200_TRY(e->c.precision == B200_PREC_TF32 ? gemm_tf32_launch(dn, st, pdl) : gemm_ffma_launch(dn, st, pdl));
        if (e->tp) B200_TRY(tp_allreduce(e->tp, e->x, static_cast<size_t>(n) * H, st, false, e->status));
    }
    GemvArgs lm;
    lm.w = e->lm_head;
    lm.K = H;
    lm.N = e->V;
    lm.M = 1;
    lm.x = e->x + static_cast<int64_t>(n - 1) * H;
    lm.gamma = e->out_norm;
    lm.eps = e->c.rms_eps;
    lm.out = want_logits ? e->logits : nullptr;
    lm.epi = GEMV_ARGMAX;
    lm.part_val = e->am_val;
    lm.part_idx = e->am_idx;
    lm.counter = e->am_counter;
    lm.status = e->status;
    if (e->tp) {
        lm.argmax_out = e->am_idx + e->am_slots;
        lm.best_val_out = e->am_val + e->am_slots;
        lm.idx_offset = e->vocab_off;
        B200_TRY(gemv_launch(lm, st, pdl));
        B200_TRY(tp_select_token(e->tp, e->am_val + e->am_slots, e->am_idx + e->am_slots, e->tp_pairs, e->token, e->token_log,
                                 e->log_pos, e->log_cap, e->n_past_dev, n, st, false, e->status));
    } else {
        lm.argmax_out = e->token;
        lm.token_log = e->token_log;
        lm.log_pos = e->log_pos;
        lm.log_cap = e->log_cap;
        lm.n_past = e->n_past_dev;
        lm.n_past_add = n;
        B200_TRY(gemv_launch(lm, st, pdl));
    }
    return B200_OK;
}

// Device n_past := the host's committed n_past (after a failed step).
int restore_n_past(b200_engine *e) {
    e->pinned_io[e->io_tok + 3] = static_cast<int32_t>(e->n_past);
    B200_TRY(cudaMemcpyAsync(e->n_past_dev, e->pinned_io + e->io_tok + 3, 4, cudaMemcpyHostToDevice, e->stream));
    B200_TRY(cudaStreamSynchronize(e->stream));
    return B200_OK;
}

// Host wait bound of a tensor-parallel step (B200_TP_TIMEOUT_MS, default 60 s).
int64_t tp_timeout_ms() {
    const char *v = std::getenv("B200_TP_TIMEOUT_MS");
    const long long x = (v && *v) ? std::atoll(v) : 60000;
    return x > 0 ? x : 60000;
}

int check_status(b200_engine *e) {
    // into pinned memory: an asynchronous copy to pageable memory would block here
    // until the stream drains, before the bounded wait below could begin
    int32_t *ps = e->pinned_io + e->io_tok + 4;
    *ps = 0;
    B200_TRY(cudaMemcpyAsync(ps, e->status, 4, cudaMemcpyDeviceToHost, e->stream));
    if (e->tp) {
        const int rc = tp_sync(e->tp, e->stream, tp_timeout_ms());
        if (rc != B200_OK) return rc;
    }
    B200_TRY(cudaStreamSynchronize(e->stream));
    const int32_t s = *ps;
    if (s == 0) return B200_OK;
    B200_TRY(cudaMemsetAsync(e->status, 0, 4, e->stream));
    // an aborted step may leave argmax tickets and attention split counters behind
    B200_TRY(cudaMemsetAsync(e->am_counter, 0, 4, e->stream));
    if (e->attn_ws_bytes) B200_TRY(cudaMemsetAsync(e->attn_ws, 0, e->attn_ws_bytes, e->stream));
    B200_TRY(cudaStreamSynchronize(e->stream));
    if (s == B200_DEV_BAD_LOGITS) return B200_ERR_NUMERIC;
    if (s == B200_DEV_TIMEOUT) return B200_ERR_TIMEOUT;
    if (s == B200_DEV_BAD_TOKEN || s == B200_DEV_BAD_POSITION) return B200_ERR_OUT_OF_RANGE;
    return B200_ERR_DEVICE_CHECK;
}

// Accounts for n single-launch decode steps about to be enqueued on the engine
// stream. Tags repeat after kMkTagPeriod launches; before kMkClearEvery launches
// have run since the last clear, the tagged words and the launch counter are
// cleared together (stream-ordered, before the launches), so no word left by an
// earlier launch can carry a tag of a later one.
int mk_account(b200_engine *e, int64_t n) {
    if (!e->use_mk || n <= 0) return B200_OK;
    if (e->mk_since_clear + n > kMkClearEvery) {
        B200_TRY(cudaMemsetAsync(e->mk_words, 0, e->mk_words_bytes, e->stream));
        B200_TRY(cudaMemsetAsync(e->mk.launches, 0, 8, e->stream));
        e->mk_since_clear = 0;
    }
    e->mk_since_clear += n;
    return B200_OK;
}

int build_graph(b200_engine *e) {
    if (e->graph_exec) return B200_OK;
    B200_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int rc = B200_OK;
    if (e->use_mk) {
        MkParams p = e->mk;
        p.trace = nullptr;
        rc = from_cuda(mk_launch(p, e->stream));
    } else {
        rc = enqueue_small_step(e, e->token, 1, false, 1, true);
    }
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (rc != B200_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    B200_TRY(ce);
    e->graph = g;
    B200_TRY(cudaGraphInstantiate(&e->graph_exec, g, 0));
    return B200_OK;
}

}  // namespace

extern "C" {

int b200_engine_create(const b200_qwen3_config *cfg, int device, b200_engine **out) {
    if (!cfg || !out) return B200_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    const b200_qwen3_config c = *cfg;
    const int W = c.tp_world > 0 ? c.tp_world : 1;
    if (c.n_embd <= 0 || c.n_layer <= 0 || c.n_head <= 0 || c.n_head_kv <= 0 || c.head_dim <= 0 || c.n_ff <= 0 ||
        c.n_vocab <= 0 || c.kv_capacity <= 0 || c.max_batch <= 0 || c.n_head % c.n_head_kv)
        return B200_ERR_INVALID_ARGUMENT;
    if (c.tp_rank < 0 || c.tp_rank >= W || c.n_head % W || c.n_head_kv % W || c.n_ff % W || c.n_vocab % W)
        return B200_ERR_INVALID_ARGUMENT;
    if ((c.n_embd & 3) || (c.head_dim != 64 && c.head_dim != 128) || c.kv_capacity > c.n_ctx_train)
        return B200_ERR_NOT_SUPPORTED;
    if (!c.tied && false) return B200_ERR_NOT_SUPPORTED;
    DeviceGuard dg(device);
    auto *e = new b200_engine();
    e->c = c;
    e->c.tp_world = W;
    e->device = device;
    e->H = c.n_embd;
    e->D = c.head_dim;
    e->Hq = c.n_head / W;
    e->Hkv = c.n_head_kv / W;
    e->F = c.n_ff / W;
    e->V = c.n_vocab / W;
    e->vocab_off = static_cast<int64_t>(c.tp_rank) * e->V;
    e->qkv_rows = (e->Hq + 2 * e->Hkv) * e->D;
    if (((e->F) & 3) || ((e->Hq * e->D) & 3)) {
        delete e;
        return B200_ERR_NOT_SUPPORTED;
    }
    const int64_t H = e->H, D = e->D, F = e->F, V = e->V, NL = c.n_layer;
    const int64_t cap = c.kv_capacity, MB = c.max_batch;

    // ---- weight arena: embedding (full, replicated), per-layer packed, final norm, LM head
    const size_t A = 256;
    size_t off = 0;
    auto take = [&](int64_t floats) {
        const size_t o = off;
        off = align_up(off + static_cast<size_t>(floats) * 4, A);
        return o;
    };
    const size_t o_embd = take(static_cast<int64_t>(c.n_vocab) * H);
    const size_t o_onorm = take(H);
    const size_t o_freq = take(D / 2);
    size_t o_lm = 0;
    if (!c.tied) o_lm = take(V * H);
    std::vector<size_t> lo(NL * 8);
    for (int64_t l = 0; l < NL; ++l) {
        lo[l * 8 + 0] = take(H);                                   // attn_norm
        lo[l * 8 + 1] = take(static_cast<int64_t>(e->qkv_rows) * H); // wqkv
        lo[l * 8 + 2] = take(D);                                   // q_norm
        lo[l * 8 + 3] = take(D);                                   // k_norm
        lo[l * 8 + 4] = take(H * e->Hq * D);                       // wo [H][Hq*D]
        lo[l * 8 + 5] = take(H);                                   // ffn_norm
        lo[l * 8 + 6] = take(2 * F * H);                           // wgu interleaved
        lo[l * 8 + 7] = take(H * F);                               // wdown [H][F]
    }
    e->w_bytes = off;
    // ---- KV arena: per layer K block [cap][Hkv][D] then V block (NaiveKVStorage layout)
    const size_t kv_layer = align_up(static_cast<size_t>(cap * e->Hkv * D) * 4, A) * 2;
    e->kv_bytes = kv_layer * NL;
    // ---- activation arena
    e->attn_splits = attn_decode_splits(cap, e->Hkv);
    e->attn_ws_bytes = attn_decode_ws_bytes(D, e->Hq, e->Hkv, e->attn_splits);
    off = 0;
    const size_t o_x = take(MB * H), o_xn = take(MB * H), o_qkv = take(MB * e->qkv_rows);
    const size_t o_q = take(MB * e->Hq * D), o_attn = take(MB * e->Hq * D), o_h = take(MB * F);
    const size_t o_logits = take(V);
    const size_t o_ids = take(MB), o_tok = take(4), o_np = take(4), o_st = take(4);
    e->log_cap = 65536;
    const size_t o_log = take(e->log_cap), o_logpos = take(4);
    const size_t o_aws = off;
    off = align_up(off + e->attn_ws_bytes, A);
    e->am_slots = std::max(gemv_argmax_slots(V, H), mk_grid());
    const size_t o_amv = take(e->am_slots + 64), o_ami = take(e->am_slots + 64), o_amc = take(64);
    const size_t o_pairs = take(2 * W + 64);
    e->trace_cap = 5 * c.n_layer + 8;
    const size_t o_trace = take(2 * 8 * static_cast<int64_t>(e->trace_cap));
    // split-K workspace of the prefill GEMMs: 8 Mi floats (bounded by the launcher)
    e->gemm_ws_floats = int64_t(8) << 20;
    const size_t o_gws = take(e->gemm_ws_floats);
    const size_t o_mkl = take(static_cast<int64_t>(sizeof(MkLayer) / 4 + 1) * NL);
    MkParams shape;
    shape.Hq = e->Hq;
    shape.D = static_cast<int>(D);
    // tagged activation words of the single-launch decode step (8 bytes each)
    const size_t o_tx = take(2 * H), o_tqkv = take(2 * static_cast<int64_t>(e->qkv_rows));
    const size_t o_th = take(2 * F);
    const size_t o_tpo = take(2 * static_cast<int64_t>(mk_po_words(shape)));
    const size_t o_tpml = take(2 * static_cast<int64_t>(mk_pml_words(shape)));
    const size_t o_tao = take(2 * static_cast<int64_t>(e->Hq) * D);
    const size_t o_withhold = take(64);
    const size_t o_mkl_n = take(64);
    e->act_bytes = off;

    cudaError_t err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaMalloc(&e->w_arena, e->w_bytes);
    if (c.external_kv) e->kv_bytes = 0;  // the caller binds each layer's KV object (b200_engine_bind_kv)
    if (err == cudaSuccess && e->kv_bytes) err = cudaMalloc(&e->kv_arena, e->kv_bytes);
    if (err == cudaSuccess) err = cudaMalloc(&e->act_arena, e->act_bytes);
    e->io_tok = (static_cast<int64_t>(c.max_batch) + 15) / 16 * 16;
    if (err == cudaSuccess) err = cudaMallocHost(&e->pinned_io, static_cast<size_t>(e->io_tok + 16) * 4);
    if (err != cudaSuccess) {
        b200_engine_destroy(e);
        cudaGetLastError();
        return err == cudaErrorMemoryAllocation ? B200_ERR_NO_MEMORY : B200_ERR_CUDA;
    }
    auto wf = [&](size_t o) { return reinterpret_cast<float *>(e->w_arena + o); };
    auto af = [&](size_t o) { return reinterpret_cast<float *>(e->act_arena + o); };
    auto ai = [&](size_t o) { return reinterpret_cast<int32_t *>(e->act_arena + o); };
    e->tok_embd = wf(o_embd);
    e->out_norm = wf(o_onorm);
    e->freq = wf(o_freq);
    e->lm_head = c.tied ? e->tok_embd + e->vocab_off * H : wf(o_lm);
    e->L.resize(NL);
    for (int64_t l = 0; l < NL; ++l) {
        LayerW &w = e->L[l];
        w.attn_norm = wf(lo[l * 8 + 0]);
        w.wqkv = wf(lo[l * 8 + 1]);
        w.q_norm = wf(lo[l * 8 + 2]);
        w.k_norm = wf(lo[l * 8 + 3]);
        w.wo = wf(lo[l * 8 + 4]);
        w.ffn_norm = wf(lo[l * 8 + 5]);
        w.wgu = wf(lo[l * 8 + 6]);
        w.wdown = wf(lo[l * 8 + 7]);
        if (e->kv_arena) {
            w.kc = reinterpret_cast<float *>(e->kv_arena + kv_layer * l);
            w.vc = reinterpret_cast<float *>(e->kv_arena + kv_layer * l + kv_layer / 2);
        }
    }
    e->x = af(o_x);
    e->xn = af(o_xn);
    e->qkv = af(o_qkv);
    e->q = af(o_q);
    e->attn = af(o_attn);
    e->h = af(o_h);
    e->logits = af(o_logits);
    e->ids = ai(o_ids);
    e->token = ai(o_tok);
    e->n_past_dev = ai(o_np);
    e->status = ai(o_st);
    e->token_log = ai(o_log);
    e->log_pos = ai(o_logpos);
    e->attn_ws = e->act_arena + o_aws;
    e->am_val = af(o_amv);
    e->am_idx = ai(o_ami);
    e->am_counter = reinterpret_cast<unsigned *>(e->act_arena + o_amc);
    e->tp_pairs = af(o_pairs);
    e->trace_buf = reinterpret_cast<unsigned long long *>(e->act_arena + o_trace);
    e->gemm_ws = af(o_gws);
    e->mk_layers = reinterpret_cast<MkLayer *>(e->act_arena + o_mkl);
    auto aw = [&](size_t o) { return reinterpret_cast<unsigned long long *>(e->act_arena + o); };
    e->mk.tx = aw(o_tx);
    e->mk.tqkv = aw(o_tqkv);
    e->mk.th = aw(o_th);
    e->mk.tpo = aw(o_tpo);
    e->mk.tpml = aw(o_tpml);
    e->mk.tao = aw(o_tao);
    e->mk.withhold = ai(o_withhold);  // zeroed with the arena below: no injection
    e->mk.launches = reinterpret_cast<unsigned long long *>(e->act_arena + o_mkl_n);
    e->mk_words = e->act_arena + o_tx;
    e->mk_words_bytes = o_withhold - o_tx;  // the tagged words (tx .. tao)
    err = cudaMemsetAsync(e->act_arena, 0, e->act_bytes, e->stream);
    if (err == cudaSuccess && e->kv_arena) err = cudaMemsetAsync(e->kv_arena, 0, e->kv_bytes, e->stream);
    std::vector<float> hf(D / 2);
    b200_rope_freqs(c.rope_theta, D, hf.data());
    if (err == cudaSuccess) err = cudaMemcpyAsync(e->freq, hf.data(), hf.size() * 4, cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    if (err != cudaSuccess) {
        b200_engine_destroy(e);
        return B200_ERR_CUDA;
    }
    // weights still to be provided
    e->missing = {"token_embd.weight", "output_norm.weight"};
    if (!c.tied) e->missing.push_back("output.weight");
    static const char *per_layer[] = {"attn_norm", "attn_q",   "attn_k",   "attn_v",  "attn_output", "attn_q_norm",
                                      "attn_k_norm", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
    for (int l = 0; l < c.n_layer; ++l)
        for (const char *p : per_layer) e->missing.push_back("blk." + std::to_string(l) + "." + p + ".weight");
    *out = e;
    return B200_OK;
}

void b200_engine_destroy(b200_engine *e) {
    if (!e) return;
    DeviceGuard dg(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    // the decode graph holds NCCL operations under tensor parallelism: released first
    if (e->graph_exec) cudaGraphExecDestroy(e->graph_exec);
    if (e->graph) cudaGraphDestroy(e->graph);
    if (e->tp) tp_destroy(e->tp);
    cudaFree(e->w_arena);
    cudaFree(e->kv_arena);
    cudaFree(e->act_arena);
    if (e->pinned_io) cudaFreeHost(e->pinned_io);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

int b200_engine_memory(const b200_engine *e, size_t *weights, size_t *kv, size_t *act) {
    if (!e) return B200_ERR_INVALID_ARGUMENT;
    if (weights) *weights = e->w_bytes;
    if (kv) *kv = e->kv_bytes;
    if (act) *act = e->act_bytes;
    return B200_OK;
}

}  // extern "C"

namespace {

// Where one GGUF tensor lives in the engine's weight arena: `rows` rows of `width`
// floats, taken from the host tensor at src_off + row * spitch (floats) and stored
// at dst + row * dpitch. Every weight is one such block: whole tensors, this rank's
// row or column shard, the q / k / v rows of the fused QKV matrix, the interleaved
// gate / up rows.
struct WeightBlock {
    float *dst = nullptr;
    int64_t dpitch = 0, src_off = 0, spitch = 0, width = 0, rows = 0;
};

// The block of tensor `name` (n elements in its GGUF shape); B200_ERR_INVALID_ARGUMENT
// for an unknown name or a wrong size.
int weight_block(b200_engine *e, const std::string &nm, int64_t n, WeightBlock *out) {
    const b200_qwen3_config &c = e->c;
    const int64_t r = c.tp_rank;
    const int64_t H = e->H, D = e->D, F = e->F, V = e->V;
    const int64_t Hq_all = c.n_head, Hkv_all = c.n_head_kv;
    auto whole = [&](float *dst, int64_t floats) {  // a vector: one row
        *out = WeightBlock{dst, floats, 0, floats, floats, 1};
        return B200_OK;
    };
    // rows [row0, row0 + rows) of a [N][K] matrix, into dst with pitch dpitch
    auto rows_of = [&](float *dst, int64_t dpitch, int64_t K, int64_t row0, int64_t rows) {
        *out = WeightBlock{dst, dpitch, row0 * K, K, K, rows};
        return B200_OK;
    };
    int layer = -1;
    const char *rest = nullptr;
    if (nm == "token_embd.weight") {  // full on every rank (the gather needs any row)
        if (n != static_cast<int64_t>(c.n_vocab) * H) return B200_ERR_INVALID_ARGUMENT;
        return rows_of(e->tok_embd, H, H, 0, c.n_vocab);
    }
    if (nm == "output_norm.weight") return n == H ? whole(e->out_norm, H) : B200_ERR_INVALID_ARGUMENT;
    if (nm == "output.weight") {
        if (c.tied || n != static_cast<int64_t>(c.n_vocab) * H) return B200_ERR_INVALID_ARGUMENT;
        return rows_of(e->lm_head, H, H, e->vocab_off, V);  // this rank's vocabulary rows
    }
    if (!parse_layer(nm.c_str(), &layer, &rest) || layer < 0 || layer >= c.n_layer) return B200_ERR_INVALID_ARGUMENT;
    LayerW &w = e->L[layer];
    const std::string p(rest);
    if (p == "attn_norm.weight" || p == "ffn_norm.weight")
        return n == H ? whole(p[0] == 'a' ? w.attn_norm : w.ffn_norm, H) : B200_ERR_INVALID_ARGUMENT;
    if (p == "attn_q_norm.weight" || p == "attn_k_norm.weight")
        return n == D ? whole(p[5] == 'q' ? w.q_norm : w.k_norm, D) : B200_ERR_INVALID_ARGUMENT;
    if (p == "attn_q.weight") {
        if (n != Hq_all * D * H) return B200_ERR_INVALID_ARGUMENT;
        return rows_of(w.wqkv, H, H, r * e->Hq * D, e->Hq * D);
    }
    if (p == "attn_k.weight" || p == "attn_v.weight") {
        if (n != Hkv_all * D * H) return B200_ERR_INVALID_ARGUMENT;
        float *dst = w.wqkv + (e->Hq + (p[5] == 'k' ? 0 : e->Hkv)) * D * H;
        return rows_of(dst, H, H, r * e->Hkv * D, e->Hkv * D);
    }
    if (p == "attn_output.weight") {
        // [H][Hq*D]: this rank's column block (row-split for tensor parallelism)
        if (n != H * Hq_all * D) return B200_ERR_INVALID_ARGUMENT;
        const int64_t kc = e->Hq * D;
        *out = WeightBlock{w.wo, kc, r * kc, Hq_all * D, kc, H};
        return B200_OK;
    }
    if (p == "ffn_gate.weight" || p == "ffn_up.weight") {
        // interleaved: packed row 2i = gate row i, 2i+1 = up row i
        if (n != static_cast<int64_t>(c.n_ff) * H) return B200_ERR_INVALID_ARGUMENT;
        *out = WeightBlock{w.wgu + (p[4] == 'g' ? 0 : H), 2 * H, r * F * H, H, H, F};
        return B200_OK;
    }
    if (p == "ffn_down.weight") {
        if (n != H * static_cast<int64_t>(c.n_ff)) return B200_ERR_INVALID_ARGUMENT;
        *out = WeightBlock{w.wdown, F, r * F, static_cast<int64_t>(c.n_ff), F, H};
        return B200_OK;
    }
    return B200_ERR_INVALID_ARGUMENT;
}

// Rows [a, b) of a block between the host tensor and the arena (one 2-D copy).
cudaError_t copy_rows(const WeightBlock &wb, float *host, int64_t a, int64_t b, cudaMemcpyKind kind, cudaStream_t st) {
    float *dev = wb.dst + a * wb.dpitch;
    float *hst = host + wb.src_off + a * wb.spitch;
    if (kind != cudaMemcpyDeviceToHost)
        return cudaMemcpy2DAsync(dev, wb.dpitch * 4, hst, wb.spitch * 4, wb.width * 4, b - a, kind, st);
    return cudaMemcpy2DAsync(hst, wb.spitch * 4, dev, wb.dpitch * 4, wb.width * 4, b - a, kind, st);
}

void mark_loaded(b200_engine *e, const std::string &nm) {
    for (size_t i = 0; i < e->missing.size(); ++i)
        if (e->missing[i] == nm) {
            e->missing.erase(e->missing.begin() + i);
            return;
        }
}

// ---- minimal GGUF v3 reader (gguf_parser.cpp:100-125 reads the same layout):
// header, metadata records (skipped except general.alignment), tensor infos.
struct GgufTensor {
    std::string name;
    int64_t n = 0;
    uint32_t type = 0;
    uint64_t offset = 0;
};

struct GgufFile {
    const unsigned char *base = nullptr;
    size_t size = 0, pos = 0;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if (pos + sizeof(T) > size) {
            ok = false;
            return v;
        }
        std::memcpy(&v, base + pos, sizeof(T));
        pos += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > size - pos) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char *>(base + pos), n);
        pos += n;
        return s;
    }
    // skips one metadata value of GGUF type t
    void skip(uint32_t t, int depth = 0) {
        static const size_t fixed[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t == 8) {
            str();
        } else if (t == 9) {
            const uint32_t et = get<uint32_t>();
            const uint64_t cnt = get<uint64_t>();
            if (!ok || depth > 2) {
                ok = false;
                return;
            }
            if (et != 8 && et != 9 && et < 13) {
                if (cnt > (size - pos) / fixed[et]) {
                    ok = false;
                    return;
                }
                pos += cnt * fixed[et];
            } else {
                for (uint64_t i = 0; i < cnt && ok; ++i) skip(et, depth + 1);
            }
        } else if (t < 13) {
            if (fixed[t] > size - pos) {
                ok = false;
                return;
            }
            pos += fixed[t];
        } else {
            ok = false;
        }
    }
};

}  // namespace

extern "C" {

int b200_engine_set_weight(b200_engine *e, const char *name, const float *host, int64_t n) {
    if (!e || !name || !host) return B200_ERR_INVALID_ARGUMENT;
    if (e->finalized) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    WeightBlock wb;
    const int rc = weight_block(e, name, n, &wb);
    if (rc != B200_OK) return rc;
    // cudaMemcpyDefault: the source may be host memory or device memory (unified addressing)
    cudaError_t err = copy_rows(wb, const_cast<float *>(host), 0, wb.rows, cudaMemcpyDefault, e->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);  // the source may be released after return
    if (err != cudaSuccess) return from_cuda(err);
    mark_loaded(e, name);
    return B200_OK;
}

int b200_engine_get_weight(b200_engine *e, const char *name, float *host_out, int64_t n) {
    if (!e || !name || !host_out) return B200_ERR_INVALID_ARGUMENT;
    if (e->c.tp_world != 1) return B200_ERR_NOT_SUPPORTED;
    DeviceGuard dg(e->device);
    WeightBlock wb;
    const int rc = weight_block(e, name, n, &wb);
    if (rc != B200_OK) return rc;
    cudaError_t err = copy_rows(wb, host_out, 0, wb.rows, cudaMemcpyDeviceToHost, e->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    return from_cuda(err);
}

int b200_engine_load_gguf(b200_engine *e, const char *path, int64_t staging_bytes) {
    if (!e || !path || e->finalized) return B200_ERR_INVALID_ARGUMENT;
    if (staging_bytes <= 0) staging_bytes = int64_t(256) << 20;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return B200_ERR_INVALID_ARGUMENT;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 24) {
        close(fd);
        return B200_ERR_INVALID_ARGUMENT;
    }
    const size_t fsize = static_cast<size_t>(sb.st_size);
    void *map = mmap(nullptr, fsize, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return B200_ERR_INVALID_ARGUMENT;
    madvise(map, fsize, MADV_SEQUENTIAL);
    GgufFile g{static_cast<const unsigned char *>(map), fsize};
    int rc = B200_OK;
    std::vector<GgufTensor> ts;
    uint64_t align = 32;
    if (g.get<uint32_t>() != 0x46554747u || g.get<uint32_t>() != 3u) rc = B200_ERR_INVALID_ARGUMENT;
    const uint64_t n_tensors = g.get<uint64_t>(), n_kv = g.get<uint64_t>();
    for (uint64_t i = 0; rc == B200_OK && g.ok && i < n_kv; ++i) {
        const std::string key = g.str();
        const uint32_t t = g.get<uint32_t>();
        if (key == "general.alignment" && t == 4) {
            align = g.get<uint32_t>();
            if (align == 0 || (align & (align - 1))) rc = B200_ERR_INVALID_ARGUMENT;
        } else {
            g.skip(t);
        }
    }
    for (uint64_t i = 0; rc == B200_OK && g.ok && i < n_tensors; ++i) {
        GgufTensor t;
        t.name = g.str();
        const uint32_t nd = g.get<uint32_t>();
        t.n = 1;
        for (uint32_t d = 0; d < nd && d < 4; ++d) t.n *= static_cast<int64_t>(g.get<uint64_t>());
        if (nd > 4) rc = B200_ERR_INVALID_ARGUMENT;
        t.type = g.get<uint32_t>();
        t.offset = g.get<uint64_t>();
        ts.push_back(std::move(t));
    }
    if (!g.ok) rc = B200_ERR_INVALID_ARGUMENT;
    const size_t data0 = (g.pos + align - 1) / align * align;
    // validate every tensor before the first copy
    std::vector<WeightBlock> blocks(ts.size());
    for (size_t i = 0; rc == B200_OK && i < ts.size(); ++i) {
        const GgufTensor &t = ts[i];
        if (t.type != 0 /* F32 */ || t.n <= 0 || t.offset > fsize || data0 + t.offset + 4 * static_cast<uint64_t>(t.n) > fsize)
            rc = B200_ERR_INVALID_ARGUMENT;
        else
            rc = weight_block(e, t.name, t.n, &blocks[i]);
    }
    DeviceGuard dg(e->device);
    // Pinned staging ring: the host copies row blocks of the mapping into a slot
    // while the copy engine drains the previous slots; a slot is reused once the
    // event recorded after its last copy has completed. One sync at the end.
    constexpr int kSlots = 4;
    const size_t slot_bytes = std::max<size_t>(static_cast<size_t>(staging_bytes) / kSlots, size_t(1) << 20);
    unsigned char *pinned = nullptr;
    cudaEvent_t ev[kSlots] = {};
    bool used[kSlots] = {};
    cudaError_t err = cudaSuccess;
    if (rc == B200_OK) err = cudaMallocHost(&pinned, slot_bytes * kSlots);
    for (int i = 0; err == cudaSuccess && i < kSlots; ++i) err = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
    int slot = 0;
    for (size_t i = 0; rc == B200_OK && err == cudaSuccess && i < ts.size(); ++i) {
        const WeightBlock &wb = blocks[i];
        const float *src = reinterpret_cast<const float *>(g.base + data0 + ts[i].offset);
        const int64_t row_bytes = wb.width * 4;
        if (row_bytes > static_cast<int64_t>(slot_bytes)) {
            rc = B200_ERR_INVALID_ARGUMENT;  // a single row larger than a slot
            break;
        }
        const int64_t rows_per_slot = static_cast<int64_t>(slot_bytes) / row_bytes;
        for (int64_t a = 0; a < wb.rows && err == cudaSuccess; a += rows_per_slot) {
            const int64_t b = std::min(wb.rows, a + rows_per_slot);
            if (used[slot]) err = cudaEventSynchronize(ev[slot]);
            if (err != cudaSuccess) break;
            float *stage = reinterpret_cast<float *>(pinned + slot * slot_bytes);
            for (int64_t row = a; row < b; ++row)
                std::memcpy(stage + (row - a) * wb.width, src + wb.src_off + row * wb.spitch, row_bytes);
            // the staged rows are packed: source pitch = width
            err = cudaMemcpy2DAsync(wb.dst + a * wb.dpitch, wb.dpitch * 4, stage, row_bytes, row_bytes, b - a,
                                    cudaMemcpyHostToDevice, e->stream);
            if (err == cudaSuccess) err = cudaEventRecord(ev[slot], e->stream);
            used[slot] = true;
            slot = (slot + 1) % kSlots;
        }
    }
    const cudaError_t serr = cudaStreamSynchronize(e->stream);
    if (err == cudaSuccess) err = serr;
    for (int i = 0; i < kSlots; ++i)
        if (ev[i]) cudaEventDestroy(ev[i]);
    if (pinned) cudaFreeHost(pinned);
    munmap(map, fsize);
    if (rc != B200_OK) return rc;
    if (err != cudaSuccess) return from_cuda(err);
    for (const GgufTensor &t : ts) mark_loaded(e, t.name);
    return B200_OK;
}

int b200_engine_init_random(b200_engine *e, uint64_t seed, float std) {
    if (!e || e->finalized) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    cudaStream_t st = e->stream;
    const int64_t H = e->H, D = e->D, F = e->F;
    uint32_t id = 1;
    auto normal = [&](float *p, int64_t n) {
        fill_normal_kernel<<<1184, 256, 0, st>>>(p, n, seed + 0x9E3779B97F4A7C15ull * e->c.tp_rank, id++, std);
        return cudaGetLastError();
    };
    auto ones = [&](float *p, int64_t n) {
        fill_value_kernel<<<296, 256, 0, st>>>(p, n, 1.0f);
        return cudaGetLastError();
    };
    // Shards are generated per rank (each rank's weights are its own draw); the
    // embedding table is replicated, so it uses the rank-independent stream.
    fill_normal_kernel<<<1184, 256, 0, st>>>(e->tok_embd, static_cast<int64_t>(e->c.n_vocab) * H, seed, 0u, std);
    B200_TRY(cudaGetLastError());
    B200_TRY(ones(e->out_norm, H));
    if (!e->c.tied) B200_TRY(normal(e->lm_head, static_cast<int64_t>(e->V) * H));
    for (auto &w : e->L) {
        B200_TRY(ones(w.attn_norm, H));
        B200_TRY(ones(w.ffn_norm, H));
        B200_TRY(ones(w.q_norm, D));
        B200_TRY(ones(w.k_norm, D));
        B200_TRY(normal(w.wqkv, static_cast<int64_t>(e->qkv_rows) * H));
        B200_TRY(normal(w.wo, H * e->Hq * D));
        B200_TRY(normal(w.wgu, 2 * F * H));
        B200_TRY(normal(w.wdown, H * F));
    }
    B200_TRY(cudaStreamSynchronize(st));
    e->missing.clear();
    return B200_OK;
}

int b200_engine_finalize(b200_engine *e) {
    if (!e) return B200_ERR_INVALID_ARGUMENT;
    if (!e->missing.empty()) {
        std::fprintf(stderr, "b200_engine_finalize: %zu weights missing (first: %s)\n", e->missing.size(),
                     e->missing[0].c_str());
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (e->c.tp_world > 1 && !e->tp) return B200_ERR_INVALID_ARGUMENT;
    for (const LayerW &w : e->L)
        if (!w.kc || !w.vc) {
            std::fprintf(stderr, "b200_engine_finalize: a layer's KV object is not bound\n");
            return B200_ERR_INVALID_ARGUMENT;
        }
    DeviceGuard dg(e->device);
    // Single-launch decode step where the shape allows it (one GPU only).
    MkParams &p = e->mk;
    p.n_layer = e->c.n_layer;
    p.H = e->H;
    p.D = e->D;
    p.Hq = e->Hq;
    p.Hkv = e->Hkv;
    p.F = e->F;
    p.V = e->V;
    p.eps = e->c.rms_eps;
    p.n_ctx = e->c.kv_capacity;
    p.tok_embd = e->tok_embd;
    p.out_norm = e->out_norm;
    p.lm_head = e->lm_head;
    p.freq = e->freq;
    p.logits = e->logits;  // V floats per step, so eval() can return logits from the graph step
    p.token = e->token;
    p.n_past = e->n_past_dev;
    p.status = e->status;
    p.token_log = e->token_log;
    p.log_pos = e->log_pos;
    p.log_cap = e->log_cap;
    p.am_val = e->am_val;
    p.am_idx = e->am_idx;
    p.am_counter = e->am_counter;
    p.layers = e->mk_layers;
    // AUTO takes the single-launch kernel wherever it supports the shape (it is the
    // faster of the two on one GPU); MULTI forces the multi-kernel chain.
    e->use_mk = e->c.decode_mode != B200_DECODE_MULTI && e->c.tp_world == 1 && mk_supported(p) &&
                mk_grid() <= e->am_slots;
    if (e->use_mk) {
        std::vector<MkLayer> tab(e->c.n_layer);
        for (int l = 0; l < e->c.n_layer; ++l) {
            const LayerW &w = e->L[l];
            tab[l] = MkLayer{w.attn_norm, w.wqkv, w.q_norm, w.k_norm, w.wo, w.ffn_norm, w.wgu, w.wdown, w.kc, w.vc};
        }
        B200_TRY(cudaMemcpy(e->mk_layers, tab.data(), sizeof(MkLayer) * tab.size(), cudaMemcpyHostToDevice));
    }
    e->finalized = true;
    return B200_OK;
}

int b200_engine_reset(b200_engine *e) {
    if (!e) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    B200_TRY(cudaMemsetAsync(e->n_past_dev, 0, 4, e->stream));
    B200_TRY(cudaStreamSynchronize(e->stream));
    e->n_past = 0;
    return B200_OK;
}

int64_t b200_engine_n_past(const b200_engine *e) { return e ? e->n_past : -1; }

int b200_engine_set_precision(b200_engine *e, int32_t precision) {
    if (!e || (precision != B200_PREC_FFMA && precision != B200_PREC_TF32)) return B200_ERR_INVALID_ARGUMENT;
    e->c.precision = precision;
    return B200_OK;
}

int b200_engine_inject_withhold(b200_engine *e, int32_t cta, int32_t after_steps) {
    if (!e || !e->finalized || after_steps < 0) return B200_ERR_INVALID_ARGUMENT;
    if (!e->use_mk) return B200_ERR_NOT_SUPPORTED;
    if (cta >= mk_grid()) return B200_ERR_OUT_OF_RANGE;
    DeviceGuard dg(e->device);
    const int32_t v[2] = {cta < 0 ? 0 : cta + 1, cta < 0 ? 0 : after_steps};
    B200_TRY(cudaMemcpyAsync(e->mk.withhold, v, 8, cudaMemcpyHostToDevice, e->stream));
    B200_TRY(cudaStreamSynchronize(e->stream));
    return B200_OK;
}

int b200_engine_set_decode_launch_counter(b200_engine *e, uint64_t launches) {
    if (!e || !e->finalized) return B200_ERR_INVALID_ARGUMENT;
    if (!e->use_mk) return B200_ERR_NOT_SUPPORTED;
    DeviceGuard dg(e->device);
    const unsigned long long tickets = static_cast<unsigned long long>(launches) * mk_grid();
    B200_TRY(cudaMemcpyAsync(e->mk.launches, &tickets, 8, cudaMemcpyHostToDevice, e->stream));
    B200_TRY(cudaStreamSynchronize(e->stream));
    return B200_OK;
}

int b200_engine_decode_launches(const b200_engine *e) {
    if (!e || !e->finalized) return -B200_ERR_INVALID_ARGUMENT;
    if (e->use_mk) return 1;
    return 5 * e->c.n_layer + 1 + (e->tp ? 2 : 0);
}

}  // extern "C"

namespace {

// One eval step; the last row's logits go to `last_logits` (host or, with
// logits_on_device, device memory of this engine's device; nullable).
int eval_to(b200_engine *e, const int32_t *host_ids, int64_t n, float *last_logits, bool logits_on_device,
            int32_t *host_token) {
    float *host_last_logits = last_logits;
    if (!e || !host_ids || n <= 0) return B200_ERR_INVALID_ARGUMENT;
    if (!e->finalized) return B200_ERR_INVALID_ARGUMENT;
    if (n > e->c.max_batch) return B200_ERR_INVALID_ARGUMENT;
    if (e->n_past + n > e->c.kv_capacity) return B200_ERR_OUT_OF_RANGE;
    for (int64_t i = 0; i < n; ++i)
        if (host_ids[i] < 0 || host_ids[i] >= e->c.n_vocab) return B200_ERR_OUT_OF_RANGE;
    DeviceGuard dg(e->device);
    cudaStream_t st = e->stream;
    const bool want_logits = host_last_logits != nullptr;
    int rc;
    // one token: the captured decode step (under tensor parallelism it holds the NCCL
    // all-reduces and the token all-gather; logits are not returned there)
    if (n == 1 && (e->c.tp_world > 1 || !want_logits || e->use_mk)) {
        // graph-replayed decode: the token slot is the embedding input
        e->pinned_io[0] = host_ids[0];
        B200_TRY(cudaMemcpyAsync(e->token, e->pinned_io, 4, cudaMemcpyHostToDevice, st));
        rc = build_graph(e);
        if (rc == B200_OK) rc = mk_account(e, 1);
        if (rc != B200_OK) return rc;
        B200_TRY(cudaGraphLaunch(e->graph_exec, st));
    } else {
        std::memcpy(e->pinned_io, host_ids, n * 4);
        B200_TRY(cudaMemcpyAsync(e->ids, e->pinned_io, n * 4, cudaMemcpyHostToDevice, st));
        if (n <= 4)
            rc = enqueue_small_step(e, e->ids, static_cast<int>(n), want_logits, static_cast<int>(n), true);
        else
            rc = enqueue_prefill(e, static_cast<int>(n), want_logits);
        if (rc != B200_OK) return rc;
    }
    B200_TRY(cudaMemcpyAsync(e->pinned_io + e->io_tok, e->token, 4, cudaMemcpyDeviceToHost, st));
    if (want_logits && e->c.tp_world == 1)
        B200_TRY(cudaMemcpyAsync(last_logits, e->logits, static_cast<size_t>(e->V) * 4,
                                 logits_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
    rc = check_status(e);  // synchronizes
    if (rc != B200_OK) {
        // nothing committed: restore n_past (a failed restore is the error reported)
        const int rr = restore_n_past(e);
        return rr != B200_OK ? rr : rc;
    }
    if (host_token) *host_token = e->pinned_io[e->io_tok];
    e->n_past += n;
    return B200_OK;
}

}  // namespace

extern "C" {

int b200_engine_eval(b200_engine *e, const int32_t *host_ids, int64_t n, float *host_last_logits,
                     int32_t *host_token) {
    return eval_to(e, host_ids, n, host_last_logits, false, host_token);
}

int b200_engine_eval_device(b200_engine *e, const int32_t *host_ids, int64_t n, float *dev_last_logits,
                            int32_t *host_token) {
    return eval_to(e, host_ids, n, dev_last_logits, true, host_token);
}

int b200_engine_set_n_past(b200_engine *e, int64_t n_past) {
    if (!e || n_past < 0 || n_past > e->c.kv_capacity) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    e->n_past = n_past;
    return restore_n_past(e);
}

int b200_engine_set_rope_freqs(b200_engine *e, const float *host_freq) {
    if (!e || !host_freq) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    B200_TRY(cudaMemcpyAsync(e->freq, host_freq, static_cast<size_t>(e->D / 2) * 4, cudaMemcpyHostToDevice, e->stream));
    B200_TRY(cudaStreamSynchronize(e->stream));
    return B200_OK;
}

int b200_engine_bind_kv(b200_engine *e, int32_t layer, float *k_base, float *v_base) {
    if (!e || !e->c.external_kv || layer < 0 || layer >= e->c.n_layer || !k_base || !v_base) return B200_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(k_base) | reinterpret_cast<uintptr_t>(v_base)) & 15) return B200_ERR_INVALID_ARGUMENT;
    LayerW &w = e->L[layer];
    if (w.kc == k_base && w.vc == v_base) return B200_OK;
    DeviceGuard dg(e->device);
    w.kc = k_base;
    w.vc = v_base;
    if (e->finalized) {
        // the captured decode step holds the old KV addresses: capture it again at the
        // next step; the single-launch step reads them from its device layer table
        if (e->graph_exec) B200_TRY(cudaGraphExecDestroy(e->graph_exec));
        if (e->graph) B200_TRY(cudaGraphDestroy(e->graph));
        e->graph_exec = nullptr;
        e->graph = nullptr;
        if (e->use_mk) {
            const MkLayer ml{w.attn_norm, w.wqkv, w.q_norm, w.k_norm, w.wo, w.ffn_norm, w.wgu, w.wdown, w.kc, w.vc};
            B200_TRY(cudaMemcpyAsync(e->mk_layers + layer, &ml, sizeof ml, cudaMemcpyHostToDevice, e->stream));
            B200_TRY(cudaStreamSynchronize(e->stream));
        }
    }
    return B200_OK;
}

int b200_engine_generate(b200_engine *e, int64_t n_steps, int32_t *host_tokens) {
    if (!e || n_steps < 0 || !e->finalized) return B200_ERR_INVALID_ARGUMENT;
    if (e->n_past + n_steps > e->c.kv_capacity) return B200_ERR_OUT_OF_RANGE;
    if (n_steps > e->log_cap) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    cudaStream_t st = e->stream;
    int rc = build_graph(e);
    if (rc == B200_OK) rc = mk_account(e, n_steps);
    if (rc != B200_OK) return rc;
    // the input token, restored if a step fails (each completed step advances the
    // device token and n_past)
    int32_t *saved_tok = e->pinned_io + e->io_tok + 2;
    B200_TRY(cudaMemcpyAsync(saved_tok, e->token, 4, cudaMemcpyDeviceToHost, st));
    B200_TRY(cudaMemsetAsync(e->log_pos, 0, 4, st));
    for (int64_t i = 0; i < n_steps; ++i) B200_TRY(cudaGraphLaunch(e->graph_exec, st));
    if (host_tokens && n_steps > 0)
        B200_TRY(cudaMemcpyAsync(host_tokens, e->token_log, n_steps * 4, cudaMemcpyDeviceToHost, st));
    rc = check_status(e);
    if (rc != B200_OK) {
        // Nothing is committed: the steps before the failing one advanced the device
        // n_past and token; both go back to the state before the call, so the next
        // eval / generate continues from the last committed position (the KV rows
        // those steps wrote are overwritten then).
        int rr = restore_n_past(e);
        if (rr == B200_OK) {
            const cudaError_t ce = cudaMemcpyAsync(e->token, saved_tok, 4, cudaMemcpyHostToDevice, st);
            rr = from_cuda(ce == cudaSuccess ? cudaStreamSynchronize(st) : ce);
        }
        return rr != B200_OK ? rr : rc;
    }
    e->n_past += n_steps;
    return B200_OK;
}

int b200_engine_profile_step(b200_engine *e, char *names, int name_len, float *us, int max_ops) {
    if (!e || !e->finalized || !names || !us || max_ops <= 0 || name_len <= 1) return B200_ERR_INVALID_ARGUMENT;
    if (e->tp || e->n_past + 1 > e->c.kv_capacity) return B200_ERR_NOT_SUPPORTED;
    DeviceGuard dg(e->device);
    cudaStream_t st = e->stream;
    // One eager decode step (no graph, no programmatic overlap) with an event after
    // every launch. n_past and the token slot are restored afterwards, so the step
    // leaves no trace beyond a KV row that the next real step overwrites.
    int32_t saved[2];
    B200_TRY(cudaMemcpyAsync(&saved[0], e->n_past_dev, 4, cudaMemcpyDeviceToHost, st));
    B200_TRY(cudaMemcpyAsync(&saved[1], e->token, 4, cudaMemcpyDeviceToHost, st));
    std::vector<cudaEvent_t> evs;
    std::vector<const char *> nms;
    cudaEvent_t start;
    B200_TRY(cudaEventCreate(&start));
    B200_TRY(cudaEventRecord(start, st));
    e->prof_events = &evs;
    e->prof_names = &nms;
    const int rc = enqueue_small_step(e, e->token, 1, false, 1, false);
    e->prof_events = nullptr;
    e->prof_names = nullptr;
    cudaError_t err = cudaStreamSynchronize(st);
    std::vector<std::string> uniq;
    std::vector<float> tot;
    cudaEvent_t prev = start;
    for (size_t i = 0; i < evs.size() && err == cudaSuccess; ++i) {
        float ms = 0.f;
        err = cudaEventElapsedTime(&ms, prev, evs[i]);
        prev = evs[i];
        size_t k = 0;
        while (k < uniq.size() && uniq[k] != nms[i]) ++k;
        if (k == uniq.size()) {
            uniq.push_back(nms[i]);
            tot.push_back(0.f);
        }
        tot[k] += ms * 1000.f;
    }
    for (auto ev : evs) cudaEventDestroy(ev);
    cudaEventDestroy(start);
    cudaMemcpyAsync(e->n_past_dev, &saved[0], 4, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(e->token, &saved[1], 4, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
    if (rc != B200_OK) return rc;
    if (err != cudaSuccess) return from_cuda(err);
    const int n = static_cast<int>(uniq.size() < static_cast<size_t>(max_ops) ? uniq.size() : max_ops);
    for (int i = 0; i < n; ++i) {
        std::strncpy(names + static_cast<size_t>(i) * name_len, uniq[i].c_str(), name_len - 1);
        names[static_cast<size_t>(i) * name_len + name_len - 1] = 0;
        us[i] = tot[i];
    }
    return n;
}

int b200_engine_trace_step(b200_engine *e, unsigned long long *host_trace, int max_kernels) {
    if (!e || !e->finalized || !host_trace || max_kernels <= 0) return B200_ERR_INVALID_ARGUMENT;
    if (e->tp || e->n_past + 1 > e->c.kv_capacity) return B200_ERR_NOT_SUPPORTED;
    DeviceGuard dg(e->device);
    cudaStream_t st = e->stream;
    // One decode step captured and replayed exactly like the production graph,
    // with every launch stamping the global timer; n_past and the token slot are
    // restored afterwards.
    int32_t saved[2];
    B200_TRY(cudaMemcpyAsync(&saved[0], e->n_past_dev, 4, cudaMemcpyDeviceToHost, st));
    B200_TRY(cudaMemcpyAsync(&saved[1], e->token, 4, cudaMemcpyDeviceToHost, st));
    std::vector<unsigned long long> init(static_cast<size_t>(e->trace_cap) * 8, 0ull);
    for (int i = 0; i < e->trace_cap; ++i) init[8 * i + 3] = ~0ull;
    B200_TRY(cudaMemcpyAsync(e->trace_buf, init.data(), init.size() * 8, cudaMemcpyHostToDevice, st));
    B200_TRY(cudaStreamSynchronize(st));
    e->trace_on = true;
    e->trace_n = 0;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaError_t err = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    int rc = B200_OK;
    int n = 0;
    if (err == cudaSuccess) {
        if (e->use_mk) {
            MkParams p = e->mk;
            p.trace = e->trace_buf;
            rc = mk_account(e, 1);
            if (rc == B200_OK) rc = from_cuda(mk_launch(p, st));
            n = 5 * e->c.n_layer + 1;
        } else {
            rc = enqueue_small_step(e, e->token, 1, false, 1, true);
        }
        err = cudaStreamEndCapture(st, &g);
    }
    e->trace_on = false;
    if (!e->use_mk) n = e->trace_n;
    if (err == cudaSuccess && rc == B200_OK) err = cudaGraphInstantiate(&ge, g, 0);
    if (err == cudaSuccess && rc == B200_OK) err = cudaGraphLaunch(ge, st);
    if (err == cudaSuccess && rc == B200_OK)
        err = cudaMemcpyAsync(init.data(), e->trace_buf, static_cast<size_t>(n) * 64, cudaMemcpyDeviceToHost, st);
    cudaError_t serr = cudaStreamSynchronize(st);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    cudaMemcpyAsync(e->n_past_dev, &saved[0], 4, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(e->token, &saved[1], 4, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
    if (rc != B200_OK) return rc;
    if (err != cudaSuccess) return from_cuda(err);
    if (serr != cudaSuccess) return from_cuda(serr);
    const int out = n < max_kernels ? n : max_kernels;
    std::memcpy(host_trace, init.data(), static_cast<size_t>(out) * 64);
    return out;
}

void *b200_engine_stream(b200_engine *e) { return e ? e->stream : nullptr; }

int b200_engine_read_status(b200_engine *e, int32_t *status) {
    if (!e || !status) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    B200_TRY(cudaMemcpy(status, e->status, 4, cudaMemcpyDeviceToHost));
    return B200_OK;
}

int b200_tp_unique_id(unsigned char out_id[128]) { return tp_unique_id(out_id); }

int b200_engine_tp_init(b200_engine *e, const unsigned char id[128]) {
    if (!e || !id || e->c.tp_world < 2) return B200_ERR_INVALID_ARGUMENT;
    DeviceGuard dg(e->device);
    int rc = tp_create(&e->tp, id, e->c.tp_rank, e->c.tp_world);
    if (rc != B200_OK) return rc;
    // the decode path's all-reduces (at most 4 rows of H) and token selection over
    // NVLink peer memory; NCCL where a peer is not reachable (B200_TP_NCCL=1 forces it)
    const char *force = std::getenv("B200_TP_NCCL");
    if (!(force && force[0] == '1')) {
        rc = tp_p2p_init(e->tp, 4 * static_cast<int64_t>(e->H) + 2 * e->c.tp_world, e->stream);
        if (rc != B200_OK && rc != B200_ERR_NOT_SUPPORTED) return rc;
    }
    return B200_OK;
}

int b200_engine_tp_peer_exchange(const b200_engine *e) { return e && e->tp && tp_p2p_ready(e->tp) ? 1 : 0; }

}  // extern "C"
