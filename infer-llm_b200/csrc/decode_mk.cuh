// Persistent single-launch decode step (one token through every layer + LM head).
#pragma once

#include "common.cuh"

namespace b200 {

struct MkLayer {
    const float *attn_norm, *wqkv, *q_norm, *k_norm, *wo, *ffn_norm, *wgu, *wdown;
    float *kc, *vc;  // KV object of the layer: K block [cap][Hkv][D], V block
};

struct MkParams {
    const MkLayer *layers = nullptr;  // device array [n_layer]
    int n_layer = 0;
    int H = 0, D = 0, Hq = 0, Hkv = 0, F = 0, V = 0;
    float eps = 0.f;
    int64_t n_ctx = 0;                 // KV capacity (positions must stay below)
    const float *tok_embd = nullptr, *out_norm = nullptr, *lm_head = nullptr, *freq = nullptr;
    // Activations exchanged between CTAs, as tagged words: (phase tag << 32) | float
    // bits, written with one 64-bit store each. A reader waits for the tag of the
    // phase it needs instead of a grid barrier; tags are unique per launch.
    unsigned long long *tx = nullptr;    // residual [H]
    unsigned long long *tqkv = nullptr;  // [(Hq + 2 Hkv) D]
    unsigned long long *th = nullptr;    // SwiGLU output [F]
    unsigned long long *tpo = nullptr;   // attention split partial outputs [max_splits][Hq][D]
    unsigned long long *tpml = nullptr;  // attention split (max, sum) [max_splits][Hq][2]
    unsigned long long *tao = nullptr;   // merged attention output [Hq][D]
    // Tickets: every CTA of every launch takes one (64-bit: never wraps), launch =
    // ticket / gridDim.x; the tag base is derived from the launch modulo
    // kMkTagPeriod. The engine clears this counter together with the tagged words
    // above before kMkClearEvery launches have run since the last clear, so no word
    // can be as old as one tag period.
    unsigned long long *launches = nullptr;
    float *logits = nullptr;           // [V] or nullptr
    int32_t *token = nullptr;          // in: token of this step; out: greedy next token
    int32_t *n_past = nullptr;         // advanced by 1 at the end of the step
    int32_t *status = nullptr;
    int32_t *token_log = nullptr, *log_pos = nullptr;
    int32_t log_cap = 0;
    float *am_val = nullptr;           // [gridDim.x] per-CTA argmax partials
    int32_t *am_idx = nullptr;
    unsigned *am_counter = nullptr;    // zero at launch; the last CTA re-zeroes it
    unsigned long long *trace = nullptr;  // optional: [5 n_layer + 1] x 8 words (phase stamps)
    int max_inflight = 16;             // ring copies outstanding per CTA (set by mk_launch)
    int split_keys = 32;               // keys per attention split (set by mk_launch)
    // Failure injection for tests (two device ints, zero = none): CTA
    // (withhold[0] - 1) does not publish its layer-0 QKV outputs, as if it had
    // stopped, so the CTAs waiting for them run into their bounded waits; it lets
    // withhold[1] launches pass first (counting them down).
    int32_t *withhold = nullptr;
};

// Tags are (launch mod kMkTagPeriod + 1) * 256 + phase: 32-bit, never 0 (cleared
// words never match). Launches between two clears stay below kMkClearEvery.
constexpr unsigned long long kMkTagPeriod = (1ull << 24) - 1;
constexpr long long kMkClearEvery = 1ll << 23;

// True if the megakernel supports this model shape on this device.
bool mk_supported(const MkParams &p);
int mk_max_splits();
// Words of the split-partial buffers tpo / tpml.
size_t mk_po_words(const MkParams &p);
size_t mk_pml_words(const MkParams &p);
// Enqueues the cooperative launch.
cudaError_t mk_launch(const MkParams &p, cudaStream_t stream);
int mk_grid();
int mk_max_inflight();
int mk_split_keys();

}  // namespace b200
