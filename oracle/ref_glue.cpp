// oracle/ref_glue.cpp -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
//
// A thin extern "C" surface over the Infer-LLM reference engine, compiled
// together with the reference's own sources (see oracle/Makefile). It lets the
// Python tests and bench.py's reference leg call:
//   * single reference CPU ops (a Graph with one OpFactory node executed by
//     CPUBackend::compute), the checker that pins oracle/cpu_ops.c, and
//   * the reference end-to-end CPU path: GGUF load, Qwen3Model::build_graph,
//     Scheduler::execute, read_logits and the greedy Sampler, with the request
//     loop of benchmarks/cpu/bench.cpp (Runner::evaluate, bench.cpp:177-219).
// Nothing in the product library links or calls this file.
//
// Built with INFERLLM_WITH_CUDA (oracle/Makefile `ref-b200`), the same glue also
// creates the reference engine on its own CUDA backend (cuda_backend.cpp) whose
// CUDA_F32::compute_* kernels are the B200 library's (infer-llm_b200/integration/
// kernel_b200.cpp): the reference host code driving the product, end to end, as the
// drop-in check. Device placement follows benchmarks/cuda/bench.cpp:146-160,397-410
// (layers and KV on cuda:<d>, embedding on the CPU, synchronize after each step).

#include "backend.hpp"
#include "backends/cpu_backend.hpp"
#include "gguf_parser.hpp"
#include "graph.hpp"
#include "model.hpp"
#include "op_factory.hpp"
#include "sampler.hpp"
#include "scheduler.hpp"
#include "kvcache/kvcacheManager.hpp"
#include "kvcache/KVStorages/naiveKVStorage.hpp"
#include "kvcache/KVStrategys/contiguousKVStrategy.hpp"
#include "paged_kv_strategy.hpp"

#ifdef INFERLLM_WITH_CUDA
#include <cuda_runtime_api.h>
#endif
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <memory>
#include <numeric>
#include <streambuf>
#include <string>
#include <vector>

namespace {

// The reference engine prints progress to std::cout on every call; the glue
// silences it for the duration of each call (as bench.cpp:110-119 does).
class Quiet {
    struct Sink : std::streambuf {
        int_type overflow(int_type c) override { return traits_type::not_eof(c); }
        std::streamsize xsputn(const char *, std::streamsize n) override { return n; }
    } sink_;
    std::streambuf *old_;

public:
    Quiet() : old_(std::cout.rdbuf(&sink_)) {}
    ~Quiet() { std::cout.rdbuf(old_); }
};

std::unique_ptr<Backend> g_cpu;
int g_cpu_threads = -1;

Backend *cpu_backend(int threads) {
    if (g_cpu && (threads <= 0 || threads == g_cpu_threads)) return g_cpu.get();
    Quiet q;
    if (threads > 0) setenv("INFERLLM_THREADS", std::to_string(threads).c_str(), 1);
    static bool registered = false;
    if (!registered) {
        register_all_backends();
        registered = true;
    }
    auto &reg = BackendRegistry::instance();
    reg.probe_all();
    g_cpu.reset();
    auto b = reg.create("cpu", PoolConfig{});
    if (!b) return nullptr;
    g_cpu = std::move(*b);
    g_cpu_threads = static_cast<const CPUBackend *>(g_cpu.get())->get_n_threads();
    return g_cpu.get();
}

Tensor *leaf(Graph &g, const char *name, DataType type, std::initializer_list<int64_t> shape,
             const void *data, Backend *b) {
    auto t = std::make_unique<Tensor>(name, type, shape);
    t->data = const_cast<void *>(data);
    t->backend = b;
    t->device = DeviceType::CPU;
    return g.add_node(std::move(t));
}

int run_one(Graph &g, Tensor *out, void *out_data, Backend *b) {
    out->data = out_data;
    out->backend = b;
    g.mark_output(out);
    if (!g.compute()) return -2;
    if (!b->compute(g)) return -3;
    return 0;
}

}  // namespace

extern "C" {

int ref_set_threads(int threads) {
    Backend *b = cpu_backend(threads);
    return b ? g_cpu_threads : -1;
}

int ref_mul_mat(const float *w, const float *x, float *out, int64_t K, int64_t N, int64_t M) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    Graph g;
    Tensor *W = leaf(g, "w", GGML_TYPE_F32, {K, N}, w, b);
    Tensor *X = leaf(g, "x", GGML_TYPE_F32, {K, M}, x, b);
    return run_one(g, OpFactory::mul_mat(g, W, X), out, b);
}

int ref_rms_norm(const float *x, const float *gamma, float *out, int64_t D, int64_t rows, float eps) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    Graph g;
    Tensor *X = leaf(g, "x", GGML_TYPE_F32, {D, rows}, x, b);
    Tensor *G = leaf(g, "gamma", GGML_TYPE_F32, {D}, gamma, b);
    return run_one(g, OpFactory::rms_norm(g, X, G, eps), out, b);
}

// Copies the reference's own host RoPE angle table (GraphContext, graph.cpp:92-135).
int ref_rope_theta_table(float theta, uint32_t head_dim, uint32_t n_ctx, float *out) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    GraphContext ctx(b);
    auto t = ctx.get_rope_theta_table(theta, head_dim, n_ctx);
    if (!t) return -2;
    std::memcpy(out, (*t)->data, sizeof(float) * (head_dim / 2) * static_cast<size_t>(n_ctx));
    return 0;
}

int ref_rope(const float *x, const int32_t *pos, float theta, uint32_t n_ctx, float *out,
             int64_t D, int64_t H, int64_t T) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    GraphContext ctx(b);
    auto table = ctx.get_rope_theta_table(theta, static_cast<uint32_t>(D), n_ctx);
    if (!table) return -2;
    Graph g;
    Tensor *X = leaf(g, "x", GGML_TYPE_F32, {D, H, T}, x, b);
    Tensor *P = leaf(g, "pos", GGML_TYPE_I32, {T}, pos, b);
    return run_one(g, OpFactory::rope(g, X, P, *table), out, b);
}

int ref_flash_attn(const float *qp, const float *kp, const float *vp, float *out, int64_t D,
                   int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tkv, int64_t n_past) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    Graph g;
    Tensor *Q = leaf(g, "q", GGML_TYPE_F32, {D, Hq, Tq}, qp, b);
    Tensor *K = leaf(g, "k", GGML_TYPE_F32, {D, Hkv, Tkv}, kp, b);
    Tensor *V = leaf(g, "v", GGML_TYPE_F32, {D, Hkv, Tkv}, vp, b);
    AttnParams p;
    p.n_head = static_cast<uint32_t>(Hq);
    p.n_head_kv = static_cast<uint32_t>(Hkv);
    p.head_dim = static_cast<uint32_t>(D);
    p.scale = 1.0f / std::sqrt(float(D));
    p.causal = true;
    p.n_ctx = static_cast<uint32_t>(n_past);
    return run_one(g, OpFactory::flash_attn(g, Q, K, V, p), out, b);
}

int ref_silu(const float *x, float *out, int64_t n) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    Graph g;
    Tensor *X = leaf(g, "x", GGML_TYPE_F32, {n}, x, b);
    return run_one(g, OpFactory::silu(g, X), out, b);
}

int ref_binary(int op, const float *a, const float *bb, float *out, int64_t n) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    Graph g;
    Tensor *A = leaf(g, "a", GGML_TYPE_F32, {n}, a, b);
    Tensor *B = leaf(g, "b", GGML_TYPE_F32, {n}, bb, b);
    return run_one(g, op == 0 ? OpFactory::add(g, A, B) : OpFactory::mul(g, A, B), out, b);
}

int ref_get_rows(const float *table, const int32_t *ids, float *out, int64_t D, int64_t n,
                 int64_t n_rows) {
    Backend *b = cpu_backend(0);
    if (!b) return -1;
    Quiet q;
    Graph g;
    Tensor *T = leaf(g, "table", GGML_TYPE_F32, {D, n_rows}, table, b);
    Tensor *I = leaf(g, "ids", GGML_TYPE_I32, {n}, ids, b);
    return run_one(g, OpFactory::embedding(g, T, I), out, b);
}

int32_t ref_sample_greedy(const float *logits, int64_t n) {
    Sampler s;
    auto r = s.sample(std::span<const float>(logits, static_cast<size_t>(n)));
    return r ? *r : -1;
}

// ---------------------------------------------------------------------------
// End-to-end reference CPU engine (one sequence at a time).

struct RefEngine {
    std::unique_ptr<Backend> gpu;  // the reference CUDA backend, or null (CPU engine)
    std::unique_ptr<ModelBase> model;
    std::unique_ptr<KVCacheManager> cache;
    std::unique_ptr<GraphContext> ctx;
    std::vector<Backend *> devices;
    std::unique_ptr<Scheduler> scheduler;
    SequenceId seq = kInvalidSequenceId;
    Tensor *tokens = nullptr, *pos = nullptr;
    std::vector<int32_t> ids, positions;
    int64_t n_vocab = 0;
};

static void *engine_create(const char *gguf_path, int threads, int64_t capacity, int cuda_device) {
    Backend *b = cpu_backend(threads);
    if (!b) return nullptr;
    Quiet q;
    std::unique_ptr<Backend> gpu;
    if (cuda_device >= 0) {
        auto g = BackendRegistry::instance().create("cuda:" + std::to_string(cuda_device), PoolConfig{});
        if (!g) return nullptr;
        gpu = std::move(*g);
    }
    Backend *dev = gpu ? gpu.get() : b;  // where the layers and the KV cache live
    auto gguf = GGUFContext::load(gguf_path);
    if (!gguf) return nullptr;
    auto arch = gguf->metadata().get_meta<std::string>("general.architecture");
    if (!arch) return nullptr;
    auto n_layer = gguf->metadata().get_meta<uint32_t>(*arch + ".block_count");
    auto kv_heads = gguf->metadata().get_meta<uint32_t>(*arch + ".attention.head_count_kv");
    auto kd = gguf->metadata().get_meta<uint32_t>(*arch + ".attention.key_length");
    auto vd = gguf->metadata().get_meta<uint32_t>(*arch + ".attention.value_length");
    if (!n_layer || !kv_heads || !kd || !vd) return nullptr;
    static bool models_registered = false;
    if (!models_registered) {
        register_all_models();
        models_registered = true;
    }
    auto e = std::make_unique<RefEngine>();
    e->gpu = std::move(gpu);
    auto model = ModelBase::load_model(std::move(*gguf));
    if (!model) return nullptr;
    e->model = std::move(*model);
    if (!e->model->load_hparams() || !e->model->load_weight()) return nullptr;
    e->devices = e->gpu ? std::vector<Backend *>{dev, b} : std::vector<Backend *>{b};
    PlacementConfig placement;
    placement.n_ctx = static_cast<uint32_t>(capacity);
    if (!e->model->plan_weights_placement(e->devices, placement)) return nullptr;
    std::vector<KVLayerSpec> layers(*n_layer, KVLayerSpec{.n_kv_heads = *kv_heads,
                                                           .k_head_dim = *kd,
                                                           .v_head_dim = *vd,
                                                           .k_type = GGML_TYPE_F32,
                                                           .v_type = GGML_TYPE_F32});
    e->cache = std::make_unique<KVCacheManager>(
        std::make_unique<ContiguousKVStrategy>(std::make_unique<NaiveKVStorage>()));
    std::vector<Backend *> placement_layers(layers.size(), dev);
    KVCacheConfig config{.layers = layers.size(), .max_tokens_per_sequence = static_cast<size_t>(capacity)};
    if (!e->cache->init(layers, placement_layers, config)) return nullptr;
    e->ctx = std::make_unique<GraphContext>(b);
    e->scheduler = std::make_unique<Scheduler>(e->devices);
    e->tokens = e->ctx->make_tensor("bench_tokens", DataType::GGML_TYPE_I32, {1});
    e->pos = e->ctx->make_tensor("bench_positions", DataType::GGML_TYPE_I32, {1});
    for (Tensor *t : {e->tokens, e->pos}) {
        t->tensorRole = TensorRole::TNESOR_ROLE_INPUT;
        t->backend = b;
        t->device = DeviceType::CPU;
    }
    e->ctx->set_input_tokens(e->tokens);
    e->ctx->set_input_pos(e->pos);
    auto seq = e->cache->create_sequence();
    if (!seq) return nullptr;
    e->seq = *seq;
    if (!e->ctx->set_kv_cache(e->cache.get(), e->seq)) return nullptr;
    return e.release();
}

void *ref_engine_create(const char *gguf_path, int threads, int64_t capacity) {
    return engine_create(gguf_path, threads, capacity, -1);
}

// The reference engine on its CUDA backend (null unless built with INFERLLM_WITH_CUDA).
void *ref_engine_create_cuda(const char *gguf_path, int threads, int64_t capacity, int device) {
#ifdef INFERLLM_WITH_CUDA
    return engine_create(gguf_path, threads, capacity, device);
#else
    (void)gguf_path, (void)threads, (void)capacity, (void)device;
    return nullptr;
#endif
}

void ref_engine_destroy(void *h) {
    auto *e = static_cast<RefEngine *>(h);
    if (!e) return;
    Quiet q;
    (void)e->ctx->release_kv_access();
    if (e->seq != kInvalidSequenceId) (void)e->cache->release_sequence(e->seq);
    delete e;
}

// Starts a new request: drops the sequence's KV and creates a fresh one.
int ref_engine_reset(void *h) {
    auto *e = static_cast<RefEngine *>(h);
    Quiet q;
    if (!e->ctx->release_kv_access()) return -1;
    if (!e->cache->release_sequence(e->seq)) return -1;
    if (!e->ctx->set_kv_cache(nullptr, kInvalidSequenceId)) return -1;
    auto seq = e->cache->create_sequence();
    if (!seq) return -1;
    e->seq = *seq;
    if (!e->ctx->set_kv_cache(e->cache.get(), e->seq)) return -1;
    return 0;
}

// Drives infer-llm_b200/integration/paged_kv_strategy.cpp through the reference's
// own KVCacheManager + NaiveKVStorage on the CPU backend: two appends of `first` and
// `second` tokens across block boundaries (views written and read back through the
// manager's segment views), an aborted append (its blocks freed again), and the
// block table the paged kernels take. Returns 0, or the number of the failed check.
// out[0] = segments of the second append's readable view, out[1] = blocks held.
int ref_paged_kv_selftest(int64_t block_tokens, int64_t n_layer, int64_t first, int64_t second, int64_t *out) {
    Backend *cpu = cpu_backend(0);
    if (!cpu) return 1;
    Quiet q;
    constexpr std::size_t Hkv = 2, D = 8, HD = Hkv * D;
    std::vector<KVLayerSpec> layers(static_cast<size_t>(n_layer),
                                    KVLayerSpec{.n_kv_heads = Hkv, .k_head_dim = D, .v_head_dim = D,
                                                .k_type = GGML_TYPE_F32, .v_type = GGML_TYPE_F32});
    auto strategy = std::make_unique<PagedKVStrategy>(std::make_unique<NaiveKVStorage>());
    PagedKVStrategy *paged = strategy.get();
    KVCacheManager mgr(std::move(strategy));
    std::vector<Backend *> place(layers.size(), cpu);
    KVCacheConfig cfg{.layers = layers.size(), .max_tokens_per_sequence = 4096,
                      .block_tokens = static_cast<size_t>(block_tokens)};
    if (!mgr.init(layers, place, cfg)) return 2;
    auto seq = mgr.create_sequence();
    if (!seq) return 3;
    auto value = [](size_t layer, size_t pos, bool is_v) { return float(layer * 100000 + pos * 2 + (is_v ? 1 : 0)); };
    // append [0, first) then [first, first + second); write the new rows through the
    // writable segments, then read every row back through the readable segments
    size_t done = 0;
    for (int64_t n : {first, second}) {
        if (!mgr.reserve_append(*seq, static_cast<size_t>(n))) return 4;
        for (size_t l = 0; l < layers.size(); ++l) {
            auto acc = mgr.acquire_layer(*seq, l);
            if (!acc) return 5;
            size_t pos = done;
            for (size_t i = 0; i < acc->writable.k.size(); ++i) {
                const KVSegmentView &ks = acc->writable.k[i], &vs = acc->writable.v[i];
                if (ks.token_begin != pos || ks.token_count == 0 || ks.token_count > cfg.block_tokens) return 6;
                for (size_t t = 0; t < ks.token_count; ++t)
                    for (size_t e = 0; e < HD; ++e) {
                        static_cast<float *>(ks.view.data)[t * HD + e] = value(l, pos + t, false);
                        static_cast<float *>(vs.view.data)[t * HD + e] = value(l, pos + t, true);
                    }
                pos += ks.token_count;
            }
            if (pos != done + static_cast<size_t>(n)) return 7;
            size_t rpos = 0;
            for (size_t i = 0; i < acc->readable.k.size(); ++i) {
                const KVSegmentView &ks = acc->readable.k[i], &vs = acc->readable.v[i];
                if (ks.token_begin != rpos) return 8;
                for (size_t t = 0; t < ks.token_count; ++t)
                    for (size_t e = 0; e < HD; e += 7)
                        if (static_cast<float *>(ks.view.data)[t * HD + e] != value(l, rpos + t, false) ||
                            static_cast<float *>(vs.view.data)[t * HD + e] != value(l, rpos + t, true))
                            return 9;
                rpos += ks.token_count;
            }
            if (rpos != pos) return 10;
            if (l == 0 && out) out[0] = static_cast<int64_t>(acc->readable.k.size());
            if (!mgr.release_layer(*acc)) return 11;
        }
        if (!mgr.commit_append(*seq)) return 12;
        done += static_cast<size_t>(n);
    }
    const size_t held = paged->blocks(*seq, 0);
    if (held != (done + cfg.block_tokens - 1) / cfg.block_tokens) return 13;
    // an aborted append gives its new blocks back
    if (!mgr.reserve_append(*seq, cfg.block_tokens + 1)) return 14;
    if (paged->blocks(*seq, 0) <= held) return 15;
    if (!mgr.abort_append(*seq)) return 16;
    if (paged->blocks(*seq, 0) != held) return 17;
    // the kernels' block table: position p at k[p / bt] + (p % bt) * HD
    std::vector<void *> kt, vt;
    if (!paged->block_table(*seq, n_layer - 1, done, kt, vt)) return 18;
    for (size_t p = 0; p < done; ++p) {
        const float *kb = static_cast<const float *>(kt[p / cfg.block_tokens]);
        const float *vb = static_cast<const float *>(vt[p / cfg.block_tokens]);
        const size_t o = (p % cfg.block_tokens) * HD;
        if (kb[o] != value(n_layer - 1, p, false) || vb[o + HD - 1] != value(n_layer - 1, p, true)) return 19;
    }
    if (out) out[1] = static_cast<int64_t>(held);
    if (!mgr.release_sequence(*seq)) return 20;
    return 0;
}

// The device backend of an engine (null for a CPU engine): lets a test query the
// backend a drop-in build registered (b200_backend_counters).
void *ref_engine_backend(void *h) { return static_cast<RefEngine *>(h)->gpu.get(); }

// One evaluation step (prefill when n > 1, decode when n == 1), the body of
// bench.cpp Runner::evaluate. Writes the last row's logits (if non-null) and
// returns the greedy token, or a negative code.
int32_t ref_engine_eval(void *h, const int32_t *ids, int64_t n, float *last_logits) {
    auto *e = static_cast<RefEngine *>(h);
    Quiet q;
    auto n_past = e->cache->length(e->seq);
    if (!n_past) return -1;
    if (!e->cache->reserve_append(e->seq, static_cast<size_t>(n))) return -2;
    e->ids.assign(ids, ids + n);
    e->positions.resize(static_cast<size_t>(n));
    std::iota(e->positions.begin(), e->positions.end(), static_cast<int32_t>(*n_past));
    const int64_t bytes = n * static_cast<int64_t>(sizeof(int32_t));
    for (Tensor *t : {e->tokens, e->pos}) {
        t->dims = {n, 1, 1, 1};
        t->strides = {static_cast<int64_t>(sizeof(int32_t)), bytes, bytes, bytes};
    }
    e->tokens->data = e->ids.data();
    e->pos->data = e->positions.data();
    int32_t token = -3;
    {
        auto graph = e->model->build_graph(*e->ctx);
        if (!graph) goto fail;
        if (!graph->compute()) goto fail;
        if (!e->scheduler->execute(*graph)) goto fail;
#ifdef INFERLLM_WITH_CUDA
        if (e->gpu && cudaDeviceSynchronize() != cudaSuccess) goto fail;  // bench.cpp:210-213
#endif
        auto logits = read_logits(*graph->outputs().front(), static_cast<size_t>(n - 1));
        if (!logits) goto fail;
        if (last_logits) std::memcpy(last_logits, logits->data(), sizeof(float) * logits->size());
        e->n_vocab = static_cast<int64_t>(logits->size());
        Sampler s;
        auto tok = s.sample(*logits);
        token = tok ? *tok : -4;
    }
    if (!e->ctx->release_kv_access()) return -5;
    if (!e->cache->commit_append(e->seq)) return -6;
    return token;
fail:
    (void)e->ctx->release_kv_access();
    (void)e->cache->abort_append(e->seq);
    return -3;
}

}  // extern "C"
