// The B200 "cuda" backend: a drop-in for the reference's src/backends/cuda_backend.cpp.
//
// A maintainer keeps the reference's engine (model graph, scheduler, KV cache
// manager, activation manager) and builds this file instead of cuda_backend.cpp, with
// integration/kernel_b200.cpp instead of src/kernels/cuda/kernel_f32.cu, linked with
// libb200infer.so (oracle/Makefile `ref-b200be` builds exactly that). It registers
// the backend under the reference's name "cuda" (cuda_backend.cpp:41-51), with the
// reference's probe (one "cuda:<i>" per device, free bytes as memory_bytes), and
// implements every virtual of Backend (include/backend.hpp:43-115):
//
//  * alloc / free: WEIGHTS one device allocation per request (the model asks once per
//    device for its whole weight arena, model.cpp:545-575); KVCACHE and ACTIVATION
//    come from two pre-sized device arenas reserved at the first request of each
//    kind (B200_KV_ARENA_MB / B200_ACT_ARENA_MB, default 4096 / 1024 MiB), carved
//    with a bump pointer that rewinds once every block of the arena is free -- no
//    cudaMalloc per KV object or per activation plan (the reference's NaivePool
//    mallocs each, naivePool.hpp:6-21). A request that does not fit falls back to
//    its own allocation.
//  * copy_tensor_set / _get: synchronous host <-> device copies, as the reference's
//    (the sampler reads logits right after, sampler.cpp:31).
//  * copy_tensor_high: device sources are copied at once (peer copy across devices);
//    host sources (the CPU embedding rows, the positions, the RoPE angle table) are
//    deferred to compute(), which performs them only if it runs the graph op by op.
//  * compute(Graph&): a subgraph that is a whole Qwen3 step (Qwen3.cpp:4-136: every
//    layer from the embedding rows to the logits) runs on the B200 engine
//    (b200_engine_*): the embedding gathered on the device from the token ids, no
//    angle-table upload (the engine keeps the 64 frequencies, row 1 of the table),
//    the K / V of the step appended in place to the reference's own KV objects (the
//    engine binds them), the fused kernel sequence or single-launch decode step, and
//    the last row's logits written into the graph's logits tensor (read_logits takes
//    row M - 1; rows 0..M-2 are not computed). Any other subgraph runs node by node
//    through CUDA_F32::compute_* (kernel_b200.cpp) on the backend's stream, as
//    cuda_backend.cpp:181-238 does.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "b200_infer.h"
#include "backend.hpp"
#include "cuda_util.hpp"
#include "kernels/cuda/kernel_f32.hpp"
#include "op_params.hpp"
#include "tensor.hpp"

namespace {

std::unexpected<std::error_code> fail(std::errc e) { return std::unexpected(std::make_error_code(e)); }

// A pre-sized device arena: bump allocation (256-byte aligned), rewound when every
// block handed out has been freed.
class DeviceArena {
public:
    ~DeviceArena() {
        if (base_) cudaFree(base_);
        for (auto &kv : own_) cudaFree(kv.first);
    }
    void *alloc(size_t bytes, size_t reserve_bytes) {
        if (!base_ && reserve_bytes && cudaMalloc(&base_, reserve_bytes) == cudaSuccess) {
            cap_ = reserve_bytes;
        } else if (!base_) {
            cudaGetLastError();
        }
        const size_t need = (bytes + 255) / 256 * 256;
        if (base_ && top_ + need <= cap_) {
            void *p = static_cast<char *>(base_) + top_;
            top_ += need;
            ++live_;
            return p;
        }
        void *p = nullptr;  // does not fit: its own allocation
        if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        own_[p] = bytes;
        return p;
    }
    void free(void *p) {
        auto it = own_.find(p);
        if (it != own_.end()) {
            cudaFree(p);
            own_.erase(it);
            return;
        }
        if (base_ && p >= base_ && p < static_cast<char *>(base_) + cap_ && live_ > 0 && --live_ == 0) top_ = 0;
    }

private:
    void *base_ = nullptr;
    size_t cap_ = 0, top_ = 0, live_ = 0;
    std::map<void *, size_t> own_;
};

size_t env_mb(const char *name, size_t def_mb) {
    const char *v = std::getenv(name);
    const long long x = (v && *v) ? std::atoll(v) : static_cast<long long>(def_mb);
    return static_cast<size_t>(x > 0 ? x : 0) << 20;
}

// Prefill precision of the engine steps: B200_PREFILL_PRECISION=tf32 selects the
// tcgen05 TF32 prefill (GEMMs and attention, the stated 2e-3 logit bound); anything
// else, or unset, the exact F32 path. Decode is exact either way.
int32_t prefill_precision() {
    const char *v = std::getenv("B200_PREFILL_PRECISION");
    return (v && std::strcmp(v, "tf32") == 0) ? B200_PREC_TF32 : B200_PREC_FFMA;
}

bool named(const Tensor *t, const std::string &n) { return t && t->name == n; }

// The host tensor behind a scheduler copy ("<name>_##copy##", src[0] = the source).
const Tensor *host_source(const Tensor *t) {
    if (!t) return nullptr;
    if (t->backend && t->backend->is_host()) return t;
    const Tensor *s = t->src[0];
    if (s && s->backend && s->backend->is_host() && t->name == s->name + "_##copy##") return s;
    return nullptr;
}

class B200Backend final : public Backend {
public:
    B200Backend(int device_id, DeviceInfo info, const PoolConfig &cfg) : Backend(device_id, std::move(info), cfg) {
        cudaSetDevice(_device_id);
        check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    }
    ~B200Backend() override {
        cudaSetDevice(_device_id);
        if (engine_) b200_engine_destroy(engine_);
        for (void *p : weights_) cudaFree(p);
        kv_.reset();
        act_.reset();
        if (stream_) cudaStreamDestroy(stream_);
    }

    DeviceType device_type() const override { return DeviceType::CUDA; }
    std::string device_name() const override { return "CUDA:" + std::to_string(_device_id); }
    bool supports_op(OperationType, const Tensor &) const override { return true; }
    bool is_host() const override { return false; }

    std::expected<void *, std::error_code> alloc(BufferKind kind, size_t bytes) override {
        cudaSetDevice(_device_id);
        void *p = nullptr;
        switch (kind) {
            case BufferKind::WEIGHTS:
                if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
                    cudaGetLastError();
                    return fail(std::errc::not_enough_memory);
                }
                weights_.push_back(p);
                return p;
            case BufferKind::KVCACHE:
                p = kv_->alloc(bytes, env_mb("B200_KV_ARENA_MB", 4096));
                break;
            case BufferKind::ACTIVATION:
                p = act_->alloc(bytes, env_mb("B200_ACT_ARENA_MB", 1024));
                break;
            default:
                return fail(std::errc::invalid_argument);
        }
        if (!p) return fail(std::errc::not_enough_memory);
        return p;
    }

    void free(BufferKind kind, void *ptr) override {
        if (!ptr) return;
        cudaSetDevice(_device_id);
        switch (kind) {
            case BufferKind::WEIGHTS:
                for (size_t i = 0; i < weights_.size(); ++i)
                    if (weights_[i] == ptr) {
                        cudaFree(ptr);
                        weights_.erase(weights_.begin() + static_cast<long>(i));
                        break;
                    }
                break;
            case BufferKind::KVCACHE: kv_->free(ptr); break;
            case BufferKind::ACTIVATION: act_->free(ptr); break;
            default: break;
        }
    }

    std::expected<void, std::error_code> copy_tensor_set(Tensor *t, const void *data, size_t offset,
                                                         size_t size) override {
        if (!t || !t->data || !data || offset + size > t->byte_size()) return fail(std::errc::invalid_argument);
        cudaSetDevice(_device_id);
        if (auto r = check_cuda(cudaMemcpyAsync(static_cast<char *>(t->data) + offset, data, size,
                                                cudaMemcpyHostToDevice, stream_));
            !r)
            return r;
        return check_cuda(cudaStreamSynchronize(stream_));
    }

    std::expected<void, std::error_code> copy_tensor_get(const Tensor *t, void *data, size_t offset,
                                                         size_t size) override {
        if (!t || !t->data || !data || offset + size > t->byte_size()) return fail(std::errc::invalid_argument);
        cudaSetDevice(_device_id);
        if (auto r = check_cuda(cudaMemcpyAsync(data, static_cast<const char *>(t->data) + offset, size,
                                                cudaMemcpyDeviceToHost, stream_));
            !r)
            return r;
        return check_cuda(cudaStreamSynchronize(stream_));
    }

    std::expected<bool, std::error_code> copy_tensor_high(const Tensor *src, Tensor *dst) const override {
        if (!src || !dst || !src->backend || !dst->backend || !src->data || !dst->data) return false;
        auto *self = const_cast<B200Backend *>(this);
        if (src->backend->is_host()) {  // performed by compute() if the graph runs op by op
            self->pending_.push_back({src, dst});
            return true;
        }
        auto *peer = dynamic_cast<const B200Backend *>(src->backend);
        if (!peer) return false;
        cudaSetDevice(_device_id);
        const cudaError_t e = peer->_device_id == _device_id
                                  ? cudaMemcpyAsync(dst->data, src->data, src->byte_size(), cudaMemcpyDeviceToDevice,
                                                    stream_)
                                  : cudaMemcpyPeerAsync(dst->data, _device_id, src->data, peer->_device_id,
                                                        src->byte_size(), stream_);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if (auto r = check_cuda(cudaStreamSynchronize(stream_)); !r) return std::unexpected(r.error());
        return true;
    }

    std::expected<void, std::error_code> compute(Graph &g) override {
        cudaSetDevice(_device_id);
        Step st;
        if (match_step(g, &st)) {
            auto r = run_step(st);
            pending_.clear();
            if (r || r.error() != std::make_error_code(std::errc::not_supported)) return r;
            // the engine declined (e.g. a prefill longer than its activation arena):
            // the same step op by op below
            st = Step{};
        }
        return run_ops(g);
    }

    // steps the engine ran / subgraphs run op by op (for tests)
    long engine_steps = 0, op_graphs = 0;

private:
    struct Pending {
        const Tensor *src;
        Tensor *dst;
    };
    struct Step {
        int n_layer = 0;
        int64_t M = 0, n_past = 0;
        const int32_t *ids = nullptr;   // host token ids [M]
        const float *embd = nullptr;    // host token_embd [V][H]
        const float *table = nullptr;   // host RoPE angle table [n_ctx][D/2]
        int64_t n_ctx_train = 0;
        float eps = 0.f;
        std::map<std::string, const Tensor *> w;  // weights of the subgraph by name
        std::vector<float *> kc, vc;    // the layers' KV objects (K block, V block)
        Tensor *logits = nullptr;
    };

    // Runs deferred host -> device copies, then every node through CUDA_F32.
    std::expected<void, std::error_code> run_ops(Graph &g) {
        ++op_graphs;
        for (const Pending &p : pending_)
            if (auto r = check_cuda(cudaMemcpyAsync(p.dst->data, p.src->data, p.src->byte_size(),
                                                    cudaMemcpyHostToDevice, stream_));
                !r) {
                pending_.clear();
                return r;
            }
        pending_.clear();
        for (Tensor *node : g.nodes()) {
            if (node->op == OperationType::GGML_OP_NONE) continue;
            auto r = dispatch(node);
            if (!r) {
                std::cerr << "[b200] compute failed at node: " << node->name << " op=" << static_cast<int>(node->op)
                          << "\n";
                return r;
            }
        }
        return {};
    }

    std::expected<void, std::error_code> dispatch(Tensor *n) {
        switch (n->op) {
            case OperationType::GGML_OP_ADD: return check_cuda(CUDA_F32::compute_add(n, stream_));
            case OperationType::GGML_OP_MUL: return check_cuda(CUDA_F32::compute_mul(n, stream_));
            case OperationType::GGML_OP_UNARY: {
                uint32_t op = 0;
                std::memcpy(&op, &n->op_params[0], 4);
                if (static_cast<OperationType_unary_op>(op) == OperationType_unary_op::GGML_UNARY_OP_SILU)
                    return check_cuda(CUDA_F32::compute_silu(n, stream_));
                return fail(std::errc::not_supported);
            }
            case OperationType::GGML_OP_RMS_NORM: return check_cuda(CUDA_F32::compute_rms_norm(n, stream_));
            case OperationType::GGML_OP_GET_ROWS: return check_cuda(CUDA_F32::compute_get_rows(n, stream_));
            case OperationType::GGML_OP_MUL_MAT: return check_cuda(CUDA_F32::compute_mul_mat(n, stream_));
            case OperationType::GGML_OP_RESHAPE: return check_cuda(CUDA_F32::compute_reshape(n, stream_));
            case OperationType::GGML_OP_ROPE: return check_cuda(CUDA_F32::compute_rope(n, stream_));
            case OperationType::GGML_OP_FLASH_ATTN_EXT: return check_cuda(CUDA_F32::compute_flash_attn(n, stream_));
            case OperationType::GGML_OP_CPY: return check_cuda(CUDA_F32::compute_cpy(n, stream_));
            case OperationType::GGML_OP_VIEW: return check_cuda(CUDA_F32::compute_view(n, stream_));
            case OperationType::GGML_OP_NONE: return {};
            default: return fail(std::errc::not_supported);
        }
    }

    // True if `g` is one whole Qwen3 step as Qwen3Model::build_graph emits it (node
    // names and ops of Qwen3.cpp:46-129: 26 nodes per layer, the final norm, the
    // logits), with everything the engine needs reachable on the host or this device.
    bool match_step(const Graph &g, Step *s) const {
        const auto &nodes = g.nodes();
        if (nodes.size() < 28 || (nodes.size() - 2) % 26) return false;
        const int L = static_cast<int>((nodes.size() - 2) / 26);
        Tensor *lg = nodes.back();
        if (!named(lg, "logits") || lg->op != OperationType::GGML_OP_MUL_MAT || !lg->data || lg->dims[2] != 1) return false;
        std::map<std::string, const Tensor *> by_name;
        for (Tensor *n : nodes) {
            if (n->backend != this) return false;
            by_name[n->name] = n;
            for (size_t i = 0; i < TENSOR_MAX_SRC && n->src[i]; ++i) {
                const Tensor *w = n->src[i];
                if (static_cast<uint8_t>(w->tensorRole) & static_cast<uint8_t>(TensorRole::TENSOR_ROLE_WEIGHT)) {
                    if (w->backend != this || !w->data || w->dataType != DataType::GGML_TYPE_F32) return false;
                    s->w[w->name] = w;
                }
            }
        }
        auto node = [&](const std::string &n) -> const Tensor * {
            auto it = by_name.find(n);
            return it == by_name.end() ? nullptr : it->second;
        };
        static const char *per_layer[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm",
                                          "attn_k_norm", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
        for (int l = 0; l < L; ++l)
            for (const char *p : per_layer)
                if (!s->w.count("blk." + std::to_string(l) + "." + p + ".weight")) return false;
        if (!s->w.count("output_norm.weight") || !s->w.count("output.weight")) return false;
        // embedding rows from the CPU gather of the token ids (or its copy)
        const Tensor *an0 = node("attn_norm_0");
        if (!an0 || an0->op != OperationType::GGML_OP_RMS_NORM) return false;
        const Tensor *emb = an0->src[0];
        if (emb && emb->op != OperationType::GGML_OP_GET_ROWS) emb = emb->src[0];
        if (!emb || emb->op != OperationType::GGML_OP_GET_ROWS) return false;
        const Tensor *table_w = emb->src[0], *ids = emb->src[1];
        if (!table_w || !ids || !table_w->backend || !table_w->backend->is_host() || !ids->backend ||
            !ids->backend->is_host() || ids->dataType != DataType::GGML_TYPE_I32 || !ids->data || !table_w->data)
            return false;
        s->ids = static_cast<const int32_t *>(ids->data);
        s->embd = static_cast<const float *>(table_w->data);
        s->M = ids->dims[0];
        if (s->M <= 0 || lg->dims[1] != s->M) return false;
        std::memcpy(&s->eps, &an0->op_params[0], sizeof s->eps);
        // positions n_past .. n_past + M - 1 and the angle table, on the host
        const Tensor *rq = node("rope_q_0");
        if (!rq || rq->op != OperationType::GGML_OP_ROPE) return false;
        const Tensor *pos = host_source(rq->src[1]), *tab = host_source(rq->src[2]);
        if (!pos || !tab || !pos->data || !tab->data) return false;
        s->table = static_cast<const float *>(tab->data);
        s->n_ctx_train = tab->dims[1];
        s->kc.resize(L);
        s->vc.resize(L);
        const Tensor *qn = s->w.at("blk.0.attn_q_norm.weight");
        const int64_t D = qn->dims[0];
        const int64_t Hkv = s->w.at("blk.0.attn_k.weight")->dims[1] / D;
        for (int l = 0; l < L; ++l) {
            const Tensor *fa = node("flash_attn_" + std::to_string(l));
            if (!fa || fa->op != OperationType::GGML_OP_FLASH_ATTN_EXT || !fa->src[1] || !fa->src[2]) return false;
            AttnParams ap{};
            std::memcpy(&ap, fa->op_params, sizeof ap);
            if (!ap.causal || ap.sliding_window || std::fabs(ap.scale * std::sqrt(static_cast<float>(D)) - 1.f) > 1e-6f)
                return false;
            if (l == 0) s->n_past = ap.n_ctx;
            if (ap.n_ctx != s->n_past) return false;
            const Tensor *k = fa->src[1], *v = fa->src[2];
            if (k->backend != this || v->backend != this || !k->data || !v->data || k->dims[1] != Hkv ||
                k->dims[0] != D || k->dims[2] != s->n_past + s->M)
                return false;
            s->kc[l] = static_cast<float *>(k->data);
            s->vc[l] = static_cast<float *>(v->data);
        }
        const int32_t *p = static_cast<const int32_t *>(pos->data);
        for (int64_t i = 0; i < s->M; ++i)
            if (p[i] != s->n_past + i) return false;
        s->n_layer = L;
        s->logits = lg;
        return true;
    }

    std::expected<void, std::error_code> run_step(const Step &s) {
        const Tensor *wq = s.w.at("blk.0.attn_q.weight"), *wk = s.w.at("blk.0.attn_k.weight");
        const Tensor *qn = s.w.at("blk.0.attn_q_norm.weight"), *wg = s.w.at("blk.0.ffn_gate.weight");
        const Tensor *out = s.w.at("output.weight");
        const int64_t H = wq->dims[0], D = qn->dims[0], V = out->dims[1];
        // the KV objects' capacity: the V block follows the K block (naiveKVStorage.cpp:28-40)
        const int64_t Hkv = wk->dims[1] / D;
        const int64_t cap = (reinterpret_cast<const char *>(s.vc[0]) - reinterpret_cast<const char *>(s.kc[0])) /
                            (Hkv * D * 4);
        b200_qwen3_config c{};
        c.n_vocab = static_cast<int32_t>(V);
        c.n_embd = static_cast<int32_t>(H);
        c.n_layer = s.n_layer;
        c.n_head = static_cast<int32_t>(wq->dims[1] / D);
        c.n_head_kv = static_cast<int32_t>(Hkv);
        c.head_dim = static_cast<int32_t>(D);
        c.n_ff = static_cast<int32_t>(wg->dims[1]);
        c.n_ctx_train = static_cast<int32_t>(s.n_ctx_train);
        c.rope_theta = 0.f;  // the frequencies come from the angle table
        c.rms_eps = s.eps;
        c.tied = 0;          // the reference keeps a device copy named output.weight
        c.kv_capacity = static_cast<int32_t>(cap);
        c.precision = prefill_precision();
        c.tp_world = 1;
        c.external_kv = 1;
        c.max_batch = static_cast<int32_t>(std::max<int64_t>(s.M, 512));
        if (cap < s.n_past + s.M) return fail(std::errc::invalid_argument);
        if (engine_ && (std::memcmp(&c, &cfg_, offsetof(b200_qwen3_config, kv_capacity)) != 0 ||
                        c.kv_capacity != cfg_.kv_capacity || s.M > cfg_.max_batch)) {
            if (s.M > cfg_.max_batch && std::memcmp(&c, &cfg_, offsetof(b200_qwen3_config, kv_capacity)) == 0 &&
                c.kv_capacity == cfg_.kv_capacity)
                return fail(std::errc::not_supported);  // a longer batch than the engine's arena: op by op
            b200_engine_destroy(engine_);
            engine_ = nullptr;
        }
        if (!engine_) {
            if (auto r = create_engine(c, s); !r) return r;
        }
        for (int l = 0; l < s.n_layer; ++l)
            if (b200_engine_bind_kv(engine_, l, s.kc[l], s.vc[l]) != B200_OK) return fail(std::errc::io_error);
        if (b200_engine_n_past(engine_) != s.n_past && b200_engine_set_n_past(engine_, s.n_past) != B200_OK)
            return fail(std::errc::io_error);
        int32_t tok = 0;
        float *last = static_cast<float *>(s.logits->data) + (s.M - 1) * V;
        const int rc = b200_engine_eval_device(engine_, s.ids, s.M, last, &tok);
        if (rc != B200_OK) {
            std::cerr << "[b200] engine step failed: " << b200_status_string(rc) << "\n";
            return fail(rc == B200_ERR_OUT_OF_RANGE ? std::errc::result_out_of_range : std::errc::io_error);
        }
        ++engine_steps;
        return {};
    }

    std::expected<void, std::error_code> create_engine(const b200_qwen3_config &c, const Step &s) {
        b200_engine *e = nullptr;
        if (b200_engine_create(&c, _device_id, &e) != B200_OK) return fail(std::errc::not_enough_memory);
        auto bad = [&]() {
            b200_engine_destroy(e);
            return fail(std::errc::io_error);
        };
        // weights: device tensors of this backend (device-to-device) and the host
        // embedding table (gathered on the device from now on)
        for (const auto &kv : s.w)
            if (b200_engine_set_weight(e, kv.first.c_str(), static_cast<const float *>(kv.second->data),
                                       static_cast<int64_t>(kv.second->element_count())) != B200_OK)
                return bad();
        if (b200_engine_set_weight(e, "token_embd.weight", s.embd, static_cast<int64_t>(c.n_vocab) * c.n_embd) !=
            B200_OK)
            return bad();
        // rotation frequencies: row 1 of the angle table is exactly freq (graph.cpp:119-131)
        if (s.n_ctx_train < 2 || b200_engine_set_rope_freqs(e, s.table + c.head_dim / 2) != B200_OK) return bad();
        for (int l = 0; l < s.n_layer; ++l)
            if (b200_engine_bind_kv(e, l, s.kc[l], s.vc[l]) != B200_OK) return bad();
        if (b200_engine_finalize(e) != B200_OK) return bad();
        engine_ = e;
        cfg_ = c;
        return {};
    }

    cudaStream_t stream_ = nullptr;
    std::vector<void *> weights_;
    std::unique_ptr<DeviceArena> kv_ = std::make_unique<DeviceArena>();
    std::unique_ptr<DeviceArena> act_ = std::make_unique<DeviceArena>();
    std::vector<Pending> pending_;
    b200_engine *engine_ = nullptr;
    b200_qwen3_config cfg_{};
};

std::vector<DeviceInfo> probe_b200_devices() {
    std::vector<DeviceInfo> out;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return out;
    }
    int prev = 0;
    const bool restore = cudaGetDevice(&prev) == cudaSuccess;
    for (int i = 0; i < n; ++i) {
        size_t free_b = 0, total_b = 0;
        if (cudaSetDevice(i) != cudaSuccess || cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        out.push_back({"cuda:" + std::to_string(i), DeviceType::CUDA, free_b});
    }
    if (restore) cudaSetDevice(prev);
    return out;
}

}  // namespace

void register_cuda_backend() {
    BackendRegistry::instance().register_backend(
        "cuda", []() { return probe_b200_devices(); },
        [](int device_id, DeviceInfo info, const PoolConfig &cfg) -> std::unique_ptr<Backend> {
            return std::make_unique<B200Backend>(device_id, std::move(info), cfg);
        });
}

// Counters of the B200 backend on `b` (steps the engine ran, subgraphs run op by
// op); -1 if `b` is not one. For tests and benchmarks.
extern "C" int b200_backend_counters(const void *b, long *engine_steps, long *op_graphs) {
    auto *bb = dynamic_cast<const B200Backend *>(static_cast<const Backend *>(b));
    if (!bb) return -1;
    if (engine_steps) *engine_steps = bb->engine_steps;
    if (op_graphs) *op_graphs = bb->op_graphs;
    return 0;
}
