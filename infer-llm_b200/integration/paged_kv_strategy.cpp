// Paged KV strategy (see paged_kv_strategy.hpp): positions map to fixed-size block
// objects; contiguous ranges of a block become one slice each.
#include "paged_kv_strategy.hpp"

#include "kvcache/kvstorage.hpp"

namespace {
std::unexpected<std::error_code> fail(std::errc e) { return std::unexpected(std::make_error_code(e)); }
}  // namespace

PagedKVStrategy::~PagedKVStrategy() { (void)clear_sequence(); }

std::expected<void, std::error_code> PagedKVStrategy::init(std::span<const KVLayerSpec> layers,
                                                           std::span<Backend *const> backend_layer,
                                                           const KVCacheConfig &config) {
    if (!_storage || layers.size() != backend_layer.size() || config.layers != layers.size() || config.block_tokens == 0)
        return fail(std::errc::invalid_argument);
    if (auto r = _storage->init(layers, backend_layer); !r) return std::unexpected(r.error());
    _layers.assign(layers.begin(), layers.end());
    _cfg = config;
    return {};
}

std::expected<void, std::error_code> PagedKVStrategy::create_sequence(SequenceId id) {
    if (id == kInvalidSequenceId) return fail(std::errc::invalid_argument);
    auto [it, inserted] = _sequences.try_emplace(id);
    if (!inserted) return fail(std::errc::file_exists);
    it->second.blocks.assign(_cfg.layers, {});
    return {};
}

void PagedKVStrategy::free_blocks(Sequence &s, std::size_t keep) noexcept {
    for (auto &layer_blocks : s.blocks) {
        while (layer_blocks.size() > keep) {
            _storage->free(layer_blocks.back());
            layer_blocks.pop_back();
        }
    }
}

std::expected<void, std::error_code> PagedKVStrategy::reserve_append(SequenceId id, TokenRange range) {
    auto it = _sequences.find(id);
    if (it == _sequences.end()) return fail(std::errc::invalid_argument);
    Sequence &s = it->second;
    if (s.pending) return fail(std::errc::device_or_resource_busy);
    const std::size_t limit = _cfg.max_tokens_per_sequence;
    if (limit && (range.begin > limit || range.count > limit - range.begin)) return fail(std::errc::not_enough_memory);
    const std::size_t bt = _cfg.block_tokens;
    const std::size_t need = (range.end() + bt - 1) / bt;
    const std::size_t have = s.blocks.empty() ? 0 : s.blocks.front().size();
    for (std::size_t layer = 0; layer < s.blocks.size(); ++layer) {
        while (s.blocks[layer].size() < need) {
            auto b = _storage->alloc(layer, bt);
            if (!b) {  // all layers or none
                free_blocks(s, have);
                return std::unexpected(b.error());
            }
            s.blocks[layer].push_back(*b);
        }
    }
    s.committed_blocks = have;
    s.pending = true;
    return {};
}

std::expected<void, std::error_code> PagedKVStrategy::commit_append(SequenceId id, TokenRange) {
    auto it = _sequences.find(id);
    if (it == _sequences.end()) return fail(std::errc::invalid_argument);
    it->second.pending = false;
    return {};
}

std::expected<void, std::error_code> PagedKVStrategy::abort_append(SequenceId id, TokenRange) {
    auto it = _sequences.find(id);
    if (it == _sequences.end()) return fail(std::errc::invalid_argument);
    Sequence &s = it->second;
    if (s.pending) free_blocks(s, s.committed_blocks);  // the blocks this append added
    s.pending = false;
    return {};
}

std::expected<void, std::error_code> PagedKVStrategy::release_sequence(SequenceId id) {
    auto it = _sequences.find(id);
    if (it == _sequences.end()) return fail(std::errc::invalid_argument);
    free_blocks(it->second, 0);
    _sequences.erase(it);
    return {};
}

std::expected<void, std::error_code> PagedKVStrategy::clear_sequence() {
    for (auto &kv : _sequences) free_blocks(kv.second, 0);
    _sequences.clear();
    return {};
}

std::expected<KVMapping, std::error_code> PagedKVStrategy::lookup(SequenceId id, std::size_t layer,
                                                                  TokenRange range) const {
    auto it = _sequences.find(id);
    if (it == _sequences.end() || layer >= it->second.blocks.size()) return fail(std::errc::invalid_argument);
    const auto &blocks = it->second.blocks[layer];
    const std::size_t bt = _cfg.block_tokens;
    if (range.end() > blocks.size() * bt) return fail(std::errc::not_enough_memory);  // not reserved
    KVMapping m;
    for (std::size_t p = range.begin; p < range.end();) {
        const std::size_t b = p / bt, off = p % bt, n = std::min(bt - off, range.end() - p);
        const KVSlice slice{.storage_id = blocks[b], .token_offset = off, .token_count = n};
        m.k.push_back(slice);
        m.v.push_back(slice);
        p += n;
    }
    return m;
}

std::expected<void, std::error_code> PagedKVStrategy::block_table(SequenceId id, std::size_t layer, std::size_t tokens,
                                                                  std::vector<void *> &k, std::vector<void *> &v) {
    auto it = _sequences.find(id);
    if (it == _sequences.end() || layer >= it->second.blocks.size()) return fail(std::errc::invalid_argument);
    const auto &blocks = it->second.blocks[layer];
    const std::size_t n = (tokens + _cfg.block_tokens - 1) / _cfg.block_tokens;
    if (n > blocks.size()) return fail(std::errc::not_enough_memory);
    k.clear();
    v.clear();
    for (std::size_t i = 0; i < n; ++i) {
        auto obj = _storage->acquire(blocks[i], layer);  // the object's current addresses
        if (!obj) return std::unexpected(obj.error());
        k.push_back(obj->k_base);
        v.push_back(obj->v_base);
        _storage->release_access(blocks[i]);
    }
    return {};
}

std::size_t PagedKVStrategy::blocks(SequenceId id, std::size_t layer) const {
    auto it = _sequences.find(id);
    if (it == _sequences.end() || layer >= it->second.blocks.size()) return 0;
    return it->second.blocks[layer].size();
}
