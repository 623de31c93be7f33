// Paged KV strategy for the reference's KV cache manager: the block_tokens > 0 case
// of KVCacheConfig (include/kvcache/kvutil.hpp:43-44) that the reference declares
// but leaves unimplemented (its one strategy is ContiguousKVStrategy).
//
// Every (sequence, layer) holds a list of blocks; a block is one KV storage object
// of capacity block_tokens (KVStorage::alloc, so NaiveKVStorage places each block
// through Backend::alloc(KVCACHE)), and logical position p of the sequence lives in
// block p / block_tokens at token p % block_tokens. reserve_append allocates the
// blocks a pending range needs (all layers, or none), abort_append frees them again,
// release_sequence frees all of a sequence's blocks. lookup (the strategy's one
// extension point, kvstrategy.hpp) turns a token range into one KVSlice per block
// it touches, so acquire_layer hands out one segment view per block. block_table
// gives the blocks' K / V base addresses in position order: the k_blocks / v_blocks
// tables of b200_paged_kv_write / b200_flash_attn_paged (include/b200_infer.h).
#pragma once

#include <expected>
#include <memory>
#include <span>
#include <system_error>
#include <unordered_map>
#include <vector>

#include "kvcache/kvstrategy.hpp"

class PagedKVStrategy : public KVStrategy {
public:
    explicit PagedKVStrategy(std::unique_ptr<KVStorage> storage) noexcept : KVStrategy(std::move(storage)) {}
    ~PagedKVStrategy() override;

    std::expected<void, std::error_code> init(std::span<const KVLayerSpec> layers, std::span<Backend *const> backend_layer,
                                              const KVCacheConfig &config) override;
    std::expected<void, std::error_code> create_sequence(SequenceId id) override;
    std::expected<void, std::error_code> reserve_append(SequenceId id, TokenRange range) override;
    std::expected<void, std::error_code> commit_append(SequenceId id, TokenRange range) override;
    std::expected<void, std::error_code> abort_append(SequenceId id, TokenRange range) override;
    std::expected<void, std::error_code> release_sequence(SequenceId id) override;
    std::expected<void, std::error_code> clear_sequence() override;

    // K / V base addresses of the blocks holding positions [0, tokens) of one layer,
    // in position order (the block tables of the paged kernels).
    std::expected<void, std::error_code> block_table(SequenceId id, std::size_t layer, std::size_t tokens,
                                                     std::vector<void *> &k, std::vector<void *> &v);
    // Blocks a sequence holds in one layer (committed and pending).
    std::size_t blocks(SequenceId id, std::size_t layer) const;

protected:
    std::expected<KVMapping, std::error_code> lookup(SequenceId id, std::size_t layer, TokenRange range) const override;

private:
    struct Sequence {
        std::vector<std::vector<StorageId>> blocks;  // [layer][block]
        std::size_t committed_blocks = 0;            // blocks per layer before the pending append
        bool pending = false;
    };
    void free_blocks(Sequence &s, std::size_t keep) noexcept;
    std::unordered_map<SequenceId, Sequence> _sequences;
};
