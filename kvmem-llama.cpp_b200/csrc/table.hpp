// Host block table: block registry, the always-kept part of a selection and
// the working-set diff (plan). Pure host C++; the GPU context drives it.
//
// Semantics follow KvMemStore (kvmem/include/kvmem/kvmem_store.hpp:329-491,
// kvmem/src/host/kvmem_store.cpp) for the TopK policy without media ranges,
// plus the tier effect of KvMemRuntime::spill_outgoing / admit_incoming
// (kvmem/src/host/kvmem_runtime.cpp:225-249) with no CPU/NVMe tier.
#pragma once

#include <cstdint>
#include <vector>

namespace kvmret {

struct TableConfig {
    uint32_t block_tokens = 128;
    uint32_t budget_blocks = 0;
    uint32_t sink_blocks = 1;
    uint32_t recent_blocks = 0;
    bool immutable_source_k = false;
    uint32_t refresh_remaps = 8;             // immutable_refresh_remaps
    uint64_t refresh_abs_delta = 262144;     // immutable_refresh_abs_delta_tokens
    uint64_t max_baked = 262144;             // immutable_max_baked_position
};

struct Block {
    uint32_t pos0 = 0;        // orig_pos_start
    uint32_t n_tok = 0;
    bool on_gpu = true;       // KvTier::GPU is the registration default
    bool in_ws = false;       // in_working_set
    int64_t baked = -1;       // baked_pos
    uint32_t remap_count = 0;
    uint64_t remap_delta = 0;
};

struct Remap {
    uint32_t id, n_tok;
    int32_t from, to;
    bool resident, skip, raw;
};

struct Plan {
    std::vector<uint32_t> stage_in, stage_out;
    std::vector<Remap> remaps;
    uint32_t window_tokens = 0;
    uint32_t overlap = 0;
    uint32_t reused = 0;
};

class BlockTable {
public:
    explicit BlockTable(const TableConfig &c) : cfg_(c) {}
    const TableConfig &config() const { return cfg_; }
    uint32_t n_blocks() const { return static_cast<uint32_t>(blocks_.size()); }
    uint32_t n_tokens() const { return total_; }
    const std::vector<Block> &blocks() const { return blocks_; }

    // register_append: extend the partial tail block, then open new blocks.
    void append(uint32_t n_tok);

    // Always-kept ids of a top-k selection over the first n blocks. kept[] is
    // resized to n. Returns the count still to be filled by score (0 if
    // everything fits, in which case kept[] marks every block).
    uint32_t keep(uint32_t n, const uint32_t *mandatory, uint32_t n_mandatory,
                  std::vector<uint8_t> &kept, uint32_t &kept_count) const;
    uint32_t keep(const uint32_t *mandatory, uint32_t n_mandatory, std::vector<uint8_t> &kept,
                  uint32_t &kept_count) const {
        return keep(n_blocks(), mandatory, n_mandatory, kept, kept_count);
    }

    // KvMemStore::truncate_to (kvmem/src/host/kvmem_store.cpp:207-227): drop
    // the blocks that start at or after n_tokens, shrink the trailing one.
    void truncate(uint32_t n_tokens);

    // set_block_tier(id, KvTier::GPU) (kvmem/src/host/kvmem_store.cpp:250-277):
    // a block placed on the GPU outside a selection (a decode block bound to a
    // reserve slot, src/adapter/llama-memory-kvmem.cpp:2349-2362).
    void set_on_gpu(uint32_t id) {
        if (id < blocks_.size()) blocks_[id].on_gpu = true;
    }

    // set_selection (+ the runtime's tier effect). ids need not be sorted.
    Plan set_selection(const uint32_t *ids, uint32_t n_ids, bool force_raw_refresh);

    // KvMemStore::clear_working_set (kvmem/include/kvmem/kvmem_store.hpp:470-472,
    // kvmem/src/host/kvmem_store.cpp:897-901): no block is in the working set
    // any more; the registry and the baked positions stay. drop_gpu also takes
    // every block out of the GPU tier (the context's pool reset, which the
    // reference's store has no counterpart for).
    void clear_working_set(bool drop_gpu);

private:
    TableConfig cfg_;
    std::vector<Block> blocks_;
    uint32_t total_ = 0;
};

}  // namespace kvmret
