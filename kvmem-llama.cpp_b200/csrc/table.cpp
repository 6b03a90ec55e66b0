#include "table.hpp"

#include <algorithm>

namespace kvmret {

// KvMemStore::register_append, kvmem/src/host/kvmem_store.cpp:179-205.
void BlockTable::append(uint32_t n_tok) {
    const uint32_t bt = cfg_.block_tokens;
    uint32_t left = n_tok;
    if (!blocks_.empty() && blocks_.back().n_tok < bt) {
        const uint32_t take = std::min(bt - blocks_.back().n_tok, left);
        blocks_.back().n_tok += take;
        total_ += take;
        left -= take;
    }
    while (left > 0) {
        Block b;
        b.pos0 = total_;
        b.n_tok = std::min(bt, left);
        b.baked = b.pos0;
        blocks_.push_back(b);
        total_ += b.n_tok;
        left -= b.n_tok;
    }
}

// pick_topk_ungrouped up to the score fill, kvmem/src/host/kvmem_store.cpp:482-534:
// sink prefix, mandatory newest-first while budget lasts, recent suffix.
uint32_t BlockTable::keep(uint32_t n, const uint32_t *mandatory, uint32_t n_mandatory,
                          std::vector<uint8_t> &kept, uint32_t &kept_count) const {
    kept.assign(n, 0);
    kept_count = 0;
    if (n == 0) return 0;
    const uint32_t budget = cfg_.budget_blocks;
    if (budget == 0 || n <= budget) {
        std::fill(kept.begin(), kept.end(), 1);
        kept_count = n;
        return 0;
    }
    auto take = [&](uint32_t id) {
        if (id < n && !kept[id]) {
            kept[id] = 1;
            ++kept_count;
        }
    };
    const uint32_t sink = std::min(cfg_.sink_blocks, n);
    const uint32_t recent = std::min(cfg_.recent_blocks, n);
    for (uint32_t i = 0; i < sink && kept_count < budget; ++i) take(i);
    for (uint32_t i = n_mandatory; i > 0 && kept_count < budget; --i) take(mandatory[i - 1]);
    for (uint32_t i = 0; i < recent && kept_count < budget; ++i) take(n - 1 - i);
    return budget - kept_count;
}

// KvMemStore::set_selection, kvmem/src/host/kvmem_store.cpp:758-882, then the
// tier effect of spill_outgoing / admit_incoming (kvmem_runtime.cpp:225-249):
// stage-out blocks leave the GPU tier, stage-in blocks enter it.
Plan BlockTable::set_selection(const uint32_t *ids, uint32_t n_ids, bool force_raw) {
    const uint32_t n = n_blocks();
    std::vector<uint32_t> sel(ids, ids + n_ids);
    std::sort(sel.begin(), sel.end());
    sel.erase(std::unique(sel.begin(), sel.end()), sel.end());
    sel.erase(std::remove_if(sel.begin(), sel.end(), [&](uint32_t id) { return id >= n; }),
              sel.end());

    Plan p;
    std::vector<uint8_t> now(n, 0), was(n, 0);
    for (uint32_t id : sel) now[id] = 1;
    for (uint32_t i = 0; i < n; ++i) {
        was[i] = blocks_[i].in_ws;
        if (was[i] && now[i]) ++p.overlap;
    }
    for (uint32_t i = 0; i < n; ++i) {
        if (blocks_[i].on_gpu && !now[i]) {
            p.stage_out.push_back(i);
            blocks_[i].in_ws = false;
        }
    }
    uint32_t wpos = 0;
    p.remaps.reserve(sel.size());
    for (uint32_t id : sel) {
        Block &b = blocks_[id];
        if (was[id] && b.on_gpu) ++p.reused;
        const bool cold = !b.on_gpu;
        if (!b.in_ws) p.stage_in.push_back(id);
        const int64_t w = static_cast<int64_t>(wpos);
        const bool same = b.baked == w;
        Remap r;
        r.id = id;
        r.n_tok = b.n_tok;
        r.from = static_cast<int32_t>(b.baked);
        r.to = static_cast<int32_t>(wpos);
        r.resident = !cold;
        r.skip = same && (!cfg_.immutable_source_k || r.resident) && !force_raw;
        r.raw = false;
        const uint64_t delta = static_cast<uint64_t>(b.baked > w ? b.baked - w : w - b.baked);
        if (cfg_.immutable_source_k && (cold || !same)) {
            const bool by_count =
                cfg_.refresh_remaps > 0 && b.remap_count >= cfg_.refresh_remaps;
            const uint64_t lim = cfg_.refresh_abs_delta;
            const bool by_delta =
                lim > 0 && (b.remap_delta >= lim || delta >= lim - std::min(b.remap_delta, lim));
            const bool out_of_range =
                cfg_.max_baked > 0 &&
                (b.baked < 0 || static_cast<uint64_t>(b.baked) + b.n_tok > cfg_.max_baked);
            r.raw = cold || by_count || by_delta || out_of_range;
        }
        if (cfg_.immutable_source_k && force_raw) r.raw = true;
        p.remaps.push_back(r);
        b.in_ws = true;
        if (!r.skip) {
            if (r.raw) {
                b.remap_count = 0;
                b.remap_delta = 0;
            } else {
                ++b.remap_count;
                b.remap_delta += delta;
            }
        }
        b.baked = w;
        wpos += b.n_tok;
    }
    p.window_tokens = wpos;
    for (uint32_t id : p.stage_out) blocks_[id].on_gpu = false;
    for (uint32_t id : p.stage_in) blocks_[id].on_gpu = true;
    return p;
}

void BlockTable::truncate(uint32_t n_tokens) {
    if (n_tokens >= total_) return;
    while (!blocks_.empty() && blocks_.back().pos0 >= n_tokens) {
        total_ -= blocks_.back().n_tok;
        blocks_.pop_back();
    }
    if (!blocks_.empty()) {
        Block &last = blocks_.back();
        if (last.pos0 + last.n_tok > n_tokens) {
            const uint32_t keep_tok = n_tokens - last.pos0;
            total_ -= last.n_tok - keep_tok;
            last.n_tok = keep_tok;
        }
    }
}

void BlockTable::clear_working_set(bool drop_gpu) {
    for (Block &b : blocks_) {
        b.in_ws = false;
        if (drop_gpu) b.on_gpu = false;
    }
}

}  // namespace kvmret
