// C-ABI shim over the reference's own libkvmem, compiled from the reference
// sources (kvmem/src/host/*.cpp) into oracle/_ref/. TEST INFRASTRUCTURE ONLY:
// it lets the tests pin the oracle restatement against the reference code
// itself (selection, plan, mean-K, RoPE). Nothing here is shipped.

#include "kvmem/kvmem_runtime.hpp"
#include "kvmem/kvmem_store.hpp"
#include "kvmem/raw_kv_store.hpp"
#include "kvmem/rope.hpp"

#include <cstring>
#include <vector>

#define REF_API extern "C" __attribute__((visibility("default")))

// kvmem_store.cpp pick_topk_blocks via a fresh store of n full blocks.
REF_API uint32_t ref_pick_topk(const double *scores, uint32_t n, uint32_t block_tokens,
                               uint32_t budget_blocks, uint32_t sink_blocks,
                               uint32_t recent_blocks, const uint32_t *mandatory,
                               uint32_t n_mandatory, uint32_t *out) {
    kvmem::KvMemStoreConfig cfg;
    cfg.block_tokens = block_tokens;
    cfg.select_budget = budget_blocks * block_tokens;
    cfg.sink_blocks = sink_blocks;
    cfg.recent_blocks = recent_blocks;
    kvmem::KvMemStore s(cfg);
    s.register_append(n * block_tokens);
    s.set_retrieval_scores(std::vector<double>(scores, scores + n));
    std::vector<uint32_t> mand(mandatory, mandatory + n_mandatory);
    const auto sel = s.pick_topk_blocks(mand);
    for (size_t i = 0; i < sel.size(); ++i) out[i] = sel[i];
    return static_cast<uint32_t>(sel.size());
}

struct RefRuntime {
    kvmem::KvMemRuntime rt;
    explicit RefRuntime(kvmem::KvMemRuntimeConfig c) : rt(std::move(c)) {}
};

REF_API void *ref_runtime_create(uint32_t block_tokens, uint32_t budget_blocks,
                                 uint32_t sink_blocks, int immutable_source_k) {
    kvmem::KvMemRuntimeConfig c;
    c.store.block_tokens = block_tokens;
    c.store.select_budget = budget_blocks * block_tokens;
    c.store.sink_blocks = sink_blocks;
    c.store.immutable_source_k = immutable_source_k != 0;
    return new RefRuntime(c);
}
REF_API void ref_runtime_free(void *p) { delete static_cast<RefRuntime *>(p); }
REF_API void ref_runtime_append(void *p, uint32_t n_tokens) {
    static_cast<RefRuntime *>(p)->rt.register_append(n_tokens);
}

// The store's clear_working_set, reached through the runtime's store().
REF_API void ref_runtime_clear_working_set(void *p) {
    static_cast<RefRuntime *>(p)->rt.store().clear_working_set();
}

// prepare_selection (set_selection) + finish_reselect (spill then admit).
REF_API void ref_runtime_select(void *p, const uint32_t *ids, uint32_t n_ids,
                                int force_raw_refresh, uint32_t *stage_in,
                                uint32_t *stage_out, int32_t *remaps, uint32_t *counts) {
    auto &rt = static_cast<RefRuntime *>(p)->rt;
    const auto plan = rt.prepare_selection(std::vector<uint32_t>(ids, ids + n_ids),
                                           force_raw_refresh != 0);
    rt.finish_reselect();
    for (size_t i = 0; i < plan.stage_in.size(); ++i) stage_in[i] = plan.stage_in[i];
    for (size_t i = 0; i < plan.stage_out.size(); ++i) stage_out[i] = plan.stage_out[i];
    for (size_t i = 0; i < plan.remaps.size(); ++i) {
        const auto &r = plan.remaps[i];
        int32_t *o = remaps + 7 * i;
        o[0] = static_cast<int32_t>(r.block_id);
        o[1] = static_cast<int32_t>(r.n_tokens);
        o[2] = r.from_base;
        o[3] = r.to_base;
        o[4] = r.working_k_resident ? 1 : 0;
        o[5] = r.skip ? 1 : 0;
        o[6] = r.raw_refresh ? 1 : 0;
    }
    counts[0] = static_cast<uint32_t>(plan.stage_in.size());
    counts[1] = static_cast<uint32_t>(plan.stage_out.size());
    counts[2] = static_cast<uint32_t>(plan.remaps.size());
    counts[3] = plan.total_window_tokens;
    counts[4] = plan.selection_overlap_blocks;
    counts[5] = plan.gpu_reused_blocks;
}

// RawKvStore::write_layer_mean_k + mean_k for one (block, layer).
REF_API void ref_mean_k_f32(const float *k_rows, uint32_t n_tok, uint32_t n_embd_k,
                            uint32_t block_tokens, float *out) {
    kvmem::RawKvStoreConfig c;
    c.n_layer = 1;
    c.n_embd_k = n_embd_k;
    c.n_embd_v = n_embd_k;
    c.block_tokens = block_tokens;
    kvmem::RawKvStore s(c);
    s.write_layer_mean_k(0, n_tok, 0, k_rows);
    s.mean_k(0, 0, out);
}

REF_API void ref_rope_neox(const float *k, uint32_t n_tok, uint32_t n_head,
                           uint32_t n_embd_head, uint32_t n_rot, int32_t pos0,
                           float freq_base, float freq_scale, float *out) {
    kvmem::RopeConfig c;
    c.n_rot = n_rot;
    c.n_embd_head = n_embd_head;
    c.n_head_kv = n_head;
    c.freq_base = freq_base;
    c.freq_scale = freq_scale;
    kvmem::rope_neox_apply(c, k, n_tok, pos0, out);
}

// The stage-in work of one retrieval step on the host cores, for the CPU
// reference arm of the benchmark: every unit is one (block, layer) of the
// window. Its K (n_tok rows of n_head x n_embd_head f16) is converted to f32,
// rotated by the reference's rope_neox_apply at the unit's window base, and
// rounded back to f16 (F16C conversions, round to nearest even); its V bytes
// are copied. Units [u0, u1) of the arrays; a caller splits the units over
// its threads.
REF_API void ref_rope_units_f16(const uint16_t *const *k_src, uint16_t *const *k_dst,
                                const uint8_t *const *v_src, uint8_t *const *v_dst,
                                uint64_t v_bytes, const int32_t *pos0, uint32_t u0, uint32_t u1,
                                uint32_t n_tok, uint32_t n_head, uint32_t n_embd_head,
                                float freq_base, float freq_scale) {
    kvmem::RopeConfig c;
    c.n_rot = n_embd_head;
    c.n_embd_head = n_embd_head;
    c.n_head_kv = n_head;
    c.freq_base = freq_base;
    c.freq_scale = freq_scale;
    const size_t n = static_cast<size_t>(n_tok) * n_head * n_embd_head;
    std::vector<float> x(n), y(n);
    for (uint32_t u = u0; u < u1; ++u) {
        const _Float16 *src = reinterpret_cast<const _Float16 *>(k_src[u]);
        _Float16 *dst = reinterpret_cast<_Float16 *>(k_dst[u]);
        for (size_t i = 0; i < n; ++i) x[i] = static_cast<float>(src[i]);
        kvmem::rope_neox_apply(c, x.data(), n_tok, pos0[u], y.data());
        for (size_t i = 0; i < n; ++i) dst[i] = static_cast<_Float16>(y[i]);
        if (v_bytes) std::memcpy(v_dst[u], v_src[u], v_bytes);
    }
}

// Byte copies [i0, i1) of a list (the staging memcpy of stage-in blocks).
REF_API void ref_copy_list(const uint8_t *const *src, uint8_t *const *dst, const uint64_t *nbytes,
                           uint32_t i0, uint32_t i1) {
    for (uint32_t i = i0; i < i1; ++i) std::memcpy(dst[i], src[i], nbytes[i]);
}

// KvMemRuntime::truncate_to and the store's set_block_tier(id, GPU), for the
// host-table tests of truncation and decode-block placement.
REF_API void ref_runtime_truncate(void *p, uint32_t token_pos) {
    static_cast<RefRuntime *>(p)->rt.truncate_to(token_pos);
}
REF_API void ref_runtime_set_tier_gpu(void *p, uint32_t block_id) {
    static_cast<RefRuntime *>(p)->rt.store().set_block_tier(block_id, kvmem::KvTier::GPU, -1, -1);
}

// The reference's own snapshot archive of n_tok tokens per layer, stored the
// way this library stores them: unrotated K rows (k_row_bytes 0 = f16) with
// their f32 values for the running sum, and V as packed rows. The bytes of
// RawKvStore::snapshot_write through a SnapshotWriter into `out`; returns the
// archive size (also when it exceeds cap, without writing past it).
#include "kvmem/snapshot.hpp"

REF_API uint64_t ref_snapshot_rows(uint32_t n_layer, uint32_t n_embd, uint32_t block_tokens,
                                   uint64_t k_row_bytes, uint64_t v_row_bytes, uint32_t n_tok,
                                   const uint8_t *k_rows, const float *k_f32,
                                   const uint8_t *v_rows, uint8_t *out, uint64_t cap,
                                   uint64_t *hash) {
    kvmem::RawKvStoreConfig c;
    c.n_layer = n_layer;
    c.n_embd_k = n_embd;
    c.n_embd_v = n_embd;
    c.block_tokens = block_tokens;
    c.k_row_bytes = k_row_bytes;
    c.v_gpu_row_bytes = v_row_bytes;
    kvmem::RawKvStore s(c);
    const uint64_t krow = k_row_bytes ? k_row_bytes : 2ull * n_embd;
    for (uint32_t l = 0; l < n_layer; ++l) {
        s.write_layer_k_rows(0, n_tok, l, k_rows + static_cast<size_t>(l) * n_tok * krow,
                             k_f32 ? k_f32 + static_cast<size_t>(l) * n_tok * n_embd : nullptr);
        s.write_layer_v_gpu(0, n_tok, l, v_rows + static_cast<size_t>(l) * n_tok * v_row_bytes);
    }
    uint64_t pos = 0;
    kvmem::SnapshotWriter w([&](const void *p, size_t n) {
        if (pos + n <= cap) std::memcpy(out + pos, p, n);
        pos += n;
    });
    s.snapshot_write(w);
    if (hash) *hash = w.hash();
    return w.bytes();
}
