// kvmret oracle — TEST INFRASTRUCTURE ONLY.
//
// A plain CPU restatement of KVMem's per-step KV retrieval path, used by the
// tests, the smoke check and the bench's CPU-baseline arm as the checker. The
// product library never links, loads or calls anything in this directory.
//
// Every function restates one reference function; the citation is given as
// path:line inside the zyf32453/kvmem-llama.cpp tree. Floating-point
// operations follow the reference's types and loop order exactly. This file
// must be compiled with -ffp-contract=off and without -march=native so that
// no multiply-add is fused (x86-64 baseline g++, as the reference is built).
//
// Parity pins: the selection / plan / mean-K / RoPE functions are checked in
// the tests against the reference's own libkvmem (built from its sources into
// oracle/_ref) and against the known answers of the reference's unit tests.
// The scorer, the query accumulation and the dequant / FWHT / requant kernels
// live in reference files that cannot be compiled here (they need the absent
// llama.cpp / ggml headers); they are restated line by line, and for those
// three functions parity is unpinned (no reference golden vector exists).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <vector>

#define ORC_API extern "C" __attribute__((visibility("default")))

namespace {

// kvmem/src/host/raw_kv_store.cpp:33-67 (f32 -> f16, round to nearest even).
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, sizeof(x));
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t exp = static_cast<int32_t>((x >> 23) & 0xffu) - 127 + 15;
    uint32_t man = x & 0x7fffffu;
    if ((x & 0x7fffffffu) == 0) return static_cast<uint16_t>(sign);
    if (((x >> 23) & 0xffu) == 0xffu) return static_cast<uint16_t>(sign | 0x7c00u | (man ? 0x200u : 0));
    if (exp <= 0) {
        if (exp < -10) return static_cast<uint16_t>(sign);
        man |= 0x800000u;
        const uint32_t t = static_cast<uint32_t>(14 - exp);
        uint32_t half = man >> t;
        const uint32_t rem = man & ((1u << t) - 1u);
        if (rem > (1u << (t - 1)) || (rem == (1u << (t - 1)) && (half & 1u))) half += 1;
        return static_cast<uint16_t>(sign | half);
    }
    if (exp >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    uint32_t half = (static_cast<uint32_t>(exp) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half += 1;
    return static_cast<uint16_t>(sign | half);
}

// kvmem/src/host/raw_kv_store.cpp:69-96 (f16 -> f32, exact).
float f16_to_f32(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t out;
    if (exp == 0) {
        if (man == 0) {
            out = sign;
        } else {
            exp = 1;
            while ((man & 0x400u) == 0) { man <<= 1; exp--; }
            man &= 0x3ffu;
            out = sign | ((exp + 127 - 15) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        out = sign | 0x7f800000u | (man << 13);
    } else {
        out = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &out, sizeof(f));
    return f;
}

}  // namespace

ORC_API uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
ORC_API float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

ORC_API void orc_f32_to_f16_n(const float *src, uint16_t *dst, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = f32_to_f16(src[i]);
}
ORC_API void orc_f16_to_f32_n(const uint16_t *src, float *dst, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = f16_to_f32(src[i]);
}

// ---------------------------------------------------------------------------
// S2 — block summary (mean pre-RoPE K).
// kvmem/src/host/raw_kv_store.cpp:215-234 (add_mean_f32: token-order F32 sum,
// zeroed at off == 0) and :987-1007 (mean_k: sum * (1.0f / mean_tokens), the
// accumulator is never normalised in place). The K rows reach the sum as f32
// converted from the f16 capture (src/adapter/llama-memory-kvmem.cpp:3405-3414).
//
// k_rows: token-major [n_tok][n_embd] f16.  mean_out: [n_embd] f32.
ORC_API void orc_mean_k_f16(const uint16_t *k_rows, uint32_t n_tok, uint32_t n_embd,
                            float *mean_out) {
    std::vector<float> sum(n_embd, 0.0f);
    for (uint32_t t = 0; t < n_tok; ++t) {
        const uint16_t *row = k_rows + static_cast<size_t>(t) * n_embd;
        for (uint32_t d = 0; d < n_embd; ++d) sum[d] += f16_to_f32(row[d]);
    }
    if (n_tok == 0) {
        std::fill_n(mean_out, n_embd, 0.0f);
        return;
    }
    const float inv = 1.0f / static_cast<float>(n_tok);
    for (uint32_t d = 0; d < n_embd; ++d) mean_out[d] = sum[d] * inv;
}

// Same, over many (block, layer) units laid out [unit][n_tok][n_embd] -> [unit][n_embd].
ORC_API void orc_mean_k_f16_batch(const uint16_t *k, uint64_t n_units, uint32_t n_tok,
                                  uint32_t n_embd, float *mean_out) {
    for (uint64_t u = 0; u < n_units; ++u)
        orc_mean_k_f16(k + u * static_cast<size_t>(n_tok) * n_embd, n_tok, n_embd,
                       mean_out + u * n_embd);
}

// ---------------------------------------------------------------------------
// S1 — query accumulation.
// src/adapter/llama-memory-kvmem.cpp:3417-3432 (harvest_from_host 'q') and
// :3470-3483 (harvest_capture 'q'): every query-span row is added to
// q_sum_[il] in order, and q_count_[il] is incremented per row.
// reset_query_acc :3300-3315 zeroes both.
//
// q_sum: [qdim] f32 for one layer; rows: [n_rows][qdim] f32.
ORC_API void orc_query_add(float *q_sum, uint32_t *q_count, const float *rows,
                           uint32_t n_rows, uint32_t qdim) {
    for (uint32_t i = 0; i < n_rows; ++i) {
        const float *src = rows + static_cast<size_t>(i) * qdim;
        for (uint32_t d = 0; d < qdim; ++d) q_sum[d] += src[d];
        (*q_count)++;
    }
}

// ---------------------------------------------------------------------------
// S3 — query-to-block scoring.
// src/adapter/llama-memory-kvmem.cpp:4149-4196 (llama_memory_kvmem::score_retrieval).
//
// mean:  [n_blocks][n_layer][n_head_kv * d_head] f32 (the mean_k() of every
//        (block, layer); zeros where absent, as mean_k returns).
// has:   [n_blocks] nonzero when the block holds data (raw_->has_block).
// q_sum: [n_layer][n_head * d_head] f32; q_count: [n_layer].
// scores: [n_blocks] f64.
ORC_API void orc_score(const float *mean, const uint8_t *has, const float *q_sum,
                       const uint32_t *q_count, uint32_t n_blocks, uint32_t n_layer,
                       uint32_t n_head, uint32_t n_head_kv, uint32_t d_head,
                       double *scores) {
    const uint32_t n_embd_k = n_head_kv * d_head;
    const uint32_t g = n_head_kv == 0 ? 1 : n_head / n_head_kv;
    std::vector<float> qh(d_head);
    for (uint32_t b = 0; b < n_blocks; ++b) {
        scores[b] = 0.0;
        if (!has[b]) continue;
        double acc = 0;
        uint32_t nlay = 0;
        for (uint32_t il = 0; il < n_layer; ++il) {
            if (q_count[il] == 0) continue;
            const float *mk = mean + (static_cast<size_t>(b) * n_layer + il) * n_embd_k;
            double layer = 0;
            const float invq = 1.0f / static_cast<float>(q_count[il] * std::max(1u, g));
            for (uint32_t h = 0; h < n_head_kv; ++h) {
                std::fill(qh.begin(), qh.end(), 0.0f);
                for (uint32_t gi = 0; gi < g; ++gi) {
                    const uint32_t qh_i = h * g + gi;
                    if (qh_i >= n_head) break;
                    const float *q = q_sum + static_cast<size_t>(il) * n_head * d_head +
                                     static_cast<size_t>(qh_i) * d_head;
                    for (uint32_t d = 0; d < d_head; ++d) qh[d] += q[d];
                }
                const float *kh = mk + static_cast<size_t>(h) * d_head;
                float dot = 0, nq = 0, nk = 0;
                for (uint32_t d = 0; d < d_head; ++d) {
                    const float qv = qh[d] * invq;
                    dot += qv * kh[d];
                    nq += qv * qv;
                    nk += kh[d] * kh[d];
                }
                layer += dot / (std::sqrt(nq) * std::sqrt(nk) + 1e-6f);
            }
            acc += layer / static_cast<double>(std::max(1u, n_head_kv));
            nlay++;
        }
        scores[b] = nlay ? acc / nlay : 0;
    }
}

// S3 split for layer sharding: the per-(layer, block) term layer / n_head_kv of
// score_retrieval (:4186-4188) for a contiguous range of layers, and the
// layer-ordered reduction acc / nlay (:4189-4193). Composing the two over all
// layers in order is orc_score.
// terms: [n_layer][n_blocks] f64 (0 for inactive layers); active: [n_layer].
ORC_API void orc_score_terms(const float *mean, const float *q_sum, const uint32_t *q_count,
                             uint32_t n_blocks, uint32_t n_layer, uint32_t n_head,
                             uint32_t n_head_kv, uint32_t d_head, double *terms,
                             uint8_t *active) {
    const uint32_t n_embd_k = n_head_kv * d_head;
    const uint32_t g = n_head_kv == 0 ? 1 : n_head / n_head_kv;
    std::vector<float> qh(d_head);
    for (uint32_t il = 0; il < n_layer; ++il) {
        active[il] = q_count[il] != 0;
        for (uint32_t b = 0; b < n_blocks; ++b) {
            double &out = terms[static_cast<size_t>(il) * n_blocks + b];
            out = 0.0;
            if (q_count[il] == 0) continue;
            const float *mk = mean + (static_cast<size_t>(b) * n_layer + il) * n_embd_k;
            double layer = 0;
            const float invq = 1.0f / static_cast<float>(q_count[il] * std::max(1u, g));
            for (uint32_t h = 0; h < n_head_kv; ++h) {
                std::fill(qh.begin(), qh.end(), 0.0f);
                for (uint32_t gi = 0; gi < g; ++gi) {
                    const uint32_t qh_i = h * g + gi;
                    if (qh_i >= n_head) break;
                    const float *q = q_sum + static_cast<size_t>(il) * n_head * d_head +
                                     static_cast<size_t>(qh_i) * d_head;
                    for (uint32_t d = 0; d < d_head; ++d) qh[d] += q[d];
                }
                const float *kh = mk + static_cast<size_t>(h) * d_head;
                float dot = 0, nq = 0, nk = 0;
                for (uint32_t d = 0; d < d_head; ++d) {
                    const float qv = qh[d] * invq;
                    dot += qv * kh[d];
                    nq += qv * qv;
                    nk += kh[d] * kh[d];
                }
                layer += dot / (std::sqrt(nq) * std::sqrt(nk) + 1e-6f);
            }
            out = layer / static_cast<double>(std::max(1u, n_head_kv));
        }
    }
}

ORC_API void orc_score_reduce(const double *terms, const uint8_t *active, const uint8_t *has,
                              uint32_t n_blocks, uint32_t n_layer, double *scores) {
    for (uint32_t b = 0; b < n_blocks; ++b) {
        double acc = 0;
        uint32_t nlay = 0;
        for (uint32_t il = 0; il < n_layer; ++il) {
            if (!active[il]) continue;
            acc += terms[static_cast<size_t>(il) * n_blocks + b];
            nlay++;
        }
        scores[b] = (has[b] && nlay) ? acc / nlay : 0;
    }
}

// ---------------------------------------------------------------------------
// S6 — top-k block selection, TopK policy.
// kvmem/src/host/kvmem_store.cpp:357-359 (pick_topk_blocks -> constrain_media,
// which returns its input unchanged when no media ranges are set, :364) and
// :482-623 (pick_topk_ungrouped): all blocks when n <= budget; else the sink
// prefix, then mandatory ids newest-first while the budget lasts, then the
// `recent` suffix, then the best remaining by (score desc, id desc) via
// nth_element. Returned ascending.
//
// tie_higher_id: 1 = the reference's tie-break (higher id wins, :602-609);
//                0 = lower id wins (the alternative convention).
// Returns the number of ids written to out (capacity >= min(n, budget)).
ORC_API uint32_t orc_pick_topk(const double *scores, uint32_t n, uint32_t budget,
                               uint32_t sink_blocks, uint32_t recent_blocks,
                               const uint32_t *mandatory, uint32_t n_mandatory,
                               int tie_higher_id, uint32_t *out) {
    if (n == 0) return 0;
    if (budget == 0 || n <= budget) {
        for (uint32_t i = 0; i < n; ++i) out[i] = i;
        return n;
    }
    const uint32_t sink = std::min(sink_blocks, n);
    const uint32_t recent = std::min(recent_blocks, n);
    std::vector<bool> kept(n, false);
    uint32_t kept_count = 0;
    auto keep = [&](uint32_t id) {
        if (id < n && !kept[id]) { kept[id] = true; ++kept_count; }
    };
    for (uint32_t i = 0; i < sink && kept_count < budget; ++i) keep(i);
    for (size_t i = n_mandatory; i > 0 && kept_count < budget; --i) keep(mandatory[i - 1]);
    for (uint32_t i = 0; i < recent && kept_count < budget; ++i) keep(n - 1 - i);
    if (kept_count < budget) {
        std::vector<uint32_t> cand;
        cand.reserve(n - kept_count);
        for (uint32_t i = 0; i < n; ++i) if (!kept[i]) cand.push_back(i);
        const uint32_t need = budget - kept_count;
        auto better = [&](uint32_t a, uint32_t b) {
            if (scores[a] != scores[b]) return scores[a] > scores[b];
            return tie_higher_id ? a > b : a < b;
        };
        if (need < cand.size()) {
            std::nth_element(cand.begin(), cand.begin() + need, cand.end(), better);
            cand.resize(need);
        }
        for (uint32_t id : cand) keep(id);
    }
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; ++i) if (kept[i]) out[m++] = i;
    return m;
}

// ---------------------------------------------------------------------------
// S7 — selection diff and window remap plan (default profile: stage-in and
// stage-out optimised, immutable_source_k off unless asked).
// kvmem/src/host/kvmem_store.cpp:179-205 (register_append),
// :758-882 (set_selection), :268-289 (set_block_tier, optimize_stage_out on).
// The runtime's spill/admit (kvmem/src/host/kvmem_runtime.cpp:225-249,
// :269-341) is reduced to its tier effect with no CPU/NVMe tier configured:
// stage_out -> tier CPU, gpu_slot -1; stage_in -> tier GPU.
namespace {
struct OrcBlock {
    uint32_t orig_pos_start = 0, n_tokens = 0;
    bool gpu = true;  // KvTier::GPU is the registration default
    int64_t baked_pos = -1;
    uint32_t remap_count = 0;
    uint64_t remap_abs_delta = 0;
    bool in_working_set = false;
};
struct OrcStore {
    uint32_t block_tokens = 128;
    bool immutable_source_k = false;
    uint32_t refresh_remaps = 8;
    uint64_t refresh_abs_delta = 262144;
    uint64_t max_baked = 262144;
    uint32_t total_tokens = 0;
    std::vector<OrcBlock> blocks;
};
}  // namespace

ORC_API void *orc_store_create(uint32_t block_tokens, int immutable_source_k) {
    auto *s = new OrcStore();
    s->block_tokens = block_tokens;
    s->immutable_source_k = immutable_source_k != 0;
    return s;
}
ORC_API void orc_store_free(void *p) { delete static_cast<OrcStore *>(p); }

ORC_API void orc_store_append(void *p, uint32_t n_new) {
    auto &s = *static_cast<OrcStore *>(p);
    uint32_t remaining = n_new;
    if (!s.blocks.empty() && s.blocks.back().n_tokens < s.block_tokens) {
        const uint32_t take = std::min(s.block_tokens - s.blocks.back().n_tokens, remaining);
        s.blocks.back().n_tokens += take;
        remaining -= take;
        s.total_tokens += take;
    }
    while (remaining > 0) {
        OrcBlock b;
        b.orig_pos_start = s.total_tokens;
        b.n_tokens = std::min(s.block_tokens, remaining);
        b.baked_pos = b.orig_pos_start;
        s.blocks.push_back(b);
        s.total_tokens += b.n_tokens;
        remaining -= b.n_tokens;
    }
}

ORC_API uint32_t orc_store_block_count(void *p) {
    return static_cast<uint32_t>(static_cast<OrcStore *>(p)->blocks.size());
}
ORC_API uint32_t orc_store_block_tokens(void *p, uint32_t id) {
    return static_cast<OrcStore *>(p)->blocks[id].n_tokens;
}

// KvMemStore::truncate_to (kvmem/src/host/kvmem_store.cpp:207-227): pop the
// blocks that start at or past token_pos, shrink the trailing one.
ORC_API void orc_store_truncate(void *p, uint32_t token_pos) {
    auto &s = *static_cast<OrcStore *>(p);
    if (token_pos >= s.total_tokens) return;
    while (!s.blocks.empty() && s.blocks.back().orig_pos_start >= token_pos) {
        s.total_tokens -= s.blocks.back().n_tokens;
        s.blocks.pop_back();
    }
    if (!s.blocks.empty()) {
        OrcBlock &last = s.blocks.back();
        if (last.orig_pos_start + last.n_tokens > token_pos) {
            const uint32_t keep = token_pos - last.orig_pos_start;
            s.total_tokens -= last.n_tokens - keep;
            last.n_tokens = keep;
        }
    }
}

// set_block_tier(id, KvTier::GPU) (kvmem/src/host/kvmem_store.cpp:250-277),
// as the adapter does for a decode block it gives a reserve slot
// (src/adapter/llama-memory-kvmem.cpp:2349-2362).
ORC_API void orc_store_set_tier_gpu(void *p, uint32_t id) {
    auto &s = *static_cast<OrcStore *>(p);
    if (id < s.blocks.size()) s.blocks[id].gpu = true;
}

// KvMemStore::clear_working_set (kvmem/src/host/kvmem_store.cpp:897-901): no
// block stays in the working set; tiers and baked positions are kept.
// drop_gpu (no reference counterpart) also moves every block off the GPU tier.
ORC_API void orc_store_clear_working_set(void *p, int drop_gpu) {
    for (OrcBlock &b : static_cast<OrcStore *>(p)->blocks) {
        b.in_working_set = false;
        if (drop_gpu) b.gpu = false;
    }
}

// Plan output arrays are caller-sized to block_count entries.
// remap rows: block_id, n_tokens, from_base, to_base, working_k_resident, skip, raw_refresh.
// counts[0..5]: n_stage_in, n_stage_out, n_remaps, total_window_tokens,
//               selection_overlap_blocks, gpu_reused_blocks.
ORC_API void orc_store_set_selection(void *p, const uint32_t *ids_in, uint32_t n_ids,
                                     int force_raw_refresh, uint32_t *stage_in,
                                     uint32_t *stage_out, int32_t *remaps /*[n][7]*/,
                                     uint32_t *counts) {
    auto &s = *static_cast<OrcStore *>(p);
    const uint32_t nb = static_cast<uint32_t>(s.blocks.size());
    std::vector<uint32_t> sel(ids_in, ids_in + n_ids);
    std::sort(sel.begin(), sel.end());
    sel.erase(std::unique(sel.begin(), sel.end()), sel.end());
    sel.erase(std::remove_if(sel.begin(), sel.end(), [&](uint32_t id) { return id >= nb; }),
              sel.end());
    std::vector<bool> now(nb, false), was(nb, false);
    for (uint32_t id : sel) now[id] = true;
    uint32_t n_in = 0, n_out = 0, n_rm = 0, overlap = 0, reused = 0;
    for (uint32_t i = 0; i < nb; ++i) {
        was[i] = s.blocks[i].in_working_set;
        if (was[i] && now[i]) ++overlap;
    }
    for (uint32_t i = 0; i < nb; ++i) {
        OrcBlock &b = s.blocks[i];
        if (b.gpu && !now[i]) {
            stage_out[n_out++] = i;
            b.in_working_set = false;
        }
    }
    uint32_t window_pos = 0;
    for (uint32_t id : sel) {
        OrcBlock &b = s.blocks[id];
        if (was[id] && b.gpu) ++reused;
        const bool cold = !b.gpu;
        if (!b.in_working_set) stage_in[n_in++] = id;
        const bool same = b.baked_pos == static_cast<int64_t>(window_pos);
        const bool resident = !cold;
        bool skip = same && (!s.immutable_source_k || resident) && !force_raw_refresh;
        bool raw = false;
        const uint64_t delta = static_cast<uint64_t>(
            b.baked_pos > static_cast<int64_t>(window_pos) ? b.baked_pos - window_pos
                                                           : window_pos - b.baked_pos);
        if (s.immutable_source_k && (cold || !same)) {
            const bool remap_limit = s.refresh_remaps > 0 && b.remap_count >= s.refresh_remaps;
            const bool delta_limit =
                s.refresh_abs_delta > 0 &&
                (b.remap_abs_delta >= s.refresh_abs_delta ||
                 delta >= s.refresh_abs_delta - std::min<uint64_t>(b.remap_abs_delta,
                                                                   s.refresh_abs_delta));
            const bool out_of_range =
                s.max_baked > 0 &&
                (b.baked_pos < 0 || static_cast<uint64_t>(b.baked_pos) + b.n_tokens > s.max_baked);
            raw = cold || remap_limit || delta_limit || out_of_range;
        }
        if (s.immutable_source_k && force_raw_refresh) raw = true;
        int32_t *r = remaps + 7 * n_rm++;
        r[0] = static_cast<int32_t>(id);
        r[1] = static_cast<int32_t>(b.n_tokens);
        r[2] = static_cast<int32_t>(b.baked_pos);
        r[3] = static_cast<int32_t>(window_pos);
        r[4] = resident ? 1 : 0;
        r[5] = skip ? 1 : 0;
        r[6] = raw ? 1 : 0;
        b.in_working_set = true;
        if (!skip) {
            if (raw) { b.remap_count = 0; b.remap_abs_delta = 0; }
            else { ++b.remap_count; b.remap_abs_delta += delta; }
        }
        b.baked_pos = static_cast<int64_t>(window_pos);
        window_pos += b.n_tokens;
    }
    // Runtime effect (spill_outgoing then admit_incoming, no lower tier).
    for (uint32_t k = 0; k < n_out; ++k) s.blocks[stage_out[k]].gpu = false;
    for (uint32_t k = 0; k < n_in; ++k) s.blocks[stage_in[k]].gpu = true;
    counts[0] = n_in;
    counts[1] = n_out;
    counts[2] = n_rm;
    counts[3] = window_pos;
    counts[4] = overlap;
    counts[5] = reused;
}

// ---------------------------------------------------------------------------
// S12 — NeoX RoPE.
// kvmem/src/host/rope.cpp:8-45 (rope_neox_apply): theta_i = pow(base, -2i/n_rot)
// * scale in float; per pair (i, i+half) at position pos0 + t:
//   (x0*c - x1*s, x0*s + x1*c), dims >= n_rot copied.
// k: token-major [n_tok][n_head][n_embd_head] f32.
ORC_API void orc_rope_neox(const float *k, uint32_t n_tok, uint32_t n_head,
                           uint32_t n_embd_head, uint32_t n_rot, int32_t pos0,
                           float freq_base, float freq_scale, float *out) {
    const uint32_t half = n_rot / 2;
    std::vector<float> theta(half);
    for (uint32_t i = 0; i < half; ++i) {
        theta[i] = std::pow(freq_base, -2.0f * static_cast<float>(i) / static_cast<float>(n_rot));
        theta[i] *= freq_scale;
    }
    const uint32_t tok_stride = n_head * n_embd_head;
    for (uint32_t t = 0; t < n_tok; ++t) {
        const float pos = static_cast<float>(pos0 + static_cast<int32_t>(t));
        for (uint32_t h = 0; h < n_head; ++h) {
            const float *src = k + static_cast<size_t>(t) * tok_stride + h * n_embd_head;
            float *dst = out + static_cast<size_t>(t) * tok_stride + h * n_embd_head;
            for (uint32_t i = 0; i < half; ++i) {
                const float c = std::cos(pos * theta[i]);
                const float s = std::sin(pos * theta[i]);
                const float x0 = src[i];
                const float x1 = src[i + half];
                dst[i] = x0 * c - x1 * s;
                dst[i + half] = x0 * s + x1 * c;
            }
            for (uint32_t i = n_rot; i < n_embd_head; ++i) dst[i] = src[i];
        }
    }
}

// theta table exactly as the host RoPE computes it (rope.cpp:20-24).
ORC_API void orc_rope_theta(uint32_t n_rot, float freq_base, float freq_scale, float *theta) {
    for (uint32_t i = 0; i < n_rot / 2; ++i) {
        theta[i] = std::pow(freq_base, -2.0f * static_cast<float>(i) / static_cast<float>(n_rot));
        theta[i] *= freq_scale;
    }
}

// Window K for one f16 block: f16 unrotated K -> f32 -> RoPE at pos0 -> f16 RNE.
ORC_API void orc_rope_block_f16(const uint16_t *k, uint32_t n_tok, uint32_t n_head,
                                uint32_t n_embd_head, uint32_t n_rot, int32_t pos0,
                                float freq_base, float freq_scale, uint16_t *out) {
    const size_t n = static_cast<size_t>(n_tok) * n_head * n_embd_head;
    std::vector<float> a(n), b(n);
    for (size_t i = 0; i < n; ++i) a[i] = f16_to_f32(k[i]);
    orc_rope_neox(a.data(), n_tok, n_head, n_embd_head, n_rot, pos0, freq_base, freq_scale,
                  b.data());
    for (size_t i = 0; i < n; ++i) out[i] = f32_to_f16(b[i]);
}

// ---------------------------------------------------------------------------
// S13 — q8_0 / q4_0 dequant, FWHT and requant (the stage-in K item path).
// src/adapter/llama-kvmem-stagein.cu:133-143 (dequant_q8_0), :145-158
// (dequant_q4_0), :105-131 (fwht_kernel: scale applied on input, butterfly
// stages h = 1, 2, 4, ...), :181-199 (quant_q8_0), :201-234 (quant_q4_0), and
// the per-item order dequant -> RoPE -> FWHT -> quant at :746-785.
// Blocks: q8_0 = {f16 d; int8 qs[32]} (34 B), q4_0 = {f16 d; u8 qs[16]} (18 B).
ORC_API void orc_dequant_q8_0(const uint8_t *x, float *y, uint64_t n_blocks) {
    for (uint64_t i = 0; i < n_blocks; ++i) {
        const uint8_t *b = x + i * 34;
        uint16_t dh;
        std::memcpy(&dh, b, 2);
        const float d = f16_to_f32(dh);
        for (int j = 0; j < 32; ++j)
            y[i * 32 + j] = static_cast<float>(static_cast<int8_t>(b[2 + j])) * d;
    }
}

ORC_API void orc_dequant_q4_0(const uint8_t *x, float *y, uint64_t n_blocks) {
    for (uint64_t i = 0; i < n_blocks; ++i) {
        const uint8_t *b = x + i * 18;
        uint16_t dh;
        std::memcpy(&dh, b, 2);
        const float d = f16_to_f32(dh);
        for (int j = 0; j < 16; ++j) {
            const int x0 = (b[2 + j] & 0x0F) - 8;
            const int x1 = (b[2 + j] >> 4) - 8;
            y[i * 32 + j] = static_cast<float>(x0) * d;
            y[i * 32 + j + 16] = static_cast<float>(x1) * d;
        }
    }
}

ORC_API void orc_quant_q8_0(const float *x, uint8_t *y, uint64_t n_blocks) {
    for (uint64_t i = 0; i < n_blocks; ++i) {
        const float *src = x + i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(src[j]));
        const float d = amax / 127.0f;
        const float id = d ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        uint8_t *b = y + i * 34;
        std::memcpy(b, &dh, 2);
        for (int j = 0; j < 32; ++j)
            b[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(std::round(src[j] * id)));
    }
}

ORC_API void orc_quant_q4_0(const float *x, uint8_t *y, uint64_t n_blocks) {
    for (uint64_t i = 0; i < n_blocks; ++i) {
        const float *src = x + i * 32;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = src[j];
            if (amax < std::fabs(v)) { amax = std::fabs(v); vmax = v; }
        }
        const float d = vmax / -8.0f;
        const float id = d ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        uint8_t *b = y + i * 18;
        std::memcpy(b, &dh, 2);
        for (int j = 0; j < 16; ++j) {
            const float x0 = src[j] * id;
            const float x1 = src[j + 16] * id;
            int xi0 = static_cast<int>(x0 + 8.5f);
            int xi1 = static_cast<int>(x1 + 8.5f);
            if (xi0 > 15) xi0 = 15;
            if (xi1 > 15) xi1 = 15;
            b[2 + j] = static_cast<uint8_t>((xi0 & 15) | ((xi1 & 15) << 4));
        }
    }
}

// In-place FWHT over rows of length n (n in {64, 128, 256, 512}).
ORC_API void orc_fwht(float *x, uint64_t n_rows, uint32_t n) {
    const float scale = 1.0f / std::sqrt(static_cast<float>(n));
    std::vector<float> tmp(n);
    for (uint64_t r = 0; r < n_rows; ++r) {
        float *row = x + r * n;
        for (uint32_t i = 0; i < n; ++i) tmp[i] = row[i] * scale;
        for (uint32_t h = 1; h < n; h *= 2)
            for (uint32_t i = 0; i < n; i += 2 * h)
                for (uint32_t j = 0; j < h; ++j) {
                    const float a = tmp[i + j];
                    const float b = tmp[i + j + h];
                    tmp[i + j] = a + b;
                    tmp[i + j + h] = a - b;
                }
        for (uint32_t i = 0; i < n; ++i) row[i] = tmp[i];
    }
}

// Hadamard by explicit matrix, src/adapter/llama-kvmem-quant.h:250-302
// (kvmem_hadamard_matrix + kvmem_hadamard_rows). A cross-check of orc_fwht.
ORC_API void orc_hadamard_rows(float *rows, uint64_t n_rows, uint32_t n_head,
                               uint32_t n_embd_head, uint32_t nrot) {
    std::vector<float> H(static_cast<size_t>(nrot) * nrot, 0.0f);
    H[0] = 1.0f / std::sqrt(static_cast<float>(nrot));
    for (uint32_t s = 1; s < nrot; s *= 2)
        for (uint32_t i = 0; i < s; ++i)
            for (uint32_t j = 0; j < s; ++j) {
                const float v = H[static_cast<size_t>(i) * nrot + j];
                H[static_cast<size_t>(i + s) * nrot + j] = v;
                H[static_cast<size_t>(i) * nrot + j + s] = v;
                H[static_cast<size_t>(i + s) * nrot + j + s] = -v;
            }
    std::vector<float> tmp(nrot);
    const uint64_t row = static_cast<uint64_t>(n_head) * n_embd_head;
    for (uint64_t t = 0; t < n_rows; ++t)
        for (uint32_t h = 0; h < n_head; ++h)
            for (uint32_t off = 0; off < n_embd_head; off += nrot) {
                float *x = rows + t * row + static_cast<uint64_t>(h) * n_embd_head + off;
                for (uint32_t i = 0; i < nrot; ++i) {
                    float acc = 0.0f;
                    for (uint32_t j = 0; j < nrot; ++j) acc += H[static_cast<size_t>(i) * nrot + j] * x[j];
                    tmp[i] = acc;
                }
                std::memcpy(x, tmp.data(), nrot * sizeof(float));
            }
}

// Window K for one q8_0 block: dequant -> RoPE at pos0 -> FWHT(nrot, 0 = off)
// -> q8_0. k_q8: [n_tok][n_head*n_embd_head/32] q8_0 blocks.
ORC_API void orc_rope_block_q8_0(const uint8_t *k_q8, uint32_t n_tok, uint32_t n_head,
                                 uint32_t n_embd_head, uint32_t n_rot, int32_t pos0,
                                 float freq_base, float freq_scale, uint32_t fwht_n,
                                 uint8_t *out) {
    const size_t n = static_cast<size_t>(n_tok) * n_head * n_embd_head;
    std::vector<float> a(n), b(n);
    orc_dequant_q8_0(k_q8, a.data(), n / 32);
    orc_rope_neox(a.data(), n_tok, n_head, n_embd_head, n_rot, pos0, freq_base, freq_scale,
                  b.data());
    if (fwht_n) orc_fwht(b.data(), n / fwht_n, fwht_n);
    orc_quant_q8_0(b.data(), out, n / 32);
}

// The same item path for q4_0 K (dequant_q4_0 / quant_q4_0, stagein.cu:145-158,
// :201-234). k_q4: [n_tok][n_head*n_embd_head/32] q4_0 blocks.
ORC_API void orc_rope_block_q4_0(const uint8_t *k_q4, uint32_t n_tok, uint32_t n_head,
                                 uint32_t n_embd_head, uint32_t n_rot, int32_t pos0,
                                 float freq_base, float freq_scale, uint32_t fwht_n,
                                 uint8_t *out) {
    const size_t n = static_cast<size_t>(n_tok) * n_head * n_embd_head;
    std::vector<float> a(n), b(n);
    orc_dequant_q4_0(k_q4, a.data(), n / 32);
    orc_rope_neox(a.data(), n_tok, n_head, n_embd_head, n_rot, pos0, freq_base, freq_scale,
                  b.data());
    if (fwht_n) orc_fwht(b.data(), n / fwht_n, fwht_n);
    orc_quant_q4_0(b.data(), out, n / 32);
}

// ---------------------------------------------------------------------------
// Host stage-in of one step for the benchmark's CPU arms when the reference
// library was not built: units [u0, u1) of (block, layer) K rotated with
// orc_rope_block_f16 at their window bases, V bytes copied; and a list of
// byte copies (the staging memcpy).
ORC_API void orc_rope_units_f16(const uint16_t *const *k_src, uint16_t *const *k_dst,
                                const uint8_t *const *v_src, uint8_t *const *v_dst,
                                uint64_t v_bytes, const int32_t *pos0, uint32_t u0, uint32_t u1,
                                uint32_t n_tok, uint32_t n_head, uint32_t n_embd_head,
                                float freq_base, float freq_scale) {
    for (uint32_t u = u0; u < u1; ++u) {
        orc_rope_block_f16(k_src[u], n_tok, n_head, n_embd_head, n_embd_head, pos0[u], freq_base,
                           freq_scale, k_dst[u]);
        if (v_bytes) std::memcpy(v_dst[u], v_src[u], v_bytes);
    }
}

// q8_0 K units: dequant -> RoPE -> FWHT -> requant (orc_rope_block_q8_0).
ORC_API void orc_rope_units_q8_0(const uint8_t *const *k_src, uint8_t *const *k_dst,
                                 const uint8_t *const *v_src, uint8_t *const *v_dst,
                                 uint64_t v_bytes, const int32_t *pos0, uint32_t u0, uint32_t u1,
                                 uint32_t n_tok, uint32_t n_head, uint32_t n_embd_head,
                                 float freq_base, float freq_scale, uint32_t fwht_n) {
    for (uint32_t u = u0; u < u1; ++u) {
        orc_rope_block_q8_0(k_src[u], n_tok, n_head, n_embd_head, n_embd_head, pos0[u], freq_base,
                            freq_scale, fwht_n, k_dst[u]);
        if (v_bytes) std::memcpy(v_dst[u], v_src[u], v_bytes);
    }
}

ORC_API void orc_copy_list(const uint8_t *const *src, uint8_t *const *dst, const uint64_t *nbytes,
                           uint32_t i0, uint32_t i1) {
    for (uint32_t i = i0; i < i1; ++i) std::memcpy(dst[i], src[i], nbytes[i]);
}
