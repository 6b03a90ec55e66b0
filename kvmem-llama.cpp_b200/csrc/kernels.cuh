// Kernel launchers shared by the context and the C ABI. All launches are
// asynchronous on the given stream and return the launch's cudaError_t.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace kvmret {

// One window-assembly job: rebuild window slot `win_slot` of every layer from
// HBM pool slot `pool_slot` (or, for a fresh block, from block `block` of the
// mapped host repository, also filling the pool slot), K rotated at positions
// pos0 .. pos0 + n_tok - 1.
struct Job {
    uint32_t pool_slot;
    uint32_t win_slot;
    int32_t pos0;
    uint32_t n_tok;
    uint32_t block;
    uint32_t pad[3];
};
static_assert(sizeof(Job) == 32, "Job is 32 bytes");

// RoPE frequencies theta_i = freq_base^(-2i/n_rot) * freq_scale, computed on
// the host exactly as the reference's host RoPE does; passed by value.
struct Theta {
    float v[128];
};

struct AssembleGeom {
    uint32_t n_layer;
    uint32_t n_head_kv;
    uint32_t d_head;
    uint32_t block_tokens;
    uint64_t k_row;         // bytes per K token row (window and pool)
    uint64_t v_row;         // bytes per V token row
    uint64_t unit_k;        // pool/repo bytes of the K part of one (block, layer) unit
    uint64_t unit;          // pool/repo bytes of one (block, layer) unit (K part + V part)
    uint64_t win_k_layer;   // window K bytes per layer
    uint64_t win_v_layer;   // window V bytes per layer
    int32_t k_type;
    uint32_t fwht_n;        // 0 = no Hadamard on requantised K
    float fwht_scale;       // 1 / sqrt(fwht_n), computed on the host
};

// S1: q_sum[l][e] += sum over rows (row order), f16 or f32 rows [L][n_rows][qdim];
// q_count (optional, device) += n_rows per layer; assign: start from zero.
cudaError_t launch_query_add(float *q_sum, const void *rows, bool rows_f16, uint32_t n_layer,
                             uint32_t n_rows, uint32_t qdim, cudaStream_t st,
                             uint32_t *q_count = nullptr, bool assign = false);

// S3 prologue: per (layer, kv head) the scaled group query and its squared norm.
// With flag_col set, each layer's query flag (1.0 / 0.0) is also written to
// flag_col[l * cstride + cstride - 1] (the packed exchange row).
cudaError_t launch_qprep(const float *q_sum, const uint32_t *q_count, float *qv, float *nq,
                         uint8_t *active, uint32_t n_layer, uint32_t n_head,
                         uint32_t n_head_kv, uint32_t d_head, cudaStream_t st,
                         double *flag_col = nullptr, uint32_t cstride = 0);

// S3: per (layer, block) term layer_sum / n_head_kv into contrib rows of
// cstride doubles (0 = ncap).
// Peer-memory exchange of the layer-sharded score rows (NVLink, no
// collective), pull form: every rank's scoring writes its rows into its own
// exchange region; the last CTA then publishes the step in every rank's flag
// array (flags[p] is rank p's array, one word per rank); counter is a device
// word the last CTA uses to know every CTA has finished. The reductions read
// the peers' rows from their regions (RowSource).
constexpr int kMaxRanks = 8;
struct Peers {
    uint32_t *flags[kMaxRanks];
    uint32_t *counter;
    uint32_t n, rank, step, n_layer;
};
// Where the reduction finds the rows of the global layers: layer g of rank
// g / l_local at base[g / l_local] + (g % l_local) * stride (n_ranks = 0: the
// rows are contiguous at `contrib`).
struct RowSource {
    const double *base[kMaxRanks];
    uint32_t l_local, n_ranks;
};

cudaError_t launch_score(const float *summ, const float *qv, const float *nq,
                         const uint8_t *active, double *contrib, uint32_t n_layer,
                         uint32_t n_head_kv, uint32_t d_head, uint32_t ncap,
                         uint32_t n_blocks, cudaStream_t st, uint32_t cstride = 0,
                         const Peers *peers = nullptr);

// S3 epilogue: layer-ordered sum, / number of layers with a query. With
// active == nullptr the flags are read from each row's last column.
// With wait_flags, each CTA first waits (at most 2 s) until every one of the
// wait_n ranks' flags has reached wait_step; on a timeout it sets *err.
cudaError_t launch_reduce(const double *contrib, const uint8_t *active, uint32_t n_layer,
                          uint32_t stride, const uint8_t *has_block, uint32_t n_blocks,
                          double *scores, cudaStream_t st, const uint32_t *wait_flags = nullptr,
                          uint32_t wait_n = 0, uint32_t wait_step = 0, uint32_t *err = nullptr,
                          const RowSource *rows = nullptr);

// S6: sel[b] = kept[b] || (rank of b among non-kept blocks < need).
cudaError_t launch_select(const double *scores, const uint8_t *kept, uint32_t n_blocks,
                          uint32_t need, int tie_higher_id, uint8_t *sel, cudaStream_t st);

// S10-S13: window assembly from the HBM pool. One launch rebuilds n_jobs
// window slots on every layer. With jobs == nullptr the jobs are synthesised:
// job i covers tokens [i*T, min((i+1)*T, synth_ntok)) of a contiguous run,
// pool slot i -> window slot i, positions from synth_pos0. gtab is the cos/sin
// table, [position][n_rot/4] x {c_2j, c_2j+1, s_2j, s_2j+1}, covering every
// position the launch uses (the f16 form may pass null: evaluate on the fly;
// quantised K requires it).
struct AsmLaunch {
    const Job *jobs;
    // Device job counts {moved, fresh} written by the plan kernel (nullptr: the
    // launch's n_jobs jobs are all moved jobs). Moved jobs sit at jobs[0..),
    // fresh jobs at jobs[fresh_offset..); CTAs beyond the counts exit at once.
    const uint32_t *counts;
    uint32_t *work;         // with counts: work counter (zeroed by the plan kernel); the
                            // quantised form's fresh-item counter
    uint32_t *work_moved;   // the quantised form's moved-item counter (zeroed by the plan)
    uint32_t fresh_offset;
    uint32_t n_groups;      // layer groups per job (set by the launcher)
    const uint8_t *repo;    // device alias of the mapped pinned repository (fresh jobs)
    uint8_t *pool_w;        // writable pool base (fresh jobs fill their slot)
    const uint8_t *pool;
    uint64_t slot_bytes;
    uint8_t *win_k;
    uint8_t *win_v;
    const float4 *gtab;
    int32_t synth_pos0;
    uint32_t synth_ntok;
    Theta theta;
    AssembleGeom g;
};
cudaError_t launch_assemble(const AsmLaunch &a, uint32_t n_jobs, cudaStream_t st);

// Device plan of one step (S7/S9-S11 physical part): from the selection flags,
// the chronological window (ids ascending, bases = running token sums), the
// HBM pool slots (release of blocks that left unless caching, LRU eviction,
// allocation in slot order), the moved / fresh job lists, the window update,
// and counts {n_moved, n_fresh, n_sel, window_tokens, error, moved_tokens,
// fresh_tokens} plus the selected ids for the host.
struct PlanArgs {
    const uint8_t *sel;
    const uint32_t *blk_ntok;
    uint32_t n_blocks, win_slots, pool_slots, step;
    int pool_cache;
    int32_t *win_id;
    int32_t *win_base;
    uint32_t *win_ntok;
    int32_t *blk_slot;
    int32_t *slot_blk;
    uint32_t *slot_ntok;
    uint32_t *slot_used;
    Job *jobs;          // [2 * win_slots]: moved, then fresh at + win_slots
    uint32_t *counts;   // [9]: 8 read back per step, [7] and [8] work counters
    uint32_t *ids;      // [win_slots]
    uint32_t *ext_err;  // optional: a nonzero word here (read and cleared) fails the step as 0x100
};
cudaError_t launch_plan(const PlanArgs &a, cudaStream_t st);
size_t plan_smem_bytes(uint32_t win_slots, uint32_t pool_slots);

// cos/sin table of positions [0, n_pos) for the window (see AsmLaunch::gtab).
cudaError_t launch_rope_table(float4 *cs, uint32_t n_pos, uint32_t half, const Theta &th,
                              cudaStream_t st, int32_t pos_base = 0);

// S2 + S14: summaries of the appended tokens and the repository rows.
struct AppendArgs {
    const uint16_t *k_cap;   // [L][n][E] f16
    const uint8_t *k_rows;   // [L][n][k_row]
    const uint8_t *v_rows;   // [L][n][v_row]
    uint32_t pos0, n_tok;
    uint32_t n_layer, n_head_kv, d_head, block_tokens, ncap;
    uint64_t k_row, v_row, unit_k, unit;
    float *summ;             // [L][Hkv][D][ncap]
    uint32_t *blk_ntok;      // [ncap] tokens per block (kept current for the device plan)
    float *tail_sum;         // [L][E] running sum of the trailing partial block
    uint8_t *has_block;      // [ncap]
    uint8_t *repo_dev;       // device alias of the mapped pinned repository
};
cudaError_t launch_append(const AppendArgs &a, cudaStream_t st);

// f16 rows -> q8_0 (q8 = true) or q4_0 blocks of 32 elements.
cudaError_t launch_quantize(const uint16_t *x, uint8_t *y, uint64_t n_blocks, bool q8,
                            cudaStream_t st);

// ---- gen-reserve placement: decode blocks bound to reserve window slots ----
// One binding: window slot `win_slot` (RoPE base `base`) and pool slot
// `pool_slot` now hold `block`, whose first `n_exist` rows are already in the
// pool slot; `evict_block` (>= 0) loses its pool slot.
struct GenBind {
    uint32_t block, win_slot, pool_slot, n_exist;
    int32_t base, evict_block;
};
constexpr int kMaxGenBinds = 64;  // = kMaxGenSegs: every touched block may bind
struct GenBinds {
    GenBind b[kMaxGenBinds];
    uint32_t n, step;
    int32_t *win_id;
    int32_t *win_base;
    uint32_t *win_ntok;
    int32_t *blk_slot;
    int32_t *slot_blk;
    uint32_t *slot_ntok;
    uint32_t *slot_used;
};
cudaError_t launch_gen_bind(const GenBinds &g, cudaStream_t st);

// Rows of one bound block written into its window slot (K rotated at the
// slot's base + row, V copied) and its pool slot (unrotated): rows
// [rebuild_lo, new_lo) from the pool slot, rows [new_lo, new_hi) from the
// caller's append rows starting at append token tok0.
struct GenSeg {
    uint32_t block, rebuild_lo, new_lo, new_hi, tok0;
};
constexpr int kMaxGenSegs = 64;
struct GenWrite {
    GenSeg seg[kMaxGenSegs];
    uint32_t n_seg, n_tok_append, win_slots;
    const uint8_t *k_rows;  // [n_layer][n_tok_append][k_row] unrotated K
    const uint8_t *v_rows;  // [n_layer][n_tok_append][v_row]
    uint8_t *pool;
    uint64_t slot_bytes;
    uint8_t *win_k;
    uint8_t *win_v;
    const float4 *gtab;     // the window's position table
    const int32_t *win_id;
    const int32_t *win_base;
    const int32_t *blk_slot;
    uint32_t *win_ntok;
    uint32_t *slot_ntok;
    uint32_t *err;          // set to 1 when a bound block is not in the window
    AssembleGeom g;
};
static_assert(kMaxGenBinds >= kMaxGenSegs, "every block an append touches may need a binding");
cudaError_t launch_gen_write(const GenWrite &a, cudaStream_t st);

// Truncation (KvMemStore::truncate_to + RawKvStore::truncate_to): blocks
// [nb_new, nb_old) leave the block set, the pool and the window; with
// tail_ntok > 0 block nb_new - 1 keeps tail_ntok tokens.
struct TruncArgs {
    uint32_t nb_new, nb_old, tail_ntok, pool_slots, win_slots;
    uint8_t *has_block;
    uint32_t *blk_ntok;
    int32_t *blk_slot;
    int32_t *slot_blk;
    uint32_t *slot_ntok;
    int32_t *win_id;
    uint32_t *win_ntok;
};
cudaError_t launch_truncate(const TruncArgs &a, cudaStream_t st);
// The summary and running tail sum of a partial f16 block recomputed from the
// repository's first n_tok unrotated K rows (token-order f32 sum, * 1/n_tok).
cudaError_t launch_resum(const AppendArgs &a, uint32_t block, uint32_t n_tok, cudaStream_t st);

struct CopyOp {
    const uint8_t *src;
    uint8_t *dst;
    uint64_t nbytes;
};
cudaError_t launch_copy_ops(const CopyOp *ops, int n, cudaStream_t st);

}  // namespace kvmret
