/*
 * kvmret — B200-native KVMem per-step KV retrieval path, C ABI.
 *
 * The path: score the current GQA query against per-block mean-key summaries,
 * pick a deterministic block top-k (sink + mandatory pinning), diff it against
 * the current working set, stage the selected 128-token blocks from the pinned
 * host repository / HBM block pool into a chronologically ordered window with
 * K re-rotated (RoPE) at its window position (dequant -> RoPE -> FWHT -> requant
 * for q8_0 K), and append completed blocks back to the repository with their
 * summaries.
 *
 * Every entry point returns an int status (KVMRET_OK == 0, negative on error);
 * kvmret_last_error() describes the last failure on the calling thread. No C++
 * exception crosses this boundary. Pointers named *_dev are device pointers,
 * *_host are host pointers. A context is bound to one CUDA device and must not
 * be used concurrently from two threads (the reference's rule for an execution
 * state, src/adapter/llama-kvmem-hooks.h:46-50).
 *
 * Reference interfaces replaced (paths inside zyf32453/kvmem-llama.cpp) are
 * cited per function.
 */
#ifndef KVMRET_H
#define KVMRET_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVMRET_OK 0
#define KVMRET_ERR_ARG (-1)     /* bad argument or size out of range */
#define KVMRET_ERR_CUDA (-2)    /* a CUDA runtime call failed */
#define KVMRET_ERR_STATE (-3)   /* call not valid in the current state */
#define KVMRET_ERR_NOMEM (-4)   /* device or pinned host allocation failed */

/* KV element formats; values are ggml_type ids (F16 = 1, Q4_0 = 2, Q8_0 = 8). */
#define KVMRET_TYPE_F16 1
#define KVMRET_TYPE_Q4_0 2
#define KVMRET_TYPE_Q8_0 8

typedef struct kvmret_ctx kvmret_ctx;
typedef struct kvmret_table kvmret_table;

/*
 * Context configuration. Mirrors the parts of llama_kvmem_params
 * (src/adapter/llama-kvmem-hooks.h:19-39), KvMemStoreConfig
 * (kvmem/include/kvmem/kvmem_store.hpp:231-327) and the adapter's model
 * geometry / RoPE config (src/adapter/llama-memory-kvmem.cpp:929-944) that the
 * retrieval path reads.
 */
typedef struct kvmret_config {
    uint32_t n_layer;        /* layers held by this context (a shard) */
    uint32_t n_head;         /* query heads */
    uint32_t n_head_kv;      /* KV heads */
    uint32_t d_head;         /* head dim: 64, 128 or 256 */
    uint32_t block_tokens;   /* tokens per block (reference default 128) */
    uint32_t max_blocks;     /* history capacity in blocks */
    uint32_t budget_blocks;  /* selection budget W (select_budget / block_tokens) */
    uint32_t reserve_blocks; /* gen-reserve window slots beyond the budget */
    uint32_t sink_blocks;    /* always-kept prefix (reference default 1) */
    uint32_t recent_blocks;  /* always-kept suffix (reference default 0) */
    uint32_t pool_blocks;    /* HBM raw-block pool slots; 0 -> budget + reserve */
    int32_t k_type;          /* KVMRET_TYPE_F16 or KVMRET_TYPE_Q8_0 */
    int32_t v_type;          /* KVMRET_TYPE_F16, _Q8_0 or _Q4_0 (copied as bytes) */
    int32_t attn_rot_k;      /* FWHT on re-roped quantised K: -1 auto (on for
                                quantised K, n_embd_head % 64 == 0), 0 off, 1 on */
    int32_t tie_higher_id;   /* top-k tie-break: 1 higher id (reference), 0 lower */
    int32_t pool_cache;      /* 1: keep evicted blocks in free pool slots as a cache */
    int32_t immutable_source_k; /* KvMemStoreConfig::immutable_source_k (plan flags) */
    uint32_t n_rot;          /* rotated dims (== d_head for NeoX full rotary) */
    float freq_base;         /* rope_freq_base */
    float freq_scale;        /* rope_freq_scale */
    int32_t device;          /* CUDA device ordinal */
} kvmret_config;

/* Counters for one apply step; the KVMEM_RETR_SUM buckets of
 * src/adapter/llama-memory-kvmem.cpp:4198-4216 that this path owns. */
typedef struct kvmret_step_stats {
    uint32_t n_selected;      /* blocks in the new window */
    uint32_t n_stage_in;      /* plan.stage_in (newly in the working set) */
    uint32_t n_stage_out;     /* plan.stage_out */
    uint32_t n_skip;          /* plan remaps with skip set */
    uint32_t n_h2d_blocks;    /* blocks read from the host repository this step */
    uint32_t n_assembled;     /* window slots rewritten (new + moved) */
    uint32_t n_moved;         /* window slots rewritten from a resident block */
    uint32_t total_window_tokens;
    uint64_t h2d_bytes;       /* host -> device bytes of the stage-in (host link) */
    uint64_t assemble_bytes;  /* HBM bytes read + written by window assembly */
} kvmret_step_stats;

/* Defaults as the reference CLI/server recipes use them. */
void kvmret_config_default(kvmret_config *cfg);

/* Bytes of one token row of a format (e.g. q8_0 of 1024 elements = 1088). */
uint64_t kvmret_row_bytes(int32_t type, uint32_t n_elems);

const char *kvmret_last_error(void);
const char *kvmret_version(void);

/* ---- context (llama_kvmem_execution_create / kvmem_gpu_state_create,
 *      src/adapter/llama-kvmem-stagein.cu:345-354; llama_memory_kvmem ctor,
 *      src/adapter/llama-memory-kvmem.cpp:829-998) ---- */
int kvmret_create(const kvmret_config *cfg, kvmret_ctx **out);
void kvmret_destroy(kvmret_ctx *ctx);
/* The context's compute stream (cudaStream_t). */
void *kvmret_stream(kvmret_ctx *ctx);
int kvmret_sync(kvmret_ctx *ctx);

/* ---- host repository (RawKvStore, kvmem/include/kvmem/raw_kv_store.hpp:40-170):
 *      pinned, mapped host memory laid out [block][layer][K rows | V rows]. ---- */
void *kvmret_repo_host(kvmret_ctx *ctx);
uint64_t kvmret_repo_unit_bytes(kvmret_ctx *ctx);  /* one (block, layer): K + V */
uint64_t kvmret_repo_k_bytes(kvmret_ctx *ctx);     /* K part of a unit */

/*
 * Append tokens [pos0, pos0 + n_tok) for every layer of the context
 * (S14 + S2). Replaces the harvest path: RawKvStore::write_layer_mean_k
 * (kvmem/src/host/raw_kv_store.cpp:685-705), write_layer_k_gpu / v_gpu
 * (:600-683), KvMemStore::register_append (kvmem/src/host/kvmem_store.cpp:
 * 179-205) and harvest_full_blocks_async (src/adapter/llama-memory-kvmem.cpp:
 * 3692-3729). pos0 must equal the current token count.
 *   k_cap_dev: [n_layer][n_tok][n_head_kv * d_head] f16 pre-RoPE K (summary source)
 *   k_rows_dev: [n_layer][n_tok][k row bytes] unrotated K in k_type (NULL: use
 *               k_cap_dev, valid only when k_type is F16)
 *   v_rows_dev: [n_layer][n_tok][v row bytes] V in v_type
 * The summary of every touched block is its F32 token-order mean.
 */
int kvmret_append(kvmret_ctx *ctx, uint32_t pos0, uint32_t n_tok, const uint16_t *k_cap_dev,
                  const void *k_rows_dev, const void *v_rows_dev);
uint32_t kvmret_n_blocks(kvmret_ctx *ctx);
uint32_t kvmret_n_tokens(kvmret_ctx *ctx);
/* KvMemRuntime::truncate_to (kvmem/src/host/kvmem_runtime.cpp:94-112,
 * KvMemStore::truncate_to kvmem/src/host/kvmem_store.cpp:207-227,
 * RawKvStore::truncate_to kvmem/src/host/raw_kv_store.cpp:1096-1126): keep
 * the first n_tokens tokens. Blocks past them leave the store, the HBM pool
 * and the window; a partial last block keeps its first tokens, its f16
 * summary rebuilt from the repository's K rows (quantised K: block
 * boundaries only, since the repository holds no f16 K). Collects steps in
 * flight first. */
int kvmret_truncate(kvmret_ctx *ctx, uint32_t n_tokens);

/* ---- gen-reserve placement (S15): the adapter's prepare_working_set after
 *      a retrieval (src/adapter/llama-memory-kvmem.cpp:2314-2365: "pin the
 *      working set and place decode tokens into gen_reserve slots"), its
 *      alloc_slot (:1720-1741) and the cell mapping of kvmem_fill_slot_info
 *      (src/adapter/llama-kvmem-batch.cpp:5-58). ----
 * kvmret_gen_begin: from now on every block that kvmret_append touches (the
 * decode blocks: the block holding the next token and those after it) gets a
 * window slot of its own when it has none (the first free slot: it is the
 * newest block, so that is its chronological place, RoPE base = the window's
 * token count), plus an HBM pool slot, and each append writes its tokens into
 * that window slot (K rotated at base + offset; quantised K dequantised,
 * rotated, Hadamard-transformed and requantised) and into the pool slot, so
 * attention sees them at once. These blocks stay in every later window beyond
 * the budget (the top-k of later steps runs over the blocks before them),
 * using the reserve_blocks slots. An append that finds no free window or pool
 * slot fails with KVMRET_ERR_STATE ("no free GPU slot for block N") and
 * changes nothing. An append may touch at most 64 blocks in this mode.
 * kvmret_gen_end: the decode blocks become ordinary blocks for the next
 * selection; reports KVMRET_ERR_STATE if a bound block was ever missing from
 * the window when its tokens were written. */
int kvmret_gen_begin(kvmret_ctx *ctx);
int kvmret_gen_end(kvmret_ctx *ctx);
/* First decode block of gen mode (0xffffffff when gen mode is off). */
uint32_t kvmret_gen_first_block(kvmret_ctx *ctx);
/* Cache cell of each token position [pos0, pos0 + n_tok): window slot of its
 * block * block_tokens + offset in the block, -1 when the block is not in the
 * window (kvmem_fill_slot_info, src/adapter/llama-kvmem-batch.cpp:5-58).
 * Waits for the context stream. */
int kvmret_cells(kvmret_ctx *ctx, uint32_t pos0, uint32_t n_tok, int32_t *cells_out);
/* Summaries in the order the reference's mean_k returns them:
 * out [n_blocks][n_layer][n_head_kv * d_head] f32 (host). */
int kvmret_get_summaries(kvmret_ctx *ctx, float *out_host);

/* ---- query accumulation (S1): q_sum_ / q_count_ of the adapter,
 *      src/adapter/llama-memory-kvmem.cpp:3417-3432, reset :3300-3315,
 *      llama_kvmem_get_query / set_query (src/adapter/llama-kvmem-hooks.h:247-248). ---- */
int kvmret_query_reset(kvmret_ctx *ctx);
/* q_dev: [n_layer][n_rows][n_head * d_head], f16 or f32. */
int kvmret_query_add_f16(kvmret_ctx *ctx, const uint16_t *q_dev, uint32_t n_rows);
int kvmret_query_add_f32(kvmret_ctx *ctx, const float *q_dev, uint32_t n_rows);
/* Host copies of the accumulator: q_sum [n_layer][n_head * d_head], q_count [n_layer]. */
int kvmret_query_set(kvmret_ctx *ctx, const float *q_sum_host, const uint32_t *q_count_host);
int kvmret_query_get(kvmret_ctx *ctx, float *q_sum_host, uint32_t *q_count_host);

/* ---- scoring (S3): llama_memory_kvmem::score_retrieval,
 *      src/adapter/llama-memory-kvmem.cpp:4149-4196 ---- */
/* Score every block; if scores_host != NULL copy the n_blocks f64 scores out. */
int kvmret_score(kvmret_ctx *ctx, double *scores_host);
/* Layer-sharded form: the per-(layer, block) terms layer_sum / n_head_kv (f64)
 * of this context's layers, without the reduction, as exchange rows of
 * kvmret_contrib_stride(ctx) doubles: row l holds the terms of blocks
 * [0, n_blocks) and, in its LAST column, 1.0 if layer l has query rows else
 * 0.0 — so one all-gather of [n_layer][stride] per shard carries everything.
 * contrib_out_dev == NULL writes the context's own buffer (kvmret_contrib_dev). */
int kvmret_score_layers(kvmret_ctx *ctx, double *contrib_out_dev);
const double *kvmret_contrib_dev(kvmret_ctx *ctx);
uint32_t kvmret_contrib_stride(kvmret_ctx *ctx);
/* Reduce the gathered rows of ALL layers of the model, in layer order
 * (contrib_all_dev [n_layer_all][stride], shards concatenated by layer). */
int kvmret_score_reduce(kvmret_ctx *ctx, const double *contrib_all_dev, uint32_t n_layer_all);

/* ---- selection (S5/S6): llama_memory_kvmem::preview_retrieval
 *      (src/adapter/llama-memory-kvmem.cpp:4327-4347) -> KvMemRuntime::
 *      preview_reselect -> KvMemStore::pick_topk_blocks
 *      (kvmem/src/host/kvmem_store.cpp:357-359, 482-623) ---- */
/* Top-k over the current scores (after kvmret_score or kvmret_score_reduce).
 * mandatory: block ids that consume budget, kept newest-first (retrieval_mandatory,
 * src/adapter/llama-memory-kvmem.cpp:4306-4325). ids_out (capacity
 * budget_blocks) receives the selection ascending; *n_out its length. */
int kvmret_select(kvmret_ctx *ctx, const uint32_t *mandatory, uint32_t n_mandatory,
                  uint32_t *ids_out, uint32_t *n_out);
/* kvmret_score + kvmret_select. */
int kvmret_preview(kvmret_ctx *ctx, const uint32_t *mandatory, uint32_t n_mandatory,
                   uint32_t *ids_out, uint32_t *n_out);

/* ---- apply (S7-S13): llama_memory_kvmem::apply_selection
 *      (src/adapter/llama-memory-kvmem.cpp:4424-4543): KvMemStore::set_selection
 *      (kvmem/src/host/kvmem_store.cpp:758-882), layout_gpu_slots_by_orig_pos
 *      (src/adapter/llama-memory-kvmem.cpp:1958-2289), write_block_to_gpu
 *      (:4000-4071) and kvmem_stagein_flush (src/adapter/llama-kvmem-stagein.cu:
 *      669-790). Enqueued on the context stream; the window is valid once the
 *      stream reaches this point. ---- */
int kvmret_apply_selection(kvmret_ctx *ctx, const uint32_t *ids, uint32_t n_ids,
                           kvmret_step_stats *stats);
/* Asynchronous step: top-k over the current scores (after kvmret_score or
 * kvmret_score_reduce), device plan and window assembly, all enqueued on the
 * context stream with no host synchronisation; fresh blocks are read from the
 * mapped pinned repository by the assembly itself. Up to 4 steps may be in
 * flight; kvmret_step_collect returns the oldest one's selection and stats
 * (waiting for its readback) and replays it in the host block table. */
int kvmret_select_apply_async(kvmret_ctx *ctx, const uint32_t *mandatory, uint32_t n_mandatory);
int kvmret_step_collect(kvmret_ctx *ctx, uint32_t *ids_out, uint32_t *n_out,
                        kvmret_step_stats *stats);
/* KvMemStore::clear_working_set (kvmem/include/kvmem/kvmem_store.hpp:470-472,
 * kvmem/src/host/kvmem_store.cpp:897-901): the working set becomes empty (a
 * new session over the same history); blocks, summaries and the repository
 * stay, and blocks still in the HBM pool are rebuilt from it by the next
 * step. drop_pool != 0 also forgets the pool's contents and LRU history, so
 * the next step stages its whole selection from the host repository, as
 * right after kvmret_create. Collects any step still in flight first. */
int kvmret_clear_working_set(kvmret_ctx *ctx, int drop_pool);
/* Residency policy of the HBM block pool for later steps (the config's
 * pool_cache): 1 keeps blocks that left the window in idle pool slots as a
 * cache (least recently used evicted first), 0 frees a block's slot as soon
 * as the block leaves the window, so only the working set stays on the GPU —
 * the reference's residency (KvMemRuntime::spill_outgoing,
 * kvmem/src/host/kvmem_runtime.cpp:225-249). Collects any step in flight. */
int kvmret_set_pool_cache(kvmret_ctx *ctx, int on);
/* HBM-resident history: copies the stored blocks of [first_block,
 * first_block + n_blocks) that hold no pool slot into free pool slots (lowest
 * free slot first, no eviction; stops when the pool is full), so that later
 * steps move them from HBM instead of reading the host repository. The
 * placed blocks count as least recently used. Needs pool caching on
 * (KVMRET_ERR_STATE otherwise); size the pool with kvmret_config.pool_blocks.
 * Drains the context; the copies are done on return. No reference
 * counterpart: a residency choice of this library (the reference keeps only
 * the window on the GPU). */
int kvmret_pool_prefetch(kvmret_ctx *ctx, uint32_t first_block, uint32_t n_blocks,
                         uint32_t *n_placed);
/* llama_kvmem_apply_retrieval (src/adapter/llama-memory-kvmem.cpp:4778-4782,
 * apply_retrieval :4419-4422): preview + apply. ids_out may be NULL. */
int kvmret_apply_retrieval(kvmret_ctx *ctx, const uint32_t *mandatory, uint32_t n_mandatory,
                           uint32_t *ids_out, uint32_t *n_out, kvmret_step_stats *stats);

/* The last plan's remap rows, 7 int32 each: block_id, n_tokens, from_base,
 * to_base, working_k_resident, skip, raw_refresh (KvMemRemap,
 * kvmem/include/kvmem/kvmem_store.hpp:75-95). Capacity budget_blocks rows. */
int kvmret_last_plan(kvmret_ctx *ctx, int32_t *remaps_out, uint32_t *n_remaps,
                     uint32_t *stage_in_out, uint32_t *n_stage_in,
                     uint32_t *stage_out_out, uint32_t *n_stage_out);

/* ---- window (where attention reads; the llama_kv_cache K/V layer tensors) ---- */
/* Device base of layer `layer`'s K / V window: rows of kvmret_row_bytes(type,
 * n_head_kv * d_head), cell = window_slot * block_tokens + token. */
void *kvmret_window_k(kvmret_ctx *ctx, uint32_t layer);
void *kvmret_window_v(kvmret_ctx *ctx, uint32_t layer);
uint32_t kvmret_window_slots(kvmret_ctx *ctx);
/* Current window: block id and RoPE base of each occupied slot (host). */
int kvmret_window_layout(kvmret_ctx *ctx, uint32_t *ids_out, int32_t *bases_out, uint32_t *n_out);
/* Copy window slots [slot0, slot0 + n_slots) of one layer's K (is_v = 0) or V
 * to host memory after the context stream drains (read_gpu_block,
 * src/adapter/llama-memory-kvmem.cpp:4600-4650). */
int kvmret_window_read(kvmret_ctx *ctx, uint32_t layer, int is_v, uint32_t slot0,
                       uint32_t n_slots, void *out_host);

/* ---- per-step timing: the KVMEM_PERF retrieval buckets
 *      (src/adapter/llama-memory-kvmem.cpp:4198-4216, struct
 *      src/adapter/llama-memory-kvmem.h:357-382), measured with CUDA events on
 *      the stream each kernel or copy runs on. ---- */
typedef struct kvmret_prof {
    uint64_t launches;        /* kernels launched by the context since reset */
    uint32_t n_score, n_asm;  /* timed scoring / assembly launches */
    uint32_t dropped;         /* regions not timed (event pool exhausted) */
    double score_ms;          /* scoring kernel */
    double asm_ms;            /* window assembly (moved and fresh slots in one launch) */
    uint64_t score_bytes;     /* summary bytes the scoring read */
    uint64_t asm_hbm_bytes;   /* HBM bytes the assemblies read + wrote (collected steps) */
    uint64_t asm_link_bytes;  /* host-link bytes fresh slots read (collected steps) */
    uint32_t n_gemm, pad_;    /* timed prefill-scorer GEMM launches */
    double gemm_ms;           /* prefill-scorer tensor-core GEMM */
    double gemm_flops;        /* its algorithmic FLOPs (2 * tokens * blocks * K) */
} kvmret_prof;
/* Reset the counters and turn event timing on (1) or off (0). */
int kvmret_prof_enable(kvmret_ctx *ctx, int on);
/* Drain the streams, resolve the recorded events and return the totals. */
int kvmret_prof_read(kvmret_ctx *ctx, kvmret_prof *out);

/* ---- stateless kernels on caller buffers (the kvmem_stagein_* / kvmem_d2d /
 *      kvmem_meank surface, src/adapter/llama-kvmem-stagein.h:1-67). `stream`
 *      is a cudaStream_t (NULL = legacy default stream). ---- */
/* RoPE f16 K rows [n_tok][n_head_kv][d_head] at positions pos0 + t
 * (kvmem_stagein_rope_neox, src/adapter/llama-kvmem-stagein.cu:534-569). */
int kvmret_rope_f16(const uint16_t *k_dev, uint16_t *out_dev, uint32_t n_tok, uint32_t n_head_kv,
                    uint32_t d_head, uint32_t n_rot, int32_t pos0, float freq_base,
                    float freq_scale, void *stream);
/* q8_0 K rows: dequant -> RoPE at pos0 -> FWHT(fwht_n, 0 = off) -> q8_0
 * (kvmem_stagein_enqueue_k + flush, src/adapter/llama-kvmem-stagein.cu:813-855, 746-785). */
int kvmret_rope_q8_0(const void *k_dev, void *out_dev, uint32_t n_tok, uint32_t n_head_kv,
                     uint32_t d_head, uint32_t n_rot, int32_t pos0, float freq_base,
                     float freq_scale, uint32_t fwht_n, void *stream);
/* The same for q4_0 K rows (dequant_q4_0 / quant_q4_0,
 * src/adapter/llama-kvmem-stagein.cu:145-158, 201-234). */
int kvmret_rope_q4_0(const void *k_dev, void *out_dev, uint32_t n_tok, uint32_t n_head_kv,
                     uint32_t d_head, uint32_t n_rot, int32_t pos0, float freq_base,
                     float freq_scale, uint32_t fwht_n, void *stream);
/* Block top-k on caller buffers (KvMemStore::pick_topk_ungrouped,
 * kvmem/src/host/kvmem_store.cpp:594-616, the score fill after its keep set): sel_dev[b] = 1
 * for every kept block (kept_dev[b] != 0) and for the `need` best of the
 * others under (score desc, id: higher wins when tie_higher_id, else lower);
 * 0 elsewhere. -0.0 and +0.0 tie. One CTA, radix selection, O(n) per pass. */
int kvmret_topk_select(const double *scores_dev, const uint8_t *kept_dev, uint32_t n,
                       uint32_t need, int tie_higher_id, uint8_t *sel_dev, void *stream);
/* ---- layer-sharded exchange over NVLink peer memory (no collective
 *      library). One context per rank, each holding n_layer of
 *      the world * n_layer layers in rank order. Set-up (once): every rank
 *      calls kvmret_exchange_export, the 64-byte handles are all-gathered by
 *      the caller (any host channel), every rank calls kvmret_exchange_import.
 *      Per step, kvmret_score_exchange replaces kvmret_score_layers + the
 *      caller's all-gather + kvmret_score_reduce: the scoring kernel writes this
 *      rank's per-layer terms into its own exchange region (two halves,
 *      alternating by step) and publishes the step in every rank's flag array;
 *      the reduction waits (at most 2 s; a timeout is reported by the next
 *      collect as plan error 0x100) for every rank's step, then reads every
 *      rank's rows from its region over NVLink and reduces all layers in global
 *      order. Then kvmret_select_apply_async as usual. ---- */
int kvmret_exchange_export(kvmret_ctx *ctx, uint32_t world, void *handle_out);
int kvmret_exchange_import(kvmret_ctx *ctx, uint32_t rank, uint32_t world, const void *handles);
int kvmret_score_exchange(kvmret_ctx *ctx);

/* ---- conversation stores: several conversations time-multiplexed on one
 *      context's window and HBM pool (llama_kvmem_store_create / _switch /
 *      _rows / _bytes / _destroy, src/adapter/llama-kvmem-hooks.h:107-151;
 *      swap_conv / detach_conv / attach_conv,
 *      src/adapter/llama-memory-kvmem.cpp:1217-1714). ----
 * A store holds one conversation: its pinned host repository, block table,
 * block summaries (kept in HBM while parked), running tail sum and query
 * accumulator. kvmret_store_create makes a new empty store with the context's
 * geometry. kvmret_store_swap collects every step in flight, then exchanges
 * the context's active conversation with the one in `store` (by pointer:
 * nothing is copied; on return `store` holds the outgoing conversation),
 * empties the window and the HBM pool, and stages the incoming
 * conversation's working set back into the window from its repository.
 * *restaged (optional) = 1 when the incoming conversation has a working set
 * in the window, 0 when it has none (an empty or never-selected store). A
 * store belongs to the context's device; it may be swapped into any context
 * made with the same configuration. */
typedef struct kvmret_store kvmret_store;
int kvmret_store_create(kvmret_ctx *ctx, kvmret_store **out);
int kvmret_store_swap(kvmret_ctx *ctx, kvmret_store *store, int *restaged);
/* Tokens held by a (parked) store, and its host repository bytes. */
uint32_t kvmret_store_rows(const kvmret_store *store);
uint64_t kvmret_store_bytes(const kvmret_store *store);
void kvmret_store_destroy(kvmret_store *store);

/* ---- NVMe raw tier (NvmeKvTier, kvmem/include/kvmem/nvme_kv_tier.hpp:113-430):
 *      a file arena of fixed-size slots, each holding one block's bytes,
 *      with positional I/O (several host threads may transfer at once). ----
 * slot_count = total_bytes / slot_bytes (0 disables the tier). A block takes
 * the lowest free slot; kvmret_nvme_place with evict != 0 gives a full arena's
 * least recently used block (by write, read or touch order) up, reported in
 * *evicted. Slot-range transfers must stay inside their slot. Span batches
 * (one caller buffer) merge runs of full-slot spans whose file offsets and
 * buffer ranges are both contiguous into one system call. direct_read opens a
 * second O_DIRECT descriptor used for reads whose buffer, file offset and
 * size are 4096-byte aligned (others read buffered); drop_page_cache advises
 * the kernel to drop each transferred range; the backing file loses its
 * directory entry at once unless durable. Errors: KVMRET_ERR_ARG for bad
 * arguments, KVMRET_ERR_STATE for a failed or out-of-range transfer, a full
 * arena or a block that is not resident. */
typedef struct kvmret_nvme kvmret_nvme;
typedef struct kvmret_nvme_config {
    const char *dir;
    const char *file_name;     /* NULL: "kvmret_nvme.bin" */
    uint64_t total_bytes;
    uint64_t slot_bytes;
    int32_t durable;
    int32_t direct_read;
    int32_t drop_page_cache;
    int32_t pad_;
} kvmret_nvme_config;
typedef struct kvmret_nvme_span {
    int32_t slot;
    uint32_t pad_;
    uint64_t buffer_offset;
    uint64_t bytes;
} kvmret_nvme_span;
typedef struct kvmret_nvme_stats {
    uint64_t bytes, syscalls, direct_bytes, cache_drop_bytes, cache_drop_failures;
} kvmret_nvme_stats;
int kvmret_nvme_create(const kvmret_nvme_config *cfg, kvmret_nvme **out);
void kvmret_nvme_destroy(kvmret_nvme *t);
uint32_t kvmret_nvme_slot_count(kvmret_nvme *t);
uint32_t kvmret_nvme_free_slots(kvmret_nvme *t);
int kvmret_nvme_direct_reads(kvmret_nvme *t);
int kvmret_nvme_path(kvmret_nvme *t, char *out, uint32_t cap);
int32_t kvmret_nvme_block_slot(kvmret_nvme *t, uint32_t block);
int32_t kvmret_nvme_lru_victim(kvmret_nvme *t);
/* The block's slot (placing it: lowest free slot, else the LRU block's with
 * evict != 0), -1 when the arena is full or disabled. */
int32_t kvmret_nvme_place(kvmret_nvme *t, uint32_t block, int evict, int32_t *evicted);
int kvmret_nvme_release(kvmret_nvme *t, uint32_t block);
int kvmret_nvme_touch(kvmret_nvme *t, uint32_t block);
int kvmret_nvme_write_block(kvmret_nvme *t, uint32_t block, const void *data, uint64_t bytes);
int kvmret_nvme_read_block(kvmret_nvme *t, uint32_t block, void *data, uint64_t bytes);
int kvmret_nvme_write_range(kvmret_nvme *t, int32_t slot, uint64_t offset, const void *data,
                            uint64_t bytes);
int kvmret_nvme_read_range(kvmret_nvme *t, int32_t slot, uint64_t offset, void *data,
                           uint64_t bytes);
int kvmret_nvme_write_spans(kvmret_nvme *t, const kvmret_nvme_span *spans, uint32_t n,
                            const void *buffer, uint64_t buffer_bytes, kvmret_nvme_stats *stats);
int kvmret_nvme_read_spans(kvmret_nvme *t, const kvmret_nvme_span *spans, uint32_t n,
                           void *buffer, uint64_t buffer_bytes, kvmret_nvme_stats *stats);
/* The context's pinned repository and a tier whose slot_bytes hold at least
 * one repository block (all the context's layers, kvmret_repo_unit_bytes *
 * n_layer): kvmret_repo_spill writes the blocks' repository bytes to the tier
 * (placing them, evicting least recently used blocks of a full arena);
 * kvmret_repo_fill reads resident blocks back into the repository (O_DIRECT
 * when the tier has direct reads and the sizes are 4096-aligned), after every
 * step in flight has been collected, so later steps stage them from there —
 * the reference's NVMe -> pinned staging path
 * (kvmem/src/host/raw_kv_store.cpp load_k_nvme / load_v_gpu_nvme). */
int kvmret_repo_spill(kvmret_ctx *ctx, kvmret_nvme *t, const uint32_t *blocks, uint32_t n,
                      kvmret_nvme_stats *stats);
int kvmret_repo_fill(kvmret_ctx *ctx, kvmret_nvme *t, const uint32_t *blocks, uint32_t n,
                     kvmret_nvme_stats *stats);

/* ---- snapshot archive of a context's conversation: the reference's
 *      RawKvStore stream (RawKvStore::snapshot_write / snapshot_read,
 *      kvmem/src/host/raw_kv_store.cpp:1225-1287; framing and hash of
 *      SnapshotWriter / SnapshotReader, kvmem/include/kvmem/snapshot.hpp). ----
 * Layout (little-endian): u32 magic 0x31564b52; u32 n_layer, n_embd_k,
 * n_embd_v, block_tokens; u64 k_row_bytes (0 = f16 K), k_gpu_row_bytes (0),
 * v_gpu_row_bytes (the V row); u64 block count; per block a u64 section size
 * and per layer: u32 n_tokens, k_gpu_tokens (0), v_gpu_tokens, mean_tokens;
 * u8 k_gpu_fmt (0), v_gpu_fmt (1); then five vectors, each a u64 element count
 * and the elements: k (block_tokens unrotated K rows, zero past n_tokens), v
 * (empty), k_gpu (empty), v_gpu (block_tokens V rows, zero past n_tokens),
 * k_sum (n_embd_k f32: the token-order sum of the block's K; for quantised K,
 * whose f16 rows are not kept, a full block's summary with mean_tokens 1).
 * The hash is 64-bit FNV-1a over every byte. kvmret_snapshot_write with
 * buf == NULL reports the size only; it collects steps in flight first.
 * kvmret_snapshot_read fills an empty context (no tokens) made with the same
 * geometry: repository, summaries, running tail sum and block table; its
 * working set starts empty. A mismatched or malformed archive is rejected
 * with KVMRET_ERR_ARG and leaves the context empty. */
int kvmret_snapshot_write(kvmret_ctx *ctx, void *buf, uint64_t cap, uint64_t *len,
                          uint64_t *hash);
int kvmret_snapshot_read(kvmret_ctx *ctx, const void *buf, uint64_t len, uint64_t *hash);

/* ---- session lanes (config 5: several conversations per GPU, stepped
 *      together; the reference keeps one KvMemStore per lane,
 *      src/adapter/llama-memory-kvmem.cpp:1624-1714) ----
 * A group of contexts on one device (same layer count and block capacity).
 * Each lane's kernels run on the lane's own stream, forked from and joined to
 * `stream`, so the lanes overlap on the GPU. The lanes' score terms share one
 * exchange buffer, lane-major: rows_out [n_lanes][n_layer][kvmret_contrib_stride]. */
typedef struct kvmret_lanes kvmret_lanes;
int kvmret_lanes_create(kvmret_ctx *const *lanes, uint32_t n_lanes, kvmret_lanes **out);
void kvmret_lanes_destroy(kvmret_lanes *g);
/* Per-layer score terms of every lane's accumulated query (kvmret_score_layers per lane). */
int kvmret_lanes_score_layers(kvmret_lanes *g, double *rows_out, void *stream);
/* rows_all: [n_ranks][n_lanes][n_layer][stride], the all-gather of every rank's
 * rows_out in layer order (n_ranks = 1: rows_out itself). Per lane: reduce over
 * all n_ranks * n_layer layers, top-k (mandatory[i], n_mandatory[i]; both may be
 * null), plan and window assembly, enqueued without host synchronisation;
 * collect each lane with kvmret_step_collect. */
int kvmret_lanes_select_apply_async(kvmret_lanes *g, const double *rows_all, uint32_t n_ranks,
                                    const uint32_t *const *mandatory,
                                    const uint32_t *n_mandatory, void *stream);

/* ---- prefill scoring (an extension: the reference scores the MEAN query of a
 *      span, src/adapter/llama-memory-kvmem.cpp:4149-4196; here every token of
 *      a prefill chunk is scored) ----
 * q_dev: [n_layer][n_tok][n_head * d_head] f16 pre-RoPE queries of the chunk.
 * score(t, b) = mean over layers l and KV heads g of the cosine between the
 * token's group query sum_{h in g} q[l][t][h] and block b's summary, computed
 * from unit-length f16 operands on the tensor cores with f32 accumulation.
 * sel_dev[max_blocks] receives 1 for every block in some token's top_k (by
 * score, ties by the config's tie rule), else 0. scores_dev (optional):
 * [n_tok][n_blocks] f32. n_sel_out (optional, host): number of selected blocks;
 * passing it makes the call synchronous and reports a GEMM pipeline timeout. */
int kvmret_prefill_score(kvmret_ctx *ctx, const uint16_t *q_dev, uint32_t n_tok, uint32_t top_k,
                         uint8_t *sel_dev, float *scores_dev, uint32_t *n_sel_out);
/* C = alpha * A * B^T on the tensor cores: A [m][k], B [n][k] f16 row-major,
 * C [m][n] f32; m % 128 == 0, n % 16 == 0, k % 64 == 0, 16-byte aligned
 * operands. C is computed in 128 x 256 tiles (the last tile of a row may be
 * partial). err_dev (optional device word) is set to 1 if the kernel's
 * pipeline gave up waiting. The prefill scorer's contraction. */
int kvmret_gemm_f16_nt(const uint16_t *a_dev, const uint16_t *b_dev, float *c_dev, uint32_t m,
                       uint32_t n, uint32_t k, float alpha, uint32_t *err_dev, void *stream);
/* The same with a caller workspace of kvmret_gemm_ws_bytes(m, n, k) bytes
 * (0: none needed, ws_dev may be NULL). When the tiles would leave enough SMs
 * idle for it to pay, the grid is one CTA per SM: a CTA per tile runs the
 * first k-steps of its tile in lockstep with the others (the k-slices of A
 * and B shared in L2), the remaining CTAs split the k tails of all tiles, and
 * a second launch adds the pieces in a fixed order, so results repeat run to
 * run. */
size_t kvmret_gemm_ws_bytes(uint32_t m, uint32_t n, uint32_t k);
int kvmret_gemm_f16_nt_ws(const uint16_t *a_dev, const uint16_t *b_dev, float *c_dev, uint32_t m,
                          uint32_t n, uint32_t k, float alpha, uint32_t *err_dev, float *ws_dev,
                          size_t ws_bytes, void *stream);
/* f16 values -> q8_0 / q4_0 blocks (n_elems a multiple of 32): the quantisers
 * of kvmem_stagein_quantize (src/adapter/llama-kvmem-stagein.cu:181-234,
 * 616-642), used to build quantised cache rows and repository bytes. */
int kvmret_quantize_f16(const uint16_t *src_dev, void *dst_dev, int32_t type, uint64_t n_elems,
                        void *stream);
/* Batched byte copies on the context stream, at most 8192 per call
 * (kvmem_d2d_batched, src/adapter/llama-kvmem-stagein.cu:1002-1035, which uses
 * its execution state's preallocated op buffer the same way). */
int kvmret_d2d_batched(kvmret_ctx *ctx, const void *const *src, void *const *dst,
                       const uint64_t *nbytes, int n);

/* ---- allocation-free scoring. No counterpart in the reference: this entry
 *      point exists for callers that cannot allocate device memory (code that
 *      runs inside an allocator hook, under a memory manager that owns the whole
 *      device, or on a serving path where cudaMalloc is forbidden). ----
 *
 * Same scores as kvmret_score, from caller-owned inputs and output:
 *   summ_dev      [n_layer][n_head_kv][d_head][summ_stride] f32 block summaries
 *                 (the context's own layout), 16-byte aligned, summ_stride a
 *                 multiple of 64 and >= n_blocks
 *   q_sum_dev     [n_layer][n_head * d_head] f32 query sums
 *   q_count_dev   [n_layer] u32 query row counts
 *   has_block_dev [n_blocks] u8, nonzero where the block holds data
 *   scores_dev    [n_blocks] f64 output
 * It calls no allocator. Its scratch is one file-scope device array of
 * KVMRET_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until
 * exit; a call needing more (n_layer * summ_stride * 8 bytes plus the query
 * scratch) is rejected with KVMRET_ERR_ARG. The first call on each device,
 * with that device current, looks up the array's device address: make it
 * before any stream capture. The address is cached per CUDA context; after a
 * cudaDeviceReset the next call looks it up again (again, not while a capture
 * is under way). Calls share the array (each call writes every
 * scratch byte it reads, so nothing needs clearing); calls that overlap on the
 * GPU race. `stream` is a cudaStream_t (NULL = legacy default stream). */
#define KVMRET_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
int kvmret_score_noalloc(const float *summ_dev, uint32_t summ_stride, const float *q_sum_dev,
                         const uint32_t *q_count_dev, const uint8_t *has_block_dev,
                         uint32_t n_blocks, uint32_t n_layer, uint32_t n_head,
                         uint32_t n_head_kv, uint32_t d_head, double *scores_dev, void *stream);

/* ---- host block table: the selection / plan logic alone, no GPU needed
 *      (KvMemStore, kvmem/include/kvmem/kvmem_store.hpp:329-491). ---- */
int kvmret_table_create(const kvmret_config *cfg, kvmret_table **out);
void kvmret_table_destroy(kvmret_table *t);
int kvmret_table_append(kvmret_table *t, uint32_t n_tokens);
uint32_t kvmret_table_n_blocks(kvmret_table *t);
/* The always-kept part of a selection: sink, mandatory newest-first, recent
 * (kvmem/src/host/kvmem_store.cpp:497-534). kept_out [n_blocks] u8; returns
 * via *need the number of blocks still to fill by score (0 when all fit). */
int kvmret_table_keep(kvmret_table *t, const uint32_t *mandatory, uint32_t n_mandatory,
                      uint8_t *kept_out, uint32_t *kept_count, uint32_t *need);
/* set_selection + the runtime's spill/admit tier effect. remaps_out rows as
 * kvmret_last_plan; counts_out[6]: n_stage_in, n_stage_out, n_remaps,
 * total_window_tokens, selection_overlap_blocks, gpu_reused_blocks. */
/* KvMemStore::clear_working_set (kvmem/src/host/kvmem_store.cpp:897-901);
 * drop_gpu != 0 also takes every block out of the GPU tier. */
int kvmret_table_clear_working_set(kvmret_table *t, int drop_gpu);
/* KvMemStore::truncate_to (kvmem/src/host/kvmem_store.cpp:207-227). */
int kvmret_table_truncate(kvmret_table *t, uint32_t n_tokens);
/* set_block_tier(id, KvTier::GPU) (kvmem/src/host/kvmem_store.cpp:250-277):
 * the tier change of a decode block given a reserve slot. */
int kvmret_table_set_on_gpu(kvmret_table *t, uint32_t block_id);
int kvmret_table_set_selection(kvmret_table *t, const uint32_t *ids, uint32_t n_ids,
                               int force_raw_refresh, uint32_t *stage_in_out,
                               uint32_t *stage_out_out, int32_t *remaps_out,
                               uint32_t *counts_out);

#ifdef __cplusplus
}
#endif
#endif /* KVMRET_H */
