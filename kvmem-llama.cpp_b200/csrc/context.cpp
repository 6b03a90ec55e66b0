// Retrieval context: device state of one shard (layers) of one session and
// the host orchestration of a retrieval step. Implements the C ABI of
// include/kvmret.h; no C++ exception leaves this file.
//
// A step runs entirely on the device once it is enqueued: query accumulation,
// scoring, the exact top-k, the device plan (window diff, HBM pool slots, job
// lists) and the window assembly, which reads fresh blocks straight from the
// mapped pinned repository. The selected ids and the plan counts come back
// through a pinned readback ring; the host block table replays each selection
// when it is collected, which keeps the reference's plan metadata (stage-in /
// stage-out lists, remap rows) without the host ever sitting between the
// selection and the assembly.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <new>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "kvmret.h"
#include "prefill.cuh"
#include "table.hpp"

using kvmret::Job;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                              \
    do {                                                                                      \
        const cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                                \
            return fail(KVMRET_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_));            \
    } while (0)

#define TRY(x)                                                                                \
    do {                                                                                      \
        const int r_ = (x);                                                                   \
        if (r_ != KVMRET_OK) return r_;                                                       \
    } while (0)

// Makes a context's device current for the length of an entry point and gives
// the caller back its own current device on return.
class DeviceScope {
public:
    DeviceScope() = default;
    DeviceScope(const DeviceScope &) = delete;
    DeviceScope &operator=(const DeviceScope &) = delete;
    cudaError_t enter(int dev) {
        if (dev < 0) return cudaSuccess;
        int cur = 0;
        cudaError_t e = cudaGetDevice(&cur);
        if (e != cudaSuccess || cur == dev) return e;
        e = cudaSetDevice(dev);
        if (e == cudaSuccess) prev_ = cur;
        return e;
    }
    ~DeviceScope() {
        if (prev_ >= 0) cudaSetDevice(prev_);
    }

private:
    int prev_ = -1;
};

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

bool type_ok(int32_t t) {
    return t == KVMRET_TYPE_F16 || t == KVMRET_TYPE_Q8_0 || t == KVMRET_TYPE_Q4_0;
}

// Host theta exactly as rope_neox_apply computes it (kvmem/src/host/rope.cpp:20-24).
kvmret::Theta make_theta(uint32_t n_rot, float base, float scale) {
    kvmret::Theta t{};
    for (uint32_t i = 0; i < n_rot / 2 && i < 128; ++i) {
        t.v[i] = std::pow(base, -2.0f * static_cast<float>(i) / static_cast<float>(n_rot));
        t.v[i] *= scale;
    }
    return t;
}

// FWHT size applied to quantised K (kvmem_hadamard_nrot_k,
// src/adapter/llama-kvmem-quant.h:238-244).
uint32_t hadamard_nrot_k(uint32_t d_head) {
    uint32_t nrot = 64;
    do {
        nrot *= 2;
    } while (d_head % nrot == 0);
    return nrot / 2;
}

constexpr int kRing = 4;          // readback slots (steps in flight before a collect)
constexpr size_t kEventPool = 8192;
enum { PR_SCORE = 0, PR_ASM, PR_GEMM };
enum { OP_APPEND = 0, OP_TRUNCATE, OP_ON_GPU };  // deferred block-table operations

}  // namespace

namespace kvmret {
int set_error(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace kvmret

struct kvmret_ctx {
    kvmret_config cfg{};
    // geometry
    uint32_t E = 0, qdim = 0, ncap = 0, win_slots = 0, pool_slots = 0;
    uint32_t cstride = 0;  // exchange row: ncap score terms, padding, query flag last
    uint64_t k_row = 0, v_row = 0, unit_k = 0, unit = 0, slot_bytes = 0;
    uint64_t win_k_layer = 0, win_v_layer = 0;
    kvmret::AssembleGeom geom{};
    kvmret::Theta theta{};
    // device: scoring
    float *summ = nullptr, *tail_sum = nullptr, *q_sum = nullptr, *qv = nullptr, *nq = nullptr;
    uint32_t *q_count_dev = nullptr;
    uint8_t *has_block = nullptr, *active = nullptr, *kept_dev = nullptr, *sel_dev = nullptr;
    double *contrib = nullptr, *scores = nullptr;
    // device: window, pool and plan state
    uint8_t *pool = nullptr, *win_k = nullptr, *win_v = nullptr;
    // cos/sin of every window position, [pos][n_rot/4] x {c_2j, c_2j+1, s_2j, s_2j+1}
    float4 *rope_tab = nullptr;
    int32_t *d_win_id = nullptr, *d_win_base = nullptr, *d_blk_slot = nullptr,
            *d_slot_blk = nullptr;
    uint32_t *d_win_ntok = nullptr, *d_blk_ntok = nullptr, *d_slot_ntok = nullptr,
             *d_slot_used = nullptr, *d_counts = nullptr, *d_ids = nullptr;
    Job *jobs_dev = nullptr;
    kvmret::CopyOp *ops_dev = nullptr;
    // device: prefill scorer (allocated on first use). pf_a: unit group
    // queries [pf_rows][K] f16; pf_b: unit summaries [pf_nrows][K] f16, rows
    // below mhat_valid current; pf_s: scores [pf_rows][pf_nrows] f32.
    uint16_t *pf_a = nullptr, *pf_b = nullptr;
    float *pf_s = nullptr, *pf_ws = nullptr;  // pf_ws: the GEMM's split partials
    size_t pf_ws_bytes = 0;
    uint32_t *pf_err = nullptr;
    uint32_t pf_rows = 0, pf_nrows = 0, mhat_valid = 0;
    // layer-sharded exchange over peer memory (kvmret_exchange_*): one region
    // per rank = 2 halves (step parity) of this rank's [n_layer][cstride]
    // rows, then flags [kMaxRanks], counter, err; peer regions opened via
    // CUDA IPC and read by the reduction
    uint8_t *ex_region = nullptr;
    uint8_t *ex_peer[kvmret::kMaxRanks] = {};
    uint32_t ex_world = 0, ex_rank = 0, ex_step = 0;
    uint64_t ex_half = 0;  // doubles per half
    uint64_t ex_tail = 0;  // byte offset of the flags
    // host
    uint8_t *repo_host = nullptr, *repo_dev = nullptr;
    uint8_t *pin_flags = nullptr;  // kept / selection flags staging
    uint32_t *pin_rb = nullptr;    // readback ring: kRing x (8 counts + win_slots ids)
    cudaEvent_t ev_rb[kRing] = {};
    int rb_head = 0, rb_pending = 0;
    uint32_t step = 0;
    std::vector<uint32_t> q_count;  // host mirror of q_count_dev
    bool q_dirty = true;            // qv / nq / active must be recomputed
    bool q_reset_pending = true;    // q_sum / q_count_dev hold a stale query
    std::vector<uint8_t> kept_cached;  // last kept flags uploaded
    bool kept_valid = false;
    kvmret::BlockTable table;
    // Tokens appended so far, in call (= stream) order; launches size their
    // block loops from it. The block table above lags: it replays each step's
    // selection when the step is collected, so appends, truncations and tier
    // changes made while steps are in flight reach it after the steps that
    // were enqueued before them (deferred table operations).
    uint32_t live_tokens = 0;
    struct TableOp {
        uint32_t after_step;
        int kind;
        uint32_t arg;
    };
    std::deque<TableOp> deferred;
    uint32_t rb_step[kRing] = {};  // step number of each readback slot
    // gen-reserve placement (kvmret_gen_begin / kvmret_gen_end): blocks from
    // gen_first on receive their decode tokens in the window and stay in every
    // window beyond the budget; gen_bound marks those holding a window slot
    bool gen_on = false;
    uint32_t gen_first = 0;
    std::vector<uint8_t> gen_bound;
    uint32_t *d_gen_err = nullptr;
    kvmret::Plan last_plan;
    kvmret_step_stats last_stats{};
    cudaStream_t st = nullptr;
    // timing (kvmret_prof_*): event pool and pending (begin, end, kind)
    struct Region {
        cudaEvent_t a, b;
        int kind;
    };
    bool prof_on = false;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_next = 0;
    std::vector<Region> pending;
    kvmret_prof prof{};

    explicit kvmret_ctx(const kvmret::TableConfig &tc) : table(tc) {}
    uint32_t *rb(int slot) { return pin_rb + static_cast<size_t>(slot) * (8 + win_slots); }
    uint32_t live_blocks() const {
        return (live_tokens + cfg.block_tokens - 1) / cfg.block_tokens;
    }
};

struct kvmret_table {
    kvmret::BlockTable t;
    explicit kvmret_table(const kvmret::TableConfig &c) : t(c) {}
};

namespace {

kvmret::TableConfig table_config(const kvmret_config &c) {
    kvmret::TableConfig tc;
    tc.block_tokens = c.block_tokens;
    tc.budget_blocks = c.budget_blocks;
    tc.sink_blocks = c.sink_blocks;
    tc.recent_blocks = c.recent_blocks;
    tc.immutable_source_k = c.immutable_source_k != 0;
    return tc;
}

int validate(const kvmret_config &c) {
    if (c.n_layer == 0 || c.n_head == 0 || c.n_head_kv == 0 || c.n_head % c.n_head_kv)
        return fail(KVMRET_ERR_ARG, "bad head geometry (n_layer %u, n_head %u, n_head_kv %u)",
                    c.n_layer, c.n_head, c.n_head_kv);
    if (c.d_head != 64 && c.d_head != 128 && c.d_head != 256)
        return fail(KVMRET_ERR_ARG, "d_head %u not in {64, 128, 256}", c.d_head);
    if (c.n_rot != c.d_head)
        return fail(KVMRET_ERR_ARG, "n_rot %u must equal d_head %u (full NeoX rotary)", c.n_rot,
                    c.d_head);
    if (c.block_tokens == 0 || static_cast<uint64_t>(c.block_tokens) * c.d_head > 32768)
        return fail(KVMRET_ERR_ARG, "block_tokens %u too large for d_head %u", c.block_tokens,
                    c.d_head);
    if (c.max_blocks == 0 || c.budget_blocks == 0)
        return fail(KVMRET_ERR_ARG, "max_blocks and budget_blocks must be > 0");
    if (c.k_type != KVMRET_TYPE_F16 && c.k_type != KVMRET_TYPE_Q8_0 &&
        c.k_type != KVMRET_TYPE_Q4_0)
        return fail(KVMRET_ERR_ARG, "k_type %d unsupported (f16, q8_0 or q4_0)", c.k_type);
    if (!type_ok(c.v_type)) return fail(KVMRET_ERR_ARG, "v_type %d unsupported", c.v_type);
    const uint64_t kr = kvmret_row_bytes(c.k_type, c.n_head_kv * c.d_head);
    const uint64_t vr = kvmret_row_bytes(c.v_type, c.n_head_kv * c.d_head);
    if (kr % 16 || vr % 16)
        return fail(KVMRET_ERR_ARG, "row bytes %llu / %llu not multiples of 16",
                    (unsigned long long)kr, (unsigned long long)vr);
    const uint32_t win = c.budget_blocks + c.reserve_blocks;
    const uint32_t pool = c.pool_blocks ? c.pool_blocks : win;
    if (pool < c.budget_blocks)
        return fail(KVMRET_ERR_ARG, "pool_blocks %u < budget_blocks %u", pool, c.budget_blocks);
    if (win > 4096 || pool > 8192)
        return fail(KVMRET_ERR_ARG, "window of %u slots / pool of %u slots exceeds 4096 / 8192",
                    win, pool);
    if (c.freq_base <= 0.0f) return fail(KVMRET_ERR_ARG, "freq_base must be > 0");
    return KVMRET_OK;
}

// Begin a timed region on stream `s`; returns the region index or -1.
int prof_begin(kvmret_ctx *c, cudaStream_t s, int kind) {
    if (!c->prof_on) return -1;
    if (c->ev_next + 2 > c->ev_pool.size()) {
        ++c->prof.dropped;
        return -1;
    }
    kvmret_ctx::Region r{c->ev_pool[c->ev_next], c->ev_pool[c->ev_next + 1], kind};
    c->ev_next += 2;
    if (cudaEventRecord(r.a, s) != cudaSuccess) return -1;
    c->pending.push_back(r);
    return static_cast<int>(c->pending.size() - 1);
}

void prof_end(kvmret_ctx *c, cudaStream_t s, int idx) {
    if (idx >= 0) cudaEventRecord(c->pending[idx].b, s);
}

void free_all(kvmret_ctx *c) {
    DeviceScope ds;
    ds.enter(c->cfg.device);
    if (c->st) cudaStreamSynchronize(c->st);
    for (uint32_t p = 0; p < kvmret::kMaxRanks; ++p)
        if (c->ex_peer[p] && c->ex_peer[p] != c->ex_region) cudaIpcCloseMemHandle(c->ex_peer[p]);
    if (c->ex_region) cudaFree(c->ex_region);
    void *dev[] = {c->summ, c->tail_sum, c->q_sum, c->qv, c->nq, c->q_count_dev, c->has_block,
                   c->active, c->kept_dev, c->sel_dev, c->contrib, c->scores, c->pool,
                   c->win_k, c->win_v, c->jobs_dev, c->ops_dev, c->rope_tab, c->d_win_id,
                   c->d_win_base, c->d_blk_slot, c->d_slot_blk, c->d_win_ntok, c->d_blk_ntok,
                   c->d_slot_ntok, c->d_slot_used, c->d_counts, c->d_ids, c->pf_a, c->pf_b,
                   c->pf_s, c->pf_ws, c->pf_err, c->d_gen_err};
    for (void *p : dev)
        if (p) cudaFree(p);
    if (c->repo_host) cudaFreeHost(c->repo_host);
    if (c->pin_flags) cudaFreeHost(c->pin_flags);
    if (c->pin_rb) cudaFreeHost(c->pin_rb);
    for (cudaEvent_t e : c->ev_pool) cudaEventDestroy(e);
    for (cudaEvent_t e : c->ev_rb)
        if (e) cudaEventDestroy(e);
    if (c->st) cudaStreamDestroy(c->st);
}

template <typename T>
int dmalloc(T **p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    const cudaError_t e = cudaMalloc(reinterpret_cast<void **>(p), bytes);
    if (e != cudaSuccess) {
        *p = nullptr;
        return fail(e == cudaErrorMemoryAllocation ? KVMRET_ERR_NOMEM : KVMRET_ERR_CUDA,
                    "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    return KVMRET_OK;
}

template <typename T>
int hmalloc(T **p, size_t bytes, unsigned flags) {
    const cudaError_t e = cudaHostAlloc(reinterpret_cast<void **>(p), bytes, flags);
    if (e != cudaSuccess) {
        *p = nullptr;
        return fail(KVMRET_ERR_NOMEM, "pinned host allocation of %zu bytes: %s", bytes,
                    cudaGetErrorString(e));
    }
    return KVMRET_OK;
}

// NUMA node of a GPU's PCIe attachment (-1 when unknown).
int gpu_numa_node(int device) {
    char bus[32] = {};
    if (cudaDeviceGetPCIBusId(bus, sizeof(bus), device) != cudaSuccess) return -1;
    for (char *q = bus; *q; ++q) *q = static_cast<char>(std::tolower(*q));
    char path[128];
    std::snprintf(path, sizeof(path), "/sys/bus/pci/devices/%s/numa_node", bus);
    FILE *f = std::fopen(path, "r");
    if (!f) return -1;
    int node = -1;
    if (std::fscanf(f, "%d", &node) != 1) node = -1;
    std::fclose(f);
    return node;
}

// Pinned allocation whose pages are placed on `node` (preferred policy for
// the calling thread while the driver pins them), so the GPU reads its
// repository without crossing the inter-socket link. Falls back silently to
// the default placement.
template <typename T>
int hmalloc_near(T **p, size_t bytes, unsigned flags, int node) {
    constexpr long kMpolDefault = 0, kMpolPreferred = 1;
    bool bound = false;
    if (node >= 0 && node < 64) {
        unsigned long mask = 1ul << node;
        bound = syscall(SYS_set_mempolicy, kMpolPreferred, &mask, 64ul) == 0;
    }
    const int rc = hmalloc(p, bytes, flags);
    if (bound) syscall(SYS_set_mempolicy, kMpolDefault, nullptr, 0ul);
    return rc;
}

int create_impl(const kvmret_config &cfg, kvmret_ctx *c, DeviceScope &ds) {
    c->cfg = cfg;
    const kvmret_config &k = c->cfg;
    CK(ds.enter(k.device));
    c->E = k.n_head_kv * k.d_head;
    c->qdim = k.n_head * k.d_head;
    c->ncap = static_cast<uint32_t>(align_up(k.max_blocks, 128));
    c->cstride = c->ncap + 64;
    c->k_row = kvmret_row_bytes(k.k_type, c->E);
    c->v_row = kvmret_row_bytes(k.v_type, c->E);
    c->unit_k = align_up(static_cast<uint64_t>(k.block_tokens) * c->k_row, 256);
    c->unit = c->unit_k + align_up(static_cast<uint64_t>(k.block_tokens) * c->v_row, 256);
    c->slot_bytes = c->unit * k.n_layer;
    c->win_slots = k.budget_blocks + k.reserve_blocks;
    c->pool_slots = k.pool_blocks ? k.pool_blocks : c->win_slots;
    c->win_k_layer = static_cast<uint64_t>(c->win_slots) * k.block_tokens * c->k_row;
    c->win_v_layer = static_cast<uint64_t>(c->win_slots) * k.block_tokens * c->v_row;
    c->theta = make_theta(k.n_rot, k.freq_base, k.freq_scale);
    const bool quant_k = k.k_type != KVMRET_TYPE_F16;
    const bool rot = k.attn_rot_k < 0 ? (quant_k && k.d_head % 64 == 0) : k.attn_rot_k != 0;
    const uint32_t fwht_n = (rot && quant_k) ? hadamard_nrot_k(k.d_head) : 0;
    kvmret::AssembleGeom &g = c->geom;
    g.n_layer = k.n_layer;
    g.n_head_kv = k.n_head_kv;
    g.d_head = k.d_head;
    g.block_tokens = k.block_tokens;
    g.k_row = c->k_row;
    g.v_row = c->v_row;
    g.unit_k = c->unit_k;
    g.unit = c->unit;
    g.win_k_layer = c->win_k_layer;
    g.win_v_layer = c->win_v_layer;
    g.k_type = k.k_type;
    g.fwht_n = fwht_n;
    g.fwht_scale = fwht_n ? 1.0f / std::sqrt(static_cast<float>(fwht_n)) : 0.0f;

    CK(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking));
    for (auto &e : c->ev_rb) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));

    const size_t L = k.n_layer, W = c->win_slots, P = c->pool_slots;
    TRY(dmalloc(&c->summ, L * c->E * c->ncap * sizeof(float)));
    TRY(dmalloc(&c->tail_sum, 2 * L * c->E * sizeof(float)));
    TRY(dmalloc(&c->q_sum, L * c->qdim * sizeof(float)));
    TRY(dmalloc(&c->qv, L * c->E * sizeof(float)));
    TRY(dmalloc(&c->nq, L * k.n_head_kv * sizeof(float)));
    TRY(dmalloc(&c->q_count_dev, L * sizeof(uint32_t)));
    TRY(dmalloc(&c->has_block, c->ncap));
    TRY(dmalloc(&c->active, L));
    TRY(dmalloc(&c->kept_dev, c->ncap));
    TRY(dmalloc(&c->sel_dev, c->ncap));
    TRY(dmalloc(&c->contrib, L * c->cstride * sizeof(double)));
    TRY(dmalloc(&c->scores, c->ncap * sizeof(double)));
    TRY(dmalloc(&c->pool, P * c->slot_bytes));
    TRY(dmalloc(&c->win_k, L * c->win_k_layer));
    TRY(dmalloc(&c->win_v, L * c->win_v_layer));
    TRY(dmalloc(&c->jobs_dev, 2 * W * sizeof(Job)));
    TRY(dmalloc(&c->ops_dev, 8192 * sizeof(kvmret::CopyOp)));
    const uint32_t n_pos = c->win_slots * k.block_tokens;
    TRY(dmalloc(&c->rope_tab, static_cast<size_t>(n_pos) * (k.n_rot / 4) * sizeof(float4)));
    TRY(dmalloc(&c->d_win_id, W * sizeof(int32_t)));
    TRY(dmalloc(&c->d_win_base, W * sizeof(int32_t)));
    TRY(dmalloc(&c->d_win_ntok, W * sizeof(uint32_t)));
    TRY(dmalloc(&c->d_blk_slot, c->ncap * sizeof(int32_t)));
    TRY(dmalloc(&c->d_blk_ntok, c->ncap * sizeof(uint32_t)));
    TRY(dmalloc(&c->d_slot_blk, P * sizeof(int32_t)));
    TRY(dmalloc(&c->d_slot_ntok, P * sizeof(uint32_t)));
    TRY(dmalloc(&c->d_slot_used, P * sizeof(uint32_t)));
    TRY(dmalloc(&c->d_counts, 16 * sizeof(uint32_t)));
    TRY(dmalloc(&c->d_ids, W * sizeof(uint32_t)));
    TRY(dmalloc(&c->d_gen_err, 16));
    CK(cudaMemsetAsync(c->d_gen_err, 0, 16, c->st));
    CK(cudaMemsetAsync(c->summ, 0, L * c->E * c->ncap * sizeof(float), c->st));
    CK(cudaMemsetAsync(c->tail_sum, 0, 2 * L * c->E * sizeof(float), c->st));
    CK(cudaMemsetAsync(c->q_sum, 0, L * c->qdim * sizeof(float), c->st));
    CK(cudaMemsetAsync(c->has_block, 0, c->ncap, c->st));
    CK(cudaMemsetAsync(c->contrib, 0, L * c->cstride * sizeof(double), c->st));
    CK(cudaMemsetAsync(c->scores, 0, c->ncap * sizeof(double), c->st));
    CK(cudaMemsetAsync(c->d_win_id, 0xff, W * sizeof(int32_t), c->st));  // -1: empty
    CK(cudaMemsetAsync(c->d_win_base, 0, W * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_win_ntok, 0, W * sizeof(uint32_t), c->st));
    CK(cudaMemsetAsync(c->d_blk_slot, 0xff, c->ncap * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_blk_ntok, 0, c->ncap * sizeof(uint32_t), c->st));
    CK(cudaMemsetAsync(c->d_slot_blk, 0xff, P * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_slot_ntok, 0, P * sizeof(uint32_t), c->st));
    CK(cudaMemsetAsync(c->d_slot_used, 0, P * sizeof(uint32_t), c->st));
    CK(kvmret::launch_rope_table(c->rope_tab, n_pos, k.n_rot / 2, c->theta, c->st));

    const size_t repo_bytes = static_cast<size_t>(k.max_blocks) * c->slot_bytes;
    TRY(hmalloc_near(&c->repo_host, repo_bytes, cudaHostAllocMapped | cudaHostAllocPortable,
                     gpu_numa_node(k.device)));
    CK(cudaHostGetDevicePointer(reinterpret_cast<void **>(&c->repo_dev), c->repo_host, 0));
    TRY(hmalloc(&c->pin_flags, c->ncap, cudaHostAllocDefault));
    TRY(hmalloc(&c->pin_rb, kRing * (8 + W) * sizeof(uint32_t), cudaHostAllocDefault));
    c->q_count.assign(L, 0);
    c->gen_bound.assign(c->ncap, 0);
    CK(cudaStreamSynchronize(c->st));
    return KVMRET_OK;
}

void apply_table_op(kvmret_ctx *c, int kind, uint32_t arg) {
    if (kind == OP_APPEND) c->table.append(arg);
    else if (kind == OP_TRUNCATE) c->table.truncate(arg);
    else c->table.set_on_gpu(arg);
}

// A block-table operation in stream order: applied now when no step is in
// flight, else after the newest enqueued step has been collected.
void table_op(kvmret_ctx *c, int kind, uint32_t arg) {
    if (c->rb_pending == 0) apply_table_op(c, kind, arg);
    else c->deferred.push_back({c->step, kind, arg});
}

void apply_deferred(kvmret_ctx *c, uint32_t upto_step) {
    while (!c->deferred.empty() &&
           static_cast<int32_t>(c->deferred.front().after_step - upto_step) <= 0) {
        const auto op = c->deferred.front();
        c->deferred.pop_front();
        apply_table_op(c, op.kind, op.arg);
    }
}

// Readback of the oldest uncollected step: wait for it, replay its selection
// in the host block table (the plan metadata) and fill the stats.
int collect_one(kvmret_ctx *c, uint32_t *ids_out, uint32_t *n_out) {
    const int slot = (c->rb_head - c->rb_pending + kRing) % kRing;
    CK(cudaEventSynchronize(c->ev_rb[slot]));
    const uint32_t *r = c->rb(slot);
    const uint32_t n_moved = r[0], n_fresh = r[1], n_sel = r[2], err = r[4];
    --c->rb_pending;
    if (err) {
        apply_deferred(c, c->rb_step[slot]);
        return fail(KVMRET_ERR_STATE, "device plan error 0x%x (window or pool too small)", err);
    }
    const uint32_t *ids = r + 8;
    c->last_plan = c->table.set_selection(ids, n_sel, false);
    apply_deferred(c, c->rb_step[slot]);
    kvmret_step_stats &s = c->last_stats;
    std::memset(&s, 0, sizeof(s));
    s.n_selected = n_sel;
    s.n_stage_in = static_cast<uint32_t>(c->last_plan.stage_in.size());
    s.n_stage_out = static_cast<uint32_t>(c->last_plan.stage_out.size());
    for (const auto &rm : c->last_plan.remaps) s.n_skip += rm.skip ? 1u : 0u;
    s.n_h2d_blocks = n_fresh;
    s.n_assembled = n_moved + n_fresh;
    s.n_moved = n_moved;
    s.total_window_tokens = r[3];
    const uint64_t row = c->k_row + c->v_row, L = c->cfg.n_layer;
    s.h2d_bytes = static_cast<uint64_t>(r[6]) * row * L;
    s.assemble_bytes = 2ull * (static_cast<uint64_t>(r[5]) + r[6]) * row * L;
    c->prof.asm_hbm_bytes += s.assemble_bytes;
    c->prof.asm_link_bytes += s.h2d_bytes;
    if (ids_out) std::copy(ids, ids + n_sel, ids_out);
    if (n_out) *n_out = n_sel;
    return KVMRET_OK;
}

int drain(kvmret_ctx *c) {
    while (c->rb_pending > 0) TRY(collect_one(c, nullptr, nullptr));
    return KVMRET_OK;
}

// Device plan + assembly from the selection flags in sel_dev, then an
// asynchronous readback of the ids and counts.
int plan_and_assemble(kvmret_ctx *c) {
    if (c->rb_pending == kRing) TRY(collect_one(c, nullptr, nullptr));
    ++c->step;
    kvmret::PlanArgs pa{};
    pa.sel = c->sel_dev;
    pa.blk_ntok = c->d_blk_ntok;
    pa.n_blocks = c->live_blocks();
    pa.win_slots = c->win_slots;
    pa.pool_slots = c->pool_slots;
    pa.step = c->step;
    pa.pool_cache = c->cfg.pool_cache;
    pa.win_id = c->d_win_id;
    pa.win_base = c->d_win_base;
    pa.win_ntok = c->d_win_ntok;
    pa.blk_slot = c->d_blk_slot;
    pa.slot_blk = c->d_slot_blk;
    pa.slot_ntok = c->d_slot_ntok;
    pa.slot_used = c->d_slot_used;
    pa.jobs = c->jobs_dev;
    pa.counts = c->d_counts;
    pa.ids = c->d_ids;
    pa.ext_err = c->ex_world > 1 ? reinterpret_cast<uint32_t *>(c->ex_region + c->ex_tail +
                                                               4 * (kvmret::kMaxRanks + 1))
                                 : nullptr;
    CK(kvmret::launch_plan(pa, c->st));
    kvmret::AsmLaunch al{};
    al.jobs = c->jobs_dev;
    al.counts = c->d_counts;
    al.work = c->d_counts + 7;
    al.work_moved = c->d_counts + 8;
    al.fresh_offset = c->win_slots;
    al.repo = c->repo_dev;
    al.pool_w = c->pool;
    al.pool = c->pool;
    al.slot_bytes = c->slot_bytes;
    al.win_k = c->win_k;
    al.win_v = c->win_v;
    al.gtab = c->rope_tab;
    al.theta = c->theta;
    al.g = c->geom;
    const int pr = prof_begin(c, c->st, PR_ASM);
    CK(kvmret::launch_assemble(al, 2 * c->win_slots, c->st));
    prof_end(c, c->st, pr);
    c->prof.launches += 2;
    // the plan's counts and ids go back to the host after the assembly, so the
    // two small copies do not sit between the plan and the assembly
    const int slot = c->rb_head;
    c->rb_step[slot] = c->step;
    uint32_t *r = c->rb(slot);
    CK(cudaMemcpyAsync(r, c->d_counts, 8 * sizeof(uint32_t), cudaMemcpyDeviceToHost, c->st));
    CK(cudaMemcpyAsync(r + 8, c->d_ids, c->win_slots * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                       c->st));
    CK(cudaEventRecord(c->ev_rb[slot], c->st));
    c->rb_head = (c->rb_head + 1) % kRing;
    ++c->rb_pending;
    return KVMRET_OK;
}

// Upload the kept flags of the top-k (sink, mandatory newest-first, recent)
// when they changed; returns `need` through *need.
int upload_kept(kvmret_ctx *c, const uint32_t *mandatory, uint32_t n_mand, uint32_t *need) {
    std::vector<uint8_t> kept;
    uint32_t kept_count = 0;
    const uint32_t n = c->live_blocks();
    // in gen mode the decode blocks from gen_first on are kept beyond the
    // budget; the top-k runs over the blocks before them
    const uint32_t g0 = (c->gen_on && c->gen_first < n) ? c->gen_first : n;
    *need = c->table.keep(g0, mandatory, n_mand, kept, kept_count);
    kept.resize(n, 1);
    if (!c->kept_valid || kept != c->kept_cached) {
        CK(cudaStreamSynchronize(c->st));  // the staging buffer may still feed an earlier copy
        std::copy(kept.begin(), kept.begin() + n, c->pin_flags);
        CK(cudaMemcpyAsync(c->kept_dev, c->pin_flags, n, cudaMemcpyHostToDevice, c->st));
        c->kept_cached.swap(kept);
        c->kept_valid = true;
    }
    return KVMRET_OK;
}

int select_device(kvmret_ctx *c, const uint32_t *mandatory, uint32_t n_mand) {
    uint32_t need = 0;
    TRY(upload_kept(c, mandatory, n_mand, &need));
    const uint32_t n = c->live_blocks();
    if (need > 0) {
        CK(kvmret::launch_select(c->scores, c->kept_dev, n, need, c->cfg.tie_higher_id,
                                 c->sel_dev, c->st));
        c->prof.launches += 1;
    } else if (n) {
        CK(cudaMemcpyAsync(c->sel_dev, c->kept_dev, n, cudaMemcpyDeviceToDevice, c->st));
    }
    return KVMRET_OK;
}

// Per-(layer, block) terms into rows of cstride doubles (out == nullptr: the
// context's buffer); the layer's query flag goes to the last column of its row.
// A reset is folded into the next query_add; anything that reads the query
// state before such an add clears it here instead.
int settle_query(kvmret_ctx *c) {
    if (!c->q_reset_pending) return KVMRET_OK;
    CK(cudaMemsetAsync(c->q_sum, 0, static_cast<size_t>(c->cfg.n_layer) * c->qdim * sizeof(float),
                       c->st));
    CK(cudaMemsetAsync(c->q_count_dev, 0, c->cfg.n_layer * sizeof(uint32_t), c->st));
    c->q_reset_pending = false;
    return KVMRET_OK;
}

int score_layers_impl(kvmret_ctx *c, double *out) {
    double *dst = out ? out : c->contrib;
    if (out) c->q_dirty = true;  // the flag column of a caller buffer is written by qprep
    TRY(settle_query(c));
    if (c->q_dirty) {
        CK(kvmret::launch_qprep(c->q_sum, c->q_count_dev, c->qv, c->nq, c->active,
                                c->cfg.n_layer, c->cfg.n_head, c->cfg.n_head_kv, c->cfg.d_head,
                                c->st, dst, c->cstride));
        c->prof.launches += 1;
        c->q_dirty = false;
    }
    const uint32_t n = c->live_blocks();
    const int pr = prof_begin(c, c->st, PR_SCORE);
    CK(kvmret::launch_score(c->summ, c->qv, c->nq, c->active, dst, c->cfg.n_layer,
                            c->cfg.n_head_kv, c->cfg.d_head, c->ncap, n, c->st, c->cstride));
    prof_end(c, c->st, pr);
    c->prof.score_bytes += static_cast<uint64_t>(c->cfg.n_layer) * c->E * ((n + 63) / 64 * 64) *
                           sizeof(float);
    c->prof.launches += n ? 1 : 0;
    return KVMRET_OK;
}

int reduce_impl(kvmret_ctx *c, const double *rows, uint32_t n_layer_all, const uint8_t *active) {
    CK(kvmret::launch_reduce(rows, active, n_layer_all, c->cstride, c->has_block,
                             c->live_blocks(), c->scores, c->st));
    c->prof.launches += 1;
    return KVMRET_OK;
}

#define GUARD(expr)                                                                           \
    try {                                                                                     \
        expr;                                                                                 \
    } catch (const std::bad_alloc &) {                                                        \
        return fail(KVMRET_ERR_NOMEM, "host allocation failed");                             \
    } catch (...) {                                                                           \
        return fail(KVMRET_ERR_STATE, "internal error");                                     \
    }

// First statement of an entry point on a context: the context's device is
// current until the function returns.
#define NEED_CTX(c)                                                                           \
    if (!(c)) return fail(KVMRET_ERR_ARG, "null context");                                   \
    DeviceScope dscope_;                                                                      \
    if (const cudaError_t de_ = dscope_.enter((c)->cfg.device); de_ != cudaSuccess)           \
    return fail(KVMRET_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(de_))

int preview_impl(kvmret_ctx *c, const uint32_t *mandatory, uint32_t n_mand, uint32_t *ids_out,
                 uint32_t *n_out) {
    if (!n_out) return fail(KVMRET_ERR_ARG, "n_out is NULL");
    TRY(select_device(c, mandatory, n_mand));
    const uint32_t n = c->live_blocks();
    CK(cudaMemcpyAsync(c->pin_flags, c->sel_dev, n, cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    c->kept_valid = false;  // the staging buffer now holds the selection
    uint32_t m = 0;
    for (uint32_t i = 0; i < n; ++i)
        if (c->pin_flags[i]) {
            if (ids_out) ids_out[m] = i;
            ++m;
        }
    *n_out = m;
    return KVMRET_OK;
}

int apply_impl(kvmret_ctx *c, const uint32_t *ids, uint32_t n_ids, kvmret_step_stats *stats) {
    TRY(drain(c));
    const uint32_t nb = c->live_blocks();
    std::vector<uint8_t> flags(c->ncap, 0);
    uint32_t uniq = 0;
    for (uint32_t i = 0; i < n_ids; ++i)
        if (ids[i] < nb && !flags[ids[i]]) {
            flags[ids[i]] = 1;
            ++uniq;
        }
    // in gen mode the decode blocks stay in every window
    if (c->gen_on)
        for (uint32_t b = c->gen_first; b < nb; ++b)
            if (!flags[b]) {
                flags[b] = 1;
                ++uniq;
            }
    if (uniq > c->win_slots)
        return fail(KVMRET_ERR_ARG, "selection of %u blocks exceeds %u window slots", uniq,
                    c->win_slots);
    CK(cudaStreamSynchronize(c->st));
    std::copy(flags.begin(), flags.begin() + nb, c->pin_flags);
    c->kept_valid = false;
    if (nb) CK(cudaMemcpyAsync(c->sel_dev, c->pin_flags, nb, cudaMemcpyHostToDevice, c->st));
    TRY(plan_and_assemble(c));
    TRY(collect_one(c, nullptr, nullptr));
    if (stats) *stats = c->last_stats;
    return KVMRET_OK;
}

}  // namespace

extern "C" {

void kvmret_config_default(kvmret_config *c) {
    if (!c) return;
    std::memset(c, 0, sizeof(*c));
    c->n_layer = 1;
    c->n_head = 32;
    c->n_head_kv = 8;
    c->d_head = 128;
    c->block_tokens = 128;
    c->max_blocks = 256;
    c->budget_blocks = 32;
    c->reserve_blocks = 0;
    c->sink_blocks = 1;
    c->recent_blocks = 0;
    c->pool_blocks = 0;
    c->k_type = KVMRET_TYPE_F16;
    c->v_type = KVMRET_TYPE_F16;
    c->attn_rot_k = -1;
    c->tie_higher_id = 1;
    c->pool_cache = 0;
    c->immutable_source_k = 0;
    c->n_rot = 128;
    c->freq_base = 1000000.0f;
    c->freq_scale = 1.0f;
    c->device = 0;
}

uint64_t kvmret_row_bytes(int32_t type, uint32_t n) {
    switch (type) {
    case KVMRET_TYPE_F16: return 2ull * n;
    case KVMRET_TYPE_Q8_0: return n % 32 ? 0 : (n / 32) * 34ull;
    case KVMRET_TYPE_Q4_0: return n % 32 ? 0 : (n / 32) * 18ull;
    default: return 0;
    }
}

const char *kvmret_last_error(void) { return g_err.c_str(); }
const char *kvmret_version(void) { return "kvmret 0.2 sm_100a"; }

int kvmret_create(const kvmret_config *cfg, kvmret_ctx **out) {
    if (!cfg || !out) return fail(KVMRET_ERR_ARG, "null argument");
    *out = nullptr;
    TRY(validate(*cfg));
    kvmret_ctx *c = nullptr;
    GUARD(c = new kvmret_ctx(table_config(*cfg)));
    DeviceScope ds;  // create_impl makes the context's device current
    int r = KVMRET_ERR_STATE;
    try {
        r = create_impl(*cfg, c, ds);
    } catch (...) {
        r = fail(KVMRET_ERR_NOMEM, "host allocation failed during create");
    }
    if (r != KVMRET_OK) {
        const std::string keep = g_err;
        free_all(c);
        delete c;
        g_err = keep;
        return r;
    }
    *out = c;
    return KVMRET_OK;
}

void kvmret_destroy(kvmret_ctx *c) {
    if (!c) return;
    free_all(c);
    delete c;
}

void *kvmret_stream(kvmret_ctx *c) { return c ? static_cast<void *>(c->st) : nullptr; }

int kvmret_sync(kvmret_ctx *c) {
    NEED_CTX(c);
    CK(cudaStreamSynchronize(c->st));
    GUARD(return drain(c));
}

void *kvmret_repo_host(kvmret_ctx *c) { return c ? c->repo_host : nullptr; }
uint64_t kvmret_repo_unit_bytes(kvmret_ctx *c) { return c ? c->unit : 0; }
uint64_t kvmret_repo_k_bytes(kvmret_ctx *c) { return c ? c->unit_k : 0; }
uint32_t kvmret_n_blocks(kvmret_ctx *c) { return c ? c->live_blocks() : 0; }
uint32_t kvmret_n_tokens(kvmret_ctx *c) { return c ? c->live_tokens : 0; }

namespace {

kvmret::AppendArgs append_args(kvmret_ctx *c) {
    kvmret::AppendArgs a{};
    a.n_layer = c->cfg.n_layer;
    a.n_head_kv = c->cfg.n_head_kv;
    a.d_head = c->cfg.d_head;
    a.block_tokens = c->cfg.block_tokens;
    a.ncap = c->ncap;
    a.k_row = c->k_row;
    a.v_row = c->v_row;
    a.unit_k = c->unit_k;
    a.unit = c->unit;
    a.summ = c->summ;
    a.blk_ntok = c->d_blk_ntok;
    a.tail_sum = c->tail_sum;
    a.has_block = c->has_block;
    a.repo_dev = c->repo_dev;
    return a;
}

// Gen mode, before an append of tokens [pos0, pos0 + n_tok): every touched
// block without a window slot gets one (prepare_working_set's alloc_slot for
// incoming blocks, llama-memory-kvmem.cpp:2349-2365). The reference's pool
// of GPU slots is budget + gen_reserve; here a bound block takes the first
// free window slot (it is the newest block, so that is its chronological
// place; its RoPE base is the window's token count) and an HBM pool slot (a
// free one, else the least recently used pooled block outside the window).
// With no free window or pool slot the append fails before anything is
// enqueued ("no free GPU slot", as the reference reports and then truncates
// the store back). Fills the write list of the touched blocks.
int gen_prepare(kvmret_ctx *c, uint32_t pos0, uint32_t n_tok, kvmret::GenWrite &gw) {
    const uint32_t T = c->cfg.block_tokens;
    const uint32_t b_lo = pos0 / T, b_hi = (pos0 + n_tok - 1) / T;
    if (b_hi - b_lo + 1 > static_cast<uint32_t>(kvmret::kMaxGenSegs))
        return fail(KVMRET_ERR_ARG, "gen mode: an append may touch at most %d blocks (%u tokens)",
                    kvmret::kMaxGenSegs, (kvmret::kMaxGenSegs - 1) * T);
    std::vector<uint32_t> rebuild_lo(b_hi - b_lo + 1, ~0u);
    bool need = false;
    for (uint32_t b = b_lo; b <= b_hi; ++b) need |= !c->gen_bound[b];
    if (need) {
        const uint32_t W = c->win_slots, P = c->pool_slots;
        std::vector<int32_t> win_id(W), win_base(W), slot_blk(P), blk_slot(b_hi - b_lo + 1);
        std::vector<uint32_t> win_ntok(W), slot_used(P);
        CK(cudaStreamSynchronize(c->st));
        CK(cudaMemcpy(win_id.data(), c->d_win_id, W * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(win_base.data(), c->d_win_base, W * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(win_ntok.data(), c->d_win_ntok, W * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(slot_blk.data(), c->d_slot_blk, P * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(slot_used.data(), c->d_slot_used, P * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(blk_slot.data(), c->d_blk_slot + b_lo, blk_slot.size() * 4,
                      cudaMemcpyDeviceToHost));
        std::vector<uint8_t> in_win(c->ncap, 0);
        for (int32_t id : win_id)
            if (id >= 0 && static_cast<uint32_t>(id) < c->ncap) in_win[id] = 1;
        kvmret::GenBinds gb{};
        gb.step = c->step;
        for (uint32_t b = b_lo; b <= b_hi; ++b) {
            if (c->gen_bound[b]) continue;
            const uint32_t n_exist = pos0 > b * T ? std::min(T, pos0 - b * T) : 0;
            uint32_t ws = 0;
            int32_t base = 0;
            if (in_win[b]) {
                while (win_id[ws] != static_cast<int32_t>(b)) ++ws;
                // a window slot holding all the block's rows needs nothing;
                // one left behind by appends made outside gen mode is
                // rebuilt in place from the repository's rows
                if (win_ntok[ws] == n_exist) continue;
                base = win_base[ws];
            } else {
                while (ws < W && win_id[ws] >= 0) ++ws;
                if (ws == W)
                    return fail(KVMRET_ERR_STATE,
                                "no free GPU slot for block %u (all %u window slots hold blocks)",
                                b, W);
                for (uint32_t i = 0; i < ws; ++i) base += static_cast<int32_t>(win_ntok[i]);
            }
            int32_t ps = blk_slot[b - b_lo], evict = -1;
            if (ps < 0) {
                for (uint32_t k = 0; k < P && ps < 0; ++k)
                    if (slot_blk[k] < 0) ps = static_cast<int32_t>(k);
            }
            if (ps < 0) {  // least recently used pooled block outside the window
                for (uint32_t k = 0; k < P; ++k) {
                    const int32_t o = slot_blk[k];
                    if (o < 0 || in_win[o]) continue;
                    if (ps < 0 || slot_used[k] < slot_used[ps]) ps = static_cast<int32_t>(k);
                }
                if (ps < 0)
                    return fail(KVMRET_ERR_STATE,
                                "no free GPU slot for block %u (all %u pool slots hold window "
                                "blocks)", b, P);
                evict = slot_blk[ps];
            }
            kvmret::GenBind &gbi = gb.b[gb.n++];
            gbi.block = b;
            gbi.win_slot = ws;
            gbi.pool_slot = static_cast<uint32_t>(ps);
            gbi.n_exist = n_exist;
            gbi.base = base;
            gbi.evict_block = evict;
            // host mirrors for the next binding of this append: the block
            // fills up to its final token count before the next one starts
            win_id[ws] = static_cast<int32_t>(b);
            win_ntok[ws] = std::min(T, pos0 + n_tok - b * T);
            slot_blk[ps] = static_cast<int32_t>(b);
            in_win[b] = 1;
            rebuild_lo[b - b_lo] = 0;
        }
        // enqueue: the existing rows of partial blocks into their pool slots,
        // then the bindings
        for (uint32_t i = 0; i < gb.n; ++i)
            if (gb.b[i].n_exist)
                CK(cudaMemcpyAsync(c->pool + static_cast<uint64_t>(gb.b[i].pool_slot) * c->slot_bytes,
                                   c->repo_host + static_cast<uint64_t>(gb.b[i].block) * c->slot_bytes,
                                   c->slot_bytes, cudaMemcpyHostToDevice, c->st));
        gb.win_id = c->d_win_id;
        gb.win_base = c->d_win_base;
        gb.win_ntok = c->d_win_ntok;
        gb.blk_slot = c->d_blk_slot;
        gb.slot_blk = c->d_slot_blk;
        gb.slot_ntok = c->d_slot_ntok;
        gb.slot_used = c->d_slot_used;
        CK(kvmret::launch_gen_bind(gb, c->st));
        c->prof.launches += gb.n ? 1 : 0;
        for (uint32_t i = 0; i < gb.n; ++i) table_op(c, OP_ON_GPU, gb.b[i].block);
        for (uint32_t b = b_lo; b <= b_hi; ++b) c->gen_bound[b] = 1;
    }
    gw.n_seg = 0;
    for (uint32_t b = b_lo; b <= b_hi; ++b) {
        kvmret::GenSeg &sg = gw.seg[gw.n_seg++];
        sg.block = b;
        sg.new_lo = std::max(pos0, b * T) - b * T;
        sg.new_hi = std::min(pos0 + n_tok, (b + 1) * T) - b * T;
        sg.rebuild_lo = rebuild_lo[b - b_lo] == 0 ? 0 : sg.new_lo;
        sg.tok0 = b * T + sg.new_lo - pos0;
    }
    return KVMRET_OK;
}

}  // namespace

int kvmret_append(kvmret_ctx *c, uint32_t pos0, uint32_t n_tok, const uint16_t *k_cap,
                  const void *k_rows, const void *v_rows) {
    NEED_CTX(c);
    if (pos0 != c->live_tokens)
        return fail(KVMRET_ERR_ARG, "append at %u, store holds %u tokens", pos0, c->live_tokens);
    if (n_tok == 0) return KVMRET_OK;
    const uint64_t cap = static_cast<uint64_t>(c->cfg.max_blocks) * c->cfg.block_tokens;
    if (static_cast<uint64_t>(pos0) + n_tok > cap)
        return fail(KVMRET_ERR_ARG, "append of %u tokens exceeds capacity %llu", n_tok,
                    (unsigned long long)cap);
    if (!k_cap || !v_rows) return fail(KVMRET_ERR_ARG, "k_cap and v_rows are required");
    if (!k_rows) {
        if (c->cfg.k_type != KVMRET_TYPE_F16)
            return fail(KVMRET_ERR_ARG, "k_rows required for quantised K");
        k_rows = k_cap;
    }
    kvmret::GenWrite gw{};
    if (c->gen_on) GUARD(TRY(gen_prepare(c, pos0, n_tok, gw)));
    kvmret::AppendArgs a = append_args(c);
    a.k_cap = k_cap;
    a.k_rows = static_cast<const uint8_t *>(k_rows);
    a.v_rows = static_cast<const uint8_t *>(v_rows);
    a.pos0 = pos0;
    a.n_tok = n_tok;
    CK(kvmret::launch_append(a, c->st));
    c->prof.launches += 2;
    if (c->gen_on) {  // the decode tokens into the window and the pool
        gw.n_tok_append = n_tok;
        gw.win_slots = c->win_slots;
        gw.k_rows = a.k_rows;
        gw.v_rows = a.v_rows;
        gw.pool = c->pool;
        gw.slot_bytes = c->slot_bytes;
        gw.win_k = c->win_k;
        gw.win_v = c->win_v;
        gw.gtab = c->rope_tab;
        gw.win_id = c->d_win_id;
        gw.win_base = c->d_win_base;
        gw.blk_slot = c->d_blk_slot;
        gw.win_ntok = c->d_win_ntok;
        gw.slot_ntok = c->d_slot_ntok;
        gw.err = c->d_gen_err;
        gw.g = c->geom;
        CK(kvmret::launch_gen_write(gw, c->st));
        c->prof.launches += 1;
    }
    // the prefill scorer's unit summaries of the touched blocks are stale now
    c->mhat_valid = std::min(c->mhat_valid, pos0 / c->cfg.block_tokens);
    c->live_tokens += n_tok;
    GUARD(table_op(c, OP_APPEND, n_tok));
    c->kept_valid = false;
    return KVMRET_OK;
}

int kvmret_truncate(kvmret_ctx *c, uint32_t n_tokens) {
    NEED_CTX(c);
    if (n_tokens > c->live_tokens)
        return fail(KVMRET_ERR_ARG, "truncate to %u tokens, store holds %u", n_tokens,
                    c->live_tokens);
    if (n_tokens == c->live_tokens) return KVMRET_OK;
    const uint32_t T = c->cfg.block_tokens;
    const uint32_t tail = n_tokens % T;
    if (tail && c->cfg.k_type != KVMRET_TYPE_F16)
        return fail(KVMRET_ERR_ARG,
                    "quantised K: truncate to a block boundary (the repository holds no f16 K "
                    "to rebuild a partial block's summary from)");
    GUARD(TRY(drain(c)));
    const uint32_t nb_old = c->live_blocks();
    const uint32_t nb_new = (n_tokens + T - 1) / T;
    kvmret::TruncArgs ta{};
    ta.nb_new = nb_new;
    ta.nb_old = nb_old;
    ta.tail_ntok = tail;
    ta.pool_slots = c->pool_slots;
    ta.win_slots = c->win_slots;
    ta.has_block = c->has_block;
    ta.blk_ntok = c->d_blk_ntok;
    ta.blk_slot = c->d_blk_slot;
    ta.slot_blk = c->d_slot_blk;
    ta.slot_ntok = c->d_slot_ntok;
    ta.win_id = c->d_win_id;
    ta.win_ntok = c->d_win_ntok;
    CK(kvmret::launch_truncate(ta, c->st));
    if (tail) CK(kvmret::launch_resum(append_args(c), nb_new - 1, tail, c->st));
    c->prof.launches += tail ? 2 : 1;
    GUARD(c->table.truncate(n_tokens));
    c->live_tokens = n_tokens;
    for (uint32_t b = nb_new; b < nb_old && b < c->ncap; ++b) c->gen_bound[b] = 0;
    if (c->gen_on) c->gen_first = std::min(c->gen_first, n_tokens / T);
    c->mhat_valid = std::min(c->mhat_valid, n_tokens / T);
    c->kept_valid = false;
    CK(cudaStreamSynchronize(c->st));
    return KVMRET_OK;
}

int kvmret_gen_begin(kvmret_ctx *c) {
    NEED_CTX(c);
    if (c->gen_on) return fail(KVMRET_ERR_STATE, "gen mode is already on");
    c->gen_on = true;
    c->gen_first = c->live_tokens / c->cfg.block_tokens;
    std::fill(c->gen_bound.begin(), c->gen_bound.end(), 0);
    c->kept_valid = false;
    return KVMRET_OK;
}

int kvmret_gen_end(kvmret_ctx *c) {
    NEED_CTX(c);
    if (!c->gen_on) return KVMRET_OK;
    uint32_t err = 0;
    CK(cudaMemcpyAsync(&err, c->d_gen_err, sizeof(err), cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    c->gen_on = false;
    c->kept_valid = false;
    if (err) {
        CK(cudaMemset(c->d_gen_err, 0, sizeof(err)));
        return fail(KVMRET_ERR_STATE, "a decode block bound to the window was missing from it "
                                      "when its tokens were written");
    }
    return KVMRET_OK;
}

int kvmret_cells(kvmret_ctx *c, uint32_t pos0, uint32_t n_tok, int32_t *cells_out) {
    NEED_CTX(c);
    if (n_tok && !cells_out) return fail(KVMRET_ERR_ARG, "null output");
    if (static_cast<uint64_t>(pos0) + n_tok > c->live_tokens)
        return fail(KVMRET_ERR_ARG, "positions [%u, %u) beyond the %u stored tokens", pos0,
                    pos0 + n_tok, c->live_tokens);
    std::vector<int32_t> win_id;
    GUARD(win_id.resize(c->win_slots));
    CK(cudaStreamSynchronize(c->st));
    CK(cudaMemcpy(win_id.data(), c->d_win_id, c->win_slots * 4, cudaMemcpyDeviceToHost));
    const uint32_t T = c->cfg.block_tokens;
    int32_t cur_b = -1, cur_s = -1;
    for (uint32_t i = 0; i < n_tok; ++i) {
        const uint32_t p = pos0 + i, b = p / T;
        if (static_cast<int32_t>(b) != cur_b) {
            cur_b = static_cast<int32_t>(b);
            cur_s = -1;
            for (uint32_t k = 0; k < c->win_slots; ++k)
                if (win_id[k] == cur_b) cur_s = static_cast<int32_t>(k);
        }
        cells_out[i] = cur_s < 0 ? -1 : cur_s * static_cast<int32_t>(T) + static_cast<int32_t>(p - b * T);
    }
    return KVMRET_OK;
}

uint32_t kvmret_gen_first_block(kvmret_ctx *c) {
    return (c && c->gen_on) ? c->gen_first : 0xffffffffu;
}

int kvmret_get_summaries(kvmret_ctx *c, float *out) {
    NEED_CTX(c);
    if (!out) return fail(KVMRET_ERR_ARG, "null output");
    const uint32_t n = c->live_blocks(), L = c->cfg.n_layer, E = c->E;
    std::vector<float> tmp;
    GUARD(tmp.resize(static_cast<size_t>(L) * E * c->ncap));
    CK(cudaMemcpyAsync(tmp.data(), c->summ, tmp.size() * sizeof(float), cudaMemcpyDeviceToHost,
                       c->st));
    CK(cudaStreamSynchronize(c->st));
    for (uint32_t b = 0; b < n; ++b)
        for (uint32_t l = 0; l < L; ++l)
            for (uint32_t e = 0; e < E; ++e)
                out[(static_cast<size_t>(b) * L + l) * E + e] =
                    tmp[(static_cast<size_t>(l) * E + e) * c->ncap + b];
    return KVMRET_OK;
}

int kvmret_query_reset(kvmret_ctx *c) {
    NEED_CTX(c);
    std::fill(c->q_count.begin(), c->q_count.end(), 0u);
    c->q_reset_pending = true;  // the next add assigns instead of adding
    c->q_dirty = true;
    return KVMRET_OK;
}

static int query_add(kvmret_ctx *c, const void *q, bool f16, uint32_t n_rows) {
    NEED_CTX(c);
    if (!q) return fail(KVMRET_ERR_ARG, "null query");
    if (n_rows == 0) return KVMRET_OK;
    CK(kvmret::launch_query_add(c->q_sum, q, f16, c->cfg.n_layer, n_rows, c->qdim, c->st,
                                c->q_count_dev, c->q_reset_pending));
    c->q_reset_pending = false;
    c->prof.launches += 1;
    for (auto &x : c->q_count) x += n_rows;
    c->q_dirty = true;
    return KVMRET_OK;
}

int kvmret_query_add_f16(kvmret_ctx *c, const uint16_t *q, uint32_t n_rows) {
    return query_add(c, q, true, n_rows);
}
int kvmret_query_add_f32(kvmret_ctx *c, const float *q, uint32_t n_rows) {
    return query_add(c, q, false, n_rows);
}

int kvmret_query_set(kvmret_ctx *c, const float *q_sum, const uint32_t *q_count) {
    NEED_CTX(c);
    if (!q_sum || !q_count) return fail(KVMRET_ERR_ARG, "null query state");
    CK(cudaMemcpyAsync(c->q_sum, q_sum,
                       static_cast<size_t>(c->cfg.n_layer) * c->qdim * sizeof(float),
                       cudaMemcpyHostToDevice, c->st));
    for (uint32_t l = 0; l < c->cfg.n_layer; ++l) c->q_count[l] = q_count[l];
    CK(cudaMemcpyAsync(c->q_count_dev, c->q_count.data(), c->cfg.n_layer * sizeof(uint32_t),
                       cudaMemcpyHostToDevice, c->st));
    c->q_reset_pending = false;
    c->q_dirty = true;
    CK(cudaStreamSynchronize(c->st));
    return KVMRET_OK;
}

int kvmret_query_get(kvmret_ctx *c, float *q_sum, uint32_t *q_count) {
    NEED_CTX(c);
    TRY(settle_query(c));
    if (q_sum) {
        CK(cudaMemcpyAsync(q_sum, c->q_sum,
                           static_cast<size_t>(c->cfg.n_layer) * c->qdim * sizeof(float),
                           cudaMemcpyDeviceToHost, c->st));
        CK(cudaStreamSynchronize(c->st));
    }
    if (q_count)
        for (uint32_t l = 0; l < c->cfg.n_layer; ++l) q_count[l] = c->q_count[l];
    return KVMRET_OK;
}

int kvmret_score(kvmret_ctx *c, double *scores_host) {
    NEED_CTX(c);
    TRY(score_layers_impl(c, nullptr));
    TRY(reduce_impl(c, c->contrib, c->cfg.n_layer, c->active));
    if (scores_host) {
        CK(cudaMemcpyAsync(scores_host, c->scores, c->live_blocks() * sizeof(double),
                           cudaMemcpyDeviceToHost, c->st));
        CK(cudaStreamSynchronize(c->st));
    }
    return KVMRET_OK;
}

int kvmret_score_layers(kvmret_ctx *c, double *contrib_out) {
    NEED_CTX(c);
    return score_layers_impl(c, contrib_out);
}

const double *kvmret_contrib_dev(kvmret_ctx *c) { return c ? c->contrib : nullptr; }
uint32_t kvmret_contrib_stride(kvmret_ctx *c) { return c ? c->cstride : 0; }

int kvmret_score_reduce(kvmret_ctx *c, const double *contrib_all, uint32_t n_layer_all) {
    NEED_CTX(c);
    if (!contrib_all || n_layer_all == 0) return fail(KVMRET_ERR_ARG, "bad contribution buffer");
    return reduce_impl(c, contrib_all, n_layer_all, nullptr);
}

int kvmret_prof_enable(kvmret_ctx *c, int on) {
    NEED_CTX(c);
    CK(cudaStreamSynchronize(c->st));
    GUARD(TRY(drain(c)));
    if (on && c->ev_pool.empty()) {
        GUARD(c->ev_pool.resize(kEventPool, nullptr));
        for (auto &e : c->ev_pool) CK(cudaEventCreate(&e));
    }
    c->prof = kvmret_prof{};
    c->pending.clear();
    c->ev_next = 0;
    c->prof_on = on != 0;
    return KVMRET_OK;
}

int kvmret_prof_read(kvmret_ctx *c, kvmret_prof *out) {
    NEED_CTX(c);
    if (!out) return fail(KVMRET_ERR_ARG, "null output");
    CK(cudaStreamSynchronize(c->st));
    GUARD(TRY(drain(c)));
    for (const auto &r : c->pending) {
        float ms = 0.0f;
        CK(cudaEventElapsedTime(&ms, r.a, r.b));
        if (r.kind == PR_SCORE) {
            c->prof.score_ms += ms;
            ++c->prof.n_score;
        } else if (r.kind == PR_GEMM) {
            c->prof.gemm_ms += ms;
            ++c->prof.n_gemm;
        } else {
            c->prof.asm_ms += ms;
            ++c->prof.n_asm;
        }
    }
    c->pending.clear();
    c->ev_next = 0;
    *out = c->prof;
    return KVMRET_OK;
}

int kvmret_select(kvmret_ctx *c, const uint32_t *mandatory, uint32_t n_mand, uint32_t *ids_out,
                  uint32_t *n_out) {
    NEED_CTX(c);
    if (n_mand && !mandatory) return fail(KVMRET_ERR_ARG, "null mandatory list");
    GUARD(return preview_impl(c, mandatory, n_mand, ids_out, n_out));
}

int kvmret_preview(kvmret_ctx *c, const uint32_t *mandatory, uint32_t n_mand, uint32_t *ids_out,
                   uint32_t *n_out) {
    NEED_CTX(c);
    TRY(kvmret_score(c, nullptr));
    return kvmret_select(c, mandatory, n_mand, ids_out, n_out);
}

int kvmret_apply_selection(kvmret_ctx *c, const uint32_t *ids, uint32_t n_ids,
                           kvmret_step_stats *stats) {
    NEED_CTX(c);
    if (n_ids && !ids) return fail(KVMRET_ERR_ARG, "null id list");
    GUARD(return apply_impl(c, ids, n_ids, stats));
}

int kvmret_clear_working_set(kvmret_ctx *c, int drop_pool) {
    NEED_CTX(c);
    GUARD(TRY(drain(c)));
    GUARD(c->table.clear_working_set(drop_pool != 0));
    // the window loses every block, decode blocks bound to it included
    std::fill(c->gen_bound.begin(), c->gen_bound.end(), 0);
    // an empty window: every slot of the next selection is rebuilt, from the
    // pool where the block is still pooled, else from the host repository
    const size_t W = c->win_slots, P = c->pool_slots;
    CK(cudaMemsetAsync(c->d_win_id, 0xff, W * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_win_base, 0, W * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_win_ntok, 0, W * sizeof(uint32_t), c->st));
    if (drop_pool) {  // the pool as created: no block pooled, no LRU history
        CK(cudaMemsetAsync(c->d_blk_slot, 0xff, c->ncap * sizeof(int32_t), c->st));
        CK(cudaMemsetAsync(c->d_slot_blk, 0xff, P * sizeof(int32_t), c->st));
        CK(cudaMemsetAsync(c->d_slot_ntok, 0, P * sizeof(uint32_t), c->st));
        CK(cudaMemsetAsync(c->d_slot_used, 0, P * sizeof(uint32_t), c->st));
    }
    c->last_plan = kvmret::Plan{};
    return KVMRET_OK;
}

int kvmret_set_pool_cache(kvmret_ctx *c, int on) {
    NEED_CTX(c);
    GUARD(TRY(drain(c)));
    // the next plan frees every pooled block outside its window when caching
    // is off (its release pass scans all pool slots)
    c->cfg.pool_cache = on != 0;
    return KVMRET_OK;
}

int kvmret_pool_prefetch(kvmret_ctx *c, uint32_t first_block, uint32_t n_blocks,
                         uint32_t *n_placed) {
    NEED_CTX(c);
    if (n_placed) *n_placed = 0;
    if (!c->cfg.pool_cache) return fail(KVMRET_ERR_STATE, "pool prefetch needs pool caching on");
    GUARD(TRY(drain(c)));
    CK(cudaStreamSynchronize(c->st));
    const uint32_t nb = c->live_blocks();
    const uint32_t b0 = std::min(first_block, nb);
    const uint32_t b1 = static_cast<uint32_t>(
        std::min<uint64_t>(nb, static_cast<uint64_t>(first_block) + n_blocks));
    if (b0 >= b1) return KVMRET_OK;
    const uint32_t P = c->pool_slots, T = c->cfg.block_tokens;
    std::vector<int32_t> slot_blk(P), blk_slot(b1 - b0);
    std::vector<uint32_t> slot_ntok(P), slot_used(P);
    CK(cudaMemcpy(slot_blk.data(), c->d_slot_blk, P * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(slot_ntok.data(), c->d_slot_ntok, P * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(slot_used.data(), c->d_slot_used, P * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(blk_slot.data(), c->d_blk_slot + b0, blk_slot.size() * 4,
                  cudaMemcpyDeviceToHost));
    // lowest free slot first; runs of consecutive blocks in consecutive slots
    // become one copy
    struct Run { uint32_t b, s, n; };
    std::vector<Run> runs;
    uint32_t s = 0, placed = 0;
    for (uint32_t b = b0; b < b1; ++b) {
        if (blk_slot[b - b0] >= 0) continue;
        while (s < P && slot_blk[s] >= 0) ++s;
        if (s == P) break;
        slot_blk[s] = static_cast<int32_t>(b);
        blk_slot[b - b0] = static_cast<int32_t>(s);
        slot_ntok[s] = std::min(T, c->live_tokens - b * T);
        slot_used[s] = 0;  // least recently used: the first to go when room is needed
        if (!runs.empty() && runs.back().b + runs.back().n == b && runs.back().s + runs.back().n == s)
            ++runs.back().n;
        else
            GUARD(runs.push_back({b, s, 1}));
        ++placed;
        ++s;
    }
    for (const Run &r : runs)
        CK(cudaMemcpyAsync(c->pool + static_cast<uint64_t>(r.s) * c->slot_bytes,
                           c->repo_host + static_cast<uint64_t>(r.b) * c->slot_bytes,
                           static_cast<uint64_t>(r.n) * c->slot_bytes, cudaMemcpyHostToDevice,
                           c->st));
    CK(cudaMemcpyAsync(c->d_slot_blk, slot_blk.data(), P * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->d_slot_ntok, slot_ntok.data(), P * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->d_slot_used, slot_used.data(), P * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->d_blk_slot + b0, blk_slot.data(), blk_slot.size() * 4,
                       cudaMemcpyHostToDevice, c->st));
    CK(cudaStreamSynchronize(c->st));  // the host vectors are the copies' sources
    if (n_placed) *n_placed = placed;
    return KVMRET_OK;
}

int kvmret_select_apply_async(kvmret_ctx *c, const uint32_t *mandatory, uint32_t n_mand) {
    NEED_CTX(c);
    if (n_mand && !mandatory) return fail(KVMRET_ERR_ARG, "null mandatory list");
    GUARD(TRY(select_device(c, mandatory, n_mand)));
    GUARD(return plan_and_assemble(c));
}

int kvmret_step_collect(kvmret_ctx *c, uint32_t *ids_out, uint32_t *n_out,
                        kvmret_step_stats *stats) {
    NEED_CTX(c);
    if (c->rb_pending == 0) return fail(KVMRET_ERR_STATE, "no step to collect");
    GUARD(TRY(collect_one(c, ids_out, n_out)));
    if (stats) *stats = c->last_stats;
    return KVMRET_OK;
}

int kvmret_apply_retrieval(kvmret_ctx *c, const uint32_t *mandatory, uint32_t n_mand,
                           uint32_t *ids_out, uint32_t *n_out, kvmret_step_stats *stats) {
    NEED_CTX(c);
    TRY(kvmret_score(c, nullptr));
    GUARD(TRY(drain(c)));
    TRY(kvmret_select_apply_async(c, mandatory, n_mand));
    return kvmret_step_collect(c, ids_out, n_out, stats);
}

int kvmret_last_plan(kvmret_ctx *c, int32_t *remaps, uint32_t *n_remaps, uint32_t *stage_in,
                     uint32_t *n_stage_in, uint32_t *stage_out, uint32_t *n_stage_out) {
    NEED_CTX(c);
    GUARD(TRY(drain(c)));
    const kvmret::Plan &p = c->last_plan;
    if (n_remaps) *n_remaps = static_cast<uint32_t>(p.remaps.size());
    if (remaps)
        for (size_t i = 0; i < p.remaps.size(); ++i) {
            const auto &r = p.remaps[i];
            int32_t *o = remaps + 7 * i;
            o[0] = static_cast<int32_t>(r.id);
            o[1] = static_cast<int32_t>(r.n_tok);
            o[2] = r.from;
            o[3] = r.to;
            o[4] = r.resident;
            o[5] = r.skip;
            o[6] = r.raw;
        }
    if (n_stage_in) *n_stage_in = static_cast<uint32_t>(p.stage_in.size());
    if (stage_in) std::copy(p.stage_in.begin(), p.stage_in.end(), stage_in);
    if (n_stage_out) *n_stage_out = static_cast<uint32_t>(p.stage_out.size());
    if (stage_out) std::copy(p.stage_out.begin(), p.stage_out.end(), stage_out);
    return KVMRET_OK;
}

void *kvmret_window_k(kvmret_ctx *c, uint32_t layer) {
    return (c && layer < c->cfg.n_layer) ? c->win_k + layer * c->win_k_layer : nullptr;
}
void *kvmret_window_v(kvmret_ctx *c, uint32_t layer) {
    return (c && layer < c->cfg.n_layer) ? c->win_v + layer * c->win_v_layer : nullptr;
}
uint32_t kvmret_window_slots(kvmret_ctx *c) { return c ? c->win_slots : 0; }

int kvmret_window_layout(kvmret_ctx *c, uint32_t *ids, int32_t *bases, uint32_t *n_out) {
    NEED_CTX(c);
    if (!n_out) return fail(KVMRET_ERR_ARG, "null argument");
    std::vector<int32_t> wid, wb;
    GUARD(wid.resize(c->win_slots));
    GUARD(wb.resize(c->win_slots));
    CK(cudaMemcpyAsync(wid.data(), c->d_win_id, c->win_slots * sizeof(int32_t),
                       cudaMemcpyDeviceToHost, c->st));
    CK(cudaMemcpyAsync(wb.data(), c->d_win_base, c->win_slots * sizeof(int32_t),
                       cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    uint32_t n = 0;
    while (n < c->win_slots && wid[n] >= 0) {
        if (ids) ids[n] = static_cast<uint32_t>(wid[n]);
        if (bases) bases[n] = wb[n];
        ++n;
    }
    *n_out = n;
    return KVMRET_OK;
}

int kvmret_window_read(kvmret_ctx *c, uint32_t layer, int is_v, uint32_t slot0, uint32_t n_slots,
                       void *out) {
    NEED_CTX(c);
    if (!out || layer >= c->cfg.n_layer || slot0 + static_cast<uint64_t>(n_slots) > c->win_slots)
        return fail(KVMRET_ERR_ARG, "window read out of range");
    const uint64_t row = is_v ? c->v_row : c->k_row;
    const uint64_t span = static_cast<uint64_t>(c->cfg.block_tokens) * row;
    const uint8_t *base = (is_v ? c->win_v + layer * c->win_v_layer
                                : c->win_k + layer * c->win_k_layer) + slot0 * span;
    CK(cudaStreamSynchronize(c->st));
    CK(cudaMemcpy(out, base, n_slots * span, cudaMemcpyDeviceToHost));
    return KVMRET_OK;
}

namespace {
// Stateless RoPE over a contiguous run of n_tok rows at positions pos0 ..:
// a temporary cos/sin table of those positions (indexed from 0), then the
// assembly kernel's stateless form, chunks of 128 rows.
int rope_stateless(kvmret::AsmLaunch &al, uint32_t n_tok, uint32_t n_rot, int32_t pos0,
                   cudaStream_t st) {
    float4 *tab = nullptr;
    const size_t tab_bytes = static_cast<size_t>(n_tok) * (n_rot / 4) * sizeof(float4);
    CK(cudaMallocAsync(reinterpret_cast<void **>(&tab), tab_bytes, st));
    al.synth_pos0 = 0;
    al.synth_ntok = n_tok;
    al.gtab = tab;
    cudaError_t e = kvmret::launch_rope_table(tab, n_tok, n_rot / 2, al.theta, st, pos0);
    if (e == cudaSuccess) e = kvmret::launch_assemble(al, (n_tok + 127) / 128, st);
    const cudaError_t ef = cudaFreeAsync(tab, st);
    CK(e);
    CK(ef);
    return KVMRET_OK;
}
}  // namespace

int kvmret_rope_f16(const uint16_t *k, uint16_t *out, uint32_t n_tok, uint32_t n_head_kv,
                    uint32_t d_head, uint32_t n_rot, int32_t pos0, float freq_base,
                    float freq_scale, void *stream) {
    if (!k || !out || n_head_kv == 0) return fail(KVMRET_ERR_ARG, "bad rope arguments");
    if ((d_head != 64 && d_head != 128 && d_head != 256) || n_rot != d_head)
        return fail(KVMRET_ERR_ARG, "rope needs d_head in {64,128,256} and n_rot == d_head");
    if (n_tok == 0) return KVMRET_OK;
    kvmret::AssembleGeom g{};
    g.n_layer = 1;
    g.n_head_kv = n_head_kv;
    g.d_head = d_head;
    g.block_tokens = 128;
    g.k_row = 2ull * n_head_kv * d_head;
    g.k_type = KVMRET_TYPE_F16;
    kvmret::AsmLaunch al{};
    al.pool = reinterpret_cast<const uint8_t *>(k);
    al.slot_bytes = 128 * g.k_row;
    al.win_k = reinterpret_cast<uint8_t *>(out);
    al.theta = make_theta(n_rot, freq_base, freq_scale);
    al.g = g;
    return rope_stateless(al, n_tok, n_rot, pos0, static_cast<cudaStream_t>(stream));
}

int kvmret_topk_select(const double *scores, const uint8_t *kept, uint32_t n, uint32_t need,
                       int tie_higher_id, uint8_t *sel, void *stream) {
    if (n == 0) return KVMRET_OK;
    if (!scores || !kept || !sel) return fail(KVMRET_ERR_ARG, "null buffer");
    CK(kvmret::launch_select(scores, kept, n, need, tie_higher_id ? 1 : 0, sel,
                             static_cast<cudaStream_t>(stream)));
    return KVMRET_OK;
}

namespace {
int rope_quant(int32_t type, const void *k, void *out, uint32_t n_tok, uint32_t n_head_kv,
               uint32_t d_head, uint32_t n_rot, int32_t pos0, float freq_base, float freq_scale,
               uint32_t fwht_n, void *stream) {
    if (!k || !out || n_head_kv == 0) return fail(KVMRET_ERR_ARG, "bad rope arguments");
    if ((d_head != 64 && d_head != 128 && d_head != 256) || n_rot != d_head)
        return fail(KVMRET_ERR_ARG, "rope needs d_head in {64,128,256} and n_rot == d_head");
    if (fwht_n != 0 && fwht_n != d_head)
        return fail(KVMRET_ERR_ARG, "fwht_n must be 0 or d_head");
    const uint64_t row = kvmret_row_bytes(type, n_head_kv * d_head);
    if (row % 16) return fail(KVMRET_ERR_ARG, "quantised K row of %llu bytes not 16-aligned",
                              (unsigned long long)row);
    if (n_tok == 0) return KVMRET_OK;
    kvmret::AssembleGeom g{};
    g.n_layer = 1;
    g.n_head_kv = n_head_kv;
    g.d_head = d_head;
    g.block_tokens = 128;
    g.k_row = row;
    g.k_type = type;
    g.fwht_n = fwht_n;
    g.fwht_scale = fwht_n ? 1.0f / std::sqrt(static_cast<float>(fwht_n)) : 0.0f;
    kvmret::AsmLaunch al{};
    al.pool = static_cast<const uint8_t *>(k);
    al.slot_bytes = 128 * row;
    al.win_k = static_cast<uint8_t *>(out);
    al.theta = make_theta(n_rot, freq_base, freq_scale);
    al.g = g;
    return rope_stateless(al, n_tok, n_rot, pos0, static_cast<cudaStream_t>(stream));
}
}  // namespace

int kvmret_rope_q8_0(const void *k, void *out, uint32_t n_tok, uint32_t n_head_kv,
                     uint32_t d_head, uint32_t n_rot, int32_t pos0, float freq_base,
                     float freq_scale, uint32_t fwht_n, void *stream) {
    return rope_quant(KVMRET_TYPE_Q8_0, k, out, n_tok, n_head_kv, d_head, n_rot, pos0, freq_base,
                      freq_scale, fwht_n, stream);
}

int kvmret_rope_q4_0(const void *k, void *out, uint32_t n_tok, uint32_t n_head_kv,
                     uint32_t d_head, uint32_t n_rot, int32_t pos0, float freq_base,
                     float freq_scale, uint32_t fwht_n, void *stream) {
    return rope_quant(KVMRET_TYPE_Q4_0, k, out, n_tok, n_head_kv, d_head, n_rot, pos0, freq_base,
                      freq_scale, fwht_n, stream);
}

int kvmret_quantize_f16(const uint16_t *src, void *dst, int32_t type, uint64_t n_elems,
                        void *stream) {
    if (!src || !dst) return fail(KVMRET_ERR_ARG, "null buffer");
    if (type != KVMRET_TYPE_Q8_0 && type != KVMRET_TYPE_Q4_0)
        return fail(KVMRET_ERR_ARG, "type must be q8_0 or q4_0");
    if (n_elems % 32 || (reinterpret_cast<uintptr_t>(src) & 15))
        return fail(KVMRET_ERR_ARG, "n_elems must be a multiple of 32 and src 16-byte aligned");
    CK(kvmret::launch_quantize(src, static_cast<uint8_t *>(dst), n_elems / 32,
                               type == KVMRET_TYPE_Q8_0, static_cast<cudaStream_t>(stream)));
    return KVMRET_OK;
}

int kvmret_d2d_batched(kvmret_ctx *c, const void *const *src, void *const *dst,
                       const uint64_t *nbytes, int n) {
    NEED_CTX(c);
    if (n <= 0) return KVMRET_OK;
    if (!src || !dst || !nbytes || n > 8192)
        return fail(KVMRET_ERR_ARG, "bad batched copy (n %d, max 8192)", n);
    std::vector<kvmret::CopyOp> ops;
    GUARD(ops.resize(n));
    for (int i = 0; i < n; ++i)
        ops[i] = {static_cast<const uint8_t *>(src[i]), static_cast<uint8_t *>(dst[i]), nbytes[i]};
    CK(cudaMemcpyAsync(c->ops_dev, ops.data(), n * sizeof(kvmret::CopyOp), cudaMemcpyHostToDevice,
                       c->st));
    CK(kvmret::launch_copy_ops(c->ops_dev, n, c->st));
    return KVMRET_OK;
}

int kvmret_table_create(const kvmret_config *cfg, kvmret_table **out) {
    if (!cfg || !out) return fail(KVMRET_ERR_ARG, "null argument");
    GUARD(*out = new kvmret_table(table_config(*cfg)));
    return KVMRET_OK;
}
void kvmret_table_destroy(kvmret_table *t) { delete t; }
int kvmret_table_append(kvmret_table *t, uint32_t n) {
    if (!t) return fail(KVMRET_ERR_ARG, "null table");
    GUARD(t->t.append(n));
    return KVMRET_OK;
}
uint32_t kvmret_table_n_blocks(kvmret_table *t) { return t ? t->t.n_blocks() : 0; }

int kvmret_table_keep(kvmret_table *t, const uint32_t *mandatory, uint32_t n_mand,
                      uint8_t *kept_out, uint32_t *kept_count, uint32_t *need) {
    if (!t || (n_mand && !mandatory)) return fail(KVMRET_ERR_ARG, "null argument");
    std::vector<uint8_t> kept;
    uint32_t kc = 0, nd = 0;
    GUARD(nd = t->t.keep(mandatory, n_mand, kept, kc));
    if (kept_out) std::copy(kept.begin(), kept.end(), kept_out);
    if (kept_count) *kept_count = kc;
    if (need) *need = nd;
    return KVMRET_OK;
}

int kvmret_table_truncate(kvmret_table *t, uint32_t n_tokens) {
    if (!t) return fail(KVMRET_ERR_ARG, "null argument");
    GUARD(t->t.truncate(n_tokens));
    return KVMRET_OK;
}

int kvmret_table_set_on_gpu(kvmret_table *t, uint32_t block_id) {
    if (!t) return fail(KVMRET_ERR_ARG, "null argument");
    t->t.set_on_gpu(block_id);
    return KVMRET_OK;
}

int kvmret_table_clear_working_set(kvmret_table *t, int drop_gpu) {
    if (!t) return fail(KVMRET_ERR_ARG, "null argument");
    GUARD(t->t.clear_working_set(drop_gpu != 0));
    return KVMRET_OK;
}

int kvmret_table_set_selection(kvmret_table *t, const uint32_t *ids, uint32_t n_ids,
                               int force_raw, uint32_t *stage_in, uint32_t *stage_out,
                               int32_t *remaps, uint32_t *counts) {
    if (!t || (n_ids && !ids)) return fail(KVMRET_ERR_ARG, "null argument");
    kvmret::Plan p;
    GUARD(p = t->t.set_selection(ids, n_ids, force_raw != 0));
    if (stage_in) std::copy(p.stage_in.begin(), p.stage_in.end(), stage_in);
    if (stage_out) std::copy(p.stage_out.begin(), p.stage_out.end(), stage_out);
    if (remaps)
        for (size_t i = 0; i < p.remaps.size(); ++i) {
            const auto &r = p.remaps[i];
            int32_t *o = remaps + 7 * i;
            o[0] = static_cast<int32_t>(r.id);
            o[1] = static_cast<int32_t>(r.n_tok);
            o[2] = r.from;
            o[3] = r.to;
            o[4] = r.resident;
            o[5] = r.skip;
            o[6] = r.raw;
        }
    if (counts) {
        counts[0] = static_cast<uint32_t>(p.stage_in.size());
        counts[1] = static_cast<uint32_t>(p.stage_out.size());
        counts[2] = static_cast<uint32_t>(p.remaps.size());
        counts[3] = p.window_tokens;
        counts[4] = p.overlap;
        counts[5] = p.reused;
    }
    return KVMRET_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Prefill scoring (an extension of score_retrieval, which scores the mean
// query of a span, llama-memory-kvmem.cpp:4149-4196): every token of a chunk
// against every block, per-token top-k, union.

int kvmret_gemm_f16_nt(const uint16_t *a, const uint16_t *b, float *c, uint32_t m, uint32_t n,
                       uint32_t k, float alpha, uint32_t *err, void *stream) {
    if (!a || !b || !c) return fail(KVMRET_ERR_ARG, "null operand");
    // the epilogue writes C with 16-byte vector stores
    if (reinterpret_cast<uintptr_t>(c) & 15)
        return fail(KVMRET_ERR_ARG, "gemm output must be 16-byte aligned");
    if (m == 0 || m % 128 || n == 0 || n % 16 || k % 64 || k == 0)
        return fail(KVMRET_ERR_ARG, "gemm needs m %% 128 == 0, n %% 16 == 0, k %% 64 == 0");
    CUtensorMap ma, mb;
    CK(kvmret::make_gemm_maps(a, b, m, n, k, &ma, &mb));
    CK(kvmret::launch_gemm_f16_nt(ma, mb, c, m, n, k, alpha, err,
                                  static_cast<cudaStream_t>(stream)));
    return KVMRET_OK;
}

size_t kvmret_gemm_ws_bytes(uint32_t m, uint32_t n, uint32_t k) {
    return kvmret::gemm_ws_bytes(m, n, k);
}

int kvmret_gemm_f16_nt_ws(const uint16_t *a, const uint16_t *b, float *c, uint32_t m, uint32_t n,
                          uint32_t k, float alpha, uint32_t *err, float *ws, size_t ws_bytes,
                          void *stream) {
    if (!a || !b || !c) return fail(KVMRET_ERR_ARG, "null operand");
    if ((reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(ws)) & 15)
        return fail(KVMRET_ERR_ARG, "gemm output and workspace must be 16-byte aligned");
    if (m == 0 || m % 128 || n == 0 || n % 16 || k % 64 || k == 0)
        return fail(KVMRET_ERR_ARG, "gemm needs m %% 128 == 0, n %% 16 == 0, k %% 64 == 0");
    const size_t need = kvmret::gemm_ws_bytes(m, n, k);
    if (need && (!ws || ws_bytes < need))
        return fail(KVMRET_ERR_ARG, "gemm workspace of %zu bytes, %zu needed", ws_bytes, need);
    CUtensorMap ma, mb;
    CK(kvmret::make_gemm_maps(a, b, m, n, k, &ma, &mb));
    CK(kvmret::launch_gemm_f16_nt(ma, mb, c, m, n, k, alpha, err,
                                  static_cast<cudaStream_t>(stream), ws, ws_bytes));
    return KVMRET_OK;
}

int kvmret_prefill_score(kvmret_ctx *c, const uint16_t *q, uint32_t n_tok, uint32_t top_k,
                         uint8_t *sel, float *scores, uint32_t *n_sel_out) {
    NEED_CTX(c);
    if (!q || !sel || n_tok == 0 || top_k == 0)
        return fail(KVMRET_ERR_ARG, "prefill scoring needs q, sel, n_tok > 0, top_k > 0");
    const uint32_t L = c->cfg.n_layer, Hkv = c->cfg.n_head_kv, D = c->cfg.d_head;
    const uint32_t nb = c->live_blocks();
    CK(cudaMemsetAsync(sel, 0, c->cfg.max_blocks, c->st));
    if (nb == 0) {
        if (n_sel_out) *n_sel_out = 0;
        return KVMRET_OK;
    }
    const uint64_t K = static_cast<uint64_t>(L) * Hkv * D;
    if (K % 64 || K > (1ull << 31)) return fail(KVMRET_ERR_ARG, "prefill K = %llu unsupported",
                                               (unsigned long long)K);
    const uint32_t rows = (n_tok + 127) / 128 * 128;
    const uint32_t nrows = (c->ncap + 255) / 256 * 256;
    if (!c->pf_b) {
        TRY(dmalloc(&c->pf_b, static_cast<size_t>(nrows) * K * 2));
        CK(cudaMemsetAsync(c->pf_b, 0, static_cast<size_t>(nrows) * K * 2, c->st));
        TRY(dmalloc(&c->pf_err, 16));
        CK(cudaMemsetAsync(c->pf_err, 0, 16, c->st));
        c->pf_nrows = nrows;
        c->mhat_valid = 0;
    }
    if (c->pf_rows < rows) {
        if (c->pf_a) cudaFree(c->pf_a);
        if (c->pf_s) cudaFree(c->pf_s);
        c->pf_a = nullptr;
        c->pf_s = nullptr;
        c->pf_rows = 0;
        TRY(dmalloc(&c->pf_a, static_cast<size_t>(rows) * K * 2));
        TRY(dmalloc(&c->pf_s, static_cast<size_t>(rows) * nrows * sizeof(float)));
        CK(cudaMemsetAsync(c->pf_a, 0, static_cast<size_t>(rows) * K * 2, c->st));
        c->pf_rows = rows;
    }
    const uint32_t n_used = (nb + 15) / 16 * 16;  // C's row length (a multiple of 16)
    CK(kvmret::launch_mhat(c->summ, c->pf_b, L, Hkv, D, c->ncap, c->mhat_valid, nb, K, c->st));
    c->mhat_valid = nb;
    CK(kvmret::launch_qhat(q, c->pf_a, L, n_tok, c->cfg.n_head, Hkv, D, K, c->st));
    CUtensorMap ma, mb;
    CK(kvmret::make_gemm_maps(c->pf_a, c->pf_b, rows, n_used, static_cast<uint32_t>(K), &ma,
                              &mb));
    // the pipeline-timeout word reports on this launch only
    CK(cudaMemsetAsync(c->pf_err, 0, sizeof(uint32_t), c->st));
    const int pr = prof_begin(c, c->st, PR_GEMM);
    const size_t ws_need = kvmret::gemm_ws_bytes(rows, n_used, static_cast<uint32_t>(K));
    if (ws_need > c->pf_ws_bytes) {  // the split form's partial tiles
        if (c->pf_ws) cudaFree(c->pf_ws);
        c->pf_ws = nullptr;
        c->pf_ws_bytes = 0;
        TRY(dmalloc(&c->pf_ws, ws_need));
        c->pf_ws_bytes = ws_need;
    }
    CK(kvmret::launch_gemm_f16_nt(ma, mb, c->pf_s, rows, n_used, static_cast<uint32_t>(K),
                                  1.0f / static_cast<float>(L * Hkv), c->pf_err, c->st,
                                  c->pf_ws, c->pf_ws_bytes));
    prof_end(c, c->st, pr);
    if (c->prof_on) c->prof.gemm_flops += 2.0 * n_tok * nb * static_cast<double>(K);
    CK(kvmret::launch_topk_union(c->pf_s, n_used, n_tok, nb, top_k, c->cfg.tie_higher_id, sel,
                                 c->st));
    c->prof.launches += 4;
    if (scores)
        CK(cudaMemcpy2DAsync(scores, static_cast<size_t>(nb) * sizeof(float), c->pf_s,
                             static_cast<size_t>(n_used) * sizeof(float), nb * sizeof(float),
                             n_tok, cudaMemcpyDeviceToDevice, c->st));
    if (n_sel_out) {
        std::vector<uint8_t> h(nb);
        uint32_t err = 0;
        CK(cudaMemcpyAsync(h.data(), sel, nb, cudaMemcpyDeviceToHost, c->st));
        CK(cudaMemcpyAsync(&err, c->pf_err, sizeof(err), cudaMemcpyDeviceToHost, c->st));
        CK(cudaStreamSynchronize(c->st));
        if (err) return fail(KVMRET_ERR_CUDA, "tensor-core GEMM gave up waiting (pipeline stall)");
        uint32_t n = 0;
        for (uint8_t f : h) n += f != 0;
        *n_sel_out = n;
    }
    return KVMRET_OK;
}

// ---------------------------------------------------------------------------
// Session lanes (config 5): one context per lane on the same device, stepped
// together. Each lane's kernels run on its own stream, forked from and joined
// to the caller's stream, so the lanes' scoring and window assembly overlap
// on the GPU; the lanes' score terms share one exchange buffer, so a
// layer-sharded group needs one collective per step for all lanes.

struct kvmret_lanes {
    std::vector<kvmret_ctx *> ctx;
    uint32_t L_local = 0, cstride = 0;
    cudaEvent_t fork = nullptr;
    std::vector<cudaEvent_t> join;
    double *scratch = nullptr;  // per lane [n_ranks * L_local][cstride], gathered rows
    uint64_t scratch_rows = 0;
};

namespace {

void lanes_free(kvmret_lanes *g) {
    if (!g) return;
    DeviceScope ds;
    if (!g->ctx.empty()) ds.enter(g->ctx[0]->cfg.device);
    for (kvmret_ctx *c : g->ctx) cudaStreamSynchronize(c->st);
    if (g->scratch) cudaFree(g->scratch);
    if (g->fork) cudaEventDestroy(g->fork);
    for (cudaEvent_t e : g->join)
        if (e) cudaEventDestroy(e);
    delete g;
}

// fork: every lane stream waits for the caller's stream
int lanes_fork(kvmret_lanes *g, cudaStream_t caller) {
    CK(cudaEventRecord(g->fork, caller));
    for (kvmret_ctx *c : g->ctx) CK(cudaStreamWaitEvent(c->st, g->fork, 0));
    return KVMRET_OK;
}
// join: the caller's stream waits for every lane stream
int lanes_join(kvmret_lanes *g, cudaStream_t caller) {
    for (size_t i = 0; i < g->ctx.size(); ++i) {
        CK(cudaEventRecord(g->join[i], g->ctx[i]->st));
        CK(cudaStreamWaitEvent(caller, g->join[i], 0));
    }
    return KVMRET_OK;
}

}  // namespace

int kvmret_lanes_create(kvmret_ctx *const *lanes, uint32_t n, kvmret_lanes **out) {
    if (!lanes || n == 0 || !out) return fail(KVMRET_ERR_ARG, "need lanes and an output");
    *out = nullptr;
    for (uint32_t i = 0; i < n; ++i) {
        if (!lanes[i]) return fail(KVMRET_ERR_ARG, "lane %u is null", i);
        const kvmret_config &a = lanes[0]->cfg, &b = lanes[i]->cfg;
        if (a.device != b.device || a.n_layer != b.n_layer || lanes[i]->cstride != lanes[0]->cstride)
            return fail(KVMRET_ERR_ARG, "lane %u: device, layer count and block capacity must match",
                        i);
        for (uint32_t j = 0; j < i; ++j)
            if (lanes[j] == lanes[i]) return fail(KVMRET_ERR_ARG, "lane %u repeated", i);
    }
    kvmret_lanes *g = new (std::nothrow) kvmret_lanes;
    if (!g) return fail(KVMRET_ERR_NOMEM, "out of host memory");
    g->ctx.assign(lanes, lanes + n);
    g->L_local = lanes[0]->cfg.n_layer;
    g->cstride = lanes[0]->cstride;
    DeviceScope ds;
    ds.enter(lanes[0]->cfg.device);
    g->join.assign(n, nullptr);
    cudaError_t e = cudaEventCreateWithFlags(&g->fork, cudaEventDisableTiming);
    for (uint32_t i = 0; i < n && e == cudaSuccess; ++i)
        e = cudaEventCreateWithFlags(&g->join[i], cudaEventDisableTiming);
    if (e != cudaSuccess) {
        lanes_free(g);
        return fail(KVMRET_ERR_CUDA, "event creation failed: %s", cudaGetErrorString(e));
    }
    *out = g;
    return KVMRET_OK;
}

void kvmret_lanes_destroy(kvmret_lanes *g) { lanes_free(g); }

int kvmret_lanes_score_layers(kvmret_lanes *g, double *rows_out, void *stream) {
    if (!g || !rows_out) return fail(KVMRET_ERR_ARG, "bad lanes call");
    NEED_CTX(g->ctx[0]);
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    TRY(lanes_fork(g, caller));
    const uint64_t lane_rows = static_cast<uint64_t>(g->L_local) * g->cstride;
    for (size_t i = 0; i < g->ctx.size(); ++i)
        TRY(kvmret_score_layers(g->ctx[i], rows_out + i * lane_rows));
    return lanes_join(g, caller);
}

int kvmret_lanes_select_apply_async(kvmret_lanes *g, const double *rows_all, uint32_t n_ranks,
                                    const uint32_t *const *mandatory,
                                    const uint32_t *n_mandatory, void *stream) {
    if (!g || !rows_all || n_ranks == 0) return fail(KVMRET_ERR_ARG, "bad lanes call");
    NEED_CTX(g->ctx[0]);
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    const uint32_t n = static_cast<uint32_t>(g->ctx.size());
    const uint64_t lane_rows = static_cast<uint64_t>(g->L_local) * g->cstride;
    const uint64_t need = static_cast<uint64_t>(n) * n_ranks * lane_rows;
    if (n_ranks > 1 && g->scratch_rows < need) {
        if (g->scratch) cudaFree(g->scratch);
        g->scratch = nullptr;
        g->scratch_rows = 0;
        TRY(dmalloc(&g->scratch, need * sizeof(double)));
        g->scratch_rows = need;
    }
    TRY(lanes_fork(g, caller));
    for (uint32_t i = 0; i < n; ++i) {
        kvmret_ctx *c = g->ctx[i];
        const double *rows = rows_all + i * lane_rows;
        if (n_ranks > 1) {
            // rows_all is [rank][lane][L_local][cstride]: gather this lane's rows
            // of every rank into [rank * L_local][cstride] (global layer order)
            double *dst = g->scratch + static_cast<uint64_t>(i) * n_ranks * lane_rows;
            CK(cudaMemcpy2DAsync(dst, lane_rows * sizeof(double), rows,
                                 static_cast<size_t>(n) * lane_rows * sizeof(double),
                                 lane_rows * sizeof(double), n_ranks, cudaMemcpyDeviceToDevice,
                                 c->st));
            rows = dst;
        }
        TRY(kvmret_score_reduce(c, rows, n_ranks * g->L_local));
        const uint32_t nm = n_mandatory ? n_mandatory[i] : 0;
        TRY(kvmret_select_apply_async(c, nm && mandatory ? mandatory[i] : nullptr, nm));
    }
    return lanes_join(g, caller);
}

// ---------------------------------------------------------------------------
// Conversation stores (the reference's per-conversation host bundle, swapped
// under one GPU working set: llama_memory_kvmem::swap_conv / detach_conv /
// attach_conv, src/adapter/llama-memory-kvmem.cpp:1217-1714; C API
// llama_kvmem_store_create / _switch / _rows / _bytes / _destroy,
// src/adapter/llama-kvmem-hooks.h:107-151). A store owns one conversation's
// state: its pinned host repository, block table, block summaries (kept in
// HBM while parked, so the scorer never waits for them), running tail sum,
// per-block token counts and data flags, and query accumulator. The window
// and the HBM pool belong to the context and are shared by every store.

struct kvmret_store {
    int device = 0;
    float *summ = nullptr, *tail_sum = nullptr, *q_sum = nullptr;
    uint32_t *q_count_dev = nullptr, *d_blk_ntok = nullptr;
    uint8_t *has_block = nullptr;
    int32_t *d_blk_slot = nullptr;
    uint8_t *repo_host = nullptr, *repo_dev = nullptr;
    uint64_t repo_bytes = 0;
    kvmret::BlockTable table;
    kvmret::Plan last_plan;
    uint32_t live_tokens = 0;
    std::vector<uint32_t> q_count;
    bool q_reset_pending = true;
    bool gen_on = false;
    uint32_t gen_first = 0;
    std::vector<uint8_t> gen_bound;
    explicit kvmret_store(const kvmret::TableConfig &tc) : table(tc) {}
};

namespace {

void store_free(kvmret_store *s) {
    if (!s) return;
    DeviceScope ds;
    ds.enter(s->device);
    void *dev[] = {s->summ, s->tail_sum, s->q_sum, s->q_count_dev, s->d_blk_ntok,
                   s->has_block, s->d_blk_slot};
    for (void *p : dev)
        if (p) cudaFree(p);
    if (s->repo_host) cudaFreeHost(s->repo_host);
    delete s;
}

// The per-conversation members of a context and of a store change places.
void exchange_conversation(kvmret_ctx *c, kvmret_store *s) {
    std::swap(c->summ, s->summ);
    std::swap(c->tail_sum, s->tail_sum);
    std::swap(c->q_sum, s->q_sum);
    std::swap(c->q_count_dev, s->q_count_dev);
    std::swap(c->d_blk_ntok, s->d_blk_ntok);
    std::swap(c->has_block, s->has_block);
    std::swap(c->d_blk_slot, s->d_blk_slot);
    std::swap(c->repo_host, s->repo_host);
    std::swap(c->repo_dev, s->repo_dev);
    std::swap(c->table, s->table);
    std::swap(c->last_plan, s->last_plan);
    std::swap(c->live_tokens, s->live_tokens);
    std::swap(c->q_count, s->q_count);
    std::swap(c->q_reset_pending, s->q_reset_pending);
    std::swap(c->gen_on, s->gen_on);
    std::swap(c->gen_first, s->gen_first);
    std::swap(c->gen_bound, s->gen_bound);
}

}  // namespace

int kvmret_store_create(kvmret_ctx *c, kvmret_store **out) {
    NEED_CTX(c);
    if (!out) return fail(KVMRET_ERR_ARG, "null output");
    *out = nullptr;
    kvmret_store *s = new (std::nothrow) kvmret_store(table_config(c->cfg));
    if (!s) return fail(KVMRET_ERR_NOMEM, "out of host memory");
    s->device = c->cfg.device;
    const size_t L = c->cfg.n_layer, E = c->E;
    int rc = KVMRET_OK;
    auto run = [&]() -> int {
        TRY(dmalloc(&s->summ, L * E * c->ncap * sizeof(float)));
        TRY(dmalloc(&s->tail_sum, 2 * L * E * sizeof(float)));
        TRY(dmalloc(&s->q_sum, L * c->qdim * sizeof(float)));
        TRY(dmalloc(&s->q_count_dev, L * sizeof(uint32_t)));
        TRY(dmalloc(&s->d_blk_ntok, c->ncap * sizeof(uint32_t)));
        TRY(dmalloc(&s->has_block, c->ncap));
        TRY(dmalloc(&s->d_blk_slot, c->ncap * sizeof(int32_t)));
        CK(cudaMemsetAsync(s->summ, 0, L * E * c->ncap * sizeof(float), c->st));
        CK(cudaMemsetAsync(s->tail_sum, 0, 2 * L * E * sizeof(float), c->st));
        CK(cudaMemsetAsync(s->q_sum, 0, L * c->qdim * sizeof(float), c->st));
        CK(cudaMemsetAsync(s->q_count_dev, 0, L * sizeof(uint32_t), c->st));
        CK(cudaMemsetAsync(s->d_blk_ntok, 0, c->ncap * sizeof(uint32_t), c->st));
        CK(cudaMemsetAsync(s->has_block, 0, c->ncap, c->st));
        CK(cudaMemsetAsync(s->d_blk_slot, 0xff, c->ncap * sizeof(int32_t), c->st));
        s->repo_bytes = static_cast<uint64_t>(c->cfg.max_blocks) * c->slot_bytes;
        TRY(hmalloc_near(&s->repo_host, s->repo_bytes, cudaHostAllocMapped | cudaHostAllocPortable,
                         gpu_numa_node(c->cfg.device)));
        CK(cudaHostGetDevicePointer(reinterpret_cast<void **>(&s->repo_dev), s->repo_host, 0));
        s->q_count.assign(L, 0);
        s->gen_bound.assign(c->ncap, 0);
        CK(cudaStreamSynchronize(c->st));
        return KVMRET_OK;
    };
    try {
        rc = run();
    } catch (...) {
        rc = fail(KVMRET_ERR_NOMEM, "host allocation failed");
    }
    if (rc != KVMRET_OK) {
        const std::string keep = g_err;
        store_free(s);
        g_err = keep;
        return rc;
    }
    *out = s;
    return KVMRET_OK;
}

int kvmret_store_swap(kvmret_ctx *c, kvmret_store *s, int *restaged) {
    NEED_CTX(c);
    if (!s || s->device != c->cfg.device)
        return fail(KVMRET_ERR_ARG, "store made for another device or null");
    // quiesce: every step in flight collected, its selection replayed in the
    // outgoing store's table, and the stream drained
    GUARD(TRY(drain(c)));
    CK(cudaStreamSynchronize(c->st));
    GUARD(exchange_conversation(c, s));
    // the window and the pool held the outgoing conversation's blocks (its K
    // and V are already in its repository, written at append): empty both
    const size_t W = c->win_slots, P = c->pool_slots;
    CK(cudaMemsetAsync(c->d_win_id, 0xff, W * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_win_base, 0, W * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_win_ntok, 0, W * sizeof(uint32_t), c->st));
    CK(cudaMemsetAsync(c->d_slot_blk, 0xff, P * sizeof(int32_t), c->st));
    CK(cudaMemsetAsync(c->d_slot_ntok, 0, P * sizeof(uint32_t), c->st));
    CK(cudaMemsetAsync(c->d_slot_used, 0, P * sizeof(uint32_t), c->st));
    CK(cudaMemsetAsync(c->d_blk_slot, 0xff, c->ncap * sizeof(int32_t), c->st));
    c->kept_valid = false;
    c->q_dirty = true;
    c->mhat_valid = 0;
    c->deferred.clear();
    GUARD(std::fill(c->gen_bound.begin(), c->gen_bound.end(), 0));
    // the incoming store's working set is staged back into the window from its
    // repository (the reference's attach rebuilds it from host RAM)
    std::vector<uint32_t> ws;
    GUARD(for (uint32_t b = 0; b < c->table.n_blocks(); ++b) if (c->table.blocks()[b].in_ws)
              ws.push_back(b));
    if (!ws.empty()) {
        kvmret_step_stats st{};
        GUARD(TRY(apply_impl(c, ws.data(), static_cast<uint32_t>(ws.size()), &st)));
    }
    if (restaged) *restaged = ws.empty() ? 0 : 1;
    return KVMRET_OK;
}

uint32_t kvmret_store_rows(const kvmret_store *s) { return s ? s->live_tokens : 0; }

uint64_t kvmret_store_bytes(const kvmret_store *s) {
    return s ? s->repo_bytes : 0;
}

void kvmret_store_destroy(kvmret_store *s) { store_free(s); }

// ---------------------------------------------------------------------------
// Repository blocks to and from the NVMe raw tier.

int kvmret_repo_spill(kvmret_ctx *c, kvmret_nvme *t, const uint32_t *blocks, uint32_t n,
                      kvmret_nvme_stats *stats) {
    NEED_CTX(c);
    if (!t || (n && !blocks)) return fail(KVMRET_ERR_ARG, "null argument");
    if (stats) std::memset(stats, 0, sizeof(*stats));
    GUARD(TRY(drain(c)));
    CK(cudaStreamSynchronize(c->st));  // appends write the repository from the GPU
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t b = blocks[i];
        if (b >= c->live_blocks()) return fail(KVMRET_ERR_ARG, "block %u is not stored", b);
        int32_t evicted = -1;
        const int32_t slot = kvmret_nvme_place(t, b, 1, &evicted);
        if (slot < 0) return fail(KVMRET_ERR_STATE, "NVMe tier has no slot for block %u", b);
        kvmret_nvme_span sp{slot, 0, 0, c->slot_bytes};
        kvmret_nvme_stats st{};
        // one span at the block's own offset in the repository
        sp.buffer_offset = static_cast<uint64_t>(b) * c->slot_bytes;
        TRY(kvmret_nvme_write_spans(t, &sp, 1, c->repo_host,
                                    static_cast<uint64_t>(c->cfg.max_blocks) * c->slot_bytes, &st));
        if (stats) {
            stats->bytes += st.bytes;
            stats->syscalls += st.syscalls;
            stats->direct_bytes += st.direct_bytes;
            stats->cache_drop_bytes += st.cache_drop_bytes;
            stats->cache_drop_failures += st.cache_drop_failures;
        }
    }
    return KVMRET_OK;
}

int kvmret_repo_fill(kvmret_ctx *c, kvmret_nvme *t, const uint32_t *blocks, uint32_t n,
                     kvmret_nvme_stats *stats) {
    NEED_CTX(c);
    if (!t || (n && !blocks)) return fail(KVMRET_ERR_ARG, "null argument");
    if (stats) std::memset(stats, 0, sizeof(*stats));
    // no step in flight may be reading the repository while it is rewritten
    GUARD(TRY(drain(c)));
    CK(cudaStreamSynchronize(c->st));
    std::vector<kvmret_nvme_span> spans;
    GUARD(spans.reserve(n));
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t b = blocks[i];
        if (b >= c->live_blocks()) return fail(KVMRET_ERR_ARG, "block %u is not stored", b);
        const int32_t slot = kvmret_nvme_block_slot(t, b);
        if (slot < 0) return fail(KVMRET_ERR_STATE, "block %u is not on the NVMe tier", b);
        GUARD(spans.push_back({slot, 0, static_cast<uint64_t>(b) * c->slot_bytes, c->slot_bytes}));
        kvmret_nvme_touch(t, b);
    }
    return kvmret_nvme_read_spans(t, spans.data(), n, c->repo_host,
                                  static_cast<uint64_t>(c->cfg.max_blocks) * c->slot_bytes, stats);
}

// ---------------------------------------------------------------------------
// Snapshot archive (the reference's RawKvStore stream).

namespace {

constexpr uint32_t kSnapMagic = 0x31564b52u;
constexpr uint64_t kFnvOffset = 14695981039346656037ull, kFnvPrime = 1099511628211ull;

struct SnapOut {
    uint8_t *buf;
    uint64_t cap, len = 0, hash = kFnvOffset;
    bool hashing, overflow = false;
    void put(const void *p, uint64_t n) {
        const uint8_t *b = static_cast<const uint8_t *>(p);
        if (buf) {
            if (len + n > cap) overflow = true;
            else std::memcpy(buf + len, b, n);
        }
        if (hashing)
            for (uint64_t i = 0; i < n; ++i) hash = (hash ^ b[i]) * kFnvPrime;
        len += n;
    }
    void zeros(uint64_t n) {
        static const uint8_t z[4096] = {};
        while (n) {
            const uint64_t k = std::min<uint64_t>(n, sizeof(z));
            put(z, k);
            n -= k;
        }
    }
    template <typename T> void scalar(T v) { put(&v, sizeof(v)); }
};

struct SnapIn {
    const uint8_t *p;
    uint64_t left, hash = kFnvOffset;
    bool hashing;
    bool read(void *dst, uint64_t n) {
        if (n > left) return false;
        if (dst) std::memcpy(dst, p, n);
        if (hashing)
            for (uint64_t i = 0; i < n; ++i) hash = (hash ^ p[i]) * kFnvPrime;
        p += n;
        left -= n;
        return true;
    }
    template <typename T> bool scalar(T &v) { return read(&v, sizeof(v)); }
};

}  // namespace

int kvmret_snapshot_write(kvmret_ctx *c, void *buf, uint64_t cap, uint64_t *len,
                          uint64_t *hash) {
    NEED_CTX(c);
    if (!len) return fail(KVMRET_ERR_ARG, "null length");
    GUARD(TRY(drain(c)));
    CK(cudaStreamSynchronize(c->st));
    const uint32_t L = c->cfg.n_layer, E = c->E, T = c->cfg.block_tokens;
    const uint32_t nb = c->live_blocks();
    const bool f16 = c->cfg.k_type == KVMRET_TYPE_F16;
    // quantised K keeps no f16 rows: full blocks export their summary (with
    // mean_tokens 1), the partial newest block its running sum
    std::vector<float> summ, tail;
    if (!f16 && buf && nb) {
        GUARD(summ.resize(static_cast<size_t>(L) * E * c->ncap));
        GUARD(tail.resize(static_cast<size_t>(L) * E));
        CK(cudaMemcpy(summ.data(), c->summ, summ.size() * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(tail.data(), c->tail_sum, tail.size() * 4, cudaMemcpyDeviceToHost));
    }
    SnapOut o{static_cast<uint8_t *>(buf), cap};
    o.hashing = hash != nullptr && buf != nullptr;
    o.scalar(kSnapMagic);
    o.scalar(L);
    o.scalar(E);
    o.scalar(E);
    o.scalar(T);
    o.scalar<uint64_t>(f16 ? 0 : c->k_row);
    o.scalar<uint64_t>(0);
    o.scalar<uint64_t>(c->v_row);
    o.scalar<uint64_t>(nb);
    const uint64_t kb = static_cast<uint64_t>(T) * c->k_row, vb = static_cast<uint64_t>(T) * c->v_row;
    const uint64_t layer_bytes = 4 * 4 + 2 + 5 * 8 + kb + vb + static_cast<uint64_t>(E) * 4;
    std::vector<float> sum;
    GUARD(sum.resize(E));
    for (uint32_t b = 0; b < nb; ++b) {
        o.scalar<uint64_t>(layer_bytes * L);
        const uint32_t n = std::min(T, c->live_tokens - b * T);
        for (uint32_t l = 0; l < L; ++l) {
            const uint8_t *unit = c->repo_host + (static_cast<uint64_t>(b) * L + l) * c->unit;
            const uint32_t mean_tokens = f16 ? n : (n == T ? 1u : n);
            o.scalar(n);
            o.scalar<uint32_t>(0);
            o.scalar(n);
            o.scalar(mean_tokens);
            o.scalar<uint8_t>(0);
            o.scalar<uint8_t>(1);
            o.scalar<uint64_t>(kb);  // k: block_tokens unrotated rows
            o.put(unit, static_cast<uint64_t>(n) * c->k_row);
            o.zeros(kb - static_cast<uint64_t>(n) * c->k_row);
            o.scalar<uint64_t>(0);   // v
            o.scalar<uint64_t>(0);   // k_gpu
            o.scalar<uint64_t>(vb);  // v_gpu
            o.put(unit + c->unit_k, static_cast<uint64_t>(n) * c->v_row);
            o.zeros(vb - static_cast<uint64_t>(n) * c->v_row);
            o.scalar<uint64_t>(E);   // k_sum
            if (!buf) {
                o.len += static_cast<uint64_t>(E) * 4;
                continue;
            }
            if (f16) {  // the token-order f32 sum of the stored f16 rows
                const uint16_t *k = reinterpret_cast<const uint16_t *>(unit);
                std::fill(sum.begin(), sum.end(), 0.0f);
                for (uint32_t t = 0; t < n; ++t)
                    for (uint32_t e = 0; e < E; ++e) {
                        __half_raw hr;
                        hr.x = k[static_cast<size_t>(t) * E + e];
                        sum[e] += __half2float(__half(hr));
                    }
            } else {
                for (uint32_t e = 0; e < E; ++e)
                    sum[e] = n == T ? summ[(static_cast<size_t>(l) * E + e) * c->ncap + b]
                                    : tail[static_cast<size_t>(l) * E + e];
            }
            o.put(sum.data(), static_cast<uint64_t>(E) * 4);
        }
    }
    *len = o.len;
    if (buf && o.overflow)
        return fail(KVMRET_ERR_ARG, "snapshot of %llu bytes exceeds the %llu-byte buffer",
                    (unsigned long long)o.len, (unsigned long long)cap);
    if (hash) *hash = o.hash;
    return KVMRET_OK;
}

int kvmret_snapshot_read(kvmret_ctx *c, const void *buf, uint64_t len, uint64_t *hash) {
    NEED_CTX(c);
    if (!buf) return fail(KVMRET_ERR_ARG, "null buffer");
    if (c->live_tokens) return fail(KVMRET_ERR_STATE, "snapshot read needs an empty context");
    GUARD(TRY(drain(c)));
    CK(cudaStreamSynchronize(c->st));
    const uint32_t L = c->cfg.n_layer, E = c->E, T = c->cfg.block_tokens;
    const bool f16 = c->cfg.k_type == KVMRET_TYPE_F16;
    SnapIn in{static_cast<const uint8_t *>(buf), len};
    in.hashing = hash != nullptr;
    uint32_t u32[5];
    uint64_t u64[4];
    for (uint32_t &x : u32)
        if (!in.scalar(x)) return fail(KVMRET_ERR_ARG, "truncated snapshot");
    for (uint64_t &x : u64)
        if (!in.scalar(x)) return fail(KVMRET_ERR_ARG, "truncated snapshot");
    if (u32[0] != kSnapMagic || u32[1] != L || u32[2] != E || u32[3] != E || u32[4] != T ||
        u64[0] != (f16 ? 0 : c->k_row) || u64[1] != 0 || u64[2] != c->v_row)
        return fail(KVMRET_ERR_ARG, "snapshot made with another geometry");
    const uint64_t nb = u64[3];
    if (nb > c->cfg.max_blocks)
        return fail(KVMRET_ERR_ARG, "snapshot holds %llu blocks, capacity %u",
                    (unsigned long long)nb, c->cfg.max_blocks);
    std::vector<float> summ, tail;
    std::vector<uint32_t> ntok;
    std::vector<uint8_t> has;
    GUARD(summ.assign(static_cast<size_t>(L) * E * c->ncap, 0.0f));
    GUARD(tail.assign(static_cast<size_t>(L) * E, 0.0f));
    GUARD(ntok.assign(c->ncap, 0));
    GUARD(has.assign(c->ncap, 0));
    std::vector<float> ks;
    GUARD(ks.resize(E));
    uint32_t total = 0;
    for (uint64_t b = 0; b < nb; ++b) {
        uint64_t size = 0;
        if (!in.scalar(size) || size > in.left) return fail(KVMRET_ERR_ARG, "truncated snapshot");
        const uint64_t before = in.left;
        uint32_t n_blk = 0;
        bool blk_has = true;
        for (uint32_t l = 0; l < L; ++l) {
            uint32_t n, kgt, vgt, mt;
            uint8_t kf, vf;
            if (!in.scalar(n) || !in.scalar(kgt) || !in.scalar(vgt) || !in.scalar(mt) ||
                !in.scalar(kf) || !in.scalar(vf))
                return fail(KVMRET_ERR_ARG, "truncated snapshot");
            if (std::max({n, kgt, vgt, mt}) > T || kf > 1 || vf > 1 || kgt != 0 || vgt != n ||
                (l > 0 && n != n_blk) || n == 0)
                return fail(KVMRET_ERR_ARG, "snapshot block %llu: token counts this store "
                                            "cannot hold", (unsigned long long)b);
            n_blk = n;
            uint8_t *unit = c->repo_host + (b * L + l) * c->unit;
            uint64_t cnt = 0;
            // k: at least the block's rows, at most a block
            if (!in.scalar(cnt) || cnt < static_cast<uint64_t>(n) * c->k_row ||
                cnt > static_cast<uint64_t>(T) * c->k_row)
                return fail(KVMRET_ERR_ARG, "snapshot block %llu: bad K rows", (unsigned long long)b);
            if (!in.read(unit, static_cast<uint64_t>(n) * c->k_row) ||
                !in.read(nullptr, cnt - static_cast<uint64_t>(n) * c->k_row))
                return fail(KVMRET_ERR_ARG, "truncated snapshot");
            if (!in.scalar(cnt) || cnt != 0 || !in.scalar(cnt) || cnt != 0)
                return fail(KVMRET_ERR_ARG, "snapshot block %llu: host V or packed K rows this "
                                            "store does not keep", (unsigned long long)b);
            if (!in.scalar(cnt) || cnt < static_cast<uint64_t>(n) * c->v_row ||
                cnt > static_cast<uint64_t>(T) * c->v_row)
                return fail(KVMRET_ERR_ARG, "snapshot block %llu: bad V rows", (unsigned long long)b);
            if (!in.read(unit + c->unit_k, static_cast<uint64_t>(n) * c->v_row) ||
                !in.read(nullptr, cnt - static_cast<uint64_t>(n) * c->v_row))
                return fail(KVMRET_ERR_ARG, "truncated snapshot");
            if (!in.scalar(cnt) || (mt && cnt != E) || cnt > E)
                return fail(KVMRET_ERR_ARG, "snapshot block %llu: bad K sum", (unsigned long long)b);
            if (!in.read(cnt ? ks.data() : nullptr, cnt * 4))
                return fail(KVMRET_ERR_ARG, "truncated snapshot");
            if (mt) {  // mean = sum * (1 / mean_tokens), as the append computes it
                const float inv = 1.0f / static_cast<float>(mt);
                for (uint32_t e = 0; e < E; ++e)
                    summ[(static_cast<size_t>(l) * E + e) * c->ncap + b] = ks[e] * inv;
                if (n < T && mt == n)
                    std::copy(ks.begin(), ks.end(), tail.begin() + static_cast<size_t>(l) * E);
            } else {
                blk_has = false;
            }
        }
        if (before - in.left != size)
            return fail(KVMRET_ERR_ARG, "snapshot block %llu: section size mismatch",
                        (unsigned long long)b);
        if (b + 1 < nb && n_blk != T)
            return fail(KVMRET_ERR_ARG, "snapshot block %llu is partial but not the last",
                        (unsigned long long)b);
        ntok[b] = n_blk;
        has[b] = blk_has ? 1 : 0;
        total += n_blk;
    }
    if (in.left) return fail(KVMRET_ERR_ARG, "%llu trailing snapshot bytes",
                             (unsigned long long)in.left);
    CK(cudaMemcpy(c->summ, summ.data(), summ.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->tail_sum, tail.data(), tail.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->d_blk_ntok, ntok.data(), ntok.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->has_block, has.data(), has.size(), cudaMemcpyHostToDevice));
    GUARD(c->table.append(total));
    c->live_tokens = total;
    c->kept_valid = false;
    c->mhat_valid = 0;
    if (hash) *hash = in.hash;
    return KVMRET_OK;
}

// ---------------------------------------------------------------------------
// Layer-sharded exchange over NVLink peer memory: each rank's scoring kernel
// writes its rows straight into every rank's receive buffer and publishes a
// step flag; each rank's reduction waits for all flags (bounded) and reduces
// all layers in global order. No collective library is involved.

int kvmret_exchange_export(kvmret_ctx *c, uint32_t world, void *handle_out) {
    NEED_CTX(c);
    if (world < 2 || world > kvmret::kMaxRanks || !handle_out)
        return fail(KVMRET_ERR_ARG, "exchange needs 2..%d ranks and a handle buffer",
                    kvmret::kMaxRanks);
    if (c->ex_region) return fail(KVMRET_ERR_STATE, "exchange already set up");
    const uint64_t half = static_cast<uint64_t>(c->cfg.n_layer) * c->cstride;
    const uint64_t tail = align_up(2 * half * sizeof(double), 256);
    const uint64_t bytes = tail + 256;
    TRY(dmalloc(&c->ex_region, bytes));
    CK(cudaMemset(c->ex_region, 0, bytes));
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, c->ex_region));
    std::memcpy(handle_out, &h, sizeof(h));
    c->ex_half = half;
    c->ex_tail = tail;
    c->ex_world = world;
    return KVMRET_OK;
}

int kvmret_exchange_import(kvmret_ctx *c, uint32_t rank, uint32_t world, const void *handles) {
    NEED_CTX(c);
    if (!c->ex_region || world != c->ex_world || rank >= world || !handles)
        return fail(KVMRET_ERR_ARG, "export first, with the same rank count");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    for (uint32_t p = 0; p < world; ++p) {
        if (p == rank) {
            c->ex_peer[p] = c->ex_region;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + 64ull * p, sizeof(h));
        void *ptr = nullptr;
        CK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        c->ex_peer[p] = static_cast<uint8_t *>(ptr);
    }
    c->ex_rank = rank;
    return KVMRET_OK;
}

int kvmret_score_exchange(kvmret_ctx *c) {
    NEED_CTX(c);
    if (!c->ex_region || !c->ex_peer[c->ex_rank])
        return fail(KVMRET_ERR_STATE, "exchange not set up");
    const uint32_t W = c->ex_world, L = c->cfg.n_layer;
    const uint32_t step = ++c->ex_step;
    const uint64_t half_off = (step & 1u) * c->ex_half;
    double *local = reinterpret_cast<double *>(c->ex_region) + half_off;
    kvmret::Peers pr{};
    kvmret::RowSource rs{};
    for (uint32_t p = 0; p < W; ++p) {
        pr.flags[p] = reinterpret_cast<uint32_t *>(c->ex_peer[p] + c->ex_tail);
        rs.base[p] = reinterpret_cast<const double *>(c->ex_peer[p]) + half_off;
    }
    rs.l_local = L;
    rs.n_ranks = W;
    uint32_t *tail = reinterpret_cast<uint32_t *>(c->ex_region + c->ex_tail);
    pr.counter = tail + kvmret::kMaxRanks;
    pr.n = W;
    pr.rank = c->ex_rank;
    pr.step = step;
    pr.n_layer = L;
    // qprep writes the query flags into the local rows' last column; the
    // scoring kernel writes the terms beside them and signals every rank
    c->q_dirty = true;
    TRY(settle_query(c));
    CK(kvmret::launch_qprep(c->q_sum, c->q_count_dev, c->qv, c->nq, c->active, L, c->cfg.n_head,
                            c->cfg.n_head_kv, c->cfg.d_head, c->st, local, c->cstride));
    c->q_dirty = false;
    const uint32_t n = c->live_blocks();
    const int prs = prof_begin(c, c->st, PR_SCORE);
    CK(kvmret::launch_score(c->summ, c->qv, c->nq, c->active, local, L, c->cfg.n_head_kv,
                            c->cfg.d_head, c->ncap, n, c->st, c->cstride, &pr));
    prof_end(c, c->st, prs);
    c->prof.score_bytes += static_cast<uint64_t>(L) * c->E * ((n + 63) / 64 * 64) * sizeof(float);
    CK(kvmret::launch_reduce(nullptr, nullptr, W * L, c->cstride, c->has_block, n, c->scores,
                             c->st, tail, W, step, tail + kvmret::kMaxRanks + 1, &rs));
    c->prof.launches += 3;
    return KVMRET_OK;
}
