// Allocation-free scorer: kvmret_score_noalloc.
//
// For callers that cannot allocate device memory at all: code running where
// cudaMalloc is unavailable or forbidden (inside an allocator hook or a custom
// memory manager that owns every byte of the device, or a host that must not
// perform allocations on its serving path). They pass their own inputs and
// output; the scratch this scorer needs between its kernels (the prepared
// query, its norms, the per-layer query flags and the per-(layer, block)
// score terms) lives in one file-scope device array instead of memory from
// cudaMalloc.
//
// The array is KVMRET_NOALLOC_SCRATCH_BYTES (8 MiB) and every GPU that loads
// this library holds it until the process exits. Its device address is looked
// up once per device and CUDA context, with that device current, on the first
// call made in that context; make that first call before any CUDA stream
// capture begins. After cudaDeviceReset the device gets a new context and the
// next call looks the address up again (the module is loaded anew). All
// calls on a device share the array and it keeps the previous call's
// contents: every byte a call reads is written by the same call first, so
// nothing needs clearing, but two calls whose work overlaps on the GPU (for
// example on two streams) race on it.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "kernels.cuh"
#include "kvmret.h"

namespace kvmret {
int set_error(int code, const char *msg);  // context.cpp: feeds kvmret_last_error()
}

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KVMRET_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
// per device: the context the address was looked up in, and the address
struct ScratchEntry {
    void *ctx;
    void *ptr;
};
ScratchEntry g_scratch_dev[kMaxDevices] = {};

// cuCtxGetCurrent through the runtime's driver entry-point table (the library
// does not link the driver library itself).
typedef int (*CtxGetCurrentFn)(void **);
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<CtxGetCurrentFn>(nullptr);
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    return fn;
}

void *current_ctx() {
    void *ctx = nullptr;
    const CtxGetCurrentFn fn = ctx_get_current();
    if (!fn || fn(&ctx) != 0) return nullptr;
    return ctx;
}

int nerr(int code, const std::string &msg) { return kvmret::set_error(code, msg.c_str()); }

uint64_t up256(uint64_t v) { return (v + 255) / 256 * 256; }

// Device address of the scratch array on the current device.
int scratch_for_current_device(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return nerr(KVMRET_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return nerr(KVMRET_ERR_ARG, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    ScratchEntry &ent = g_scratch_dev[dev];
    void *ctx = ent.ptr ? current_ctx() : nullptr;
    if (!ent.ptr || !ctx || ctx != ent.ctx) {
        // first call in this context (or a context we cannot identify): look
        // the address up, which also makes the device's context current
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return nerr(KVMRET_ERR_CUDA,
                        std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
        ent.ptr = p;
        ent.ctx = current_ctx();
    }
    *out = ent.ptr;
    return KVMRET_OK;
}

}  // namespace

extern "C" int kvmret_score_noalloc(const float *summ_dev, uint32_t summ_stride,
                                    const float *q_sum_dev, const uint32_t *q_count_dev,
                                    const uint8_t *has_block_dev, uint32_t n_blocks,
                                    uint32_t n_layer, uint32_t n_head, uint32_t n_head_kv,
                                    uint32_t d_head, double *scores_dev, void *stream) {
    if (!summ_dev || !q_sum_dev || !q_count_dev || !has_block_dev || !scores_dev)
        return nerr(KVMRET_ERR_ARG, "null pointer argument");
    if (n_layer == 0 || n_head == 0 || n_head_kv == 0 || n_head % n_head_kv)
        return nerr(KVMRET_ERR_ARG, "bad head geometry");
    if (d_head != 64 && d_head != 128 && d_head != 256)
        return nerr(KVMRET_ERR_ARG, "d_head must be 64, 128 or 256");
    if (summ_stride % 64 || summ_stride < n_blocks || (reinterpret_cast<uintptr_t>(summ_dev) & 15))
        return nerr(KVMRET_ERR_ARG,
                    "summ_stride must be a multiple of 64 and >= n_blocks; summ_dev 16-byte aligned");
    const uint64_t b_contrib = up256(static_cast<uint64_t>(n_layer) * summ_stride * sizeof(double));
    const uint64_t b_qv = up256(static_cast<uint64_t>(n_layer) * n_head_kv * d_head * sizeof(float));
    const uint64_t b_nq = up256(static_cast<uint64_t>(n_layer) * n_head_kv * sizeof(float));
    const uint64_t b_act = up256(n_layer);
    const uint64_t need = b_contrib + b_qv + b_nq + b_act;
    if (need > KVMRET_NOALLOC_SCRATCH_BYTES) {
        char buf[200];
        snprintf(buf, sizeof(buf),
                 "scratch of %llu bytes needed (n_layer %u x stride %u) exceeds the %u-byte limit",
                 static_cast<unsigned long long>(need), n_layer, summ_stride,
                 static_cast<unsigned>(KVMRET_NOALLOC_SCRATCH_BYTES));
        return nerr(KVMRET_ERR_ARG, buf);
    }
    void *base = nullptr;
    const int rc = scratch_for_current_device(&base);
    if (rc != KVMRET_OK) return rc;
    unsigned char *p = static_cast<unsigned char *>(base);
    double *contrib = reinterpret_cast<double *>(p);
    float *qv = reinterpret_cast<float *>(p + b_contrib);
    float *nq = reinterpret_cast<float *>(p + b_contrib + b_qv);
    uint8_t *active = p + b_contrib + b_qv + b_nq;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = kvmret::launch_qprep(q_sum_dev, q_count_dev, qv, nq, active, n_layer, n_head,
                                         n_head_kv, d_head, st);
    if (e == cudaSuccess)
        e = kvmret::launch_score(summ_dev, qv, nq, active, contrib, n_layer, n_head_kv, d_head,
                                 summ_stride, n_blocks, st);
    if (e == cudaSuccess)
        e = kvmret::launch_reduce(contrib, active, n_layer, summ_stride, has_block_dev, n_blocks,
                                  scores_dev, st);
    if (e != cudaSuccess) return nerr(KVMRET_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
    return KVMRET_OK;
}
