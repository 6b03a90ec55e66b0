// sm_100a kernels of the retrieval path. The file is compiled with
// -fmad=false and every floating-point operation whose rounding the reference
// fixes is written with an explicit _rn intrinsic, so no multiply-add is
// fused anywhere on this path.
#include "kernels.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>
#include <utility>

#include <cub/block/block_scan.cuh>

#include "kvmret.h"

namespace kvmret {
namespace {

// Programmatic dependent launch: the step's kernels are launched so that each
// may be scheduled while its predecessor on the stream drains; every such
// kernel calls dep_wait() (griddepcontrol.wait) before it reads anything its
// predecessors wrote, which returns once they have completed and their writes
// are visible.
template <typename... KArgs, typename... Args>
cudaError_t launch_dep(void (*kfn)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, std::forward<Args>(args)...);
}

__device__ __forceinline__ void dep_wait() { cudaGridDependencySynchronize(); }


__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f2h(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

// ---------------------------------------------------------------------------
// S1: q_sum += rows, row order (llama-memory-kvmem.cpp:3417-3432); with
// assign, q_sum = the rows' sum (a reset folded into the first add).
template <typename T>
__global__ void query_add_kernel(float *__restrict__ q_sum, const T *__restrict__ rows,
                                 uint32_t n_rows, uint32_t qdim, uint32_t *__restrict__ q_count,
                                 int assign) {
    dep_wait();
    const uint32_t l = blockIdx.y;
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    // the row count lives on the device; assign = the first add after a reset
    if (q_count && blockIdx.x == 0 && threadIdx.x == 0)
        q_count[l] = assign ? n_rows : q_count[l] + n_rows;
    if (e >= qdim) return;
    float s = assign ? 0.0f : q_sum[static_cast<size_t>(l) * qdim + e];
    const T *src = rows + static_cast<size_t>(l) * n_rows * qdim + e;
    for (uint32_t r = 0; r < n_rows; ++r) {
        float v;
        if constexpr (sizeof(T) == 2) v = h2f(src[static_cast<size_t>(r) * qdim]);
        else v = src[static_cast<size_t>(r) * qdim];
        s = __fadd_rn(s, v);
    }
    q_sum[static_cast<size_t>(l) * qdim + e] = s;
}

// ---------------------------------------------------------------------------
// S3 prologue (score_retrieval :4162-4185, hoisted): for each (layer, kv head)
// qv[d] = (sum over the group's heads of q_sum, in head order) * invq and
// nq = sequential sum of qv*qv. Both depend only on the query, so the
// per-block loop of the reference recomputes the same values.
__global__ void qprep_kernel(const float *__restrict__ q_sum, const uint32_t *__restrict__ q_count,
                             float *__restrict__ qv, float *__restrict__ nq,
                             uint8_t *__restrict__ active, uint32_t n_head, uint32_t n_head_kv,
                             uint32_t d_head, double *__restrict__ flag_col, uint32_t cstride) {
    dep_wait();
    extern __shared__ float sv[];
    const uint32_t l = blockIdx.x, h = blockIdx.y;
    const uint32_t g = n_head_kv == 0 ? 1 : n_head / n_head_kv;
    const uint32_t cnt = q_count[l];
    const float invq = __fdiv_rn(1.0f, static_cast<float>(cnt * (g > 1u ? g : 1u)));
    const float *qs = q_sum + static_cast<size_t>(l) * n_head * d_head;
    for (uint32_t d = threadIdx.x; d < d_head; d += blockDim.x) {
        float s = 0.0f;
        for (uint32_t gi = 0; gi < g; ++gi) {
            const uint32_t qh = h * g + gi;
            if (qh >= n_head) break;
            s = __fadd_rn(s, qs[static_cast<size_t>(qh) * d_head + d]);
        }
        const float v = __fmul_rn(s, invq);
        sv[d] = v;
        qv[(static_cast<size_t>(l) * n_head_kv + h) * d_head + d] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (uint32_t d = 0; d < d_head; ++d) a = __fadd_rn(a, __fmul_rn(sv[d], sv[d]));
        nq[static_cast<size_t>(l) * n_head_kv + h] = a;
        if (h == 0) {
            active[l] = cnt != 0;
            // packed exchange form: the layer's query flag in the last column of its row
            if (flag_col) flag_col[static_cast<size_t>(l) * cstride + cstride - 1] = cnt ? 1.0 : 0.0;
        }
    }
}

// ---------------------------------------------------------------------------
// Exchange signal, run by every CTA of a scoring launch at its end (its rows,
// and the layer query flags qprep wrote in the rows' last column, are in this
// rank's own exchange region). A CTA's stores are ordered before its increment
// of the device counter (gpu-scope fence); the last CTA, having observed every
// increment, fences at system scope and publishes the step number in every
// rank's flag slot for this rank with a release store. A reader acquires the
// flag before it reads the rows over NVLink.
__device__ void exchange_signal(const Peers &peers) {
    __threadfence();
    __syncthreads();
    __shared__ uint32_t s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(peers.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        *peers.counter = 0;
        for (uint32_t p = 0; p < peers.n; ++p)
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.flags[p] + peers.rank),
                         "r"(peers.step)
                         : "memory");
    }
}

// The exchange signal alone, for a rank whose history holds no block yet: its
// peers still wait for this rank's step flag (and its layers' query flags).
__global__ void exchange_signal_kernel(const __grid_constant__ Peers peers) {
    dep_wait();
    exchange_signal(peers);
}

// ---------------------------------------------------------------------------
// S3: a unit = one layer x TILE blocks (64: lane j walks blocks 2j, 2j+1 with
// float2 loads; 32: one block per lane). Summaries are block-minor
// [L][Hkv][D][ncap], so each d step of a warp reads 256 (128) contiguous
// bytes, and each block's dot / norm is accumulated strictly in d order
// (score_retrieval :4179-4185). Warp w handles heads w, w + 8, ...; the
// per-layer head sum is taken in head order from shared memory.
// d-rows per batch of the 32-block form (two batches in flight per lane)
#ifndef KVMRET_SCORE_RB
#define KVMRET_SCORE_RB 16
#endif
template <int D, int V>
__global__ void __launch_bounds__(256) score_kernel(const float *__restrict__ summ,
                                                    const float *__restrict__ qv,
                                                    const float *__restrict__ nq,
                                                    const uint8_t *__restrict__ active,
                                                    double *__restrict__ contrib,
                                                    uint32_t n_head_kv, uint32_t ncap,
                                                    uint32_t cstride, uint32_t tiles,
                                                    uint32_t n_units, uint32_t per_cta,
                                                    const __grid_constant__ Peers peers) {
    dep_wait();
    constexpr uint32_t TILE = 32 * V;  // blocks per unit: V per lane
    using VecT = typename std::conditional<V == 2, float2, float>::type;
    extern __shared__ float smem[];
    float *sq = smem;                       // [Hkv][D]
    float *cosb = smem + n_head_kv * D;     // [Hkv][TILE]
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
    const size_t dstep = ncap / V;  // vector stride between d rows
    // units (layer, tile of TILE blocks), layer-major; this CTA's contiguous
    // share, so every CTA carries the same number of units
    const uint32_t u0 = blockIdx.x * per_cta, u1 = min(n_units, u0 + per_cta);
    uint32_t l_loaded = ~0u;
    for (uint32_t u = u0; u < u1; ++u) {
        const uint32_t l = u / tiles;
        const uint32_t b0 = (u % tiles) * TILE;
        double *out = contrib + static_cast<size_t>(l) * cstride + b0;
        if (!active[l]) {
            for (uint32_t t = threadIdx.x; t < TILE; t += blockDim.x) out[t] = 0.0;
            continue;
        }
        if (l != l_loaded) {
            __syncthreads();  // the previous unit's readers of sq are done
            for (uint32_t i = threadIdx.x; i < n_head_kv * D; i += blockDim.x)
                sq[i] = qv[static_cast<size_t>(l) * n_head_kv * D + i];
            l_loaded = l;
        }
        __syncthreads();
        for (uint32_t h = warp; h < n_head_kv; h += nwarp) {
            const VecT *p = reinterpret_cast<const VecT *>(
                                summ + (static_cast<size_t>(l) * n_head_kv + h) * D * ncap + b0) +
                            lane;
            const float *qh = sq + h * D;
            float d0 = 0.f, d1 = 0.f, n0 = 0.f, n1 = 0.f;
            if constexpr (V == 2) {  // bandwidth-bound form: 2 x 16 rows per batch
#pragma unroll 2
                for (int dd = 0; dd < D; dd += 16) {
                    float2 k[16];
#pragma unroll
                    for (int v = 0; v < 16; ++v)
                        k[v] = __ldg(p + static_cast<size_t>(dd + v) * dstep);
#pragma unroll
                    for (int v = 0; v < 16; ++v) {
                        const float q = qh[dd + v];
                        d0 = __fadd_rn(d0, __fmul_rn(q, k[v].x));
                        d1 = __fadd_rn(d1, __fmul_rn(q, k[v].y));
                        n0 = __fadd_rn(n0, __fmul_rn(k[v].x, k[v].x));
                        n1 = __fadd_rn(n1, __fmul_rn(k[v].y, k[v].y));
                    }
                }
            } else {
                // latency-bound form (few layers): the next 16 d rows are loaded
                // before the current ones are consumed (the compiler barrier
                // keeps the loads ahead of the dependent sums)
                constexpr int RB = KVMRET_SCORE_RB < D ? KVMRET_SCORE_RB : D;
                float cur[RB], nxt[RB];
#pragma unroll
                for (int v = 0; v < RB; ++v) cur[v] = __ldg(p + static_cast<size_t>(v) * dstep);
#pragma unroll 1
                for (int dd = 0; dd < D; dd += RB) {
                    if (dd + RB < D) {
#pragma unroll
                        for (int v = 0; v < RB; ++v)
                            nxt[v] = __ldg(p + static_cast<size_t>(dd + RB + v) * dstep);
                    }
                    asm volatile("" ::: "memory");
#pragma unroll
                    for (int v = 0; v < RB; ++v) {
                        const float q = qh[dd + v];
                        d0 = __fadd_rn(d0, __fmul_rn(q, cur[v]));
                        n0 = __fadd_rn(n0, __fmul_rn(cur[v], cur[v]));
                    }
#pragma unroll
                    for (int v = 0; v < RB; ++v) cur[v] = nxt[v];
                }
            }
            const float sn = __fsqrt_rn(nq[static_cast<size_t>(l) * n_head_kv + h]);
            float *cb = cosb + h * TILE + lane * V;
            cb[0] = __fdiv_rn(d0, __fadd_rn(__fmul_rn(sn, __fsqrt_rn(n0)), 1e-6f));
            if constexpr (V == 2)
                cb[1] = __fdiv_rn(d1, __fadd_rn(__fmul_rn(sn, __fsqrt_rn(n1)), 1e-6f));
        }
        __syncthreads();
        // layer += cos (double, head order); term = layer / n_head_kv (:4186-4188).
        for (uint32_t t = threadIdx.x; t < TILE; t += blockDim.x) {
            double layer = 0.0;
            for (uint32_t h = 0; h < n_head_kv; ++h)
                layer = __dadd_rn(layer, static_cast<double>(cosb[h * TILE + t]));
            out[t] = __ddiv_rn(layer, static_cast<double>(n_head_kv));
        }
    }
    if (peers.n > 1) exchange_signal(peers);
}

// S3 epilogue (:4189-4193): acc over layers in order, score = acc / nlay.
// Row of global layer g: local rows (L2-coherent loads), or a rank's row in
// its exchange region, read over NVLink with system-scope relaxed loads (after
// the acquire of that rank's step flag).
__device__ __forceinline__ double row_load(const double *contrib, const RowSource &rs,
                                           uint32_t g, uint32_t stride, uint32_t col) {
    if (rs.n_ranks == 0) return __ldcg(contrib + static_cast<size_t>(g) * stride + col);
    const uint32_t p = g / rs.l_local;
    const double *ptr = rs.base[p] + static_cast<size_t>(g - p * rs.l_local) * stride + col;
    double v;
    asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(ptr) : "memory");
    return v;
}

__global__ void __launch_bounds__(128)
    reduce_kernel(const double *__restrict__ contrib, const uint8_t *__restrict__ active,
                  uint32_t n_layer, uint32_t stride, const uint8_t *__restrict__ has_block,
                  uint32_t n_blocks, double *__restrict__ scores, const uint32_t *wait_flags,
                  uint32_t wait_n, uint32_t wait_step, uint32_t *err,
                  const __grid_constant__ RowSource rs) {
    dep_wait();
    if (wait_flags) {  // peer-memory exchange: every rank's rows of this step have landed
        if (threadIdx.x == 0) {
            uint64_t t0 = 0;
            for (uint32_t p = 0; p < wait_n; ++p) {
                for (uint32_t i = 0;; ++i) {
                    uint32_t v;
                    asm volatile("ld.acquire.sys.global.u32 %0, [%1];"
                                 : "=r"(v)
                                 : "l"(wait_flags + p)
                                 : "memory");
                    if (static_cast<int32_t>(v - wait_step) >= 0) break;
                    uint64_t now;
                    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(now));
                    if (i == 0) t0 = now;
                    if (now - t0 > 2000000000ull) {  // 2 s: a rank is gone
                        atomicExch(err, 1u);
                        break;
                    }
                    __nanosleep(200);
                }
            }
        }
        __syncthreads();
    }
    // the layers that carry a query, once per CTA
    extern __shared__ uint8_t s_act[];
    for (uint32_t l = threadIdx.x; l < n_layer; l += blockDim.x)
        s_act[l] = active ? active[l] : (row_load(contrib, rs, l, stride, stride - 1) != 0.0);
    __syncthreads();
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    if (!has_block[b]) {
        scores[b] = 0.0;
        return;
    }
    double acc = 0.0;
    uint32_t nlay = 0;
    // 16 rows per batch; the next batch's loads are issued before the current
    // one is summed, so each batch's latency (an NVLink round trip for a
    // peer's rows) overlaps the previous one
    double cur[16], nxt[16];
#pragma unroll
    for (uint32_t u = 0; u < 16; ++u)
        cur[u] = (u < n_layer && s_act[u]) ? row_load(contrib, rs, u, stride, b) : 0.0;
    for (uint32_t l0 = 0; l0 < n_layer; l0 += 16) {
        if (l0 + 16 < n_layer) {
#pragma unroll
            for (uint32_t u = 0; u < 16; ++u) {
                const uint32_t l = l0 + 16 + u;
                nxt[u] = (l < n_layer && s_act[l]) ? row_load(contrib, rs, l, stride, b) : 0.0;
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < 16; ++u) {  // summed strictly in layer order
            const uint32_t l = l0 + u;
            if (l < n_layer && s_act[l]) {
                acc = __dadd_rn(acc, cur[u]);
                ++nlay;
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < 16; ++u) cur[u] = nxt[u];
    }
    scores[b] = nlay ? __ddiv_rn(acc, static_cast<double>(nlay)) : 0.0;
}

// ---------------------------------------------------------------------------
// Block-wide radix selection of the k smallest of a set of u64 keys.
// Each pass takes the keys still in doubt, skips the bits they all share (a
// min / max reduction), histograms the next 11 bits (2048 bins in shared
// memory) and keeps only the bin holding the k-th
// key; keys below it are in, keys above it out. Once the keys in doubt fit
// the candidate list they are compacted into it, so later passes touch only
// those (a few after the first pass on spread-out data). Work is O(n) for
// the first pass; the loop ends when the whole bin is in (exact threshold) or
// when every key left in doubt is equal (a tie group, for the caller to
// split by a second key).
struct SelSmem {
    uint32_t hist[2048];
    uint64_t wmin[32], wmax[32];
    uint32_t wcnt[32];
    uint64_t mn, mx, thr;
    uint32_t k, m, listed, mode, n_valid, cnt_new, done, claimed;
};

enum : uint32_t { kSelNone = 0, kSelAll = 1, kSelExact = 2, kSelTie = 3 };

// Block min / max / count of (mn, mx, cnt) into s.mn, s.mx and the return value.
__device__ __forceinline__ uint32_t block_minmax(uint64_t mn, uint64_t mx, uint32_t cnt,
                                                 SelSmem &s) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const uint64_t a = __shfl_xor_sync(0xffffffffu, mn, o);
        const uint64_t b = __shfl_xor_sync(0xffffffffu, mx, o);
        mn = a < mn ? a : mn;
        mx = b > mx ? b : mx;
        cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    }
    if (lane == 0) {
        s.wmin[warp] = mn;
        s.wmax[warp] = mx;
        s.wcnt[warp] = cnt;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t w = 1; w < nw; ++w) {
            mn = s.wmin[w] < mn ? s.wmin[w] : mn;
            mx = s.wmax[w] > mx ? s.wmax[w] : mx;
            cnt += s.wcnt[w];
        }
        s.mn = mn;
        s.mx = mx;
        s.wcnt[0] = cnt;
    }
    __syncthreads();
    const uint32_t total = s.wcnt[0];
    __syncthreads();  // s.wcnt is reused by the next reduction
    return total;
}

// Appends index i to `list` (warp-aggregated slot claim). Every lane of the
// warp calls it; `take` says whether this lane appends.
template <class IdxT>
__device__ __forceinline__ void list_push(bool take, uint32_t i, IdxT *list, uint32_t *count) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t m = __ballot_sync(0xffffffffu, take);
    if (!m) return;
    uint32_t base = 0;
    const uint32_t leader = static_cast<uint32_t>(__ffs(m) - 1);
    if (lane == leader) base = atomicAdd(count, static_cast<uint32_t>(__popc(m)));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (take) list[base + __popc(m & ((1u << lane) - 1))] = static_cast<IdxT>(i);
}

// key_of(i, key) -> bool (false: i is not a candidate), i < n. Every thread of
// the block calls this; blockDim.x is a multiple of 32. `la` / `lb` are two
// candidate lists of `cap` entries each (cap may be 0). On return s.mode is
//   kSelNone  (k == 0 or no candidate),
//   kSelAll   (k >= the candidate count),
//   kSelExact (exactly k candidates have key <= s.thr), or
//   kSelTie   (fewer than k have key < s.thr, and the s.k still missing are
//              to be taken from the keys equal to s.thr),
// and s.n_valid is the candidate count.
template <class IdxT, class KeyFn>
__device__ void block_select_u64(uint32_t n, uint32_t k, KeyFn key_of, IdxT *la, IdxT *lb,
                                 uint32_t cap, SelSmem &s) {
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s.cnt_new = 0;
    __syncthreads();
    // pass 0: count, range, and the list when everything fits
    uint64_t mn = ~0ull, mx = 0;
    uint32_t cnt = 0;
    const bool fits_all = n <= cap;
    for (uint32_t base = 0; base < n; base += blockDim.x) {
        const uint32_t i = base + tid;
        uint64_t key = 0;
        const bool v = i < n && key_of(i, key);
        if (v) {
            mn = key < mn ? key : mn;
            mx = key > mx ? key : mx;
            ++cnt;
        }
        if (fits_all) list_push(v, i, la, &s.cnt_new);
    }
    const uint32_t total = block_minmax(mn, mx, cnt, s);
    if (tid == 0) {
        s.n_valid = total;
        s.k = k;
        s.m = total;
        s.listed = fits_all ? 1u : 0u;
        s.done = 1;
        if (k == 0 || total == 0) s.mode = kSelNone;
        else if (k >= total) s.mode = kSelAll;
        else if (s.mn == s.mx) s.mode = kSelTie, s.thr = s.mn;
        else s.done = 0;
    }
    __syncthreads();
    IdxT *cur = la, *nxt = lb;
    while (!s.done) {
        const uint64_t lo = s.mn, hi_k = s.mx;
        const uint32_t top = 63u - static_cast<uint32_t>(__clzll(static_cast<long long>(lo ^ hi_k)));
        const uint32_t shift = top >= 10 ? top - 10 : 0;
        const uint32_t nb = 1u << (top - shift + 1);
        const uint64_t above = top == 63 ? 0ull : (lo >> (top + 1));  // bits all keys in doubt share
        const bool listed = s.listed;
        const uint32_t kk = s.k, m = s.m;
        for (uint32_t b = tid; b < nb; b += blockDim.x) s.hist[b] = 0;
        __syncthreads();
        const uint32_t span = listed ? m : n;
        for (uint32_t base = 0; base < span; base += blockDim.x) {  // warp-uniform trip count
            const uint32_t j = base + tid;
            uint64_t key = 0;
            bool act = false;
            if (j < span) {
                act = key_of(listed ? static_cast<uint32_t>(cur[j]) : j, key);
                if (act && !listed && top < 63) act = (key >> (top + 1)) == above;
                if (act && !listed) act = key >= lo && key <= hi_k;
            }
            const uint32_t dg = act ? static_cast<uint32_t>(key >> shift) & (nb - 1) : 0xffffffffu;
            if (act) atomicAdd(&s.hist[dg], 1u);
        }
        __syncthreads();
        {  // thread t owns bins [t * per, (t + 1) * per); block-wide prefix sum
            const uint32_t per = (nb + blockDim.x - 1) / blockDim.x;  // <= 2 at 1024 threads
            uint32_t sum = 0;
            for (uint32_t j = 0; j < per; ++j) {
                const uint32_t b = tid * per + j;
                sum += b < nb ? s.hist[b] : 0u;
            }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= static_cast<uint32_t>(o)) incl += t;
            }
            if (lane == 31) s.wcnt[warp] = incl;
            __syncthreads();
            if (warp == 0) {
                const uint32_t nw = blockDim.x >> 5;
                const uint32_t v = lane < nw ? s.wcnt[lane] : 0u;
                uint32_t wi = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
                    if (lane >= static_cast<uint32_t>(o)) wi += t;
                }
                if (lane < nw) s.wcnt[lane] = wi - v;  // exclusive prefix of the warps
                if (lane == 0) s.claimed = 0;
            }
            __syncthreads();
            const uint32_t excl = s.wcnt[warp] + incl - sum;
            if (excl < kk && kk <= excl + sum) {  // exactly one thread
                uint32_t cum = excl, d = tid * per, cd = 0;
                for (uint32_t j = 0; j < per; ++j) {
                    const uint32_t b = tid * per + j;
                    const uint32_t c = b < nb ? s.hist[b] : 0u;
                    if (cum + c >= kk) {
                        d = b;
                        cd = c;
                        break;
                    }
                    cum += c;
                }
                const uint32_t rem = kk - cum;
                const uint64_t pre = (top == 63 ? 0ull : (above << (top + 1))) |
                                     (static_cast<uint64_t>(d) << shift);
                if (rem == cd) {  // the whole bin is in
                    s.mode = kSelExact;
                    s.thr = pre | ((1ull << shift) - 1);
                    s.done = 1;
                } else if (shift == 0) {  // one key value, more copies than needed
                    s.mode = kSelTie;
                    s.thr = pre;
                    s.k = rem;
                    s.done = 1;
                } else {  // keep the bin: keys in [pre, pre + 2^shift)
                    s.k = rem;
                    s.m = cd;
                    s.mn = pre;
                    s.mx = pre | ((1ull << shift) - 1);
                }
                s.cnt_new = 0;
                s.claimed = 1;
            }
            __syncthreads();
            if (tid == 0 && !s.claimed) {  // unreachable for fixed keys; ends the loop regardless
                s.mode = kSelAll;
                s.done = 1;
            }
        }
        __syncthreads();
        if (s.done) break;
        // narrow to the kept bin: its exact range, and the list when it fits
        const uint64_t blo = s.mn, bhi = s.mx;
        const bool to_list = s.m <= cap;
        mn = ~0ull;
        mx = 0;
        cnt = 0;
        for (uint32_t base = 0; base < span; base += blockDim.x) {
            const uint32_t j = base + tid;
            uint64_t key = 0;
            bool act = false;
            uint32_t i = j;
            if (j < span) {
                i = listed ? static_cast<uint32_t>(cur[j]) : j;
                act = key_of(i, key) && key >= blo && key <= bhi;
            }
            if (act) {
                mn = key < mn ? key : mn;
                mx = key > mx ? key : mx;
                ++cnt;
            }
            if (to_list) list_push(act, i, nxt, &s.cnt_new);
        }
        block_minmax(mn, mx, cnt, s);
        if (tid == 0) {
            s.listed = to_list ? 1u : 0u;
            if (s.mn == s.mx) {  // every key left in doubt is equal
                s.mode = kSelTie;
                s.thr = s.mn;
                s.done = 1;
            }
        }
        if (to_list) {
            IdxT *t = cur;
            cur = nxt;
            nxt = t;
        }
        __syncthreads();
    }
    __syncthreads();
}

// Order-preserving map of a double onto u64 (-0.0 taken as +0.0, since the
// reference's comparisons do not separate them).
__device__ __forceinline__ uint64_t score_key(double x) {
    if (x == 0.0) x = 0.0;
    const uint64_t u = static_cast<uint64_t>(__double_as_longlong(x));
    return (u >> 63) ? ~u : (u | (1ull << 63));
}

// ---------------------------------------------------------------------------
// S6: block top-k. Block b (not kept) is chosen iff fewer than `need` other
// candidates beat it under (score desc, id by tie rule) — the set nth_element
// returns for that strict total order (kvmem_store.cpp:600-616). One CTA: a
// radix selection of the `need` best scores (smallest complemented keys);
// when the boundary falls inside a group of equal scores, a second selection
// over the ids of that group settles it by the tie rule. STAGED (n up to
// kSelectStagedMax): every key is loaded once, all loads in flight, into
// shared memory (a kept block's key is ~0, which no score maps to), and the
// passes run from there; beyond it the passes read the scores from global
// memory.
constexpr uint32_t kSelectStagedMax = 16384;
constexpr uint32_t kSelectListCap = 16384;
// Up to KVMRET_SEL_SMALL_N blocks the selection runs with fewer threads: each
// pass has several block-wide barriers, cheaper with fewer warps (2048
// blocks: 8.7 us with 512 threads, 9.4 us with 1024, 10.8 us with 256).
#ifndef KVMRET_SEL_SMALL_N
#define KVMRET_SEL_SMALL_N 4096
#endif
#ifndef KVMRET_SEL_SMALL_THREADS
#define KVMRET_SEL_SMALL_THREADS 512
#endif

template <bool STAGED>
__global__ void __launch_bounds__(1024) select_radix_kernel(const double *__restrict__ scores,
                                                            const uint8_t *__restrict__ kept,
                                                            uint32_t n, uint32_t need, int tie_high,
                                                            uint8_t *__restrict__ sel,
                                                            uint32_t cap) {
    dep_wait();
    extern __shared__ __align__(16) uint8_t sel_sm[];
    __shared__ SelSmem ss;
    using IdxT = typename std::conditional<STAGED, uint16_t, uint32_t>::type;
    uint64_t *s_key = reinterpret_cast<uint64_t *>(sel_sm);
    IdxT *la = reinterpret_cast<IdxT *>(sel_sm + (STAGED ? static_cast<size_t>(n) * 8 : 0));
    IdxT *lb = la + cap;
    constexpr uint64_t kKept = ~0ull;
    if (STAGED) {
        constexpr uint32_t U = 8;
        for (uint32_t base = 0; base < n; base += U * blockDim.x) {
            double v[U];
            uint8_t kp[U];
#pragma unroll
            for (uint32_t u = 0; u < U; ++u) {
                const uint32_t i = base + u * blockDim.x + threadIdx.x;
                v[u] = i < n ? scores[i] : 0.0;
                kp[u] = i < n ? kept[i] : 1;
            }
#pragma unroll
            for (uint32_t u = 0; u < U; ++u) {
                const uint32_t i = base + u * blockDim.x + threadIdx.x;
                if (i < n) s_key[i] = kp[u] ? kKept : ~score_key(v[u]);
            }
        }
        __syncthreads();
    }
    auto skey = [&](uint32_t i) -> uint64_t {
        if (STAGED) return s_key[i];
        return kept[i] ? kKept : ~score_key(scores[i]);
    };
    auto key1 = [&](uint32_t i, uint64_t &key) -> bool {
        key = skey(i);
        return key != kKept;
    };
    block_select_u64(n, need, key1, la, lb, cap, ss);
    const uint32_t mode1 = ss.mode;
    const uint64_t t1 = ss.thr;
    const uint32_t k2 = ss.k;
    uint32_t mode2 = kSelNone;
    uint64_t t2 = 0;
    if (mode1 == kSelTie) {  // the boundary group: equal scores, split by id
        auto key2 = [&](uint32_t i, uint64_t &key) -> bool {
            if (skey(i) != t1) return false;
            key = tie_high ? static_cast<uint64_t>(~i) : static_cast<uint64_t>(i);
            return true;
        };
        // the keys below the group are in; the group's k2 best by id join them
        __syncthreads();
        block_select_u64(n, k2, key2, la, lb, cap, ss);
        mode2 = ss.mode;
        t2 = ss.thr;
    }
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const uint64_t key = skey(i);
        uint8_t v;
        if (key == kKept || mode1 == kSelAll) {
            v = 1;
        } else if (mode1 == kSelNone) {
            v = 0;
        } else if (mode1 == kSelExact) {
            v = key <= t1;
        } else if (key != t1) {
            v = key < t1;
        } else {
            const uint64_t ik = tie_high ? static_cast<uint64_t>(~i) : static_cast<uint64_t>(i);
            v = mode2 == kSelAll || (mode2 == kSelExact && ik <= t2);
        }
        sel[i] = v;
    }
}

// ---------------------------------------------------------------------------
// RoPE table: cos / sin of the float angle pos * theta[i] (rope.cpp:27-33).
// The angle is the reference's float product; cos and sin are evaluated in
// double and rounded once to float, i.e. correctly rounded, so the table does
// not add the few-ulp error of a float sincos. Window positions come from a
// per-context table built once at creation; the stateless entry points build a
// temporary table for their positions.
__device__ __forceinline__ float2 rope_cs(int32_t pos, float theta) {
    const float ang = __fmul_rn(static_cast<float>(pos), theta);
    double s, c;
    sincos(static_cast<double>(ang), &s, &c);
    return make_float2(__double2float_rn(c), __double2float_rn(s));
}

// Position table: cs[p][j] = {c_2j, c_2j+1, s_2j, s_2j+1} of position
// pos_base + p, for p in [0, n_pos).
__global__ void rope_table_kernel(float4 *__restrict__ cs, uint32_t n_pos, uint32_t half,
                                  int32_t pos_base, const __grid_constant__ Theta th) {
    const uint32_t hp = half / 2;
    const size_t n = static_cast<size_t>(n_pos) * hp;
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < n;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int32_t pos = pos_base + static_cast<int32_t>(idx / hp);
        const uint32_t j = static_cast<uint32_t>(idx % hp);
        const float2 u = rope_cs(pos, th.v[2 * j]), v = rope_cs(pos, th.v[2 * j + 1]);
        cs[idx] = make_float4(u.x, v.x, u.y, v.y);
    }
}

// Items per thread whose loads are issued together (tunable at build time).
#ifndef KVMRET_F16_UNROLL
#define KVMRET_F16_UNROLL 2
#endif

template <int D>
__device__ __forceinline__ void rope_chunk_f16(const uint4 &lo, const uint4 &hi, uint4 &olo,
                                               uint4 &ohi, const float4 *__restrict__ cs) {
    const uint16_t *a = reinterpret_cast<const uint16_t *>(&lo);
    const uint16_t *b = reinterpret_cast<const uint16_t *>(&hi);
    uint16_t *oa = reinterpret_cast<uint16_t *>(&olo);
    uint16_t *ob = reinterpret_cast<uint16_t *>(&ohi);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        const float4 t = __ldg(cs + e / 2);
        float x0 = h2f(a[e]), x1 = h2f(b[e]);
        oa[e] = f2h(__fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.z)));
        ob[e] = f2h(__fadd_rn(__fmul_rn(x0, t.z), __fmul_rn(x1, t.x)));
        x0 = h2f(a[e + 1]);
        x1 = h2f(b[e + 1]);
        oa[e + 1] = f2h(__fsub_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.w)));
        ob[e + 1] = f2h(__fadd_rn(__fmul_rn(x0, t.w), __fmul_rn(x1, t.y)));
    }
}

// f16 K: rows [n_tok][Hkv][D] f16, 16-byte chunks of the low and high halves;
// row r is token r / n_head_kv at table row tab + token * D/4. raw_dst (fresh
// blocks) also receives the unrotated rows; src is then host memory read with
// plain loads.
template <int D, bool FRESH>
__device__ __forceinline__ void rope_rows_f16(const uint8_t *__restrict__ src,
                                              uint8_t *__restrict__ dst,
                                              const float4 *__restrict__ tab, uint32_t n_tok,
                                              uint32_t n_head_kv, uint8_t *__restrict__ raw_dst,
                                              uint32_t tid = threadIdx.x,
                                              uint32_t nthr = blockDim.x) {
    constexpr int HALF = D / 2, CPR = HALF / 8, U = KVMRET_F16_UNROLL;
    const uint32_t n_items = n_tok * n_head_kv * CPR;
    for (uint32_t w0 = tid; w0 < n_items; w0 += U * nthr) {
        uint4 lo[U], hi[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {  // all loads first
            const uint32_t w = w0 + u * nthr;
            if (w >= n_items) break;
            const uint32_t row = w / CPR, j = w % CPR;
            const uint4 *sp = reinterpret_cast<const uint4 *>(src + static_cast<size_t>(row) * D * 2);
            if constexpr (FRESH) {
                lo[u] = sp[j];
                hi[u] = sp[CPR + j];
                uint4 *rp = reinterpret_cast<uint4 *>(raw_dst + static_cast<size_t>(row) * D * 2);
                rp[j] = lo[u];
                rp[CPR + j] = hi[u];
            } else {
                lo[u] = __ldg(sp + j);
                hi[u] = __ldg(sp + CPR + j);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t w = w0 + u * nthr;
            if (w >= n_items) break;
            const uint32_t row = w / CPR, j = w % CPR, t = row / n_head_kv;
            uint4 olo, ohi;
            rope_chunk_f16<D>(lo[u], hi[u], olo, ohi, tab + static_cast<size_t>(t) * (D / 4) + 4 * j);
            uint4 *dp = reinterpret_cast<uint4 *>(dst + static_cast<size_t>(row) * D * 2);
            dp[j] = olo;
            dp[CPR + j] = ohi;
        }
    }
}

// 16-byte vector copies by the whole CTA. copy16 reads through the read-only
// global path (__ldg), so its source must be global memory; copy16_host
// reads host memory (mapped pinned) with plain loads and writes one or two
// destinations. Four loads are in flight per thread.
__device__ __forceinline__ void copy16(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                       uint64_t nbytes, uint32_t tid = threadIdx.x,
                                       uint32_t nthr = blockDim.x) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    const uint64_t n = nbytes / 16, step = nthr;
    uint64_t w = tid;
    for (; w + 3 * step < n; w += 4 * step) {
        const uint4 v0 = __ldg(s + w), v1 = __ldg(s + w + step);
        const uint4 v2 = __ldg(s + w + 2 * step), v3 = __ldg(s + w + 3 * step);
        d[w] = v0;
        d[w + step] = v1;
        d[w + 2 * step] = v2;
        d[w + 3 * step] = v3;
    }
    for (; w < n; w += step) d[w] = __ldg(s + w);
}
__device__ __forceinline__ void copy16_host(const uint8_t *src, uint8_t *__restrict__ dst,
                                            uint8_t *__restrict__ dst2, uint64_t nbytes,
                                            uint32_t tid = threadIdx.x,
                                            uint32_t nthr = blockDim.x) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    uint4 *d2 = reinterpret_cast<uint4 *>(dst2);
    const uint64_t n = nbytes / 16, step = nthr;
    uint64_t w = tid;
    for (; w + 3 * step < n; w += 4 * step) {
        const uint4 v0 = s[w], v1 = s[w + step], v2 = s[w + 2 * step], v3 = s[w + 3 * step];
        d[w] = v0;
        d[w + step] = v1;
        d[w + 2 * step] = v2;
        d[w + 3 * step] = v3;
        if (d2) {
            d2[w] = v0;
            d2[w + step] = v1;
            d2[w + 2 * step] = v2;
            d2[w + 3 * step] = v3;
        }
    }
    for (; w < n; w += step) {
        const uint4 v = s[w];
        d[w] = v;
        if (d2) d2[w] = v;
    }
}

// One CTA's share of an assembly launch: which job, which layer group.
struct JobView {
    uint32_t pool_slot, win_slot, n_tok, block, group;
    int32_t pos0;
    bool fresh;
};

// Returns false when the CTA has no job (beyond the device counts).
__device__ __forceinline__ bool decode_job(const AsmLaunch &a, JobView &v) {
    v.group = blockIdx.y;
    v.fresh = false;
    v.block = 0;
    if (a.jobs) {
        uint32_t j = blockIdx.x;
        if (a.counts) {
            // 1-D grid: every (fresh job, layer group) CTA first, so the host-link
            // reads start at once and overlap the moves; then the moved jobs.
            const uint32_t G = gridDim.y == 1 ? a.n_groups : 1;
            const uint32_t half = a.fresh_offset * G;
            const uint32_t idx = blockIdx.x;
            if (idx < half) {
                j = idx / G;
                v.group = idx % G;
                if (j >= a.counts[1]) return false;
                j += a.fresh_offset;
                v.fresh = true;
            } else {
                j = (idx - half) / G;
                v.group = (idx - half) % G;
                if (j >= a.counts[0]) return false;
            }
        }
        const Job *jp = a.jobs + j;
        v.pool_slot = jp->pool_slot;
        v.win_slot = jp->win_slot;
        v.pos0 = jp->pos0;
        v.n_tok = jp->n_tok;
        v.block = jp->block;
    } else {  // stateless form: chunk i of a contiguous run of rows
        v.pool_slot = blockIdx.x;
        v.win_slot = blockIdx.x;
        v.pos0 = a.synth_pos0 + static_cast<int32_t>(blockIdx.x * a.g.block_tokens);
        v.n_tok = min(a.g.block_tokens, a.synth_ntok - blockIdx.x * a.g.block_tokens);
    }
    return true;
}

constexpr int kAsmThreads = 512;

// One (job, layer) unit of the f16 assembly: K re-roped from the unrotated
// copy (pool, or host repository for a fresh job, which is also copied into
// its pool slot) at the job's window base; V copied.
template <int D>
__device__ __forceinline__ void assemble_unit_f16(const AsmLaunch &a, const JobView &jv,
                                                  uint32_t l, const float4 *tab,
                                                  uint32_t tid = threadIdx.x,
                                                  uint32_t nthr = blockDim.x) {
    const AssembleGeom &g = a.g;
    const uint8_t *slot = jv.fresh ? a.repo + static_cast<uint64_t>(jv.block) * a.slot_bytes
                                   : a.pool + static_cast<uint64_t>(jv.pool_slot) * a.slot_bytes;
    const uint8_t *src = slot + static_cast<uint64_t>(l) * g.unit;
    uint8_t *raw = jv.fresh ? a.pool_w + static_cast<uint64_t>(jv.pool_slot) * a.slot_bytes +
                                  static_cast<uint64_t>(l) * g.unit
                            : nullptr;
    uint8_t *dk = a.win_k + static_cast<uint64_t>(l) * g.win_k_layer +
                  static_cast<uint64_t>(jv.win_slot) * g.block_tokens * g.k_row;
    if (raw)
        rope_rows_f16<D, true>(src, dk, tab, jv.n_tok, g.n_head_kv, raw, tid, nthr);
    else
        rope_rows_f16<D, false>(src, dk, tab, jv.n_tok, g.n_head_kv, nullptr, tid, nthr);
    if (g.v_row) {
        uint8_t *dv = a.win_v + static_cast<uint64_t>(l) * g.win_v_layer +
                      static_cast<uint64_t>(jv.win_slot) * g.block_tokens * g.v_row;
        const uint64_t vb = static_cast<uint64_t>(jv.n_tok) * g.v_row;
        if (raw)
            copy16_host(src + g.unit_k, dv, raw + g.unit_k, vb, tid, nthr);
        else
            copy16(src + g.unit_k, dv, vb, tid, nthr);
    }
}

#ifndef KVMRET_F16_MINB
#define KVMRET_F16_MINB 2
#endif
// the fresh (host-link) work of a launch is cut into about this many units
#ifndef KVMRET_F16_FRESH_UNITS
#define KVMRET_F16_FRESH_UNITS 16
#endif
// S10-S12, f16 K. With device counts (the GPU-resident step) the grid is
// persistent (one wave) and CTAs take work units from a device counter: first
// the fresh jobs (host-link bound, started at once), then the moved jobs, one
// (job, layer) unit at a time, so the CTAs finish together (no partial last
// wave). cos/sin come from the position table through L1.
// Without counts (stateless form): CTA = one chunk, layer 0.
template <int D>
__global__ void __launch_bounds__(kAsmThreads, KVMRET_F16_MINB)
    assemble_kernel(const __grid_constant__ AsmLaunch a) {
    dep_wait();
    constexpr uint32_t PAIRS = D / 4;
    JobView jv;
    if (!a.counts) {
        if (!decode_job(a, jv)) return;
        assemble_unit_f16<D>(a, jv, 0, a.gtab + static_cast<size_t>(jv.pos0) * PAIRS);
        return;
    }
    __shared__ uint32_t s_unit;
    const uint32_t L = a.g.n_layer;
    // fresh jobs are host-link bound for most of the launch: about 16 fresh
    // units (each CTA keeps ~32 KB of host loads in flight) saturate the link
    // without taking more CTAs away from the HBM-bound moved units
    const uint32_t LF = min(L, max(1u, (a.counts[1] * L + KVMRET_F16_FRESH_UNITS - 1) /
                                           KVMRET_F16_FRESH_UNITS)),
                   gf = (L + LF - 1) / LF;
    const uint32_t n_fu = a.counts[1] * gf;
    const uint32_t n_units = n_fu + a.counts[0] * L;
    for (;;) {
        if (threadIdx.x == 0) s_unit = atomicAdd(a.work, 1u);
        __syncthreads();
        const uint32_t u = s_unit;
        __syncthreads();  // every thread has read s_unit before it is overwritten
        if (u >= n_units) break;
        uint32_t j, l0, l1;
        if (u < n_fu) {
            j = a.fresh_offset + u / gf;
            l0 = (u % gf) * LF;
            l1 = min(L, l0 + LF);
            jv.fresh = true;
        } else {
            const uint32_t v = u - n_fu;
            j = v / L;
            l0 = v % L;
            l1 = l0 + 1;
            jv.fresh = false;
        }
        const Job *jp = a.jobs + j;
        jv.pool_slot = jp->pool_slot;
        jv.win_slot = jp->win_slot;
        jv.pos0 = jp->pos0;
        jv.n_tok = jp->n_tok;
        jv.block = jp->block;
        const float4 *tab = a.gtab + static_cast<size_t>(jv.pos0) * PAIRS;
        for (uint32_t l = l0; l < l1; ++l) assemble_unit_f16<D>(a, jv, l, tab);
    }
}

// ---------------------------------------------------------------------------
// S13, quantised K: dequant (llama-kvmem-stagein.cu:133-158) -> RoPE ->
// FWHT (:105-131) -> requant (:181-234), per K head row of D elements.
//
// Register layout. A row is held by LPR = D/64 lanes; sub-lane q holds quant
// block q (elements 32q .. 32q+31) in xl[] and block LPR+q (elements
// D/2+32q ..) in xh[]. Every RoPE pair (i, i+D/2) and every quant block is
// then inside one lane; of the FWHT's strides 1 .. D/2, the strides 1-16 and
// D/2 run in registers and only 32 .. D/4 cross lanes (log2(LPR) shuffle
// stages, none for D = 64). A warp holds 32/LPR rows, which is always 64
// quant blocks: 2176 bytes of q8_0 or 1152 of q4_0 (one "segment").
//
// Data movement. Segments are contiguous in the pool and in the window. Each
// warp streams its segments, and the V rows in segment-sized pieces, through
// kQStages shared-memory stages with 16-byte cp.async copies (fresh jobs:
// plain loads from the mapped host repository, also written to the pool
// slot), converts K in place, and writes each piece back with 16-byte
// stores. A K stage also receives the cos/sin rows of the tokens the
// segment spans when they fit kQTabBytes.
//
// Byte access. Quant blocks (34 or 18 bytes) start at offsets that are 0 or 2
// mod 4 (rows are 4-byte multiples); a block is read as whole 32-bit words
// from the enclosing aligned word and realigned with byte permutes, and
// written as whole words plus one 16-bit store at the unaligned end, so no
// two lanes write the same byte.
//
// Arithmetic. Pairs of elements go through packed f32x2 operations, each of
// which rounds both halves exactly like the scalar operation.
template <int KT> struct QBlk;
template <> struct QBlk<0> {  // q8_0 {f16 d; int8 q[32]}
    static constexpr int bytes = 34, words = 8;
};
template <> struct QBlk<1> {  // q4_0 {f16 d; u8 q[16]: lo nibble j, hi nibble j+16}
    static constexpr int bytes = 18, words = 4;
};

// Launch shape (tunable at build time): threads per CTA, pipeline stages per
// warp, resident CTAs per SM the register allocation is sized for.
#ifndef KVMRET_Q_THREADS
#define KVMRET_Q_THREADS 256
#endif
#ifndef KVMRET_Q_STAGES
#define KVMRET_Q_STAGES 4
#endif
#ifndef KVMRET_Q_MINB
#define KVMRET_Q_MINB 2
#endif
constexpr int kQThreads = KVMRET_Q_THREADS;
constexpr int kQStages = KVMRET_Q_STAGES;
constexpr int kQSegBlocks = 64;   // quant blocks per warp segment
constexpr int kQTabBytes = 1024;  // staged cos/sin bytes per K segment

typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float a, float b) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(f32x2 r, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// a * b + c with one rounding; used only with b = +-1, where it equals the
// correctly rounded c + a or c - a.
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// round-half-away-from-zero (C roundf) for |y| < 2^23: truncate y + s, s =
// copysign(0.5 - 2^-25, y) (the float just below one half). Exactness: for
// |y| >= 1 the sum is exact or rounds only across the binade edge, where
// truncation already gives the rounded value; for |y| < 1 the only
// candidates for a wrong carry are the ties y = +-0.5 (sum 1 - 2^-25 rounds
// to 1, as wanted) and y = +-(0.5 - 2^-25) (sum 1 - 2^-24, exact, truncates
// to 0). Checked against the host roundf on every float of magnitude < 256.
// The truncation is the conversion to an integer (toward zero), whose low
// byte is then the int8.
__device__ __forceinline__ int round_away_int(float y) {
    return __float2int_rz(__fadd_rn(y, copysignf(0.49999997f, y)));
}

// Reads the quant block at byte offset o of a shared-memory segment: scale
// bits and the payload as words (payload byte 4j+k = byte k of p[j]).
template <int KT>
__device__ __forceinline__ void load_qblock(const uint8_t *seg, uint32_t o, uint32_t &d16,
                                            uint32_t (&p)[QBlk<KT>::words]) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(seg + (o & ~3u));
    const bool odd = o & 2u;
    uint32_t prev = w[0];
    d16 = odd ? (prev >> 16) : (prev & 0xffffu);
    const uint32_t sel = odd ? 0x7654u : 0x5432u;
#pragma unroll
    for (int j = 0; j < QBlk<KT>::words; ++j) {
        const uint32_t nx = w[j + 1];
        p[j] = __byte_perm(prev, nx, sel);
        prev = nx;
    }
}

template <int KT>
__device__ __forceinline__ void store_qblock(uint8_t *seg, uint32_t o, uint32_t d16,
                                             const uint32_t (&p)[QBlk<KT>::words]) {
    constexpr int NW = QBlk<KT>::words;
    const bool odd = o & 2u;
    uint32_t *w = reinterpret_cast<uint32_t *>(seg + (odd ? o + 2 : o));
    const uint32_t sel = odd ? 0x7654u : 0x5432u;
    uint32_t prev = d16 << 16;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        w[k] = __byte_perm(prev, p[k], sel);
        prev = p[k];
    }
    *reinterpret_cast<uint16_t *>(seg + (odd ? o : o + 4 * NW)) =
        static_cast<uint16_t>(odd ? d16 : (p[NW - 1] >> 16));
}

// Float of a small integer from the low byte of a magic-biased word:
// bits 0x4B0000xx are the float 2^23 + xx, exact.
__device__ __forceinline__ float byte_float(uint32_t word, uint32_t k) {
    return __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7440u | k));
}

template <int KT>
__device__ __forceinline__ void dequant_qblock(uint32_t d16, const uint32_t (&p)[QBlk<KT>::words],
                                               float (&x)[32]) {
    const float d = h2f(static_cast<uint16_t>(d16));
    const f32x2 D2 = pk2(d, d);
    if constexpr (KT == 0) {  // x = float(int8) * d
        const f32x2 M2 = pk2(8388736.0f, 8388736.0f);  // 2^23 + 128
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t u = p[j] ^ 0x80808080u;  // int8 s -> s + 128
#pragma unroll
            for (int k = 0; k < 4; k += 2)
                upk2(mul2(sub2(pk2(byte_float(u, k), byte_float(u, k + 1)), M2), D2),
                     x[4 * j + k], x[4 * j + k + 1]);
        }
    } else {  // x = (nibble - 8) * d
        const f32x2 M2 = pk2(8388616.0f, 8388616.0f);  // 2^23 + 8
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lo = p[j] & 0x0F0F0F0Fu, hi = (p[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
                upk2(mul2(sub2(pk2(byte_float(lo, k), byte_float(lo, k + 1)), M2), D2),
                     x[4 * j + k], x[4 * j + k + 1]);
                upk2(mul2(sub2(pk2(byte_float(hi, k), byte_float(hi, k + 1)), M2), D2),
                     x[16 + 4 * j + k], x[16 + 4 * j + k + 1]);
            }
        }
    }
}

__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t b0, uint32_t b1, uint32_t b2,
                                                   uint32_t b3) {
    return __byte_perm(__byte_perm(b0, b1, 0x0040u), __byte_perm(b2, b3, 0x0040u), 0x5410u);
}

// x / 127 correctly rounded, by division by a constant known in advance
// (Brisebarre, Muller and Raina, IEEE Trans. Computers 53(8), 2004): with
// zh = RN(1/127) and zl = RN(1/127 - zh), RN(x zh + RN(x zl)) is the
// correctly rounded quotient. Checked against IEEE division on every
// non-negative float: it holds for all x >= 2^-100 (below that x zl loses
// bits to underflow), so smaller x take the division.
__device__ __forceinline__ float div127_rn(float x) {
    if (!(x >= 0x1p-100f)) return __fdiv_rn(x, 127.0f);
    return __fmaf_rn(x, 0x1.020408p-7f, __fmul_rn(x, 0x1.020408p-35f));
}

template <int KT>
__device__ __forceinline__ void requant_qblock(const float (&x)[32], uint32_t &d16,
                                               uint32_t (&p)[QBlk<KT>::words]) {
    if constexpr (KT == 0) {  // quant_q8_0: d = amax / 127, q = round(x / d)
        // max |x| by a tree (max is exact, so the order is free); the initial
        // 0 of the sequential form is the last operand.
        float m[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) m[e] = fmaxf(fabsf(x[e]), fabsf(x[e + 16]));
#pragma unroll
        for (int w = 8; w >= 1; w /= 2)
#pragma unroll
            for (int e = 0; e < w; ++e) m[e] = fmaxf(m[e], m[e + w]);
        const float amax = fmaxf(0.0f, m[0]);
        const float dq = div127_rn(amax);
        const float id = dq != 0.0f ? __frcp_rn(dq) : 0.0f;
        d16 = f2h(dq);
        const f32x2 ID2 = pk2(id, id);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t b[4];
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
                float y0, y1;
                upk2(mul2(pk2(x[4 * j + k], x[4 * j + k + 1]), ID2), y0, y1);
                b[k] = static_cast<uint32_t>(round_away_int(y0));
                b[k + 1] = static_cast<uint32_t>(round_away_int(y1));
            }
            p[j] = pack_low_bytes(b[0], b[1], b[2], b[3]);
        }
    } else {  // quant_q4_0: d = vmax / -8 (vmax: first element of largest |x|)
        float amax = 0.0f, vmax = 0.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const float a = fabsf(x[e]);
            if (amax < a) {
                amax = a;
                vmax = x[e];
            }
        }
        const float dq = __fmul_rn(vmax, -0.125f);  // = vmax / -8, the same rounding
        const float id = dq != 0.0f ? __frcp_rn(dq) : 0.0f;
        d16 = f2h(dq);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t b[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = 4 * j + k;
                const int x0 = min(__float2int_rz(__fadd_rn(__fmul_rn(x[i], id), 8.5f)), 15);
                const int x1 = min(__float2int_rz(__fadd_rn(__fmul_rn(x[i + 16], id), 8.5f)), 15);
                b[k] = static_cast<uint32_t>((x0 & 15) | ((x1 & 15) << 4));
            }
            p[j] = pack_low_bytes(b[0], b[1], b[2], b[3]);
        }
    }
}

// In-lane butterflies of stride h (2 <= h <= 16) over one 32-element block,
// two pairs per packed operation.
template <int H>
__device__ __forceinline__ void fwht_stage2(float (&x)[32]) {
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        if (e & H) continue;
        const f32x2 a = pk2(x[e], x[e + 1]), b = pk2(x[e + H], x[e + H + 1]);
        upk2(add2(a, b), x[e], x[e + 1]);
        upk2(sub2(a, b), x[e + H], x[e + H + 1]);
    }
}

// RoPE of a lane's 32 pairs from cos/sin pairs t4[0..15] = {c, c', s, s'}.
__device__ __forceinline__ void rope_pairs(float (&xl)[32], float (&xh)[32], const float4 *t4) {
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        const float4 cs = t4[e / 2];
        const f32x2 X0 = pk2(xl[e], xl[e + 1]), X1 = pk2(xh[e], xh[e + 1]);
        const f32x2 C = pk2(cs.x, cs.y), S = pk2(cs.z, cs.w);
        upk2(sub2(mul2(X0, C), mul2(X1, S)), xl[e], xl[e + 1]);
        upk2(add2(mul2(X0, S), mul2(X1, C)), xh[e], xh[e + 1]);
    }
}

// n / d for n * d < 2^32 (m = ceil(2^32 / d)).
struct FastDiv {
    uint64_t m;
    __device__ explicit FastDiv(uint32_t d) : m((0x100000000ull + d - 1) / d) {}
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        return static_cast<uint32_t>((static_cast<uint64_t>(n) * m) >> 32);
    }
};

// n / d for every 32-bit n: division by an invariant integer with a
// multiply-high and a shift (Granlund and Montgomery, 1994): l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, t = mulhi(m, n),
// n / d = (t + ((n - t) >> 1)) >> (l - 1).
struct DivU32 {
    uint32_t m, l;
    __host__ __device__ explicit DivU32(uint32_t d)
        : m(0), l(d > 1 ? 32u - static_cast<uint32_t>(__builtin_clz(d - 1)) : 0u) {
        if (l) m = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        if (l == 0) return n;
        const uint32_t t = __umulhi(m, n);
        return (t + ((n - t) >> 1)) >> (l - 1);
    }
};

// Converts the rows of one K segment in place. The row of lane pair r is job
// row row_base + r (token (row_base + r) / n_head_kv); its cos/sin pairs are
// tab[(token - tab_tok0) * D/4 + j] (a staged shared-memory slice or the
// position table).
template <int D, int KT>
__device__ __forceinline__ void convert_row(uint8_t *seg, uint32_t lane, uint32_t n_rows_seg,
                                            uint32_t row_base, const FastDiv &hkv,
                                            uint32_t n_rows, const float4 *tab,
                                            uint32_t tab_tok0, uint32_t fwht_n,
                                            float fwht_scale) {
    constexpr int LPR = D / 64, BB = QBlk<KT>::bytes, NW = QBlk<KT>::words;
    constexpr uint32_t HEAD_BYTES = (D / 32) * BB;
    const uint32_t r = lane / LPR, q = lane % LPR;
    const uint32_t R = min(row_base + r, n_rows - 1);  // idle lanes recompute a valid row
    const uint32_t tok = hkv.div(R);
    const uint32_t o_lo = r * HEAD_BYTES + BB * q;
    const uint32_t o_hi = r * HEAD_BYTES + BB * (LPR + q);
    float xl[32], xh[32];
    {
        uint32_t d16, p[NW];
        load_qblock<KT>(seg, o_lo, d16, p);
        dequant_qblock<KT>(d16, p, xl);
        load_qblock<KT>(seg, o_hi, d16, p);
        dequant_qblock<KT>(d16, p, xh);
    }
    // RoPE, pair (i, i + D/2) with i = 32q + e: (x0 c - x1 s, x0 s + x1 c).
    rope_pairs(xl, xh, tab + (tok - tab_tok0) * (D / 4) + 16 * q);
    if (fwht_n) {  // fwht_n == D: scale on input, then strides 1, 2, ..., D/2
        const f32x2 sc = pk2(fwht_scale, fwht_scale);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
            upk2(mul2(pk2(xl[e], xl[e + 1]), sc), xl[e], xl[e + 1]);
            upk2(mul2(pk2(xh[e], xh[e + 1]), sc), xh[e], xh[e + 1]);
        }
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
            float u = xl[e], v = xl[e + 1];
            xl[e] = __fadd_rn(u, v);
            xl[e + 1] = __fsub_rn(u, v);
            u = xh[e];
            v = xh[e + 1];
            xh[e] = __fadd_rn(u, v);
            xh[e + 1] = __fsub_rn(u, v);
        }
        fwht_stage2<2>(xl); fwht_stage2<2>(xh);
        fwht_stage2<4>(xl); fwht_stage2<4>(xh);
        fwht_stage2<8>(xl); fwht_stage2<8>(xh);
        fwht_stage2<16>(xl); fwht_stage2<16>(xh);
#pragma unroll
        for (int m = 1; m < LPR; m *= 2) {  // stride 32m: partner sub-lane q ^ m
            const float sg = (q & m) ? -1.0f : 1.0f;
            const f32x2 S2 = pk2(sg, sg);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                const float pl0 = __shfl_xor_sync(0xffffffffu, xl[e], m);
                const float pl1 = __shfl_xor_sync(0xffffffffu, xl[e + 1], m);
                const float ph0 = __shfl_xor_sync(0xffffffffu, xh[e], m);
                const float ph1 = __shfl_xor_sync(0xffffffffu, xh[e + 1], m);
                upk2(fma2(pk2(xl[e], xl[e + 1]), S2, pk2(pl0, pl1)), xl[e], xl[e + 1]);
                upk2(fma2(pk2(xh[e], xh[e + 1]), S2, pk2(ph0, ph1)), xh[e], xh[e + 1]);
            }
        }
#pragma unroll
        for (int e = 0; e < 32; e += 2) {  // stride D/2
            const f32x2 u = pk2(xl[e], xl[e + 1]), v = pk2(xh[e], xh[e + 1]);
            upk2(add2(u, v), xl[e], xl[e + 1]);
            upk2(sub2(u, v), xh[e], xh[e + 1]);
        }
    }
    uint32_t dl, dh, pl[NW], ph[NW];
    requant_qblock<KT>(xl, dl, pl);
    requant_qblock<KT>(xh, dh, ph);
    __syncwarp();
    if (r < n_rows_seg) {
        store_qblock<KT>(seg, o_lo, dl, pl);
        store_qblock<KT>(seg, o_hi, dh, ph);
    }
    __syncwarp();
}

__device__ __forceinline__ void cp_async16(uint8_t *smem_dst, const uint8_t *gsrc) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// A warp's walk over the CTA's work items: for each of its layers, the K
// segments then the V pieces of the job's (block, layer) unit, dealt to the
// warps round-robin. Advancing costs no division.
struct ItemIter {
    uint32_t l, s;  // layer, index within the layer's items
    __device__ __forceinline__ void advance(uint32_t step, uint32_t per_layer) {
        s += step;
        while (s >= per_layer) {
            s -= per_layer;
            ++l;
        }
    }
};

template <int D, int KT>
__global__ void __launch_bounds__(kQThreads, KVMRET_Q_MINB)
    assemble_quant_kernel(const __grid_constant__ AsmLaunch a, uint32_t layers_per_cta) {
    dep_wait();
    extern __shared__ __align__(16) uint8_t smem_raw[];
    constexpr uint32_t SEG = kQSegBlocks * QBlk<KT>::bytes;
    constexpr uint32_t STAGE = SEG + kQTabBytes;
    constexpr uint32_t PAIRS = D / 4, TAB_TOK = kQTabBytes / (PAIRS * sizeof(float4));
    constexpr uint32_t HEAD_BYTES = (D / 32) * QBlk<KT>::bytes;
    constexpr uint32_t RPW = SEG / HEAD_BYTES;
    const AssembleGeom &g = a.g;
    JobView jv;
    if (!decode_job(a, jv)) return;
    const uint32_t l0 = jv.group * layers_per_cta;
    const uint32_t l1 = min(g.n_layer, l0 + layers_per_cta);
    const bool fresh = jv.fresh;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    uint8_t *wbuf = smem_raw + static_cast<size_t>(warp) * kQStages * STAGE;
    const uint8_t *slot = fresh ? a.repo + static_cast<uint64_t>(jv.block) * a.slot_bytes
                                : a.pool + static_cast<uint64_t>(jv.pool_slot) * a.slot_bytes;
    uint8_t *raw_slot =
        fresh ? a.pool_w + static_cast<uint64_t>(jv.pool_slot) * a.slot_bytes : nullptr;
    const uint32_t kbytes = jv.n_tok * static_cast<uint32_t>(g.k_row);
    const uint32_t vbytes = jv.n_tok * static_cast<uint32_t>(g.v_row);
    const uint32_t nseg_k = (kbytes + SEG - 1) / SEG;
    const uint32_t per_layer = nseg_k + (vbytes + SEG - 1) / SEG;
    const uint32_t n_rows = jv.n_tok * g.n_head_kv;
    const FastDiv hkv(g.n_head_kv);
    const uint64_t wk = static_cast<uint64_t>(jv.win_slot) * g.block_tokens * g.k_row;
    const uint64_t wv = static_cast<uint64_t>(jv.win_slot) * g.block_tokens * g.v_row;
    // the launcher always supplies a table for quantised K
    const float4 *gtab_job = a.gtab + static_cast<size_t>(jv.pos0) * PAIRS;

    // item fields: source, destination, byte count, rows and spanned tokens
    auto src_of = [&](const ItemIter &x, uint32_t &off, uint32_t &bytes, bool &is_v) {
        is_v = x.s >= nseg_k;
        off = (is_v ? x.s - nseg_k : x.s) * SEG;
        bytes = min(SEG, (is_v ? vbytes : kbytes) - off);
        return slot + static_cast<uint64_t>(x.l) * g.unit + (is_v ? g.unit_k : 0) + off;
    };
    auto tokens = [&](uint32_t off, uint32_t &t0, uint32_t &nt) {
        const uint32_t row_base = off / HEAD_BYTES;
        t0 = hkv.div(row_base);
        nt = hkv.div(min(row_base + RPW, n_rows) - 1) - t0 + 1;
    };
    if (per_layer == 0) return;
    ItemIter cur{l0, 0}, pre{l0, 0};
    cur.advance(warp, per_layer);
    pre.advance(warp, per_layer);
    auto issue = [&](uint32_t k) {  // prefetch this warp's k-th item into stage k % kQStages
        if (pre.l < l1) {
            uint32_t off, bytes, t0, nt;
            bool is_v;
            const uint8_t *src = src_of(pre, off, bytes, is_v);
            uint8_t *dst = wbuf + (k % kQStages) * STAGE;
            for (uint32_t c = lane; c < bytes / 16; c += 32) cp_async16(dst + 16 * c, src + 16 * c);
            if (!is_v) {
                tokens(off, t0, nt);
                if (nt <= TAB_TOK) {
                    const uint8_t *ts = reinterpret_cast<const uint8_t *>(gtab_job + t0 * PAIRS);
                    for (uint32_t c = lane; c < nt * PAIRS; c += 32)
                        cp_async16(dst + SEG + 16 * c, ts + 16 * c);
                }
            }
            pre.advance(nwarp, per_layer);
        }
        cp_async_commit();
    };
    if (!fresh) {
#pragma unroll
        for (int k = 0; k < kQStages - 1; ++k) issue(k);
    }
    for (uint32_t k = 0; cur.l < l1; ++k, cur.advance(nwarp, per_layer)) {
        uint32_t off, bytes, t0 = 0, nt = 0;
        bool is_v;
        const uint8_t *src = src_of(cur, off, bytes, is_v);
        uint8_t *buf = wbuf + (k % kQStages) * STAGE;
        if (fresh) {
            const uint4 *sp = reinterpret_cast<const uint4 *>(src);
            uint4 *rp = reinterpret_cast<uint4 *>(raw_slot + (src - slot));
            uint4 *bp = reinterpret_cast<uint4 *>(buf);
            for (uint32_t c = lane; c < bytes / 16; c += 32) {
                const uint4 v = sp[c];
                bp[c] = v;
                rp[c] = v;
            }
            __syncwarp();
        } else {
            issue(k + kQStages - 1);
            cp_async_wait<kQStages - 1>();
            __syncwarp();
        }
        uint8_t *dst = is_v ? a.win_v + static_cast<uint64_t>(cur.l) * g.win_v_layer + wv + off
                            : a.win_k + static_cast<uint64_t>(cur.l) * g.win_k_layer + wk + off;
        if (!is_v) {
            tokens(off, t0, nt);
            const bool staged = !fresh && nt <= TAB_TOK;
            const uint32_t row_base = off / HEAD_BYTES;
            convert_row<D, KT>(buf, lane, min(RPW, n_rows - row_base), row_base, hkv, n_rows,
                               staged ? reinterpret_cast<const float4 *>(buf + SEG) : gtab_job,
                               staged ? t0 : 0u, g.fwht_n, g.fwht_scale);
        }
        uint4 *dp = reinterpret_cast<uint4 *>(dst);
        const uint4 *bp = reinterpret_cast<const uint4 *>(buf);
        for (uint32_t c = lane; c < bytes / 16; c += 32) dp[c] = bp[c];
        __syncwarp();
    }
    if (!fresh) cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// S13, the GPU-resident step's quantised-K assembly: persistent warps fed by
// TMA bulk copies.
//
// Work: the flat sequence of items (job, layer, piece) over all fresh jobs,
// then all moved jobs; a piece is kQItemSegs 16-row K segments (converted one
// after the other) or the layer's whole V part (copied global to global by
// the warp's lanes, with no stage: V needs no conversion, and one item per V
// part keeps the per-item bookkeeping off the issue slots). Warps take chunks
// of kQChunk items from two counters the plan zeroes, so all warps finish
// together: the first warp of every CTA takes fresh chunks (host-link reads)
// until none is left and then moved ones, the other warps take moved chunks
// only, so the host-link reads and the HBM moves overlap. A warp streams its
// items through a ring of kQTmaStages shared-memory stages: one lane resolves
// the next item into the stage's descriptor and issues a 1-D bulk copy
// (cp.async.bulk, no multicast, this GPU's memory only) of its bytes
// (optionally also the cos/sin rows of the tokens a K segment spans, else
// those come from the position table through L1), completing on the stage's
// mbarrier, kQTmaStages - 2 items ahead of the item being converted; the
// converted stage goes back to the window with a bulk store. The conversion
// and the per-item bookkeeping (about 1,200 warp instructions per 16-row
// segment in all) bound the kernel, not the copies. Fresh items (host
// repository, read over the host link) are read with plain loads by the
// lanes, which also write them to their pool slot.
// Every mbarrier wait is bounded (2 s); on a timeout the warp records error
// 0x200 in the plan's error word, waits (bounded) for the copies it issued,
// and stops.
#ifndef KVMRET_Q_CHUNK
#define KVMRET_Q_CHUNK 8
#endif
// 1: a K stage also receives the cos/sin rows of its tokens (else they are
// read from the position table through L1)
#ifndef KVMRET_Q_TAB
#define KVMRET_Q_TAB 0
#endif
// 1: the GPU-resident step's quantised assembly runs the TMA-fed persistent
// kernel below; 0: the per-job kernel above (cp.async)
#ifndef KVMRET_Q_TMA
#define KVMRET_Q_TMA 1
#endif
// 16-byte loads a lane keeps in flight while it copies a V part
#ifndef KVMRET_Q_VU
#define KVMRET_Q_VU 16
#endif
// 16-row K segments per work item (one bulk copy, one descriptor), and the
// stages of a warp's ring: two segments per item halve the per-item
// bookkeeping (measured 6.6 % faster than one), and three stages of 4352
// bytes keep two CTAs of 8 warps per SM
#ifndef KVMRET_Q_ITEM_SEGS
#define KVMRET_Q_ITEM_SEGS 2
#endif
#ifndef KVMRET_Q_TMA_STAGES
#define KVMRET_Q_TMA_STAGES 3
#endif
constexpr uint32_t kQChunk = KVMRET_Q_CHUNK;
constexpr uint32_t kQItemSegs = KVMRET_Q_ITEM_SEGS;
constexpr uint32_t kQTmaStages = KVMRET_Q_TMA_STAGES;
// 1: a K item that follows the previous one in the same (job, layer) is
// resolved by stepping that item's addresses; 2: the same, checked against
// the full resolution (a mismatch sets 0x400 in the plan's error word)
#ifndef KVMRET_Q_CURSOR
#define KVMRET_Q_CURSOR 1
#endif
constexpr uint32_t kQCursor = KVMRET_Q_CURSOR;
constexpr uint32_t kQVUnroll = KVMRET_Q_VU;
constexpr uint32_t kQTmaTab = KVMRET_Q_TAB ? kQTabBytes : 0;
constexpr uint32_t kQNone = 0xffffffffu;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if (i == 0) t0 = globaltimer_ns();
        else if ((i & 63) == 0 && globaltimer_ns() - t0 > 2000000000ull) return false;
    }
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void bulk_store(void *dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                 "r"(src), "r"(bytes)
                 : "memory");
}

// One item of the sequence, resolved: where its bytes come from and go to.
struct QItem {
    const uint8_t *src;   // pool (moved) or host repository (fresh)
    uint8_t *raw;         // fresh: its pool slot bytes, else null
    uint8_t *dst;         // window bytes
    const float4 *tab;    // K: cos/sin rows of the job's first token
    uint32_t bytes, off, n_rows, is_v;
};

// The job of the last resolved item, kept by the issuing lane: a chunk's
// items almost always share one job, so its fields are read from global
// memory once per job instead of once per item.
struct JobCache {
    uint32_t ji = 0xffffffffu;
    Job job;
};

// Item idx of the sequence: per job, per layer, the nk K segments of SEG
// bytes, then the layer's whole V part as one item (copied directly).
template <int D, int KT>
__device__ __forceinline__ bool q_item(const AsmLaunch &a, uint32_t idx, uint32_t n_fresh,
                                       uint32_t per_job, const DivU32 &div_job, uint32_t nk,
                                       const DivU32 &div_items, JobCache &jc, QItem &it,
                                       uint32_t &si_out, uint32_t &ktotal_out) {
    constexpr uint32_t SEG = kQItemSegs * kQSegBlocks * QBlk<KT>::bytes;
    const AssembleGeom &g = a.g;
    const bool fresh = idx < n_fresh * per_job;
    const uint32_t rel = fresh ? idx : idx - n_fresh * per_job;
    const uint32_t j = div_job.div(rel), rem = rel - j * per_job;
    const uint32_t l = div_items.div(rem), si = rem - l * (nk + 1);
    const uint32_t ji = fresh ? a.fresh_offset + j : j;
    if (jc.ji != ji) {
        jc.job = a.jobs[ji];
        jc.ji = ji;
    }
    const Job *jp = &jc.job;
    const uint32_t n_tok = jp->n_tok;
    si_out = si;
    ktotal_out = n_tok * static_cast<uint32_t>(g.k_row);
    it.is_v = si >= nk;
    it.off = it.is_v ? 0u : si * SEG;
    const uint32_t total = n_tok * static_cast<uint32_t>(it.is_v ? g.v_row : g.k_row);
    if (it.off >= total) return false;  // past a partial block's rows
    it.bytes = it.is_v ? total : min(SEG, total - it.off);
    const uint64_t part = static_cast<uint64_t>(l) * g.unit + (it.is_v ? g.unit_k : 0) + it.off;
    const uint32_t ws = jp->win_slot;
    it.dst = it.is_v ? a.win_v + static_cast<uint64_t>(l) * g.win_v_layer +
                           static_cast<uint64_t>(ws) * g.block_tokens * g.v_row + it.off
                     : a.win_k + static_cast<uint64_t>(l) * g.win_k_layer +
                           static_cast<uint64_t>(ws) * g.block_tokens * g.k_row + it.off;
    if (fresh) {
        it.src = a.repo + static_cast<uint64_t>(jp->block) * a.slot_bytes + part;
        it.raw = a.pool_w + static_cast<uint64_t>(jp->pool_slot) * a.slot_bytes + part;
    } else {
        it.src = a.pool + static_cast<uint64_t>(jp->pool_slot) * a.slot_bytes + part;
        it.raw = nullptr;
    }
    it.tab = a.gtab + static_cast<size_t>(jp->pos0) * (D / 4);
    it.n_rows = n_tok * g.n_head_kv;
    return true;
}

// A stage's item, resolved once at issue time by the issuing lane.
struct QDesc {
    QItem it;
    uint32_t idx;    // item index, kQNone: the sequence has ended
    uint32_t kind;   // 0 nothing to do, 1 moved K (bulk-loaded), 2 fresh K (plain loads),
                     // 3 V (copied directly by the warp)
    uint32_t t0;     // first token of a K segment
    uint32_t staged; // its cos/sin rows are in the stage
    uint32_t si;     // the item's index within its (job, layer)
    uint32_t ktotal; // K bytes of its (job, layer)
};

template <int D, int KT>
__global__ void __launch_bounds__(kQThreads, KVMRET_Q_MINB)
    assemble_quant_tma_kernel(const __grid_constant__ AsmLaunch a) {
    dep_wait();
    constexpr uint32_t SEG = kQSegBlocks * QBlk<KT>::bytes;  // one warp's 16 rows
    constexpr uint32_t SEGI = kQItemSegs * SEG;               // a K item
    constexpr uint32_t STAGE = SEGI + kQTmaTab;
    constexpr uint32_t PAIRS = D / 4, TAB_TOK = kQTmaTab / (PAIRS * sizeof(float4));
    constexpr uint32_t HEAD_BYTES = (D / 32) * QBlk<KT>::bytes;
    constexpr uint32_t RPW = SEG / HEAD_BYTES, RPI = kQItemSegs * RPW;
    constexpr uint32_t S = kQTmaStages, P = kQTmaStages - 2;
    static_assert(kQTmaStages >= 3, "the ring needs a stage for the store in flight");
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const AssembleGeom &g = a.g;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    uint8_t *wbuf = smem_raw + warp * S * STAGE;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw + nwarp * S * STAGE) + warp * S;
    QDesc *desc = reinterpret_cast<QDesc *>(smem_raw + nwarp * S * (STAGE + 8)) + warp * S;
    const uint32_t T = g.block_tokens;
    const uint32_t nk = (T * static_cast<uint32_t>(g.k_row) + SEGI - 1) / SEGI;
    const uint32_t n_items_job = nk + 1, per_job = g.n_layer * n_items_job;
    const DivU32 div_job(per_job), div_items(n_items_job);
    const uint32_t n_moved = a.counts[0], n_fresh = a.counts[1];
    const uint32_t n_fi = n_fresh * per_job, n_mi = n_moved * per_job;  // items per kind
    const FastDiv hkv(g.n_head_kv);
    if (lane == 0) {
        for (uint32_t s = 0; s < S; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bars + s))
                         : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();

    // the warp's item sequence, kept by lane 0 alone: chunks from a work
    // counter; kind 0 = fresh items (counter a.work), 1 = moved items
    // (a.work_moved). The chunk after the current one is claimed when the
    // current one starts, so the atomic's result arrives while the chunk's
    // items are converted (a claim past the end is harmless: it is ignored).
    uint32_t kind = warp == 0 ? 0u : 1u;
    auto claim = [&]() { return atomicAdd(kind == 0 ? a.work : a.work_moved, 1u); };
    auto n_of = [&]() { return kind == 0 ? n_fi : n_mi; };
    auto chunks = [&]() { return (n_of() + kQChunk - 1) / kQChunk; };
    uint32_t cur_chunk = 0, next_chunk = 0, pos = 0;
    if (lane == 0) {
        cur_chunk = claim();
        next_chunk = claim();
    }
    JobCache jc;
    auto next_item = [&]() -> uint32_t {  // lane 0 only
        for (;;) {
            if (cur_chunk >= chunks()) {
                if (kind == 1) return kQNone;
                kind = 1;  // fresh work done: join the moves
                cur_chunk = claim();
                next_chunk = claim();
                pos = 0;
                continue;
            }
            const uint32_t idx = cur_chunk * kQChunk + pos;
            if (pos < kQChunk && idx < n_of()) {
                ++pos;
                return kind == 0 ? idx : n_fi + idx;
            }
            cur_chunk = next_chunk;
            pos = 0;
            if (cur_chunk < chunks()) next_chunk = claim();
        }
    };
    // issue (lane 0): resolve the next item into the stage's descriptor, arm
    // the stage's barrier and start its bulk copies (moved items)
    auto issue = [&](uint32_t k) {
        if (lane != 0) return;
        const uint32_t s = k % S;
        const uint32_t idx = next_item();
        QDesc &d = desc[s];
        d.idx = idx;
        d.kind = 0;
        d.staged = 0;
        d.t0 = 0;
        if (idx == kQNone) return;
        bool ok;
        const QDesc &pd = desc[(k + S - 1) % S];  // the item issued before this one
        if (kQCursor && k > 0 && idx == pd.idx + 1 && (pd.kind == 1 || pd.kind == 2) &&
            pd.si + 1 < nk) {
            // the next K piece of the same (job, layer): the previous one, one
            // piece further on
            QItem it = pd.it;
            it.off += SEGI;
            ok = it.off < pd.ktotal;
            if (ok) {
                it.bytes = min(SEGI, pd.ktotal - it.off);
                it.src += SEGI;
                it.dst += SEGI;
                if (it.raw) it.raw += SEGI;
            }
            d.si = pd.si + 1;
            d.ktotal = pd.ktotal;
            if (kQCursor == 2) {  // checked form: the full resolution decides
                QItem ref;
                uint32_t rsi, rkt;
                const bool rok = q_item<D, KT>(a, idx, n_fresh, per_job, div_job, nk, div_items,
                                               jc, ref, rsi, rkt);
                if (rok != ok || rsi != d.si || rkt != d.ktotal ||
                    (ok && (ref.src != it.src || ref.dst != it.dst || ref.raw != it.raw ||
                            ref.tab != it.tab || ref.bytes != it.bytes || ref.off != it.off ||
                            ref.n_rows != it.n_rows || ref.is_v != it.is_v)))
                    atomicOr(const_cast<uint32_t *>(a.counts) + 4, 0x400u);
                it = ref;
                ok = rok;
            }
            d.it = it;
        } else {
            ok = q_item<D, KT>(a, idx, n_fresh, per_job, div_job, nk, div_items, jc, d.it, d.si,
                               d.ktotal);
        }
        if (!ok) return;
        if (d.it.is_v) {
            d.kind = 3;
            return;
        }
        uint32_t tab_bytes = 0;
        {
            const uint32_t row_base = d.it.off / HEAD_BYTES;
            d.t0 = hkv.div(row_base);
            const uint32_t nt = hkv.div(min(row_base + RPI, d.it.n_rows) - 1) - d.t0 + 1;
            if (!d.it.raw && nt <= TAB_TOK) {
                tab_bytes = nt * PAIRS * static_cast<uint32_t>(sizeof(float4));
                d.staged = 1;
            }
        }
        if (d.it.raw) {
            d.kind = 2;
            return;
        }
        d.kind = 1;
        const uint32_t bar = smem_addr(bars + s);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                     "r"(d.it.bytes + tab_bytes)
                     : "memory");
        const uint32_t buf = smem_addr(wbuf + s * STAGE);
        bulk_load(buf, d.it.src, d.it.bytes, bar);
        if (tab_bytes) bulk_load(buf + SEGI, d.it.tab + d.t0 * PAIRS, tab_bytes, bar);
    };

    uint32_t phase = 0;  // bit s: parity of stage s's next completion
    uint32_t issued = 0;
    for (; issued < P; ++issued) issue(issued);
    __syncwarp();
    bool failed = false;
    uint32_t c = 0;
    for (;; ++c) {
        const uint32_t s = c % S;
        const QDesc &d = desc[s];
        if (d.idx == kQNone) break;
        // the stage of item c + P last served item c + P - S, whose store
        // must have read its bytes; the store of item c - 1 may still run
        if (lane == 0)
            asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(S - P - 1)
                         : "memory");
        __syncwarp();
        issue(issued++);
        __syncwarp();
        const uint32_t dk = d.kind;
        if (dk == 3) {  // V: global to global, kQVUnroll x 16 bytes in flight per lane
            const QItem &it = d.it;
            const uint4 *sp = reinterpret_cast<const uint4 *>(it.src);
            uint4 *dp = reinterpret_cast<uint4 *>(it.dst);
            uint4 *rp = reinterpret_cast<uint4 *>(it.raw);
            const uint32_t nq = it.bytes / 16;
            constexpr uint32_t U = kQVUnroll;
            uint32_t q0 = 0;
            for (; q0 + 32 * U <= nq; q0 += 32 * U) {
                uint4 v[U];
#pragma unroll
                for (uint32_t u = 0; u < U; ++u) v[u] = sp[q0 + u * 32 + lane];
#pragma unroll
                for (uint32_t u = 0; u < U; ++u) {
                    dp[q0 + u * 32 + lane] = v[u];
                    if (rp) rp[q0 + u * 32 + lane] = v[u];
                }
            }
            for (uint32_t q = q0 + lane; q < nq; q += 32) {
                const uint4 v = sp[q];
                dp[q] = v;
                if (rp) rp[q] = v;
            }
        } else if (dk != 0) {
            uint8_t *buf = wbuf + s * STAGE;
            const QItem &it = d.it;
            if (dk == 2) {  // fresh: plain loads over the host link, also into the pool
                const uint4 *sp = reinterpret_cast<const uint4 *>(it.src);
                uint4 *rp = reinterpret_cast<uint4 *>(it.raw);
                uint4 *bp = reinterpret_cast<uint4 *>(buf);
                for (uint32_t q = lane; q < it.bytes / 16; q += 32) {
                    const uint4 v = sp[q];
                    bp[q] = v;
                    rp[q] = v;
                }
                __syncwarp();
            } else {
                if (!mbar_wait_bounded(smem_addr(bars + s), (phase >> s) & 1u)) {
                    failed = true;
                    break;
                }
                phase ^= 1u << s;
            }
#pragma unroll 1
            for (uint32_t h = 0; h < kQItemSegs; ++h) {  // the item's 16-row segments
                const uint32_t row_base = it.off / HEAD_BYTES + h * RPW;
                if (row_base >= it.n_rows) break;
                convert_row<D, KT>(buf + h * SEG, lane, min(RPW, it.n_rows - row_base), row_base,
                                   hkv, it.n_rows,
                                   d.staged ? reinterpret_cast<const float4 *>(buf + SEGI)
                                            : it.tab,
                                   d.staged ? d.t0 : 0u, g.fwht_n, g.fwht_scale);
            }
            // the lanes' writes to the stage before the bulk store reads it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) bulk_store(it.dst, smem_addr(buf), it.bytes);
        }
        if (lane == 0) asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    if (failed) {
        atomicOr(const_cast<uint32_t *>(a.counts) + 4, 0x200u);
        // wait (bounded) for the bulk loads this warp issued and has not
        // consumed: items c .. issued - 1
        for (uint32_t k = c; k < issued; ++k) {
            const uint32_t s = k % S;
            if (desc[s].kind != 1) continue;
            mbar_wait_bounded(smem_addr(bars + s), (phase >> s) & 1u);
            phase ^= 1u << s;
        }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
}

// ---------------------------------------------------------------------------
// S15, gen-reserve placement (llama-memory-kvmem.cpp:2314-2365, alloc_slot
// :1720-1741). The host chose the slots; one thread records every binding in
// order (a binding may evict the block an earlier one displaced).
__global__ void gen_bind_kernel(const __grid_constant__ GenBinds g) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    for (uint32_t i = 0; i < g.n; ++i) {
        const GenBind &b = g.b[i];
        if (b.evict_block >= 0) g.blk_slot[b.evict_block] = -1;
        g.win_id[b.win_slot] = static_cast<int32_t>(b.block);
        g.win_base[b.win_slot] = b.base;
        g.win_ntok[b.win_slot] = b.n_exist;
        g.blk_slot[b.block] = static_cast<int32_t>(b.pool_slot);
        g.slot_blk[b.pool_slot] = static_cast<int32_t>(b.block);
        g.slot_ntok[b.pool_slot] = b.n_exist;
        g.slot_used[b.pool_slot] = g.step;
    }
}

// The window and pool slots of a bound block, looked up on the device (a step
// may have moved the block to another window slot since it was bound).
__device__ __forceinline__ bool gen_slots(const GenWrite &a, uint32_t block, uint32_t &ws,
                                          uint32_t &ps, int32_t &base) {
    __shared__ int32_t s_ws;
    if (threadIdx.x == 0) s_ws = -1;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < a.win_slots; i += blockDim.x)
        if (a.win_id[i] == static_cast<int32_t>(block)) s_ws = static_cast<int32_t>(i);
    __syncthreads();
    const int32_t w = s_ws, p = a.blk_slot[block];
    if (w < 0 || p < 0) {
        if (threadIdx.x == 0) atomicExch(a.err, 1u);
        return false;
    }
    ws = static_cast<uint32_t>(w);
    ps = static_cast<uint32_t>(p);
    base = a.win_base[w];
    return true;
}

// f16 K: CTA = (layer, bound block).
template <int D>
__global__ void __launch_bounds__(256) gen_write_f16_kernel(const __grid_constant__ GenWrite a) {
    dep_wait();
    constexpr uint32_t PAIRS = D / 4;
    const AssembleGeom &g = a.g;
    const uint32_t l = blockIdx.x;
    const GenSeg sg = a.seg[blockIdx.y];
    uint32_t ws, ps;
    int32_t base;
    if (!gen_slots(a, sg.block, ws, ps, base)) return;
    uint8_t *pk = a.pool + static_cast<uint64_t>(ps) * a.slot_bytes + static_cast<uint64_t>(l) * g.unit;
    uint8_t *pv = pk + g.unit_k;
    uint8_t *wk = a.win_k + static_cast<uint64_t>(l) * g.win_k_layer +
                  static_cast<uint64_t>(ws) * g.block_tokens * g.k_row;
    uint8_t *wv = a.win_v + static_cast<uint64_t>(l) * g.win_v_layer +
                  static_cast<uint64_t>(ws) * g.block_tokens * g.v_row;
    if (sg.new_lo > sg.rebuild_lo) {  // rows already in the pool slot
        const uint32_t n = sg.new_lo - sg.rebuild_lo;
        rope_rows_f16<D, false>(pk + sg.rebuild_lo * g.k_row, wk + sg.rebuild_lo * g.k_row,
                                a.gtab + static_cast<size_t>(base + sg.rebuild_lo) * PAIRS, n,
                                g.n_head_kv, nullptr);
        copy16(pv + sg.rebuild_lo * g.v_row, wv + sg.rebuild_lo * g.v_row,
               static_cast<uint64_t>(n) * g.v_row);
    }
    const uint32_t n = sg.new_hi - sg.new_lo;
    const uint64_t row0 = static_cast<uint64_t>(l) * a.n_tok_append + sg.tok0;
    rope_rows_f16<D, true>(a.k_rows + row0 * g.k_row, wk + sg.new_lo * g.k_row,
                           a.gtab + static_cast<size_t>(base + sg.new_lo) * PAIRS, n,
                           g.n_head_kv, pk + sg.new_lo * g.k_row);
    copy16_host(a.v_rows + row0 * g.v_row, wv + sg.new_lo * g.v_row, pv + sg.new_lo * g.v_row,
                static_cast<uint64_t>(n) * g.v_row);
    if (l == 0 && threadIdx.x == 0) {
        a.win_ntok[ws] = sg.new_hi;
        a.slot_ntok[ps] = sg.new_hi;
    }
}

// Quantised K: CTA = (layer, bound block), each warp converts 16-row
// segments in shared memory (rows from the pool below new_lo, from the caller
// above it, the latter also stored unrotated into the pool slot).
constexpr int kGenQWarps = 4;
template <int D, int KT>
__global__ void __launch_bounds__(32 * kGenQWarps) gen_write_quant_kernel(const __grid_constant__ GenWrite a) {
    dep_wait();
    constexpr uint32_t SEG = kQSegBlocks * QBlk<KT>::bytes;
    constexpr uint32_t HEAD_BYTES = (D / 32) * QBlk<KT>::bytes;
    constexpr uint32_t RPW = SEG / HEAD_BYTES;
    constexpr uint32_t PAIRS = D / 4;
    __shared__ __align__(16) uint8_t sm[kGenQWarps][SEG];
    const AssembleGeom &g = a.g;
    const uint32_t l = blockIdx.x;
    const GenSeg sg = a.seg[blockIdx.y];
    uint32_t ws, ps;
    int32_t base;
    if (!gen_slots(a, sg.block, ws, ps, base)) return;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t kr = static_cast<uint32_t>(g.k_row), vr = static_cast<uint32_t>(g.v_row);
    uint8_t *pk = a.pool + static_cast<uint64_t>(ps) * a.slot_bytes + static_cast<uint64_t>(l) * g.unit;
    uint8_t *pv = pk + g.unit_k;
    uint8_t *wk = a.win_k + static_cast<uint64_t>(l) * g.win_k_layer +
                  static_cast<uint64_t>(ws) * g.block_tokens * g.k_row;
    uint8_t *wv = a.win_v + static_cast<uint64_t>(l) * g.win_v_layer +
                  static_cast<uint64_t>(ws) * g.block_tokens * g.v_row;
    const uint64_t row0 = static_cast<uint64_t>(l) * a.n_tok_append + sg.tok0;
    const uint8_t *ck = a.k_rows + row0 * kr;  // caller row of token new_lo
    const uint32_t n_rows = (sg.new_hi - sg.rebuild_lo) * g.n_head_kv;
    const uint32_t kbytes = (sg.new_hi - sg.rebuild_lo) * kr;
    const uint32_t lo_bytes = (sg.new_lo - sg.rebuild_lo) * kr;  // bytes served by the pool
    const FastDiv hkv(g.n_head_kv);
    const float4 *tab = a.gtab + static_cast<size_t>(base + sg.rebuild_lo) * PAIRS;
    uint8_t *buf = sm[warp];
    for (uint32_t off = warp * SEG; off < kbytes; off += kGenQWarps * SEG) {
        const uint32_t bytes = min(SEG, kbytes - off);
        for (uint32_t c = lane; c < bytes / 16; c += 32) {
            const uint32_t o = off + 16 * c;
            uint4 v;
            if (o < lo_bytes) {
                v = *reinterpret_cast<const uint4 *>(pk + sg.rebuild_lo * kr + o);
            } else {
                v = *reinterpret_cast<const uint4 *>(ck + (o - lo_bytes));
                *reinterpret_cast<uint4 *>(pk + sg.rebuild_lo * kr + o) = v;  // unrotated
            }
            *reinterpret_cast<uint4 *>(buf + 16 * c) = v;
        }
        __syncwarp();
        const uint32_t row_base = off / HEAD_BYTES;
        convert_row<D, KT>(buf, lane, min(RPW, n_rows - row_base), row_base, hkv, n_rows, tab, 0u,
                           g.fwht_n, g.fwht_scale);
        uint4 *dp = reinterpret_cast<uint4 *>(wk + sg.rebuild_lo * kr + off);
        for (uint32_t c = lane; c < bytes / 16; c += 32) dp[c] = reinterpret_cast<const uint4 *>(buf)[c];
        __syncwarp();
    }
    // V rows: pool part, then the caller's part (also into the pool)
    if (sg.new_lo > sg.rebuild_lo)
        copy16(pv + sg.rebuild_lo * vr, wv + sg.rebuild_lo * vr,
               static_cast<uint64_t>(sg.new_lo - sg.rebuild_lo) * vr);
    copy16_host(a.v_rows + row0 * vr, wv + sg.new_lo * vr, pv + sg.new_lo * vr,
                static_cast<uint64_t>(sg.new_hi - sg.new_lo) * vr);
    if (l == 0 && threadIdx.x == 0) {
        a.win_ntok[ws] = sg.new_hi;
        a.slot_ntok[ps] = sg.new_hi;
    }
}

// ---------------------------------------------------------------------------
// Truncation: the dropped blocks leave the block set, the HBM pool and the
// window (they are the newest blocks, so they sit at the window's end).
__global__ void __launch_bounds__(1024) truncate_kernel(const __grid_constant__ TruncArgs a) {
    for (uint32_t b = a.nb_new + threadIdx.x; b < a.nb_old; b += blockDim.x) {
        a.has_block[b] = 0;
        a.blk_ntok[b] = 0;
        a.blk_slot[b] = -1;
    }
    // the kept partial block: its window and pool copies hold valid rows only
    // up to tail_ntok (later appends may bring other tokens)
    const int32_t part = a.tail_ntok ? static_cast<int32_t>(a.nb_new) - 1 : -1;
    for (uint32_t s = threadIdx.x; s < a.pool_slots; s += blockDim.x) {
        if (a.slot_blk[s] >= static_cast<int32_t>(a.nb_new)) a.slot_blk[s] = -1;
        else if (a.slot_blk[s] == part) a.slot_ntok[s] = min(a.slot_ntok[s], a.tail_ntok);
    }
    for (uint32_t i = threadIdx.x; i < a.win_slots; i += blockDim.x) {
        if (a.win_id[i] >= static_cast<int32_t>(a.nb_new)) {
            a.win_id[i] = -1;
            a.win_ntok[i] = 0;
        } else if (a.win_id[i] == part) {
            a.win_ntok[i] = min(a.win_ntok[i], a.tail_ntok);
        }
    }
    if (threadIdx.x == 0 && a.tail_ntok && a.nb_new) a.blk_ntok[a.nb_new - 1] = a.tail_ntok;
}

// The summary of a truncated partial f16 block from the repository's K rows
// (the same token-order sum as append_summary_kernel; RawKvStore::truncate_to
// recomputes it from the stored K, raw_kv_store.cpp:1096-1126). CTA = layer.
__global__ void resum_kernel(AppendArgs a, uint32_t block, uint32_t n_tok) {
    const uint32_t l = blockIdx.x;
    const uint32_t E = a.n_head_kv * a.d_head;
    const float inv = __fdiv_rn(1.0f, static_cast<float>(n_tok));
    const uint16_t *k = reinterpret_cast<const uint16_t *>(
        a.repo_dev + (static_cast<uint64_t>(block) * a.n_layer + l) * a.unit);
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) {
        float s = 0.0f;
        for (uint32_t t = 0; t < n_tok; ++t) s = __fadd_rn(s, h2f(k[static_cast<size_t>(t) * E + e]));
        const uint32_t h = e / a.d_head, d = e % a.d_head;
        a.summ[((static_cast<size_t>(l) * a.n_head_kv + h) * a.d_head + d) * a.ncap + block] =
            __fmul_rn(s, inv);
        a.tail_sum[static_cast<size_t>(l) * E + e] = s;
    }
}

// ---------------------------------------------------------------------------
// S2 + S14: summaries of the appended tokens. CTA = (layer, touched block);
// thread e sums its channel over the block's new tokens in token order,
// continuing the trailing partial block's running sum
// (raw_kv_store.cpp:215-234), and stores sum * (1 / tokens) (:1000-1005).
__global__ void append_summary_kernel(AppendArgs a, const float *tail_in, float *tail_out) {
    dep_wait();
    const uint32_t l = blockIdx.x;
    const uint32_t E = a.n_head_kv * a.d_head;
    const uint32_t T = a.block_tokens;
    const uint32_t b = a.pos0 / T + blockIdx.y;
    const uint32_t tb = max(a.pos0, b * T);
    const uint32_t te = min(a.pos0 + a.n_tok, (b + 1) * T);
    const uint32_t off = tb - b * T;
    const uint32_t cnt = off + (te - tb);
    const float inv = __fdiv_rn(1.0f, static_cast<float>(cnt));
    const uint16_t *src = a.k_cap + static_cast<size_t>(l) * a.n_tok * E;
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) {
        float s = off == 0 ? 0.0f : tail_in[static_cast<size_t>(l) * E + e];
        for (uint32_t t = tb; t < te; ++t)
            s = __fadd_rn(s, h2f(src[static_cast<size_t>(t - a.pos0) * E + e]));
        const uint32_t h = e / a.d_head, d = e % a.d_head;
        a.summ[((static_cast<size_t>(l) * a.n_head_kv + h) * a.d_head + d) * a.ncap + b] =
            __fmul_rn(s, inv);
        if (cnt < T) tail_out[static_cast<size_t>(l) * E + e] = s;
    }
    if (l == 0 && threadIdx.x == 0) {
        a.has_block[b] = 1;
        if (a.blk_ntok) a.blk_ntok[b] = cnt;
    }
}

// Repository rows: each (layer, token) K and V row goes to
// repo[block][layer][K | V] + token offset, over the mapped host pointer.
__global__ void append_repo_kernel(AppendArgs a) {
    dep_wait();
    const uint32_t l = blockIdx.y;
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (warp >= a.n_tok) return;
    const uint32_t pos = a.pos0 + warp;
    const uint32_t b = pos / a.block_tokens, off = pos % a.block_tokens;
    uint8_t *unit = a.repo_dev + (static_cast<uint64_t>(b) * a.n_layer + l) * a.unit;
    const uint4 *ks = reinterpret_cast<const uint4 *>(
        a.k_rows + (static_cast<uint64_t>(l) * a.n_tok + warp) * a.k_row);
    uint4 *kd = reinterpret_cast<uint4 *>(unit + off * a.k_row);
    for (uint64_t w = lane; w < a.k_row / 16; w += 32) kd[w] = __ldg(ks + w);
    const uint4 *vs = reinterpret_cast<const uint4 *>(
        a.v_rows + (static_cast<uint64_t>(l) * a.n_tok + warp) * a.v_row);
    uint4 *vd = reinterpret_cast<uint4 *>(unit + a.unit_k + off * a.v_row);
    for (uint64_t w = lane; w < a.v_row / 16; w += 32) vd[w] = __ldg(vs + w);
}

// f16 rows -> q8_0 / q4_0 rows, one thread per 32-element block
// (quant_q8_0 / quant_q4_0, llama-kvmem-stagein.cu:181-234).
__global__ void quantize_kernel(const uint16_t *__restrict__ x, uint8_t *__restrict__ y,
                                uint64_t n_blocks, int q8) {
    const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (i >= n_blocks) return;
    float v[32];
    const uint4 *src = reinterpret_cast<const uint4 *>(x + i * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 w = __ldg(src + c);
        const uint16_t *h = reinterpret_cast<const uint16_t *>(&w);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[c * 8 + e] = h2f(h[e]);
    }
    if (q8) {
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint8_t *b = y + i * 34;
        *reinterpret_cast<uint16_t *>(b) = f2h(d);
#pragma unroll
        for (int j = 0; j < 32; ++j)
            b[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(roundf(__fmul_rn(v[j], id))));
    } else {
        float amax = 0.0f, vmax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (amax < fabsf(v[j])) {
                amax = fabsf(v[j]);
                vmax = v[j];
            }
        const float d = __fdiv_rn(vmax, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint8_t *b = y + i * 18;
        *reinterpret_cast<uint16_t *>(b) = f2h(d);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            int x0 = static_cast<int>(__fadd_rn(__fmul_rn(v[j], id), 8.5f));
            int x1 = static_cast<int>(__fadd_rn(__fmul_rn(v[j + 16], id), 8.5f));
            x0 = x0 > 15 ? 15 : x0;
            x1 = x1 > 15 ? 15 : x1;
            b[2 + j] = static_cast<uint8_t>((x0 & 15) | ((x1 & 15) << 4));
        }
    }
}

// ---------------------------------------------------------------------------
// Device plan (one CTA). Every array index below derives from n_blocks,
// win_slots and pool_slots, whose sizes the host checked against the buffers.
// 512 threads: the plan is bound by its block-wide barriers and scans, which
// cost less with fewer warps (config 2, 8-layer cut: 10.5 us against 13.9 us
// with 1024 threads and 12.2 us with 256)
#ifndef KVMRET_PLAN_THREADS
#define KVMRET_PLAN_THREADS 512
#endif
constexpr int kPlanThreads = KVMRET_PLAN_THREADS;

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs a) {
    dep_wait();
    using Scan = cub::BlockScan<uint32_t, kPlanThreads>;
    __shared__ typename Scan::TempStorage ts;
    __shared__ uint32_t s_err, s_mtok, s_ftok;
    __shared__ SelSmem rsm;
    extern __shared__ __align__(16) uint32_t psm[];
    const uint32_t W = a.win_slots, P = a.pool_slots, tid = threadIdx.x;
    uint32_t *s_ids = psm;
    int32_t *s_base = reinterpret_cast<int32_t *>(psm + W);
    uint32_t *s_ntok = psm + 2 * W;
    int32_t *s_slot = reinterpret_cast<int32_t *>(psm + 3 * W);
    uint32_t *s_flag = psm + 4 * W;  // bit 0: stage from the host, bit 1: needs a slot
    uint32_t *s_free = psm + 5 * W;  // [P]
    uint32_t *s_cu = psm + 5 * W + P;  // [P] eviction key: slot_used, ~0u if not a candidate
    uint32_t *s_ev = psm + 5 * W + 2 * P;  // [P] evicted slots in slot order
    if (tid == 0) s_err = a.ext_err ? atomicExch(a.ext_err, 0u) : 0u;  // consumed once
    __syncthreads();
    if (s_err) {  // a rank's score rows never arrived: keep the window, pool and plan as they are
        if (tid == 0) {
            for (int i = 0; i < 9; ++i) a.counts[i] = 0;
            a.counts[4] = 0x100u;
        }
        return;
    }
    if (tid == 0) s_mtok = 0, s_ftok = 0;

    // 1. selected ids ascending with their chronological bases
    const uint32_t n = a.n_blocks;
    const uint32_t C = (n + kPlanThreads - 1) / kPlanThreads;
    const uint32_t b0 = min(n, tid * C), b1 = min(n, b0 + C);
    uint32_t cnt = 0, tok = 0;
    for (uint32_t b = b0; b < b1; ++b)
        if (a.sel[b]) ++cnt, tok += a.blk_ntok[b];
    uint32_t pos, total, tpos, ttotal;
    Scan(ts).ExclusiveSum(cnt, pos, total);
    __syncthreads();
    Scan(ts).ExclusiveSum(tok, tpos, ttotal);
    __syncthreads();
    for (uint32_t b = b0; b < b1; ++b)
        if (a.sel[b]) {
            if (pos < W) {
                s_ids[pos] = b;
                s_base[pos] = static_cast<int32_t>(tpos);
                s_ntok[pos] = a.blk_ntok[b];
            }
            ++pos;
            tpos += a.blk_ntok[b];
        }
    if (tid == 0 && total > W) s_err = 1;
    const uint32_t n_sel = min(total, W);
    __syncthreads();

    // 2. without caching, blocks that left the selection give their slot back
    if (!a.pool_cache)
        for (uint32_t s = tid; s < P; s += kPlanThreads) {
            const int32_t b = a.slot_blk[s];
            if (b >= 0 && !a.sel[b]) {
                a.slot_blk[s] = -1;
                a.blk_slot[b] = -1;
            }
        }
    __syncthreads();

    // 3. which window blocks need their pool copy (re)staged, and a slot
    const uint32_t Cw = (n_sel + kPlanThreads - 1) / kPlanThreads;
    const uint32_t i0 = min(n_sel, tid * Cw), i1 = min(n_sel, i0 + Cw);
    uint32_t need = 0;
    for (uint32_t i = i0; i < i1; ++i) {
        const int32_t sl = a.blk_slot[s_ids[i]];
        uint32_t f = 0;
        if (sl < 0) f = 3, ++need;
        else if (a.slot_ntok[sl] != s_ntok[i]) f = 1;
        s_slot[i] = sl;
        s_flag[i] = f;
    }
    uint32_t need_rank, n_need;
    Scan(ts).ExclusiveSum(need, need_rank, n_need);
    __syncthreads();
    const uint32_t Cp = (P + kPlanThreads - 1) / kPlanThreads;
    const uint32_t p0 = min(P, tid * Cp), p1 = min(P, p0 + Cp);
    uint32_t fc = 0;
    for (uint32_t s = p0; s < p1; ++s) fc += a.slot_blk[s] < 0 ? 1u : 0u;
    uint32_t frank, n_free;
    Scan(ts).ExclusiveSum(fc, frank, n_free);
    __syncthreads();
    for (uint32_t s = p0; s < p1; ++s)
        if (a.slot_blk[s] < 0) s_free[frank++] = s;
    __syncthreads();
    if (n_need > n_free) {  // cache mode: evict least recently used blocks outside the window
        const uint32_t deficit = n_need - n_free;
        // Candidates are pooled blocks outside the new window, ordered by
        // (slot_used, slot). Their key is staged in shared memory (~0u marks a
        // non-candidate; slot_used never reaches it); a radix selection finds
        // the `deficit` least recently used, which are then ranked among
        // themselves so that the k-th victim takes free-list position k.
        for (uint32_t s = tid; s < P; s += kPlanThreads) {
            const int32_t b = a.slot_blk[s];
            s_cu[s] = (b < 0 || a.sel[b]) ? 0xffffffffu : a.slot_used[s];
        }
        __syncthreads();
        auto lru_key = [&](uint32_t s, uint64_t &key) -> bool {
            const uint32_t u = s_cu[s];
            if (u == 0xffffffffu) return false;
            key = (static_cast<uint64_t>(u) << 32) | s;
            return true;
        };
        // the two candidate lists of the selection (u16 slots) live in s_ev
        // until the victims are known
        uint16_t *la = reinterpret_cast<uint16_t *>(s_ev);
        block_select_u64(P, deficit, lru_key, la, la + P, P, rsm);
        const uint32_t mode = rsm.mode, n_cand = rsm.n_valid;
        const uint64_t thr = rsm.thr;  // keys are distinct: never a tie
        uint32_t ec = 0;
        for (uint32_t s = p0; s < p1; ++s) {
            uint64_t key;
            if (lru_key(s, key) && (mode == kSelAll || (mode >= kSelExact && key <= thr))) ++ec;
        }
        uint32_t erank, n_ev;
        Scan(ts).ExclusiveSum(ec, erank, n_ev);
        __syncthreads();
        for (uint32_t s = p0; s < p1; ++s) {
            uint64_t key;
            if (lru_key(s, key) && (mode == kSelAll || (mode >= kSelExact && key <= thr)))
                s_ev[erank++] = s;
        }
        __syncthreads();
        // n_ev <= deficit <= the window's stage-ins: the quadratic rank below
        // is bounded by the blocks this step copies from the host
        for (uint32_t k = tid; k < n_ev; k += kPlanThreads) {
            const uint32_t s = s_ev[k];
            const uint64_t key = (static_cast<uint64_t>(s_cu[s]) << 32) | s;
            uint32_t r = 0;
            for (uint32_t j = 0; j < n_ev; ++j) {
                const uint32_t s2 = s_ev[j];
                r += ((static_cast<uint64_t>(s_cu[s2]) << 32) | s2) < key ? 1u : 0u;
            }
            s_free[n_free + r] = s;
            a.blk_slot[a.slot_blk[s]] = -1;
        }
        __syncthreads();
        for (uint32_t k = tid; k < n_ev; k += kPlanThreads) a.slot_blk[s_free[n_free + k]] = -1;
        if (tid == 0 && n_cand < deficit) s_err |= 2;
        n_free += n_ev;
        __syncthreads();
    }
    for (uint32_t i = i0; i < i1; ++i)
        if (s_flag[i] & 2) {
            const uint32_t k = need_rank++;
            if (k < n_free) {
                const uint32_t s = s_free[k];
                s_slot[i] = static_cast<int32_t>(s);
                a.blk_slot[s_ids[i]] = static_cast<int32_t>(s);
                a.slot_blk[s] = static_cast<int32_t>(s_ids[i]);
            } else {
                atomicOr(&s_err, 4u);
            }
        }
    __syncthreads();

    // 4. job lists and the new window
    uint32_t mv = 0, fr = 0;
    for (uint32_t i = i0; i < i1; ++i) {
        const bool stage = s_flag[i] & 1;
        const bool changed = a.win_id[i] != static_cast<int32_t>(s_ids[i]) ||
                             a.win_base[i] != s_base[i] || a.win_ntok[i] != s_ntok[i];
        fr += stage ? 1u : 0u;
        mv += (!stage && changed) ? 1u : 0u;
    }
    uint32_t mrank, n_moved, frk, n_fresh;
    Scan(ts).ExclusiveSum(mv, mrank, n_moved);
    __syncthreads();
    Scan(ts).ExclusiveSum(fr, frk, n_fresh);
    __syncthreads();
    for (uint32_t i = i0; i < i1; ++i) {
        const bool stage = s_flag[i] & 1;
        const bool changed = a.win_id[i] != static_cast<int32_t>(s_ids[i]) ||
                             a.win_base[i] != s_base[i] || a.win_ntok[i] != s_ntok[i];
        const int32_t sl = s_slot[i];
        if (sl >= 0 && (stage || changed)) {
            Job j{};
            j.pool_slot = static_cast<uint32_t>(sl);
            j.win_slot = i;
            j.pos0 = s_base[i];
            j.n_tok = s_ntok[i];
            j.block = s_ids[i];
            if (stage) {
                a.jobs[W + frk++] = j;
                a.slot_ntok[sl] = s_ntok[i];
                atomicAdd(&s_ftok, s_ntok[i]);
            } else {
                a.jobs[mrank++] = j;
                atomicAdd(&s_mtok, s_ntok[i]);
            }
        }
        if (sl >= 0) a.slot_used[sl] = a.step;
        a.win_id[i] = static_cast<int32_t>(s_ids[i]);
        a.win_base[i] = s_base[i];
        a.win_ntok[i] = s_ntok[i];
        a.ids[i] = s_ids[i];
    }
    for (uint32_t i = n_sel + tid; i < W; i += kPlanThreads) {
        a.win_id[i] = -1;
        a.win_ntok[i] = 0;
    }
    __syncthreads();
    if (tid == 0) {
        a.counts[0] = n_moved;
        a.counts[1] = n_fresh;
        a.counts[2] = n_sel;
        a.counts[3] = ttotal;
        a.counts[4] = s_err;
        a.counts[5] = s_mtok;
        a.counts[6] = s_ftok;
        a.counts[7] = 0;  // the assembly's work counters
        a.counts[8] = 0;
    }
}

__global__ void copy_ops_kernel(const CopyOp *__restrict__ ops, int n) {
    const int i = blockIdx.x;
    if (i >= n) return;
    const CopyOp op = ops[i];
    if (!op.src || !op.dst || op.nbytes == 0) return;
    const uintptr_t al = reinterpret_cast<uintptr_t>(op.src) | reinterpret_cast<uintptr_t>(op.dst);
    if ((al & 15u) == 0 && (op.nbytes & 15u) == 0) {
        copy16(op.src, op.dst, op.nbytes);
        return;
    }
    for (uint64_t j = threadIdx.x; j < op.nbytes; j += blockDim.x) op.dst[j] = op.src[j];
}

// Layers per CTA: up to 8 (one RoPE table serves them all), fewer when the
// launch has few jobs so the grid still covers every SM several times.
uint32_t layers_per_cta(uint32_t n_jobs, uint32_t n_layer) {
    const uint64_t units = static_cast<uint64_t>(n_jobs) * n_layer;
    uint64_t lpc = units / (148ull * 8);
    lpc = lpc < 1 ? 1 : (lpc > 8 ? 8 : lpc);
    return static_cast<uint32_t>(lpc < n_layer ? lpc : n_layer);
}

uint32_t layers_per_cta_for(const AsmLaunch &a, uint32_t n_jobs) {
    // With device counts the job total is unknown here; n_jobs is then the
    // grid's upper bound and the layer split follows the layer count alone.
    return a.counts ? (a.g.n_layer <= 8 ? 1u : a.g.n_layer <= 16 ? 2u
                                             : a.g.n_layer <= 32 ? 4u : 8u)
                    : layers_per_cta(n_jobs, a.g.n_layer);
}

template <int D>
cudaError_t launch_assemble_t(const AsmLaunch &a, uint32_t n_jobs, cudaStream_t st) {
    auto kfn = assemble_kernel<D>;
    if (!a.counts) {
        return launch_dep(kfn, dim3(n_jobs), dim3(kAsmThreads), 0, st, a);
    }
    // persistent: as many CTAs as fit on the device at once
    static int per_sm = 0, n_sm = 0;
    if (per_sm == 0) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess)
            e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kAsmThreads, 0);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) per_sm = 1;
    }
    return launch_dep(kfn, dim3(static_cast<uint32_t>(per_sm * n_sm)), dim3(kAsmThreads), 0, st,
                      a);
}

template <int D, int KT>
cudaError_t launch_assemble_quant_t(const AsmLaunch &a, uint32_t n_jobs, cudaStream_t st) {
    if (a.counts && KVMRET_Q_TMA) {  // the GPU-resident step: persistent TMA-fed warps
        constexpr uint32_t STAGE = kQItemSegs * kQSegBlocks * QBlk<KT>::bytes + kQTmaTab;
        const size_t smem =
            static_cast<size_t>(kQThreads / 32) * kQTmaStages * (STAGE + 8 + sizeof(QDesc));
        auto kfn = assemble_quant_tma_kernel<D, KT>;
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        static int per_sm = 0, n_sm = 0;
        if (e == cudaSuccess && per_sm == 0) {
            int dev = 0;
            e = cudaGetDevice(&dev);
            if (e == cudaSuccess)
                e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kQThreads, smem);
            if (per_sm < 1) per_sm = 1;
        }
        if (e != cudaSuccess) return e;
        return launch_dep(kfn, dim3(static_cast<uint32_t>(per_sm * n_sm)), dim3(kQThreads), smem,
                          st, a);
    }
    const uint32_t lpc = layers_per_cta_for(a, n_jobs);
    const uint32_t groups = (a.g.n_layer + lpc - 1) / lpc;
    AsmLaunch al = a;
    al.n_groups = groups;
    const dim3 grid = a.counts ? dim3(n_jobs * groups, 1) : dim3(n_jobs, groups);
    const size_t smem = static_cast<size_t>(kQThreads / 32) * kQStages *
                        (kQSegBlocks * QBlk<KT>::bytes + kQTabBytes);
    auto kfn = assemble_quant_kernel<D, KT>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_dep(kfn, grid, dim3(kQThreads), smem, st, al, lpc);
}

}  // namespace

cudaError_t launch_query_add(float *q_sum, const void *rows, bool rows_f16, uint32_t n_layer,
                             uint32_t n_rows, uint32_t qdim, cudaStream_t st, uint32_t *q_count,
                             bool assign) {
    const dim3 grid((qdim + 255) / 256, n_layer);
    const int as = assign ? 1 : 0;
    if (rows_f16)
        return launch_dep(query_add_kernel<uint16_t>, grid, dim3(256), 0, st, q_sum,
                          static_cast<const uint16_t *>(rows), n_rows, qdim, q_count, as);
    return launch_dep(query_add_kernel<float>, grid, dim3(256), 0, st, q_sum,
                      static_cast<const float *>(rows), n_rows, qdim, q_count, as);
}

cudaError_t launch_qprep(const float *q_sum, const uint32_t *q_count, float *qv, float *nq,
                         uint8_t *active, uint32_t n_layer, uint32_t n_head, uint32_t n_head_kv,
                         uint32_t d_head, cudaStream_t st, double *flag_col, uint32_t cstride) {
    return launch_dep(qprep_kernel, dim3(n_layer, n_head_kv), dim3(d_head), d_head * sizeof(float), st,
                      
        q_sum, q_count, qv, nq, active, n_head, n_head_kv, d_head, flag_col, cstride);
    
}

template <int D, int V>
cudaError_t launch_score_tv(const float *summ, const float *qv, const float *nq,
                            const uint8_t *active, double *contrib, uint32_t n_layer,
                            uint32_t n_head_kv, uint32_t ncap, uint32_t tiles, uint32_t slots,
                            size_t smem, cudaStream_t st, uint32_t cstride, const Peers &peers) {
    const uint32_t n_units = tiles * n_layer;
    const uint32_t per_cta = (n_units + slots - 1) / slots;
    const uint32_t grid = (n_units + per_cta - 1) / per_cta;
    return launch_dep(score_kernel<D, V>, dim3(grid), dim3(256), smem, st, summ, qv, nq, active,
                      contrib, n_head_kv, ncap, cstride, tiles, n_units, per_cta, peers);
}

// As many units per CTA as it takes for one wave of resident CTAs, then as few
// CTAs as carry them all: every CTA gets the same share. With fewer 64-block
// units than resident CTAs (few layers per GPU) the tile shrinks to 32 blocks
// so more CTAs keep loads in flight. Measured (score kernel, one GPU, live):
// 8 layers 24.6 us (32-block) against 39.2 us (64-block), 16 layers 41.1
// against 47.0, 32 layers 71.9 against 64.9 (there the 64-block tiles fill
// the resident CTAs and their float2 loads win).
template <int D>
cudaError_t launch_score_t(const float *summ, const float *qv, const float *nq,
                           const uint8_t *active, double *contrib, uint32_t n_layer,
                           uint32_t n_head_kv, uint32_t ncap, uint32_t n_blocks, cudaStream_t st,
                           uint32_t cstride, const Peers &peers) {
    int per_sm = 0, n_sm = 0, dev = 0;
    const size_t smem64 = static_cast<size_t>(n_head_kv) * (D + 64) * sizeof(float);
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, score_kernel<D, 2>, 256, smem64);
    if (e != cudaSuccess) return e;
    const uint32_t slots = static_cast<uint32_t>(std::max(1, per_sm) * std::max(1, n_sm));
    const uint32_t tiles64 = (n_blocks + 63) / 64;
    if (tiles64 * n_layer >= slots)
        return launch_score_tv<D, 2>(summ, qv, nq, active, contrib, n_layer, n_head_kv, ncap,
                                     tiles64, slots, smem64, st, cstride, peers);
    const size_t smem32 = static_cast<size_t>(n_head_kv) * (D + 32) * sizeof(float);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, score_kernel<D, 1>, 256, smem32);
    if (e != cudaSuccess) return e;
    const uint32_t slots1 = static_cast<uint32_t>(std::max(1, per_sm) * std::max(1, n_sm));
    return launch_score_tv<D, 1>(summ, qv, nq, active, contrib, n_layer, n_head_kv, ncap,
                                 (n_blocks + 31) / 32, slots1, smem32, st, cstride, peers);
}

cudaError_t launch_score(const float *summ, const float *qv, const float *nq,
                         const uint8_t *active, double *contrib, uint32_t n_layer,
                         uint32_t n_head_kv, uint32_t d_head, uint32_t ncap, uint32_t n_blocks,
                         cudaStream_t st, uint32_t cstride, const Peers *peers_in) {
    if (cstride == 0) cstride = ncap;
    if (n_blocks == 0) {
        if (peers_in && peers_in->n > 1)
            return launch_dep(exchange_signal_kernel, dim3(1), dim3(256), 0, st, *peers_in);
        return cudaSuccess;
    }
    Peers none{};
    const Peers &peers = peers_in ? *peers_in : none;
    switch (d_head) {
    case 64:
        return launch_score_t<64>(summ, qv, nq, active, contrib, n_layer, n_head_kv, ncap,
                                   n_blocks, st, cstride, peers);
    case 128:
        return launch_score_t<128>(summ, qv, nq, active, contrib, n_layer, n_head_kv, ncap,
                                   n_blocks, st, cstride, peers);
    case 256:
        return launch_score_t<256>(summ, qv, nq, active, contrib, n_layer, n_head_kv, ncap,
                                   n_blocks, st, cstride, peers);
    default:
        return cudaErrorInvalidValue;
    }
}

cudaError_t launch_reduce(const double *contrib, const uint8_t *active, uint32_t n_layer,
                          uint32_t stride, const uint8_t *has_block, uint32_t n_blocks,
                          double *scores, cudaStream_t st, const uint32_t *wait_flags,
                          uint32_t wait_n, uint32_t wait_step, uint32_t *err,
                          const RowSource *rows) {
    // with an exchange to wait for, one CTA still takes part in the step
    // protocol when there is nothing to reduce
    if (n_blocks == 0 && !wait_flags) return cudaSuccess;
    RowSource none{};
    return launch_dep(reduce_kernel, dim3(std::max(1u, (n_blocks + 127) / 128)), dim3(128), n_layer, st,
                      contrib, active, n_layer, stride, has_block, n_blocks, scores, wait_flags,
                      wait_n, wait_step, err, rows ? *rows : none);
}

cudaError_t launch_select(const double *scores, const uint8_t *kept, uint32_t n_blocks,
                          uint32_t need, int tie_higher_id, uint8_t *sel, cudaStream_t st) {
    if (n_blocks == 0) return cudaSuccess;
    if (n_blocks <= kSelectStagedMax) {  // keys (8 B) and two u16 lists per block
        const size_t smem = static_cast<size_t>(n_blocks) * (8 + 2 * 2);
        auto kfn = select_radix_kernel<true>;
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        // small sets: fewer warps make the block-wide barriers of each pass cheaper
        const uint32_t threads = n_blocks <= KVMRET_SEL_SMALL_N ? KVMRET_SEL_SMALL_THREADS : 1024;
        return launch_dep(kfn, dim3(1), dim3(threads), smem, st, scores, kept, n_blocks, need,
                          tie_higher_id, sel, n_blocks);
    }
    const size_t smem = 2ull * kSelectListCap * sizeof(uint32_t);
    auto kfn = select_radix_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_dep(kfn, dim3(1), dim3(1024), smem, st, scores, kept, n_blocks, need,
                      tie_higher_id, sel, kSelectListCap);
}

cudaError_t launch_assemble(const AsmLaunch &a, uint32_t n_jobs, cudaStream_t st) {
    if (n_jobs == 0) return cudaSuccess;
    const bool q8 = a.g.k_type == KVMRET_TYPE_Q8_0, q4 = a.g.k_type == KVMRET_TYPE_Q4_0;
    switch (a.g.d_head) {
    case 64: return q8 ? launch_assemble_quant_t<64, 0>(a, n_jobs, st)
                  : q4 ? launch_assemble_quant_t<64, 1>(a, n_jobs, st)
                       : launch_assemble_t<64>(a, n_jobs, st);
    case 128: return q8 ? launch_assemble_quant_t<128, 0>(a, n_jobs, st)
                   : q4 ? launch_assemble_quant_t<128, 1>(a, n_jobs, st)
                        : launch_assemble_t<128>(a, n_jobs, st);
    case 256: return q8 ? launch_assemble_quant_t<256, 0>(a, n_jobs, st)
                   : q4 ? launch_assemble_quant_t<256, 1>(a, n_jobs, st)
                        : launch_assemble_t<256>(a, n_jobs, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_rope_table(float4 *cs, uint32_t n_pos, uint32_t half, const Theta &th,
                              cudaStream_t st, int32_t pos_base) {
    if (n_pos == 0) return cudaSuccess;
    rope_table_kernel<<<1184, 256, 0, st>>>(cs, n_pos, half, pos_base, th);
    return cudaGetLastError();
}

cudaError_t launch_append(const AppendArgs &a, cudaStream_t st) {
    if (a.n_tok == 0) return cudaSuccess;
    const uint32_t T = a.block_tokens;
    const uint32_t nb = (a.pos0 + a.n_tok - 1) / T - a.pos0 / T + 1;
    // Ping-pong the tail sum when the append spans blocks: the first touched
    // block reads the old tail while the last one may write the new tail in
    // the same launch. Within one block (a decode token) each thread reads and
    // then writes only its own channel, so the tail is updated in place.
    const size_t E = static_cast<size_t>(a.n_head_kv) * a.d_head;
    float *tail_in = a.tail_sum;
    float *tail_out = nb == 1 ? tail_in : a.tail_sum + static_cast<size_t>(a.n_layer) * E;
    cudaError_t e = launch_dep(append_summary_kernel, dim3(a.n_layer, nb), dim3(256), 0, st, a,
                               static_cast<const float *>(tail_in), tail_out);
    if (e != cudaSuccess) return e;
    if (nb > 1) {
        e = cudaMemcpyAsync(tail_in, tail_out, static_cast<size_t>(a.n_layer) * E * sizeof(float),
                            cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return e;
    }
    const uint32_t warps_per_cta = 8;
    return launch_dep(append_repo_kernel,
                      dim3((a.n_tok + warps_per_cta - 1) / warps_per_cta, a.n_layer),
                      dim3(warps_per_cta * 32), 0, st, a);
}

cudaError_t launch_quantize(const uint16_t *x, uint8_t *y, uint64_t n_blocks, bool q8,
                            cudaStream_t st) {
    if (n_blocks == 0) return cudaSuccess;
    quantize_kernel<<<static_cast<unsigned>((n_blocks + 255) / 256), 256, 0, st>>>(x, y, n_blocks,
                                                                                   q8 ? 1 : 0);
    return cudaGetLastError();
}

size_t plan_smem_bytes(uint32_t win_slots, uint32_t pool_slots) {
    return (5ull * win_slots + 3ull * pool_slots) * sizeof(uint32_t);
}

cudaError_t launch_plan(const PlanArgs &a, cudaStream_t st) {
    const size_t smem = plan_smem_bytes(a.win_slots, a.pool_slots);
    cudaError_t e = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_dep(plan_kernel, dim3(1), dim3(kPlanThreads), smem, st, a);
}

cudaError_t launch_gen_bind(const GenBinds &g, cudaStream_t st) {
    if (g.n == 0) return cudaSuccess;
    gen_bind_kernel<<<1, 32, 0, st>>>(g);
    return cudaGetLastError();
}

cudaError_t launch_gen_write(const GenWrite &a, cudaStream_t st) {
    if (a.n_seg == 0) return cudaSuccess;
    const dim3 grid(a.g.n_layer, a.n_seg);
    const bool q8 = a.g.k_type == KVMRET_TYPE_Q8_0, q4 = a.g.k_type == KVMRET_TYPE_Q4_0;
    const dim3 qb(32 * kGenQWarps);
    switch (a.g.d_head) {
    case 64:
        return q8   ? launch_dep(gen_write_quant_kernel<64, 0>, grid, qb, 0, st, a)
               : q4 ? launch_dep(gen_write_quant_kernel<64, 1>, grid, qb, 0, st, a)
                    : launch_dep(gen_write_f16_kernel<64>, grid, dim3(256), 0, st, a);
    case 128:
        return q8   ? launch_dep(gen_write_quant_kernel<128, 0>, grid, qb, 0, st, a)
               : q4 ? launch_dep(gen_write_quant_kernel<128, 1>, grid, qb, 0, st, a)
                    : launch_dep(gen_write_f16_kernel<128>, grid, dim3(256), 0, st, a);
    case 256:
        return q8   ? launch_dep(gen_write_quant_kernel<256, 0>, grid, qb, 0, st, a)
               : q4 ? launch_dep(gen_write_quant_kernel<256, 1>, grid, qb, 0, st, a)
                    : launch_dep(gen_write_f16_kernel<256>, grid, dim3(256), 0, st, a);
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_truncate(const TruncArgs &a, cudaStream_t st) {
    truncate_kernel<<<1, 1024, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_resum(const AppendArgs &a, uint32_t block, uint32_t n_tok, cudaStream_t st) {
    if (n_tok == 0) return cudaSuccess;
    resum_kernel<<<a.n_layer, 256, 0, st>>>(a, block, n_tok);
    return cudaGetLastError();
}

cudaError_t launch_copy_ops(const CopyOp *ops, int n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    copy_ops_kernel<<<n, 256, 0, st>>>(ops, n);
    return cudaGetLastError();
}

}  // namespace kvmret
