// Dense f16 GEMM on the sm_100a tensor cores (tcgen05), C = alpha * A * B^T
// with A [M][K] and B [N][K] f16 row-major (both K-major) and C [M][N] f32.
// It is the contraction of the prefill scorer (a chunk's normalised group
// queries against every block's normalised summary, all layers and KV heads
// stacked along K) and is exported on its own as kvmret_gemm_f16_nt.
//
// A CTA computes 128 x 256 tiles of C (or k-ranges of them, below) with the
// accumulator in tensor memory (two 256-column f32 buffers of the SM's 512
// TMEM columns); the last tile of a row may be partial (its columns past n
// are loaded as zeros and not stored). Warp roles:
//   warp 0      TMA producer: 2-D tiled loads of A (128 x 64) and B (256 x 64)
//               into a 4-stage shared-memory ring, 128-byte swizzle, no
//               multicast; completion by mbarrier transaction counts;
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma
//               (kind::f16, M = 128, N = 256, K = 16; four per 64-wide stage)
//               and commits each stage back to the producer, and the finished
//               accumulator to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns at a time (warp w
//               reads TMEM lanes 32 * (w % 4) ..), scale, 16-byte stores.
// (A 240-wide tile, 144 CTAs instead of 128 for a 2048 x 2048 product, was
// built and measured: no faster, 0.448 against 0.445 ms at config 4. The
// tiles' L2-to-SM traffic, not the idle SMs, sets the pace.)
// Every mbarrier wait is bounded; on a timeout the CTA records an error in
// *err, stops issuing, drains what it issued (bounded), frees its TMEM and
// returns.
#include "gemm_tc.cuh"

#include <cuda_fp16.h>

#include <algorithm>

namespace kvmret {
namespace {

constexpr int kGemmThreads = 192;
constexpr int kTileM = 128, kTileN = 256, kTileK = 64, kStages = 4;
constexpr uint32_t kStageA = kTileM * kTileK * 2;  // 16 KiB
constexpr uint32_t kStageB = kTileN * kTileK * 2;  // 32 KiB
constexpr uint32_t kStageBytes = kStageA + kStageB;
constexpr uint32_t kTmemCols = 512;  // two 256-column accumulators
constexpr uint64_t kWaitNs = 2000000000ull;  // a pipeline wait gives up after 2 s

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Wait for the phase with the given parity to complete; gives up (false)
// after kWaitNs of wall time.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
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
        if (i == 0) {
            t0 = global_ns();
        } else if ((i & 63) == 0 && global_ns() - t0 > kWaitNs) {
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x,
                                            int32_t y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// 8-row x 128-byte atoms stacked every 1024 bytes (stride byte offset), the
// leading byte offset unused (1), descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) |
           (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: D f32, A and B f16, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(kTileN >> 3) << 17) |
                            (static_cast<uint32_t>(kTileM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t tmem_c, uint64_t da, uint64_t db,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            tmem_c),
        "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
        " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
        " [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Work split. With one tile per CTA (x == n_ktiles, gridDim.x == n_tiles)
// every CTA runs its tile's whole K and writes C. When the tiles would leave
// SMs idle (n_tiles < SM count) the grid is one CTA per SM: CTA g < n_tiles
// (a "main" CTA) runs k-steps [0, x) of tile g, all main CTAs in lockstep so
// each k-slice of A and B is shared in L2 as in the one-tile form, and writes
// its raw sums into C; the remaining H CTAs ("helpers") split the tails
// [x, n_ktiles) of all tiles, in tile order, into equal contiguous ranges and
// write each piece raw into the workspace slot (tile, piece); then
// gemm_fixup_kernel sets C = alpha * (C + the tile's pieces in order), so the
// result does not depend on timing. x = total k-steps / SM count, so every
// SM gets the same share. The accumulator is double-buffered in TMEM
// (2 x 256 columns): the MMAs of a helper's next piece overlap the epilogue
// of its previous one.
struct GemmSplit {
    uint32_t n_ktiles, tiles_n, n_tiles;
    uint32_t x;      // k-steps of a main CTA; n_ktiles: one tile per CTA
    uint32_t helpers, pieces;  // helper CTAs; workspace slots per tile
};

__device__ __forceinline__ uint64_t range_begin(uint64_t total, uint32_t g, uint32_t n) {
    return total * g / n;
}
// the helper whose tail range holds tail k-step j
__device__ __forceinline__ uint32_t tail_owner(uint64_t j, uint64_t total, uint32_t n) {
    const uint64_t guess = j * n / total;
    uint32_t h = guess < n - 1 ? static_cast<uint32_t>(guess) : n - 1;
    while (h + 1 < n && range_begin(total, h + 1, n) <= j) ++h;
    while (h > 0 && range_begin(total, h, n) > j) --h;
    return h;
}

// One CTA's run of segments (tile, k0 .. k1) and where each one goes.
struct SegWalk {
    GemmSplit sp;
    uint32_t role;   // 0: a tile per CTA, 1: main, 2: helper
    uint64_t it, it1, tail_total;
    uint32_t h;
    __device__ SegWalk(const GemmSplit &s, uint32_t g) : sp(s) {
        if (sp.x == sp.n_ktiles) {
            role = 0;
            it = static_cast<uint64_t>(g) * sp.n_ktiles;
            it1 = it + sp.n_ktiles;
        } else if (g < sp.n_tiles) {
            role = 1;
            it = 0;
            it1 = sp.x;
        } else {
            role = 2;
            h = g - sp.n_tiles;
            tail_total = static_cast<uint64_t>(sp.n_tiles) * (sp.n_ktiles - sp.x);
            it = range_begin(tail_total, h, sp.helpers);
            it1 = range_begin(tail_total, h + 1, sp.helpers);
        }
    }
    __device__ bool more() const { return it < it1; }
    // the current segment; kind 0: C scaled, 1: C raw, 2: workspace slot
    __device__ void get(uint32_t &t, uint32_t &k0, uint32_t &k1, uint32_t &kind,
                        uint32_t &slot) const {
        slot = 0;
        if (role == 0) {
            t = static_cast<uint32_t>(it / sp.n_ktiles);
            k0 = 0;
            k1 = sp.n_ktiles;
            kind = 0;
        } else if (role == 1) {
            t = blockIdx.x;
            k0 = 0;
            k1 = sp.x;
            kind = 1;
        } else {
            const uint32_t L = sp.n_ktiles - sp.x;
            t = static_cast<uint32_t>(it / L);
            const uint32_t off = static_cast<uint32_t>(it - static_cast<uint64_t>(t) * L);
            const uint64_t len = it1 - it < L - off ? it1 - it : L - off;
            k0 = sp.x + off;
            k1 = k0 + static_cast<uint32_t>(len);
            kind = 2;
            slot = t * sp.pieces +
                   (h - tail_owner(static_cast<uint64_t>(t) * L, tail_total, sp.helpers));
        }
    }
    __device__ void next(uint32_t k0, uint32_t k1) { it += k1 - k0; }
};

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_nt_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, float *__restrict__ c,
                       uint32_t ldc, const __grid_constant__ GemmSplit sp, float alpha,
                       float *__restrict__ ws, uint32_t *err) {
    extern __shared__ uint8_t smem_raw[];
    // stages must start on 1024-byte boundaries (the swizzle atom)
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *const smem = smem_raw + (base - raw);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    // bars[0..S): stage full, [S..2S): stage empty, [2S, 2S+1]: accumulator b
    // full, [2S+2, 2S+3]: accumulator b drained by the epilogue
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kStages + 4);
    __shared__ uint32_t s_fail;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](uint32_t s) { return bar0 + 8u * s; };
    auto empty_bar = [&](uint32_t s) { return bar0 + 8u * (kStages + s); };
    auto acc_full = [&](uint32_t b) { return bar0 + 8u * (2 * kStages + b); };
    auto acc_empty = [&](uint32_t b) { return bar0 + 8u * (2 * kStages + 2 + b); };
    const uint32_t tiles_n = sp.tiles_n;

    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int s = 0; s < 2 * kStages + 2; ++s) mbar_init(bar0 + 8u * s, 1);
        mbar_init(acc_empty(0), 4);  // one arrival per epilogue warp
        mbar_init(acc_empty(1), 4);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a))
                     : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b))
                     : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // producer
            uint32_t q = 0;  // k-steps issued (the stage ring runs across segments)
            bool stop = false;
            for (SegWalk sw(sp, blockIdx.x); sw.more() && !stop;) {
                uint32_t t, k0, k1, kind, slot;
                sw.get(t, k0, k1, kind, slot);
                const int32_t m0 = static_cast<int32_t>((t / tiles_n) * kTileM);
                const int32_t n0 = static_cast<int32_t>((t % tiles_n) * kTileN);
                for (uint32_t k = k0; k < k1; ++k) {
                    const uint32_t s = q % kStages, round = q / kStages;
                    if ((round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1u)) ||
                        *static_cast<volatile uint32_t *>(&s_fail)) {
                        stop = true;
                        break;
                    }
                    const uint32_t sa = base + s * kStageBytes;
                    mbar_expect_tx(full_bar(s), kStageBytes);
                    tma_load_2d(sa, &map_a, static_cast<int32_t>(k * kTileK), m0, full_bar(s));
                    tma_load_2d(sa + kStageA, &map_b, static_cast<int32_t>(k * kTileK), n0,
                                full_bar(s));
                    ++q;
                }
                sw.next(k0, k1);
            }
            if (stop) {  // gave up: drain the loads already issued (bounded)
                atomicExch(&s_fail, 1u);
                for (uint32_t j = (q > kStages ? q - kStages : 0); j < q; ++j)
                    mbar_wait(full_bar(j % kStages), (j / kStages) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            uint32_t q = 0, j = 0;
            bool stop = false;
            for (SegWalk sw(sp, blockIdx.x); sw.more() && !stop; ++j) {
                uint32_t t, k0, k1, kind, slot;
                sw.get(t, k0, k1, kind, slot);
                const uint32_t b = j & 1u;
                // the epilogue has drained this buffer's previous segment
                if (j >= 2 && !mbar_wait(acc_empty(b), ((j >> 1) - 1) & 1u)) {
                    stop = true;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + b * kTileN;
                for (uint32_t k = k0; k < k1; ++k) {
                    const uint32_t s = q % kStages;
                    if (!mbar_wait(full_bar(s), (q / kStages) & 1u) ||
                        *static_cast<volatile uint32_t *>(&s_fail)) {
                        stop = true;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sa = base + s * kStageBytes;
                    const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + kStageA);
#pragma unroll
                    for (uint32_t kk = 0; kk < kTileK / 16; ++kk)  // +32 bytes per K = 16 slice
                        mma_f16(acc, da + 2 * kk, db + 2 * kk, (k != k0 || kk != 0) ? 1u : 0u);
                    mma_commit(empty_bar(s));
                    ++q;
                }
                // arrives once every MMA issued above has completed (on a stop
                // too, so the epilogue wakes and sees the failure)
                mma_commit(acc_full(b));
                sw.next(k0, k1);
            }
            if (stop) atomicExch(&s_fail, 1u);
        }
    } else {  // epilogue, warps 2..5
        const uint32_t qd = warp & 3u;
        uint32_t j = 0;
        for (SegWalk sw(sp, blockIdx.x); sw.more(); ++j) {
            uint32_t t, k0, k1, kind, slot;
            sw.get(t, k0, k1, kind, slot);
            const uint32_t b = j & 1u;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full(b), (j >> 1) & 1u));
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (!ok || *static_cast<volatile uint32_t *>(&s_fail)) {
                if (lane == 0) atomicExch(&s_fail, 1u);
                break;
            }
            const uint32_t r = 32 * qd + lane;
            float *dst_row;
            const float scale = kind == 0 ? alpha : 1.0f;
            const uint32_t n0 = (t % tiles_n) * kTileN;
            // columns of C this tile holds (ldc = n; a row's last tile may be
            // partial); a workspace slot takes the whole tile
            const uint32_t ncols =
                kind < 2 ? min(static_cast<uint32_t>(kTileN), ldc - n0) : kTileN;
            if (kind < 2)
                dst_row = c + static_cast<size_t>((t / tiles_n) * kTileM + r) * ldc + n0;
            else
                dst_row = ws + (static_cast<size_t>(slot) * kTileM + r) * kTileN;
            const uint32_t tacc = tmem + ((32 * qd) << 16) + b * kTileN;
#pragma unroll 1
            for (uint32_t col = 0; col < ncols; col += 32) {  // ncols: a multiple of 16
                uint32_t v[32];
                tmem_ld32(tacc + col, v);
                float4 *dst = reinterpret_cast<float4 *>(dst_row + col);
#pragma unroll
                for (uint32_t e = 0; e < 8; ++e)
                    if (col + 4 * e < ncols)
                        dst[e] = make_float4(scale * __uint_as_float(v[4 * e]),
                                             scale * __uint_as_float(v[4 * e + 1]),
                                             scale * __uint_as_float(v[4 * e + 2]),
                                             scale * __uint_as_float(v[4 * e + 3]));
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(acc_empty(b))
                             : "memory");
            sw.next(k0, k1);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && s_fail && err) atomicExch(err, 1u);
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// C = alpha * (the main CTA's sums in C + the helpers' pieces of the tile, in
// order). One CTA per tile; columns past n (= ldc) are skipped.
__global__ void __launch_bounds__(256)
    gemm_fixup_kernel(float *__restrict__ c, uint32_t ldc, const float *__restrict__ ws,
                      const __grid_constant__ GemmSplit sp, float alpha, const uint32_t *err) {
    if (err && *err) return;  // the product gave up: C is not valid anyway
    const uint32_t t = blockIdx.x, L = sp.n_ktiles - sp.x;
    const uint64_t tail_total = static_cast<uint64_t>(sp.n_tiles) * L;
    const uint64_t a = static_cast<uint64_t>(t) * L;
    const uint32_t n_pieces = tail_owner(a + L - 1, tail_total, sp.helpers) -
                              tail_owner(a, tail_total, sp.helpers) + 1;
    const uint32_t m0 = (t / sp.tiles_n) * kTileM, n0 = (t % sp.tiles_n) * kTileN;
    for (uint32_t e = threadIdx.x; e < kTileM * kTileN / 4; e += blockDim.x) {
        const uint32_t r = e / (kTileN / 4), c4 = e % (kTileN / 4);
        if (n0 + 4 * c4 >= ldc) continue;
        float4 *cp = reinterpret_cast<float4 *>(c + static_cast<size_t>(m0 + r) * ldc + n0) + c4;
        float4 acc = *cp;
        for (uint32_t p = 0; p < n_pieces; ++p) {
            const float4 v = reinterpret_cast<const float4 *>(
                ws + (static_cast<size_t>(t * sp.pieces + p) * kTileM + r) * kTileN)[c4];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        *cp = make_float4(alpha * acc.x, alpha * acc.y, alpha * acc.z, alpha * acc.w);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// 2-D f16 tensor {k, rows}, row stride k * 2 bytes, box {64, box_rows}, 128-byte swizzle.
cudaError_t encode_kmajor(CUtensorMap *map, const void *base, uint32_t rows, uint32_t k,
                          uint32_t box_rows) {
    const EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {k, rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int sm_count() {
    static int n = [] {
        int dev = 0, v = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return 0;
        return v;
    }();
    return n;
}

bool shape_ok(uint32_t m, uint32_t n, uint32_t k) {
    return m && m % kTileM == 0 && n && n % 16 == 0 && k && k % kTileK == 0;
}

// The split of an m x n x k product on this device (x == n_ktiles: none).
GemmSplit plan_split(uint32_t m, uint32_t n, uint32_t k) {
    GemmSplit sp{};
    sp.tiles_n = (n + kTileN - 1) / kTileN;
    sp.n_tiles = sp.tiles_n * (m / kTileM);
    sp.n_ktiles = k / kTileK;
    sp.x = sp.n_ktiles;
    const int n_sm = sm_count();
    if (n_sm <= 0 || sp.n_tiles >= static_cast<uint32_t>(n_sm)) return sp;
    const uint64_t total = static_cast<uint64_t>(sp.n_tiles) * sp.n_ktiles;
    // x near total / SMs, the one whose busiest CTA takes the least time; no
    // split unless that beats a whole tile per CTA. A helper's k-step counts
    // 1.25 of a main CTA's: its tail slices are not shared in L2 with CTAs in
    // lockstep, and one SM's TMA stream from DRAM runs ~25 % slower than the
    // tensor pipe (measured: 128 tiles, K = 65536, 479 us split against
    // 449 us a tile per CTA; 32 tiles 179 us against 398 us).
    uint64_t best = 4ull * sp.n_ktiles;  // in quarter k-steps
    for (uint64_t x = total / n_sm; x <= total / n_sm + 1; ++x) {
        if (x == 0 || x >= sp.n_ktiles) continue;
        const uint64_t tail = static_cast<uint64_t>(sp.n_tiles) * (sp.n_ktiles - x);
        const uint64_t h = std::min<uint64_t>(static_cast<uint64_t>(n_sm) - sp.n_tiles, tail);
        const uint64_t load = std::max<uint64_t>(4 * x, (5 * tail + h - 1) / h);
        if (load < best) {
            best = load;
            sp.x = static_cast<uint32_t>(x);
            sp.helpers = static_cast<uint32_t>(h);
        }
    }
    if (sp.x == sp.n_ktiles) return sp;
    const uint32_t L = sp.n_ktiles - sp.x;
    const uint64_t share = static_cast<uint64_t>(sp.n_tiles) * L / sp.helpers;  // >= 1
    // a tail of L k-steps meets at most ceil(L / share) + 1 helper ranges
    sp.pieces = static_cast<uint32_t>((L + share - 1) / share + 1);
    return sp;
}

size_t smem_bytes() {
    return kStages * static_cast<size_t>(kStageBytes) + 1024 /* alignment */ +
           (2 * kStages + 4) * 8 + 16;
}
}  // namespace

cudaError_t make_gemm_maps(const void *a, const void *b, uint32_t m, uint32_t n, uint32_t k,
                           CUtensorMap *map_a, CUtensorMap *map_b) {
    if (!shape_ok(m, n, k)) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15)
        return cudaErrorInvalidValue;
    cudaError_t e = encode_kmajor(map_a, a, m, k, kTileM);
    if (e == cudaSuccess) e = encode_kmajor(map_b, b, n, k, kTileN);
    return e;
}

size_t gemm_ws_bytes(uint32_t m, uint32_t n, uint32_t k) {
    if (!shape_ok(m, n, k)) return 0;
    const GemmSplit sp = plan_split(m, n, k);
    if (sp.x == sp.n_ktiles) return 0;
    return static_cast<size_t>(sp.n_tiles) * sp.pieces * kTileM * kTileN * sizeof(float);
}

cudaError_t launch_gemm_f16_nt(const CUtensorMap &map_a, const CUtensorMap &map_b, float *c,
                               uint32_t m, uint32_t n, uint32_t k, float alpha, uint32_t *err,
                               cudaStream_t st, float *ws, size_t ws_bytes) {
    if (!shape_ok(m, n, k)) return cudaErrorInvalidValue;
    const size_t smem = smem_bytes();
    cudaError_t e = cudaFuncSetAttribute(gemm_f16_nt_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    GemmSplit sp = plan_split(m, n, k);
    const size_t need = static_cast<size_t>(sp.n_tiles) * sp.pieces * kTileM * kTileN * 4;
    if (sp.x != sp.n_ktiles && (!ws || ws_bytes < need)) {  // no room: a tile per CTA
        sp.x = sp.n_ktiles;
        sp.helpers = sp.pieces = 0;
    }
    const uint32_t grid = sp.x == sp.n_ktiles ? sp.n_tiles : sp.n_tiles + sp.helpers;
    gemm_f16_nt_kernel<<<grid, kGemmThreads, smem, st>>>(map_a, map_b, c, n, sp, alpha, ws, err);
    e = cudaGetLastError();
    if (e != cudaSuccess || sp.x == sp.n_ktiles) return e;
    gemm_fixup_kernel<<<sp.n_tiles, 256, 0, st>>>(c, n, ws, sp, alpha, err);
    return cudaGetLastError();
}

}  // namespace kvmret
