// Prefill scorer operands and per-token selection (an extension of the
// reference's scorer: score_retrieval, llama-memory-kvmem.cpp:4149-4196,
// scores the MEAN query of a span; this path scores every token of a prefill
// chunk and takes the union of the per-token top-k).
//
//   qhat:  for layer l, token t, KV head g: the group query
//          qg = sum_{h < G} q[l][t][g*G + h] (f32, head order), normalised to
//          unit length, stored f16 in row t of A at column (l*Hkv + g)*D + d;
//   mhat:  the block summary m[l][g][b] normalised to unit length, f16, row b
//          of B at the same columns;
//   A * B^T * 1/(L*Hkv) is then the mean over layers and KV heads of the
//   cosine of each token's group query with each block's mean key
//   (gemm_tc.cu, tensor cores);
//   topk_union: per token, the top_k blocks by (score desc, block id by the
//          tie rule) among the blocks with data; union over the tokens.
#include "prefill.cuh"

#include <cub/block/block_scan.cuh>
#include <cuda_fp16.h>

namespace kvmret {
namespace {

template <int D>
__global__ void qhat_kernel(const uint16_t *__restrict__ q, uint16_t *__restrict__ a,
                            uint32_t n_tok, uint32_t n_head, uint32_t n_head_kv, uint64_t lda) {
    constexpr int EPL = D / 32;
    const uint32_t t = blockIdx.x, l = blockIdx.y;
    const uint32_t g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (g >= n_head_kv) return;
    const uint32_t G = n_head / n_head_kv;
    const uint16_t *row = q + (static_cast<uint64_t>(l) * n_tok + t) * n_head * D;
    float s[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) s[e] = 0.0f;
    for (uint32_t h = 0; h < G; ++h) {
        const uint16_t *src = row + static_cast<uint64_t>(g * G + h) * D + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e)
            s[e] = __fadd_rn(s[e], __half2float(__ushort_as_half(src[e])));
    }
    float n2 = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) n2 = __fadd_rn(n2, __fmul_rn(s[e], s[e]));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) n2 = __fadd_rn(n2, __shfl_xor_sync(0xffffffffu, n2, o));
    const float inv = n2 > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(n2)) : 0.0f;
    uint16_t *dst = a + static_cast<uint64_t>(t) * lda +
                    (static_cast<uint64_t>(l) * n_head_kv + g) * D + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = __half_as_ushort(__float2half_rn(__fmul_rn(s[e], inv)));
}

// CTA = (32 blocks, KV head, layer). Summaries are block-minor
// [L][Hkv][D][ncap]; the tile is transposed through shared memory.
template <int D>
__global__ void mhat_kernel(const float *__restrict__ summ, uint16_t *__restrict__ b,
                            uint32_t ncap, uint32_t n_head_kv, uint32_t b_lo, uint32_t b_hi,
                            uint64_t ldb) {
    __shared__ float tile[D][33];
    __shared__ float inv[32];
    const uint32_t b0 = b_lo + blockIdx.x * 32, g = blockIdx.y, l = blockIdx.z;
    const float *src = summ + (static_cast<uint64_t>(l) * n_head_kv + g) * D * ncap;
    for (uint32_t i = threadIdx.x; i < D * 32; i += blockDim.x) {
        const uint32_t d = i / 32, j = i % 32;
        tile[d][j] = (b0 + j < b_hi) ? src[static_cast<uint64_t>(d) * ncap + b0 + j] : 0.0f;
    }
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
    for (uint32_t j = warp; j < 32; j += nwarp) {
        float n2 = 0.0f;
        for (uint32_t d = lane; d < D; d += 32) n2 = __fadd_rn(n2, __fmul_rn(tile[d][j], tile[d][j]));
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) n2 = __fadd_rn(n2, __shfl_xor_sync(0xffffffffu, n2, o));
        if (lane == 0) inv[j] = n2 > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(n2)) : 0.0f;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < D * 32; i += blockDim.x) {
        const uint32_t j = i / D, d = i % D;
        if (b0 + j >= b_hi) continue;
        b[static_cast<uint64_t>(b0 + j) * ldb + (static_cast<uint64_t>(l) * n_head_kv + g) * D + d] =
            __half_as_ushort(__float2half_rn(__fmul_rn(tile[d][j], inv[j])));
    }
}

// Order-preserving map of a float to an unsigned key.
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kTopkThreads = 256;

// CTA = one token. Radix select (4 x 8 bits) of the top_k-th largest key,
// then the keys above it and, among the keys equal to it, the first ones by
// the tie rule (higher block id first when tie_high).
__global__ void __launch_bounds__(kTopkThreads)
    topk_union_kernel(const float *__restrict__ s, uint64_t lds, uint32_t n_blocks,
                      uint32_t top_k, int tie_high, uint8_t *__restrict__ sel) {
    using Scan = cub::BlockScan<uint32_t, kTopkThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask, s_need;
    extern __shared__ uint32_t keys[];
    const float *row = s + static_cast<uint64_t>(blockIdx.x) * lds;
    if (n_blocks <= top_k) {
        for (uint32_t b = threadIdx.x; b < n_blocks; b += blockDim.x) sel[b] = 1;
        return;
    }
    for (uint32_t b = threadIdx.x; b < n_blocks; b += blockDim.x) keys[b] = fkey(row[b]);
    if (threadIdx.x == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_need = top_k;  // rank (from the top) still to place inside the current prefix
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (uint32_t b = threadIdx.x; b < n_blocks; b += blockDim.x) {
            const uint32_t k = keys[b];
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {  // walk the digits from the top
            uint32_t need = s_need, d = 255;
            for (;; --d) {
                if (hist[d] >= need || d == 0) break;
                need -= hist[d];
            }
            s_need = need;
            s_prefix = prefix | (d << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    const uint32_t thr = s_prefix, need_eq = s_need;  // need_eq equal keys are taken
    // block ids with key == thr, ranked in id order by a block-wide scan over
    // contiguous per-thread ranges
    const uint32_t per = (n_blocks + kTopkThreads - 1) / kTopkThreads;
    const uint32_t lo = threadIdx.x * per, hi = min(n_blocks, lo + per);
    uint32_t cnt = 0;
    for (uint32_t b = lo; b < hi; ++b) cnt += keys[b] == thr;
    uint32_t before, total;
    Scan(scan_tmp).ExclusiveSum(cnt, before, total);
    for (uint32_t b = lo; b < hi; ++b) {
        const uint32_t k = keys[b];
        bool take = k > thr;
        if (k == thr) {
            const uint32_t r = tie_high ? total - 1 - before : before;  // rank by the tie rule
            take = r < need_eq;
            ++before;
        }
        if (take) sel[b] = 1;
    }
}

}  // namespace

cudaError_t launch_qhat(const uint16_t *q, uint16_t *a, uint32_t n_layer, uint32_t n_tok,
                        uint32_t n_head, uint32_t n_head_kv, uint32_t d_head, uint64_t lda,
                        cudaStream_t st) {
    if (n_tok == 0) return cudaSuccess;
    const dim3 grid(n_tok, n_layer);
    const uint32_t threads = 32 * n_head_kv;
    if (threads > 1024) return cudaErrorInvalidValue;
    switch (d_head) {
    case 64: qhat_kernel<64><<<grid, threads, 0, st>>>(q, a, n_tok, n_head, n_head_kv, lda); break;
    case 128: qhat_kernel<128><<<grid, threads, 0, st>>>(q, a, n_tok, n_head, n_head_kv, lda); break;
    case 256: qhat_kernel<256><<<grid, threads, 0, st>>>(q, a, n_tok, n_head, n_head_kv, lda); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_mhat(const float *summ, uint16_t *b, uint32_t n_layer, uint32_t n_head_kv,
                        uint32_t d_head, uint32_t ncap, uint32_t b_lo, uint32_t b_hi,
                        uint64_t ldb, cudaStream_t st) {
    if (b_hi <= b_lo) return cudaSuccess;
    const dim3 grid((b_hi - b_lo + 31) / 32, n_head_kv, n_layer);
    switch (d_head) {
    case 64: mhat_kernel<64><<<grid, 256, 0, st>>>(summ, b, ncap, n_head_kv, b_lo, b_hi, ldb); break;
    case 128: mhat_kernel<128><<<grid, 256, 0, st>>>(summ, b, ncap, n_head_kv, b_lo, b_hi, ldb); break;
    case 256: mhat_kernel<256><<<grid, 256, 0, st>>>(summ, b, ncap, n_head_kv, b_lo, b_hi, ldb); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_topk_union(const float *s, uint64_t lds, uint32_t n_tok, uint32_t n_blocks,
                              uint32_t top_k, int tie_high, uint8_t *sel, cudaStream_t st) {
    if (n_tok == 0 || n_blocks == 0) return cudaSuccess;
    const size_t smem = static_cast<size_t>(n_blocks) * sizeof(uint32_t);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(topk_union_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    topk_union_kernel<<<n_tok, kTopkThreads, smem, st>>>(s, lds, n_blocks, top_k, tie_high, sel);
    return cudaGetLastError();
}

}  // namespace kvmret
