// Prefill scorer kernels (prefill.cu) and the tensor-core GEMM they feed
// (gemm_tc.cuh).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm_tc.cuh"

namespace kvmret {

// A[t][(l*Hkv + g)*D + d] = unit-length group query of token t, layer l, KV head g (f16).
// q: [n_layer][n_tok][n_head * d_head] f16.
cudaError_t launch_qhat(const uint16_t *q, uint16_t *a, uint32_t n_layer, uint32_t n_tok,
                        uint32_t n_head, uint32_t n_head_kv, uint32_t d_head, uint64_t lda,
                        cudaStream_t st);
// B[b][(l*Hkv + g)*D + d] = unit-length summary of block b (f16), blocks [b_lo, b_hi).
cudaError_t launch_mhat(const float *summ, uint16_t *b, uint32_t n_layer, uint32_t n_head_kv,
                        uint32_t d_head, uint32_t ncap, uint32_t b_lo, uint32_t b_hi,
                        uint64_t ldb, cudaStream_t st);
// sel[b] = 1 for every block in some token's top_k (rows of s: [n_tok][lds] f32).
cudaError_t launch_topk_union(const float *s, uint64_t lds, uint32_t n_tok, uint32_t n_blocks,
                              uint32_t top_k, int tie_high, uint8_t *sel, cudaStream_t st);

}  // namespace kvmret
