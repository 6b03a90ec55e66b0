// Tensor-core GEMM of the prefill scorer (sm_100a tcgen05): C = alpha * A * B^T,
// A [m][k] and B [n][k] f16 row-major, C [m][n] f32; m % 128 == 0,
// n % 16 == 0, k % 64 == 0. The tensor maps describe A and B as 2-D f16
// tensors {k, rows} with 64 x 128 (A) and 64 x 256 (B) boxes and 128-byte
// swizzle (make_gemm_maps builds them).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace kvmret {

// Workspace the split form of an m x n x k product needs on the current
// device (0: it runs a tile per CTA): the helpers' partial 128 x 256 f32
// tiles. With at least that much, a product whose tiles would leave SMs idle
// runs one CTA per SM (main CTAs in lockstep plus helpers on the k tails) and
// a fix-up launch; otherwise, or without a workspace, a tile per CTA.
size_t gemm_ws_bytes(uint32_t m, uint32_t n, uint32_t k);
cudaError_t launch_gemm_f16_nt(const CUtensorMap &map_a, const CUtensorMap &map_b, float *c,
                               uint32_t m, uint32_t n, uint32_t k, float alpha, uint32_t *err,
                               cudaStream_t st, float *ws = nullptr, size_t ws_bytes = 0);
// Encodes the two tensor maps (driver entry point looked up once).
cudaError_t make_gemm_maps(const void *a, const void *b, uint32_t m, uint32_t n, uint32_t k,
                           CUtensorMap *map_a, CUtensorMap *map_b);

}  // namespace kvmret
