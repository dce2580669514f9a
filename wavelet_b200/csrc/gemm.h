// Host API of the tcgen05 GEMM family (gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace wb {

enum GemmEpilogue : int {
  kEpiBF16 = 0,    // C(bf16) = alpha * acc (+ bias)
  kEpiF32 = 1,     // C(fp32) = alpha * acc
  kEpiF32Acc = 2,  // C(fp32) += alpha * acc
};

struct GemmArgs {
  // A(m, k): K-major -> A[m * lda + k];  MN-major -> A[k * lda + m]
  const void* A = nullptr;
  int64_t lda = 0;
  bool a_mn = false;
  // B(n, k): K-major -> B[n * ldb + k];  MN-major -> B[k * ldb + n]
  const void* B = nullptr;
  int64_t ldb = 0;
  bool b_mn = false;
  void* C = nullptr;  // row-major [M, ldc]
  int64_t ldc = 0;
  const void* bias = nullptr;  // bf16 [N] (kEpiBF16 only)
  const void* res = nullptr;   // bf16 [M, ldr] residual added to C (kEpiBF16 only)
  int64_t ldr = 0;
  float alpha = 1.0f;
  int epi = kEpiBF16;
  int M = 0, N = 0, K = 0;
  // Grouped (MoE expert) modes.  0: dense.
  // 1 (M-grouped): A rows are expert segments padded to 128; tile_group[m_tile]
  //   gives the expert; B holds every expert's weights stacked along its outer
  //   dimension (b_outer rows in total) and expert g starts at g * b_group_stride.
  // 2 (K-grouped): C[g] (rows g*M .. g*M+M-1) = A_g^T B_g where A_g / B_g are the
  //   token rows [k_start[g], k_start[g] + k_len[g]) of MN-major A and B.
  int group_mode = 0;
  const int* tile_group = nullptr;
  int64_t b_group_stride = 0;
  int64_t b_outer = 0;
  const int* k_start = nullptr;
  const int* k_len = nullptr;
  int groups = 0;
};

void gemm_bf16(const GemmArgs& g, cudaStream_t stream);

}  // namespace wb
