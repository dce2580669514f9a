// Host API of the tcgen05 GEMM family (gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace wb {

enum GemmEpilogue : int {
  kEpiBF16 = 0,    // C(bf16) = alpha * acc (+ bias)
  kEpiF32 = 1,     // C(fp32) = alpha * acc
  kEpiF32Acc = 2,  // C(fp32) += alpha * acc
  // C(bf16) = alpha * acc stored straight into peer memory: the GEMM half of a
  // fused GEMM -> all-reduce / reduce-scatter (see peer_* below).
  kEpiPeerBF16 = 3,
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
  // Second operand pair (dense mode): C (op)= alpha * (A B^T + A2 B2^T), with
  // A2 / B2 of the same majorness as A / B and inner dimension K2.  This is
  // the LoRA-fused linear: A2 = s * X A_lora^T, B2 = B_lora (forward), or
  // A2 = s * dY B_lora, B2 = A_lora (dgrad).
  const void* A2 = nullptr;
  int64_t lda2 = 0;
  const void* B2 = nullptr;
  int64_t ldb2 = 0;
  int K2 = 0;
  // NF4 B operand (dense mode, K-major A, bf16 out): B is dequantised on the
  // fly from 4-bit codes.  The weight W is [q_rows, q_cols] row-major with
  // two codes per byte (element 2i in the high nibble) and one fp32 absmax
  // per 64 consecutive elements of a row.  b_mn=false: B(n,k) = W[n][k];
  // b_mn=true: B(n,k) = W[k][n].  q_cols must be a multiple of 64.
  const uint8_t* q = nullptr;
  const float* q_absmax = nullptr;
  int64_t q_rows = 0, q_cols = 0;
  float q_lut[16] = {0};
  // kEpiPeerBF16 (dense mode): peer[r] is rank r's receive buffer (fabric
  // memory, mapped on this rank) and this rank's partial product lands at
  // element peer_off + row * ldc + col of it.  peer_rs_rows == 0: every rank
  // gets every row (all-reduce); > 0: row m goes only to rank m / peer_rs_rows,
  // at row m % peer_rs_rows (reduce-scatter).  Stores start at the next rank
  // (rank-rotated) so the ranks do not all write the same peer at once.
  void* peer[8] = {nullptr};
  int peer_world = 0;
  int peer_rank = 0;
  int64_t peer_off = 0;
  int64_t peer_rs_rows = 0;
  // Dense mode cuts the tiles of a small last wave into K-pieces reduced in a
  // per-device workspace (gemm.cu, "tail-wave split"); true keeps whole tiles.
  bool no_split = false;
};

void gemm_bf16(const GemmArgs& g, cudaStream_t stream);

}  // namespace wb
