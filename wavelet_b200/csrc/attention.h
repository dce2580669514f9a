// Host API of the sm_100a attention kernels (attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace wb {

struct AttnArgs {
  const void* q = nullptr;  // [T, Hq, 128], row stride q_row elements
  const void* k = nullptr;  // [T, Hk, 128]
  const void* v = nullptr;
  int64_t q_row = 0, k_row = 0, v_row = 0;
  void* o = nullptr;        // [T, Hq, 128]
  int64_t o_row = 0;
  float* lse = nullptr;     // [Hq, T]
  const int* cu_seqlens = nullptr;  // device int32 [nseq + 1]
  int nseq = 0, max_seqlen = 0, T = 0, Hq = 0, Hk = 0, head_dim = 128;
  float scale = 0.f;
  // Optional separate key sequences (context parallelism): k/v are [Tk, Hk,
  // 128] and sequence i's keys are rows cu_seqlens_k[i] .. cu_seqlens_k[i+1].
  // Its queries are the LAST Lq positions of those Lk keys (causal mask
  // aligned bottom-right: query j sees keys <= j + Lk - Lq).  Requires
  // Lk >= Lq and (Lk - Lq) % 128 == 0 for every sequence.
  const int* cu_seqlens_k = nullptr;
  int max_seqlen_k = 0, Tk = 0;
};

struct AttnBwdArgs {
  AttnArgs f;               // forward inputs (q, k, v, o, lse, cu_seqlens, ...)
  const void* dout = nullptr;  // [T, Hq, 128] contiguous
  void* dq = nullptr;          // [T, Hq, 128] contiguous
  void* dk = nullptr;          // [T, Hk, 128] contiguous
  void* dv = nullptr;          // [T, Hk, 128] contiguous
  float* delta = nullptr;      // [Hq, T] scratch
  float* part_dk = nullptr;    // [T, Hq, 128] fp32 scratch (GQA: per-q-head partials)
  float* part_dv = nullptr;
};

void attn_fwd(const AttnArgs& a, cudaStream_t stream);
void attn_bwd(const AttnBwdArgs& a, cudaStream_t stream);
// attn_bwd with caller-provided Delta scratch (a.delta) and error word;
// returns 0 on success (no exceptions, no allocation).
int attn_bwd_explicit(const AttnBwdArgs& a, int* err, cudaStream_t stream);

}  // namespace wb
