// Host API of the generator kernels (decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace wb {

struct DecodeArgs {
  const void* q = nullptr;  // [nseq, Hq, 128] rows of q_row elements
  int64_t q_row = 0;
  const void* k_cache = nullptr;  // [num_blocks, block_size, Hk, 128]
  const void* v_cache = nullptr;
  const int* block_tables = nullptr;  // [nseq, max_blocks]
  int max_blocks = 0;
  const int* ctx_lens = nullptr;  // [nseq]
  void* out = nullptr;            // [nseq, Hq, 128] rows of out_row elements
  int64_t out_row = 0;
  float* part_o = nullptr;   // [nseq, Hq, splits, 128] when splits > 1
  float* part_ml = nullptr;  // [nseq, Hq, splits, 2]
  int nseq = 0, Hq = 0, Hk = 0, block_size = 0, splits = 1;
  int64_t cache_rows = 0;  // num_blocks * block_size (TMA view of the cache)
  float scale = 0.f;
};

void kv_append(const void* k, int64_t k_row, const void* v, int64_t v_row, void* k_cache, void* v_cache,
               const int* slot, int T, int Hk, int block_size, cudaStream_t st);
void decode_attention(const DecodeArgs& a, cudaStream_t st);
void sample_tokens(const void* z, int64_t ldz, int rows, int V, const float* inv_tau, const float* thresh,
                   float min_p, uint64_t seed, const int64_t* row_ids, int64_t* out_tok, float* out_lp,
                   cudaStream_t st, const int64_t* seed_dev = nullptr);
// Per-row sampling threshold in logit units for top-k (top_k[i] > 0) and
// top-p (top_p[i] < 1, softmax of z * inv_tau): keep z >= out[i]; -inf where
// neither applies.  top_k / top_p / inv_tau may be null (off).
void sample_thresholds(const void* z, int64_t ldz, int rows, int V, const int* top_k, const float* top_p,
                       const float* inv_tau, float* out, cudaStream_t st);
void decode_advance(const int64_t* tok, const float* lp, int64_t* ids, int32_t* pos, int32_t* ctx, int32_t* slots,
                    const int32_t* bt, int max_blocks, int block_size, int64_t* win_tok, float* win_lp, int win_ld,
                    int32_t* step, int64_t* seed, int rows, cudaStream_t st);

}  // namespace wb
