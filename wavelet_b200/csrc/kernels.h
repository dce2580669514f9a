// Host API of the bandwidth-bound kernels (kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace wb {

void rmsnorm_fwd(const void* x, const void* res, void* h_out, const void* w, void* y, float* rstd,
                 int rows, int H, float eps, cudaStream_t st);
// dw (optional, fp32, +=) is reduced through part: fp32 scratch of
// rmsnorm_dw_splits(rows) x H elements (reproducible order).
int rmsnorm_dw_splits(int rows);
void rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* dres,
                 void* dx, float* dw, float* part, int rows, int H, cudaStream_t st);
void qk_norm_rope_fwd(void* qkv, int64_t row_stride, int n_q, int n_k, const int* pos,
                      const float* inv_freq, const void* q_w, const void* k_w, float* rstd,
                      int tokens, float eps, cudaStream_t st);
void qk_norm_rope_bwd(void* dqkv, int64_t drow_stride, const void* qkv_pre, int64_t row_stride,
                      int n_q, int n_k, const int* pos, const float* inv_freq, const void* q_w,
                      const void* k_w, const float* rstd, float* dq_w, float* dk_w, int tokens,
                      cudaStream_t st);
void swiglu_fwd(const void* gu, void* h, int64_t rows, int I, cudaStream_t st);
void swiglu_bwd(const void* gu, const void* dh, void* dgu, int64_t rows, int I, cudaStream_t st);
void embedding_fwd(const void* table, const int64_t* ids, void* out, int64_t T, int H, int64_t V,
                   cudaStream_t st);
void embedding_bwd(const void* dy, const int64_t* ids, float* dtable, int64_t T, int H, int64_t V,
                   cudaStream_t st);
void splitk_reduce(const float* ws, int S, int64_t M, int N, void* out, int64_t ldc, const void* bias, const void* res,
                   int64_t ldr, float alpha, cudaStream_t st);
void nf4_dequant(const void* codes, const float* absmax, void* out, int64_t numel, const float* lut,
                 cudaStream_t st);
// AdamW with 8-bit block-scaled moments (256 elements per fp32 scale, log
// codes; see kernels.cu).  m8 / v8: n codes; am / av: ceil(n / 256) scales.
void adamw8_step(float* p, const float* g, int8_t* m8, uint8_t* v8, float* am, float* av, void* p16, int64_t n,
                 float lr, float b1, float b2, float eps, float wd, float bc1, float bc2, const float* gscale_dev,
                 float gscale_host, cudaStream_t st);
void adamw_step(float* p, const float* g, float* m, float* v, void* p16, int64_t n, float lr,
                float b1, float b2, float eps, float wd, float bc1, float bc2,
                const float* gscale_dev, float gscale_host, cudaStream_t st);
void sumsq(const float* x, int64_t n, float* out, cudaStream_t st);
void clip_factor(const float* sumsq_v, float max_norm, float* out, cudaStream_t st);
void softmax_stats(const void* z, int64_t ldz, int rows, int V, const int64_t* target,
                   float inv_tau, float* lse, float* lp, float* ent, cudaStream_t st);
void softmax_grad(void* z, int64_t ldz, int rows, int V, const int64_t* target, float inv_tau,
                  const float* lse, const float* ent, const float* dlp, const float* dent,
                  cudaStream_t st);

}  // namespace wb
