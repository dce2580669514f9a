// Bandwidth-bound sm_100a kernels of the trainer and generator:
//   RMSNorm forward/backward (optionally fused with the residual add),
//   per-head QK-RMSNorm + rotary embedding forward/backward (in place on the
//   packed qkv activation), SwiGLU forward/backward, embedding gather and
//   scatter-add backward, fused flat AdamW with bf16 shadow write, squared
//   norm / finite reduction, and the row-wise softmax statistics used by the
//   chunked LM-head log-prob / entropy / cross-entropy path.
//
// The reference implements these with Liger/Triton or HF eager torch ops
// (trainer/model.py Liger patches; kernels/swiglu.py:12-83 for SwiGLU;
// trainer/losses.py:600-1004 for the chunked log-prob head; trainer/optim.py
// for AdamW).  All math is fp32 in registers; tensors are bf16 unless noted.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace wb {

namespace {

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float r = (l < nw) ? red[l] : 0.f;
  r = warp_sum(r);
  return r;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

// ------------------------------------------------------------------ RMSNorm
// One warp per row; 8 bf16 (16 bytes) per lane per step.
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ res,
                                   __nv_bfloat16* __restrict__ h_out,
                                   const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out,
                                   int rows, int H, float eps) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * H);
  const uint4* rr = res ? reinterpret_cast<const uint4*>(res + (int64_t)row * H) : nullptr;
  uint4* hr = h_out ? reinterpret_cast<uint4*>(h_out + (int64_t)row * H) : nullptr;
  const int nv = H >> 3;
  float ss = 0.f;
  for (int i = lane; i < nv; i += 32) {
    uint4 a = xr[i];
    if (rr) {
      uint4 b = rr[i];
      uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        pa[j] = pack_bf16(bf16_lo(pa[j]) + bf16_lo(pb[j]), bf16_hi(pa[j]) + bf16_hi(pb[j]));
      if (hr) hr[i] = a;
    }
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float u = bf16_lo(pa[j]), v = bf16_hi(pa[j]);
      ss += u * u + v * v;
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / H + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = rstd;
  const uint4* src = rr ? reinterpret_cast<const uint4*>(h_out ? h_out + (int64_t)row * H : nullptr)
                        : xr;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + (int64_t)row * H);
  for (int i = lane; i < nv; i += 32) {
    uint4 a;
    if (rr && !h_out) {
      uint4 p = xr[i], q = rr[i];
      uint32_t* pa = reinterpret_cast<uint32_t*>(&p);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&q);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        pa[j] = pack_bf16(bf16_lo(pa[j]) + bf16_lo(pb[j]), bf16_hi(pa[j]) + bf16_hi(pb[j]));
      a = p;
    } else {
      a = src[i];
    }
    uint4 ww = wr[i];
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&ww);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      po[j] = pack_bf16(bf16_lo(pa[j]) * rstd * bf16_lo(pw[j]),
                        bf16_hi(pa[j]) * rstd * bf16_hi(pw[j]));
    yr[i] = o;
  }
}

// dx = rstd * (w*dy - xhat * mean(xhat*w*dy)) (+ dres).  One warp per row,
// each CTA a contiguous run of rows.  dw is a separate column pass
// (rmsnorm_dw_kernel) so that it is summed in a fixed order.
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w,
                                   const float* __restrict__ rstd,
                                   const __nv_bfloat16* __restrict__ dy,
                                   const __nv_bfloat16* __restrict__ dres,
                                   __nv_bfloat16* __restrict__ dx, int rows, int H, int rows_per_cta) {
  const int warps = blockDim.x >> 5;
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(rows, r0 + rows_per_cta);
  const int nv = H >> 3;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  for (int row = r0 + wid; row < r1; row += warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * H);
    const uint4* dyr = reinterpret_cast<const uint4*>(dy + (int64_t)row * H);
    const float rs = rstd[row];
    float dot = 0.f;
#pragma unroll 4
    for (int i = lane; i < nv; i += 32) {
      uint4 a = xr[i], g = dyr[i], ww = wr[i];
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
      const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&ww);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dot += bf16_lo(pa[j]) * bf16_lo(pg[j]) * bf16_lo(pw[j]);
        dot += bf16_hi(pa[j]) * bf16_hi(pg[j]) * bf16_hi(pw[j]);
      }
    }
    dot = warp_sum(dot) * rs;  // sum(xhat * w * dy)
    const float mean = dot / H;
    uint4* dxr = reinterpret_cast<uint4*>(dx + (int64_t)row * H);
    const uint4* drr = dres ? reinterpret_cast<const uint4*>(dres + (int64_t)row * H) : nullptr;
#pragma unroll 4
    for (int i = lane; i < nv; i += 32) {
      uint4 a = xr[i], g = dyr[i], ww = wr[i];
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
      const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&ww);
      uint4 rres = drr ? drr[i] : make_uint4(0, 0, 0, 0);
      const uint32_t* pr = reinterpret_cast<const uint32_t*>(&rres);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float xh0 = bf16_lo(pa[j]) * rs, xh1 = bf16_hi(pa[j]) * rs;
        const float d0 = rs * (bf16_lo(pw[j]) * bf16_lo(pg[j]) - xh0 * mean) + bf16_lo(pr[j]);
        const float d1 = rs * (bf16_hi(pw[j]) * bf16_hi(pg[j]) - xh1 * mean) + bf16_hi(pr[j]);
        po[j] = pack_bf16(d0, d1);
      }
      dxr[i] = o;
    }
  }
}

// part[s, c] = sum over the rows of split s of dy[r, c] * x[r, c] * rstd[r].
// Thread = 8 consecutive columns, block = 1024 columns, grid.y = row splits.
__global__ void rmsnorm_dw_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ rstd,
                                  const __nv_bfloat16* __restrict__ dy, float* __restrict__ part, int rows, int H,
                                  int rows_per_split) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;  // chunk of 8 columns
  if (c8 * 8 >= H) return;
  const int r0 = blockIdx.y * rows_per_split;
  const int r1 = min(rows, r0 + rows_per_split);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll 4
  for (int r = r0; r < r1; ++r) {
    const uint4 a = reinterpret_cast<const uint4*>(x + (int64_t)r * H)[c8];
    const uint4 g = reinterpret_cast<const uint4*>(dy + (int64_t)r * H)[c8];
    const float rs = rstd[r];
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
    const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[2 * j] += bf16_lo(pg[j]) * bf16_lo(pa[j]) * rs;
      acc[2 * j + 1] += bf16_hi(pg[j]) * bf16_hi(pa[j]) * rs;
    }
  }
  float4* dst = reinterpret_cast<float4*>(part + (int64_t)blockIdx.y * H + c8 * 8);
  dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// dw[c] += sum_s part[s, c], splits in order (reproducible).
__global__ void colsum_add_kernel(const float* __restrict__ part, int splits, int H, float* __restrict__ dw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int k = 0; k < splits; ++k) s += part[(int64_t)k * H + c];
  dw[c] += s;
}

// ------------------------------------------------------------ QK-norm + RoPE
// One warp per (token, head) of a 128-wide head; lane l holds elements
// [4l, 4l+4); rotate-half partners live 16 lanes apart.
__global__ void qk_norm_rope_fwd_kernel(__nv_bfloat16* __restrict__ qkv, int64_t row_stride,
                                        int n_q, int n_k, const int* __restrict__ pos,
                                        const float* __restrict__ inv_freq,
                                        const __nv_bfloat16* __restrict__ q_w,
                                        const __nv_bfloat16* __restrict__ k_w,
                                        float* __restrict__ rstd_out, int tokens, float eps) {
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = n_q + n_k;
  if (gw >= tokens * heads) return;
  const int t = gw / heads, h = gw - t * heads;
  __nv_bfloat16* base = qkv + (int64_t)t * row_stride + (int64_t)h * 128;
  uint2 raw = reinterpret_cast<uint2*>(base)[lane];
  float v[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  const __nv_bfloat16* nw = (h < n_q) ? q_w : k_w;
  if (nw) {
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / 128.f + eps);
    if (lane == 0 && rstd_out) rstd_out[gw] = rs;
    uint2 wraw = reinterpret_cast<const uint2*>(nw)[lane];
    v[0] = __bfloat162float(__float2bfloat16(v[0] * rs * bf16_lo(wraw.x)));
    v[1] = __bfloat162float(__float2bfloat16(v[1] * rs * bf16_hi(wraw.x)));
    v[2] = __bfloat162float(__float2bfloat16(v[2] * rs * bf16_lo(wraw.y)));
    v[3] = __bfloat162float(__float2bfloat16(v[3] * rs * bf16_hi(wraw.y)));
  }
  const float p = static_cast<float>(pos[t]);
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float other = __shfl_xor_sync(0xffffffffu, v[j], 16);
    const int d = (lane & 15) * 4 + j;  // frequency index in [0, 64)
    float s, c;
    sincosf(p * inv_freq[d], &s, &c);
    // first half: x1*cos - x2*sin ; second half: x2*cos + x1*sin
    o[j] = (lane < 16) ? (v[j] * c - other * s) : (v[j] * c + other * s);
  }
  raw.x = pack_bf16(o[0], o[1]);
  raw.y = pack_bf16(o[2], o[3]);
  reinterpret_cast<uint2*>(base)[lane] = raw;
}

// Backward of qk_norm_rope_fwd: `dqkv` holds dL/d(rotated output) on entry and
// dL/d(pre-norm input) on exit.  `qkv_pre` is the saved pre-norm activation.
__global__ void qk_norm_rope_bwd_kernel(__nv_bfloat16* __restrict__ dqkv, int64_t drow_stride,
                                        const __nv_bfloat16* __restrict__ qkv_pre,
                                        int64_t row_stride, int n_q, int n_k,
                                        const int* __restrict__ pos,
                                        const float* __restrict__ inv_freq,
                                        const __nv_bfloat16* __restrict__ q_w,
                                        const __nv_bfloat16* __restrict__ k_w,
                                        const float* __restrict__ rstd, float* __restrict__ dq_w,
                                        float* __restrict__ dk_w, int tokens) {
  __shared__ float sdq[128], sdk[128];
  for (int i = threadIdx.x; i < 128; i += blockDim.x) sdq[i] = 0.f, sdk[i] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = n_q + n_k;
  if (gw < tokens * heads) {
    const int t = gw / heads, h = gw - t * heads;
    __nv_bfloat16* dbase = dqkv + (int64_t)t * drow_stride + (int64_t)h * 128;
    uint2 draw = reinterpret_cast<uint2*>(dbase)[lane];
    float g[4] = {bf16_lo(draw.x), bf16_hi(draw.x), bf16_lo(draw.y), bf16_hi(draw.y)};
    const float p = static_cast<float>(pos[t]);
    float gr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float other = __shfl_xor_sync(0xffffffffu, g[j], 16);
      const int d = (lane & 15) * 4 + j;
      float s, c;
      sincosf(p * inv_freq[d], &s, &c);
      // transpose of the rotation
      gr[j] = (lane < 16) ? (g[j] * c + other * s) : (g[j] * c - other * s);
    }
    const __nv_bfloat16* nw = (h < n_q) ? q_w : k_w;
    if (nw) {
      const __nv_bfloat16* xb = qkv_pre + (int64_t)t * row_stride + (int64_t)h * 128;
      uint2 xraw = reinterpret_cast<const uint2*>(xb)[lane];
      uint2 wraw = reinterpret_cast<const uint2*>(nw)[lane];
      float x[4] = {bf16_lo(xraw.x), bf16_hi(xraw.x), bf16_lo(xraw.y), bf16_hi(xraw.y)};
      float wv[4] = {bf16_lo(wraw.x), bf16_hi(wraw.x), bf16_lo(wraw.y), bf16_hi(wraw.y)};
      const float rs = rstd[gw];
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) dot += x[j] * rs * wv[j] * gr[j];
      dot = warp_sum(dot) / 128.f;
      float* sacc = (h < n_q) ? sdq : sdk;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float xh = x[j] * rs;
        atomicAdd(&sacc[lane * 4 + j], gr[j] * xh);
        gr[j] = rs * (wv[j] * gr[j] - xh * dot);
      }
    }
    draw.x = pack_bf16(gr[0], gr[1]);
    draw.y = pack_bf16(gr[2], gr[3]);
    reinterpret_cast<uint2*>(dbase)[lane] = draw;
  }
  __syncthreads();
  if (dq_w && q_w)
    for (int i = threadIdx.x; i < 128; i += blockDim.x) atomicAdd(&dq_w[i], sdq[i]);
  if (dk_w && k_w)
    for (int i = threadIdx.x; i < 128; i += blockDim.x) atomicAdd(&dk_w[i], sdk[i]);
}

// ------------------------------------------------------------------ SwiGLU
// gu row = [gate (I) | up (I)];  h = silu(gate) * up.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ h, int64_t rows, int I) {
  const int nv = I >> 3;
  const int64_t total = rows * nv;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / nv;
    const int c = static_cast<int>(idx - r * nv);
    const uint4* gr = reinterpret_cast<const uint4*>(gu + r * 2 * I);
    uint4 g = gr[c], u = gr[nv + c];
    const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
    const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      po[j] = pack_bf16(silu_f(bf16_lo(pg[j])) * bf16_lo(pu[j]),
                        silu_f(bf16_hi(pg[j])) * bf16_hi(pu[j]));
    reinterpret_cast<uint4*>(h + r * I)[c] = o;
  }
}

// dgu = [dh*u*s*(1+g*(1-s)) | dh*silu(g)],  s = sigmoid(g).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, int64_t rows, int I) {
  const int nv = I >> 3;
  const int64_t total = rows * nv;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / nv;
    const int c = static_cast<int>(idx - r * nv);
    const uint4* gr = reinterpret_cast<const uint4*>(gu + r * 2 * I);
    uint4 g = gr[c], u = gr[nv + c];
    uint4 d = reinterpret_cast<const uint4*>(dh + r * I)[c];
    const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
    const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
    const uint32_t* pd = reinterpret_cast<const uint32_t*>(&d);
    uint4 og, ou;
    uint32_t* pog = reinterpret_cast<uint32_t*>(&og);
    uint32_t* pou = reinterpret_cast<uint32_t*>(&ou);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float gg[2] = {bf16_lo(pg[j]), bf16_hi(pg[j])};
      float uu[2] = {bf16_lo(pu[j]), bf16_hi(pu[j])};
      float dd[2] = {bf16_lo(pd[j]), bf16_hi(pd[j])};
      float rg[2], ru[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float s = 1.f / (1.f + __expf(-gg[e]));
        rg[e] = dd[e] * uu[e] * s * (1.f + gg[e] * (1.f - s));
        ru[e] = dd[e] * gg[e] * s;
      }
      pog[j] = pack_bf16(rg[0], rg[1]);
      pou[j] = pack_bf16(ru[0], ru[1]);
    }
    uint4* dr = reinterpret_cast<uint4*>(dgu + r * 2 * I);
    dr[c] = og;
    dr[nv + c] = ou;
  }
}

// ------------------------------------------------------------------ embedding
__global__ void embedding_fwd_kernel(const __nv_bfloat16* __restrict__ table,
                                     const int64_t* __restrict__ ids,
                                     __nv_bfloat16* __restrict__ out, int64_t T, int H,
                                     int64_t V) {
  const int nv = H >> 3;
  const int64_t total = T * nv;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / nv;
    const int c = static_cast<int>(idx - t * nv);
    int64_t id = ids[t];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);
    reinterpret_cast<uint4*>(out + t * H)[c] = reinterpret_cast<const uint4*>(table + id * H)[c];
  }
}

__global__ void embedding_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                     const int64_t* __restrict__ ids, float* __restrict__ dtable,
                                     int64_t T, int H, int64_t V) {
  const int nv = H >> 2;
  const int64_t total = T * nv;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / nv;
    const int c = static_cast<int>(idx - t * nv);
    int64_t id = ids[t];
    if (id < 0 || id >= V) continue;
    const uint2 g = reinterpret_cast<const uint2*>(dy + t * H)[c];
    float4 v = make_float4(bf16_lo(g.x), bf16_hi(g.x), bf16_lo(g.y), bf16_hi(g.y));
    atomicAdd(reinterpret_cast<float4*>(dtable + id * H) + c, v);
  }
}

// ------------------------------------------------------------------ AdamW
// Decoupled weight decay (torch.optim.AdamW semantics) over flat fp32 buffers
// with the gradient scaled by `gscale` (token normalisation x clip factor read
// from device memory so the step needs no host sync), writing the bf16 shadow.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v,
                             __nv_bfloat16* __restrict__ p16, int64_t n, float lr, float b1,
                             float b2, float eps, float wd, float bc1, float bc2,
                             const float* __restrict__ gscale_dev, float gscale_host) {
  const float gs = gscale_host * (gscale_dev ? *gscale_dev : 1.f);
  const float step = lr / bc1;
  const float rbc2 = rsqrtf(bc2);
  const int64_t n4 = n >> 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* ap = &pp.x;
    float* ag = &gg.x;
    float* am = &mm.x;
    float* av = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = ag[j] * gs;
      am[j] = b1 * am[j] + (1.f - b1) * gj;
      av[j] = b2 * av[j] + (1.f - b2) * gj * gj;
      ap[j] = ap[j] * (1.f - lr * wd);
      ap[j] -= step * am[j] / (sqrtf(av[j]) * rbc2 + eps);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p16) {
      uint2 o;
      o.x = pack_bf16(pp.x, pp.y);
      o.y = pack_bf16(pp.z, pp.w);
      reinterpret_cast<uint2*>(p16)[i] = o;
    }
  }
  // scalar tail
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gj = g[i] * gs;
    m[i] = b1 * m[i] + (1.f - b1) * gj;
    v[i] = b2 * v[i] + (1.f - b2) * gj * gj;
    p[i] = p[i] * (1.f - lr * wd) - step * m[i] / (sqrtf(v[i]) * rbc2 + eps);
    if (p16) p16[i] = __float2bfloat16(p[i]);
  }
}

// ------------------------------------------------------------------ 8-bit AdamW
// AdamW whose moments live in 8 bits per element with one fp32 scale per
// block of 256 elements (the memory class of bitsandbytes' 8-bit Adam,
// reference trainer/optim.py:393-512; the code is this library's own).
// Codes are logarithmic, relative to the block's absolute maximum a:
//   m (signed):  c in [-127, 127], |m| = a * 2^((|c| - 127) / 8), c = 0 -> 0
//   v (>= 0):    c in [0, 255],     v = a * 2^((c - 255) / 16),   c = 0 -> 0
// i.e. a relative step of 2^(1/8) (9%) for m and 2^(1/16) (4.4%) for v over
// about 16 octaves below the block maximum.  Each step dequantises, runs the
// fp32 AdamW update, takes the new block maxima and re-quantises (round to
// nearest in the log domain).  The fp32 master weights are kept in full.
constexpr int kQ8Block = 256;

__device__ __forceinline__ float q8m_decode(int8_t c, float a) {
  if (c == 0) return 0.f;
  const int mag = c < 0 ? -c : c;
  const float v = a * exp2f((float)(mag - 127) * 0.125f);
  return c < 0 ? -v : v;
}
__device__ __forceinline__ int8_t q8m_encode(float x, float a) {
  if (!(a > 0.f) || x == 0.f) return 0;
  const float r = fabsf(x) / a;
  float l = 127.f + 8.f * log2f(r);
  int c = (int)rintf(l);
  if (c < 1) c = (r >= 0.5f * exp2f(-126.f * 0.125f)) ? 1 : 0;
  c = min(c, 127);
  return (int8_t)(x < 0.f ? -c : c);
}
__device__ __forceinline__ float q8v_decode(uint8_t c, float a) {
  return c == 0 ? 0.f : a * exp2f((float)((int)c - 255) * 0.0625f);
}
__device__ __forceinline__ uint8_t q8v_encode(float x, float a) {
  if (!(a > 0.f) || !(x > 0.f)) return 0;
  const float r = x / a;
  int c = (int)rintf(255.f + 16.f * log2f(r));
  if (c < 1) c = (r >= 0.5f * exp2f(-254.f * 0.0625f)) ? 1 : 0;
  return (uint8_t)min(c, 255);
}

__global__ void __launch_bounds__(kQ8Block) adamw8_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                          int8_t* __restrict__ m8, uint8_t* __restrict__ v8,
                                                          float* __restrict__ am, float* __restrict__ av,
                                                          __nv_bfloat16* __restrict__ p16, int64_t n, float lr,
                                                          float b1, float b2, float eps, float wd, float bc1,
                                                          float bc2, const float* __restrict__ gscale_dev,
                                                          float gscale_host) {
  __shared__ float red_m[kQ8Block / 32], red_v[kQ8Block / 32];
  const float gs = gscale_host * (gscale_dev ? *gscale_dev : 1.f);
  const float step = lr / bc1;
  const float rbc2 = rsqrtf(bc2);
  const int64_t nblk = (n + kQ8Block - 1) / kQ8Block;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const int64_t i = blk * kQ8Block + threadIdx.x;
    const bool ok = i < n;
    float m = 0.f, v = 0.f;
    if (ok) {
      const float gj = g[i] * gs;
      m = b1 * q8m_decode(m8[i], am[blk]) + (1.f - b1) * gj;
      v = b2 * q8v_decode(v8[i], av[blk]) + (1.f - b2) * gj * gj;
      float w = p[i] * (1.f - lr * wd);
      w -= step * m / (sqrtf(v) * rbc2 + eps);
      p[i] = w;
      if (p16) p16[i] = __float2bfloat16(w);
    }
    float mx_m = fabsf(m), mx_v = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx_m = fmaxf(mx_m, __shfl_xor_sync(0xffffffffu, mx_m, o));
      mx_v = fmaxf(mx_v, __shfl_xor_sync(0xffffffffu, mx_v, o));
    }
    if (lane == 0) red_m[wid] = mx_m, red_v[wid] = mx_v;
    __syncthreads();
    mx_m = red_m[0];
    mx_v = red_v[0];
#pragma unroll
    for (int w = 1; w < kQ8Block / 32; ++w) mx_m = fmaxf(mx_m, red_m[w]), mx_v = fmaxf(mx_v, red_v[w]);
    __syncthreads();  // red_* is rewritten by the next block's reduction
    if (ok) {
      m8[i] = q8m_encode(m, mx_m);
      v8[i] = q8v_encode(v, mx_v);
    }
    if (threadIdx.x == 0) am[blk] = mx_m, av[blk] = mx_v;
  }
}

// Cross-block scratch of the deterministic grid sums (one launch at a time per
// device: the optimizer's reductions run in stream order).
constexpr int kMaxSumBlocks = 1024;
__device__ float g_sum_scratch[2 * kMaxSumBlocks];
__device__ unsigned g_sum_counter;

// Sum of squares of a flat fp32 buffer added to out[0] and the non-finite
// count to out[1], in a fixed order (bit-reproducible).
__global__ void sumsq_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f, bad = 0.f;
  const int64_t n4 = n >> 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = reinterpret_cast<const float4*>(x)[i];
    s += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    bad += (isfinite(a.x) && isfinite(a.y) && isfinite(a.z) && isfinite(a.w)) ? 0.f : 1.f;
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    s += x[i] * x[i];
    bad += isfinite(x[i]) ? 0.f : 1.f;
  }
  s = block_sum(s, red);
  __syncthreads();
  bad = block_sum(bad, red);
  grid_sum2_ordered(s, bad, g_sum_scratch, &g_sum_counter, out, red);
}

// clip factor = min(1, max_norm / (sqrt(sumsq) + 1e-6)); written to out.
__global__ void clip_factor_kernel(const float* __restrict__ sumsq, float max_norm,
                                   float* __restrict__ out) {
  const float norm = sqrtf(sumsq[0]);
  float f = 1.f;
  if (max_norm > 0.f) f = fminf(1.f, max_norm / (norm + 1e-6f));
  out[0] = f;
  out[1] = norm;
}

// ------------------------------------------------------ softmax row statistics
// For each row of z (bf16 logits, temperature tau): lse of z/tau, the target
// log-prob z_t/tau - lse and the entropy lse - sum p * z/tau.  One CTA per row,
// single pass with per-thread online (max, sum, weighted-sum) merged at the end.
// The running values live in the base-2 domain (v = z * log2(e) / tau), so every
// exponential is one ex2 of a difference; the max of each 8-logit load is taken on
// packed bf16 pairs (order is kept by the positive scale); two 16-byte loads per
// thread are in flight.  Results are converted back to natural-log units.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void stats_accum8(const uint4& a, float c, float& m, float& s, float& w) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162 mx = __hmax2(__hmax2(p[0], p[1]), __hmax2(p[2], p[3]));
  const float lm = fmaxf(__low2float(mx), __high2float(mx)) * c;
  if (lm > m) {
    const float sc = ex2_approx(m - lm);  // m = -inf on the first load: sc = 0, s = w = 0
    s *= sc;
    w *= sc;
    m = lm;
  }
  const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float v0 = bf16_lo(pa[j]) * c, v1 = bf16_hi(pa[j]) * c;
    const float e0 = ex2_approx(v0 - m), e1 = ex2_approx(v1 - m);
    s += e0 + e1;
    w = fmaf(e0, v0, fmaf(e1, v1, w));
  }
}

__device__ __forceinline__ void stats_merge(float& m, float& s, float& w, float m2, float s2, float w2) {
  const float mm = fmaxf(m, m2);
  const float a = (m == -INFINITY) ? 0.f : ex2_approx(m - mm);
  const float b = (m2 == -INFINITY) ? 0.f : ex2_approx(m2 - mm);
  s = s * a + s2 * b;
  w = w * a + w2 * b;
  m = mm;
}

__global__ void softmax_stats_kernel(const __nv_bfloat16* __restrict__ z, int64_t ldz, int V,
                                     const int64_t* __restrict__ target, float inv_tau,
                                     float* __restrict__ lse_out, float* __restrict__ lp_out,
                                     float* __restrict__ ent_out) {
  constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
  __shared__ float sm[32], ss[32], sw[32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* zr = z + row * ldz;
  const float c = inv_tau * kLog2e;
  float m = -INFINITY, s = 0.f, w = 0.f;
  const int nv = V >> 3;
  const uint4* zv = reinterpret_cast<const uint4*>(zr);
  for (int i = threadIdx.x; i < nv; i += 2 * blockDim.x) {
    const int i2 = i + blockDim.x;
    const uint4 a = zv[i];
    uint4 b = a;
    if (i2 < nv) b = zv[i2];
    stats_accum8(a, c, m, s, w);
    if (i2 < nv) stats_accum8(b, c, m, s, w);
  }
  for (int i = (nv << 3) + threadIdx.x; i < V; i += blockDim.x) {
    const float v = __bfloat162float(zr[i]) * c;
    if (v > m) {
      const float sc = ex2_approx(m - v);
      s *= sc;
      w *= sc;
      m = v;
    }
    const float e = ex2_approx(v - m);
    s += e;
    w = fmaf(e, v, w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    stats_merge(m, s, w, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o),
                __shfl_xor_sync(0xffffffffu, w, o));
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sm[wid] = m, ss[wid] = s, sw[wid] = w;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
    w = lane < nw ? sw[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      stats_merge(m, s, w, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o),
                  __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) {
      const float lse = m * kLn2 + __logf(s);  // sum_j e^(z_j/tau) = 2^m * s
      lse_out[row] = lse;
      if (ent_out) ent_out[row] = lse - (w / s) * kLn2;
      if (lp_out) {
        int64_t t = target ? target[row] : -1;
        lp_out[row] = (t >= 0 && t < V) ? __bfloat162float(zr[t]) * inv_tau - lse : 0.f;
      }
    }
  }
}

// In-place: z <- dL/dz = inv_tau * [dlp * (1[j=t] - p_j) - dent * p_j * (log p_j + H)].
__global__ void softmax_grad_kernel(__nv_bfloat16* __restrict__ z, int64_t ldz, int V,
                                    const int64_t* __restrict__ target, float inv_tau,
                                    const float* __restrict__ lse, const float* __restrict__ ent,
                                    const float* __restrict__ dlp, const float* __restrict__ dent) {
  const int64_t row = blockIdx.x;
  __nv_bfloat16* zr = z + row * ldz;
  const float L = lse[row];
  const float gl = dlp ? dlp[row] : 0.f;
  const float ge = dent ? dent[row] : 0.f;
  const float Hh = (ent && dent) ? ent[row] : 0.f;
  const int64_t t = target ? target[row] : -1;
  const int nv = V >> 3;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    uint4 a = reinterpret_cast<uint4*>(zr)[i];
    uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float r[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = i * 8 + 2 * j + e;
        const float zz = (e ? bf16_hi(pa[j]) : bf16_lo(pa[j])) * inv_tau;
        const float logp = zz - L;
        const float pj = __expf(logp);
        float gv = -gl * pj - ge * pj * (logp + Hh);
        if (col == t) gv += gl;
        r[e] = gv * inv_tau;
      }
      pa[j] = pack_bf16(r[0], r[1]);
    }
    reinterpret_cast<uint4*>(zr)[i] = a;
  }
  for (int col = (nv << 3) + threadIdx.x; col < V; col += blockDim.x) {
    const float zz = __bfloat162float(zr[col]) * inv_tau;
    const float logp = zz - L;
    const float pj = __expf(logp);
    float gv = -gl * pj - ge * pj * (logp + Hh);
    if (col == t) gv += gl;
    zr[col] = __float2bfloat16(gv * inv_tau);
  }
}

// NF4 -> bf16 dequantisation (QLoRA base weights at training batch sizes:
// dequantise once, then the dense tcgen05 GEMM).  One thread = one block of
// 64 elements: 32 bytes of codes (element 2i in the high nibble) + one fp32
// absmax -> 128 bytes of bf16.  Memory-bound: 2.56 bytes moved per element.
__global__ void __launch_bounds__(256) nf4_dequant_kernel(const uint4* __restrict__ codes,
                                                          const float* __restrict__ absmax,
                                                          uint4* __restrict__ out, int64_t nblk, float4 l0,
                                                          float4 l1, float4 l2, float4 l3) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) {
    const float t[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                         l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
    lut[threadIdx.x] = t[threadIdx.x];
  }
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nblk; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 w0 = __ldcs(codes + 2 * i);
    const uint4 w1 = __ldcs(codes + 2 * i + 1);
    const float am = __ldcs(absmax + i);
    const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    uint4* dst = out + 8 * i;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 o;
      uint32_t* op = &o.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t byte = (words[c] >> (8 * j)) & 0xffu;
        op[j] = pack_bf16(lut[byte >> 4] * am, lut[byte & 15u] * am);
      }
      dst[c] = o;
    }
  }
}

// Split-K reduction: out[m, n] = bf16(alpha * sum_s ws[s, m, n] + bias[n] + res[m, n]).
// 4 columns per thread (N % 4 == 0).
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, int S, int64_t M, int N,
                                                            __nv_bfloat16* __restrict__ out, int64_t ldc,
                                                            const __nv_bfloat16* __restrict__ bias,
                                                            const __nv_bfloat16* __restrict__ res, int64_t ldr,
                                                            float alpha) {
  const int64_t n4 = N / 4;
  const int64_t total = M * n4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / n4;
    const int c = (int)(i - m * n4) * 4;
    float4 acc = reinterpret_cast<const float4*>(ws + m * N + c)[0];
    for (int s = 1; s < S; ++s) {
      const float4 v = reinterpret_cast<const float4*>(ws + ((int64_t)s * M + m) * N + c)[0];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    float r[4] = {acc.x * alpha, acc.y * alpha, acc.z * alpha, acc.w * alpha};
    if (bias) {
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] += __bfloat162float(bias[c + j]);
    }
    if (res) {
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] += __bfloat162float(res[m * ldr + c + j]);
    }
    uint2 o;
    o.x = pack_bf16(r[0], r[1]);
    o.y = pack_bf16(r[2], r[3]);
    *reinterpret_cast<uint2*>(out + m * ldc + c) = o;
  }
}

inline int grid_for(int64_t work, int threads, int cap = 148 * 16) {
  int64_t g = (work + threads - 1) / threads;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

}  // namespace

void rmsnorm_fwd(const void* x, const void* res, void* h_out, const void* w, void* y,
                 float* rstd, int rows, int H, float eps, cudaStream_t st) {
  if (H % 8) throw std::runtime_error("rmsnorm: hidden size must be a multiple of 8");
  const int threads = 256, warps = threads / 32;
  rmsnorm_fwd_kernel<<<(rows + warps - 1) / warps, threads, 0, st>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)res, (__nv_bfloat16*)h_out,
      (const __nv_bfloat16*)w, (__nv_bfloat16*)y, rstd, rows, H, eps); note_launch();
}

int rmsnorm_dw_splits(int rows) { return rows < 64 ? 1 : (rows < 4096 ? rows / 64 : 64); }

void rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* dres,
                 void* dx, float* dw, float* part, int rows, int H, cudaStream_t st) {
  if (H % 8) throw std::runtime_error("rmsnorm: hidden size must be a multiple of 8");
  if (rows <= 0) return;
  const int threads = 256;
  const int ctas = 148 * 2;
  const int rows_per_cta = (rows + ctas - 1) / ctas;
  const int grid = (rows + rows_per_cta - 1) / rows_per_cta;
  rmsnorm_bwd_kernel<<<grid, threads, 0, st>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, rstd, (const __nv_bfloat16*)dy,
      (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, rows, H, rows_per_cta); note_launch();
  if (dw) {
    const int splits = rmsnorm_dw_splits(rows);
    const int per = (rows + splits - 1) / splits;
    rmsnorm_dw_kernel<<<dim3((H / 8 + 127) / 128, splits), 128, 0, st>>>(
        (const __nv_bfloat16*)x, rstd, (const __nv_bfloat16*)dy, part, rows, H, per); note_launch();
    colsum_add_kernel<<<(H + 255) / 256, 256, 0, st>>>(part, splits, H, dw); note_launch();
  }
}

void qk_norm_rope_fwd(void* qkv, int64_t row_stride, int n_q, int n_k, const int* pos,
                      const float* inv_freq, const void* q_w, const void* k_w, float* rstd,
                      int tokens, float eps, cudaStream_t st) {
  const int threads = 256, warps = 8;
  const int64_t work = (int64_t)tokens * (n_q + n_k);
  qk_norm_rope_fwd_kernel<<<(int)((work + warps - 1) / warps), threads, 0, st>>>(
      (__nv_bfloat16*)qkv, row_stride, n_q, n_k, pos, inv_freq, (const __nv_bfloat16*)q_w,
      (const __nv_bfloat16*)k_w, rstd, tokens, eps); note_launch();
}

void qk_norm_rope_bwd(void* dqkv, int64_t drow_stride, const void* qkv_pre, int64_t row_stride,
                      int n_q, int n_k, const int* pos, const float* inv_freq, const void* q_w,
                      const void* k_w, const float* rstd, float* dq_w, float* dk_w, int tokens,
                      cudaStream_t st) {
  const int threads = 256, warps = 8;
  const int64_t work = (int64_t)tokens * (n_q + n_k);
  qk_norm_rope_bwd_kernel<<<(int)((work + warps - 1) / warps), threads, 0, st>>>(
      (__nv_bfloat16*)dqkv, drow_stride, (const __nv_bfloat16*)qkv_pre, row_stride, n_q, n_k, pos,
      inv_freq, (const __nv_bfloat16*)q_w, (const __nv_bfloat16*)k_w, rstd, dq_w, dk_w, tokens); note_launch();
}

void swiglu_fwd(const void* gu, void* h, int64_t rows, int I, cudaStream_t st) {
  if (I % 8) throw std::runtime_error("swiglu: intermediate size must be a multiple of 8");
  swiglu_fwd_kernel<<<grid_for(rows * (I / 8), 256), 256, 0, st>>>((const __nv_bfloat16*)gu,
                                                                  (__nv_bfloat16*)h, rows, I); note_launch();
}

void swiglu_bwd(const void* gu, const void* dh, void* dgu, int64_t rows, int I, cudaStream_t st) {
  if (I % 8) throw std::runtime_error("swiglu: intermediate size must be a multiple of 8");
  swiglu_bwd_kernel<<<grid_for(rows * (I / 8), 256), 256, 0, st>>>(
      (const __nv_bfloat16*)gu, (const __nv_bfloat16*)dh, (__nv_bfloat16*)dgu, rows, I); note_launch();
}

void embedding_fwd(const void* table, const int64_t* ids, void* out, int64_t T, int H, int64_t V,
                   cudaStream_t st) {
  embedding_fwd_kernel<<<grid_for(T * (H / 8), 256), 256, 0, st>>>(
      (const __nv_bfloat16*)table, ids, (__nv_bfloat16*)out, T, H, V); note_launch();
}

void embedding_bwd(const void* dy, const int64_t* ids, float* dtable, int64_t T, int H, int64_t V,
                   cudaStream_t st) {
  embedding_bwd_kernel<<<grid_for(T * (H / 4), 256), 256, 0, st>>>((const __nv_bfloat16*)dy, ids,
                                                                  dtable, T, H, V); note_launch();
}

void splitk_reduce(const float* ws, int S, int64_t M, int N, void* out, int64_t ldc, const void* bias, const void* res,
                   int64_t ldr, float alpha, cudaStream_t st) {
  if (M <= 0 || N <= 0) return;
  if (N % 4 || ldc % 4 || (res && ldr % 4)) throw std::runtime_error("splitk_reduce: N and strides must be multiples of 4");
  splitk_reduce_kernel<<<grid_for(M * (N / 4), 256, 148 * 8), 256, 0, st>>>(
      ws, S, M, N, (__nv_bfloat16*)out, ldc, (const __nv_bfloat16*)bias, (const __nv_bfloat16*)res, ldr, alpha); note_launch();
}

void nf4_dequant(const void* codes, const float* absmax, void* out, int64_t numel, const float* lut,
                 cudaStream_t st) {
  if (numel <= 0) return;
  if (numel % 64) throw std::runtime_error("nf4_dequant: numel must be a multiple of 64");
  const int64_t nblk = numel / 64;
  nf4_dequant_kernel<<<grid_for(nblk, 256, 148 * 8), 256, 0, st>>>(
      (const uint4*)codes, absmax, (uint4*)out, nblk, make_float4(lut[0], lut[1], lut[2], lut[3]),
      make_float4(lut[4], lut[5], lut[6], lut[7]), make_float4(lut[8], lut[9], lut[10], lut[11]),
      make_float4(lut[12], lut[13], lut[14], lut[15])); note_launch();
}

void adamw_step(float* p, const float* g, float* m, float* v, void* p16, int64_t n, float lr,
                float b1, float b2, float eps, float wd, float bc1, float bc2,
                const float* gscale_dev, float gscale_host, cudaStream_t st) {
  if (n <= 0) return;
  adamw_kernel<<<grid_for((n + 3) / 4, 256, 148 * 8), 256, 0, st>>>(
      p, g, m, v, (__nv_bfloat16*)p16, n, lr, b1, b2, eps, wd, bc1, bc2, gscale_dev, gscale_host); note_launch();
}

void adamw8_step(float* p, const float* g, int8_t* m8, uint8_t* v8, float* am, float* av, void* p16, int64_t n,
                 float lr, float b1, float b2, float eps, float wd, float bc1, float bc2, const float* gscale_dev,
                 float gscale_host, cudaStream_t st) {
  if (n <= 0) return;
  adamw8_kernel<<<grid_for((n + kQ8Block - 1) / kQ8Block, 1, 148 * 8), kQ8Block, 0, st>>>(
      p, g, m8, v8, am, av, (__nv_bfloat16*)p16, n, lr, b1, b2, eps, wd, bc1, bc2, gscale_dev, gscale_host);
  note_launch();
}

void sumsq(const float* x, int64_t n, float* out, cudaStream_t st) {
  if (n <= 0) return;
  static_assert(148 * 4 <= kMaxSumBlocks, "sumsq grid exceeds the scratch");
  sumsq_kernel<<<grid_for((n + 3) / 4, 256, 148 * 4), 256, 0, st>>>(x, n, out); note_launch();
}

void clip_factor(const float* sumsq_v, float max_norm, float* out, cudaStream_t st) {
  clip_factor_kernel<<<1, 1, 0, st>>>(sumsq_v, max_norm, out); note_launch();
}

void softmax_stats(const void* z, int64_t ldz, int rows, int V, const int64_t* target,
                   float inv_tau, float* lse, float* lp, float* ent, cudaStream_t st) {
  if (rows <= 0) return;
  if ((ldz % 8) || (reinterpret_cast<uintptr_t>(z) & 15))
    throw std::runtime_error("softmax_stats: rows must be 16-byte aligned");
  softmax_stats_kernel<<<rows, 512, 0, st>>>((const __nv_bfloat16*)z, ldz, V, target, inv_tau,
                                             lse, lp, ent); note_launch();
}

void softmax_grad(void* z, int64_t ldz, int rows, int V, const int64_t* target, float inv_tau,
                  const float* lse, const float* ent, const float* dlp, const float* dent,
                  cudaStream_t st) {
  if (rows <= 0) return;
  if ((ldz % 8) || (reinterpret_cast<uintptr_t>(z) & 15))
    throw std::runtime_error("softmax_grad: rows must be 16-byte aligned");
  softmax_grad_kernel<<<rows, 512, 0, st>>>((__nv_bfloat16*)z, ldz, V, target, inv_tau, lse, ent,
                                            dlp, dent); note_launch();
}

}  // namespace wb
