// Peer-memory fabric (CUDA IPC) and the fused reduce-scatter -> AdamW ->
// all-gather optimizer step over NVLink.  Layout and protocol: comm.h.
//
// Roofline of the fused step on W ranks with a flat fp32 gradient of P
// elements: each rank pulls (W-1)/W * 4P bytes of gradient over NVLink and
// pushes (W-1)/W * 2P bytes of bf16 parameters, i.e. the same bytes as NCCL's
// reduce-scatter + all-gather, but the sum, the norm, the clip, the AdamW
// update and the bf16 cast ride along with the transfer instead of running
// as separate passes over HBM.
#include <cstring>
#include <stdexcept>
#include <string>

#include "comm.h"
#include "common.cuh"

namespace wb {
namespace comm {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_sys(float* p, float v) {
  asm volatile("st.relaxed.sys.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__device__ __forceinline__ float ld_relaxed_sys(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

// Wait until *p has reached `epoch` (wrap-safe); false when the budget ran out.
__device__ bool wait_epoch(const uint32_t* p, uint32_t epoch, uint64_t budget_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (static_cast<int32_t>(ld_acquire_sys(p) - epoch) < 0) {
    if (globaltimer_ns() - t0 > budget_ns) return false;
    __nanosleep(100);
  }
  return true;
}

// One thread signals every peer, then waits for every peer.  A single thread
// keeps the acquire/release reasoning local; the kernel is latency-bound
// anyway (a few microseconds over NVSwitch).
__global__ void barrier_kernel(PeerPtrs pads, int rank, int world, uint32_t epoch, int slot_base,
                               uint64_t budget_ns, int* err) {
  if (threadIdx.x != 0) return;
  // Cumulative fence: everything this GPU wrote before this kernel (earlier
  // kernels on the stream) is ordered before the signal stores.
  __threadfence_system();
  for (int t = 0; t < world; ++t) st_release_sys(static_cast<uint32_t*>(pads.p[t]) + slot_base + rank, epoch);
  const uint32_t* mine = static_cast<const uint32_t*>(pads.p[rank]) + slot_base;
  for (int t = 0; t < world; ++t) {
    if (!wait_epoch(mine + t, epoch, budget_ns)) {
      atomicOr(err, kErrTimeoutPeer);
      return;
    }
  }
  __threadfence_system();
}

__global__ void norm_exchange_kernel(PeerPtrs pads, int rank, int world, uint32_t epoch, const float* stats,
                                     float max_norm, float* tot, uint64_t budget_ns, int* err) {
  if (threadIdx.x != 0) return;
  const float ss = stats[0], bad = stats[1];
  __threadfence_system();
  for (int t = 0; t < world; ++t) {
    uint32_t* pad = static_cast<uint32_t*>(pads.p[t]);
    float* vals = reinterpret_cast<float*>(pad + kPadNormVals) + 2 * rank;
    st_relaxed_sys(vals, ss);
    st_relaxed_sys(vals + 1, bad);
    st_release_sys(pad + kPadNormFlag + rank, epoch);  // release: orders the two value stores
  }
  const uint32_t* mine = static_cast<const uint32_t*>(pads.p[rank]);
  const float* mvals = reinterpret_cast<const float*>(mine + kPadNormVals);
  float s = 0.f, b = 0.f;
  bool ok = true;
  for (int t = 0; t < world; ++t) {  // fixed order: identical totals on every rank
    if (!wait_epoch(mine + kPadNormFlag + t, epoch, budget_ns)) {
      atomicOr(err, kErrTimeoutPeer);
      ok = false;
      break;
    }
    s += ld_relaxed_sys(mvals + 2 * t);
    b += ld_relaxed_sys(mvals + 2 * t + 1);
  }
  if (!ok) b = 1.f;  // a missing peer: treat as non-finite so no rank updates from a partial norm
  // finite gradients whose squared norm overflows: no usable clip factor, so
  // skip the step when clipping is on (with clipping off the step proceeds)
  if (!isfinite(s) && max_norm > 0.f) b += 1.f;
  float factor = 1.f;
  if (max_norm > 0.f) factor = fminf(1.f, max_norm / (sqrtf(s) + 1e-6f));
  tot[0] = s;
  tot[1] = b;
  tot[2] = factor;
}

__device__ __forceinline__ void add4(float4& a, const float4& b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  }
  return v;
}

// Each thread owns 8 consecutive floats (two 16-byte loads per rank, all
// ranks' loads issued before the adds so W*2 requests are in flight).
constexpr int kMaxSumBlocks = 1024;
__device__ float g_sum_scratch[2 * kMaxSumBlocks];
__device__ unsigned g_sum_counter;

template <int W>
__global__ void __launch_bounds__(512) rs_kernel(PeerPtrs grads, int64_t lo, int64_t n8, float scale, float* out,
                                                 float* stats, int64_t w_end, float w_lo) {
  __shared__ float red[32];
  float ss = 0.f, bad = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    // elements below w_end (a multiple of 8) enter the squared norm with weight
    // w_lo: parameters replicated over tensor-parallel ranks are counted once
    // in the cross-TP norm sum (each of the tp replicas adds 1/tp of them)
    const float wgt = (lo + 8 * i < w_end) ? w_lo : 1.f;
    float4 x0[W], x1[W];
#pragma unroll
    for (int r = 0; r < W; ++r) {
      const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(grads.p[r]) + lo) + 2 * i;
      x0[r] = src[0];
      x1[r] = src[1];
    }
    float4 a0 = x0[0], a1 = x1[0];
#pragma unroll
    for (int r = 1; r < W; ++r) {
      add4(a0, x0[r]);
      add4(a1, x1[r]);
    }
    float* e0 = &a0.x;
    float* e1 = &a1.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      e0[j] *= scale;
      e1[j] *= scale;
      ss += wgt * (e0[j] * e0[j] + e1[j] * e1[j]);
      bad += (isfinite(e0[j]) ? 0.f : 1.f) + (isfinite(e1[j]) ? 0.f : 1.f);
    }
    float4* dst = reinterpret_cast<float4*>(out) + 2 * i;
    dst[0] = a0;
    dst[1] = a1;
  }
  ss = block_sum(ss, red);
  __syncthreads();
  bad = block_sum(bad, red);
  grid_sum2_ordered(ss, bad, g_sum_scratch, &g_sum_counter, stats, red);  // fixed order: reproducible norm
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int W>
__global__ void __launch_bounds__(256) adamw_ag_kernel(PeerPtrs compute, int64_t lo, float* __restrict__ master,
                                                       const float* __restrict__ g, float* __restrict__ m,
                                                       float* __restrict__ v, int64_t n8, float lr, float b1, float b2,
                                                       float eps, float wd, float bc1, float bc2, const float* tot) {
  const bool skip = tot[1] > 0.f;
  const float gs = tot[2];
  const float step = lr / bc1;
  const float rbc2 = rsqrtf(bc2);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float4 p[2], gg[2], mm[2], vv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      p[h] = reinterpret_cast<const float4*>(master)[2 * i + h];
      gg[h] = reinterpret_cast<const float4*>(g)[2 * i + h];
      mm[h] = reinterpret_cast<const float4*>(m)[2 * i + h];
      vv[h] = reinterpret_cast<const float4*>(v)[2 * i + h];
    }
    if (!skip) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float* ap = &p[h].x;
        float* ag = &gg[h].x;
        float* am = &mm[h].x;
        float* av = &vv[h].x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float gj = ag[j] * gs;
          am[j] = b1 * am[j] + (1.f - b1) * gj;
          av[j] = b2 * av[j] + (1.f - b2) * gj * gj;
          ap[j] = ap[j] * (1.f - lr * wd);
          ap[j] -= step * am[j] / (sqrtf(av[j]) * rbc2 + eps);
        }
        reinterpret_cast<float4*>(master)[2 * i + h] = p[h];
        reinterpret_cast<float4*>(m)[2 * i + h] = mm[h];
        reinterpret_cast<float4*>(v)[2 * i + h] = vv[h];
      }
    }
    uint4 w;
    w.x = pack2(p[0].x, p[0].y);
    w.y = pack2(p[0].z, p[0].w);
    w.z = pack2(p[1].x, p[1].y);
    w.w = pack2(p[1].z, p[1].w);
#pragma unroll
    for (int r = 0; r < W; ++r)
      reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(compute.p[r]) + lo)[i] = w;
  }
}

template <int W>
__global__ void __launch_bounds__(256) ag_kernel(PeerPtrs dst, int64_t lo, const uint4* __restrict__ src, int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 w = src[i];
#pragma unroll
    for (int r = 0; r < W; ++r) reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dst.p[r]) + lo)[i] = w;
  }
}

// ---------------------------------------------------------------- expert-parallel rows
// Dispatch: row i of the send list goes to rank dst_rank[i], row dst_row[i] of
// that rank's receive buffer: out = bf16(scale[i] * x[src_row[i]]).  One warp
// per row, 16-byte stores straight into peer memory over NVLink (the gather,
// the routing-weight scale and the transfer are one pass).
__global__ void __launch_bounds__(256) rows_scatter_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                           const int64_t* __restrict__ src_row,
                                                           const int* __restrict__ dst_rank,
                                                           const int64_t* __restrict__ dst_row,
                                                           const float* __restrict__ scale, PeerPtrs dst, int64_t ldd,
                                                           int n, int H, int64_t limit_rows) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  // a row outside the destination buffer (an over-capacity layout, which the
  // layout kernel has already reported) is dropped, never written
  if (limit_rows >= 0 && (dst_row[w] < 0 || dst_row[w] >= limit_rows)) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + src_row[w] * ldx);
  uint4* out = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dst.p[dst_rank[w]]) + dst_row[w] * ldd);
  const float sc = scale ? scale[w] : 1.f;
  for (int c = lane; c < H / 8; c += 32) {
    uint4 v = src[c];
    if (scale) {
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        h[j] = __floats2bfloat162_rn(f.x * sc, f.y * sc);
      }
    }
    out[c] = v;
  }
}

// Combine: out[t] = res[t] + sum_j w[t*k+j] * src[src_rank[t*k+j]][src_row[t*k+j]]
// (fp32 accumulation in a fixed slot order; out bf16 or fp32).  One warp per
// token, plain 16-byte loads from peer memory.
template <bool F32OUT>
__global__ void __launch_bounds__(256) rows_gather_sum_kernel(PeerPtrs src, int64_t lds,
                                                              const int* __restrict__ src_rank,
                                                              const int64_t* __restrict__ src_row,
                                                              const float* __restrict__ wt, int k,
                                                              const __nv_bfloat16* __restrict__ res, int64_t ldr,
                                                              void* __restrict__ out, int64_t ldo, int T, int H,
                                                              int64_t limit_rows) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int c = lane; c < H / 8; c += 32) {
    float acc[8];
    if (res) {
      const uint4 r = reinterpret_cast<const uint4*>(res + (int64_t)t * ldr)[c];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] = f.x;
        acc[2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    for (int s = 0; s < k; ++s) {
      const int64_t i = (int64_t)t * k + s;
      if (limit_rows >= 0 && (src_row[i] < 0 || src_row[i] >= limit_rows)) continue;  // never read out of bounds
      const float wv = wt ? wt[i] : 1.f;
      const uint4 v = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(src.p[src_rank[i]]) +
                                                     src_row[i] * lds)[c];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += wv * f.x;
        acc[2 * j + 1] += wv * f.y;
      }
    }
    if constexpr (F32OUT) {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + (int64_t)t * ldo) + 2 * c;
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      uint4 o;
      o.x = pack2(acc[0], acc[1]);
      o.y = pack2(acc[2], acc[3]);
      o.z = pack2(acc[4], acc[5]);
      o.w = pack2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + (int64_t)t * ldo)[c] = o;
    }
  }
}

// Pull-gather: dst[r * n + i] = src[r][off + i] for every rank r (16-byte
// loads from peer memory; n and off multiples of 8 bf16).  Used to re-form a
// full weight tensor from its expert-parallel shards in place.
__global__ void __launch_bounds__(256) gather_from_peers_kernel(PeerPtrs src, int world, int64_t off, int64_t n8,
                                                                uint4* __restrict__ dst) {
  const int64_t total = n8 * world;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / n8);
    const int64_t j = i - (int64_t)r * n8;
    dst[i] = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(src.p[r]) + off)[j];
  }
}

// out[i] = res[i] + sum_r slots[r * stride + i] in rank order (fp32 sum, bf16
// out): the local half of the fused GEMM -> all-reduce, run after the
// barrier that orders every peer's epilogue stores into `slots`.  Every rank
// sums the same values in the same order, so all replicas agree bit for bit.
__global__ void __launch_bounds__(256) slots_sum_kernel(const __nv_bfloat16* __restrict__ slots, int world,
                                                        int64_t stride, int64_t n8,
                                                        const __nv_bfloat16* __restrict__ res,
                                                        __nv_bfloat16* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float f[8];
    if (res) {
      const uint4 w = reinterpret_cast<const uint4*>(res)[i];
      f[0] = bf16_lo(w.x), f[1] = bf16_hi(w.x), f[2] = bf16_lo(w.y), f[3] = bf16_hi(w.y);
      f[4] = bf16_lo(w.z), f[5] = bf16_hi(w.z), f[6] = bf16_lo(w.w), f[7] = bf16_hi(w.w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = 0.f;
    }
    for (int r = 0; r < world; ++r) {
      const uint4 w = reinterpret_cast<const uint4*>(slots + r * stride)[i];
      f[0] += bf16_lo(w.x), f[1] += bf16_hi(w.x), f[2] += bf16_lo(w.y), f[3] += bf16_hi(w.y);
      f[4] += bf16_lo(w.z), f[5] += bf16_hi(w.z), f[6] += bf16_lo(w.w), f[7] += bf16_hi(w.w);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]),
                                                  pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
  }
}

inline int grid_for(int64_t work, int threads, int cap) {
  int64_t b = (work + threads - 1) / threads;
  if (b < 1) b = 1;
  return static_cast<int>(b < cap ? b : cap);
}

}  // namespace comm

static void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string("wavelet_b200 fabric: ") + what + ": " + cudaGetErrorString(e));
}

void* fabric_malloc(size_t bytes) {
  void* p = nullptr;
  check(cudaMalloc(&p, bytes), "cudaMalloc");
  check(cudaMemset(p, 0, bytes), "cudaMemset");
  return p;
}

void fabric_free(void* p) {
  if (p) cudaFree(p);
}

void fabric_export(void* p, unsigned char out[64]) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  std::memcpy(out, &h, 64);
}

void* fabric_import(const unsigned char in[64]) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, in, 64);
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return p;
}

void fabric_close(void* p) {
  if (p) cudaIpcCloseMemHandle(p);
}

static void check_world(int world) {
  if (world < 1 || world > kMaxPeers) throw std::runtime_error("wavelet_b200 fabric: world size must be 1..8");
}

void peer_barrier(const PeerPtrs& pads, int rank, int world, uint32_t epoch, int slot_base, uint64_t budget_ns,
                  int* err, cudaStream_t st) {
  check_world(world);
  comm::barrier_kernel<<<1, 32, 0, st>>>(pads, rank, world, epoch, slot_base, budget_ns, err); note_launch();
}

void norm_exchange(const PeerPtrs& pads, int rank, int world, uint32_t epoch, const float* stats, float max_norm,
                   float* tot, uint64_t budget_ns, int* err, cudaStream_t st) {
  check_world(world);
  comm::norm_exchange_kernel<<<1, 32, 0, st>>>(pads, rank, world, epoch, stats, max_norm, tot, budget_ns, err); note_launch();
}

#define WB_WORLD_SWITCH(W, ...)                          \
  switch (W) {                                           \
    case 1: { constexpr int kW = 1; __VA_ARGS__; } break; \
    case 2: { constexpr int kW = 2; __VA_ARGS__; } break; \
    case 3: { constexpr int kW = 3; __VA_ARGS__; } break; \
    case 4: { constexpr int kW = 4; __VA_ARGS__; } break; \
    case 5: { constexpr int kW = 5; __VA_ARGS__; } break; \
    case 6: { constexpr int kW = 6; __VA_ARGS__; } break; \
    case 7: { constexpr int kW = 7; __VA_ARGS__; } break; \
    case 8: { constexpr int kW = 8; __VA_ARGS__; } break; \
    default: throw std::runtime_error("wavelet_b200 fabric: world size must be 1..8"); \
  }

void rs_sum_sumsq(const PeerPtrs& grads, int world, int64_t lo, int64_t n, float scale, float* out, float* stats,
                  int64_t w_end, float w_lo, cudaStream_t st) {
  if (n <= 0) return;
  if (n % 8 || lo % 8 || w_end % 8)
    throw std::runtime_error("wavelet_b200 fabric: shard and norm-weight boundary must be multiples of 8 elements");
  const int64_t n8 = n / 8;
  const int grid = comm::grid_for(n8, 512, 148 * 4);
  WB_WORLD_SWITCH(world, comm::rs_kernel<kW><<<grid, 512, 0, st>>>(grads, lo, n8, scale, out, stats, w_end, w_lo));
  note_launch();
}

void adamw_allgather(const PeerPtrs& compute, int world, int64_t lo, float* master, const float* g, float* m, float* v,
                     int64_t n, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                     const float* tot, cudaStream_t st) {
  if (n <= 0) return;
  if (n % 8 || lo % 8) throw std::runtime_error("wavelet_b200 fabric: shard must be a multiple of 8 elements");
  const int64_t n8 = n / 8;
  const int grid = comm::grid_for(n8, 256, 148 * 8);
  WB_WORLD_SWITCH(world, comm::adamw_ag_kernel<kW><<<grid, 256, 0, st>>>(compute, lo, master, g, m, v, n8, lr, b1, b2,
                                                                            eps, wd, bc1, bc2, tot)); note_launch();
}

void allgather_bf16(const PeerPtrs& dst, int world, int64_t lo, const void* src, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  if (n % 8 || lo % 8) throw std::runtime_error("wavelet_b200 fabric: shard must be a multiple of 8 elements");
  const int64_t n8 = n / 8;
  const int grid = comm::grid_for(n8, 256, 148 * 8);
  WB_WORLD_SWITCH(world, comm::ag_kernel<kW><<<grid, 256, 0, st>>>(dst, lo, static_cast<const uint4*>(src), n8)); note_launch();
}

void gather_from_peers(const PeerPtrs& src, int world, int64_t off, int64_t n, void* dst, cudaStream_t st) {
  if (n <= 0) return;
  if (n % 8 || off % 8) throw std::runtime_error("wavelet_b200 gather_from_peers: n and offset must be multiples of 8");
  comm::gather_from_peers_kernel<<<comm::grid_for(n / 8 * world, 256, 148 * 8), 256, 0, st>>>(
      src, world, off, n / 8, static_cast<uint4*>(dst)); note_launch();
}

void slots_sum(const void* slots, int world, int64_t stride, int64_t n, const void* res, void* out,
               cudaStream_t st) {
  if (n <= 0) return;
  if (n % 8 || stride % 8) throw std::runtime_error("wavelet_b200 slots_sum: n and slot stride must be multiples of 8");
  comm::slots_sum_kernel<<<comm::grid_for(n / 8, 256, 148 * 8), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(slots), world, stride, n / 8, static_cast<const __nv_bfloat16*>(res),
      static_cast<__nv_bfloat16*>(out)); note_launch();
}

void rows_scatter(const void* x, int64_t ldx, const int64_t* src_row, const int* dst_rank, const int64_t* dst_row,
                  const float* scale, const PeerPtrs& dst, int64_t ldd, int n, int H, int64_t limit_rows,
                  cudaStream_t st) {
  if (n <= 0) return;
  if (H % 8 || ldx % 8 || ldd % 8) throw std::runtime_error("wavelet_b200 rows_scatter: H and strides must be multiples of 8");
  comm::rows_scatter_kernel<<<(n + 7) / 8, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx, src_row, dst_rank,
                                                         dst_row, scale, dst, ldd, n, H, limit_rows); note_launch();
}

void rows_gather_sum(const PeerPtrs& src, int64_t lds, const int* src_rank, const int64_t* src_row, const float* w,
                     int k, const void* res, int64_t ldr, void* out, int64_t ldo, bool f32_out, int T, int H,
                     int64_t limit_rows, cudaStream_t st) {
  if (T <= 0) return;
  if (H % 8 || lds % 8 || ldo % 8 || (res && ldr % 8))
    throw std::runtime_error("wavelet_b200 rows_gather_sum: H and strides must be multiples of 8");
  const int grid = (T + 7) / 8;
  if (f32_out)
    comm::rows_gather_sum_kernel<true><<<grid, 256, 0, st>>>(src, lds, src_rank, src_row, w, k,
                                                             static_cast<const __nv_bfloat16*>(res), ldr, out, ldo, T, H,
                                                             limit_rows);
  else
    comm::rows_gather_sum_kernel<false><<<grid, 256, 0, st>>>(src, lds, src_rank, src_row, w, k,
                                                              static_cast<const __nv_bfloat16*>(res), ldr, out, ldo, T, H,
                                                             limit_rows);
  note_launch();
}

}  // namespace wb
