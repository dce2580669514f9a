// MoE routing on the device: router softmax / top-k, and the padded
// expert-major row layout that the grouped expert GEMMs consume, built
// without a host round trip (the reference reads the expert counts back to
// the host to size its all-to-all, trainer/moe.py:201-202).
//
//   moe_route     logits [T, E] fp32 -> probs [T, E], top-k experts / weights
//                 (optionally renormalised), per-expert copy counts.
//   moe_layout    all ranks' counts [ep, E] -> for every global expert the
//                 first row of this rank's copies in its owner's layout, and
//                 this rank's receive layout: per local expert the segment
//                 start / padded length / row count, and the expert of every
//                 128-row tile (-1 past the end, so the grouped GEMM skips it).
//                 A layout that does not fit the capacity of any rank sets
//                 the overflow flag (kErrEpOverflow); the layout is then
//                 empty (no tiles, zero-length segments) and every transfer
//                 of that layer is skipped: nothing is written out of bounds
//                 and nothing reads rows that were not written.
//   moe_copy_rows stable row of every (token, slot) copy in its owner's layout
//                 (copies of one expert keep (token, slot) order), and the
//                 owner rank.
//   moe_zero_pad  zero the padding rows of this rank's layout.
//   moe_put_counts  store this rank's counts into every peer's count table
//                 (expert parallelism over peer memory; a fabric barrier
//                 follows before anyone reads the table).
#include <cuda_bf16.h>
#include <stdint.h>

#include <stdexcept>

#include "comm.h"
#include "common.cuh"
#include "moe.h"

namespace wb {
namespace {

constexpr int kRouteMaxE = 256;  // 8 router logits per lane

// One warp per token.  Ties in the top-k go to the lower expert index.
__global__ void __launch_bounds__(256) moe_route_kernel(const float* __restrict__ logits, int T, int E, int k,
                                                        int norm_topk, int bf16_logits, float* __restrict__ probs,
                                                        int64_t* __restrict__ topi, float* __restrict__ topv,
                                                        float* __restrict__ w, float* __restrict__ ssum,
                                                        int* __restrict__ counts) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  constexpr int PER = kRouteMaxE / 32;
  float v[PER];
  const float* row = logits + (int64_t)t * E;
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = j * 32 + lane;
    float x = e < E ? row[e] : -INFINITY;
    if (bf16_logits && e < E) x = __bfloat162float(__float2bfloat16(x));
    v[j] = x;
    mx = fmaxf(mx, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = j * 32 + lane;
    v[j] = e < E ? __expf(v[j] - mx) : 0.f;
    sum += v[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.f / sum;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = j * 32 + lane;
    v[j] *= inv;
    if (e < E) probs[(int64_t)t * E + e] = v[j];
  }
  // top-k by k rounds of a warp arg-max over the not yet taken experts
  unsigned taken = 0;  // bit j: this lane's expert j*32+lane is taken
  float tot = 0.f;
  for (int r = 0; r < k; ++r) {
    float best = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = j * 32 + lane;
      if (e < E && !((taken >> j) & 1u) && v[j] > best) best = v[j], bi = e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (b2 > best || (b2 == best && i2 < bi)) best = b2, bi = i2;
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == 0) {
      topi[(int64_t)t * k + r] = bi;
      topv[(int64_t)t * k + r] = best;
      atomicAdd(&counts[bi], 1);
    }
    tot += best;
  }
  if (lane == 0) {
    ssum[t] = tot;
    const float sc = norm_topk ? 1.f / tot : 1.f;
    for (int r = 0; r < k; ++r) w[(int64_t)t * k + r] = topv[(int64_t)t * k + r] * sc;
  }
}

// One CTA of E threads (E <= 1024); thread ge = global expert ge = d * El + el.
__global__ void moe_layout_kernel(const int* __restrict__ allc, int ep, int me, int E, int pad, int64_t cap_rows,
                                  int cap_tiles, int64_t* __restrict__ base, int* __restrict__ tile_group,
                                  int* __restrict__ k_start, int* __restrict__ k_len, int* __restrict__ n_recv,
                                  int* __restrict__ rows_out, int* __restrict__ overflow, int* __restrict__ err) {
  extern __shared__ int sh[];
  int* padded = sh;        // [E]
  int* start = sh + E;     // [E]
  __shared__ int s_over;
  const int El = E / ep;
  const int ge = threadIdx.x;
  if (ge == 0) s_over = 0;
  int n = 0, mine_before = 0;
  if (ge < E) {
    for (int s = 0; s < ep; ++s) {
      const int c = allc[s * E + ge];
      n += c;
      if (s < me) mine_before += c;
    }
    padded[ge] = (n + pad - 1) / pad * pad;
  }
  __syncthreads();
  if (ge < E) {
    const int d = ge / El, el = ge - d * El;
    int st = 0;
    for (int j = d * El; j < d * El + el; ++j) st += padded[j];
    start[ge] = st;
    base[ge] = (int64_t)st + mine_before;
    if (el == El - 1 && (int64_t)st + padded[ge] > cap_rows) atomicOr(&s_over, 1);
  }
  for (int t = threadIdx.x; t < cap_tiles; t += blockDim.x) tile_group[t] = -1;
  __syncthreads();
  if (ge < E && ge / El == me) {
    const int el = ge - me * El;
    // an over-capacity layout is empty: no tile, no segment, no row, so no
    // kernel reads a row that nothing wrote
    k_start[el] = s_over ? 0 : start[ge];
    k_len[el] = s_over ? 0 : padded[ge];
    n_recv[el] = s_over ? 0 : n;
    if (!s_over) {
      const int t0 = start[ge] / pad, t1 = (start[ge] + padded[ge]) / pad;
      for (int t = t0; t < t1 && t < cap_tiles; ++t) tile_group[t] = el;
    }
  }
  if (threadIdx.x == 0) {
    int rows = 0;
    for (int el = 0; el < El; ++el) rows += padded[me * El + el];
    rows_out[0] = s_over ? 0 : rows;
    overflow[0] = s_over;
    if (s_over && err) atomicOr(err, kErrEpOverflow);
  }
}

// One CTA per global expert: stable rank of its copies in (token, slot) order.
__global__ void __launch_bounds__(1024) moe_copy_rows_kernel(const int64_t* __restrict__ topi, int n_copies, int El,
                                                             const int64_t* __restrict__ base,
                                                             int64_t* __restrict__ dst_row,
                                                             int* __restrict__ dst_rank) {
  __shared__ int warp_tot[32];
  __shared__ int s_run;
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (threadIdx.x == 0) s_run = 0;
  __syncthreads();
  const int64_t b = base[e];
  for (int c0 = 0; c0 < n_copies; c0 += blockDim.x) {
    const int i = c0 + threadIdx.x;
    const bool hit = i < n_copies && topi[i] == e;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) warp_tot[wid] = __popc(m);
    __syncthreads();
    int before = s_run;
    for (int w2 = 0; w2 < wid; ++w2) before += warp_tot[w2];
    if (hit) {
      dst_row[i] = b + before + __popc(m & ((1u << lane) - 1u));
      dst_rank[i] = e / El;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int add = 0;
      for (int w2 = 0; w2 < nw; ++w2) add += warp_tot[w2];
      s_run += add;
    }
    __syncthreads();
  }
}

// One CTA per local expert: rows [k_start + n, k_start + k_len) <- 0.
__global__ void moe_zero_pad_kernel(__nv_bfloat16* __restrict__ x, int64_t ldx, int H, const int* __restrict__ k_start,
                                    const int* __restrict__ k_len, const int* __restrict__ n_recv,
                                    const int* __restrict__ overflow) {
  if (overflow && overflow[0]) return;
  const int el = blockIdx.x;
  const int64_t r0 = (int64_t)k_start[el] + n_recv[el], r1 = (int64_t)k_start[el] + k_len[el];
  const int h8 = H / 8;
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int64_t i = threadIdx.x; i < (r1 - r0) * h8; i += blockDim.x) {
    const int64_t r = r0 + i / h8;
    reinterpret_cast<uint4*>(x + r * ldx)[i % h8] = z;
  }
}

__global__ void moe_put_counts_kernel(PeerPtrs dst, int world, int me, int E, const int* __restrict__ cnt) {
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    const int c = cnt[i];
    for (int r = 0; r < world; ++r) static_cast<int*>(dst.p[r])[me * E + i] = c;
  }
}

}  // namespace

void moe_route(const float* logits, int T, int E, int k, bool norm_topk, bool bf16_logits, float* probs,
               int64_t* topi, float* topv, float* w, float* ssum, int* counts, cudaStream_t st) {
  if (T <= 0) return;
  if (E > kRouteMaxE || k > 32 || k > E) throw std::runtime_error("moe_route: at most 256 experts and k <= 32");
  moe_route_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, T, E, k, norm_topk ? 1 : 0, bf16_logits ? 1 : 0, probs,
                                                topi, topv, w, ssum, counts);
  note_launch();
}

void moe_layout(const int* allc, int ep, int me, int E, int pad, int64_t cap_rows, int cap_tiles, int64_t* base,
                int* tile_group, int* k_start, int* k_len, int* n_recv, int* rows, int* overflow, int* err,
                cudaStream_t st) {
  if (E <= 0 || E > 1024 || ep <= 0 || E % ep) throw std::runtime_error("moe_layout: bad expert / rank counts");
  const int threads = (E + 31) / 32 * 32;
  moe_layout_kernel<<<1, threads, 2 * E * sizeof(int), st>>>(allc, ep, me, E, pad, cap_rows, cap_tiles, base,
                                                             tile_group, k_start, k_len, n_recv, rows, overflow, err);
  note_launch();
}

void moe_copy_rows(const int64_t* topi, int n_copies, int E, int El, const int64_t* base, int64_t* dst_row,
                   int* dst_rank, cudaStream_t st) {
  if (n_copies <= 0) return;
  moe_copy_rows_kernel<<<E, 1024, 0, st>>>(topi, n_copies, El, base, dst_row, dst_rank);
  note_launch();
}

void moe_zero_pad(void* x, int64_t ldx, int H, int El, const int* k_start, const int* k_len, const int* n_recv,
                  const int* overflow, cudaStream_t st) {
  if (El <= 0) return;
  if (H % 8 || ldx % 8) throw std::runtime_error("moe_zero_pad: H and the row stride must be multiples of 8");
  moe_zero_pad_kernel<<<El, 256, 0, st>>>(static_cast<__nv_bfloat16*>(x), ldx, H, k_start, k_len, n_recv, overflow);
  note_launch();
}

void moe_put_counts(const PeerPtrs& dst, int world, int me, int E, const int* cnt, cudaStream_t st) {
  moe_put_counts_kernel<<<1, 256, 0, st>>>(dst, world, me, E, cnt);
  note_launch();
}

}  // namespace wb
