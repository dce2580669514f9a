// Trainer -> generator policy push over peer memory (split placement: the
// trainer and the rollout generator are separate processes on one NVLink
// node).  The reference moves a policy with a layer-by-layer NCCL broadcast
// from trainer rank 0 into paused vLLM workers (transport/policy.py:355-560);
// here every trainer rank stores the part of the weights it holds straight
// into a receive slot on each generator GPU, resharding (tensor-parallel row /
// column blocks, expert-parallel expert blocks) and casting on the way, and a
// release store of the slot's epoch publishes the result.
//
//   policy_push    a segment table of 2-D blocks (rows x row_len elements,
//                  with source / destination row strides) copied from this
//                  GPU's buffer to the same offsets in up to kMaxPeers
//                  destination buffers (plain 16-byte stores over NVLink; no
//                  TMA, so nothing here reads another GPU's memory).  Every
//                  thread ends with a system-scope fence, so the stores are
//                  visible to the destination before a later publish.
//   policy_signal  one release store (system scope) of a 32-bit value into
//                  a word of every destination pad: the slot epoch, or 0 to
//                  invalidate a slot before it is rewritten.
#include <cuda_bf16.h>
#include <stdint.h>

#include <stdexcept>

#include "comm.h"
#include "common.cuh"
#include "policy.h"

namespace wb {
namespace {

// Segment row i of the table: {src_off, dst_off, rows, row_len, src_stride,
// dst_stride} in elements; prefix[i] = vectors before segment i.
__device__ __forceinline__ int find_segment(const int64_t* __restrict__ prefix, int nseg, int64_t v) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(prefix + mid) <= v) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Store to destination k < nd of dst; the loop over kMaxPeers is unrolled so
// the pointer array stays in registers / the parameter bank (no local memory).
#define WB_EACH_DST(stmt)                       \
  _Pragma("unroll") for (int k = 0; k < kMaxPeers; ++k) { \
    if (k < nd) { stmt; }                        \
  }

template <typename TS, typename TD, int V>
struct Vec;

// 8 bf16 -> 8 bf16 (one 16-byte load, one 16-byte store per destination)
template <>
struct Vec<__nv_bfloat16, __nv_bfloat16, 8> {
  static __device__ __forceinline__ void copy(const __nv_bfloat16* s, const PeerPtrs& d, int nd, int64_t so,
                                              int64_t dof) {
    const uint4 w = *reinterpret_cast<const uint4*>(s + so);
    WB_EACH_DST(*reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(d.p[k]) + dof) = w)
  }
};
// 4 fp32 -> 4 fp32
template <>
struct Vec<float, float, 4> {
  static __device__ __forceinline__ void copy(const float* s, const PeerPtrs& d, int nd, int64_t so, int64_t dof) {
    const uint4 w = *reinterpret_cast<const uint4*>(s + so);
    WB_EACH_DST(*reinterpret_cast<uint4*>(static_cast<float*>(d.p[k]) + dof) = w)
  }
};
// 8 bf16 -> 8 fp32 (exact)
template <>
struct Vec<__nv_bfloat16, float, 8> {
  static __device__ __forceinline__ void copy(const __nv_bfloat16* s, const PeerPtrs& d, int nd, int64_t so,
                                              int64_t dof) {
    const uint4 w = *reinterpret_cast<const uint4*>(s + so);
    const uint4 a = make_uint4(__float_as_uint(bf16_lo(w.x)), __float_as_uint(bf16_hi(w.x)),
                               __float_as_uint(bf16_lo(w.y)), __float_as_uint(bf16_hi(w.y)));
    const uint4 b = make_uint4(__float_as_uint(bf16_lo(w.z)), __float_as_uint(bf16_hi(w.z)),
                               __float_as_uint(bf16_lo(w.w)), __float_as_uint(bf16_hi(w.w)));
    WB_EACH_DST(reinterpret_cast<uint4*>(static_cast<float*>(d.p[k]) + dof)[0] = a;
                reinterpret_cast<uint4*>(static_cast<float*>(d.p[k]) + dof)[1] = b)
  }
};
// 8 fp32 -> 8 bf16 (round to nearest even)
template <>
struct Vec<float, __nv_bfloat16, 8> {
  static __device__ __forceinline__ void copy(const float* s, const PeerPtrs& d, int nd, int64_t so,
                                              int64_t dof) {
    const float4 a = reinterpret_cast<const float4*>(s + so)[0];
    const float4 b = reinterpret_cast<const float4*>(s + so)[1];
    const uint4 w = make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
    WB_EACH_DST(*reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(d.p[k]) + dof) = w)
  }
};

template <typename TS, typename TD>
__device__ __forceinline__ TD cast1(TS x);
template <>
__device__ __forceinline__ __nv_bfloat16 cast1(__nv_bfloat16 x) { return x; }
template <>
__device__ __forceinline__ float cast1(float x) { return x; }
template <>
__device__ __forceinline__ float cast1(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cast1(float x) { return __float2bfloat16_rn(x); }

// V > 1: every offset, stride and row length is a multiple of V (checked on
// the host); V == 1: any layout, one element per step.
template <typename TS, typename TD, int V>
__global__ void __launch_bounds__(256) policy_push_kernel(const TS* __restrict__ src, PeerPtrs dst, int nd,
                                                          const int64_t* __restrict__ seg, const int64_t* __restrict__ prefix,
                                                          int nseg, int64_t total) {
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int s = find_segment(prefix, nseg, v);
    const int64_t* g = seg + 6 * (int64_t)s;
    const int64_t j = v - __ldg(prefix + s);
    int64_t so, dof;
    if (__ldg(g + 2) == 1) {  // one contiguous run (most parameters): no division
      so = __ldg(g + 0) + j * V;
      dof = __ldg(g + 1) + j * V;
    } else {
      const int64_t row_v = __ldg(g + 3) / V;
      const int64_t r = j / row_v;
      const int64_t c = (j - r * row_v) * V;
      so = __ldg(g + 0) + r * __ldg(g + 4) + c;
      dof = __ldg(g + 1) + r * __ldg(g + 5) + c;
    }
    if constexpr (V == 1) {
      const TD x = cast1<TS, TD>(src[so]);
      WB_EACH_DST(static_cast<TD*>(dst.p[k])[dof] = x)
    } else {
      Vec<TS, TD, V>::copy(src, dst, nd, so, dof);
    }
  }
  __threadfence_system();
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void policy_signal_kernel(PeerPtrs pads, int nd, int word, uint32_t value) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    WB_EACH_DST(st_release_sys_u32(static_cast<uint32_t*>(pads.p[k]) + word, value))
  }
}

template <typename TS, typename TD, int V>
void launch_push(const void* src, const PeerPtrs& dst, int nd, const int64_t* seg, const int64_t* prefix, int nseg,
                 int64_t total, cudaStream_t st) {
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  policy_push_kernel<TS, TD, V><<<(int)blocks, 256, 0, st>>>(static_cast<const TS*>(src), dst, nd, seg, prefix, nseg,
                                                              total);
  note_launch();
}

}  // namespace

void policy_push(const void* src, int src_bf16, const PeerPtrs& dst, int nd, int dst_bf16, const int64_t* seg,
                 const int64_t* prefix, int nseg, int64_t total_vectors, int vec, cudaStream_t st) {
  if (nseg <= 0 || total_vectors <= 0) return;
  if (nd < 1 || nd > kMaxPeers) throw std::runtime_error("wavelet_b200 policy_push: 1..8 destinations");
  using bf = __nv_bfloat16;
  if (src_bf16 && dst_bf16) {
    if (vec == 8) launch_push<bf, bf, 8>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else if (vec == 1) launch_push<bf, bf, 1>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else throw std::runtime_error("wavelet_b200 policy_push: bf16 -> bf16 takes vec 8 or 1");
  } else if (!src_bf16 && !dst_bf16) {
    if (vec == 4) launch_push<float, float, 4>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else if (vec == 1) launch_push<float, float, 1>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else throw std::runtime_error("wavelet_b200 policy_push: fp32 -> fp32 takes vec 4 or 1");
  } else if (src_bf16) {
    if (vec == 8) launch_push<bf, float, 8>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else if (vec == 1) launch_push<bf, float, 1>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else throw std::runtime_error("wavelet_b200 policy_push: bf16 -> fp32 takes vec 8 or 1");
  } else {
    if (vec == 8) launch_push<float, bf, 8>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else if (vec == 1) launch_push<float, bf, 1>(src, dst, nd, seg, prefix, nseg, total_vectors, st);
    else throw std::runtime_error("wavelet_b200 policy_push: fp32 -> bf16 takes vec 8 or 1");
  }
}

void policy_signal(const PeerPtrs& pads, int nd, int word, uint32_t value, cudaStream_t st) {
  if (nd < 1 || nd > kMaxPeers) throw std::runtime_error("wavelet_b200 policy_signal: 1..8 destinations");
  policy_signal_kernel<<<1, 32, 0, st>>>(pads, nd, word, value);
  note_launch();
}

}  // namespace wb
