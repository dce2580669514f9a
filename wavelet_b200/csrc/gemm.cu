// Persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M, N] (op)= alpha * sum_k A(m, k) * B(n, k)  (+ bias[n])
//
// A and B are each either K-major (row m / n holds K contiguous elements) or
// MN-major (row k holds M / N contiguous elements), so one kernel serves the
// three GEMMs of a linear layer without any transpose:
//   forward  Y  = X  W^T : A = X  (K-major),  B = W  (K-major)
//   dgrad    dX = dY W   : A = dY (K-major),  B = W  (MN-major)
//   wgrad    dW = dY^T X : A = dY (MN-major), B = X  (MN-major)
// (the three linear GEMMs of the reference run as cuBLAS calls inside
// torch.nn.Linear, trainer/model.py; this replaces them on the GPU path).
//
// CTA layout (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: streams 128x64 A and 256x64 B tiles into a
//               4-stage shared-memory ring (128-byte swizzle, no multicast).
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256,
//               K=16) into one of two TMEM accumulators (2 x 256 columns).
//   warps 2..5  epilogue: tcgen05.ld the finished accumulator (warp w reads
//               TMEM lanes 32*(w%4)..+31 = tile rows), apply the epilogue and
//               store to global memory while the MMA warp fills the other
//               accumulator.
// Every wait is bounded (common.cuh); on timeout the CTA drains its in-flight
// TMA and MMA work, frees TMEM, reports through the error word and exits.
//
// Two extensions serve LoRA / QLoRA (reference kernels/lora.py and the
// bitsandbytes dequant + matmul it calls):
//   * a second operand pair (A2, B2, K2): after the K/64 k-blocks of A B^T
//     the producer streams K2/64 k-blocks of A2 B2^T into the same TMEM
//     accumulator, so the low-rank update costs one or two extra k-blocks of
//     the base GEMM instead of a separate GEMM plus an add;
//   * an NF4 B operand (BQ): warps 6..13 load 4-bit codes and per-64 absmax
//     scales, dequantise through a 16-entry table in shared memory and store
//     bf16 straight into the 128-byte-swizzled stage layout that TMA would
//     have produced (fence.proxy.async before arriving on the stage barrier),
//     so a frozen base weight is read at 0.5 byte per element.
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "gemm.h"
#include "tma.h"

namespace wb {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;        // 16 KB
constexpr int B_BYTES = BN * BK * 2;        // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int MN_BOX = 64;                  // MN-major TMA box width (128 bytes)
constexpr int MN_BOX_BYTES = MN_BOX * BK * 2;  // 8 KB
constexpr int NUM_THREADS = 192;
constexpr int NUM_DQ_THREADS = 256;  // NF4 dequant producers (warps 6..13)
constexpr int NUM_THREADS_Q = NUM_THREADS + NUM_DQ_THREADS;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;

struct __align__(8) Smem {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float lut[16];
};

// kEpiPeerBF16 stages each epilogue warp's [32 rows x 64 cols] bf16 slice in
// shared memory (4 KB per warp, after the barrier block) so that peer stores
// leave as whole 128-byte row segments instead of 16-byte pieces of 32 rows.
constexpr int PEER_STAGE_BYTES = 4 * 32 * 128;
constexpr size_t smem_bytes(bool peer = false) {
  return 1024 + STAGES * STAGE_BYTES + 1024 + (peer ? PEER_STAGE_BYTES : 0);
}
static_assert(sizeof(Smem) <= 1024, "barrier block must fit in front of the peer staging area");

struct Params {
  void* C;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* res;  // optional residual added in the bf16 epilogue
  int64_t ldr;
  int64_t ldc;
  float alpha;
  int M, N, K;
  int num_m, num_n, num_k;
  int* err;
  // grouped modes (GROUP template parameter)
  const int* tile_group;   // M-grouped: expert of every 128-row M tile
  int64_t b_group_stride;  // M-grouped: B outer-coordinate offset per group
  const int* k_start;      // K-grouped: first K row of every group (multiple of BK)
  const int* k_len;        // K-grouped: K rows of every group
  int groups;
  int num_k2;              // k-blocks of the second operand pair (dense mode)
  const uint8_t* q;        // NF4 B operand
  const float* q_absmax;
  int64_t q_cols;
  float lut[16];
  void* peer[8];  // kEpiPeerBF16 receive buffers (GemmArgs::peer)
  int peer_world, peer_rank;
  int64_t peer_off, peer_rs_rows;
  // split tail (dense mode): tiles >= split_first are cut into split_s K-pieces
  int split_first, split_s;
};

// Tail-wave split.  A dense GEMM whose tile count leaves a small last wave
// (e.g. 448 tiles on 148 SMs: 3 full waves + 4 tiles, so the 4th wave runs 4
// SMs while 144 idle) cuts each of the `rem` tail tiles into split_s K-ranges.
// Every piece writes its fp32 partial tile here; per (tile, 32-row quadrant)
// the last piece to finish (atomic ticket, no waiting) sums the partials in
// piece order and runs the normal epilogue.  At most 4 pieces per tile: the
// reduction is one CTA's L2 round trips, so a longer split costs more in the
// reducer than it saves in the wave.  Sized for rem * split_s <= 256
// pieces and rem <= 128 tiles (host enforces); one workspace per device, so
// tail-split GEMMs on one device run in stream order (every launch of this
// library's GEMMs shares it).  Tickets return to zero after each use.
constexpr int SPLIT_MAX_PIECES = 256;
constexpr int SPLIT_MAX_S = 4;  // pieces per tile: the reducer keeps all their loads in flight
constexpr int SPLIT_MAX_TILES = 128;
__device__ __align__(256) float g_split_ws[(size_t)SPLIT_MAX_PIECES * 128 * 256];
__device__ int g_split_ticket[SPLIT_MAX_TILES * 4];

// Tile decode shared by the three warp roles (they must agree exactly).
struct TileInfo {
  int tm, tn;
  int kb_begin, num_k;
  int64_t b_off;
  int64_t c_row_off;
  int split, piece;  // split tail: index among the split tiles and K-piece (split = -1: whole tile)
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m, int& n) {
  const int in_group = GROUP_M * num_n;
  const int gid = t / in_group;
  const int first_m = gid * GROUP_M;
  const int gsm = min(num_m - first_m, GROUP_M);
  const int r = t - gid * in_group;
  m = first_m + r % gsm;
  n = r / gsm;
}

template <int GROUP>
__device__ __forceinline__ TileInfo tile_info(int t, const Params& p) {
  TileInfo ti;
  if constexpr (GROUP == 2) {
    const int per = p.num_m * p.num_n;
    const int g = t / per;
    tile_coords(t - g * per, p.num_m, p.num_n, ti.tm, ti.tn);
    ti.kb_begin = p.k_start[g] / BK;
    ti.num_k = (p.k_len[g] + BK - 1) / BK;
    ti.b_off = 0;
    ti.c_row_off = (int64_t)g * p.M;
  } else {
    ti.split = -1;
    ti.piece = 0;
    int tile = t;
    ti.kb_begin = 0;
    ti.num_k = p.num_k;
    if (GROUP == 0 && p.split_s > 1 && t >= p.split_first) {
      const int v = t - p.split_first;
      ti.split = v / p.split_s;
      ti.piece = v - ti.split * p.split_s;
      tile = p.split_first + ti.split;
      ti.kb_begin = ti.piece * p.num_k / p.split_s;
      ti.num_k = (ti.piece + 1) * p.num_k / p.split_s - ti.kb_begin;
    }
    tile_coords(tile, p.num_m, p.num_n, ti.tm, ti.tn);
    ti.b_off = 0;
    if constexpr (GROUP == 1) {
      // a tile past the used rows of a device-built layout has group -1: no
      // k-blocks, so the producer, MMA and epilogue all skip it
      const int g = p.tile_group[ti.tm];
      if (g < 0)
        ti.num_k = 0;
      else
        ti.b_off = (int64_t)g * p.b_group_stride;
    }
    ti.c_row_off = 0;
  }
  if constexpr (GROUP == 2) ti.split = -1, ti.piece = 0;
  return ti;
}

template <int GROUP, bool BQ, int EPI>
constexpr bool kSplitCapable = (GROUP == 0 && !BQ && EPI != kEpiPeerBF16);

// Units of work: tiles, with every split tail tile counted once per K-piece.
__device__ __forceinline__ int num_units(const Params& p, int groups_mul) {
  const int tiles = p.num_m * p.num_n * groups_mul;
  return (p.split_s > 1) ? p.split_first + (tiles - p.split_first) * p.split_s : tiles;
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const Params& p, int row, int col0,
                                               const uint32_t (&v)[32], int64_t row_off) {
  if (row >= p.M) return;
  row += static_cast<int>(row_off);
  const bool full = (col0 + 32 <= p.N);
  if constexpr (EPI == kEpiBF16) {
    __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + (int64_t)row * p.ldc + col0;
    float f[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]) * p.alpha;
    if (p.bias) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) f[j] += __bfloat162float(p.bias[col0 + j]);
    }
    if (p.res) {
      const __nv_bfloat16* r = p.res + (int64_t)row * p.ldr + col0;
      if (full && ((p.ldr & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.res) & 15) == 0)) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 w = reinterpret_cast<const uint4*>(r)[q];
          f[8 * q + 0] += bf16_lo(w.x);
          f[8 * q + 1] += bf16_hi(w.x);
          f[8 * q + 2] += bf16_lo(w.y);
          f[8 * q + 3] += bf16_hi(w.y);
          f[8 * q + 4] += bf16_lo(w.z);
          f[8 * q + 5] += bf16_hi(w.z);
          f[8 * q + 6] += bf16_lo(w.w);
          f[8 * q + 7] += bf16_hi(w.w);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N) f[j] += __bfloat162float(r[j]);
      }
    }
    if (full && ((p.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0)) {
      uint4* dst = reinterpret_cast<uint4*>(c);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16(f[8 * q + 0], f[8 * q + 1]);
        w.y = pack_bf16(f[8 * q + 2], f[8 * q + 3]);
        w.z = pack_bf16(f[8 * q + 4], f[8 * q + 5]);
        w.w = pack_bf16(f[8 * q + 6], f[8 * q + 7]);
        dst[q] = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) c[j] = __float2bfloat16(f[j]);
    }
  } else if constexpr (EPI == kEpiPeerBF16) {
    // partial product -> peer receive buffers over NVLink (plain 16-byte stores)
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      w[j] = pack_bf16(__uint_as_float(v[2 * j]) * p.alpha, __uint_as_float(v[2 * j + 1]) * p.alpha);
    int64_t drow = row;
    int first = p.peer_rank + 1, count = p.peer_world;
    if (p.peer_rs_rows > 0) {
      first = static_cast<int>(row / p.peer_rs_rows);
      drow = row - (int64_t)first * p.peer_rs_rows;
      count = 1;
    }
    const bool vec = full && ((p.ldc & 7) == 0) && ((p.peer_off & 7) == 0);
    for (int i = 0; i < count; ++i) {
      int r = first + i;
      if (r >= p.peer_world) r -= p.peer_world;
      __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.peer[r]) + p.peer_off + drow * p.ldc + col0;
      if (vec) {
        uint4* dst = reinterpret_cast<uint4*>(c);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N) c[j] = __float2bfloat16(__uint_as_float(v[j]) * p.alpha);
      }
    }
  } else {
    float* c = reinterpret_cast<float*>(p.C) + (int64_t)row * p.ldc + col0;
    if (full && ((p.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0)) {
      float4* dst = reinterpret_cast<float4*>(c);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = make_float4(__uint_as_float(v[4 * q + 0]) * p.alpha,
                               __uint_as_float(v[4 * q + 1]) * p.alpha,
                               __uint_as_float(v[4 * q + 2]) * p.alpha,
                               __uint_as_float(v[4 * q + 3]) * p.alpha);
        if constexpr (EPI == kEpiF32Acc) {
          float4 o = dst[q];
          w.x += o.x;
          w.y += o.y;
          w.z += o.z;
          w.w += o.w;
        }
        dst[q] = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < p.N) {
          float w = __uint_as_float(v[j]) * p.alpha;
          if constexpr (EPI == kEpiF32Acc) w += c[j];
          c[j] = w;
        }
      }
    }
  }
}

// kEpiPeerBF16, 64 columns of this warp's 32 rows: pack to bf16, stage in
// shared memory (16-byte chunks XOR-swizzled by row), read back so that 8
// lanes hold one row's 128 contiguous bytes, and store every destination's
// copy as full 128-byte segments.  Partial column blocks use the per-thread
// path of epilogue_chunk.
__device__ __forceinline__ void peer_store64(const Params& p, int col0, const uint32_t (&v0)[32],
                                             const uint32_t (&v1)[32], uint8_t* stg, int lane, int row_base) {
  const bool full = (col0 + 64 <= p.N) && ((p.ldc & 7) == 0) && ((p.peer_off & 7) == 0);
  if (!full) {
    epilogue_chunk<kEpiPeerBF16>(p, row_base + lane, col0, v0, 0);
    if (col0 + 32 < p.N) epilogue_chunk<kEpiPeerBF16>(p, row_base + lane, col0 + 32, v1, 0);
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t* v = (j < 4) ? v0 : v1;
    const int b = (j & 3) * 8;
    uint4 w;
    w.x = pack_bf16(__uint_as_float(v[b + 0]) * p.alpha, __uint_as_float(v[b + 1]) * p.alpha);
    w.y = pack_bf16(__uint_as_float(v[b + 2]) * p.alpha, __uint_as_float(v[b + 3]) * p.alpha);
    w.z = pack_bf16(__uint_as_float(v[b + 4]) * p.alpha, __uint_as_float(v[b + 5]) * p.alpha);
    w.w = pack_bf16(__uint_as_float(v[b + 6]) * p.alpha, __uint_as_float(v[b + 7]) * p.alpha);
    *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) << 4)) = w;
  }
  __syncwarp();
  const int ch = lane & 7;
  uint4 o[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = 4 * it + (lane >> 3);
    o[it] = *reinterpret_cast<const uint4*>(stg + r * 128 + ((ch ^ (r & 7)) << 4));
  }
  __syncwarp();  // the staging slice is rewritten by the next 64 columns
  const int nd = p.peer_rs_rows > 0 ? 1 : p.peer_world;
  for (int i = 0; i < nd; ++i) {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int row = row_base + 4 * it + (lane >> 3);
      if (row >= p.M) continue;
      int r;
      int64_t drow = row;
      if (p.peer_rs_rows > 0) {
        r = static_cast<int>(row / p.peer_rs_rows);
        drow = row - (int64_t)r * p.peer_rs_rows;
      } else {
        r = p.peer_rank + 1 + i;
        if (r >= p.peer_world) r -= p.peer_world;
      }
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.peer[r]) + p.peer_off + drow * p.ldc + col0 + ch * 8;
      *reinterpret_cast<uint4*>(dst) = o[it];
    }
  }
}

// 32 bytes of codes (64 elements) -> 8 chunks of 8 bf16 at swizzled offsets.
__device__ __forceinline__ void dequant_segment(uint8_t* row_base, int swz, uint4 w0, uint4 w1, float am,
                                                const float* lut) {
  const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint32_t b = words[c];  // 4 bytes = 8 codes, little-endian byte order
    uint4 o;
    uint32_t* op = &o.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t byte = (b >> (8 * j)) & 0xffu;
      op[j] = pack_bf16(lut[byte >> 4] * am, lut[byte & 15u] * am);
    }
    *reinterpret_cast<uint4*>(row_base + ((c ^ swz) << 4)) = o;
  }
}

struct NF4Seg {
  uint4 w0, w1;
  float am;
};

// Codes + absmax of dequant thread d's segment for flat iteration `it` of
// this CTA (dense mode: every tile has nk = num_k + num_k2 iterations; the
// second-operand iterations and out-of-range rows load nothing).
template <bool B_MN>
__device__ __forceinline__ void nf4_fetch(const Params& p, int it, int nk, int num_tiles, int d, NF4Seg& sg) {
  sg.w0 = make_uint4(0, 0, 0, 0);
  sg.w1 = sg.w0;
  sg.am = 0.f;
  const int j = it / nk, kb = it - j * nk;
  const int t = blockIdx.x + j * gridDim.x;
  if (t >= num_tiles || kb >= p.num_k) return;
  int tm, tn;
  tile_coords(t, p.num_m, p.num_n, tm, tn);
  const int n0 = tn * BN, k0 = kb * BK;
  const int64_t qb = p.q_cols / 2, qa = p.q_cols / 64;
  if constexpr (!B_MN) {
    const int n = n0 + d;  // B(n, k) = W[n][k]
    if (n >= p.N) return;
    const uint4* src = reinterpret_cast<const uint4*>(p.q + (int64_t)n * qb + k0 / 2);
    sg.w0 = __ldg(src);
    sg.w1 = __ldg(src + 1);
    sg.am = __ldg(p.q_absmax + (int64_t)n * qa + kb);
  } else {
    const int kr = k0 + (d & 63), nb = n0 + (d >> 6) * 64;  // B(n, k) = W[k][n]
    if (kr >= p.K || nb >= p.N) return;
    const uint4* src = reinterpret_cast<const uint4*>(p.q + (int64_t)kr * qb + nb / 2);
    sg.w0 = __ldg(src);
    sg.w1 = __ldg(src + 1);
    sg.am = __ldg(p.q_absmax + (int64_t)kr * qa + nb / 64);
  }
}

template <bool A_MN, bool B_MN, int EPI, int GROUP, bool BQ>
__global__ void __launch_bounds__(BQ ? NUM_THREADS_Q : NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  Smem* s = reinterpret_cast<Smem*>(tiles + STAGES * STAGE_BYTES);
  volatile int* abort = &s->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = (GROUP == 0) ? num_units(p, 1) : p.num_m * p.num_n * (GROUP == 2 ? p.groups : 1);
  const int num_k2 = (GROUP == 0) ? p.num_k2 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s->full[i], BQ ? 1 + NUM_DQ_THREADS : 1);
      mbar_init(&s->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->tmem_full[i], 1);
      mbar_init(&s->tmem_empty[i], 128);
    }
    mbar_init(&s->drain, 1);
    s->abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    if (BQ)
      for (int i = 0; i < 16; ++i) s->lut[i] = p.lut[i];
  }
  if (warp == 1) {
    tmem_alloc(&s->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued[STAGES];
      uint32_t issued_phase[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = 0, issued_phase[i] = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<GROUP>(t, p);
        const int m0 = ti.tm * BM, n0 = ti.tn * BN;
        const int nk = ti.num_k + (ti.num_k > 0 ? num_k2 : 0);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&s->empty[stage], phase ^ 1, abort, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = tiles + stage * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_BYTES;
          const bool second = kb >= ti.num_k;
          const bool load_b = second || !BQ;
          mbar_arrive_expect_tx(&s->full[stage], load_b ? STAGE_BYTES : A_BYTES);
          const int k0 = second ? (kb - ti.num_k) * BK : (ti.kb_begin + kb) * BK;
          const int boff = second ? 0 : (int)ti.b_off;
          const CUtensorMap* mA = second ? &tmA2 : &tmA;
          const CUtensorMap* mB = second ? &tmB2 : &tmB;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / MN_BOX; ++j)
              tma_load_2d(mA, &s->full[stage], a_dst + j * MN_BOX_BYTES, m0 + j * MN_BOX, k0);
          } else {
            tma_load_2d(mA, &s->full[stage], a_dst, k0, m0);
          }
          if (load_b) {
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / MN_BOX; ++j)
                tma_load_2d(mB, &s->full[stage], b_dst + j * MN_BOX_BYTES, n0 + j * MN_BOX, k0 + boff);
            } else {
              tma_load_2d(mB, &s->full[stage], b_dst, k0, n0 + boff);
            }
          }
          issued[stage] = 1;
          issued_phase[stage] = phase;
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
      if (!ok || *abort) {
        // Drain: every TMA we issued must land before the CTA may exit.
        for (int i = 0; i < STAGES; ++i) {
          if (!issued[i]) continue;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s->full[i], issued_phase[i])) {
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
              atomicOr(p.err, kErrTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool any = false;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<GROUP>(t, p);
        if (ti.num_k == 0) continue;  // empty group: no MMA, no epilogue
        if (!mbar_wait(&s->tmem_empty[acc], acc_phase ^ 1, abort, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int nk = ti.num_k + num_k2;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&s->full[stage], phase, abort, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad, bd;
            if constexpr (A_MN)
              ad = smem_desc_sw128(a_addr + k * 16 * 128, MN_BOX_BYTES, 1024);
            else
              ad = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            if constexpr (B_MN)
              bd = smem_desc_sw128(b_addr + k * 16 * 128, MN_BOX_BYTES, 1024);
            else
              bd = smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&s->empty[stage]);
          any = true;
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        umma_commit(&s->tmem_full[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1;
      }
      if (any) {
        // All MMAs must retire before TMEM is released.
        umma_commit(&s->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s->drain, 0)) {
          if (globaltimer_ns() - t0 > kWaitBudgetNs) {
            atomicOr(p.err, kErrTimeoutDrain);
            break;
          }
        }
      }
    }
  } else if (BQ && warp >= NUM_THREADS / 32) {
    // ------------------------------------------------------------ NF4 dequant producers
    // Flat iteration space it -> (tile j of this CTA, k-block kb); the codes of
    // iteration it+4 are loaded into registers while iteration it is
    // converted, so four stages of global-load latency are in flight.
    const int d = threadIdx.x - NUM_THREADS;  // 0..255: one 64-element segment per stage
    const int nk = p.num_k + num_k2;
    const int my_tiles = blockIdx.x < num_tiles ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int total = my_tiles * nk;
    uint8_t* row_off;
    int swz;
    if constexpr (!B_MN) {
      row_off = tiles + A_BYTES + d * 128;
      swz = d & 7;
    } else {
      row_off = tiles + A_BYTES + (d >> 6) * MN_BOX_BYTES + (d & 63) * 128;
      swz = d & 7;
    }
    NF4Seg s0, s1, s2, s3;
    nf4_fetch<B_MN>(p, 0, nk, num_tiles, d, s0);
    nf4_fetch<B_MN>(p, 1, nk, num_tiles, d, s1);
    nf4_fetch<B_MN>(p, 2, nk, num_tiles, d, s2);
    nf4_fetch<B_MN>(p, 3, nk, num_tiles, d, s3);
    int stage = 0;
    uint32_t phase = 0;
    for (int it = 0; it < total; ++it) {
      if (!mbar_wait_warp(&s->empty[stage], phase ^ 1, abort, p.err, kErrTimeoutProducer)) break;
      if (it % nk < p.num_k) {
        dequant_segment(row_off + stage * STAGE_BYTES, swz, s0.w0, s0.w1, s0.am, s->lut);
        fence_proxy_async_shared();
      }
      mbar_arrive(&s->full[stage]);
      if (++stage == STAGES) stage = 0, phase ^= 1;
      s0 = s1;
      s1 = s2;
      s2 = s3;
      nf4_fetch<B_MN>(p, it + 4, nk, num_tiles, d, s3);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const TileInfo ti = tile_info<GROUP>(t, p);
      if (ti.num_k == 0) continue;
      if (!mbar_wait_warp(&s->tmem_full[acc], acc_phase, abort, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const int tm = ti.tm, tn = ti.tn;
      const int row = tm * BM + q * 32 + lane;
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (kSplitCapable<GROUP, BQ, EPI> && ti.split >= 0) {
        // tail piece: fp32 partial out, TMEM back to the MMA warp, then the
        // last piece of this (tile, quadrant) reduces and runs the epilogue
        float* part = g_split_ws + ((size_t)(ti.split * p.split_s + ti.piece) * BM + q * 32 + lane) * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          if (tn * BN + c >= p.N) break;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_addr + c, v);
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(part + c);
#pragma unroll
          for (int u = 0; u < 8; ++u)
            dst[u] = make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                                 __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
        }
        tc_fence_before();
        mbar_arrive(&s->tmem_empty[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1;
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&g_split_ticket[ti.split * 4 + q], 1) == p.split_s - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          const float* base = g_split_ws + ((size_t)ti.split * p.split_s * BM + q * 32 + lane) * BN;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            if (tn * BN + c >= p.N) break;
            // all pieces' loads in flight before the adds (split_s <= SPLIT_MAX_S)
            float4 w[SPLIT_MAX_S][8];
#pragma unroll
            for (int pc = 0; pc < SPLIT_MAX_S; ++pc) {
              if (pc < p.split_s) {
                const float4* src = reinterpret_cast<const float4*>(base + (size_t)pc * BM * BN + c);
#pragma unroll
                for (int u = 0; u < 8; ++u) w[pc][u] = __ldcg(src + u);
              }
            }
            float a[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = 0.f;
#pragma unroll
            for (int pc = 0; pc < SPLIT_MAX_S; ++pc) {
              if (pc < p.split_s) {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  a[4 * u] += w[pc][u].x;
                  a[4 * u + 1] += w[pc][u].y;
                  a[4 * u + 2] += w[pc][u].z;
                  a[4 * u + 3] += w[pc][u].w;
                }
              }
            }
            uint32_t v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(a[j]);
            epilogue_chunk<EPI>(p, row, tn * BN + c, v, 0);
          }
          if (lane == 0) g_split_ticket[ti.split * 4 + q] = 0;
        }
        continue;
      }
      if constexpr (EPI == kEpiPeerBF16) {
        uint8_t* stg = tiles + STAGES * STAGE_BYTES + 1024 + q * 4096;
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          if (tn * BN + c >= p.N) break;
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(t_addr + c, v0);
          tmem_ld_32x32b_x32(t_addr + c + 32, v1);
          tmem_wait_ld();
          peer_store64(p, tn * BN + c, v0, v1, stg, lane, tm * BM + q * 32);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          if (tn * BN + c >= p.N) break;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_addr + c, v);
          tmem_wait_ld();
          epilogue_chunk<EPI>(p, row, tn * BN + c, v, ti.c_row_off);
        }
      }
      tc_fence_before();
      mbar_arrive(&s->tmem_empty[acc]);
      if (++acc == 2) acc = 0, acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool A_MN, bool B_MN, int EPI, int GROUP = 0, bool BQ = false>
static void launch(const GemmArgs& g, cudaStream_t stream) {
  auto kern = gemm_kernel<A_MN, B_MN, EPI, GROUP, BQ>;
  static std::atomic<bool> attr_set[64];  // per device; cudaFuncSetAttribute is idempotent
  int dev = 0;
  cudaGetDevice(&dev);
  constexpr size_t smem = smem_bytes(EPI == kEpiPeerBF16);
  if (!attr_set[dev & 63].load(std::memory_order_acquire)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_set[dev & 63].store(true, std::memory_order_release);
  }
  // A(m,k): K-major -> rows of K; MN-major -> rows of M.
  CUtensorMap ta = A_MN ? make_tmap_2d(g.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.M, g.K, g.lda,
                                       MN_BOX, BK, CU_TENSOR_MAP_SWIZZLE_128B)
                        : make_tmap_2d(g.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.K, g.M, g.lda,
                                       BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  // B outer extent: N (K-major) or K (MN-major) rows, times the group count
  // in M-grouped mode where every group has its own weight block.
  const uint64_t b_outer = g.b_outer > 0 ? (uint64_t)g.b_outer : (uint64_t)(B_MN ? g.K : g.N);
  CUtensorMap tb;
  if (BQ)
    tb = ta;  // unused: B comes from the NF4 dequant warps
  else
    tb = B_MN ? make_tmap_2d(g.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.N, b_outer, g.ldb, MN_BOX, BK,
                             CU_TENSOR_MAP_SWIZZLE_128B)
              : make_tmap_2d(g.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.K, b_outer, g.ldb, BK, BN,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap ta2 = ta, tb2 = tb;
  if (g.K2 > 0) {
    ta2 = A_MN ? make_tmap_2d(g.A2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.M, g.K2, g.lda2, MN_BOX, BK,
                              CU_TENSOR_MAP_SWIZZLE_128B)
               : make_tmap_2d(g.A2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.K2, g.M, g.lda2, BK, BM,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    tb2 = B_MN ? make_tmap_2d(g.B2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.N, g.K2, g.ldb2, MN_BOX, BK,
                              CU_TENSOR_MAP_SWIZZLE_128B)
               : make_tmap_2d(g.B2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.K2, g.N, g.ldb2, BK, BN,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  }
  Params p;
  p.C = g.C;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(g.bias);
  p.res = reinterpret_cast<const __nv_bfloat16*>(g.res);
  p.ldr = g.ldr;
  p.ldc = g.ldc;
  p.alpha = g.alpha;
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.num_m = (g.M + BM - 1) / BM;
  p.num_n = (g.N + BN - 1) / BN;
  p.num_k = (g.K + BK - 1) / BK;
  p.err = error_word(dev);
  p.tile_group = g.tile_group;
  p.b_group_stride = g.b_group_stride;
  p.k_start = g.k_start;
  p.k_len = g.k_len;
  p.groups = g.groups;
  p.num_k2 = g.K2 > 0 ? (g.K2 + BK - 1) / BK : 0;
  p.q = g.q;
  p.q_absmax = g.q_absmax;
  p.q_cols = g.q_cols;
  for (int i = 0; i < 16; ++i) p.lut[i] = g.q_lut[i];
  for (int i = 0; i < 8; ++i) p.peer[i] = g.peer[i];
  p.peer_world = g.peer_world;
  p.peer_rank = g.peer_rank;
  p.peer_off = g.peer_off;
  p.peer_rs_rows = g.peer_rs_rows;
  p.split_first = 0;
  p.split_s = 1;
  const int tiles = p.num_m * p.num_n * (GROUP == 2 ? g.groups : 1);
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  static const bool split_off = std::getenv("WAVELET_GEMM_NO_SPLIT") != nullptr;  // A/B switch
  if (GROUP == 0 && !BQ && EPI != kEpiPeerBF16 && p.num_k2 == 0 && !g.no_split && !split_off && tiles > grid) {
    const int rem = tiles % grid;
    int S = rem > 0 ? grid / rem : 1;
    S = S < SPLIT_MAX_S ? S : SPLIT_MAX_S;
    // at least 64 k-blocks per piece: measured on B200, shorter pieces lose
    // more in the partial-tile round trip than the shorter wave saves
    // (K = 3584: 1126 -> 980 TFLOP/s split; K = 18944: 1199 -> 1308)
    S = S < p.num_k / 64 ? S : p.num_k / 64;
    if (S >= 2 && rem <= SPLIT_MAX_TILES && rem * S <= SPLIT_MAX_PIECES) {
      p.split_first = tiles - rem;
      p.split_s = S;
    }
  }
  kern<<<grid, BQ ? NUM_THREADS_Q : NUM_THREADS, smem, stream>>>(ta, tb, ta2, tb2, p); note_launch();
}

}  // namespace gemm

void gemm_bf16(const GemmArgs& g, cudaStream_t stream) {
  using namespace gemm;
  if (g.M <= 0 || g.N <= 0) return;
  if (g.group_mode == 1) {
    // expert forward / dgrad: rows of A are expert segments padded to 128
    if (!g.tile_group) throw std::runtime_error("wavelet_b200 grouped gemm: tile_group required");
    if (g.epi != kEpiBF16 || g.a_mn) throw std::runtime_error("wavelet_b200 grouped gemm: M-grouped mode is K-major A, bf16 out");
    if (g.b_mn) return launch<false, true, kEpiBF16, 1>(g, stream);
    return launch<false, false, kEpiBF16, 1>(g, stream);
  }
  if (g.group_mode == 2) {
    // K-grouped: C[g] = A_g^T B_g over K ranges [k_start[g], +k_len[g]); C = [groups * M, N] fp32.
    // MN-major A and B: expert wgrad over token segments.  K-major A (B either way):
    // split-K partials of a skinny forward / dgrad GEMM (reduced by splitk_reduce).
    if (!g.k_start || !g.k_len || g.groups <= 0) throw std::runtime_error("wavelet_b200 grouped gemm: k_start/k_len required");
    if (g.a_mn && g.b_mn) {
      if (g.epi == kEpiF32Acc) return launch<true, true, kEpiF32Acc, 2>(g, stream);
      if (g.epi == kEpiF32) return launch<true, true, kEpiF32, 2>(g, stream);
    } else if (!g.a_mn && g.epi == kEpiF32) {
      if (g.b_mn) return launch<false, true, kEpiF32, 2>(g, stream);
      return launch<false, false, kEpiF32, 2>(g, stream);
    }
    throw std::runtime_error("wavelet_b200 grouped gemm: unsupported K-grouped layout / epilogue");
  }
  if (g.K <= 0) throw std::runtime_error("wavelet_b200 gemm: K must be positive");
  if (g.K2 > 0 && (!g.A2 || !g.B2)) throw std::runtime_error("wavelet_b200 gemm: K2 > 0 needs A2 and B2");
  if (g.K2 % 64) throw std::runtime_error("wavelet_b200 gemm: K2 must be a multiple of 64 (pad the adapter rank)");
  if (g.q) {
    // NF4 base weight: forward (B K-major) or dgrad (B MN-major), bf16 out
    if (g.a_mn || g.epi != kEpiBF16) throw std::runtime_error("wavelet_b200 nf4 gemm: K-major A and bf16 output only");
    if (g.q_cols % 64) throw std::runtime_error("wavelet_b200 nf4 gemm: weight columns must be a multiple of 64");
    if (g.b_mn ? (g.K != g.q_rows || g.N != g.q_cols) : (g.N != g.q_rows || g.K != g.q_cols))
      throw std::runtime_error("wavelet_b200 nf4 gemm: weight shape does not match M/N/K");
    if (g.b_mn) return launch<false, true, kEpiBF16, 0, true>(g, stream);
    return launch<false, false, kEpiBF16, 0, true>(g, stream);
  }
  if (g.epi == kEpiPeerBF16) {
    // fused GEMM -> all-reduce / reduce-scatter: forward (B K-major) or dgrad (B MN-major)
    if (g.a_mn || g.peer_world < 1 || g.peer_world > 8 || g.peer_rank < 0 || g.peer_rank >= g.peer_world)
      throw std::runtime_error("wavelet_b200 peer gemm: K-major A and 1..8 ranks");
    for (int r = 0; r < g.peer_world; ++r)
      if (!g.peer[r]) throw std::runtime_error("wavelet_b200 peer gemm: missing peer buffer");
    if (g.peer_rs_rows > 0 && (int64_t)g.peer_world * g.peer_rs_rows < g.M)
      throw std::runtime_error("wavelet_b200 peer gemm: reduce-scatter rows do not cover M");
    if (g.b_mn) return launch<false, true, kEpiPeerBF16>(g, stream);
    return launch<false, false, kEpiPeerBF16>(g, stream);
  }
#define WB_GEMM_DISPATCH(AM, BMJ)                                               \
  if (g.a_mn == AM && g.b_mn == BMJ) {                                          \
    if (g.epi == kEpiBF16) return launch<AM, BMJ, kEpiBF16>(g, stream);         \
    if (g.epi == kEpiF32) return launch<AM, BMJ, kEpiF32>(g, stream);           \
    if (g.epi == kEpiF32Acc) return launch<AM, BMJ, kEpiF32Acc>(g, stream);     \
  }
  WB_GEMM_DISPATCH(false, false)
  WB_GEMM_DISPATCH(false, true)
  WB_GEMM_DISPATCH(true, false)
  WB_GEMM_DISPATCH(true, true)
#undef WB_GEMM_DISPATCH
  throw std::runtime_error("wavelet_b200 gemm: unsupported epilogue");
}

}  // namespace wb
