// Packed variable-length causal attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Layout: q [T, Hq, 128], k/v [T, Hk, 128] bf16 (any row stride, e.g. views
// into the packed qkv activation), sequences delimited by cu_seqlens; GQA with
// Hq % Hk == 0.  Output o [T, Hq, 128] bf16 and lse [Hq, T] fp32 (natural log).
//
// Forward, one CTA per (128-query tile, q head, sequence), 192 threads:
//   warp 0      TMA: Q tile once, then K_j / V_j tiles into a 2-stage ring.
//   warp 1      MMA: S_j = Q K_j^T into one of two TMEM S buffers (so S_{j+1}
//               overlaps the softmax of S_j), then O += P_j V_j.
//   warps 2..5  softmax: thread = query row = TMEM lane.  Reads S_j with
//               tcgen05.ld, applies the causal / sequence mask, keeps the
//               running max m and sum l in the log2 domain, writes P_j (bf16)
//               into a 128B-swizzled shared tile for the SS MMA, and rescales
//               the TMEM O row only when m grows by more than 8 (factor 256),
//               which keeps P <= 256 and the rescale rare.
// Backward: two kernels of the same shape (dK/dV per KV tile looping over the
// q tiles of every q head of the group; dQ per q tile looping over KV tiles),
// fed by a row-wise Delta = sum(dO * O) pre-pass.  No atomics.
//
// Parity: replaces the FA2/FA3/SDPA attention of the reference's HF models
// (trainer/model.py:315-360) including packed varlen (trainer/rl.py:189-229).
#include <atomic>
#include <cuda_bf16.h>
#include <math.h>

#include <stdexcept>

#include "attention.h"
#include "common.cuh"
#include "tma.h"

namespace wb {
namespace attn {

constexpr int TILE = 128;         // queries / keys per tile
constexpr int HD = 128;           // head dim
constexpr int SLAB_BYTES = TILE * 64 * 2;   // one [128 rows x 64 cols] bf16 swizzled slab = 16 KB
constexpr int TILE_BYTES = 2 * SLAB_BYTES;  // [128 x 128] bf16 = 32 KB
constexpr int NUM_THREADS = 192;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;

// idesc: M=128, N=128, bf16 in, fp32 accumulate.
constexpr uint32_t IDESC_KK = idesc_bf16_f32(128, 128, 0, 0);   // A K-major, B K-major
constexpr uint32_t IDESC_KMN = idesc_bf16_f32(128, 128, 0, 1);  // A K-major, B MN-major

// K-major [128 rows x 128 cols] tile stored as two 64-col swizzled slabs.
// Descriptor for MMA k-step kk (16 columns each, 8 steps over 128 columns).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, int kk) {
  return smem_desc_sw128(tile_addr + (kk >> 2) * SLAB_BYTES + (kk & 3) * 32, 16, 1024);
}
// MN-major [128 k-rows x 128 n-cols] tile stored as two 64-col slabs of 128
// rows each (slab = n-group, LBO = slab size).  k-step kk advances 16 rows.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_addr, int kk) {
  return smem_desc_sw128(tile_addr + kk * 16 * 128, SLAB_BYTES, 1024);
}

// Write 8 bf16 (one 16-byte chunk `c` in 0..15) of row r into a K-major
// swizzled [128 x 128] tile (two 64-column slabs).
__device__ __forceinline__ void st_tile_chunk(uint8_t* tile, int r, int c, uint4 v) {
  const int slab = c >> 3;
  const int cc = (c & 7) ^ (r & 7);
  *reinterpret_cast<uint4*>(tile + slab * SLAB_BYTES + r * 128 + cc * 16) = v;
}

struct FwdParams {
  __nv_bfloat16* o;
  float* lse;
  const int* cu;
  const int* cuk;  // key sequences (nullptr: the query sequences); see AttnArgs::cu_seqlens_k
  int64_t o_row;  // elements between consecutive tokens of o
  int Hq, Hk, T, nseq;
  float scale_log2;
  int* err;
};

struct __align__(8) FwdSmem {
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t fwd_smem_bytes() { return 1024 + TILE_BYTES /*Q*/ + 4 * TILE_BYTES /*K,V x2*/ + TILE_BYTES /*P*/ + sizeof(FwdSmem) + 64; }

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sK[2] = {base + TILE_BYTES, base + 2 * TILE_BYTES};
  uint8_t* sV[2] = {base + 3 * TILE_BYTES, base + 4 * TILE_BYTES};
  uint8_t* sP = base + 5 * TILE_BYTES;
  FwdSmem* s = reinterpret_cast<FwdSmem*>(base + 6 * TILE_BYTES);
  volatile int* abort = &s->abort;

  const int seq = blockIdx.z;
  const int h = blockIdx.y;
  const int g = h / (p.Hq / p.Hk);
  const int s0 = p.cu[seq];
  const int L = p.cu[seq + 1] - s0;
  const int ks0 = p.cuk ? p.cuk[seq] : s0;          // first key row of the sequence
  const int Lk = p.cuk ? p.cuk[seq + 1] - ks0 : L;
  const int off = Lk - L;                            // query i sits at key position i + off
  const int n_qt = (L + TILE - 1) / TILE;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // longest tiles first
  if (qt < 0) return;
  const int q0 = qt * TILE;                       // within the sequence
  const int kv_end = min(Lk, q0 + off + TILE);     // causal: keys < q0 + off + 128
  const int n_kv = (kv_end + TILE - 1) / TILE;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&s->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->kv_full[i], 1);
      mbar_init(&s->kv_empty[i], 1);
      mbar_init(&s->s_full[i], 1);
    }
    mbar_init(&s->p_full, 128);
    mbar_init(&s->pv_done, 1);
    mbar_init(&s->drain, 1);
    s->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      mbar_arrive_expect_tx(&s->q_full, TILE_BYTES);
      tma_load_2d(&tmQ, &s->q_full, sQ, h * HD, s0 + q0);
      tma_load_2d(&tmQ, &s->q_full, sQ + SLAB_BYTES, h * HD + 64, s0 + q0);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        if (j >= 2) {
          if (!mbar_wait(&s->kv_empty[st], ((j - 2) >> 1) & 1, abort, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
        }
        mbar_arrive_expect_tx(&s->kv_full[st], 2 * TILE_BYTES);
        const int krow = ks0 + j * TILE;
        tma_load_2d(&tmK, &s->kv_full[st], sK[st], g * HD, krow);
        tma_load_2d(&tmK, &s->kv_full[st], sK[st] + SLAB_BYTES, g * HD + 64, krow);
        tma_load_2d(&tmV, &s->kv_full[st], sV[st], g * HD, krow);
        tma_load_2d(&tmV, &s->kv_full[st], sV[st] + SLAB_BYTES, g * HD + 64, krow);
        issued = j + 1;
      }
      if (!ok) {
        // drain in-flight loads (the last <= 2 stages and Q)
        for (int j = max(0, issued - 2); j < issued; ++j) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s->kv_full[j & 1], (j >> 1) & 1))
            if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
        }
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s->q_full, 0))
          if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&s->q_full, 0, abort, p.err, kErrTimeoutMma);
      const uint32_t aQ = smem_u32(sQ);
      const uint32_t aP = smem_u32(sP);
      bool any = false;
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&s->kv_full[st], (j >> 1) & 1, abort, p.err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK[st]);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16_ss(tS[st], kmajor_desc(aQ, kk), kmajor_desc(aK, kk), IDESC_KK, kk > 0);
        umma_commit(&s->s_full[st]);
        any = true;
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(&s->p_full, j & 1, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aV = smem_u32(sV[j & 1]);
#pragma unroll
        for (int kk = 0; kk < TILE / 16; ++kk)
          umma_f16_ss(tO, kmajor_desc(aP, kk), mnmajor_desc(aV, kk), IDESC_KMN, (j > 0 || kk > 0));
        umma_commit(&s->kv_empty[j & 1]);
        umma_commit(&s->pv_done);
      }
      if (any) {
        // retire everything before TMEM is released
        umma_commit(&s->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s->drain, 0))
          if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int q = warp & 3;
    const int r = q * 32 + lane;        // row in tile == TMEM lane
    const int qi = q0 + r;              // query index within the sequence
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      if (!mbar_wait_warp(&s->s_full[st], (j >> 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tS[st] + lane_off + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[c * 32 + e] = __uint_as_float(v[e]) * p.scale_log2;
      }
      const int k0 = j * TILE;
      if (j == n_kv - 1) {
        const int lim = min(qi + off + 1, Lk) - k0;  // keys [0, lim) valid
#pragma unroll
        for (int e = 0; e < 128; ++e)
          if (e >= lim) sv[e] = -INFINITY;
      }
      float mt = sv[0];
#pragma unroll
      for (int e = 1; e < 128; ++e) mt = fmaxf(mt, sv[e]);
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_run = mt;
      } else if (mt > m_run + RESCALE_THRESHOLD) {
        alpha = exp2f(m_run - mt);
        m_run = mt;
        rescale = true;
      }
      // P buffer and O must be idle: wait for PV_{j-1}
      if (j > 0) {
        if (!mbar_wait_warp(&s->pv_done, (j - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
        tc_fence_after();
      }
      // tcgen05.ld/st are warp-collective: rescale the whole warp's rows
      // together when any row needs it (alpha = 1 for the others).
      if (__any_sync(0xffffffffu, rescale)) {
        l_run *= alpha;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t v[16];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
              : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
              : "r"(tO + lane_off + c * 16));
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st_32x32b_x16(tO + lane_off + c * 16, v);
        }
        tmem_wait_st();
      }
      float ls = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float pe[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pe[e] = exp2f(sv[c * 8 + e] - m_run);
          ls += pe[e];
        }
        uint4 w;
        w.x = pack_bf16(pe[0], pe[1]);
        w.y = pack_bf16(pe[2], pe[3]);
        w.z = pack_bf16(pe[4], pe[5]);
        w.w = pack_bf16(pe[6], pe[7]);
        st_tile_chunk(sP, r, c, w);
      }
      l_run += ls;
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&s->p_full);
    }
    if (ok && n_kv > 0) {
      if (mbar_wait_warp(&s->pv_done, (n_kv - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) {
        tc_fence_after();
        const bool valid = qi < L;
        const float inv_l = 1.f / l_run;
        __nv_bfloat16* orow = p.o + (int64_t)(s0 + qi) * p.o_row + (int64_t)h * HD;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tO + lane_off + c * 32, v);
          tmem_wait_ld();
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint4 w;
              w.x = pack_bf16(__uint_as_float(v[8 * u + 0]) * inv_l, __uint_as_float(v[8 * u + 1]) * inv_l);
              w.y = pack_bf16(__uint_as_float(v[8 * u + 2]) * inv_l, __uint_as_float(v[8 * u + 3]) * inv_l);
              w.z = pack_bf16(__uint_as_float(v[8 * u + 4]) * inv_l, __uint_as_float(v[8 * u + 5]) * inv_l);
              w.w = pack_bf16(__uint_as_float(v[8 * u + 6]) * inv_l, __uint_as_float(v[8 * u + 7]) * inv_l);
              dst[u] = w;
            }
          }
        }
        if (valid) p.lse[(int64_t)h * p.T + s0 + qi] = (m_run + log2f(l_run)) * 0.6931471805599453f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ------------------------------------------------------------------ backward
// delta[h, t] = sum_d dO[t, h, d] * O[t, h, d]   (one warp per (t, h))
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, int64_t o_row,
                                  const __nv_bfloat16* __restrict__ dout, float* __restrict__ delta,
                                  int T, int Hq) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * Hq) return;
  const int t = w / Hq, h = w - t * Hq;
  const uint2 a = reinterpret_cast<const uint2*>(o + (int64_t)t * o_row + h * HD)[lane];
  const uint2 b = reinterpret_cast<const uint2*>(dout + ((int64_t)t * Hq + h) * HD)[lane];
  float acc = bf16_lo(a.x) * bf16_lo(b.x) + bf16_hi(a.x) * bf16_hi(b.x) + bf16_lo(a.y) * bf16_lo(b.y) +
              bf16_hi(a.y) * bf16_hi(b.y);
  acc = warp_sum(acc);
  if (lane == 0) delta[(int64_t)h * T + t] = acc;
}

struct BwdParams {
  const float* lse;    // [Hq, T]
  const float* delta;  // [Hq, T]
  const int* cu;
  const int* cuk;      // key sequences (v2 kernels; nullptr: the query sequences)
  __nv_bfloat16* dq;   // [T, Hq, 128]
  __nv_bfloat16* dk;   // [T, Hk, 128]
  __nv_bfloat16* dv;
  int Hq, Hk, T;
  float scale, scale_log2;
  int* err;
};

__device__ __forceinline__ void ld_row128(uint32_t taddr, float (&out)[128], float mul) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(taddr + c * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e) out[c * 32 + e] = __uint_as_float(v[e]) * mul;
  }
}

// Store a 128-column fp32 TMEM row (times `mul`) as bf16 to global.
__device__ __forceinline__ void store_row128(uint32_t taddr, __nv_bfloat16* dst, float mul, bool valid) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(taddr + c * 32, v);
    tmem_wait_ld();
    if (valid) {
      uint4* d = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 w;
        w.x = pack_bf16(__uint_as_float(v[8 * u + 0]) * mul, __uint_as_float(v[8 * u + 1]) * mul);
        w.y = pack_bf16(__uint_as_float(v[8 * u + 2]) * mul, __uint_as_float(v[8 * u + 3]) * mul);
        w.z = pack_bf16(__uint_as_float(v[8 * u + 4]) * mul, __uint_as_float(v[8 * u + 5]) * mul);
        w.w = pack_bf16(__uint_as_float(v[8 * u + 6]) * mul, __uint_as_float(v[8 * u + 7]) * mul);
        d[u] = w;
      }
    }
  }
}

// Columns [0, 64) of a TMEM accumulator row (from taddr) -> 64 bf16 at dst.
__device__ __forceinline__ void store_row64(uint32_t taddr, __nv_bfloat16* dst, float mul, bool valid) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(taddr + c * 32, v);
    tmem_wait_ld();
    if (valid) {
      uint4* d = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 w;
        w.x = pack_bf16(__uint_as_float(v[8 * u + 0]) * mul, __uint_as_float(v[8 * u + 1]) * mul);
        w.y = pack_bf16(__uint_as_float(v[8 * u + 2]) * mul, __uint_as_float(v[8 * u + 3]) * mul);
        w.z = pack_bf16(__uint_as_float(v[8 * u + 4]) * mul, __uint_as_float(v[8 * u + 5]) * mul);
        w.w = pack_bf16(__uint_as_float(v[8 * u + 6]) * mul, __uint_as_float(v[8 * u + 7]) * mul);
        d[u] = w;
      }
    }
  }
}

struct __align__(8) BwdSmem {
  uint64_t a_full;      // loaded-once operands
  uint64_t b_full[2];   // per-iteration operands
  uint64_t b_empty[2];
  uint64_t s_full;
  uint64_t p_full;
  uint64_t mma_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// dK / dV: CTA per (kv tile, kv head, seq); loop over (q head in group, q tile).
// Thread = key row.  S^T = K Q^T, dP^T = V dO^T, P^T = exp2(S^T*sl2 - lse2[q]),
// dS^T = P^T (dP^T - delta[q]);  dV += P^T dO,  dK += dS^T Q.
constexpr size_t dkv_smem_bytes() { return 1024 + 2 * TILE_BYTES /*K,V*/ + 2 * TILE_BYTES /*Q,dO*/ + 2 * TILE_BYTES /*Pt,dSt*/ + sizeof(BwdSmem) + 64; }

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = base;
  uint8_t* sV = base + TILE_BYTES;
  uint8_t* sQ = base + 2 * TILE_BYTES;
  uint8_t* sDO = base + 3 * TILE_BYTES;
  uint8_t* sPt = base + 4 * TILE_BYTES;
  uint8_t* sdSt = base + 5 * TILE_BYTES;
  BwdSmem* s = reinterpret_cast<BwdSmem*>(base + 6 * TILE_BYTES);
  volatile int* abort = &s->abort;

  const int seq = blockIdx.z, g = blockIdx.y;
  const int rep = p.Hq / p.Hk;
  const int s0 = p.cu[seq];
  const int L = p.cu[seq + 1] - s0;
  const int n_t = (L + TILE - 1) / TILE;
  const int jt = static_cast<int>(blockIdx.x);  // kv tile
  if (jt >= n_t) return;
  const int k0 = jt * TILE;
  const int n_q = n_t - jt;               // causal: q tiles jt .. n_t-1
  const int n_it = rep * n_q;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&s->a_full, 1);
    mbar_init(&s->b_full[0], 1);
    mbar_init(&s->b_empty[0], 1);
    mbar_init(&s->s_full, 1);
    mbar_init(&s->p_full, 128);
    mbar_init(&s->mma_done, 1);
    mbar_init(&s->drain, 1);
    s->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&s->a_full, 2 * TILE_BYTES);
      tma_load_2d(&tmK, &s->a_full, sK, g * HD, s0 + k0);
      tma_load_2d(&tmK, &s->a_full, sK + SLAB_BYTES, g * HD + 64, s0 + k0);
      tma_load_2d(&tmV, &s->a_full, sV, g * HD, s0 + k0);
      tma_load_2d(&tmV, &s->a_full, sV + SLAB_BYTES, g * HD + 64, s0 + k0);
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        if (it > 0 && !mbar_wait(&s->b_empty[0], (it - 1) & 1, abort, p.err, kErrTimeoutProducer)) break;
        const int h = g * rep + it / n_q;
        const int qrow = s0 + (jt + it % n_q) * TILE;
        mbar_arrive_expect_tx(&s->b_full[0], 2 * TILE_BYTES);
        tma_load_2d(&tmQ, &s->b_full[0], sQ, h * HD, qrow);
        tma_load_2d(&tmQ, &s->b_full[0], sQ + SLAB_BYTES, h * HD + 64, qrow);
        tma_load_2d(&tmDO, &s->b_full[0], sDO, h * HD, qrow);
        tma_load_2d(&tmDO, &s->b_full[0], sDO + SLAB_BYTES, h * HD + 64, qrow);
        issued = it + 1;
      }
      if (*abort) {
        const uint64_t t0 = globaltimer_ns();
        while (issued > 0 && !mbar_try_wait(&s->b_full[0], (issued - 1) & 1))
          if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(&s->a_full, 0))
          if (globaltimer_ns() - t1 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&s->a_full, 0, abort, p.err, kErrTimeoutMma);
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aQ = smem_u32(sQ), aDO = smem_u32(sDO);
      const uint32_t aPt = smem_u32(sPt), adSt = smem_u32(sdSt);
      bool any = false;
      for (int it = 0; it < n_it && ok; ++it) {
        if (!mbar_wait(&s->b_full[0], it & 1, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tS, kmajor_desc(aK, kk), kmajor_desc(aQ, kk), IDESC_KK, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tdP, kmajor_desc(aV, kk), kmajor_desc(aDO, kk), IDESC_KK, kk > 0);
        umma_commit(&s->s_full);
        any = true;
        if (!mbar_wait(&s->p_full, it & 1, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tdV, kmajor_desc(aPt, kk), mnmajor_desc(aDO, kk), IDESC_KMN, (it > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tdK, kmajor_desc(adSt, kk), mnmajor_desc(aQ, kk), IDESC_KMN, (it > 0 || kk > 0));
        umma_commit(&s->b_empty[0]);
        umma_commit(&s->mma_done);
      }
      if (any) {
        umma_commit(&s->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s->drain, 0))
          if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;  // key row
    const int kj = k0 + r;        // key index within the sequence
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int h = g * rep + it / n_q;
      const int i = jt + it % n_q;  // q tile
      const int q0 = i * TILE;
      const float* lse_row = p.lse + (int64_t)h * p.T + s0 + q0;
      const float* dlt_row = p.delta + (int64_t)h * p.T + s0 + q0;
      const int qlim = L - q0;  // columns c < qlim are real queries
      if (!mbar_wait_warp(&s->s_full, it & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      float pt[128];
      ld_row128(tS + lane_off, pt, p.scale_log2);
      // causal: key kj attends to query qi iff kj <= qi; also qi < L, kj < L
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const int qi = q0 + c;
        const bool valid = (kj <= qi) && (c < qlim) && (kj < L);
        pt[c] = valid ? exp2f(pt[c] - __ldg(lse_row + c) * LOG2E) : 0.f;
      }
      if (it > 0) {
        if (!mbar_wait_warp(&s->mma_done, (it - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 w;
        w.x = pack_bf16(pt[c * 8 + 0], pt[c * 8 + 1]);
        w.y = pack_bf16(pt[c * 8 + 2], pt[c * 8 + 3]);
        w.z = pack_bf16(pt[c * 8 + 4], pt[c * 8 + 5]);
        w.w = pack_bf16(pt[c * 8 + 6], pt[c * 8 + 7]);
        st_tile_chunk(sPt, r, c, w);
      }
      // dS^T = P^T * (dP^T - delta)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tdP + lane_off + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int col = c * 32 + e;
          pt[col] *= (__uint_as_float(v[e]) - (col < qlim ? __ldg(dlt_row + col) : 0.f));
        }
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 w;
        w.x = pack_bf16(pt[c * 8 + 0], pt[c * 8 + 1]);
        w.y = pack_bf16(pt[c * 8 + 2], pt[c * 8 + 3]);
        w.z = pack_bf16(pt[c * 8 + 4], pt[c * 8 + 5]);
        w.w = pack_bf16(pt[c * 8 + 6], pt[c * 8 + 7]);
        st_tile_chunk(sdSt, r, c, w);
      }
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&s->p_full);
    }
    if (ok && n_it > 0 && mbar_wait_warp(&s->mma_done, (n_it - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const bool valid = kj < L;
      store_row128(tdV + lane_off, p.dv + ((int64_t)(s0 + kj) * p.Hk + g) * HD, 1.f, valid);
      store_row128(tdK + lane_off, p.dk + ((int64_t)(s0 + kj) * p.Hk + g) * HD, p.scale, valid);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ: CTA per (q tile, q head, seq); loop over kv tiles (2-stage K/V ring).
// S = Q K^T, dP = dO V^T, dS = P (dP - delta);  dQ += dS K.
constexpr size_t dq_smem_bytes() { return 1024 + 2 * TILE_BYTES /*Q,dO*/ + 4 * TILE_BYTES /*K,V x2*/ + TILE_BYTES /*dS*/ + sizeof(BwdSmem) + 64; }

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sDO = base + TILE_BYTES;
  uint8_t* sK[2] = {base + 2 * TILE_BYTES, base + 3 * TILE_BYTES};
  uint8_t* sV[2] = {base + 4 * TILE_BYTES, base + 5 * TILE_BYTES};
  uint8_t* sdS = base + 6 * TILE_BYTES;
  BwdSmem* s = reinterpret_cast<BwdSmem*>(base + 7 * TILE_BYTES);
  volatile int* abort = &s->abort;

  const int seq = blockIdx.z, h = blockIdx.y;
  const int g = h / (p.Hq / p.Hk);
  const int s0 = p.cu[seq];
  const int L = p.cu[seq + 1] - s0;
  const int n_qt = (L + TILE - 1) / TILE;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);
  if (qt < 0) return;
  const int q0 = qt * TILE;
  const int n_kv = (min(L, q0 + TILE) + TILE - 1) / TILE;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&s->a_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->b_full[i], 1);
      mbar_init(&s->b_empty[i], 1);
    }
    mbar_init(&s->s_full, 1);
    mbar_init(&s->p_full, 128);
    mbar_init(&s->mma_done, 1);
    mbar_init(&s->drain, 1);
    s->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  const uint32_t tS = tmem, tdP = tmem + 128, tdQ = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&s->a_full, 2 * TILE_BYTES);
      tma_load_2d(&tmQ, &s->a_full, sQ, h * HD, s0 + q0);
      tma_load_2d(&tmQ, &s->a_full, sQ + SLAB_BYTES, h * HD + 64, s0 + q0);
      tma_load_2d(&tmDO, &s->a_full, sDO, h * HD, s0 + q0);
      tma_load_2d(&tmDO, &s->a_full, sDO + SLAB_BYTES, h * HD + 64, s0 + q0);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&s->b_empty[st], ((j - 2) >> 1) & 1, abort, p.err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&s->b_full[st], 2 * TILE_BYTES);
        const int krow = s0 + j * TILE;
        tma_load_2d(&tmK, &s->b_full[st], sK[st], g * HD, krow);
        tma_load_2d(&tmK, &s->b_full[st], sK[st] + SLAB_BYTES, g * HD + 64, krow);
        tma_load_2d(&tmV, &s->b_full[st], sV[st], g * HD, krow);
        tma_load_2d(&tmV, &s->b_full[st], sV[st] + SLAB_BYTES, g * HD + 64, krow);
        issued = j + 1;
      }
      if (*abort) {
        for (int j = max(0, issued - 2); j < issued; ++j) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s->b_full[j & 1], (j >> 1) & 1))
            if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
        }
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(&s->a_full, 0))
          if (globaltimer_ns() - t1 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&s->a_full, 0, abort, p.err, kErrTimeoutMma);
      const uint32_t aQ = smem_u32(sQ), aDO = smem_u32(sDO), adS = smem_u32(sdS);
      bool any = false;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&s->b_full[st], (j >> 1) & 1, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aK = smem_u32(sK[st]), aV = smem_u32(sV[st]);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tS, kmajor_desc(aQ, kk), kmajor_desc(aK, kk), IDESC_KK, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tdP, kmajor_desc(aDO, kk), kmajor_desc(aV, kk), IDESC_KK, kk > 0);
        umma_commit(&s->s_full);
        any = true;
        if (!mbar_wait(&s->p_full, j & 1, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tdQ, kmajor_desc(adS, kk), mnmajor_desc(aK, kk), IDESC_KMN, (j > 0 || kk > 0));
        umma_commit(&s->b_empty[st]);
        umma_commit(&s->mma_done);
      }
      if (any) {
        umma_commit(&s->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s->drain, 0))
          if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const bool vq = qi < L;
    const float lse2 = vq ? p.lse[(int64_t)h * p.T + s0 + qi] * LOG2E : INFINITY;
    const float dlt = vq ? p.delta[(int64_t)h * p.T + s0 + qi] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait_warp(&s->s_full, j & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      float pr[128];
      ld_row128(tS + lane_off, pr, p.scale_log2);
      const int kb = j * TILE;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const int kj = kb + c;
        const bool valid = (kj <= qi) && (kj < L) && vq;
        pr[c] = valid ? exp2f(pr[c] - lse2) : 0.f;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tdP + lane_off + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) pr[c * 32 + e] *= (__uint_as_float(v[e]) - dlt);
      }
      if (j > 0 && !mbar_wait_warp(&s->mma_done, (j - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 w;
        w.x = pack_bf16(pr[c * 8 + 0], pr[c * 8 + 1]);
        w.y = pack_bf16(pr[c * 8 + 2], pr[c * 8 + 3]);
        w.z = pack_bf16(pr[c * 8 + 4], pr[c * 8 + 5]);
        w.w = pack_bf16(pr[c * 8 + 6], pr[c * 8 + 7]);
        st_tile_chunk(sdS, r, c, w);
      }
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&s->p_full);
    }
    if (ok && n_kv > 0 && mbar_wait_warp(&s->mma_done, (n_kv - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      store_row128(tdQ + lane_off, p.dq + ((int64_t)(s0 + qi) * p.Hq + h) * HD, p.scale, vq);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ------------------------------------------------------------ dK/dV, v2
// CTA per (kv tile of 128 keys, q head, seq): every q head of a GQA group
// works in parallel and writes fp32 partial dK/dV; a reduction kernel sums
// the group (or, with one q head per kv head, the CTA writes bf16 directly).
// Queries come in tiles of 64 through a 2-stage TMA ring, and S^T / dP^T are
// double-buffered in TMEM so the MMAs of tile i+1 overlap the softmax of i.
//   S^T = K Q^T, dP^T = V dO^T         (M=128 keys, N=64 queries, K=128)
//   P^T = exp2(S^T*sl2 - lse2[q]),  dS^T = P^T (dP^T - delta[q])
//   dV += P^T dO, dK += dS^T Q         (M=128 keys, N=128 dims, K=64 queries)
constexpr int QT = 64;
// v2 backward kernels: warp 0 TMA, warp 1 MMA, warps 2..9 softmax.  Two
// softmax warps share each TMEM lane quadrant (warp & 3) and split the 64
// columns of a tile (half = (warp - 2) / 4 takes columns 32*half..+31), so each
// SM sub-partition runs two independent exp/ALU streams.
constexpr int NUM_THREADS_BWD2 = 64 + 256;
constexpr int BWD2_SOFTMAX_THREADS = 256;
constexpr int QSLAB = QT * 64 * 2;          // [64 rows x 64 cols] bf16 = 8 KB
constexpr int QTILE_BYTES = 2 * QSLAB;      // [64 x 128] = 16 KB
constexpr int PT_BYTES = TILE * QT * 2;     // [128 keys x 64 q] = 16 KB
constexpr uint32_t IDESC_S64 = idesc_bf16_f32(128, 64, 0, 0);

__device__ __forceinline__ uint64_t kmajor64_desc(uint32_t tile, int kk) {
  return smem_desc_sw128(tile + (kk >> 2) * QSLAB + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t mnmajor64_desc(uint32_t tile, int kk) {
  return smem_desc_sw128(tile + kk * 16 * 128, QSLAB, 1024);
}
__device__ __forceinline__ uint64_t pt_desc(uint32_t tile, int kk) {
  return smem_desc_sw128(tile + kk * 32, 16, 1024);
}

struct Bwd2Params {
  BwdParams b;
  float* part_dk;  // [T, Hq, 128] fp32 (rep > 1)
  float* part_dv;
};

struct __align__(8) Bwd2Smem {
  uint64_t a_full;
  uint64_t b_full[2];
  uint64_t b_empty[2];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t mma_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t dkv2_smem_bytes() {
  return 1024 + 2 * TILE_BYTES + 4 * QTILE_BYTES + 2 * PT_BYTES + sizeof(Bwd2Smem) + 64;
}

__global__ void __launch_bounds__(NUM_THREADS_BWD2, 1)
    attn_bwd_dkv2_kernel(const __grid_constant__ CUtensorMap tmQ64, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO64,
                         Bwd2Params p2) {
  const BwdParams& p = p2.b;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = base;
  uint8_t* sV = base + TILE_BYTES;
  uint8_t* sQ[2] = {base + 2 * TILE_BYTES, base + 2 * TILE_BYTES + QTILE_BYTES};
  uint8_t* sDO[2] = {base + 2 * TILE_BYTES + 2 * QTILE_BYTES, base + 2 * TILE_BYTES + 3 * QTILE_BYTES};
  uint8_t* sPt = base + 2 * TILE_BYTES + 4 * QTILE_BYTES;
  uint8_t* sdSt = sPt + PT_BYTES;
  Bwd2Smem* s = reinterpret_cast<Bwd2Smem*>(sdSt + PT_BYTES);
  volatile int* abort = &s->abort;

  const int seq = blockIdx.z, h = blockIdx.y;
  const int rep = p.Hq / p.Hk;
  const int g = h / rep;
  const int s0 = p.cu[seq];
  const int L = p.cu[seq + 1] - s0;
  const int ks0 = p.cuk ? p.cuk[seq] : s0;
  const int Lk = p.cuk ? p.cuk[seq + 1] - ks0 : L;
  const int off = Lk - L;
  const int n_kt = (Lk + TILE - 1) / TILE;
  const int jt = n_kt - 1 - static_cast<int>(blockIdx.x);  // heaviest (earliest) tiles launch first
  if (jt < 0) return;
  const int k0 = jt * TILE;
  const int i0 = max(0, k0 - off) / QT;    // first q tile that sees these keys (causal)
  const int n_it = max(0, (L + QT - 1) / QT - i0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&s->a_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->b_full[i], 1);
      mbar_init(&s->b_empty[i], 1);
      mbar_init(&s->s_full[i], 1);
    }
    mbar_init(&s->p_full, BWD2_SOFTMAX_THREADS);
    mbar_init(&s->mma_done, 1);
    mbar_init(&s->drain, 1);
    s->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  const uint32_t tS[2] = {tmem, tmem + 64};
  const uint32_t tdP[2] = {tmem + 128, tmem + 192};
  const uint32_t tdV = tmem + 256, tdK = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&s->a_full, 2 * TILE_BYTES);
      tma_load_2d(&tmK, &s->a_full, sK, g * HD, ks0 + k0);
      tma_load_2d(&tmK, &s->a_full, sK + SLAB_BYTES, g * HD + 64, ks0 + k0);
      tma_load_2d(&tmV, &s->a_full, sV, g * HD, ks0 + k0);
      tma_load_2d(&tmV, &s->a_full, sV + SLAB_BYTES, g * HD + 64, ks0 + k0);
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int st = it & 1;
        if (it >= 2 && !mbar_wait(&s->b_empty[st], ((it - 2) >> 1) & 1, abort, p.err, kErrTimeoutProducer)) break;
        const int qrow = s0 + (i0 + it) * QT;
        mbar_arrive_expect_tx(&s->b_full[st], 2 * QTILE_BYTES);
        tma_load_2d(&tmQ64, &s->b_full[st], sQ[st], h * HD, qrow);
        tma_load_2d(&tmQ64, &s->b_full[st], sQ[st] + QSLAB, h * HD + 64, qrow);
        tma_load_2d(&tmDO64, &s->b_full[st], sDO[st], h * HD, qrow);
        tma_load_2d(&tmDO64, &s->b_full[st], sDO[st] + QSLAB, h * HD + 64, qrow);
        issued = it + 1;
      }
      if (*abort) {
        for (int it = max(0, issued - 2); it < issued; ++it) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s->b_full[it & 1], (it >> 1) & 1))
            if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
        }
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(&s->a_full, 0))
          if (globaltimer_ns() - t1 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&s->a_full, 0, abort, p.err, kErrTimeoutMma);
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV);
      const uint32_t aPt = smem_u32(sPt), adSt = smem_u32(sdSt);
      bool any = false;
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        if (!mbar_wait(&s->b_full[st], (it >> 1) & 1, abort, p.err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ[st]), aDO = smem_u32(sDO[st]);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tS[st], kmajor_desc(aK, kk), kmajor64_desc(aQ, kk), IDESC_S64, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tdP[st], kmajor_desc(aV, kk), kmajor64_desc(aDO, kk), IDESC_S64, kk > 0);
        umma_commit(&s->s_full[st]);
        any = true;
        return true;
      };
      if (ok && n_it > 0) ok = issue_s(0);
      for (int it = 0; it < n_it && ok; ++it) {
        if (it + 1 < n_it && !issue_s(it + 1)) { ok = false; break; }
        if (!mbar_wait(&s->p_full, it & 1, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ[it & 1]), aDO = smem_u32(sDO[it & 1]);
#pragma unroll
        for (int kk = 0; kk < QT / 16; ++kk)
          umma_f16_ss(tdV, pt_desc(aPt, kk), mnmajor64_desc(aDO, kk), IDESC_KMN, (it > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < QT / 16; ++kk)
          umma_f16_ss(tdK, pt_desc(adSt, kk), mnmajor64_desc(aQ, kk), IDESC_KMN, (it > 0 || kk > 0));
        umma_commit(&s->b_empty[it & 1]);
        umma_commit(&s->mma_done);
      }
      if (any) {
        umma_commit(&s->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s->drain, 0))
          if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;  // key row
    const int kj = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int half = (warp - 2) >> 2;
    const int cb = half * 32;  // this warp's 32 query columns of the tile
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int st = it & 1;
      const int q0 = (i0 + it) * QT;
      const float* lse_row = p.lse + (int64_t)h * p.T + s0 + q0;
      const float* dlt_row = p.delta + (int64_t)h * p.T + s0 + q0;
      const int qlim = L - q0;
      if (!mbar_wait_warp(&s->s_full[st], (it >> 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      float pt[32], dp[32];
      {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tS[st] + lane_off + cb, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) pt[e] = __uint_as_float(v[e]) * p.scale_log2;
        tmem_ld_32x32b_x32(tdP[st] + lane_off + cb, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) dp[e] = __uint_as_float(v[e]);
      }
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int qc = cb + c;
        const int qi = q0 + qc;
        const bool valid = (kj <= qi + off) && (qc < qlim) && (kj < Lk);
        const float pv = valid ? exp2f(pt[c] - __ldg(lse_row + qc) * LOG2E) : 0.f;
        pt[c] = pv;
        dp[c] = pv * (dp[c] - (valid ? __ldg(dlt_row + qc) : 0.f));
      }
      if (it > 0 && !mbar_wait_warp(&s->mma_done, (it - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 w;
        w.x = pack_bf16(pt[c * 8 + 0], pt[c * 8 + 1]);
        w.y = pack_bf16(pt[c * 8 + 2], pt[c * 8 + 3]);
        w.z = pack_bf16(pt[c * 8 + 4], pt[c * 8 + 5]);
        w.w = pack_bf16(pt[c * 8 + 6], pt[c * 8 + 7]);
        st_tile_chunk(sPt, r, half * 4 + c, w);
        uint4 d;
        d.x = pack_bf16(dp[c * 8 + 0], dp[c * 8 + 1]);
        d.y = pack_bf16(dp[c * 8 + 2], dp[c * 8 + 3]);
        d.z = pack_bf16(dp[c * 8 + 4], dp[c * 8 + 5]);
        d.w = pack_bf16(dp[c * 8 + 6], dp[c * 8 + 7]);
        st_tile_chunk(sdSt, r, half * 4 + c, d);
      }
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&s->p_full);
    }
    if (n_it == 0 && kj < Lk) {
      // keys that no query sees (an empty query sequence): zero gradients
      const uint4 z = make_uint4(0, 0, 0, 0);
      if (rep == 1) {
        uint4* dv4 = reinterpret_cast<uint4*>(p.dv + ((int64_t)(ks0 + kj) * p.Hk + g) * HD);
        uint4* dk4 = reinterpret_cast<uint4*>(p.dk + ((int64_t)(ks0 + kj) * p.Hk + g) * HD);
        for (int u = half * 8; u < half * 8 + 8; ++u) dv4[u] = z, dk4[u] = z;
      } else {
        uint4* dv4 = reinterpret_cast<uint4*>(p2.part_dv + ((int64_t)(ks0 + kj) * p.Hq + h) * HD);
        uint4* dk4 = reinterpret_cast<uint4*>(p2.part_dk + ((int64_t)(ks0 + kj) * p.Hq + h) * HD);
        for (int u = half * 16; u < half * 16 + 16; ++u) dv4[u] = z, dk4[u] = z;
      }
    }
    if (ok && n_it > 0 && mbar_wait_warp(&s->mma_done, (n_it - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const bool valid = kj < Lk;
      if (rep == 1) {
        store_row64(tdV + lane_off + half * 64, p.dv + ((int64_t)(ks0 + kj) * p.Hk + g) * HD + half * 64, 1.f, valid);
        store_row64(tdK + lane_off + half * 64, p.dk + ((int64_t)(ks0 + kj) * p.Hk + g) * HD + half * 64, p.scale,
                    valid);
      } else {
#pragma unroll
        for (int c = half * 2; c < half * 2 + 2; ++c) {
          uint32_t v[32], w[32];
          tmem_ld_32x32b_x32(tdV + lane_off + c * 32, v);
          tmem_ld_32x32b_x32(tdK + lane_off + c * 32, w);
          tmem_wait_ld();
          if (valid) {
            float4* dv4 = reinterpret_cast<float4*>(p2.part_dv + ((int64_t)(ks0 + kj) * p.Hq + h) * HD + c * 32);
            float4* dk4 = reinterpret_cast<float4*>(p2.part_dk + ((int64_t)(ks0 + kj) * p.Hq + h) * HD + c * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              dv4[u] = make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]), __uint_as_float(v[4 * u + 2]),
                                   __uint_as_float(v[4 * u + 3]));
              dk4[u] = make_float4(__uint_as_float(w[4 * u]), __uint_as_float(w[4 * u + 1]), __uint_as_float(w[4 * u + 2]),
                                   __uint_as_float(w[4 * u + 3]));
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dk/dv[t, g] = sum over the group's q heads of the fp32 partials (dK also
// times the softmax scale).  One warp per (token, kv head); 4 dims per lane.
__global__ void attn_dkv_reduce_kernel(const float* __restrict__ part_dk, const float* __restrict__ part_dv,
                                       __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int T, int Hq,
                                       int Hk, float scale) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * Hk) return;
  const int t = w / Hk, g = w - t * Hk;
  const int rep = Hq / Hk;
  float4 ak = make_float4(0.f, 0.f, 0.f, 0.f), av = ak;
  for (int r = 0; r < rep; ++r) {
    const int64_t off = ((int64_t)t * Hq + g * rep + r) * HD;
    const float4 k4 = reinterpret_cast<const float4*>(part_dk + off)[lane];
    const float4 v4 = reinterpret_cast<const float4*>(part_dv + off)[lane];
    ak.x += k4.x; ak.y += k4.y; ak.z += k4.z; ak.w += k4.w;
    av.x += v4.x; av.y += v4.y; av.z += v4.z; av.w += v4.w;
  }
  const int64_t o = ((int64_t)t * Hk + g) * HD;
  uint2 kk, vv;
  kk.x = pack_bf16(ak.x * scale, ak.y * scale);
  kk.y = pack_bf16(ak.z * scale, ak.w * scale);
  vv.x = pack_bf16(av.x, av.y);
  vv.y = pack_bf16(av.z, av.w);
  reinterpret_cast<uint2*>(dk + o)[lane] = kk;
  reinterpret_cast<uint2*>(dv + o)[lane] = vv;
}


// ---------------------------------------------------------------- dQ, v2
// CTA per (128-query tile, q head, seq); keys in tiles of 64 through a
// 3-stage TMA ring; S / dP double-buffered in TMEM so the next tile's MMAs
// overlap this tile's softmax.
//   S = Q K^T, dP = dO V^T   (M=128 q, N=64 keys, K=128)
//   dS = P (dP - delta)      (thread = query row)
//   dQ += dS K               (M=128 q, N=128 dims, K=64 keys)
constexpr int KT = 64;
constexpr int KV_STAGES = 3;
constexpr int DS_BYTES = TILE * KT * 2;  // [128 q x 64 keys] = 16 KB

constexpr size_t dq2_smem_bytes() {
  return 1024 + 2 * TILE_BYTES + KV_STAGES * 2 * QTILE_BYTES + DS_BYTES + sizeof(Bwd2Smem) + 64 + 64;
}

struct __align__(8) Dq2Smem {
  uint64_t a_full;
  uint64_t kv_full[KV_STAGES];
  uint64_t kv_empty[KV_STAGES];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t ds_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(NUM_THREADS_BWD2, 1)
    attn_bwd_dq2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK64,
                        const __grid_constant__ CUtensorMap tmV64, const __grid_constant__ CUtensorMap tmDO,
                        BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sDO = base + TILE_BYTES;
  uint8_t* sKV = base + 2 * TILE_BYTES;  // stage st: K at +st*2*QTILE, V at +QTILE
  uint8_t* sdS = sKV + KV_STAGES * 2 * QTILE_BYTES;
  Dq2Smem* s = reinterpret_cast<Dq2Smem*>(sdS + DS_BYTES);
  volatile int* abort = &s->abort;

  const int seq = blockIdx.z, h = blockIdx.y;
  const int g = h / (p.Hq / p.Hk);
  const int s0 = p.cu[seq];
  const int L = p.cu[seq + 1] - s0;
  const int ks0 = p.cuk ? p.cuk[seq] : s0;
  const int Lk = p.cuk ? p.cuk[seq + 1] - ks0 : L;
  const int off = Lk - L;
  const int n_qt = (L + TILE - 1) / TILE;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);
  if (qt < 0) return;
  const int q0 = qt * TILE;
  const int n_kv = (min(Lk, q0 + off + TILE) + KT - 1) / KT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&s->a_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&s->kv_full[i], 1);
      mbar_init(&s->kv_empty[i], 1);
    }
    mbar_init(&s->s_full[0], 1);
    mbar_init(&s->s_full[1], 1);
    mbar_init(&s->p_full, BWD2_SOFTMAX_THREADS);
    mbar_init(&s->ds_done, 1);
    mbar_init(&s->drain, 1);
    s->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  const uint32_t tS[2] = {tmem, tmem + 64};
  const uint32_t tdP[2] = {tmem + 128, tmem + 192};
  const uint32_t tdQ = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&s->a_full, 2 * TILE_BYTES);
      tma_load_2d(&tmQ, &s->a_full, sQ, h * HD, s0 + q0);
      tma_load_2d(&tmQ, &s->a_full, sQ + SLAB_BYTES, h * HD + 64, s0 + q0);
      tma_load_2d(&tmDO, &s->a_full, sDO, h * HD, s0 + q0);
      tma_load_2d(&tmDO, &s->a_full, sDO + SLAB_BYTES, h * HD + 64, s0 + q0);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % KV_STAGES;
        if (j >= KV_STAGES && !mbar_wait(&s->kv_empty[st], ((j - KV_STAGES) / KV_STAGES) & 1, abort, p.err, kErrTimeoutProducer)) break;
        uint8_t* kd = sKV + st * 2 * QTILE_BYTES;
        uint8_t* vd = kd + QTILE_BYTES;
        const int krow = ks0 + j * KT;
        mbar_arrive_expect_tx(&s->kv_full[st], 2 * QTILE_BYTES);
        tma_load_2d(&tmK64, &s->kv_full[st], kd, g * HD, krow);
        tma_load_2d(&tmK64, &s->kv_full[st], kd + QSLAB, g * HD + 64, krow);
        tma_load_2d(&tmV64, &s->kv_full[st], vd, g * HD, krow);
        tma_load_2d(&tmV64, &s->kv_full[st], vd + QSLAB, g * HD + 64, krow);
        issued = j + 1;
      }
      if (*abort) {
        for (int j = max(0, issued - KV_STAGES); j < issued; ++j) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s->kv_full[j % KV_STAGES], (j / KV_STAGES) & 1))
            if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
        }
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(&s->a_full, 0))
          if (globaltimer_ns() - t1 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&s->a_full, 0, abort, p.err, kErrTimeoutMma);
      const uint32_t aQ = smem_u32(sQ), aDO = smem_u32(sDO), adS = smem_u32(sdS);
      bool any = false;
      auto issue_s = [&](int j) -> bool {
        const int st = j % KV_STAGES;
        if (!mbar_wait(&s->kv_full[st], (j / KV_STAGES) & 1, abort, p.err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sKV + st * 2 * QTILE_BYTES), aV = aK + QTILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tS[j & 1], kmajor_desc(aQ, kk), kmajor64_desc(aK, kk), IDESC_S64, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tdP[j & 1], kmajor_desc(aDO, kk), kmajor64_desc(aV, kk), IDESC_S64, kk > 0);
        umma_commit(&s->s_full[j & 1]);
        any = true;
        return true;
      };
      if (ok && n_kv > 0) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(&s->p_full, j & 1, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const int st = j % KV_STAGES;
        const uint32_t aK = smem_u32(sKV + st * 2 * QTILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk)
          umma_f16_ss(tdQ, pt_desc(adS, kk), mnmajor64_desc(aK, kk), IDESC_KMN, (j > 0 || kk > 0));
        umma_commit(&s->kv_empty[st]);
        umma_commit(&s->ds_done);
      }
      if (any) {
        umma_commit(&s->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s->drain, 0))
          if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const bool vq = qi < L;
    const int half = (warp - 2) >> 2;
    const int cb = half * 32;  // this warp's 32 key columns of the tile
    const float lse2 = vq ? p.lse[(int64_t)h * p.T + s0 + qi] * LOG2E : INFINITY;
    const float dlt = vq ? p.delta[(int64_t)h * p.T + s0 + qi] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait_warp(&s->s_full[j & 1], (j >> 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      float pr[32], dp[32];
      {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tS[j & 1] + lane_off + cb, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) pr[e] = __uint_as_float(v[e]) * p.scale_log2;
        tmem_ld_32x32b_x32(tdP[j & 1] + lane_off + cb, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) dp[e] = __uint_as_float(v[e]);
      }
      const int kb = j * KT + cb;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int kj = kb + c;
        const bool valid = (kj <= qi + off) && (kj < Lk) && vq;
        const float pv = valid ? exp2f(pr[c] - lse2) : 0.f;
        pr[c] = pv * (dp[c] - dlt);
      }
      if (j > 0 && !mbar_wait_warp(&s->ds_done, (j - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 w;
        w.x = pack_bf16(pr[c * 8 + 0], pr[c * 8 + 1]);
        w.y = pack_bf16(pr[c * 8 + 2], pr[c * 8 + 3]);
        w.z = pack_bf16(pr[c * 8 + 4], pr[c * 8 + 5]);
        w.w = pack_bf16(pr[c * 8 + 6], pr[c * 8 + 7]);
        st_tile_chunk(sdS, r, half * 4 + c, w);
      }
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&s->p_full);
    }
    if (ok && n_kv > 0 && mbar_wait_warp(&s->ds_done, (n_kv - 1) & 1, abort, p.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      store_row64(tdQ + lane_off + half * 64, p.dq + ((int64_t)(s0 + qi) * p.Hq + h) * HD + half * 64, p.scale, vq);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn

static CUtensorMap head_map(const void* base, int64_t row_stride, int heads, int T) {
  // 2-D view: T rows x (heads*128) columns, pitch row_stride elements, box 64 x 128.
  return make_tmap_2d(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)heads * 128, (uint64_t)T,
                      (uint64_t)row_stride, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
}

static CUtensorMap head_map64(const void* base, int64_t row_stride, int heads, int T) {
  return make_tmap_2d(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)heads * 128, (uint64_t)T,
                      (uint64_t)row_stride, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
}

void attn_fwd(const AttnArgs& a, cudaStream_t stream) {
  using namespace attn;
  if (a.head_dim != 128) throw std::runtime_error("wavelet_b200 attention: head_dim must be 128");
  if (a.Hq % a.Hk) throw std::runtime_error("wavelet_b200 attention: Hq must be a multiple of Hk");
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> attr[64];  // per device; cudaFuncSetAttribute is idempotent
  if (!attr[dev & 63].load(std::memory_order_acquire)) {
    cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_smem_bytes());
    attr[dev & 63].store(true, std::memory_order_release);
  }
  const int Tk = a.cu_seqlens_k ? a.Tk : a.T;
  CUtensorMap mq = head_map(a.q, a.q_row, a.Hq, a.T);
  CUtensorMap mk = head_map(a.k, a.k_row, a.Hk, Tk);
  CUtensorMap mv = head_map(a.v, a.v_row, a.Hk, Tk);
  FwdParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.lse = a.lse;
  p.cu = a.cu_seqlens;
  p.cuk = a.cu_seqlens_k;
  p.o_row = a.o_row;
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.T = a.T;
  p.nseq = a.nseq;
  p.scale_log2 = a.scale * LOG2E;
  p.err = error_word(dev);
  dim3 grid((a.max_seqlen + TILE - 1) / TILE, a.Hq, a.nseq);
  attn_fwd_kernel<<<grid, NUM_THREADS, fwd_smem_bytes(), stream>>>(mq, mk, mv, p); note_launch();
}

}  // namespace wb

namespace wb {

void attn_bwd(const AttnBwdArgs& b, cudaStream_t stream) {
  using namespace attn;
  const AttnArgs& a = b.f;
  if (a.head_dim != 128) throw std::runtime_error("wavelet_b200 attention: head_dim must be 128");
  const int rep = a.Hq / a.Hk;
  if (rep > 1 && (!b.part_dk || !b.part_dv))
    throw std::runtime_error("wavelet_b200 attention: GQA backward needs fp32 partial buffers");
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> attr[64];  // per device; cudaFuncSetAttribute is idempotent
  if (!attr[dev & 63].load(std::memory_order_acquire)) {
    cudaFuncSetAttribute(attn_bwd_dkv2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dkv2_smem_bytes());
    cudaFuncSetAttribute(attn_bwd_dq2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dq2_smem_bytes());
    attr[dev & 63].store(true, std::memory_order_release);
  }
  {
    const int warps = 8;
    const int64_t work = (int64_t)a.T * a.Hq;
    attn_delta_kernel<<<(int)((work + warps - 1) / warps), warps * 32, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(a.o), a.o_row, reinterpret_cast<const __nv_bfloat16*>(b.dout),
        b.delta, a.T, a.Hq); note_launch();
  }
  const int Tk = a.cu_seqlens_k ? a.Tk : a.T;
  CUtensorMap mq = head_map(a.q, a.q_row, a.Hq, a.T);
  CUtensorMap mk = head_map(a.k, a.k_row, a.Hk, Tk);
  CUtensorMap mv = head_map(a.v, a.v_row, a.Hk, Tk);
  CUtensorMap mdo = head_map(b.dout, (int64_t)a.Hq * 128, a.Hq, a.T);
  CUtensorMap mq64 = head_map64(a.q, a.q_row, a.Hq, a.T);
  CUtensorMap mdo64 = head_map64(b.dout, (int64_t)a.Hq * 128, a.Hq, a.T);
  Bwd2Params p2;
  BwdParams& p = p2.b;
  p.lse = a.lse;
  p.delta = b.delta;
  p.cu = a.cu_seqlens;
  p.cuk = a.cu_seqlens_k;
  p.dq = reinterpret_cast<__nv_bfloat16*>(b.dq);
  p.dk = reinterpret_cast<__nv_bfloat16*>(b.dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(b.dv);
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.T = a.T;
  p.scale = a.scale;
  p.scale_log2 = a.scale * LOG2E;
  p.err = error_word(dev);
  p2.part_dk = b.part_dk;
  p2.part_dv = b.part_dv;
  const int nt = (a.max_seqlen + TILE - 1) / TILE;
  const int ntk = ((a.cu_seqlens_k ? a.max_seqlen_k : a.max_seqlen) + TILE - 1) / TILE;
  attn_bwd_dkv2_kernel<<<dim3(ntk, a.Hq, a.nseq), NUM_THREADS_BWD2, dkv2_smem_bytes(), stream>>>(mq64, mk, mv, mdo64, p2); note_launch();
  CUtensorMap mk64 = head_map64(a.k, a.k_row, a.Hk, Tk);
  CUtensorMap mv64 = head_map64(a.v, a.v_row, a.Hk, Tk);
  attn_bwd_dq2_kernel<<<dim3(nt, a.Hq, a.nseq), NUM_THREADS_BWD2, dq2_smem_bytes(), stream>>>(mq, mk64, mv64, mdo, p); note_launch();
  if (rep > 1) {
    const int warps = 8;
    const int64_t work = (int64_t)Tk * a.Hk;
    attn_dkv_reduce_kernel<<<(int)((work + warps - 1) / warps), warps * 32, 0, stream>>>(
        b.part_dk, b.part_dv, p.dk, p.dv, Tk, a.Hq, a.Hk, a.scale); note_launch();
  }
}

// Same launch sequence as attn_bwd, with the Delta scratch (b.delta) and the
// error word supplied by the caller instead of looked up / allocated here.
// Used by the allocation-free entry point (attention_noalloc.cu).
int attn_bwd_explicit(const AttnBwdArgs& b, int* err, cudaStream_t stream) {
  using namespace attn;
  const AttnArgs& a = b.f;
  if (a.head_dim != 128) return 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 2;
  static std::atomic<bool> attr[64];  // per device; cudaFuncSetAttribute is idempotent
  if (!attr[dev & 63].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(attn_bwd_dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dkv_smem_bytes()) !=
            cudaSuccess ||
        cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dq_smem_bytes()) !=
            cudaSuccess)
      return 3;
    attr[dev & 63].store(true, std::memory_order_release);
  }
  {
    const int warps = 8;
    const int64_t work = (int64_t)a.T * a.Hq;
    attn_delta_kernel<<<(int)((work + warps - 1) / warps), warps * 32, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(a.o), a.o_row, reinterpret_cast<const __nv_bfloat16*>(b.dout),
        b.delta, a.T, a.Hq); note_launch();
  }
  CUtensorMap mq, mk, mv, mdo;
  try {
    mq = head_map(a.q, a.q_row, a.Hq, a.T);
    mk = head_map(a.k, a.k_row, a.Hk, a.T);
    mv = head_map(a.v, a.v_row, a.Hk, a.T);
    mdo = head_map(b.dout, (int64_t)a.Hq * 128, a.Hq, a.T);
  } catch (const std::exception&) {
    return 4;
  }
  if (a.cu_seqlens_k) return 6;  // separate key sequences: v2 kernels (attn_bwd) only
  BwdParams p;
  p.lse = a.lse;
  p.delta = b.delta;
  p.cu = a.cu_seqlens;
  p.cuk = nullptr;
  p.dq = reinterpret_cast<__nv_bfloat16*>(b.dq);
  p.dk = reinterpret_cast<__nv_bfloat16*>(b.dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(b.dv);
  p.Hq = a.Hq;
  p.Hk = a.Hk;
  p.T = a.T;
  p.scale = a.scale;
  p.scale_log2 = a.scale * LOG2E;
  p.err = err;
  const int nt = (a.max_seqlen + TILE - 1) / TILE;
  attn_bwd_dkv_kernel<<<dim3(nt, a.Hk, a.nseq), NUM_THREADS, dkv_smem_bytes(), stream>>>(mq, mk, mv, mdo, p); note_launch();
  attn_bwd_dq_kernel<<<dim3(nt, a.Hq, a.nseq), NUM_THREADS, dq_smem_bytes(), stream>>>(mq, mk, mv, mdo, p); note_launch();
  return cudaGetLastError() == cudaSuccess ? 0 : 5;
}

}  // namespace wb
