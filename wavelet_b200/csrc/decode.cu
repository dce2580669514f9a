// Generator kernels for sm_100a: paged KV-cache append, paged decode
// attention (GQA), and fused temperature sampling with the processed
// log-prob of the sampled token.
//
// KV cache layout per layer: k_cache / v_cache [num_blocks, Hk, block_size, 128]
// bf16 (head-major pages: the tokens of one head in one block are a
// contiguous run); block_tables [num_seqs, max_blocks] int32; context_lens
// [num_seqs].
// These replace vLLM's paged attention / sampler used by the reference's
// rollout engine (inference/engine.py:776-818).
#include <atomic>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include <stdexcept>

#include "common.cuh"
#include "decode.h"
#include "tma.h"

namespace wb {
namespace {

constexpr int HD = 128;

// ------------------------------------------------------------------ append
// One warp per (token, kv head): copy 128 bf16 of K and V into the paged cache.
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ k, int64_t k_row,
                                 const __nv_bfloat16* __restrict__ v, int64_t v_row,
                                 __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                                 const int* __restrict__ slot, int T, int Hk, int block_size) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * Hk) return;
  const int t = w / Hk, h = w - t * Hk;
  const int s = slot[t];
  if (s < 0) return;
  const int blk = s / block_size, off = s - blk * block_size;  // slot = block * block_size + offset
  const int64_t dst = (((int64_t)blk * Hk + h) * block_size + off) * HD;
  reinterpret_cast<uint2*>(k_cache + dst)[lane] = reinterpret_cast<const uint2*>(k + (int64_t)t * k_row + h * HD)[lane];
  reinterpret_cast<uint2*>(v_cache + dst)[lane] = reinterpret_cast<const uint2*>(v + (int64_t)t * v_row + h * HD)[lane];
}

// ------------------------------------------------------------- decode attn
// CTA per (sequence, kv head, split).  256 threads.  For every page of the
// split: the page's K and V rows of this head are staged in shared memory
// (coalesced 16-byte loads), scores for (token, q head) pairs are computed
// from shared memory, and an online softmax accumulates O[rep][128].
// Splits > 1 write partial (m, l, O) that decode_combine merges.
constexpr int DEC_THREADS = 256;
constexpr int MAX_REP = 16;
constexpr int PAGE_MAX = 64;

__global__ void __launch_bounds__(DEC_THREADS)
    decode_attn_kernel(const __nv_bfloat16* __restrict__ q, int64_t q_row,
                       const __nv_bfloat16* __restrict__ k_cache, const __nv_bfloat16* __restrict__ v_cache,
                       const int* __restrict__ block_tables, int max_blocks, const int* __restrict__ ctx_lens,
                       __nv_bfloat16* __restrict__ out, int64_t out_row, float* __restrict__ part_o,
                       float* __restrict__ part_ml, int Hq, int Hk, int block_size, int splits,
                       float scale_log2) {
  const int seq = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int rep = Hq / Hk;
  const int L = ctx_lens[seq];
  const int n_pages = (L + block_size - 1) / block_size;
  const int pages_per = (n_pages + splits - 1) / splits;
  const int p0 = sp * pages_per, p1 = min(n_pages, p0 + pages_per);

  __shared__ __align__(16) __nv_bfloat16 sK[PAGE_MAX * HD];
  __shared__ __align__(16) __nv_bfloat16 sV[PAGE_MAX * HD];
  __shared__ float sQ[MAX_REP * HD];
  __shared__ float sS[MAX_REP * PAGE_MAX];
  __shared__ float sM[MAX_REP], sL[MAX_REP], sAlpha[MAX_REP];

  const int tid = threadIdx.x;
  for (int i = tid; i < rep * HD; i += DEC_THREADS) {
    const int r = i / HD, d = i - r * HD;
    sQ[i] = __bfloat162float(q[(int64_t)seq * q_row + (g * rep + r) * HD + d]);
  }
  if (tid < rep) {
    sM[tid] = -INFINITY;
    sL[tid] = 0.f;
  }
  // each thread owns outputs (r, d) for idx = tid + k*256 < rep*128
  float acc[MAX_REP * HD / DEC_THREADS];
  constexpr int ACC = MAX_REP * HD / DEC_THREADS;
#pragma unroll
  for (int i = 0; i < ACC; ++i) acc[i] = 0.f;
  __syncthreads();

  const int* bt = block_tables + (int64_t)seq * max_blocks;
  for (int pg = p0; pg < p1; ++pg) {
    const int blk = bt[pg];
    const int ntok = min(block_size, L - pg * block_size);
    // stage K, V rows (ntok x 128) of head g: 16-byte vectors
    const int vec_per_row = HD / 8;
    for (int i = tid; i < ntok * vec_per_row; i += DEC_THREADS) {
      const int j = i / vec_per_row, c = i - j * vec_per_row;
      const int64_t src = (((int64_t)blk * Hk + g) * block_size + j) * HD + c * 8;
      reinterpret_cast<uint4*>(sK)[j * vec_per_row + c] = *reinterpret_cast<const uint4*>(k_cache + src);
      reinterpret_cast<uint4*>(sV)[j * vec_per_row + c] = *reinterpret_cast<const uint4*>(v_cache + src);
    }
    __syncthreads();
    // scores
    for (int i = tid; i < rep * ntok; i += DEC_THREADS) {
      const int r = i / ntok, j = i - r * ntok;
      const uint4* kr = reinterpret_cast<const uint4*>(sK + j * HD);
      const float* qr = sQ + r * HD;
      float s = 0.f;
#pragma unroll 4
      for (int c = 0; c < 16; ++c) {
        const uint4 kv = kr[(c + j) & 15];  // rotate start to spread banks
        const int base = ((c + j) & 15) * 8;
        s += bf16_lo(kv.x) * qr[base + 0] + bf16_hi(kv.x) * qr[base + 1] + bf16_lo(kv.y) * qr[base + 2] +
             bf16_hi(kv.y) * qr[base + 3] + bf16_lo(kv.z) * qr[base + 4] + bf16_hi(kv.z) * qr[base + 5] +
             bf16_lo(kv.w) * qr[base + 6] + bf16_hi(kv.w) * qr[base + 7];
      }
      sS[r * PAGE_MAX + j] = s * scale_log2;
    }
    __syncthreads();
    // per-head online softmax update (one warp per head)
    const int warp = tid >> 5, lane = tid & 31;
    for (int r = warp; r < rep; r += DEC_THREADS / 32) {
      float mx = -INFINITY;
      for (int j = lane; j < ntok; j += 32) mx = fmaxf(mx, sS[r * PAGE_MAX + j]);
      mx = warp_max(mx);
      const float m_old = sM[r];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int j = lane; j < ntok; j += 32) {
        const float p = exp2f(sS[r * PAGE_MAX + j] - m_new);
        sS[r * PAGE_MAX + j] = p;
        sum += p;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float a = (m_old == -INFINITY) ? 0.f : exp2f(m_old - m_new);
        sAlpha[r] = a;
        sL[r] = sL[r] * a + sum;
        sM[r] = m_new;
      }
    }
    __syncthreads();
    // O = O * alpha + P V
#pragma unroll
    for (int i = 0; i < ACC; ++i) {
      const int idx = tid + i * DEC_THREADS;
      if (idx < rep * HD) {
        const int r = idx / HD, d = idx - r * HD;
        float o = acc[i] * sAlpha[r];
        const float* pr = sS + r * PAGE_MAX;
        for (int j = 0; j < ntok; ++j) o += pr[j] * __bfloat162float(sV[j * HD + d]);
        acc[i] = o;
      }
    }
    __syncthreads();
  }
  // write
  if (splits == 1) {
#pragma unroll
    for (int i = 0; i < ACC; ++i) {
      const int idx = tid + i * DEC_THREADS;
      if (idx < rep * HD) {
        const int r = idx / HD, d = idx - r * HD;
        const float l = sL[r];
        out[(int64_t)seq * out_row + (g * rep + r) * HD + d] = __float2bfloat16(l > 0.f ? acc[i] / l : 0.f);
      }
    }
  } else {
    const int64_t base = ((int64_t)seq * Hq + g * rep) * splits + sp;  // unused form kept simple below
    (void)base;
#pragma unroll
    for (int i = 0; i < ACC; ++i) {
      const int idx = tid + i * DEC_THREADS;
      if (idx < rep * HD) {
        const int r = idx / HD, d = idx - r * HD;
        const int h = g * rep + r;
        part_o[(((int64_t)seq * Hq + h) * splits + sp) * HD + d] = acc[i];
      }
    }
    if (tid < rep) {
      const int h = g * rep + tid;
      part_ml[(((int64_t)seq * Hq + h) * splits + sp) * 2 + 0] = sM[tid];
      part_ml[(((int64_t)seq * Hq + h) * splits + sp) * 2 + 1] = sL[tid];
    }
  }
}

// ------------------------------------------------------------ decode attention (TMA ring)
// Memory-bound by design: every (sequence, kv head) reads its K/V history
// once.  CTA per (sequence, kv head, split), 4 warps, a ring of 4 stages of 32
// tokens (K and V, 16 KB) in shared memory filled by TMA (two 64-column
// halves per tile, 128-byte swizzle, no multicast; pages are head-major so a
// stage is one contiguous 8 KB run per tensor).  Warp w owns ring slot w: it
// processes stages w, w+4, ... of the split with its own online-softmax state
// and refills its slot as soon as it has read it, so while one warp computes,
// the other slots' loads are in flight.  The four warp states merge at the
// end; splits > 1 write partials for decode_combine.
constexpr int D2_WARPS = 4;
constexpr int D2_TOK = 32;
constexpr int D2_HALF = D2_TOK * 64 * 2;  // 32 rows x 64 bf16 = 4 KB
constexpr int D2_STAGE = 4 * D2_HALF;     // K lo, K hi, V lo, V hi
constexpr int D2_MAXREP = 8;

constexpr size_t d2_smem_bytes(int rep) {
  return 1024 + (size_t)D2_WARPS * D2_STAGE + (size_t)rep * HD * 4 + D2_WARPS * 8 + 16;
}

// Both products run
// on the tensor cores with mma.sync m16n8k16 (bf16 in, fp32 accumulate):
//   S[16 x 32]  = Q[16 x 128] K^T   (rows = the rep q heads of this kv head,
//                                    padded to 16; 4 n-tiles x 8 k-steps)
//   O[16 x 128] += P[16 x 32] V     (16 n-tiles x 2 k-steps; P comes straight
//                                    from the S accumulators as A fragments)
// K fragments come from ldmatrix on the swizzled tile, V fragments from
// ldmatrix.trans.  tcgen05 needs M >= 64 while a GQA decode step has only
// rep (4..8) query rows per kv head, so the warp-level MMA is the right unit
// here; it needs about a tenth of the issue slots of a CUDA-core dot-product
// loop (measured: the scalar version was issue-bound at ~1.5 TB/s).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// byte offset of (row, 16-byte chunk c in 0..15) in a [32 x 128] bf16 tile
// stored as two 128-byte-swizzled 64-column halves
__device__ __forceinline__ uint32_t tile_off(int row, int c) {
  return (uint32_t)((c >> 3) * D2_HALF + row * 128 + (((c & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(D2_WARPS * 32)
    decode_attn3_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const __nv_bfloat16* __restrict__ q, int64_t q_row, const int* __restrict__ block_tables,
                        int max_blocks, const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out,
                        int64_t out_row, float* __restrict__ part_o, float* __restrict__ part_ml, int Hq, int Hk,
                        int block_size, int splits, float scale_log2, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + D2_WARPS * D2_STAGE);
  volatile int* abort = reinterpret_cast<volatile int*>(full + D2_WARPS);
  const int rep = Hq / Hk;
  const int seq = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int L = ctx_lens[seq];
  const int n_st = (L + D2_TOK - 1) / D2_TOK;
  const int per = (n_st + splits - 1) / splits;
  const int s0 = sp * per, s1 = min(n_st, s0 + per);
  const int* bt = block_tables + (int64_t)seq * max_blocks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < D2_WARPS; ++i) mbar_init(&full[i], 1);
    *abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  __syncthreads();
  uint8_t* slot = ring + warp * D2_STAGE;
  auto issue = [&](int st) {
    const int tok0 = st * D2_TOK;
    const int row = (bt[tok0 / block_size] * Hk + g) * block_size + tok0 % block_size;
    mbar_arrive_expect_tx(&full[warp], D2_STAGE);
    tma_load_2d(&tmK, &full[warp], slot, 0, row);
    tma_load_2d(&tmK, &full[warp], slot + D2_HALF, 64, row);
    tma_load_2d(&tmV, &full[warp], slot + 2 * D2_HALF, 0, row);
    tma_load_2d(&tmV, &full[warp], slot + 3 * D2_HALF, 64, row);
  };
  bool pending = s0 + warp < s1;
  if (lane == 0 && pending) issue(s0 + warp);

  // Q A-fragments for the 8 k-steps: rows gid (< rep) real, rows gid + 8 zero
  uint32_t qa[8][2];
  {
    const bool real = gid < rep;
    const __nv_bfloat16* qr = q + (int64_t)seq * q_row + (g * rep + (real ? gid : 0)) * HD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = real ? *reinterpret_cast<const uint32_t*>(qr + ks * 16 + tig * 2) : 0u;
      qa[ks][1] = real ? *reinterpret_cast<const uint32_t*>(qr + ks * 16 + 8 + tig * 2) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_row = -INFINITY, l_part = 0.f;
  uint32_t phase = 0;
  const uint32_t kbase = smem_u32(slot), vbase = kbase + 2 * D2_HALF;
  const int mi = lane >> 3, r8 = lane & 7;
  for (int st = s0 + warp; st < s1; st += D2_WARPS) {
    if (!mbar_wait_warp(&full[warp], phase, abort, err, kErrTimeoutProducer)) break;
    pending = false;
    phase ^= 1;
    // ---- S = Q K^T (4 n-tiles of 8 tokens)
    float sacc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        // matrices: (ks lo, ks hi, ks+1 lo, ks+1 hi) of tokens 8j..8j+7
        const int tok = 8 * j + r8;
        const int c = 2 * (ks + (mi >> 1)) + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + tile_off(tok, c), b0, b1, b2, b3);
        const uint32_t a0[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
        const uint32_t a1[4] = {qa[ks + 1][0], 0u, qa[ks + 1][1], 0u};
        mma_bf16_16816(sacc[j], a0, b0, b1);
        mma_bf16_16816(sacc[j], a1, b2, b3);
      }
    }
    // ---- online softmax on rows gid (the 4 threads of a group share a row)
    const int tbase = st * D2_TOK;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tbase + 8 * j + tig * 2 + e;
        const float v = (t < L) ? sacc[j][e] * scale_log2 : -INFINITY;
        sacc[j][e] = v;
        mx = fmaxf(mx, v);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m_row, mx);
    const float alpha = (m_row == -INFINITY) ? 0.f : exp2f(m_row - mn);
    m_row = mn;
    float ps = 0.f;
    uint32_t pa[4][2];  // P as bf16 pairs per n-tile (rows gid)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p0 = exp2f(sacc[j][0] - mn), p1 = exp2f(sacc[j][1] - mn);
      ps += p0 + p1;
      pa[j][0] = pack_bf16x2(p0, p1);
    }
    l_part = l_part * alpha + ps;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= alpha;
      o[n][1] *= alpha;
    }
    // ---- O += P V (2 k-steps of 16 tokens, 16 n-tiles of 8 dims)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const uint32_t a[4] = {pa[2 * ks][0], 0u, pa[2 * ks + 1][0], 0u};
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        // matrices: (n: tokens lo, tokens hi), (n+1: tokens lo, tokens hi)
        const int tok = 16 * ks + 8 * (mi & 1) + r8;
        const int c = n + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + tile_off(tok, c), b0, b1, b2, b3);
        mma_bf16_16816(o[n], a, b0, b1);
        mma_bf16_16816(o[n + 1], a, b2, b3);
      }
    }
    __syncwarp();
    if (st + D2_WARPS < s1) {
      if (lane == 0) {
        fence_proxy_async_shared();  // generic reads of the slot before the async-proxy refill
        issue(st + D2_WARPS);
      }
      pending = true;
    }
  }
  if (pending && lane == 0) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&full[warp], phase))
      if (globaltimer_ns() - t0 > kWaitBudgetNs) { atomicOr(err, kErrTimeoutDrain); break; }
  }
  float l_row = l_part + __shfl_xor_sync(0xffffffffu, l_part, 1);
  l_row += __shfl_xor_sync(0xffffffffu, l_row, 2);
  __syncthreads();
  float* sm = reinterpret_cast<float*>(ring);  // [warps][8] m
  float* sl = sm + D2_WARPS * 8;               // [warps][8] l
  float* so = sl + D2_WARPS * 8;               // [warps][8][128]
  if (gid < rep) {
    if (tig == 0) {
      sm[warp * 8 + gid] = m_row;
      sl[warp * 8 + gid] = l_row;
    }
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<float2*>(so + (warp * 8 + gid) * HD + 8 * n + tig * 2) = make_float2(o[n][0], o[n][1]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rep * HD; i += blockDim.x) {
    const int r = i / HD, d = i - r * HD;
    float mm = -INFINITY;
    for (int w = 0; w < D2_WARPS; ++w) mm = fmaxf(mm, sm[w * 8 + r]);
    float ll = 0.f, acc = 0.f;
    for (int w = 0; w < D2_WARPS; ++w) {
      const float mw = sm[w * 8 + r];
      if (mw == -INFINITY) continue;
      const float a = exp2f(mw - mm);
      ll += sl[w * 8 + r] * a;
      acc += so[(w * 8 + r) * HD + d] * a;
    }
    const int h = g * rep + r;
    if (splits == 1) {
      out[(int64_t)seq * out_row + h * HD + d] = __float2bfloat16(ll > 0.f ? acc / ll : 0.f);
    } else {
      part_o[(((int64_t)seq * Hq + h) * splits + sp) * HD + d] = acc;
      if (d == 0) {
        part_ml[(((int64_t)seq * Hq + h) * splits + sp) * 2 + 0] = mm;
        part_ml[(((int64_t)seq * Hq + h) * splits + sp) * 2 + 1] = ll;
      }
    }
  }
}

// Merge split partials: one warp per (seq, q head), lane covers 4 dims.
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                      __nv_bfloat16* __restrict__ out, int64_t out_row, int nseq, int Hq,
                                      int splits) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= nseq * Hq) return;
  const int seq = w / Hq, h = w - seq * Hq;
  const int64_t b = ((int64_t)seq * Hq + h) * splits;
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, part_ml[(b + s) * 2]);
  float l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < splits; ++s) {
    const float ms = part_ml[(b + s) * 2], ls = part_ml[(b + s) * 2 + 1];
    if (ls <= 0.f) continue;
    const float a = exp2f(ms - m);
    l += ls * a;
    const float4 po = reinterpret_cast<const float4*>(part_o + (b + s) * HD)[lane];
    o[0] += po.x * a;
    o[1] += po.y * a;
    o[2] += po.z * a;
    o[3] += po.w * a;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  uint2 r;
  r.x = pack_bf16(o[0] * inv, o[1] * inv);
  r.y = pack_bf16(o[2] * inv, o[3] * inv);
  reinterpret_cast<uint2*>(out + (int64_t)seq * out_row + h * HD)[lane] = r;
}

// ---------------------------------------------------------------- sampling
// Counter-based uniform from (seed, row, col, step): SplitMix64 finaliser
// (Steele, Lea & Flood 2014) — deterministic and stateless.
__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t row, uint64_t col) {
  uint64_t z = seed ^ (row * 0x9E3779B97F4A7C15ull) ^ (col * 0xD1B54A32D192ED03ull);
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= (z >> 31);
  return ((z >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
}

// One CTA per row: Gumbel-max sample of softmax(z / tau) plus the processed
// log-prob log softmax(z / tau)[sampled] (online logsumexp in the same pass).
// tau <= 0 means greedy.  Optional top-k / min-p restrict the support: they
// need the row max (min-p) or a threshold computed by a previous pass
// (top-k threshold given per row in `thresh`; -inf disables).
__global__ void sample_kernel(const __nv_bfloat16* __restrict__ z, int64_t ldz, int V,
                              const float* __restrict__ inv_tau, const float* __restrict__ thresh,
                              float min_p, uint64_t seed, const int64_t* __restrict__ row_ids,
                              int64_t* __restrict__ out_tok, float* __restrict__ out_lp,
                              const int64_t* __restrict__ seed_dev) {
  const int row = blockIdx.x;
  if (seed_dev) seed = (uint64_t)*seed_dev;  // device-resident seed (CUDA-graph replays)
  const float it = inv_tau[row];
  const bool greedy = !(it > 0.f) || isinf(it);
  const float scale = greedy ? 1.f : it;
  const float th = thresh ? thresh[row] : -INFINITY;
  const __nv_bfloat16* zr = z + (int64_t)row * ldz;
  const uint64_t rid = row_ids ? (uint64_t)row_ids[row] : (uint64_t)row;
  __shared__ float s_m[32], s_s[32], s_best[32];
  __shared__ int s_arg[32];
  __shared__ float s_rowmax;
  // pass 0 (min-p): row max of scaled logits
  float minp_cut = -INFINITY;
  if (min_p > 0.f) {
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, __bfloat162float(zr[i]) * scale);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) s_m[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? s_m[threadIdx.x] : -INFINITY;
      v = warp_max(v);
      if (threadIdx.x == 0) s_rowmax = v;
    }
    __syncthreads();
    minp_cut = s_rowmax + logf(min_p);
  }
  float m = -INFINITY, s = 0.f, best = -INFINITY;
  int arg = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float raw = __bfloat162float(zr[i]);
    const float x = raw * scale;
    if (raw < th || x < minp_cut) continue;
    if (x > m) {
      s *= __expf(m - x);
      m = x;
    }
    s += __expf(x - m);
    float key = x;
    if (!greedy) {
      const float u = uniform01(seed, rid, (uint64_t)i);
      key = x - __logf(-__logf(u));
    }
    if (key > best) {
      best = key;
      arg = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int a2 = __shfl_xor_sync(0xffffffffu, arg, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
    if (b2 > best || (b2 == best && a2 < arg)) {
      best = b2;
      arg = a2;
    }
  }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s_m[wid] = m, s_s[wid] = s, s_best[wid] = best, s_arg[wid] = arg;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? s_m[lane] : -INFINITY;
    s = lane < nw ? s_s[lane] : 0.f;
    best = lane < nw ? s_best[lane] : -INFINITY;
    arg = lane < nw ? s_arg[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int a2 = __shfl_xor_sync(0xffffffffu, arg, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
      m = mm;
      if (b2 > best || (b2 == best && a2 < arg)) {
        best = b2;
        arg = a2;
      }
    }
    if (lane == 0) {
      out_tok[row] = arg;
      out_lp[row] = __bfloat162float(zr[arg]) * scale - (m + __logf(s));
    }
  }
}

}  // namespace

void kv_append(const void* k, int64_t k_row, const void* v, int64_t v_row, void* k_cache, void* v_cache,
               const int* slot, int T, int Hk, int block_size, cudaStream_t st) {
  if (T <= 0) return;
  const int warps = 8;
  kv_append_kernel<<<(T * Hk + warps - 1) / warps, warps * 32, 0, st>>>(
      (const __nv_bfloat16*)k, k_row, (const __nv_bfloat16*)v, v_row, (__nv_bfloat16*)k_cache,
      (__nv_bfloat16*)v_cache, slot, T, Hk, block_size); note_launch();
}

void decode_attention(const DecodeArgs& a, cudaStream_t st) {
  if (a.Hq / a.Hk > MAX_REP) throw std::runtime_error("decode_attention: at most 16 q heads per kv head");
  if (a.block_size > PAGE_MAX) throw std::runtime_error("decode_attention: block_size must be <= 64");
  if (a.nseq <= 0) return;
  dim3 grid(a.nseq, a.Hk, a.splits);
  const int rep = a.Hq / a.Hk;
  if (rep <= D2_MAXREP && a.block_size % D2_TOK == 0 && a.cache_rows > 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    static std::atomic<bool> attr[64];  // per device; cudaFuncSetAttribute is idempotent
    const size_t smem = d2_smem_bytes(D2_MAXREP);
    if (!attr[dev & 63].load(std::memory_order_acquire)) {
      cudaFuncSetAttribute(decode_attn3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr[dev & 63].store(true, std::memory_order_release);
    }
    const uint64_t rows = (uint64_t)a.cache_rows * a.Hk;  // [num_blocks * Hk * block_size, 128]
    CUtensorMap tk = make_tmap_2d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, rows, HD, 64, D2_TOK,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tv = make_tmap_2d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, rows, HD, 64, D2_TOK,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    decode_attn3_kernel<<<grid, D2_WARPS * 32, smem, st>>>(
        tk, tv, (const __nv_bfloat16*)a.q, a.q_row, a.block_tables, a.max_blocks, a.ctx_lens, (__nv_bfloat16*)a.out,
        a.out_row, a.part_o, a.part_ml, a.Hq, a.Hk, a.block_size, a.splits, a.scale * 1.4426950408889634f,
        error_word(dev)); note_launch();
  } else {
  decode_attn_kernel<<<grid, DEC_THREADS, 0, st>>>(
      (const __nv_bfloat16*)a.q, a.q_row, (const __nv_bfloat16*)a.k_cache, (const __nv_bfloat16*)a.v_cache,
      a.block_tables, a.max_blocks, a.ctx_lens, (__nv_bfloat16*)a.out, a.out_row, a.part_o, a.part_ml, a.Hq, a.Hk,
      a.block_size, a.splits, a.scale * 1.4426950408889634f); note_launch();
  }
  if (a.splits > 1) {
    const int warps = 8;
    decode_combine_kernel<<<(a.nseq * a.Hq + warps - 1) / warps, warps * 32, 0, st>>>(
        a.part_o, a.part_ml, (__nv_bfloat16*)a.out, a.out_row, a.nseq, a.Hq, a.splits); note_launch();
  }
}

namespace {

// Order-preserving 16-bit key of a bf16 value: larger value -> larger key.
__device__ __forceinline__ uint32_t bf16_key(uint16_t b) { return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u); }
__device__ __forceinline__ float key_value(uint32_t k) {
  const uint16_t b = (k & 0x8000u) ? (uint16_t)(k & 0x7FFFu) : (uint16_t)(~k & 0xFFFFu);
  return __bfloat162float(__ushort_as_bfloat16(b));
}

constexpr int TH_THREADS = 1024;

// Scan 256 bins from the top (bin 255) down; returns the first bin whose
// inclusive running total reaches `target`, and the total strictly above it
// in *above*.  Runs in warp 0 (8 bins per lane), result broadcast via smem.
template <typename T>
__device__ int scan_desc(const T* bins, T target, T* above, int* s_bin, T* s_above) {
  __syncthreads();  // every thread has read the previous scan's result; the bins are complete
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    T part = 0;  // lane l owns bins 255-8l .. 248-8l (descending)
#pragma unroll
    for (int j = 0; j < 8; ++j) part += bins[255 - 8 * lane - j];
    T incl = part;  // inclusive prefix over lanes (descending bin order)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const T excl = incl - part;
    const unsigned hit = __ballot_sync(0xffffffffu, incl >= target);
    const int first = hit ? __ffs(hit) - 1 : 31;
    if (lane == first) {
      T run = excl;
      int bin = 248 - 8 * lane;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int b = 255 - 8 * lane - j;
        if (run + bins[b] >= target || j == 7) {
          bin = b;
          break;
        }
        run += bins[b];
      }
      *s_bin = bin;
      *s_above = run;
    }
  }
  __syncthreads();
  *above = *s_above;
  return *s_bin;
}

// Per row: the sampling threshold in logit units (keep z >= thresh) of the
// row's top-k (k-th largest logit) and top-p (the logit at which the sorted
// cumulative probability of softmax(z * inv_tau) first reaches p), the larger
// of the two; -inf when neither applies.  Radix select over the 16-bit bf16
// keys: one pass for the max and the softmax denominator, one histogram pass
// over the high byte (counts and probability mass), one over the low byte
// inside the selected high-byte bins.  No sort, no host round trip.
__global__ void __launch_bounds__(TH_THREADS) sample_thresh_kernel(const __nv_bfloat16* __restrict__ z, int64_t ldz,
                                                                   int V, const int* __restrict__ top_k,
                                                                   const float* __restrict__ top_p,
                                                                   const float* __restrict__ inv_tau,
                                                                   float* __restrict__ out) {
  __shared__ unsigned cnt_hi[256], cnt_lo[256];
  __shared__ float mass_hi[256], mass_lo[256];
  __shared__ float red[32];
  __shared__ int s_bin;
  __shared__ unsigned s_above_u;
  __shared__ float s_above_f;
  const int row = blockIdx.x;
  const uint16_t* zr = reinterpret_cast<const uint16_t*>(z + (int64_t)row * ldz);
  const int k = top_k ? top_k[row] : 0;
  const float p = top_p ? top_p[row] : 1.f;
  const float it = inv_tau ? inv_tau[row] : 1.f;
  const bool use_k = k > 0 && k < V;
  const bool use_p = p < 1.f && it > 0.f;
  if (!use_k && !use_p) {
    if (threadIdx.x == 0) out[row] = -INFINITY;
    return;
  }
  for (int i = threadIdx.x; i < 256; i += blockDim.x) cnt_hi[i] = 0, cnt_lo[i] = 0, mass_hi[i] = 0.f, mass_lo[i] = 0.f;
  // pass 1: row max (for a stable softmax mass)
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, __bfloat162float(__ushort_as_bfloat16(zr[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  // pass 2: high-byte histograms (count, mass) and the softmax denominator
  float tot = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const uint16_t b = zr[i];
    const uint32_t key = bf16_key(b);
    if (use_k) atomicAdd(&cnt_hi[key >> 8], 1u);
    if (use_p) {
      const float e = __expf((__bfloat162float(__ushort_as_bfloat16(b)) - mx) * it);
      tot += e;
      atomicAdd(&mass_hi[key >> 8], e);
    }
  }
  if (use_p) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = tot;
  }
  __syncthreads();
  if (use_p && threadIdx.x == 0) {
    float v = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += red[w];  // fixed order
    red[0] = v;
  }
  __syncthreads();
  tot = red[0];
  int hk = -1, hp = -1;
  unsigned above_k = 0;
  float above_p = 0.f;
  if (use_k) hk = scan_desc<unsigned>(cnt_hi, (unsigned)k, &above_k, &s_bin, &s_above_u);
  if (use_p) hp = scan_desc<float>(mass_hi, p * tot, &above_p, &s_bin, &s_above_f);
  // pass 3: low-byte histograms inside the selected high-byte bins
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const uint16_t b = zr[i];
    const uint32_t key = bf16_key(b);
    const int hi = (int)(key >> 8);
    if (hi == hk) atomicAdd(&cnt_lo[key & 255u], 1u);
    if (hi == hp) atomicAdd(&mass_lo[key & 255u], __expf((__bfloat162float(__ushort_as_bfloat16(b)) - mx) * it));
  }
  __syncthreads();
  float th = -INFINITY;
  if (use_k) {
    unsigned a2 = 0;
    const int lo = scan_desc<unsigned>(cnt_lo, (unsigned)k - above_k, &a2, &s_bin, &s_above_u);
    th = key_value(((uint32_t)hk << 8) | (uint32_t)lo);
  }
  if (use_p) {
    float a2 = 0.f;
    const int lo = scan_desc<float>(mass_lo, p * tot - above_p, &a2, &s_bin, &s_above_f);
    th = fmaxf(th, key_value(((uint32_t)hp << 8) | (uint32_t)lo));
  }
  if (threadIdx.x == 0) out[row] = th;
}

}  // namespace

void sample_thresholds(const void* z, int64_t ldz, int rows, int V, const int* top_k, const float* top_p,
                       const float* inv_tau, float* out, cudaStream_t st) {
  if (rows <= 0) return;
  sample_thresh_kernel<<<rows, TH_THREADS, 0, st>>>((const __nv_bfloat16*)z, ldz, V, top_k, top_p, inv_tau, out);
  note_launch();
}

void sample_tokens(const void* z, int64_t ldz, int rows, int V, const float* inv_tau, const float* thresh,
                   float min_p, uint64_t seed, const int64_t* row_ids, int64_t* out_tok, float* out_lp,
                   cudaStream_t st, const int64_t* seed_dev) {
  if (rows <= 0) return;
  sample_kernel<<<rows, 1024, 0, st>>>((const __nv_bfloat16*)z, ldz, V, inv_tau, thresh, min_p, seed, row_ids, out_tok,
                                       out_lp, seed_dev); note_launch();
}

// One decode step's bookkeeping on the device (so a step needs no host work):
// record the sampled token / log-prob in column step[0] of the window
// buffers, make it the next input, advance position and context length, look
// up the next KV slot in the block table, then bump the step index and the
// sampling seed.  One CTA (rows <= 1024).
__global__ void decode_advance_kernel(const int64_t* __restrict__ tok, const float* __restrict__ lp,
                                      int64_t* __restrict__ ids, int32_t* __restrict__ pos, int32_t* __restrict__ ctx,
                                      int32_t* __restrict__ slots, const int32_t* __restrict__ bt, int max_blocks,
                                      int block_size, int64_t* __restrict__ win_tok, float* __restrict__ win_lp,
                                      int win_ld, int32_t* __restrict__ step, int64_t* __restrict__ seed, int rows) {
  const int s = *step;
  __syncthreads();
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const int64_t t = tok[i];
    if (s < win_ld) {
      win_tok[(int64_t)i * win_ld + s] = t;
      win_lp[(int64_t)i * win_ld + s] = lp[i];
    }
    ids[i] = t;
    const int p = pos[i] + 1;
    pos[i] = p;
    ctx[i] = p + 1;
    const int b = min(p / block_size, max_blocks - 1);
    slots[i] = bt[(int64_t)i * max_blocks + b] * block_size + p % block_size;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *step = s + 1;
    *seed = *seed + 1;
  }
}

void decode_advance(const int64_t* tok, const float* lp, int64_t* ids, int32_t* pos, int32_t* ctx, int32_t* slots,
                    const int32_t* bt, int max_blocks, int block_size, int64_t* win_tok, float* win_lp, int win_ld,
                    int32_t* step, int64_t* seed, int rows, cudaStream_t st) {
  if (rows <= 0) return;
  if (rows > 1024) throw std::runtime_error("decode_advance: at most 1024 rows");
  decode_advance_kernel<<<1, 1024, 0, st>>>(tok, lp, ids, pos, ctx, slots, bt, max_blocks, block_size, win_tok, win_lp,
                                            win_ld, step, seed, rows); note_launch();
}

}  // namespace wb
