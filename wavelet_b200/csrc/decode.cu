// Generator kernels for sm_100a: paged KV-cache append, paged decode
// attention (GQA), and fused temperature sampling with the processed
// log-prob of the sampled token.
//
// KV cache layout per layer: k_cache / v_cache [num_blocks, block_size, Hk, 128]
// bf16; block_tables [num_seqs, max_blocks] int32; context_lens [num_seqs].
// These replace vLLM's paged attention / sampler used by the reference's
// rollout engine (inference/engine.py:776-818).
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include <stdexcept>

#include "common.cuh"
#include "decode.h"

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
  const int64_t dst = ((int64_t)s * Hk + h) * HD;  // slot = block * block_size + offset
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
      const int64_t src = (((int64_t)blk * block_size + j) * Hk + g) * HD + c * 8;
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
                              int64_t* __restrict__ out_tok, float* __restrict__ out_lp) {
  const int row = blockIdx.x;
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
      (__nv_bfloat16*)v_cache, slot, T, Hk, block_size);
}

void decode_attention(const DecodeArgs& a, cudaStream_t st) {
  if (a.Hq / a.Hk > MAX_REP) throw std::runtime_error("decode_attention: at most 16 q heads per kv head");
  if (a.block_size > PAGE_MAX) throw std::runtime_error("decode_attention: block_size must be <= 64");
  if (a.nseq <= 0) return;
  dim3 grid(a.nseq, a.Hk, a.splits);
  decode_attn_kernel<<<grid, DEC_THREADS, 0, st>>>(
      (const __nv_bfloat16*)a.q, a.q_row, (const __nv_bfloat16*)a.k_cache, (const __nv_bfloat16*)a.v_cache,
      a.block_tables, a.max_blocks, a.ctx_lens, (__nv_bfloat16*)a.out, a.out_row, a.part_o, a.part_ml, a.Hq, a.Hk,
      a.block_size, a.splits, a.scale * 1.4426950408889634f);
  if (a.splits > 1) {
    const int warps = 8;
    decode_combine_kernel<<<(a.nseq * a.Hq + warps - 1) / warps, warps * 32, 0, st>>>(
        a.part_o, a.part_ml, (__nv_bfloat16*)a.out, a.out_row, a.nseq, a.Hq, a.splits);
  }
}

void sample_tokens(const void* z, int64_t ldz, int rows, int V, const float* inv_tau, const float* thresh,
                   float min_p, uint64_t seed, const int64_t* row_ids, int64_t* out_tok, float* out_lp,
                   cudaStream_t st) {
  if (rows <= 0) return;
  sample_kernel<<<rows, 1024, 0, st>>>((const __nv_bfloat16*)z, ldz, V, inv_tau, thresh, min_p, seed, row_ids, out_tok,
                                       out_lp);
}

}  // namespace wb
