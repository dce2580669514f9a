// Peer-memory fabric and fused collective kernels (one process per GPU, all
// GPUs of one NVLink/NVSwitch node).
//
// Buffers that take part in a fused collective are allocated with
// fabric_malloc (a plain cudaMalloc allocation), exported with a CUDA IPC
// handle and opened by every peer, so each rank holds a device pointer to the
// same buffer on every other rank.  Kernels then move data with ordinary
// 16-byte loads and stores over NVLink; no kernel here issues TMA, and no
// library kernel is ever given a peer pointer.
//
// Cross-GPU ordering uses per-rank signal pads (fabric memory, zeroed once):
// rank s announces epoch e to rank t by a release store into t's pad slot s,
// and t waits with acquire loads until every slot reaches e.  Epochs only
// grow, so pads never need resetting.  Every wait is bounded by a time budget;
// on expiry the kernel ORs kErrTimeoutPeer into the device error word and
// returns.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wb {

constexpr int kMaxPeers = 8;

struct PeerPtrs {
  void* p[kMaxPeers];
};

// Signal-pad layout (uint32 words); one pad of kPadWords words per rank.
constexpr int kPadWords = 256;
constexpr int kPadBarrier = 0;     // [0, 8): barrier epochs, slot = source rank
constexpr int kPadNormFlag = 8;    // [8, 16): norm-exchange epochs
constexpr int kPadNormVals = 16;   // [16, 32): (sumsq, nonfinite) float pairs per source rank

void* fabric_malloc(size_t bytes);
void fabric_free(void* p);
// 64-byte opaque IPC handle of an allocation made by fabric_malloc.
void fabric_export(void* p, unsigned char out[64]);
void* fabric_import(const unsigned char in[64]);
void fabric_close(void* p);

// Every rank: signal all peers with `epoch`, wait until all peers signalled.
void peer_barrier(const PeerPtrs& pads, int rank, int world, uint32_t epoch, int slot_base,
                  uint64_t budget_ns, int* err, cudaStream_t st);

// out[i] = scale * sum_r grads[r][lo + i] for i < n (fixed rank order), and
// stats[0] += sum wgt(i) * out^2, stats[1] += #non-finite, where wgt = w_lo for
// global index lo + i < w_end and 1 above (w_end = 0: plain sum of squares).
// n, lo and w_end multiples of 8.
void rs_sum_sumsq(const PeerPtrs& grads, int world, int64_t lo, int64_t n, float scale, float* out,
                  float* stats, int64_t w_end, float w_lo, cudaStream_t st);

// Exchange (sumsq, nonfinite) with every peer, then write
// tot = {sumsq, nonfinite, clip factor} (fixed rank order sum).
void norm_exchange(const PeerPtrs& pads, int rank, int world, uint32_t epoch, const float* stats,
                   float max_norm, float* tot, uint64_t budget_ns, int* err, cudaStream_t st);

// AdamW on a shard whose gradient is `g` (already reduced), scaled by tot[2];
// skipped entirely when tot[1] > 0 (non-finite gradients).  Writes the bf16
// result into compute[r] + lo for every rank r (the parameter all-gather).
void adamw_allgather(const PeerPtrs& compute, int world, int64_t lo, float* master, const float* g,
                     float* m, float* v, int64_t n, float lr, float b1, float b2, float eps, float wd,
                     float bc1, float bc2, const float* tot, cudaStream_t st);

// Plain peer all-gather of a bf16 shard (used after loading a checkpoint).
void allgather_bf16(const PeerPtrs& dst, int world, int64_t lo, const void* src, int64_t n,
                    cudaStream_t st);

// dst[r * n + i] = src[r][off + i] (bf16) for every rank r: re-forms a full
// tensor from its per-rank shards (expert-parallel policy refresh).
void gather_from_peers(const PeerPtrs& src, int world, int64_t off, int64_t n, void* dst, cudaStream_t st);

// out[i] = res[i] (optional) + sum_r slots[r * stride + i], r in rank order:
// the local reduction after a kEpiPeerBF16 GEMM filled `slots` (one slot per
// source rank).  n and stride multiples of 8.
void slots_sum(const void* slots, int world, int64_t stride, int64_t n, const void* res, void* out, cudaStream_t st);

// Expert-parallel row exchange over peer memory (comm.cu): dispatch rows to
// their expert's rank / combine the k expert outputs of every token.
// limit_rows >= 0: rows at or past it (or negative) are skipped (not written /
// not read): an over-capacity layout never touches memory past the buffers.
void rows_scatter(const void* x, int64_t ldx, const int64_t* src_row, const int* dst_rank, const int64_t* dst_row,
                  const float* scale, const PeerPtrs& dst, int64_t ldd, int n, int H, int64_t limit_rows,
                  cudaStream_t st);
void rows_gather_sum(const PeerPtrs& src, int64_t lds, const int* src_rank, const int64_t* src_row, const float* w,
                     int k, const void* res, int64_t ldr, void* out, int64_t ldo, bool f32_out, int T, int H,
                     int64_t limit_rows, cudaStream_t st);

}  // namespace wb
