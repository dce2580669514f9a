// MoE routing and expert row layout on the device (moe.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"

namespace wb {

// Router: probs = softmax(logits) (logits rounded to bf16 first when
// bf16_logits), top-k experts (ties -> lower index) with their probabilities,
// w = topv / sum(topv) when norm_topk else topv, ssum = sum(topv);
// counts[e] += copies routed to e (counts must be zeroed by the caller).
void moe_route(const float* logits, int T, int E, int k, bool norm_topk, bool bf16_logits, float* probs,
               int64_t* topi, float* topv, float* w, float* ssum, int* counts, cudaStream_t st);

// Layout from all ranks' counts allc[ep][E] (global expert ge is owned by rank
// ge / (E / ep)): base[ge] = first row of this rank's copies of ge in the
// owner's padded layout; this rank's layout: k_start / k_len (padded) /
// n_recv per local expert, tile_group[t] = local expert of 128-row tile t or
// -1, rows[0] = rows used.  overflow[0] = 1 (and kErrEpOverflow in err) when
// any rank's layout exceeds cap_rows; the layout is then empty (every tile -1,
// k_start / k_len / n_recv 0, rows 0).
void moe_layout(const int* allc, int ep, int me, int E, int pad, int64_t cap_rows, int cap_tiles, int64_t* base,
                int* tile_group, int* k_start, int* k_len, int* n_recv, int* rows, int* overflow, int* err,
                cudaStream_t st);

// dst_row[i] = base[topi[i]] + rank of copy i among this rank's copies of the
// same expert in (token, slot) order; dst_rank[i] = topi[i] / El.
void moe_copy_rows(const int64_t* topi, int n_copies, int E, int El, const int64_t* base, int64_t* dst_row,
                   int* dst_rank, cudaStream_t st);

// Zero rows [k_start + n_recv, k_start + k_len) of every local expert segment
// of x (skipped when overflow[0] is set).
void moe_zero_pad(void* x, int64_t ldx, int H, int El, const int* k_start, const int* k_len, const int* n_recv,
                  const int* overflow, cudaStream_t st);

// cnt[0:E] -> dst[r][me * E : (me + 1) * E] for every rank r (peer stores).
void moe_put_counts(const PeerPtrs& dst, int world, int me, int E, const int* cnt, cudaStream_t st);

}  // namespace wb
