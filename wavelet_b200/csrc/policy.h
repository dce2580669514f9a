// Trainer -> generator policy push over peer memory (policy.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"

namespace wb {

// Copy the 2-D blocks of `seg` ([nseg, 6] int64: src_off, dst_off, rows,
// row_len, src_stride, dst_stride, in elements) from `src` into each of the nd
// destination buffers, casting between bf16 and fp32.  prefix[i] = vectors of
// `vec` elements before segment i; total_vectors = all of them.  vec > 1
// requires every offset, stride and row length to be a multiple of vec.
void policy_push(const void* src, int src_bf16, const PeerPtrs& dst, int nd, int dst_bf16, const int64_t* seg,
                 const int64_t* prefix, int nseg, int64_t total_vectors, int vec, cudaStream_t st);

// Release-store `value` into 32-bit word `word` of every destination pad,
// after a system-scope fence (ordered after earlier work on the stream).
void policy_signal(const PeerPtrs& pads, int nd, int word, uint32_t value, cudaStream_t st);

}  // namespace wb
