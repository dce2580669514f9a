// Allocation-free attention backward entry point.
//
// This entry point has no counterpart in the reference project; it exists
// for callers of this library that are not allowed to allocate GPU memory:
// code running inside a memory pool or arena that owns every byte of the
// device (so a cudaMalloc would fail or fragment it), plug-ins loaded into a
// host application that forbids device allocation after start-up, and
// launch paths that must not touch the allocator.  Such a caller passes its
// own inputs and outputs; the one scratch buffer the backward needs (the
// per-row Delta = sum(dO * O), Hq x T floats) lives in a fixed, statically
// sized device array inside this library instead of being allocated.
//
// Limit: Hq * T <= WB_ATTN_BWD_NOALLOC_MAX_ROWS (1,048,576 rows = 4 MiB of
// float scratch, held by every GPU that loads the library until the process
// exits).  Larger problems are rejected with WB_NOALLOC_ETOO_LARGE.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define WB_ATTN_BWD_NOALLOC_MAX_ROWS (1 << 20)

// Return codes
#define WB_NOALLOC_OK 0
#define WB_NOALLOC_ETOO_LARGE 1      // Hq * T exceeds WB_ATTN_BWD_NOALLOC_MAX_ROWS
#define WB_NOALLOC_EARG 2            // bad argument (null pointer, negative T / nseq / max_seqlen, Hq % Hk != 0)
#define WB_NOALLOC_ESETUP 3          // cudaGetSymbolAddress of the static scratch failed
#define WB_NOALLOC_ELAUNCH 4         // a kernel launch or TMA descriptor encode failed

#ifdef __cplusplus
extern "C" {
#endif

// Causal varlen GQA attention backward (same math and layouts as the
// library's attn_bwd; the head dimension is fixed at 128): q/k/v/o are [T, H, 128] bf16 with the given row
// strides (elements between tokens), dout/dq are contiguous [T, Hq, 128],
// dk/dv contiguous [T, Hk, 128], lse [Hq, T] fp32 from the forward,
// cu_seqlens device int32 [nseq + 1].  All pointers are device pointers on
// the current device.  Work is enqueued on `stream`; nothing is allocated.
//
// The first call on a device resolves the device address of the static
// scratch (cudaGetSymbolAddress) with that device current; make that first
// call before any stream capture.  Every call shares the same scratch, so
// calls that can overlap on the GPU (different streams, or different host
// threads, on one device) race on it: serialise them.
int wb_attn_bwd_noalloc(const void* q, int64_t q_row, const void* k, int64_t k_row, const void* v,
                        int64_t v_row, const void* o, int64_t o_row, const float* lse, const void* dout,
                        void* dq, void* dk, void* dv, const int* cu_seqlens, int nseq, int max_seqlen,
                        int T, int Hq, int Hk, float scale, cudaStream_t stream);

// Error bits the kernels of the last call(s) on `device` recorded (0 = none);
// a blocking read, for tests and diagnostics.
int wb_attn_bwd_noalloc_status(int device);

// Human-readable description of a return code.
const char* wb_attn_bwd_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
